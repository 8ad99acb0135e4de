/*
 * dg_oracle.h -- CPU restatement of DeltaGrid's recurrence hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load this library, and only as
 * the checker or the timed CPU baseline.  The product path (deltagrid_b200/)
 * never calls it.
 *
 * Parity of this restatement is pinned two ways:
 *   - golden vectors produced by the reference's own PyTorch layer
 *     (src/modules/memory.py per-step loops, src/ops/_autograd.py CPU loop,
 *     DeltaGridLayer._route_sparse_pkm), committed under tests/golden/;
 *   - the reference C++ engine itself (src/cpp/engine/src/deltagrid_math.cpp and
 *     deltagrid_fxp.cpp), compiled from its own sources into oracle/_ref/ by
 *     oracle/Makefile and driven by oracle/ref_engine_harness.cpp.
 *
 * All floating-point arrays are fp32 and dense (row-major, last index fastest).
 * Values that the reference keeps in a 16-bit storage dtype are rounded to that
 * dtype with orc_round() at exactly the points where the reference CUDA kernel
 * casts (src/cpp/delta_kernel.cu:99, :117, :898, :918).
 */
#ifndef DG_ORACLE_H
#define DG_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* storage dtype codes; identical numbering to dg_dtype in include/deltagrid_b200.h */
#define ORC_F32 0
#define ORC_F64 1
#define ORC_F16 2
#define ORC_BF16 3

/* Round an fp32 value to the storage dtype (round-to-nearest-even) and back. */
float orc_round(float x, int dtype);
void orc_round_array(float* x, int64_t n, int dtype);

/* Number of OpenMP threads the oracle uses (1 when built without OpenMP). */
int orc_num_threads(void);
void orc_set_num_threads(int n);

/*
 * Dense sequence forward with the state held in fp32 for all T steps
 * (src/cpp/delta_kernel.cu:64-121, src/modules/memory.py:524-539).
 *   v [B,H,T,Dh]  beta [B,H,T]  wk,wq [B,H,T,S]
 *   decay: [H] (dynamic_decay == 0) or [B,H,T] (dynamic_decay != 0)
 *   s_init [B,H,S,Dh] or NULL (zeros)
 *   out [B,H,T,Dh] (fp32; the caller rounds to the storage dtype)
 *   s_final [B,H,S,Dh] fp32
 *   err_out [B,H,T,Dh] residual r_t, or NULL
 */
void orc_dense_forward(int B, int H, int T, int S, int Dh,
                       const float* v, const float* beta, const float* wk, const float* wq,
                       const float* decay, int dynamic_decay, const float* s_init,
                       float* out, float* s_final, float* err_out);

/*
 * Sparse Delta-PKM sequence forward, state updated in place
 * (src/cpp/delta_kernel.cu:885-920, src/ops/_autograd.py:148-167,
 *  src/modules/memory.py:466-481).  Touched rows are rounded to state_dtype
 * after every scatter, as the reference kernel stores them every step.
 *   v [B,H,T,Dh] beta [B,H,T] wk,wq [B,H,T,A] idx [B,H,T,A] (int64)
 *   decay [H] or [B,H,T];  state [B,H,total_slots,Dh] in/out
 *   out [B,H,T,Dh] fp32 (unrounded);  saved_s_act [B,H,T,A,Dh] or NULL
 */
void orc_pkm_forward(int B, int H, int T, int A, int64_t total_slots, int Dh,
                     const float* v, const float* beta, const float* wk, const float* wq,
                     const int64_t* idx, const float* decay, int dynamic_decay,
                     float* state, int state_dtype, float* out, float* saved_s_act);

/*
 * Two-axis product-key router (src/modules/memory.py:240-289;
 * tie order of src/cpp/engine/src/deltagrid_math.cpp:142-168, pinned by
 * src/cpp/engine/tests/test_math.cpp:44-53: equal scores keep the lower index first).
 *   N tokens; k,q [N,Dh]; wk0 [G0,Dh], wk1 [G1,Dh], wq0 [G0,Dh], wq1 [G1,Dh]
 *   (nn.Linear weight layout);  q_scale: per-token scale or NULL (== 1).
 *   outputs: wk,wq [N,K*K]; idx [N,K*K] (= i0*G1 + i1, axis-0 rank major);
 *   margin [N] or NULL: min over axes of (K-th best score - (K+1)-th best score),
 *   used by tests to exclude documented near-ties.
 */
void orc_pkm_route(int64_t N, int Dh, int G0, int G1, int K,
                   const float* k, const float* q,
                   const float* wk0, const float* wk1, const float* wq0, const float* wq1,
                   const float* q_scale, float* wk, float* wq, int64_t* idx, float* margin);

/* Descending top-K with lower-index-first ties (deltagrid_math.cpp:155-167). */
void orc_topk_desc(const float* scores, int n, int K, float* vals, int32_t* idx);

/* ---------------- Q16.16 fixed-point recurrence core ---------------------- */

/* a*b in Q16.16 with round-half-up (src/cpp/engine/include/deltagrid_math_fxp.h:16-19). */
int32_t orc_fxp_mul(int32_t a, int32_t b);

/*
 * Dense Q16.16 recurrence over T steps per lane (deltagrid_fxp.cpp:380-405,
 * applied once per step as dg_memory_layer_step_fxp is).
 *   wk,wq [L,T,S] (wq already multiplied by q_scale, deltagrid_fxp.cpp:376-378)
 *   v [L,T,Dh]; beta, alpha [L,T]; state [L,S,Dh] in/out; y [L,T,Dh]
 */
void orc_fxp_dense_forward(int L, int T, int S, int Dh,
                           const int32_t* wk, const int32_t* wq, const int32_t* v,
                           const int32_t* beta, const int32_t* alpha,
                           int32_t* state, int32_t* y);

/*
 * Sparse PKM Q16.16 recurrence over T steps per lane (deltagrid_fxp.cpp:298-326).
 *   wk,wq,idx [L,T,A]; state [L,total_slots,Dh] in/out.
 */
void orc_fxp_pkm_forward(int L, int T, int A, int64_t total_slots, int Dh,
                         const int32_t* wk, const int32_t* wq, const int32_t* idx,
                         const int32_t* v, const int32_t* beta, const int32_t* alpha,
                         int32_t* state, int32_t* y);

/* Q16.16 two-axis router for one head (deltagrid_fxp.cpp:246-296), q_scale applied. */
void orc_fxp_pkm_route(int Dh, int G0, int G1, int K, const int32_t* k, const int32_t* q,
                       const int32_t* wk0, const int32_t* wk1, const int32_t* wq0,
                       const int32_t* wq1, int32_t q_scale,
                       int32_t* wk, int32_t* wq, int32_t* idx);

#ifdef __cplusplus
}
#endif
#endif
