/*
 * deltagrid_b200.h -- C ABI of the B200 (sm_100a) DeltaGrid recurrence kernels.
 *
 * Plain C: raw device pointers, element counts and dtype codes; no torch or
 * CUDA types.  `stream` is a cudaStream_t passed as void* (NULL = the legacy
 * default stream).  Every entry point is asynchronous on `stream`, validates
 * its arguments on the host, and returns DG_OK (0) or a negative dg_status.
 * Outputs are caller-owned.  No entry point keeps state between calls except
 * the per-device setup noted where it applies; calls on different streams are
 * independent.
 *
 * Tensor layouts are the reference's (src/cpp/delta_kernel.h): dense, row
 * major, batch-major [B, H, ...] unless strides are taken explicitly.
 * Reference paths below are relative to the hsameerc/deltagrid project root.
 */
#ifndef DELTAGRID_B200_H
#define DELTAGRID_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DG_ABI_VERSION 1

/* storage dtypes; the reference dispatches float, double, Half, BFloat16
   (src/cpp/binding.cpp:90-92).  Arithmetic is fp32 in every case, as there. */
typedef enum dg_dtype {
    DG_DTYPE_F32 = 0,
    DG_DTYPE_F64 = 1,
    DG_DTYPE_F16 = 2,
    DG_DTYPE_BF16 = 3
} dg_dtype;

typedef enum dg_status {
    DG_OK = 0,
    DG_ERR_INVALID_ARGUMENT = -1, /* null pointer, non-positive size, unknown dtype */
    DG_ERR_UNSUPPORTED = -2,      /* shape/dtype combination no kernel covers */
    DG_ERR_MISALIGNED = -3,       /* a pointer lacks the alignment the kernel needs */
    DG_ERR_WORKSPACE = -4,        /* workspace missing or smaller than *_workspace_size */
    DG_ERR_CUDA = -5,             /* CUDA launch/runtime error (dg_last_cuda_error) */
    DG_ERR_DEVICE_CHECK = -6,     /* a kernel's own check tripped (dg_read_device_status) */
    DG_ERR_FORMAT = -7            /* an engine file unreadable, truncated or inconsistent */
} dg_status;

/* dense-forward algorithm selector for dg_dense_forward_ex */
typedef enum dg_dense_algo {
    DG_DENSE_AUTO = 0,       /* chunkwise tensor-core kernel where it applies (f16; bf16 up to
                                256 slots), else sequential */
    DG_DENSE_SEQUENTIAL = 1, /* CUDA-core recurrence, S resident for all T (any dtype) */
    DG_DENSE_CHUNKED_TC = 2, /* chunkwise WY/UT form on tcgen05, state columns on TMEM lanes
                                (f16/bf16, Dh = 64, slots 128/256/384/512) */
    DG_DENSE_CHUNKED_TC_ROWS = 3 /* the same algebra with state rows on TMEM lanes (the
                                    earlier layout; kept as a second GPU reference) */
} dg_dense_algo;

/* PKM sequence-forward kernel selector for dg_pkm_forward_ex */
typedef enum dg_pkm_algo {
    DG_PKM_AUTO = 0,             /* warp-specialised, else pipelined, else one step at a time */
    DG_PKM_ONE_STEP = 1,         /* one CTA per lane and part, one step per iteration (any dtype) */
    DG_PKM_PIPELINED = 2,        /* rows gathered D steps ahead by the column warps (f16/bf16/f32) */
    DG_PKM_WARP_SPECIALIZED = 3  /* producer / tensor-core GEMV / update warps (f16/bf16) */
} dg_pkm_algo;

/* bits written into the optional device status word by kernel self-checks */
#define DG_DEVCHK_INDEX_RANGE 0x1 /* a slot index was outside [0, total_slots) */
#define DG_DEVCHK_DUPLICATE 0x2   /* reserved */
#define DG_DEVCHK_TIMEOUT 0x4     /* a bounded wait on an mbarrier gave up (results invalid) */

const char* dg_status_string(int status);
int dg_abi_version(void);
/* cudaError_t value of the most recent DG_ERR_CUDA on this host thread */
int dg_last_cuda_error(void);

/*
 * Dense sequence forward.
 * Replaces launch_delta_grid_forward (src/cpp/delta_kernel.cu:563-622) and the
 * kernels it launches (:34-122, :127-218); same semantics as
 * delta_grid_forward_binding (src/cpp/binding.cpp:36-113).
 *   v [B,H,T,Dh]  beta [B,H,T]  wk,wq [B,H,T,slots]
 *   decay [H] (dynamic_decay = 0) or [B,H,T] (dynamic_decay = 1)
 *   s_init [B,H,slots,Dh] or NULL (zero state)
 *   out [B,H,T,Dh]  s_final [B,H,slots,Dh]      (storage dtype)
 *   err_out [B,H,T,Dh] fp32 residuals r_t, or NULL
 *   s_final_f [B,H,slots,Dh] fp32 final state, or NULL
 * The state stays fp32 for all T and is cast once at the end (delta_kernel.cu:64-121).
 */
int dg_dense_forward(int dtype, int B, int H, int T, int slots, int dh,
                     const void* v, const void* beta, const void* wk, const void* wq,
                     const void* decay, int dynamic_decay, const void* s_init,
                     void* out, void* s_final, float* err_out, float* s_final_f,
                     void* stream);

/* dg_dense_forward with an explicit algorithm (dg_dense_algo). */
int dg_dense_forward_ex(int dtype, int B, int H, int T, int slots, int dh,
                        const void* v, const void* beta, const void* wk, const void* wq,
                        const void* decay, int dynamic_decay, const void* s_init,
                        void* out, void* s_final, float* err_out, float* s_final_f,
                        int algo, void* stream);

/* dg_dense_forward_ex with a device status word (or NULL) into which the tensor-core
 * kernel ORs DG_DEVCHK_TIMEOUT when one of its bounded waits gives up.  Same
 * reference interface as dg_dense_forward (binding.cpp:36-113). */
int dg_dense_forward_ex2(int dtype, int B, int H, int T, int slots, int dh,
                         const void* v, const void* beta, const void* wk, const void* wq,
                         const void* decay, int dynamic_decay, const void* s_init,
                         void* out, void* s_final, float* err_out, float* s_final_f,
                         int32_t* dev_status, int algo, void* stream);

/* Poll budget of the bounded waits inside the tensor-core dense kernel and the
 * warp-specialised PKM kernel (launches made after the call).  Default 4194304 polls,
 * seconds of waiting; 0 makes every such wait give up at once, which drives the
 * kernels' timeout path (DG_DEVCHK_TIMEOUT, results invalid) without a hung wait.
 * Returns the previous value.  No reference counterpart (the reference kernels have
 * no waits). */
unsigned int dg_set_wait_limit(unsigned int polls);

/*
 * Dense single decode step with (batch, head) element strides.
 * Replaces launch_delta_grid_step (src/cpp/delta_kernel.cu:624-695) and the
 * kernels :223-351; same semantics as delta_grid_step_binding (binding.cpp:130-203).
 *   v [B,H,Dh] (strides v_sb, v_sh; last dim contiguous)  beta [B,H]
 *   wk,wq [B,H,slots] (last dim contiguous)
 *   decay [H] contiguous, or [B,H] with strides (dynamic_decay = 1)
 *   s_prev, s_next [B,H,slots,Dh] contiguous; s_next may equal s_prev (in place)
 *   out [B,H,Dh] contiguous
 */
int dg_dense_step(int dtype, int B, int H, int slots, int dh,
                  const void* v, int64_t v_sb, int64_t v_sh,
                  const void* beta, int64_t beta_sb, int64_t beta_sh,
                  const void* wk, int64_t wk_sb, int64_t wk_sh,
                  const void* wq, int64_t wq_sb, int64_t wq_sh,
                  const void* decay, int dynamic_decay, int64_t decay_sb, int64_t decay_sh,
                  const void* s_prev, void* out, void* s_next, void* stream);

/*
 * Sparse Delta-PKM sequence forward, state updated in place.
 * Replaces launch_delta_grid_pkm_forward (src/cpp/delta_kernel.cu:923-944) and
 * delta_pkm_sequence_forward_kernel (:862-921); same semantics as
 * delta_pkm_forward_binding (binding.cpp:375-434).
 *   v [B,H,T,Dh] beta [B,H,T] wk,wq [B,H,T,active] idx [B,H,T,active] (int64)
 *   decay [H] or [B,H,T];  state [B,H,total_slots,Dh] (in place)
 *   out [B,H,T,Dh];  saved_s_act [B,H,T,active,Dh] gathered rows, or NULL
 *   dev_status: optional device int32; kernels OR DG_DEVCHK_* bits into it.
 * Touched rows are stored (rounded to the storage dtype) after every step,
 * as in the reference (delta_kernel.cu:918).  Slot indices outside
 * [0, total_slots) are skipped (the row reads as zero and is not written) and
 * flagged in dev_status.  Indices repeated within one step are not supported,
 * as in the reference.
 */
int dg_pkm_forward(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                   const void* v, const void* beta, const void* wk, const void* wq,
                   const int64_t* idx, const void* decay, int dynamic_decay,
                   void* state, void* out, void* saved_s_act, int32_t* dev_status,
                   void* stream);

/* Bytes of device workspace dg_pkm_forward_ex needs for this shape and kernel
 * choice (0: none).  The warp-specialised kernel stores a 16-bit hazard code per
 * row in it: B*H*T*64*2 bytes.  Call-independent; no GPU work. */
size_t dg_pkm_forward_workspace_size(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                                     int algo);

/* dg_pkm_forward with an explicit kernel choice (dg_pkm_algo) and an optional
 * caller-owned workspace (16-byte aligned, at least
 * dg_pkm_forward_workspace_size bytes; DG_ERR_WORKSPACE otherwise).  With
 * workspace == NULL a kernel that needs one takes it from the device's default
 * memory pool, stream-ordered (cudaMallocAsync / cudaFreeAsync on `stream`).
 * DG_ERR_UNSUPPORTED when the chosen kernel does not cover the call.
 * dg_pkm_forward is this call with DG_PKM_AUTO and no workspace. */
int dg_pkm_forward_ex(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                      const void* v, const void* beta, const void* wk, const void* wq,
                      const int64_t* idx, const void* decay, int dynamic_decay,
                      void* state, void* out, void* saved_s_act, int32_t* dev_status,
                      int algo, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Dense analytic backward.  Replaces delta_grid_bwd_kernel / launch_delta_grid_backward
 * (src/cpp/delta_kernel.cu:364-558, :698-731); same call as delta_grid_backward_binding
 * (binding.cpp:223-312).  s_final and err_saved are the fp32 final state and residuals
 * that dg_dense_forward writes when asked (s_final_f / err_out).  grad_s_final and
 * grad_s_init may be NULL.  A static [H] decay gets grad_decay[h] += the head's sum, so
 * the caller zeroes it first.  workspace: dg_dense_backward_workspace_size() bytes of
 * fp32 (the state and its adjoint when they do not fit on chip), else NULL.
 */
size_t dg_dense_backward_workspace_size(int B, int H, int slots, int dh);
int dg_dense_backward(int dtype, int B, int H, int T, int slots, int dh,
                      const void* grad_out, const void* grad_s_final, const void* v,
                      const void* beta, const void* wk, const void* wq, const void* decay,
                      int dynamic_decay, const float* s_final, const float* err_saved,
                      void* grad_v, void* grad_beta, void* grad_wk, void* grad_wq,
                      void* grad_decay, void* grad_s_init, float* workspace, void* stream);

/*
 * Sparse Delta-PKM analytic backward.  Replaces delta_pkm_sequence_backward_kernel /
 * launch_delta_grid_pkm_backward (src/cpp/delta_kernel.cu:971-1102); same call as
 * delta_pkm_backward_binding (binding.cpp:439-518).  grad_state [B,H,total,Dh] holds
 * grad_final_state (or zeros) on entry and the gradient of the initial state on return.
 * saved_s_act is the [B,H,T,active,Dh] rows dg_pkm_forward saved.  grad_decay may be
 * NULL (not requested); a static [H] decay gets grad_decay[h] += the head's sum (the
 * reference leaves that output unwritten), so the caller zeroes it first.  active <= 64,
 * dh <= 128.  Indices out of range are skipped and set DG_DEVCHK_INDEX_RANGE.
 */
int dg_pkm_backward(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                    const void* grad_out, const void* v, const void* beta, const void* wk,
                    const void* wq, const int64_t* idx, const void* decay, int dynamic_decay,
                    const void* saved_s_act, void* grad_state, void* grad_v, void* grad_beta,
                    void* grad_wk, void* grad_wq, void* grad_decay, int32_t* dev_status,
                    void* stream);

/* dg_pkm_forward that allocates nothing (no reference counterpart).  For callers
 * that may not allocate device memory while the recurrence runs: a serving loop
 * whose memory is reserved up front and must not grow or fragment between
 * requests, or code under a memory manager or in a context that forbids
 * allocation.  Scratch comes from a fixed 16 MiB device array inside this
 * library.  Set-up: every call made outside stream capture (its device current)
 * looks up the array's address there and caches it; a call made under capture uses
 * the cached address, so make the first call on a device before any stream capture.
 * A device reset can move the array; the next uncaptured call picks up its new
 * address (a capture recorded before the reset holds the old one).  Calls needing
 * more scratch than the array holds
 * (dg_pkm_forward_workspace_size > 16 MiB, i.e. B*H*T > 131072 on the
 * warp-specialised kernel) return DG_ERR_WORKSPACE without launching.  Calls that
 * overlap in time on one device share the array and race: serialize them. */
int dg_pkm_forward_noalloc(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                           const void* v, const void* beta, const void* wk, const void* wq,
                           const int64_t* idx, const void* decay, int dynamic_decay,
                           void* state, void* out, void* saved_s_act, int32_t* dev_status,
                           void* stream);

/*
 * Sparse Delta-PKM single decode step, state updated in place.
 * Replaces launch_delta_grid_pkm_step (src/cpp/delta_kernel.cu:829-847) and
 * delta_pkm_step_kernel (:776-827); same call as delta_grid_pkm_step_binding
 * (binding.cpp:319-370).  decay is [H], or [B,H] when dynamic_decay = 1; the
 * reference kernel reads decay[h] even for a [B,H] tensor (:795), this entry
 * point uses the per-batch value as the PyTorch path does (memory.py:582-591).
 */
int dg_pkm_step(int dtype, int B, int H, int active, int64_t total_slots, int dh,
                const void* v, const void* beta, const void* wk, const void* wq,
                const int64_t* idx, const void* decay, int dynamic_decay,
                void* state, void* out, int32_t* dev_status, void* stream);

/*
 * Q16.16 fixed-point recurrence core, bit-exact with the reference engine's
 * integer mode.  Replaces the dense loops of dg_memory_layer_step_fxp
 * (src/cpp/engine/src/deltagrid_fxp.cpp:380-405) applied once per step.
 * Lanes-first int32 layouts (one lane = one (context, head) of the engine):
 *   wk, wq [lanes,T,slots] (wq already multiplied by q_scale, :376-378)
 *   v, y [lanes,T,dh]; beta, alpha [lanes,T]; state [lanes,slots,dh] (in place)
 */
int dg_fxp_dense_forward(int lanes, int T, int slots, int dh, const int32_t* wk, const int32_t* wq,
                         const int32_t* v, const int32_t* beta, const int32_t* alpha, int32_t* state,
                         int32_t* y, void* stream);

/*
 * Q16.16 sparse PKM recurrence core, bit-exact with deltagrid_fxp.cpp:298-326.
 *   wk, wq, idx [lanes,T,active] int32 (active <= 64); state [lanes,total_slots,dh]
 *   in place (dh a multiple of 4, 16-byte aligned).  Out-of-range indices are
 *   skipped and flagged in dev_status (DG_DEVCHK_INDEX_RANGE).
 */
int dg_fxp_pkm_forward(int lanes, int T, int active, int64_t total_slots, int dh, const int32_t* wk,
                       const int32_t* wq, const int32_t* idx, const int32_t* v, const int32_t* beta,
                       const int32_t* alpha, int32_t* state, int32_t* y, int32_t* dev_status, void* stream);

/*
 * Dense slot routing, one kernel (tcgen05): wk = L2-normalise(k P_k^T) and
 * wq = (q P_q^T) * q_scale[h].  Replaces DeltaGridLayer._route_dense's linear-projection
 * branch (src/modules/memory.py:233-236, bias-free nn.Linear slot projections, :192-193)
 * and the q_scale multiply of memory.py:490-492.
 *   k, q [B,H,T,dh] (storage dtype `dtype`: f16 or bf16; dh = 64)
 *   slot_proj_k, slot_proj_q [slots, dh] (the nn.Linear weights, same dtype; slots a
 *   multiple of 64 up to 512);  q_scale [H] fp32 or NULL
 *   wk, wq [B,H,T,slots] (same dtype); every pointer 16-byte aligned
 * The products accumulate in fp32; the norm is the fp32 sum of squares, eps 1e-12 as
 * F.normalize; each output is rounded once.  Other shapes: DG_ERR_UNSUPPORTED.
 * dev_status (or NULL) gets DG_DEVCHK_TIMEOUT if a bounded wait gave up.
 */
int dg_dense_route(int dtype, int B, int H, int T, int dh, int slots, const void* k, const void* q,
                   const void* slot_proj_k, const void* slot_proj_q, const float* q_scale, void* wk, void* wq,
                   int32_t* dev_status, void* stream);

/*
 * Two-axis product-key router for Sparse Delta-PKM, fused (one kernel).
 * Replaces DeltaGridLayer._route_sparse_pkm (src/modules/memory.py:240-289) for two
 * axes without subspace slicing, and the q_scale multiply of memory.py:453-455.
 *   k, q [B,H,T,dh] (storage dtype `dtype`, dh <= 128)
 *   router_k0/router_q0 [g0,dh], router_k1/router_q1 [g1,dh] fp32 (nn.Linear weights)
 *   q_scale [H] fp32 or NULL;  top_k <= 8
 *   wk, wq [B,H,T,top_k^2] (storage dtype), idx [B,H,T,top_k^2] int64 = i0*g1 + i1
 * Scores are fp32 dot products in increasing dh order; equal scores keep the
 * lower index first (src/cpp/engine/src/deltagrid_math.cpp:155-167).
 * The tensor-core form (16-bit k, dh = 64, top_k 4 or 8; both axes of one size of
 * 32, 64, 96 or 128 rows, or each a multiple of 128 rows) keeps a split
 * copy of the router weights in a per-device buffer allocated on first use and
 * reused by later calls, which wait for the previous call's kernels (calls under
 * stream capture allocate their copy from the stream instead).  Other shapes run
 * the CUDA-core form, with the same results.
 */
int dg_pkm_route(int dtype, int B, int H, int T, int dh, int g0, int g1, int top_k, const void* k,
                 const void* q, const float* router_k0, const float* router_k1, const float* router_q0,
                 const float* router_q1, const float* q_scale, void* wk, void* wq, int64_t* idx,
                 void* stream);

/* ---------------------------------------------------------------------------
 * The reference C++ engine's files (src/cpp/engine), read and written on the
 * host so that its weights and recurrent state can drive the GPU recurrence
 * (dg_fxp_* for Q16.16 files, dg_dense_forward / dg_pkm_forward for fp32 ones).
 * ------------------------------------------------------------------------- */

/* DeltaGridBinHeader (src/cpp/engine/include/deltagrid_internal.h:65-82) */
typedef struct dg_dlg1_header {
    int32_t magic, version, model_type, precision_mode, num_layers, d_model, num_heads, kernel_size,
        thinking_cycles, input_or_vocab, output_dim, forecast_horizon, num_axes, top_k, actual_slots, flags;
} dg_dlg1_header;

#define DG_DLG1_MAX_AXES 8

typedef enum dg_dlg1_encoding {
    DG_ENC_F32 = 0, /* fp32 */
    DG_ENC_Q8 = 1,  /* int8, value = q * scale (the fp32 scale precedes the bytes) */
    DG_ENC_Q16 = 2  /* int32 Q16.16 */
} dg_dlg1_encoding;

/* one array of a DLG1 file: names follow the engine's struct fields
   ("input_weight", "memory.decay", "memory.axes_proj_k", "ffn_fc1_weight", ...) */
typedef struct dg_dlg1_array {
    char name[32];
    int32_t layer;    /* block index, -1 outside the blocks */
    int32_t axis;     /* axis of memory.axes_proj_k / _q, else -1 */
    int32_t encoding; /* dg_dlg1_encoding */
    float scale;      /* DG_ENC_Q8 dequantisation scale, else 1 */
    int64_t offset;   /* byte offset of the first element */
    int64_t count;    /* elements */
} dg_dlg1_array;

/*
 * DLG1 weights layout.  Replaces the read order of dg_load_context_from_file
 * (src/cpp/engine/src/deltagrid_math.cpp:558-761, fp32 / int8 files) and
 * deltagrid_init_context_fxp (src/cpp/engine/src/deltagrid_fxp.cpp:503-660,
 * Q16.16 files), as written by export_deltagrid_to_bin
 * (src/cpp/engine/tools/export_deltagrid_binary.py:77-237).  Fills *hdr, grid_dim
 * (up to max_axes) and up to max_arrays entries of `arrays` (NULL: count only);
 * *n_arrays = the file's array count.  DG_ERR_FORMAT for a bad magic, precision
 * or shape, a truncated file or trailing bytes; DG_ERR_WORKSPACE when `arrays`
 * is too short.  Opens and closes the file; keeps nothing.
 */
int dg_dlg1_layout(const char* path, dg_dlg1_header* hdr, int32_t* grid_dim, int max_axes, dg_dlg1_array* arrays,
                   int max_arrays, int* n_arrays);

/* DLGS state snapshot header (the six words after the magic,
   src/cpp/engine/src/deltagrid_math.cpp:779-811) */
typedef struct dg_dlgs_header {
    int32_t num_layers, d_model, num_heads, actual_slots, kernel_size, step_count;
} dg_dlgs_header;

/* per-layer element counts: conv window d_model * max(kernel_size - 1, 1), memory
   state num_heads * actual_slots * (d_model / num_heads) */
size_t dg_dlgs_conv_elems(const dg_dlgs_header* h);
size_t dg_dlgs_mem_elems(const dg_dlgs_header* h);

/* Reads and checks the header (magic, shape, file length). */
int dg_dlgs_read_header(const char* path, dg_dlgs_header* h);

/*
 * One layer of a snapshot.  Replaces dg_load_runtime_state
 * (src/cpp/engine/src/deltagrid_math.cpp:812-844) and deltagrid_load_state_fxp
 * (deltagrid_fxp.cpp:762-795) for one layer: the file's shape must equal
 * `expect` (the step count may differ).  conv_state / mem_state (either may be
 * NULL) receive 4-byte elements: fp32 for the float engine, Q16.16 for the
 * fixed-point engine; mem_state is [num_heads, actual_slots, d_model/num_heads],
 * the lanes-first layout of the GPU kernels.
 */
int dg_dlgs_read_layer(const char* path, const dg_dlgs_header* expect, int layer, void* conv_state, void* mem_state);

/*
 * Writes a snapshot.  Replaces dg_save_runtime_state (deltagrid_math.cpp:779-810)
 * and deltagrid_save_state_fxp (deltagrid_fxp.cpp:728-760); conv_layers[l] and
 * mem_layers[l] point at layer l's states (host memory, 4-byte elements).
 */
int dg_dlgs_write(const char* path, const dg_dlgs_header* h, const void* const* conv_layers,
                  const void* const* mem_layers);

/* Reads (and clears when `clear`) a device status word; synchronizes `stream`. */
int dg_read_device_status(int32_t* dev_status, int clear, int32_t* host_value, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DELTAGRID_B200_H */
