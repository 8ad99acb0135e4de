// capi.cu -- extern "C" entry points: argument checks, algorithm choice, launches.
#include "dg_common.cuh"

namespace dg_host {

static thread_local int g_last_cuda_error = 0;
static unsigned int g_wait_limit = 1u << 22;

uint32_t wait_limit() { return __atomic_load_n(&g_wait_limit, __ATOMIC_RELAXED); }

// per-device multiprocessor counts (0 = not yet queried; the count is never 0)
static int g_sm_count[64];

int sm_count(int device, int* out) {
    if (device < 0 || device >= 64) return DG_ERR_UNSUPPORTED;
    int n = __atomic_load_n(&g_sm_count[device], __ATOMIC_RELAXED);
    if (n == 0) {
        cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
        if (e != cudaSuccess) return record_cuda_error(e);
        __atomic_store_n(&g_sm_count[device], n, __ATOMIC_RELAXED);
    }
    *out = n;
    return DG_OK;
}

int record_cuda_error(cudaError_t e) {
    g_last_cuda_error = (int)e;
    return DG_ERR_CUDA;
}

// kernels implemented in the other translation units
int dense_forward_sequential(int dtype, int B, int H, int T, int S, int Dh, const void* v,
                             const void* beta, const void* wk, const void* wq, const void* decay,
                             int dynamic_decay, const void* s_init, void* out, void* s_final,
                             float* err_out, float* s_final_f, cudaStream_t stream);
int dense_forward_chunked_tc(int dtype, int B, int H, int T, int S, int Dh, const void* v,
                             const void* beta, const void* wk, const void* wq, const void* decay,
                             int dynamic_decay, const void* s_init, void* out, void* s_final,
                             float* err_out, float* s_final_f, cudaStream_t stream);
bool dense_chunked_tc_supports(int dtype, int B, int H, int T, int S, int Dh);
int dense_forward_chunked_t(int dtype, int B, int H, int T, int S, int Dh, const void* v, const void* beta,
                            const void* wk, const void* wq, const void* decay, int dynamic_decay, const void* s_init,
                            void* out, void* s_final, float* err_out, float* s_final_f, int32_t* status,
                            cudaStream_t stream);
int dense_step(int dtype, int B, int H, int S, int Dh, const void* v, int64_t v_sb, int64_t v_sh,
               const void* beta, int64_t beta_sb, int64_t beta_sh, const void* wk, int64_t wk_sb,
               int64_t wk_sh, const void* wq, int64_t wq_sb, int64_t wq_sh, const void* decay,
               int dynamic_decay, int64_t decay_sb, int64_t decay_sh, const void* s_prev,
               void* out, void* s_next, cudaStream_t stream);
int pkm_forward_v1(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v,
                   const void* beta, const void* wk, const void* wq, const int64_t* idx,
                   const void* decay, int dynamic_decay, void* state, void* out, void* saved,
                   int32_t* status, cudaStream_t stream);
bool pkm_pipe_supports(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v,
                       const void* beta, const void* wk, const void* wq, const void* idx, const void* decay,
                       int dynamic_decay, const void* state, const void* saved);
int pkm_forward_pipe(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v, const void* beta,
                     const void* wk, const void* wq, const int64_t* idx, const void* decay, int dynamic_decay,
                     void* state, void* out, int32_t* status, cudaStream_t stream);
bool pkm_ws_supports(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v, const void* beta,
                     const void* wk, const void* wq, const void* idx, const void* decay, int dynamic_decay,
                     const void* state, const void* saved);
int pkm_forward_ws(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v, const void* beta,
                   const void* wk, const void* wq, const int64_t* idx, const void* decay, int dynamic_decay,
                   void* state, void* out, void* saved, int32_t* status, void* workspace, cudaStream_t stream);
size_t pkm_ws_workspace_bytes(int B, int H, int T);

}  // namespace dg_host

using namespace dg_host;

static bool valid_dtype(int d) { return d >= DG_DTYPE_F32 && d <= DG_DTYPE_BF16; }

extern "C" {

const char* dg_status_string(int status) {
    switch (status) {
    case DG_OK: return "ok";
    case DG_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DG_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case DG_ERR_MISALIGNED: return "misaligned pointer";
    case DG_ERR_WORKSPACE: return "workspace missing or too small";
    case DG_ERR_CUDA: return "CUDA error";
    case DG_ERR_DEVICE_CHECK: return "device-side check failed";
    case DG_ERR_FORMAT: return "engine file unreadable, truncated or inconsistent";
    default: return "unknown status";
    }
}

int dg_abi_version(void) { return DG_ABI_VERSION; }

int dg_last_cuda_error(void) { return g_last_cuda_error; }

int dg_dense_forward_ex(int dtype, int B, int H, int T, int slots, int dh, const void* v,
                        const void* beta, const void* wk, const void* wq, const void* decay,
                        int dynamic_decay, const void* s_init, void* out, void* s_final,
                        float* err_out, float* s_final_f, int algo, void* stream) {
    return dg_dense_forward_ex2(dtype, B, H, T, slots, dh, v, beta, wk, wq, decay, dynamic_decay, s_init, out,
                                s_final, err_out, s_final_f, nullptr, algo, stream);
}

unsigned int dg_set_wait_limit(unsigned int polls) {
    return __atomic_exchange_n(&g_wait_limit, polls, __ATOMIC_RELAXED);
}

int dg_dense_forward_ex2(int dtype, int B, int H, int T, int slots, int dh, const void* v,
                         const void* beta, const void* wk, const void* wq, const void* decay,
                         int dynamic_decay, const void* s_init, void* out, void* s_final,
                         float* err_out, float* s_final_f, int32_t* dev_status, int algo, void* stream) {
    if (!valid_dtype(dtype) || B <= 0 || H <= 0 || T < 0 || slots <= 0 || dh <= 0)
        return DG_ERR_INVALID_ARGUMENT;
    // with T == 0 the per-step tensors are empty (their pointers may be null):
    // only the state passes through, s_final = s_init (or zeros)
    if (!decay || !s_final || (T > 0 && (!v || !beta || !wk || !wq || !out)))
        return DG_ERR_INVALID_ARGUMENT;
    if ((int64_t)B * H > 65535) return DG_ERR_UNSUPPORTED;      // grid.y limit
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (T == 0) algo = DG_DENSE_SEQUENTIAL;
    const bool tc_ok = dense_chunked_tc_supports(dtype, B, H, T, slots, dh);
    if ((algo == DG_DENSE_CHUNKED_TC || algo == DG_DENSE_CHUNKED_TC_ROWS) && !tc_ok) return DG_ERR_UNSUPPORTED;
    // AUTO keeps bf16 states of more than 256 slots on the sequential kernel: there the
    // tensor-core kernels take single bf16 copies of the state and residual operands,
    // ~2e-3 from an fp32-state recurrence, outside the 1e-3 bar (at <= 256 slots the
    // default kernel carries them as bf16 hi + lo pairs)
    const bool tc_auto = tc_ok && !(dtype == DG_DTYPE_BF16 && slots > 256);
    if (algo == DG_DENSE_CHUNKED_TC || (algo == DG_DENSE_AUTO && tc_auto))
        return dense_forward_chunked_t(dtype, B, H, T, slots, dh, v, beta, wk, wq, decay, dynamic_decay, s_init,
                                       out, s_final, err_out, s_final_f, dev_status, s);
    if (algo == DG_DENSE_CHUNKED_TC_ROWS)
        return dense_forward_chunked_tc(dtype, B, H, T, slots, dh, v, beta, wk, wq, decay,
                                        dynamic_decay, s_init, out, s_final, err_out, s_final_f, s);
    if (algo != DG_DENSE_AUTO && algo != DG_DENSE_SEQUENTIAL) return DG_ERR_INVALID_ARGUMENT;
    return dense_forward_sequential(dtype, B, H, T, slots, dh, v, beta, wk, wq, decay, dynamic_decay,
                                    s_init, out, s_final, err_out, s_final_f, s);
}

int dg_dense_forward(int dtype, int B, int H, int T, int slots, int dh, const void* v,
                     const void* beta, const void* wk, const void* wq, const void* decay,
                     int dynamic_decay, const void* s_init, void* out, void* s_final,
                     float* err_out, float* s_final_f, void* stream) {
    return dg_dense_forward_ex(dtype, B, H, T, slots, dh, v, beta, wk, wq, decay, dynamic_decay,
                               s_init, out, s_final, err_out, s_final_f, DG_DENSE_AUTO, stream);
}

int dg_dense_step(int dtype, int B, int H, int slots, int dh, const void* v, int64_t v_sb,
                  int64_t v_sh, const void* beta, int64_t beta_sb, int64_t beta_sh, const void* wk,
                  int64_t wk_sb, int64_t wk_sh, const void* wq, int64_t wq_sb, int64_t wq_sh,
                  const void* decay, int dynamic_decay, int64_t decay_sb, int64_t decay_sh,
                  const void* s_prev, void* out, void* s_next, void* stream) {
    if (!valid_dtype(dtype) || B <= 0 || H <= 0 || slots <= 0 || dh <= 0) return DG_ERR_INVALID_ARGUMENT;
    if (!v || !beta || !wk || !wq || !decay || !s_prev || !out || !s_next) return DG_ERR_INVALID_ARGUMENT;
    if ((int64_t)B * H > 65535) return DG_ERR_UNSUPPORTED;
    return dense_step(dtype, B, H, slots, dh, v, v_sb, v_sh, beta, beta_sb, beta_sh, wk, wk_sb, wk_sh,
                      wq, wq_sb, wq_sh, decay, dynamic_decay, decay_sb, decay_sh, s_prev, out, s_next,
                      static_cast<cudaStream_t>(stream));
}

size_t dg_pkm_forward_workspace_size(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                                     int algo) {
    if (!valid_dtype(dtype) || B <= 0 || H <= 0 || T <= 0 || active <= 0 || total_slots <= 0 || dh <= 0) return 0;
    if (algo != DG_PKM_AUTO && algo != DG_PKM_WARP_SPECIALIZED) return 0;
    if (algo == DG_PKM_AUTO && T < 64) return 0;
    // shape-level check only (alignment is not known here): 16-byte-aligned placeholder pointers
    const void* a = reinterpret_cast<const void*>(uintptr_t(256));
    if (!pkm_ws_supports(dtype, B, H, T, active, total_slots, dh, a, a, a, a, a, a, 0, a, a)) return 0;
    return pkm_ws_workspace_bytes(B, H, T);
}

int dg_pkm_forward_ex(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                      const void* v, const void* beta, const void* wk, const void* wq,
                      const int64_t* idx, const void* decay, int dynamic_decay, void* state, void* out,
                      void* saved_s_act, int32_t* dev_status, int algo, void* workspace,
                      size_t workspace_bytes, void* stream) {
    if (!valid_dtype(dtype) || B <= 0 || H <= 0 || T < 0 || active <= 0 || total_slots <= 0 || dh <= 0)
        return DG_ERR_INVALID_ARGUMENT;
    if (algo < DG_PKM_AUTO || algo > DG_PKM_WARP_SPECIALIZED) return DG_ERR_INVALID_ARGUMENT;
    if (!state) return DG_ERR_INVALID_ARGUMENT;
    if (T == 0) return DG_OK;              // nothing to do; per-step tensors may be empty
    if (!v || !beta || !wk || !wq || !idx || !decay || !out) return DG_ERR_INVALID_ARGUMENT;
    if ((int64_t)B * H > 65535) return DG_ERR_UNSUPPORTED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool ws = pkm_ws_supports(dtype, B, H, T, active, total_slots, dh, v, beta, wk, wq, idx, decay,
                                    dynamic_decay, state, saved_s_act);
    const bool pipe = pkm_pipe_supports(dtype, B, H, T, active, total_slots, dh, v, beta, wk, wq, idx, decay,
                                        dynamic_decay, state, saved_s_act);
    if (algo == DG_PKM_AUTO) {
        // long sequences: the warp-specialised kernel (16-bit state) or the
        // pipelined one; decode steps, saved rows and other shapes: one step at a time
        algo = T < 64 ? DG_PKM_ONE_STEP : ws ? DG_PKM_WARP_SPECIALIZED : pipe ? DG_PKM_PIPELINED : DG_PKM_ONE_STEP;
    }
    if (algo == DG_PKM_WARP_SPECIALIZED) {
        if (!ws) return DG_ERR_UNSUPPORTED;
        const size_t need = pkm_ws_workspace_bytes(B, H, T);
        if (workspace) {
            if (workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15)) return DG_ERR_WORKSPACE;
            return pkm_forward_ws(dtype, B, H, T, active, total_slots, dh, v, beta, wk, wq, idx, decay,
                                  dynamic_decay, state, out, saved_s_act, dev_status, workspace, s);
        }
        // no caller workspace: stream-ordered allocation from the device's default pool
        void* w = nullptr;
        cudaError_t e = cudaMallocAsync(&w, need, s);
        if (e != cudaSuccess) return record_cuda_error(e);
        const int rc = pkm_forward_ws(dtype, B, H, T, active, total_slots, dh, v, beta, wk, wq, idx, decay,
                                      dynamic_decay, state, out, saved_s_act, dev_status, w, s);
        e = cudaFreeAsync(w, s);
        if (rc != DG_OK) return rc;
        return e == cudaSuccess ? DG_OK : record_cuda_error(e);
    }
    if (algo == DG_PKM_PIPELINED) {
        if (!pipe) return DG_ERR_UNSUPPORTED;
        return pkm_forward_pipe(dtype, B, H, T, active, total_slots, dh, v, beta, wk, wq, idx, decay,
                                dynamic_decay, state, out, dev_status, s);
    }
    return pkm_forward_v1(dtype, B, H, T, active, total_slots, dh, v, beta, wk, wq, idx, decay,
                          dynamic_decay, state, out, saved_s_act, dev_status, s);
}

int dg_pkm_forward(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                   const void* v, const void* beta, const void* wk, const void* wq,
                   const int64_t* idx, const void* decay, int dynamic_decay, void* state, void* out,
                   void* saved_s_act, int32_t* dev_status, void* stream) {
    return dg_pkm_forward_ex(dtype, B, H, T, active, total_slots, dh, v, beta, wk, wq, idx, decay,
                             dynamic_decay, state, out, saved_s_act, dev_status, DG_PKM_AUTO, nullptr, 0, stream);
}

int dg_pkm_step(int dtype, int B, int H, int active, int64_t total_slots, int dh, const void* v,
                const void* beta, const void* wk, const void* wq, const int64_t* idx,
                const void* decay, int dynamic_decay, void* state, void* out, int32_t* dev_status,
                void* stream) {
    // a decode step is the sequence kernel with T = 1 ([B,H] decay == [B,H,1])
    return dg_pkm_forward(dtype, B, H, 1, active, total_slots, dh, v, beta, wk, wq, idx, decay,
                          dynamic_decay, state, out, nullptr, dev_status, stream);
}

int dg_read_device_status(int32_t* dev_status, int clear, int32_t* host_value, void* stream) {
    if (!dev_status || !host_value) return DG_ERR_INVALID_ARGUMENT;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(host_value, dev_status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(dev_status, 0, sizeof(int32_t), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? DG_OK : record_cuda_error(e);
}

}  // extern "C"
