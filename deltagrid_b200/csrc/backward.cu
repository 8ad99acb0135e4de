// backward.cu -- analytical backward passes of the dense and Sparse Delta-PKM
// recurrences (the reference's delta_grid_bwd_kernel, src/cpp/delta_kernel.cu:364-558,
// and delta_pkm_sequence_backward_kernel, :971-1072), walked backward in time.
//
// Dense.  With r_t the saved fp32 residuals and S_T the exact fp32 final state,
// step t (from T-1 down to 0) reconstructs S_{t-1} = (S_t - beta_t wk_t r_t^T) / alpha_t
// and carries the adjoint G (dL/dS_t, initialised from grad_s_final):
//     gr_d     = beta_t sum_m wk_tm G_md                      (grad_v_t = gr)
//     dwq_tm   = sum_d dy_td S_{t-1,md}
//     dwk_tm   = sum_d (beta_t G_md r_td - gr_d S_{t-1,md})
//     dbeta_t  = sum_md wk_tm r_td G_md,   dalpha_t = sum_md G_md S_{t-1,md}
//     G       <- alpha_t G + wq_t dy_t^T - wk_t gr^T
// grad_s_init = G after step 0; a static [H] decay gets the sum of dalpha over the
// lanes of the head.  One CTA per lane, eight warps; warp w owns a contiguous range
// of slots and lanes own columns.  The per-slot sums over columns are formed 16
// slots at a time with a transpose-reduce (16 shuffles for 16 slots) instead of one
// butterfly per slot.  S and G are fp32, in shared memory when both fit, else in a
// caller-provided fp32 workspace.
//
// PKM.  The adjoint state G (storage dtype, [B,H,total,Dh], initialised by the caller
// from grad_final_state or zeros) is gathered at the step's active rows, and with the
// rows s as the forward gathered them (saved_s_act):
//     r_d = v_d - sum_m wk_m s_md,   u_d = sum_m wk_m g_md      (grad_v = beta u)
//     dbeta = sum_d u_d r_d,  dwq_m = sum_d s_md dy_d,  dwk_m = beta sum_d (g_md r_d - s_md u_d)
//     g_md <- alpha g_md - beta wk_m u_d + wq_m dy_d             (rounded to storage)
//     dalpha = sum_md s_md g_md
// One CTA per lane; warp w owns rows w, w+8, ...; lanes own columns.  All rows are
// read before any is written back, so two active entries with the same slot in one
// step (which routing never produces) see the same adjoint row.
#include "dg_common.cuh"

namespace {

constexpr int BWD_THREADS = 256;
constexpr int BWD_WARPS = BWD_THREADS / 32;
constexpr size_t kDenseSmemMax = 220 * 1024;

// Transpose-reduce: 16 values per lane -> lanes l and l ^ 16 hold the warp-wide sum of
// value (l & 15) (4 halving stages and one cross-half add: 16 shuffles for 16 sums)
template <int HALF>
__device__ __forceinline__ void tr_stage(float (&v)[16], int lane) {
    const bool up = (lane & HALF) != 0;
#pragma unroll
    for (int i = 0; i < HALF; ++i) {
        const float send = up ? v[i] : v[i + HALF];
        const float keep = up ? v[i + HALF] : v[i];
        v[i] = keep + __shfl_xor_sync(DG_FULL_MASK, send, HALF);
    }
}
__device__ __forceinline__ float transpose_reduce(float (&v)[16], int lane) {
    tr_stage<8>(v, lane);
    tr_stage<4>(v, lane);
    tr_stage<2>(v, lane);
    tr_stage<1>(v, lane);
    return v[0] + __shfl_xor_sync(DG_FULL_MASK, v[0], 16);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(DG_FULL_MASK, x, o);
    return x;
}

// block-wide sum of one value per thread; every thread gets the total
__device__ __forceinline__ float block_sum(float x, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    x = warp_sum(x);
    __syncthreads();
    if (lane == 0) red[warp] = x;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < BWD_WARPS; ++w) t += red[w];
    return t;
}

template <typename T> __device__ __forceinline__ void atomic_add_out(T* p, float x);
template <> __device__ __forceinline__ void atomic_add_out<float>(float* p, float x) { atomicAdd(p, x); }
template <> __device__ __forceinline__ void atomic_add_out<double>(double* p, float x) { atomicAdd(p, (double)x); }
template <> __device__ __forceinline__ void atomic_add_out<__half>(__half* p, float x) { atomicAdd(p, __float2half_rn(x)); }
template <> __device__ __forceinline__ void atomic_add_out<__nv_bfloat16>(__nv_bfloat16* p, float x) {
    atomicAdd(p, __float2bfloat16_rn(x));
}

struct DenseBwdParams {
    const void *grad_out, *grad_s_final, *beta, *wk, *wq, *decay;
    const float *s_final, *err_saved;
    void *grad_v, *grad_beta, *grad_wk, *grad_wq, *grad_decay, *grad_s_init;
    float* workspace;                 // [lanes][2][slots][dh] fp32, or null when on chip
    int H, T, S, Dh, dynamic_decay;
};

template <typename T>
__global__ void __launch_bounds__(BWD_THREADS, 1) dense_bwd_kernel(DenseBwdParams p) {
    extern __shared__ __align__(16) float sm[];
    const int S = p.S, Dh = p.Dh, T_ = p.T;
    const int lane_bh = blockIdx.x, h = lane_bh % p.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t st_off = (int64_t)lane_bh * S * Dh;
    const bool on_chip = p.workspace == nullptr;
    float* st = on_chip ? sm : p.workspace + (int64_t)lane_bh * 2 * S * Dh;   // S_t    [S][Dh]
    float* gt = st + (int64_t)S * Dh;                                          // G      [S][Dh]
    float* vec = on_chip ? sm + 2 * S * Dh : sm;
    float* dy = vec;                  // [Dh]
    float* rr = dy + Dh;              // [Dh]  r_t
    float* gr = rr + Dh;              // [Dh]  beta sum_m wk G
    float* wks = gr + Dh;             // [S]
    float* wqs = wks + S;             // [S]
    float* part = wqs + S;            // [BWD_WARPS][Dh]
    float* red = part + BWD_WARPS * Dh;   // [BWD_WARPS]
    const T* grad_out = static_cast<const T*>(p.grad_out);
    const T* gsf = static_cast<const T*>(p.grad_s_final);
    const T* beta = static_cast<const T*>(p.beta);
    const T* wk = static_cast<const T*>(p.wk);
    const T* wq = static_cast<const T*>(p.wq);
    const T* decay = static_cast<const T*>(p.decay);

    for (int i = tid; i < S * Dh; i += BWD_THREADS) {
        st[i] = p.s_final[st_off + i];
        gt[i] = gsf ? dg::to_f(gsf[st_off + i]) : 0.f;
    }
    const float alpha_static = p.dynamic_decay ? 1.f : dg::to_f(decay[h]);
    const int spw = (S + BWD_WARPS - 1) / BWD_WARPS;          // slots of this warp: [m0, m1)
    const int m0 = min(S, warp * spw), m1 = min(S, m0 + spw);
    float decay_acc = 0.f;
    __syncthreads();

    for (int t = T_ - 1; t >= 0; --t) {
        const int64_t bt_i = (int64_t)lane_bh * T_ + t;
        const float alpha = p.dynamic_decay ? dg::to_f(decay[bt_i]) : alpha_static;
        const float inv_alpha = alpha != 0.f ? 1.f / alpha : 0.f;
        const float bt = dg::to_f(beta[bt_i]);
        for (int d = tid; d < Dh; d += BWD_THREADS) {
            dy[d] = dg::to_f(grad_out[bt_i * Dh + d]);
            rr[d] = p.err_saved[bt_i * Dh + d];
        }
        for (int m = tid; m < S; m += BWD_THREADS) {
            wks[m] = dg::to_f(wk[bt_i * S + m]);
            wqs[m] = dg::to_f(wq[bt_i * S + m]);
        }
        __syncthreads();
        // gr_d = beta sum_m wk_m G_md: per-warp partials over its slots, then across warps
        for (int d = lane; d < Dh; d += 32) {
            float a = 0.f;
            for (int m = m0; m < m1; ++m) a = fmaf(wks[m], gt[m * Dh + d], a);
            part[warp * Dh + d] = a;
        }
        __syncthreads();
        for (int d = tid; d < Dh; d += BWD_THREADS) {
            float a = 0.f;
#pragma unroll
            for (int w = 0; w < BWD_WARPS; ++w) a += part[w * Dh + d];
            gr[d] = bt * a;
            static_cast<T*>(p.grad_v)[bt_i * Dh + d] = dg::from_f<T>(bt * a);
        }
        __syncthreads();
        // slot sweep, 16 slots of this warp at a time
        float dbeta_l = 0.f, dalpha_l = 0.f;
        for (int mb = m0; mb < m1; mb += 16) {
            float pq[16], pk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                pq[j] = 0.f;
                pk[j] = 0.f;
                const int m = mb + j;
                if (m < m1) {
                    const float wkm = wks[m], wqm = wqs[m], rate = bt * wkm;
                    for (int d = lane; d < Dh; d += 32) {
                        const float r = rr[d], g = gt[m * Dh + d], y = dy[d], gd = gr[d];
                        const float sp = (st[m * Dh + d] - rate * r) * inv_alpha;
                        pq[j] = fmaf(y, sp, pq[j]);
                        pk[j] += bt * (g * r) - gd * sp;
                        dbeta_l = fmaf(wkm, r * g, dbeta_l);
                        dalpha_l = fmaf(g, sp, dalpha_l);
                        gt[m * Dh + d] = alpha * g + wqm * y - wkm * gd;
                        st[m * Dh + d] = sp;
                    }
                }
            }
            const float sq = transpose_reduce(pq, lane);
            const float sk = transpose_reduce(pk, lane);
            if (lane < 16 && mb + lane < m1) {
                static_cast<T*>(p.grad_wq)[bt_i * S + mb + lane] = dg::from_f<T>(sq);
                static_cast<T*>(p.grad_wk)[bt_i * S + mb + lane] = dg::from_f<T>(sk);
            }
        }
        const float tb = block_sum(dbeta_l, red);
        const float ta = block_sum(dalpha_l, red);
        if (tid == 0) {
            static_cast<T*>(p.grad_beta)[bt_i] = dg::from_f<T>(tb);
            if (p.dynamic_decay) static_cast<T*>(p.grad_decay)[bt_i] = dg::from_f<T>(ta);
            else decay_acc += ta;
        }
        __syncthreads();
    }
    if (!p.dynamic_decay && tid == 0) atomic_add_out<T>(static_cast<T*>(p.grad_decay) + h, decay_acc);
    if (p.grad_s_init) {
        T* gsi = static_cast<T*>(p.grad_s_init);
        for (int i = tid; i < S * Dh; i += BWD_THREADS) gsi[st_off + i] = dg::from_f<T>(gt[i]);
    }
}

struct PkmBwdParams {
    const void *grad_out, *v, *beta, *wk, *wq, *decay, *saved;
    const int64_t* idx;
    void *grad_state, *grad_v, *grad_beta, *grad_wk, *grad_wq, *grad_decay;
    int32_t* status;
    int64_t total;
    int H, T, A, Dh, dynamic_decay;
};

// RPW rows per warp (A <= 8 RPW), KD columns per lane (Dh <= 32 KD)
template <typename T, int RPW, int KD>
__global__ void __launch_bounds__(BWD_THREADS) pkm_bwd_kernel(PkmBwdParams p) {
    __shared__ float pu[BWD_WARPS][32 * KD];    // per-warp partials of pred and u
    __shared__ float pp[BWD_WARPS][32 * KD];
    __shared__ float rv[32 * KD], uv[32 * KD], yv[32 * KD];
    __shared__ float red[BWD_WARPS];
    const int A = p.A, Dh = p.Dh, T_ = p.T;
    const int lane_bh = blockIdx.x, h = lane_bh % p.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const T* grad_out = static_cast<const T*>(p.grad_out);
    const T* vv = static_cast<const T*>(p.v);
    const T* beta = static_cast<const T*>(p.beta);
    const T* wk = static_cast<const T*>(p.wk);
    const T* wq = static_cast<const T*>(p.wq);
    const T* decay = static_cast<const T*>(p.decay);
    const T* saved = static_cast<const T*>(p.saved);
    T* gstate = static_cast<T*>(p.grad_state) + (int64_t)lane_bh * p.total * Dh;
    const float alpha_static = p.dynamic_decay ? 1.f : dg::to_f(decay[h]);
    float decay_acc = 0.f;

    for (int t = T_ - 1; t >= 0; --t) {
        const int64_t bt_i = (int64_t)lane_bh * T_ + t;
        const float alpha = p.dynamic_decay ? dg::to_f(decay[bt_i]) : alpha_static;
        const float bt = dg::to_f(beta[bt_i]);
        float s[RPW][KD], g[RPW][KD], wkm[RPW], wqm[RPW];
        int64_t slot[RPW];
        float ap[KD], au[KD];
#pragma unroll
        for (int k = 0; k < KD; ++k) { ap[k] = 0.f; au[k] = 0.f; }
#pragma unroll
        for (int j = 0; j < RPW; ++j) {
            const int m = warp + BWD_WARPS * j;
            slot[j] = -1;
            wkm[j] = 0.f;
            wqm[j] = 0.f;
            if (m < A) {
                const int64_t x = p.idx[bt_i * A + m];
                if (x >= 0 && x < p.total) slot[j] = x;
                else if (lane == 0) dg::flag_status(p.status, DG_DEVCHK_INDEX_RANGE);
                wkm[j] = dg::to_f(wk[bt_i * A + m]);
                wqm[j] = dg::to_f(wq[bt_i * A + m]);
            }
#pragma unroll
            for (int k = 0; k < KD; ++k) {
                const int d = lane + 32 * k;
                s[j][k] = 0.f;
                g[j][k] = 0.f;
                if (m < A && d < Dh) {
                    s[j][k] = dg::to_f(saved[(bt_i * A + m) * Dh + d]);
                    if (slot[j] >= 0) g[j][k] = dg::to_f(gstate[slot[j] * Dh + d]);
                }
                ap[k] = fmaf(wkm[j], s[j][k], ap[k]);
                au[k] = fmaf(wkm[j], g[j][k], au[k]);
            }
        }
#pragma unroll
        for (int k = 0; k < KD; ++k) {
            pp[warp][lane + 32 * k] = ap[k];
            pu[warp][lane + 32 * k] = au[k];
        }
        __syncthreads();
        float dbeta_l = 0.f;
        for (int d = tid; d < Dh; d += BWD_THREADS) {
            float a = 0.f, u = 0.f;
#pragma unroll
            for (int w = 0; w < BWD_WARPS; ++w) { a += pp[w][d]; u += pu[w][d]; }
            const float r = dg::to_f(vv[bt_i * Dh + d]) - a;
            rv[d] = r;
            uv[d] = u;
            yv[d] = dg::to_f(grad_out[bt_i * Dh + d]);
            static_cast<T*>(p.grad_v)[bt_i * Dh + d] = dg::from_f<T>(bt * u);
            dbeta_l = fmaf(u, r, dbeta_l);
        }
        const float tbeta = block_sum(dbeta_l, red);      // includes the barrier that publishes rv/uv/yv
        if (tid == 0) static_cast<T*>(p.grad_beta)[bt_i] = dg::from_f<T>(tbeta);
        float dalpha_l = 0.f;
#pragma unroll
        for (int j = 0; j < RPW; ++j) {
            const int m = warp + BWD_WARPS * j;
            float q = 0.f, kq = 0.f;
#pragma unroll
            for (int k = 0; k < KD; ++k) {
                const int d = lane + 32 * k;
                if (d < Dh) {
                    q = fmaf(s[j][k], yv[d], q);
                    kq += g[j][k] * rv[d] - s[j][k] * uv[d];
                    dalpha_l = fmaf(s[j][k], g[j][k], dalpha_l);
                }
            }
            q = warp_sum(q);
            kq = warp_sum(kq);
            if (m < A) {
                if (lane == 0) {
                    static_cast<T*>(p.grad_wq)[bt_i * A + m] = dg::from_f<T>(q);
                    static_cast<T*>(p.grad_wk)[bt_i * A + m] = dg::from_f<T>(bt * kq);
                }
                if (slot[j] >= 0) {
#pragma unroll
                    for (int k = 0; k < KD; ++k) {
                        const int d = lane + 32 * k;
                        if (d < Dh)
                            gstate[slot[j] * Dh + d] =
                                dg::from_f<T>(alpha * g[j][k] - bt * wkm[j] * uv[d] + wqm[j] * yv[d]);
                    }
                }
            }
        }
        const float ta = block_sum(dalpha_l, red);        // also orders this step's writes before the next step's reads
        if (tid == 0 && p.grad_decay) {
            if (p.dynamic_decay) static_cast<T*>(p.grad_decay)[bt_i] = dg::from_f<T>(ta);
            else decay_acc += ta;
        }
        __syncthreads();
    }
    if (!p.dynamic_decay && p.grad_decay && tid == 0) atomic_add_out<T>(static_cast<T*>(p.grad_decay) + h, decay_acc);
}

size_t dense_bwd_vec_floats(int S, int Dh) { return (size_t)3 * Dh + 2 * S + BWD_WARPS * Dh + BWD_WARPS; }
bool dense_bwd_on_chip(int S, int Dh) {
    return ((size_t)2 * S * Dh + dense_bwd_vec_floats(S, Dh)) * 4 <= kDenseSmemMax;
}

template <typename T, int RPW, int KD>
int launch_pkm_bwd(const PkmBwdParams& p, int lanes, cudaStream_t s) {
    pkm_bwd_kernel<T, RPW, KD><<<lanes, BWD_THREADS, 0, s>>>(p);
    return dg_host::check_launch();
}

}  // namespace

extern "C" {

size_t dg_dense_backward_workspace_size(int B, int H, int slots, int dh) {
    if (B <= 0 || H <= 0 || slots <= 0 || dh <= 0 || dense_bwd_on_chip(slots, dh)) return 0;
    return (size_t)B * H * 2 * slots * dh * sizeof(float);
}

int dg_dense_backward(int dtype, int B, int H, int T, int slots, int dh, const void* grad_out,
                      const void* grad_s_final, const void* v, const void* beta, const void* wk, const void* wq,
                      const void* decay, int dynamic_decay, const float* s_final, const float* err_saved,
                      void* grad_v, void* grad_beta, void* grad_wk, void* grad_wq, void* grad_decay,
                      void* grad_s_init, float* workspace, void* stream) {
    (void)v;   // the residuals r_t stand in for v (the reference's kernel does not read it either)
    if (B <= 0 || H <= 0 || T < 0 || slots <= 0 || dh <= 0) return DG_ERR_INVALID_ARGUMENT;
    if (!grad_out || !beta || !wk || !wq || !decay || !s_final || !err_saved || !grad_v || !grad_beta ||
        !grad_wk || !grad_wq || !grad_decay)
        return DG_ERR_INVALID_ARGUMENT;
    const bool on_chip = dense_bwd_on_chip(slots, dh);
    if (!on_chip && !workspace) return DG_ERR_WORKSPACE;
    const size_t smem = (on_chip ? (size_t)2 * slots * dh : 0) * 4 + dense_bwd_vec_floats(slots, dh) * 4;
    if (smem > 232448) return DG_ERR_UNSUPPORTED;
    DenseBwdParams p{grad_out, grad_s_final, beta, wk, wq, decay, s_final, err_saved, grad_v, grad_beta, grad_wk,
                     grad_wq, grad_decay, grad_s_init, on_chip ? nullptr : workspace, H, T, slots, dh, dynamic_decay};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DG_DISPATCH(dtype, TT, {
        auto k = dense_bwd_kernel<TT>;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return dg_host::record_cuda_error(e);
        k<<<B * H, BWD_THREADS, smem, s>>>(p);
        return dg_host::check_launch();
    });
    return DG_ERR_INVALID_ARGUMENT;
}

int dg_pkm_backward(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh, const void* grad_out,
                    const void* v, const void* beta, const void* wk, const void* wq, const int64_t* idx,
                    const void* decay, int dynamic_decay, const void* saved_s_act, void* grad_state, void* grad_v,
                    void* grad_beta, void* grad_wk, void* grad_wq, void* grad_decay, int32_t* dev_status,
                    void* stream) {
    if (B <= 0 || H <= 0 || T < 0 || active <= 0 || total_slots <= 0 || dh <= 0) return DG_ERR_INVALID_ARGUMENT;
    if (!grad_out || !v || !beta || !wk || !wq || !idx || !decay || !saved_s_act || !grad_state || !grad_v ||
        !grad_beta || !grad_wk || !grad_wq)
        return DG_ERR_INVALID_ARGUMENT;
    if (active > 64 || dh > 128) return DG_ERR_UNSUPPORTED;    // the forward kernels' shapes
    PkmBwdParams p{grad_out, v, beta, wk, wq, decay, saved_s_act, idx, grad_state, grad_v, grad_beta, grad_wk,
                   grad_wq, grad_decay, dev_status, total_slots, H, T, active, dh, dynamic_decay};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int lanes = B * H;
    DG_DISPATCH(dtype, TT, {
        if (dh <= 64) return launch_pkm_bwd<TT, 8, 2>(p, lanes, s);
        return launch_pkm_bwd<TT, 8, 4>(p, lanes, s);
    });
    return DG_ERR_INVALID_ARGUMENT;
}

}  // extern "C"
