// dense_seq.cu -- dense delta-rule recurrence on CUDA cores (any dtype, slots <= 1024).
//
// Math (src/cpp/delta_kernel.cu:78-112, src/modules/memory.py:524-539), per
// lane (b,h) and step t:
//     y_t = wq_t^T S,   r_t = v_t - wk_t^T S,   S = alpha_t S + (beta_t wk_t) r_t^T
//
// Layout: one CTA per (lane, tile of CW columns).  Columns of S are independent
// (column d only needs v_t[d] and the per-step scalars), so the reference puts
// one thread on a column and loops over all slots (delta_kernel.cu:49).  Here
// SG threads share a column, each holding SPT slots of it in registers, and
// the two dot products are finished with an xor-butterfly over those SG lanes.
// That shortens the dependent FMA chain per step by SG and spreads a lane over
// ceil(Dh/CW) CTAs.  The prediction wk_t^T S is carried one step ahead
// (wk_{t+1}^T S_t = alpha_t wk_{t+1}^T S_{t-1} + beta_t (wk_{t+1}.wk_t) r_t), so no
// reduction sits between one step's state update and the next step's residual.
// The per-step inputs (wk, wq, v, beta, alpha) for TT steps are staged in shared
// memory as fp32 and y/r are staged for coalesced stores.
// The state stays fp32 for all T and is cast once at the end (delta_kernel.cu:116-121).
#include "dg_common.cuh"

#include <algorithm>

namespace {

struct DenseSeqParams {
    const void* v;
    const void* beta;
    const void* wk;
    const void* wq;
    const void* decay;
    const void* s_init;
    void* out;
    void* s_final;
    float* err_out;
    float* s_final_f;
    int B, H, T, S, Dh;
    int dynamic_decay;
    int TT;  // steps staged per shared-memory chunk
};

// slot m of thread group g, register j: m = 4 * (g + SG * (j / 4)) + (j % 4)
template <int SG>
__device__ __forceinline__ int slot_of(int g, int j) {
    return 4 * (g + SG * (j >> 2)) + (j & 3);
}

template <typename T, int SG, int SPT, int CW>
__global__ void __launch_bounds__(CW * SG) dense_seq_kernel(DenseSeqParams p) {
    constexpr int NT = CW * SG;
    constexpr int SP = SG * SPT;  // padded slot count
    extern __shared__ __align__(16) float sm[];
    const int TT = p.TT;
    float* wk_s = sm;                  // [TT][SP]
    float* wq_s = wk_s + TT * SP;      // [TT][SP]
    float* v_s = wq_s + TT * SP;       // [TT][CW]
    float* y_s = v_s + TT * CW;        // [TT][CW]
    float* r_s = y_s + TT * CW;        // [TT][CW]
    float* ab_s = r_s + TT * CW;       // [TT][3]  (alpha, beta, beta * wk_{t+1}.wk_t)

    const T* __restrict__ v = static_cast<const T*>(p.v);
    const T* __restrict__ beta = static_cast<const T*>(p.beta);
    const T* __restrict__ wk = static_cast<const T*>(p.wk);
    const T* __restrict__ wq = static_cast<const T*>(p.wq);
    const T* __restrict__ decay = static_cast<const T*>(p.decay);

    const int tid = threadIdx.x;
    const int g = tid % SG;
    const int cl = tid / SG;
    const int lane = blockIdx.y;             // b * H + h
    const int h = lane % p.H;
    const int c0 = blockIdx.x * CW;
    const int c = c0 + cl;
    const bool cvalid = c < p.Dh;
    const int S = p.S, Dh = p.Dh, T_ = p.T;

    float st[SPT];
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
        const int m = slot_of<SG>(g, j);
        float x = 0.f;
        if (p.s_init && cvalid && m < S)
            x = dg::to_f(static_cast<const T*>(p.s_init)[((int64_t)lane * S + m) * Dh + c]);
        st[j] = x;
    }
    const float alpha_static = p.dynamic_decay ? 1.f : dg::to_f(decay[h]);

    for (int t0 = 0; t0 < T_; t0 += TT) {
        const int nT = min(TT, T_ - t0);
        __syncthreads();
        const int64_t wbase = ((int64_t)lane * T_ + t0) * S;
        // rows of wk / wq for nT steps are one contiguous run of nT * S elements; when
        // it needs no padding (S == SP) and is 16-byte aligned, 16-byte loads put every
        // load of a thread in flight at once instead of one element per iteration
        constexpr int EV = 16 / (int)sizeof(T);            // elements per 16-byte vector
        const int64_t run = (int64_t)nT * S;
        const bool vec = S == SP && run % EV == 0 && ((uintptr_t)(wk + wbase) & 15) == 0 &&
                         ((uintptr_t)(wq + wbase) & 15) == 0;
        if (vec) {
            const uint4* wk16 = reinterpret_cast<const uint4*>(wk + wbase);
            const uint4* wq16 = reinterpret_cast<const uint4*>(wq + wbase);
            for (int i = tid; i < (int)(run / EV); i += NT) {
                const uint4 a = wk16[i], b = wq16[i];
                const T* ea = reinterpret_cast<const T*>(&a);
                const T* eb = reinterpret_cast<const T*>(&b);
#pragma unroll
                for (int e = 0; e < EV; ++e) {
                    wk_s[i * EV + e] = dg::to_f(ea[e]);
                    wq_s[i * EV + e] = dg::to_f(eb[e]);
                }
            }
            for (int i = (int)run + tid; i < TT * SP; i += NT) {      // steps past the end of T
                wk_s[i] = 0.f;
                wq_s[i] = 0.f;
            }
        } else {
            for (int i = tid; i < TT * SP; i += NT) {
                const int tt = i / SP, m = i - tt * SP;
                const bool ok = tt < nT && m < S;
                wk_s[i] = ok ? dg::to_f(wk[wbase + (int64_t)tt * S + m]) : 0.f;
                wq_s[i] = ok ? dg::to_f(wq[wbase + (int64_t)tt * S + m]) : 0.f;
            }
        }
        const int64_t vbase = ((int64_t)lane * T_ + t0) * Dh + c0;
        for (int i = tid; i < TT * CW; i += NT) {
            const int tt = i / CW, cc = i - tt * CW;
            v_s[i] = (tt < nT && c0 + cc < Dh) ? dg::to_f(v[vbase + (int64_t)tt * Dh + cc]) : 0.f;
        }
        for (int i = tid; i < nT; i += NT) {
            const int64_t bt = (int64_t)lane * T_ + t0 + i;
            ab_s[3 * i] = p.dynamic_decay ? dg::to_f(decay[bt]) : alpha_static;
            ab_s[3 * i + 1] = dg::to_f(beta[bt]);
            ab_s[3 * i + 2] = 0.f;
        }
        __syncthreads();
        // beta_t (wk_{t+1} . wk_t) for t < nT - 1: with it each step's prediction follows
        // from the one before (below).  Row i starts at slot i mod SP, so the threads of a
        // warp read distinct banks.
        for (int i = tid; i < nT - 1; i += NT) {
            const float* a = wk_s + i * SP;
            const float* b = a + SP;
            float g0 = 0.f, g1 = 0.f;
#pragma unroll 4
            for (int n = 0; n < SP; n += 2) {
                const int m0 = (i + n) & (SP - 1), m1 = (i + n + 1) & (SP - 1);
                g0 = fmaf(a[m0], b[m0], g0);
                g1 = fmaf(a[m1], b[m1], g1);
            }
            ab_s[3 * i + 2] = ab_s[3 * i + 1] * (g0 + g1);
        }
        __syncthreads();

        // pr = wk_t . S_{t-1} for the chunk's first step, reduced directly
        float pr;
        {
            const float4* wk4 = reinterpret_cast<const float4*>(wk_s);
            float p0 = 0.f, p1 = 0.f;
#pragma unroll
            for (int j4 = 0; j4 < SPT / 4; ++j4) {
                const float4 b = wk4[g + SG * j4];
                p0 = fmaf(b.x, st[4 * j4 + 0], p0);
                p1 = fmaf(b.y, st[4 * j4 + 1], p1);
                p0 = fmaf(b.z, st[4 * j4 + 2], p0);
                p1 = fmaf(b.w, st[4 * j4 + 3], p1);
            }
            pr = p0 + p1;
#pragma unroll
            for (int o = 1; o < SG; o <<= 1) pr += __shfl_xor_sync(DG_FULL_MASK, pr, o);
        }

        // Step t reduces y_t = wq_t . S_{t-1} and x = wk_{t+1} . S_{t-1} together; then
        //     wk_{t+1} . S_t = alpha_t x + beta_t (wk_{t+1} . wk_t) r_t,
        // so the next step's residual needs no reduction of S_t, and the state update can
        // issue before this step's butterflies finish.  Consecutive steps' reductions
        // overlap (two steps per unrolled body).
#pragma unroll 2
        for (int tt = 0; tt < nT; ++tt) {
            const float4* wk4 = reinterpret_cast<const float4*>(wk_s + tt * SP);
            const float4* wq4 = reinterpret_cast<const float4*>(wq_s + tt * SP);
            const float4* wn4 = reinterpret_cast<const float4*>(wk_s + min(tt + 1, nT - 1) * SP);
            float y0 = 0.f, y1 = 0.f, x0 = 0.f, x1 = 0.f;
#pragma unroll
            for (int j4 = 0; j4 < SPT / 4; ++j4) {
                const float4 a = wq4[g + SG * j4];
                const float4 b = wn4[g + SG * j4];
                y0 = fmaf(a.x, st[4 * j4 + 0], y0);
                x0 = fmaf(b.x, st[4 * j4 + 0], x0);
                y1 = fmaf(a.y, st[4 * j4 + 1], y1);
                x1 = fmaf(b.y, st[4 * j4 + 1], x1);
                y0 = fmaf(a.z, st[4 * j4 + 2], y0);
                x0 = fmaf(b.z, st[4 * j4 + 2], x0);
                y1 = fmaf(a.w, st[4 * j4 + 3], y1);
                x1 = fmaf(b.w, st[4 * j4 + 3], x1);
            }
            const float al = ab_s[3 * tt], bt = ab_s[3 * tt + 1], bg = ab_s[3 * tt + 2];
            const float r = v_s[tt * CW + cl] - pr;
#pragma unroll
            for (int j4 = 0; j4 < SPT / 4; ++j4) {
                const float4 b = wk4[g + SG * j4];
                st[4 * j4 + 0] = fmaf(al, st[4 * j4 + 0], (bt * b.x) * r);
                st[4 * j4 + 1] = fmaf(al, st[4 * j4 + 1], (bt * b.y) * r);
                st[4 * j4 + 2] = fmaf(al, st[4 * j4 + 2], (bt * b.z) * r);
                st[4 * j4 + 3] = fmaf(al, st[4 * j4 + 3], (bt * b.w) * r);
            }
            float y = y0 + y1, x = x0 + x1;
#pragma unroll
            for (int o = 1; o < SG; o <<= 1) {
                y += __shfl_xor_sync(DG_FULL_MASK, y, o);
                x += __shfl_xor_sync(DG_FULL_MASK, x, o);
            }
            if (g == 0) {
                y_s[tt * CW + cl] = y;
                r_s[tt * CW + cl] = r;
            }
            pr = fmaf(al, x, bg * r);
        }
        __syncthreads();
        T* __restrict__ out = static_cast<T*>(p.out);
        for (int i = tid; i < nT * CW; i += NT) {
            const int tt = i / CW, cc = i - tt * CW;
            if (c0 + cc < Dh) {
                const int64_t o = vbase + (int64_t)tt * Dh + cc;
                out[o] = dg::from_f<T>(y_s[i]);
                if (p.err_out) p.err_out[o] = r_s[i];
            }
        }
    }

    T* __restrict__ s_final = static_cast<T*>(p.s_final);
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
        const int m = slot_of<SG>(g, j);
        if (cvalid && m < S) {
            const int64_t o = ((int64_t)lane * S + m) * Dh + c;
            s_final[o] = dg::from_f<T>(st[j]);
            if (p.s_final_f) p.s_final_f[o] = st[j];
        }
    }
}

template <typename T, int SG, int SPT, int CW>
int launch_seq(DenseSeqParams p, cudaStream_t stream) {
    constexpr int SP = SG * SPT;
    // Each chunk costs a round trip to stage its inputs.  When the grid fits in one wave
    // (a CTA per SM at most), shared memory is not shared between CTAs, so chunks grow
    // to 200 KB and up to 256 steps; otherwise 96 KB keeps two CTAs per SM.
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    int nsm = 0;
    const int rc = dg_host::sm_count(dev, &nsm);
    if (rc != DG_OK) return rc;
    const int64_t ctas = (int64_t)((p.Dh + CW - 1) / CW) * p.B * p.H;
    const bool one_wave = ctas <= nsm;
    const size_t kSmemBudget = (one_wave ? 200 : 96) * 1024;
    const size_t per_step = (2 * SP + 3 * CW + 3) * sizeof(float);
    int TT = (int)std::min<size_t>(one_wave ? 256 : 64, kSmemBudget / per_step);
    TT = std::max(1, std::min(TT, p.T));
    p.TT = TT;
    const size_t smem = per_step * TT;
    auto kern = dense_seq_kernel<T, SG, SPT, CW>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    }
    dim3 grid((p.Dh + CW - 1) / CW, p.B * p.H);
    kern<<<grid, CW * SG, smem, stream>>>(p);
    return dg_host::check_launch();
}

template <typename T>
int dispatch_seq(const DenseSeqParams& p, cudaStream_t s) {
    if (p.S <= 8) return launch_seq<T, 2, 4, 64>(p, s);
    if (p.S <= 16) return launch_seq<T, 4, 4, 32>(p, s);
    if (p.S <= 32) return launch_seq<T, 4, 8, 32>(p, s);
    if (p.S <= 64) return launch_seq<T, 8, 8, 16>(p, s);
    if (p.S <= 128) return launch_seq<T, 8, 16, 16>(p, s);
    if (p.S <= 256) return launch_seq<T, 16, 16, 16>(p, s);
    if (p.S <= 512) return launch_seq<T, 16, 32, 16>(p, s);
    if (p.S <= 1024) return launch_seq<T, 32, 32, 8>(p, s);
    return DG_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------------------
// single decode step (delta_kernel.cu:223-351): reads S once, writes S_next.
// Thread (c, g): column c = tid % CW (coalesced rows), slot group g = tid / CW
// holding slots m = g + NG*i.  Partial dot products are reduced across slot
// groups through shared memory; s_next may alias s_prev (each element is read
// and then written by the same thread only).
// ---------------------------------------------------------------------------
struct DenseStepParams {
    const void* v; int64_t v_sb, v_sh;
    const void* beta; int64_t beta_sb, beta_sh;
    const void* wk; int64_t wk_sb, wk_sh;
    const void* wq; int64_t wq_sb, wq_sh;
    const void* decay; int dynamic_decay; int64_t decay_sb, decay_sh;
    const void* s_prev; void* out; void* s_next;
    int B, H, S, Dh;
};

template <typename T, int CW, int NG, int MAXPER>
__global__ void __launch_bounds__(CW * NG) dense_step_kernel(DenseStepParams p) {
    __shared__ float red[2][NG][CW];
    __shared__ float rr[CW];
    const int tid = threadIdx.x;
    const int cl = tid % CW, g = tid / CW;
    const int lane = blockIdx.y;
    const int b = lane / p.H, h = lane % p.H;
    const int c = blockIdx.x * CW + cl;
    const bool cvalid = c < p.Dh;
    const int S = p.S, Dh = p.Dh;
    const T* wk = static_cast<const T*>(p.wk) + b * p.wk_sb + h * p.wk_sh;
    const T* wq = static_cast<const T*>(p.wq) + b * p.wq_sb + h * p.wq_sh;
    const T* sp = static_cast<const T*>(p.s_prev) + (int64_t)lane * S * Dh;
    T* sn = static_cast<T*>(p.s_next) + (int64_t)lane * S * Dh;

    float sv[MAXPER];
    float y = 0.f, pr = 0.f;
#pragma unroll
    for (int i = 0; i < MAXPER; ++i) {
        const int m = g + NG * i;
        float x = 0.f;
        if (m < S && cvalid) x = dg::to_f(sp[(int64_t)m * Dh + c]);
        sv[i] = x;
        if (m < S) {
            y = fmaf(dg::to_f(wq[m]), x, y);
            pr = fmaf(dg::to_f(wk[m]), x, pr);
        }
    }
    red[0][g][cl] = y;
    red[1][g][cl] = pr;
    __syncthreads();
    if (g == 0) {
        float ys = 0.f, ps = 0.f;
#pragma unroll
        for (int k = 0; k < NG; ++k) { ys += red[0][k][cl]; ps += red[1][k][cl]; }
        if (cvalid) {
            const T* v = static_cast<const T*>(p.v) + b * p.v_sb + h * p.v_sh;
            static_cast<T*>(p.out)[(int64_t)lane * Dh + c] = dg::from_f<T>(ys);
            rr[cl] = dg::to_f(v[c]) - ps;
        } else {
            rr[cl] = 0.f;
        }
    }
    __syncthreads();
    const T* decay = static_cast<const T*>(p.decay);
    const float al = p.dynamic_decay ? dg::to_f(decay[b * p.decay_sb + h * p.decay_sh]) : dg::to_f(decay[h]);
    const float bt = dg::to_f(static_cast<const T*>(p.beta)[b * p.beta_sb + h * p.beta_sh]);
    const float r = rr[cl];
#pragma unroll
    for (int i = 0; i < MAXPER; ++i) {
        const int m = g + NG * i;
        if (m < S && cvalid) sn[(int64_t)m * Dh + c] = dg::from_f<T>(fmaf(al, sv[i], (bt * dg::to_f(wk[m])) * r));
    }
}

// Decode step, vectorised: one CTA of 256 threads per lane, the lane's S x 64 state
// held in registers as 16-byte vectors (NV per thread, read once with coalesced
// 16-byte loads: 4 KB per pass of the CTA).  Thread t owns, in pass w, row
// w * RPW + t / NG and the CPV columns (t % NG) * CPV ..; y and pred are summed over
// its rows, then over the threads of its column group (shuffles, then across warps in
// shared memory); the new rows go back as 16-byte stores.  The whole lane is read
// before any of it is written, so s_next may alias s_prev.
constexpr int STEPV_THREADS = 256;
template <typename T, int NV>
__global__ void __launch_bounds__(STEPV_THREADS) dense_step_vec_kernel(DenseStepParams p) {
    constexpr int CPV = 16 / (int)sizeof(T);            // columns per 16-byte vector
    constexpr int NG = 64 / CPV;                         // column groups (Dh = 64)
    constexpr int RPW = STEPV_THREADS / NG;              // rows per pass
    __shared__ float red[2][STEPV_THREADS / 32][64];
    __shared__ float rr[64];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cg = tid % NG, rsub = tid / NG;
    const int ln = blockIdx.x, b = ln / p.H, h = ln % p.H;
    const int S = p.S;
    const T* wk = static_cast<const T*>(p.wk) + b * p.wk_sb + h * p.wk_sh;
    const T* wq = static_cast<const T*>(p.wq) + b * p.wq_sb + h * p.wq_sh;
    const uint8_t* sp = static_cast<const uint8_t*>(p.s_prev) + (int64_t)ln * S * 64 * sizeof(T);
    uint8_t* sn = static_cast<uint8_t*>(p.s_next) + (int64_t)ln * S * 64 * sizeof(T);

    uint4 sv[NV];
    float wkv[NV];
#pragma unroll
    for (int w = 0; w < NV; ++w) {
        const int m = w * RPW + rsub;
        sv[w] = dg::ld16(sp + ((int64_t)m * 64 + cg * CPV) * sizeof(T));
        wkv[w] = dg::to_f(wk[m]);
    }
    float ya[CPV], pa[CPV];
#pragma unroll
    for (int i = 0; i < CPV; ++i) { ya[i] = 0.f; pa[i] = 0.f; }
#pragma unroll
    for (int w = 0; w < NV; ++w) {
        const float wqm = dg::to_f(wq[w * RPW + rsub]);
        const T* e = reinterpret_cast<const T*>(&sv[w]);
#pragma unroll
        for (int i = 0; i < CPV; ++i) {
            const float x = dg::to_f(e[i]);
            ya[i] = fmaf(wqm, x, ya[i]);
            pa[i] = fmaf(wkv[w], x, pa[i]);
        }
    }
    // threads of a column group: lanes l with l % NG equal, then the warps
#pragma unroll
    for (int o = NG; o < 32; o <<= 1) {
#pragma unroll
        for (int i = 0; i < CPV; ++i) {
            ya[i] += __shfl_xor_sync(DG_FULL_MASK, ya[i], o);
            pa[i] += __shfl_xor_sync(DG_FULL_MASK, pa[i], o);
        }
    }
    if (lane < NG) {
#pragma unroll
        for (int i = 0; i < CPV; ++i) {
            red[0][warp][cg * CPV + i] = ya[i];
            red[1][warp][cg * CPV + i] = pa[i];
        }
    }
    __syncthreads();
    if (tid < 64) {
        float y = 0.f, pr = 0.f;
#pragma unroll
        for (int k = 0; k < STEPV_THREADS / 32; ++k) { y += red[0][k][tid]; pr += red[1][k][tid]; }
        const T* v = static_cast<const T*>(p.v) + b * p.v_sb + h * p.v_sh;
        static_cast<T*>(p.out)[(int64_t)ln * 64 + tid] = dg::from_f<T>(y);
        rr[tid] = dg::to_f(v[tid]) - pr;
    }
    __syncthreads();
    const T* decay = static_cast<const T*>(p.decay);
    const float al = p.dynamic_decay ? dg::to_f(decay[b * p.decay_sb + h * p.decay_sh]) : dg::to_f(decay[h]);
    const float bt = dg::to_f(static_cast<const T*>(p.beta)[b * p.beta_sb + h * p.beta_sh]);
    float r[CPV];
#pragma unroll
    for (int i = 0; i < CPV; ++i) r[i] = rr[cg * CPV + i];
#pragma unroll
    for (int w = 0; w < NV; ++w) {
        const int m = w * RPW + rsub;
        const float c = bt * wkv[w];
        const T* e = reinterpret_cast<const T*>(&sv[w]);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int i = 0; i < CPV; ++i) oe[i] = dg::from_f<T>(fmaf(al, dg::to_f(e[i]), c * r[i]));
        dg::st16(sn + ((int64_t)m * 64 + cg * CPV) * sizeof(T), o);
    }
}

// Decode step, staged: the same thread mapping and arithmetic as dense_step_vec_kernel,
// but the lane's state goes to shared memory through cp.async (16 bytes a copy) instead
// of registers, so a thread keeps only its accumulators (wk and wq are re-read, from
// L1).  NT threads per lane (256 here): 5 lanes per SM for bf16 at 256 slots (160 KB
// of state in flight instead of 2 lanes' 64 KB), 3 for fp32 (64 KB each).  Each thread
// reads back only the vectors it copied (cp.async.wait_all orders them for that thread).
template <typename T, int NV, int NT>
__global__ void __launch_bounds__(NT, NT == 256 ? 5 : 6) dense_step_staged_kernel(DenseStepParams p) {
    constexpr int CPV = 16 / (int)sizeof(T);
    constexpr int NG = 64 / CPV;
    constexpr int RPW = NT / NG;
    extern __shared__ __align__(16) uint8_t st_smem[];               // [S][64] state of the lane
    __shared__ float red[2][NT / 32][64];
    __shared__ float rr[64];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cg = tid % NG, rsub = tid / NG;
    const int ln = blockIdx.x, b = ln / p.H, h = ln % p.H;
    const int S = p.S;
    const T* wk = static_cast<const T*>(p.wk) + b * p.wk_sb + h * p.wk_sh;
    const T* wq = static_cast<const T*>(p.wq) + b * p.wq_sb + h * p.wq_sh;
    const uint8_t* sp = static_cast<const uint8_t*>(p.s_prev) + (int64_t)ln * S * 64 * sizeof(T);
    uint8_t* sn = static_cast<uint8_t*>(p.s_next) + (int64_t)ln * S * 64 * sizeof(T);
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(st_smem));
#pragma unroll
    for (int w = 0; w < NV; ++w) {
        const int64_t off = ((int64_t)(w * RPW + rsub) * 64 + cg * CPV) * sizeof(T);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sbase + (uint32_t)off), "l"(sp + off)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_all;" ::: "memory");
    float ya[CPV], pa[CPV];
#pragma unroll
    for (int i = 0; i < CPV; ++i) { ya[i] = 0.f; pa[i] = 0.f; }
#pragma unroll
    for (int w = 0; w < NV; ++w) {
        const uint4 sv = *reinterpret_cast<const uint4*>(st_smem + ((w * RPW + rsub) * 64 + cg * CPV) * sizeof(T));
        const float wqm = dg::to_f(wq[w * RPW + rsub]), wkm = dg::to_f(wk[w * RPW + rsub]);
        const T* e = reinterpret_cast<const T*>(&sv);
#pragma unroll
        for (int i = 0; i < CPV; ++i) {
            const float x = dg::to_f(e[i]);
            ya[i] = fmaf(wqm, x, ya[i]);
            pa[i] = fmaf(wkm, x, pa[i]);
        }
    }
#pragma unroll
    for (int o = NG; o < 32; o <<= 1) {
#pragma unroll
        for (int i = 0; i < CPV; ++i) {
            ya[i] += __shfl_xor_sync(DG_FULL_MASK, ya[i], o);
            pa[i] += __shfl_xor_sync(DG_FULL_MASK, pa[i], o);
        }
    }
    if (lane < NG) {
#pragma unroll
        for (int i = 0; i < CPV; ++i) {
            red[0][warp][cg * CPV + i] = ya[i];
            red[1][warp][cg * CPV + i] = pa[i];
        }
    }
    __syncthreads();
    if (tid < 64) {
        float y = 0.f, pr = 0.f;
#pragma unroll
        for (int k = 0; k < NT / 32; ++k) { y += red[0][k][tid]; pr += red[1][k][tid]; }
        const T* v = static_cast<const T*>(p.v) + b * p.v_sb + h * p.v_sh;
        static_cast<T*>(p.out)[(int64_t)ln * 64 + tid] = dg::from_f<T>(y);
        rr[tid] = dg::to_f(v[tid]) - pr;
    }
    __syncthreads();
    const T* decay = static_cast<const T*>(p.decay);
    const float al = p.dynamic_decay ? dg::to_f(decay[b * p.decay_sb + h * p.decay_sh]) : dg::to_f(decay[h]);
    const float bt = dg::to_f(static_cast<const T*>(p.beta)[b * p.beta_sb + h * p.beta_sh]);
    float r[CPV];
#pragma unroll
    for (int i = 0; i < CPV; ++i) r[i] = rr[cg * CPV + i];
#pragma unroll
    for (int w = 0; w < NV; ++w) {
        const int64_t off = ((int64_t)(w * RPW + rsub) * 64 + cg * CPV) * sizeof(T);
        const uint4 sv = *reinterpret_cast<const uint4*>(st_smem + off);
        const float c = bt * dg::to_f(wk[w * RPW + rsub]);
        const T* e = reinterpret_cast<const T*>(&sv);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int i = 0; i < CPV; ++i) oe[i] = dg::from_f<T>(fmaf(al, dg::to_f(e[i]), c * r[i]));
        dg::st16(sn + off, o);
    }
}

template <typename T, int NV, int NT>
int launch_step_staged(const DenseStepParams& p, cudaStream_t s) {
    const int smem = p.S * 64 * (int)sizeof(T);
    auto kern = dense_step_staged_kernel<T, NV, NT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    }
    kern<<<p.B * p.H, NT, smem, s>>>(p);
    return dg_host::check_launch();
}

template <typename T, int NV>
int launch_step_vec(const DenseStepParams& p, cudaStream_t s) {
    dense_step_vec_kernel<T, NV><<<p.B * p.H, STEPV_THREADS, 0, s>>>(p);
    return dg_host::check_launch();
}

template <typename T>
int dispatch_step(const DenseStepParams& p, cudaStream_t s) {
    // the vectorised kernel: Dh = 64, 16-byte aligned state, and a lane state of 1, 2,
    // 4, 8 or 16 passes of 4 KB (e.g. 256 slots in bf16 = 8 passes)
    if (p.Dh == 64 && sizeof(T) <= 4) {
        const int64_t lane_bytes = (int64_t)p.S * 64 * sizeof(T);
        const bool al = ((uintptr_t)p.s_prev & 15) == 0 && ((uintptr_t)p.s_next & 15) == 0;
        if (al && lane_bytes % (STEPV_THREADS * 16) == 0) {
            // 16-bit state up to 32 KB a lane: staged through shared memory, 5 lanes per SM
            // (128 threads a lane, 6 lanes per SM, measured slower: each thread's loop doubles)
            if constexpr (sizeof(T) == 2) {
                switch (lane_bytes / (STEPV_THREADS * 16)) {
                case 1: return launch_step_staged<T, 1, 256>(p, s);
                case 2: return launch_step_staged<T, 2, 256>(p, s);
                case 4: return launch_step_staged<T, 4, 256>(p, s);
                case 8: return launch_step_staged<T, 8, 256>(p, s);
                default: break;
                }
            }
            // fp32 state up to 64 KB a lane (256 slots): staged as well, 3 lanes per SM
            if constexpr (sizeof(T) == 4) {
                switch (lane_bytes / (STEPV_THREADS * 16)) {
                case 1: return launch_step_staged<T, 1, 256>(p, s);
                case 2: return launch_step_staged<T, 2, 256>(p, s);
                case 4: return launch_step_staged<T, 4, 256>(p, s);
                case 8: return launch_step_staged<T, 8, 256>(p, s);
                case 16: return launch_step_staged<T, 16, 256>(p, s);
                default: break;
                }
            }
            switch (lane_bytes / (STEPV_THREADS * 16)) {
            case 1: return launch_step_vec<T, 1>(p, s);
            case 2: return launch_step_vec<T, 2>(p, s);
            case 4: return launch_step_vec<T, 4>(p, s);
            case 8: return launch_step_vec<T, 8>(p, s);
            case 16: return launch_step_vec<T, 16>(p, s);
            default: break;
            }
        }
    }
    constexpr int CW = 32, NG = 8;
    dim3 grid((p.Dh + CW - 1) / CW, p.B * p.H);
    if (p.S <= NG * 4) dense_step_kernel<T, CW, NG, 4><<<grid, CW * NG, 0, s>>>(p);
    else if (p.S <= NG * 16) dense_step_kernel<T, CW, NG, 16><<<grid, CW * NG, 0, s>>>(p);
    else if (p.S <= NG * 64) dense_step_kernel<T, CW, NG, 64><<<grid, CW * NG, 0, s>>>(p);
    else if (p.S <= NG * 128) dense_step_kernel<T, CW, NG, 128><<<grid, CW * NG, 0, s>>>(p);
    else return DG_ERR_UNSUPPORTED;
    return dg_host::check_launch();
}

}  // namespace

namespace dg_host {

int dense_forward_sequential(int dtype, int B, int H, int T, int S, int Dh, const void* v,
                             const void* beta, const void* wk, const void* wq, const void* decay,
                             int dynamic_decay, const void* s_init, void* out, void* s_final,
                             float* err_out, float* s_final_f, cudaStream_t stream) {
    DenseSeqParams p{v, beta, wk, wq, decay, s_init, out, s_final, err_out, s_final_f,
                     B, H, T, S, Dh, dynamic_decay, 1};
    DG_DISPATCH(dtype, Ty, return dispatch_seq<Ty>(p, stream));
    return DG_ERR_INVALID_ARGUMENT;
}

int dense_step(int dtype, int B, int H, int S, int Dh, const void* v, int64_t v_sb, int64_t v_sh,
               const void* beta, int64_t beta_sb, int64_t beta_sh, const void* wk, int64_t wk_sb,
               int64_t wk_sh, const void* wq, int64_t wq_sb, int64_t wq_sh, const void* decay,
               int dynamic_decay, int64_t decay_sb, int64_t decay_sh, const void* s_prev,
               void* out, void* s_next, cudaStream_t stream) {
    DenseStepParams p{v, v_sb, v_sh, beta, beta_sb, beta_sh, wk, wk_sb, wk_sh, wq, wq_sb, wq_sh,
                      decay, dynamic_decay, decay_sb, decay_sh, s_prev, out, s_next, B, H, S, Dh};
    DG_DISPATCH(dtype, Ty, return dispatch_step<Ty>(p, stream));
    return DG_ERR_INVALID_ARGUMENT;
}

}  // namespace dg_host
