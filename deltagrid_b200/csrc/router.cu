// router.cu -- two-axis product-key router for Sparse Delta-PKM (fused).
//
// For every token n and axis a (src/modules/memory.py:258-279):
//     s_a = W_k,a k_n            (G_a scores, fp32)
//     (val, i_a) = top-K(s_a)    (descending; equal scores keep the lower index
//                                 first, the order of src/cpp/engine/src/deltagrid_math.cpp:155-167)
//     u_k,a = val / max(|val|, 1e-12)
//     u_q,a = normalize(W_q,a[i_a] q_n)       (queries read at the key's indices)
// then the Kronecker product over the two axes:
//     wk = u_k,0 (x) u_k,1,   wq = (u_q,0 (x) u_q,1) * q_scale[h],   idx = i_0 * G_1 + i_1
//
// Layout: a CTA routes 32 tokens with 256 threads, 8 threads per token.  The
// router weights stream through shared memory 128 rows at a time; thread
// (token, sub) scores rows sub, sub+8, ... of each chunk and keeps a running
// top-K in registers; the 8 partial lists of a token are merged by a K-round
// tournament over shuffles inside the token's 8-lane group.  Scores are fp32
// dot products over Dh in increasing index order, each product and sum rounded
// separately (no FMA contraction), so they equal a sequential scalar loop bit
// for bit and the selected indices are deterministic.
#include "dg_common.cuh"

namespace {

constexpr int TN = 32;          // tokens per CTA
constexpr int SUB = 8;          // threads per token
constexpr int GC = 128;         // router rows per shared-memory chunk
constexpr int MAXK = 8;
constexpr int MAXDH = 128;

struct RouterParams {
    const void* k;
    const void* q;
    const float* wk[2];
    const float* wq[2];
    const float* q_scale;       // [H] or null
    void* out_wk;
    void* out_wq;
    int64_t* out_idx;
    int64_t N;
    int H, T, Dh, G[2], K;
};

// (value desc, index asc) ordering: true when (a, ia) ranks before (b, ib)
__device__ __forceinline__ bool ranks_before(float a, int ia, float b, int ib) {
    return a > b || (a == b && ia < ib);
}

template <typename T>
__global__ void __launch_bounds__(256) router_kernel(RouterParams p) {
    extern __shared__ __align__(16) float sm[];
    const int Dh = p.Dh;
    const int LDW = Dh + 1;
    float* ks = sm;                               // [TN][Dh]
    float* qs = ks + TN * Dh;                     // [TN][Dh]
    float* wsh = qs + TN * Dh;                    // [GC][Dh+1]
    float* res = wsh + GC * LDW;                  // [TN][2 axes][2][MAXK] u_k, u_q
    int* resi = reinterpret_cast<int*>(res + TN * 2 * 2 * MAXK);   // [TN][2][MAXK]

    const int tid = threadIdx.x, tl = tid / SUB, sub = tid % SUB, lane = tid & 31;
    const int64_t n0 = (int64_t)blockIdx.x * TN;
    const int K = p.K;
    const T* gk = static_cast<const T*>(p.k);
    const T* gq = static_cast<const T*>(p.q);

    for (int i = tid; i < TN * Dh; i += blockDim.x) {
        const int64_t n = n0 + i / Dh;
        const int d = i % Dh;
        ks[i] = n < p.N ? dg::to_f(gk[n * Dh + d]) : 0.f;
        qs[i] = n < p.N ? dg::to_f(gq[n * Dh + d]) : 0.f;
    }

    for (int ax = 0; ax < 2; ++ax) {
        const int G = ax ? p.G[1] : p.G[0];
        const float* W = ax ? p.wk[1] : p.wk[0];
        const float* WQ = ax ? p.wq[1] : p.wq[0];
        float bv[MAXK];
        int bi[MAXK];
#pragma unroll
        for (int j = 0; j < MAXK; ++j) { bv[j] = -INFINITY; bi[j] = 0x7fffffff; }
        for (int g0 = 0; g0 < G; g0 += GC) {
            const int gn = min(GC, G - g0);
            __syncthreads();
            for (int i = tid; i < gn * Dh; i += blockDim.x) {
                const int r = i / Dh, d = i % Dh;
                wsh[r * LDW + d] = W[(int64_t)(g0 + r) * Dh + d];
            }
            __syncthreads();
            constexpr int PER = GC / SUB;
            float acc[PER];
#pragma unroll
            for (int j = 0; j < PER; ++j) acc[j] = 0.f;
            const float* kr = ks + tl * Dh;
            for (int d = 0; d < Dh; ++d) {
                const float kd = kr[d];
#pragma unroll
                for (int j = 0; j < PER; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(wsh[(sub + SUB * j) * LDW + d], kd));
            }
#pragma unroll
            for (int j = 0; j < PER; ++j) {
                const int g = g0 + sub + SUB * j;
                if (sub + SUB * j < gn && ranks_before(acc[j], g, bv[MAXK - 1], bi[MAXK - 1])) {
                    // insert into the sorted list (positions >= K are never used)
                    float v = acc[j];
                    int vi = g;
#pragma unroll
                    for (int q = 0; q < MAXK; ++q) {
                        if (ranks_before(v, vi, bv[q], bi[q])) {
                            const float tv = bv[q];
                            const int ti = bi[q];
                            bv[q] = v; bi[q] = vi;
                            v = tv; vi = ti;
                        }
                    }
                }
            }
        }
        // tournament merge of the token's 8 sorted lists (lanes 8*grp .. 8*grp+7)
        float topv[MAXK];
        int topi[MAXK];
        int ptr = 0;
#pragma unroll
        for (int r = 0; r < MAXK; ++r) {
            float cv = -INFINITY;
            int ci = 0x7fffffff;
#pragma unroll
            for (int q = 0; q < MAXK; ++q)
                if (q == ptr) { cv = bv[q]; ci = bi[q]; }
            float mv = cv;
            int mi = ci;
#pragma unroll
            for (int o = 1; o < SUB; o <<= 1) {
                const float ov = __shfl_xor_sync(DG_FULL_MASK, mv, o);
                const int oi = __shfl_xor_sync(DG_FULL_MASK, mi, o);
                if (ranks_before(ov, oi, mv, mi)) { mv = ov; mi = oi; }
            }
            topv[r] = mv;
            topi[r] = mi;
            if (ci == mi && cv == mv) ++ptr;      // indices are unique: only the owner advances
        }
        (void)lane;
        // u_k = normalize(top values); u_q = normalize(W_q[top idx] . q)
        float ssk = 0.f;
#pragma unroll
        for (int r = 0; r < MAXK; ++r) ssk += (r < K) ? topv[r] * topv[r] : 0.f;
        const float nk = fmaxf(sqrtf(ssk), 1e-12f);
        // thread `sub` computes the query score of rank `sub`
        float qv = 0.f;
        int myi = 0;
#pragma unroll
        for (int r = 0; r < MAXK; ++r)
            if (r == sub) myi = topi[r];
        if (sub < K) {
            const float* wr = WQ + (int64_t)myi * Dh;
            const float* qr = qs + tl * Dh;
            for (int d = 0; d < Dh; ++d) qv = __fadd_rn(qv, __fmul_rn(__ldg(wr + d), qr[d]));
        }
        float ssq = (sub < K) ? qv * qv : 0.f;
#pragma unroll
        for (int o = 1; o < SUB; o <<= 1) ssq += __shfl_xor_sync(DG_FULL_MASK, ssq, o);
        const float nq = fmaxf(sqrtf(ssq), 1e-12f);
        float* rr = res + ((tl * 2 + ax) * 2) * MAXK;
        int* ri = resi + (tl * 2 + ax) * MAXK;
        if (sub < K) {
            float mine = 0.f;
#pragma unroll
            for (int r = 0; r < MAXK; ++r)
                if (r == sub) mine = topv[r];
            rr[sub] = mine / nk;
            rr[MAXK + sub] = qv / nq;
            ri[sub] = myi;
        }
    }
    __syncthreads();
    // Kronecker: thread `sub` writes row i = sub of the K x K product
    const int64_t n = n0 + tl;
    if (n < p.N && sub < K) {
        const int A = K * K;
        const int h = (int)((n / p.T) % p.H);
        const float qsc = p.q_scale ? p.q_scale[h] : 1.f;
        const float* r0 = res + ((tl * 2 + 0) * 2) * MAXK;
        const float* r1 = res + ((tl * 2 + 1) * 2) * MAXK;
        const int* i0 = resi + (tl * 2 + 0) * MAXK;
        const int* i1 = resi + (tl * 2 + 1) * MAXK;
        T* owk = static_cast<T*>(p.out_wk) + n * A;
        T* owq = static_cast<T*>(p.out_wq) + n * A;
        int64_t* oix = p.out_idx + n * A;
        const int i = sub;
        for (int j = 0; j < K; ++j) {
            owk[i * K + j] = dg::from_f<T>(r0[i] * r1[j]);
            owq[i * K + j] = dg::from_f<T>((r0[MAXK + i] * r1[MAXK + j]) * qsc);
            oix[i * K + j] = (int64_t)i0[i] * p.G[1] + i1[j];
        }
    }
}

}  // namespace

namespace dg_host {
bool route_tc_supports(int dtype, int dh, int g0, int g1, int top_k, const void* k, const void* q,
                       const float* rk0, const float* rk1, const float* rq0, const float* rq1, const void* wk,
                       const void* wq, const int64_t* idx);
int route_tc(int dtype, int64_t N, int H, int T, int g0, int g1, int top_k, const void* k, const void* q,
             const float* rk0, const float* rk1, const float* rq0, const float* rq1, const float* q_scale, void* wk,
             void* wq, int64_t* idx, cudaStream_t s);
}  // namespace dg_host

extern "C" int dg_pkm_route(int dtype, int B, int H, int T, int dh, int g0, int g1, int top_k, const void* k,
                            const void* q, const float* router_k0, const float* router_k1,
                            const float* router_q0, const float* router_q1, const float* q_scale, void* wk,
                            void* wq, int64_t* idx, void* stream) {
    if (B <= 0 || H <= 0 || T < 0 || dh <= 0 || g0 <= 0 || g1 <= 0 || top_k <= 0) return DG_ERR_INVALID_ARGUMENT;
    if (!k || !q || !router_k0 || !router_k1 || !router_q0 || !router_q1 || !wk || !wq || !idx)
        return DG_ERR_INVALID_ARGUMENT;
    if (top_k > MAXK || top_k > g0 || top_k > g1 || dh > MAXDH) return DG_ERR_UNSUPPORTED;
    const int64_t N = (int64_t)B * H * T;
    if (N == 0) return DG_OK;
    if (dg_host::route_tc_supports(dtype, dh, g0, g1, top_k, k, q, router_k0, router_k1, router_q0, router_q1, wk, wq,
                                   idx))
        return dg_host::route_tc(dtype, N, H, T, g0, g1, top_k, k, q, router_k0, router_k1, router_q0, router_q1,
                                 q_scale, wk, wq, idx, static_cast<cudaStream_t>(stream));
    RouterParams p{k, q, {router_k0, router_k1}, {router_q0, router_q1}, q_scale, wk, wq, idx, N, H, T, dh,
                   {g0, g1}, top_k};
    const size_t smem = (size_t)(2 * TN * dh + GC * (dh + 1) + TN * 2 * 2 * MAXK) * 4 + TN * 2 * MAXK * 4;
    const dim3 grid((unsigned)((N + TN - 1) / TN));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DG_DISPATCH(dtype, Ty, {
        auto kern = router_kernel<Ty>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return dg_host::record_cuda_error(e);
        kern<<<grid, 256, smem, s>>>(p);
    });
    return dg_host::check_launch();
}
