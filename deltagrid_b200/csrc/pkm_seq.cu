// pkm_seq.cu -- Sparse Delta-PKM recurrence: gather, delta update, scatter.
//
// Math (src/cpp/delta_kernel.cu:885-920), per lane (b,h) and step t with the
// `active` slot indices idx_t (distinct within a step):
//     s_m = S[idx_m]            y = sum_m wq_m s_m      pred = sum_m wk_m s_m
//     r = v - pred              S[idx_m] = cast(alpha s_m + (beta r) wk_m)
// Touched rows are rounded to the storage dtype every step, as the reference
// stores them every step (:918).
//
// Vector kernel layout: one CTA per lane (more when Dh needs more than 8
// warps).  Warp w owns the 16-byte column slice [w*CPW, (w+1)*CPW) of every row
// (CPW = 16 / sizeof(T)), so each gathered row slice is one 128-bit load and a
// warp needs nothing from other warps: all hazards between consecutive steps
// (a row written at t and read at t+1) stay inside one warp and are ordered by
// __syncwarp.  Lane l holds rows m = l + 32 i.  The 2*CPW partial sums (y and
// pred per column) are reduce-scattered across the warp with CPW*2-1 + log
// shuffles, r is formed on the lanes that hold pred and shuffled back.  All
// `active` gathers of a step are independent loads, so a step costs about one
// memory round trip.
#include "dg_common.cuh"

namespace {

struct PkmParams {
    const void* v;
    const void* beta;
    const void* wk;
    const void* wq;
    const int64_t* idx;
    const void* decay;
    void* state;
    void* out;
    void* saved;
    int32_t* status;
    int B, H, T, A, Dh;
    int64_t total;
    int dynamic_decay;
};

template <int NV>
struct Log2 { static constexpr int v = (NV <= 1) ? 0 : 1 + Log2<NV / 2>::v; };
template <>
struct Log2<1> { static constexpr int v = 0; };

// Sums vals[] over the 32 lanes of the warp and returns, on each lane, the sum
// of value index (lane >> (5 - log2 NV)).
template <int NV>
__device__ __forceinline__ float warp_reduce_scatter(float (&vals)[NV], int lane) {
    constexpr int LOG = Log2<NV>::v;
#pragma unroll
    for (int s = 0; s < LOG; ++s) {
        const int o = 16 >> s;
        const int half = NV >> (s + 1);
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < NV / 2; ++i) {
            if (i < half) {
                const float send = upper ? vals[i] : vals[i + half];
                const float keep = upper ? vals[i + half] : vals[i];
                vals[i] = keep + __shfl_xor_sync(DG_FULL_MASK, send, o);
            }
        }
    }
    float x = vals[0];
#pragma unroll
    for (int o = (16 >> LOG); o >= 1; o >>= 1) x += __shfl_xor_sync(DG_FULL_MASK, x, o);
    return x;
}

template <typename T, int RPL>
__global__ void __launch_bounds__(256) pkm_seq_vec_kernel(PkmParams p) {
    using V = dg::Vec16<T>;
    constexpr int CPW = V::N;           // columns per warp slice
    constexpr int NV = 2 * CPW;         // y and pred partials
    constexpr int LOG = Log2<NV>::v;
    constexpr int DUP = 5 - LOG;        // lanes per reduced value = 2^DUP

    const int lane_id = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int slice = blockIdx.x * (blockDim.x >> 5) + warp;
    const int col0 = slice * CPW;
    if (col0 >= p.Dh) return;
    const int lane = blockIdx.y;        // b * H + h
    const int h = lane % p.H;
    const int A = p.A, Dh = p.Dh, T_ = p.T;
    const int64_t total = p.total;

    const T* __restrict__ v = static_cast<const T*>(p.v);
    const T* __restrict__ beta = static_cast<const T*>(p.beta);
    const T* __restrict__ wk = static_cast<const T*>(p.wk);
    const T* __restrict__ wq = static_cast<const T*>(p.wq);
    const T* __restrict__ decay = static_cast<const T*>(p.decay);
    T* state = static_cast<T*>(p.state) + (int64_t)lane * total * Dh + col0;
    T* out = static_cast<T*>(p.out);
    T* saved = static_cast<T*>(p.saved);

    const int vi = lane_id >> DUP;                      // value index this lane ends with
    const bool leader = (lane_id & ((1 << DUP) - 1)) == 0;
    const float alpha_static = p.dynamic_decay ? 1.f : dg::to_f(decay[h]);

    for (int t = 0; t < T_; ++t) {
        const int64_t bt = (int64_t)lane * T_ + t;
        int64_t X[RPL];
        float wkv[RPL], wqv[RPL];
        bool ok[RPL];
        V rows[RPL];
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
            const int m = lane_id + 32 * i;
            X[i] = 0;
            ok[i] = false;
            wkv[i] = 0.f;
            wqv[i] = 0.f;
            if (m < A) {
                const int64_t x = p.idx[bt * A + m];
                ok[i] = (x >= 0) && (x < total);
                if (!ok[i]) dg::flag_status(p.status, DG_DEVCHK_INDEX_RANGE);
                X[i] = ok[i] ? x : 0;
                wkv[i] = dg::to_f(wk[bt * A + m]);
                wqv[i] = dg::to_f(wq[bt * A + m]);
            }
        }
#pragma unroll
        for (int i = 0; i < RPL; ++i)
            rows[i].raw = ok[i] ? dg::ld16(state + X[i] * Dh) : make_uint4(0, 0, 0, 0);

        float vals[NV];
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
            float y = 0.f, pr = 0.f;
#pragma unroll
            for (int i = 0; i < RPL; ++i) {
                const float s = rows[i].get(c);
                y = fmaf(wqv[i], s, y);
                pr = fmaf(wkv[i], s, pr);
            }
            vals[c] = y;
            vals[CPW + c] = pr;
        }
        const float red = warp_reduce_scatter<NV>(vals, lane_id);
        const float al = p.dynamic_decay ? dg::to_f(decay[bt]) : alpha_static;
        const float bta = dg::to_f(beta[bt]);
        float rloc = 0.f;
        if (vi >= CPW) {
            rloc = bta * (dg::to_f(v[bt * Dh + col0 + (vi - CPW)]) - red);   // beta * r
        } else if (leader) {
            out[bt * Dh + col0 + vi] = dg::from_f<T>(red);
        }
        float br[CPW];
#pragma unroll
        for (int c = 0; c < CPW; ++c) br[c] = __shfl_sync(DG_FULL_MASK, rloc, (CPW + c) << DUP);

#pragma unroll
        for (int i = 0; i < RPL; ++i) {
            const int m = lane_id + 32 * i;
            if (saved && m < A) dg::st16(saved + (bt * A + m) * Dh + col0, rows[i].raw);
            if (ok[i]) {
                V nv;
#pragma unroll
                for (int c = 0; c < CPW; ++c) nv.set(c, fmaf(al, rows[i].get(c), br[c] * wkv[i]));
                dg::st16(state + X[i] * Dh, nv.raw);
            }
        }
        __syncwarp();
    }
}

// Scalar fallback (any Dh, any alignment, any active count): one thread per
// column, the loop order of delta_kernel.cu:885-920.
template <typename T>
__global__ void pkm_seq_scalar_kernel(PkmParams p) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= p.Dh) return;
    const int lane = blockIdx.y;
    const int h = lane % p.H;
    const int A = p.A, Dh = p.Dh;
    const T* v = static_cast<const T*>(p.v);
    const T* beta = static_cast<const T*>(p.beta);
    const T* wk = static_cast<const T*>(p.wk);
    const T* wq = static_cast<const T*>(p.wq);
    const T* decay = static_cast<const T*>(p.decay);
    T* state = static_cast<T*>(p.state) + (int64_t)lane * p.total * Dh + d;
    T* saved = static_cast<T*>(p.saved);
    for (int t = 0; t < p.T; ++t) {
        const int64_t bt = (int64_t)lane * p.T + t;
        const float al = p.dynamic_decay ? dg::to_f(decay[bt]) : dg::to_f(decay[h]);
        float y = 0.f, pr = 0.f;
        for (int m = 0; m < A; ++m) {
            const int64_t x = p.idx[bt * A + m];
            const bool ok = x >= 0 && x < p.total;
            if (!ok && d == 0) dg::flag_status(p.status, DG_DEVCHK_INDEX_RANGE);
            const float s = ok ? dg::to_f(state[x * Dh]) : 0.f;
            if (saved) saved[(bt * A + m) * Dh + d] = dg::from_f<T>(s);
            y = fmaf(dg::to_f(wq[bt * A + m]), s, y);
            pr = fmaf(dg::to_f(wk[bt * A + m]), s, pr);
        }
        static_cast<T*>(p.out)[bt * Dh + d] = dg::from_f<T>(y);
        const float br = dg::to_f(beta[bt]) * (dg::to_f(v[bt * Dh + d]) - pr);
        for (int m = 0; m < A; ++m) {
            const int64_t x = p.idx[bt * A + m];
            if (x >= 0 && x < p.total) {
                const float s = dg::to_f(state[x * Dh]);
                state[x * Dh] = dg::from_f<T>(fmaf(al, s, br * dg::to_f(wk[bt * A + m])));
            }
        }
    }
}

template <typename T>
int dispatch_pkm(const PkmParams& p, cudaStream_t s) {
    constexpr int CPW = 16 / sizeof(T);
    const bool vec_ok = (p.Dh % CPW == 0) && ((uintptr_t)p.state % 16 == 0) &&
                        (p.saved == nullptr || (uintptr_t)p.saved % 16 == 0) && p.A <= 256;
    if (vec_ok) {
        const int slices = p.Dh / CPW;
        const int wpb = slices < 8 ? slices : 8;
        dim3 grid((slices + wpb - 1) / wpb, p.B * p.H);
        const int threads = wpb * 32;
        if (p.A <= 32) pkm_seq_vec_kernel<T, 1><<<grid, threads, 0, s>>>(p);
        else if (p.A <= 64) pkm_seq_vec_kernel<T, 2><<<grid, threads, 0, s>>>(p);
        else if (p.A <= 128) pkm_seq_vec_kernel<T, 4><<<grid, threads, 0, s>>>(p);
        else pkm_seq_vec_kernel<T, 8><<<grid, threads, 0, s>>>(p);
    } else {
        const int bs = p.Dh < 64 ? ((p.Dh + 31) / 32) * 32 : 64;
        dim3 grid((p.Dh + bs - 1) / bs, p.B * p.H);
        pkm_seq_scalar_kernel<T><<<grid, bs, 0, s>>>(p);
    }
    return dg_host::check_launch();
}

}  // namespace

namespace dg_host {

int pkm_forward_v1(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v,
                   const void* beta, const void* wk, const void* wq, const int64_t* idx,
                   const void* decay, int dynamic_decay, void* state, void* out, void* saved,
                   int32_t* status, cudaStream_t stream) {
    PkmParams p{v, beta, wk, wq, idx, decay, state, out, saved, status,
                B, H, T, A, Dh, total, dynamic_decay};
    DG_DISPATCH(dtype, Ty, return dispatch_pkm<Ty>(p, stream));
    return DG_ERR_INVALID_ARGUMENT;
}

}  // namespace dg_host
