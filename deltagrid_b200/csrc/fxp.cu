// fxp.cu -- Q16.16 fixed-point recurrence core, bit-exact with the reference engine.
//
// Dense (src/cpp/engine/src/deltagrid_fxp.cpp:380-405) and sparse PKM
// (:298-326), per lane and step:
//     yacc_d = sum_s (int64) wq_s S[s][d]    pacc_d = sum_s (int64) wk_s S[s][d]
//     y_d = (yacc_d + 2^15) >> 16            r_d = v_d - ((pacc_d + 2^15) >> 16)
//     S[s][d] = fxp(alpha, S[s][d]) + fxp(fxp(beta, wk_s), r_d)
// with fxp(a, b) = ((int64) a b + 2^15) >> 16 (include/deltagrid_math_fxp.h:16-19)
// and int32 wrap-around on the additions, as the engine's int32 arithmetic.
// Integer sums are exact and associative, so any reduction order gives the
// engine's result bit for bit.
//
// Dense: one CTA per (lane, tile of 16 columns); SG threads per column hold SPT
// slots in registers and finish the int64 sums with an xor-butterfly.
// PKM: one warp per 4-column (16-byte) slice, lane l holds rows l and l + 32,
// int64 partials reduce-scattered across the warp.
#include "dg_common.cuh"

namespace {

__device__ __forceinline__ int32_t fxp_mul(int32_t a, int32_t b) {
    return (int32_t)(((int64_t)a * (int64_t)b + (1 << 15)) >> 16);
}
__device__ __forceinline__ int32_t wrap_add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
__device__ __forceinline__ int32_t wrap_sub(int32_t a, int32_t b) { return (int32_t)((uint32_t)a - (uint32_t)b); }
__device__ __forceinline__ int64_t shfl_xor64(int64_t v, int o) {
    const int lo = __shfl_xor_sync(DG_FULL_MASK, (int)(v & 0xffffffff), o);
    const int hi = __shfl_xor_sync(DG_FULL_MASK, (int)(v >> 32), o);
    return (int64_t)(((uint64_t)(uint32_t)hi << 32) | (uint32_t)lo);
}
struct FxpDenseParams {
    const int32_t* wk;
    const int32_t* wq;
    const int32_t* v;
    const int32_t* beta;
    const int32_t* alpha;
    int32_t* state;
    int32_t* y;
    int T, S, Dh;
};

template <int SG, int SPT>
__global__ void __launch_bounds__(16 * SG) fxp_dense_kernel(FxpDenseParams p) {
    constexpr int CW = 16;
    const int tid = threadIdx.x, g = tid % SG, cl = tid / SG;
    const int lane_i = blockIdx.y;
    const int c = blockIdx.x * CW + cl;
    const bool cvalid = c < p.Dh;
    const int S = p.S, Dh = p.Dh;
    int32_t* st_g = p.state + (int64_t)lane_i * S * Dh;
    int32_t st[SPT];
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
        const int m = g + SG * j;
        st[j] = (cvalid && m < S) ? st_g[(int64_t)m * Dh + c] : 0;
    }
    for (int t = 0; t < p.T; ++t) {
        const int64_t lt = (int64_t)lane_i * p.T + t;
        const int32_t* wkt = p.wk + lt * S;
        const int32_t* wqt = p.wq + lt * S;
        int64_t ya = 0, pa = 0;
#pragma unroll
        for (int j = 0; j < SPT; ++j) {
            const int m = g + SG * j;
            if (m < S) {
                ya += (int64_t)__ldg(wqt + m) * st[j];
                pa += (int64_t)__ldg(wkt + m) * st[j];
            }
        }
#pragma unroll
        for (int o = 1; o < SG; o <<= 1) {
            ya += shfl_xor64(ya, o);
            pa += shfl_xor64(pa, o);
        }
        const int32_t yv = (int32_t)((ya + (1 << 15)) >> 16);
        const int32_t pred = (int32_t)((pa + (1 << 15)) >> 16);
        const int32_t r = cvalid ? wrap_sub(__ldg(p.v + lt * Dh + c), pred) : 0;
        if (g == 0 && cvalid) p.y[lt * Dh + c] = yv;
        const int32_t al = __ldg(p.alpha + lt), be = __ldg(p.beta + lt);
#pragma unroll
        for (int j = 0; j < SPT; ++j) {
            const int m = g + SG * j;
            if (m < S) st[j] = wrap_add(fxp_mul(al, st[j]), fxp_mul(fxp_mul(be, __ldg(wkt + m)), r));
        }
    }
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
        const int m = g + SG * j;
        if (cvalid && m < S) st_g[(int64_t)m * Dh + c] = st[j];
    }
}

struct FxpPkmParams {
    const int32_t* wk;
    const int32_t* wq;
    const int32_t* idx;
    const int32_t* v;
    const int32_t* beta;
    const int32_t* alpha;
    int32_t* state;
    int32_t* y;
    int32_t* status;
    int T, A, Dh;
    int64_t total;
};

// one warp per 4-column slice; rows m = lane + 32 i (A <= 64)
__global__ void __launch_bounds__(256) fxp_pkm_kernel(FxpPkmParams p) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int col0 = (blockIdx.x * (blockDim.x >> 5) + warp) * 4;
    if (col0 >= p.Dh) return;
    const int lane_i = blockIdx.y;
    const int A = p.A, Dh = p.Dh;
    int32_t* st = p.state + (int64_t)lane_i * p.total * Dh + col0;
    for (int t = 0; t < p.T; ++t) {
        const int64_t lt = (int64_t)lane_i * p.T + t;
        int4 rows[2];
        int32_t wkv[2], wqv[2];
        int64_t X[2];
        bool ok[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int m = lane + 32 * i;
            ok[i] = false; wkv[i] = 0; wqv[i] = 0; X[i] = 0;
            rows[i] = make_int4(0, 0, 0, 0);
            if (m < A) {
                const int32_t x = p.idx[lt * A + m];
                ok[i] = x >= 0 && (int64_t)x < p.total;
                if (!ok[i]) dg::flag_status(p.status, DG_DEVCHK_INDEX_RANGE);
                X[i] = ok[i] ? x : 0;
                wkv[i] = p.wk[lt * A + m];
                wqv[i] = p.wq[lt * A + m];
                if (ok[i]) rows[i] = *reinterpret_cast<const int4*>(st + X[i] * Dh);
            }
        }
        // partials: y (4 columns) and pred (4 columns), int64
        int64_t vals[8];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            int64_t ya = 0, pa = 0;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int32_t sv = (&rows[i].x)[c];
                ya += (int64_t)wqv[i] * sv;
                pa += (int64_t)wkv[i] * sv;
            }
            vals[c] = ya;
            vals[4 + c] = pa;
        }
        // reduce-scatter 8 values over 32 lanes: lane holds value (lane >> 2), full sum
#pragma unroll
        for (int s = 0; s < 3; ++s) {
            const int o = 16 >> s, half = 8 >> (s + 1);
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (i < half) {
                    const int64_t send = upper ? vals[i] : vals[i + half];
                    const int64_t keep = upper ? vals[i + half] : vals[i];
                    vals[i] = keep + shfl_xor64(send, o);
                }
            }
        }
        int64_t red = vals[0];
        red += shfl_xor64(red, 2);
        red += shfl_xor64(red, 1);
        const int vi = lane >> 2;
        int32_t rloc = 0;
        const int32_t rounded = (int32_t)((red + (1 << 15)) >> 16);
        if (vi >= 4) {
            rloc = wrap_sub(p.v[lt * Dh + col0 + (vi - 4)], rounded);
        } else if ((lane & 3) == 0) {
            p.y[lt * Dh + col0 + vi] = rounded;
        }
        int32_t r[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) r[c] = __shfl_sync(DG_FULL_MASK, rloc, (4 + c) << 2);
        const int32_t al = p.alpha[lt], be = p.beta[lt];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            if (ok[i]) {
                const int32_t bw = fxp_mul(be, wkv[i]);
                int4 nv;
                nv.x = wrap_add(fxp_mul(al, rows[i].x), fxp_mul(bw, r[0]));
                nv.y = wrap_add(fxp_mul(al, rows[i].y), fxp_mul(bw, r[1]));
                nv.z = wrap_add(fxp_mul(al, rows[i].z), fxp_mul(bw, r[2]));
                nv.w = wrap_add(fxp_mul(al, rows[i].w), fxp_mul(bw, r[3]));
                *reinterpret_cast<int4*>(st + X[i] * Dh) = nv;
            }
        }
        __syncwarp();
    }
}

}  // namespace

extern "C" {

int dg_fxp_dense_forward(int lanes, int T, int slots, int dh, const int32_t* wk, const int32_t* wq,
                         const int32_t* v, const int32_t* beta, const int32_t* alpha, int32_t* state, int32_t* y,
                         void* stream) {
    if (lanes <= 0 || T < 0 || slots <= 0 || dh <= 0 || !state) return DG_ERR_INVALID_ARGUMENT;
    if (T == 0) return DG_OK;
    if (!wk || !wq || !v || !beta || !alpha || !y) return DG_ERR_INVALID_ARGUMENT;
    if (lanes > 65535) return DG_ERR_UNSUPPORTED;
    FxpDenseParams p{wk, wq, v, beta, alpha, state, y, T, slots, dh};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    dim3 grid((dh + 15) / 16, lanes);
    if (slots <= 64) fxp_dense_kernel<8, 8><<<grid, 128, 0, s>>>(p);
    else if (slots <= 256) fxp_dense_kernel<16, 16><<<grid, 256, 0, s>>>(p);
    else if (slots <= 512) fxp_dense_kernel<16, 32><<<grid, 256, 0, s>>>(p);
    else return DG_ERR_UNSUPPORTED;
    return dg_host::check_launch();
}

int dg_fxp_pkm_forward(int lanes, int T, int active, int64_t total_slots, int dh, const int32_t* wk,
                       const int32_t* wq, const int32_t* idx, const int32_t* v, const int32_t* beta,
                       const int32_t* alpha, int32_t* state, int32_t* y, int32_t* dev_status, void* stream) {
    if (lanes <= 0 || T < 0 || active <= 0 || total_slots <= 0 || dh <= 0 || !state) return DG_ERR_INVALID_ARGUMENT;
    if (T == 0) return DG_OK;
    if (!wk || !wq || !idx || !v || !beta || !alpha || !y) return DG_ERR_INVALID_ARGUMENT;
    if (active > 64 || dh % 4 != 0 || lanes > 65535) return DG_ERR_UNSUPPORTED;
    if ((uintptr_t)state % 16 != 0) return DG_ERR_MISALIGNED;
    FxpPkmParams p{wk, wq, idx, v, beta, alpha, state, y, dev_status, T, active, dh, total_slots};
    const int slices = dh / 4;
    const int wpb = slices < 8 ? slices : 8;
    dim3 grid((slices + wpb - 1) / wpb, lanes);
    fxp_pkm_kernel<<<grid, 32 * wpb, 0, static_cast<cudaStream_t>(stream)>>>(p);
    return dg_host::check_launch();
}

}  // extern "C"
