// dense_chunk_tc.cu -- chunkwise (WY/UT form) dense delta-rule recurrence on tcgen05.
//
// The per-step recurrence (src/cpp/delta_kernel.cu:78-112)
//     y_t = q_t^T S,  r_t = v_t - k_t^T S,  S <- alpha_t S + beta_t k_t r_t^T
// is evaluated C = 64 steps at a time, following the chunked algebra of the
// reference's PyTorch prefill (src/modules/memory.py:325-410).  Within a chunk,
// with a_i = prod_{l<=i} alpha_l, aprev_i = a_{i-1}, Gamma_ij = aprev_i / a_j:
//     L  = strict_lower(Gamma o beta_j o K K^T),      T = (I + L)^{-1}
//     R  = T (V - aprev o (K S0))                      (the r_t of the chunk)
//     Y  = aprev o (Q S0) + strict_lower(Gamma o Q K^T) (beta o R)
//     S1 = a_{C-1} S0 + K^T diag(a_{C-1}/a_j beta_j) R
// Every product is a tensor-core MMA: [K;Q] K^T and [K;Q] S0 as one M=128
// operand, T X and Mqk R as M=128 MMAs whose other 64 rows are a zero tile,
// and the state update as S/128 M=128 MMAs accumulating into the state.
//
// Hardware mapping (one CTA per lane (b,h), 4 warps):
//   - S (slots x 64, fp32) lives in TMEM for all T steps; it is only rounded to
//     the storage dtype as an MMA operand copy, streamed 128 slots at a time
//     TMEM -> registers -> fp16 shared memory.
//   - wk / wq / v chunks arrive by TMA (3-D maps [lane][T][cols], 128B swizzle;
//     out-of-range steps of the last chunk read as zeros, which contribute
//     nothing: beta = 0 and alpha = 1 there).
//   - T = (I+L)^{-1} is formed in fp32 on CUDA cores by 16x16 block
//     forward substitution and rounded to the operand dtype.
//   - thread 0 issues TMA and MMAs; completion is tracked with mbarriers
//     (tcgen05.commit); every wait is bounded and turns into an error status.
//   - y is written per token row; s_final (and the fp32 copy) at the end.
//
// Inputs: fp16 (kind::f16).  Dh = 64, slots in {128, 256, 384, 512}.
#include "dg_common.cuh"
#include "tc_util.cuh"

#include <cuda.h>

namespace {

constexpr int CH = 64;        // steps per chunk
constexpr int DH = 64;        // head dimension handled by this kernel
constexpr uint32_t SLICE = 16384;   // 64 slots x 128 rows (K rows 0-63, Q rows 64-127) of fp16

struct ChunkParams {
    const void* beta;
    const void* decay;
    const void* s_init;
    void* out;
    void* s_final;
    float* err_out;
    float* s_final_f;
    int32_t* status;
    int H, T, nchunks, dynamic_decay;
};

template <int S>
struct Layout {
    static constexpr int NSL = S / 64;
    static constexpr int NB = S / 128;
    static constexpr uint32_t KQ = 0;
    static constexpr uint32_t S0 = KQ + NSL * SLICE;        // 2 x 16 KB
    static constexpr uint32_t TZM = S0 + 2 * 16384;         // [T | Z | Mqk] 3 x 8 KB
    static constexpr uint32_t XR = TZM + 3 * 8192;          // X, then R'
    static constexpr uint32_t VR = XR + 8192;               // V, then R*beta
    static constexpr uint32_t LT = VR + 8192;               // fp32 [64][65]
    static constexpr uint32_t PB = LT + 64 * 65 * 4;        // fp32 3 x [16][16]
    static constexpr uint32_t SC = PB + 3 * 1024;           // beta, aprev, aincl, aend (4 x 64 fp32)
    static constexpr uint32_t BAR = SC + 4 * 256 + 16;      // 8 mbarriers + tmem base
    static constexpr uint32_t BYTES = BAR + 8 * 8 + 16;
    static constexpr uint32_t ACC1 = NB * 64;               // TMEM column bases
    static constexpr uint32_t ACC2 = ACC1 + 64;
    static constexpr uint32_t ACC3 = ACC2 + 64;
    static constexpr uint32_t ACC4 = ACC3 + 64;
    static constexpr uint32_t TMEM_COLS = 512;
};

constexpr uint32_t IDESC_KK = tc::make_idesc(128, 64, 0, 0, 0);
constexpr uint32_t IDESC_KM = tc::make_idesc(128, 64, 0, 0, 1);
constexpr uint32_t IDESC_MM = tc::make_idesc(128, 64, 0, 1, 1);

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_h2(uint32_t u) {
    return __half22float2(*reinterpret_cast<__half2*>(&u));
}

// write 64 fp32 values as one 128-byte swizzled fp16 row
__device__ __forceinline__ void st_row_f16(uint8_t* tile, int row, const float* x) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 v;
        v.x = pack_h2(x[8 * c + 0], x[8 * c + 1]);
        v.y = pack_h2(x[8 * c + 2], x[8 * c + 3]);
        v.z = pack_h2(x[8 * c + 4], x[8 * c + 5]);
        v.w = pack_h2(x[8 * c + 6], x[8 * c + 7]);
        *reinterpret_cast<uint4*>(tile + tc::sw128(row, c)) = v;
    }
}

// load a TMEM row (this thread's lane) of 64 fp32 columns
__device__ __forceinline__ void ld_row64(uint32_t taddr, float* x) {
    uint32_t a[32], b[32];
    tc::tmem_ld32(taddr, a);
    tc::tmem_ld32(taddr + 32, b);
    tc::tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        x[i] = __uint_as_float(a[i]);
        x[32 + i] = __uint_as_float(b[i]);
    }
}

// bounded wait by every thread, then a collective verdict; true = failed
__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity) {
    const bool ok = tc::mbar_wait(bar, parity);
    const bool failed = __syncthreads_or(!ok) != 0;
    tc::tc_fence_after();
    return failed;
}

// (I + L)^{-1} for strictly lower L (64x64 fp32 at lt, row stride 65), by 16x16
// blocks: diagonal blocks by forward substitution, off-diagonal blocks by
//   T_ik = -D_i sum_{j=k}^{i-1} L_ij T_jk   (processed along diagonals i-k = 1, 2, 3).
// Diagonal inverses overwrite L_ii; T_ik (i > k) is stored in the unused upper block (k, i).
__device__ void invert_unit_lower(float* lt, float* pb, int tid) {
    constexpr int LD = 65;
    auto L = [&](int bi, int bk, int a, int b) -> float& { return lt[(16 * bi + a) * LD + 16 * bk + b]; };
    auto Tm = [&](int bi, int bk, int a, int b) -> float& {
        return (bi == bk) ? lt[(16 * bi + a) * LD + 16 * bi + b] : lt[(16 * bk + a) * LD + 16 * bi + b];
    };
    // diagonal blocks: thread (blk, col) solves column col of (I + L_bb) x = e_col
    float x[16];
    if (tid < 64) {
        const int blk = tid >> 4, col = tid & 15;
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            float s = (r == col) ? 1.f : 0.f;
#pragma unroll
            for (int j = 0; j < r; ++j) s -= L(blk, blk, r, j) * x[j];
            x[r] = s;
        }
    }
    __syncthreads();
    if (tid < 64) {
        const int blk = tid >> 4, col = tid & 15;
#pragma unroll
        for (int r = 0; r < 16; ++r) L(blk, blk, r, col) = x[r];
    }
    __syncthreads();
    // diagonals d = 1..3; targets (i, k = i - d)
    for (int d = 1; d <= 3; ++d) {
        const int ntarget = 4 - d;
        // P_t = sum_{j=k}^{i-1} L_ij T_jk
        for (int e = tid; e < ntarget * 256; e += 128) {
            const int t = e >> 8, a = (e >> 4) & 15, b = e & 15;
            const int i = t + d, k = t;
            float s = 0.f;
            for (int j = k; j < i; ++j)
#pragma unroll
                for (int m = 0; m < 16; ++m) s += L(i, j, a, m) * Tm(j, k, m, b);
            pb[t * 256 + a * 16 + b] = s;
        }
        __syncthreads();
        // T_ik = -D_i P_t
        for (int e = tid; e < ntarget * 256; e += 128) {
            const int t = e >> 8, a = (e >> 4) & 15, b = e & 15;
            const int i = t + d, k = t;
            float s = 0.f;
#pragma unroll
            for (int m = 0; m < 16; ++m) s += Tm(i, i, a, m) * pb[t * 256 + m * 16 + b];
            Tm(i, k, a, b) = -s;
        }
        __syncthreads();
    }
}

template <int S>
__global__ void __launch_bounds__(128, 1)
    dense_chunk_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmq,
                       const __grid_constant__ CUtensorMap tmv, ChunkParams p) {
    using Ly = Layout<S>;
    constexpr int NSL = Ly::NSL, NB = Ly::NB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kq = sm + Ly::KQ;
    uint8_t* s0b = sm + Ly::S0;
    uint8_t* tzm = sm + Ly::TZM;
    uint8_t* xr = sm + Ly::XR;
    uint8_t* vr = sm + Ly::VR;
    float* lt = reinterpret_cast<float*>(sm + Ly::LT);
    float* pb = reinterpret_cast<float*>(sm + Ly::PB);
    float* s_beta = reinterpret_cast<float*>(sm + Ly::SC);
    float* s_aprev = s_beta + 64;
    float* s_aincl = s_aprev + 64;
    float* s_aend = s_aincl + 64;
    float* s_atot = s_aend + 64;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly::BAR);
    uint64_t* bar_load = bars + 0;
    uint64_t* bar_acc1 = bars + 1;
    uint64_t* bar_acc2 = bars + 2;
    uint64_t* bar_acc3 = bars + 3;
    uint64_t* bar_acc4 = bars + 4;
    uint64_t* bar_upd = bars + 5;
    uint64_t* bar_s0 = bars + 6;     // two buffers
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lane_bh = blockIdx.x;
    const int h = lane_bh % p.H;
    const int T_ = p.T;
    const __half* beta = static_cast<const __half*>(p.beta);
    const __half* decay = static_cast<const __half*>(p.decay);

    if (warp == 0) tc::tmem_alloc(tmem_holder, Ly::TMEM_COLS);
    if (tid == 0) {
        for (int i = 0; i < 8; ++i) tc::mbar_init(bars + i, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tmk);
        tc::prefetch_tmap(&tmq);
        tc::prefetch_tmap(&tmv);
    }
    // zero tile Z (rows 64..127 of [T;Z] and rows 0..63 of [Z;Mqk])
    for (int i = tid; i < 8192 / 16; i += 128) reinterpret_cast<uint4*>(tzm + 8192)[i] = make_uint4(0, 0, 0, 0);
    tc::fence_proxy_async();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t tq = tmem + ((uint32_t)(32 * warp) << 16);   // this warp's TMEM lane quarter
    const float alpha_static = p.dynamic_decay ? 1.f : __half2float(decay[h]);

    // initial state -> TMEM (thread = slot row 128 b + 32 warp + lane)
    {
        const __half* s_init = static_cast<const __half*>(p.s_init);
        for (int b = 0; b < NB; ++b) {
            const int slot = 128 * b + 32 * warp + lane;
            uint32_t r0[32], r1[32];
            if (s_init) {
                const uint4* src = reinterpret_cast<const uint4*>(s_init + ((int64_t)lane_bh * S + slot) * DH);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint4 v = src[c];
                    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = unpack_h2(w4[e]);
                        const int col = 8 * c + 2 * e;
                        uint32_t* dst = col < 32 ? r0 : r1;
                        dst[col & 31] = __float_as_uint(f.x);
                        dst[(col & 31) + 1] = __float_as_uint(f.y);
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) { r0[i] = 0u; r1[i] = 0u; }
            }
            tc::tmem_st32(tq + 64 * b, r0);
            tc::tmem_st32(tq + 64 * b + 32, r1);
        }
        tc::tmem_wait_st();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();

    uint32_t s0_uses[2] = {0u, 0u};
    bool failed = false;
    for (int c = 0; c < p.nchunks && !failed; ++c) {
        const int t0 = c * CH;
        const uint32_t par = (uint32_t)(c & 1);
        // the previous chunk's update MMA must finish before its K tiles are
        // overwritten and before the state is read again
        if (c > 0 && wait_all(bar_upd, par ^ 1u)) { failed = true; break; }
        if (tid == 0) {
            tc::mbar_expect_tx(bar_load, NSL * SLICE + 8192);
            for (int s = 0; s < NSL; ++s) {
                tc::tma_load_3d(kq + s * SLICE, &tmk, bar_load, 64 * s, t0, lane_bh);
                tc::tma_load_3d(kq + s * SLICE + 8192, &tmq, bar_load, 64 * s, t0, lane_bh);
            }
            tc::tma_load_3d(vr, &tmv, bar_load, 0, t0, lane_bh);
        }
        if (tid < CH) {
            const int t = t0 + tid;
            const bool ok = t < T_;
            const int64_t bt = (int64_t)lane_bh * T_ + t;
            s_beta[tid] = ok ? __half2float(beta[bt]) : 0.f;
            s_aincl[tid] = ok ? (p.dynamic_decay ? __half2float(decay[bt]) : alpha_static) : 1.f;
        }
        __syncthreads();
        if (tid == 0) {
            float prod = 1.f;
            for (int i = 0; i < CH; ++i) {
                s_aprev[i] = prod;
                prod *= s_aincl[i];
                s_aincl[i] = prod;
            }
            for (int i = 0; i < CH; ++i) s_aend[i] = prod / s_aincl[i];
            *s_atot = prod;
        }
        if (wait_all(bar_load, par)) { failed = true; break; }

        // ---- G = K K^T, QK = Q K^T (TMEM ACC1: lanes 0-63 G, 64-127 QK) ----
        if (tid == 0) {
            for (int s = 0; s < NSL; ++s)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t base = tc::smem_u32(kq + s * SLICE) + 32 * kk;
                    tc::mma_f16(tmem + Ly::ACC1, tc::make_desc(base, 16, 1024), tc::make_desc(base, 16, 1024),
                                IDESC_KK, (s | kk) != 0);
                }
            tc::mma_commit(bar_acc1);
        }
        const float atot = *s_atot;

        // ---- [K;Q] S0 over 128-slot blocks; S0 streamed TMEM -> fp16 smem ----
        for (int b = 0; b < NB; ++b) {
            const int buf = b & 1;
            bool bad = false;
            if (s0_uses[buf] > 0) bad = !tc::mbar_wait(bar_s0 + buf, (s0_uses[buf] - 1) & 1u);
            tc::tc_fence_after();
            float x[64];
            ld_row64(tq + 64 * b, x);
            st_row_f16(s0b + buf * 16384, 32 * warp + lane, x);
            if (atot != 1.f) {
                uint32_t r0[32], r1[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    r0[i] = __float_as_uint(atot * x[i]);
                    r1[i] = __float_as_uint(atot * x[32 + i]);
                }
                tc::tmem_st32(tq + 64 * b, r0);
                tc::tmem_st32(tq + 64 * b + 32, r1);
                tc::tmem_wait_st();
            }
            tc::fence_proxy_async();
            tc::tc_fence_before();
            if (__syncthreads_or(bad)) { failed = true; break; }
            if (tid == 0) {
                tc::tc_fence_after();
#pragma unroll
                for (int sl = 0; sl < 2; ++sl)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t a = tc::smem_u32(kq + (2 * b + sl) * SLICE) + 32 * kk;
                        const uint32_t bb = tc::smem_u32(s0b + buf * 16384) + (sl * 4 + kk) * 2048;
                        tc::mma_f16(tmem + Ly::ACC2, tc::make_desc(a, 16, 1024), tc::make_desc(bb, 16384, 1024),
                                    IDESC_KM, (b | sl | kk) != 0);
                    }
                tc::mma_commit(bar_s0 + buf);
                if (b == NB - 1) tc::mma_commit(bar_acc2);
            }
            s0_uses[buf]++;
        }
        if (failed) break;

        // ---- L (warps 0-1) and Mqk (warps 2-3) from ACC1 ----
        if (wait_all(bar_acc1, par)) { failed = true; break; }
        {
            float g[64];
            ld_row64(tq + Ly::ACC1, g);
            const int i = 32 * (warp & 1) + lane;
            const float ap = s_aprev[i];
            if (warp < 2) {
#pragma unroll
                for (int j = 0; j < 64; ++j) lt[i * 65 + j] = (j < i) ? (ap / s_aincl[j]) * s_beta[j] * g[j] : 0.f;
            } else {
#pragma unroll
                for (int j = 0; j < 64; ++j) g[j] = (j < i) ? (ap / s_aincl[j]) * g[j] : 0.f;   // beta is in R*beta
                st_row_f16(tzm + 16384, i, g);
            }
        }
        __syncthreads();
        invert_unit_lower(lt, pb, tid);
        if (tid < 64) {
            const int i = tid;
            float row[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const int bi = i >> 4, bj = j >> 4;
                float v = 0.f;
                if (j <= i) v = (bi == bj) ? lt[i * 65 + j] : lt[(16 * bj + (i & 15)) * 65 + 16 * bi + (j & 15)];
                row[j] = v;
            }
            st_row_f16(tzm, i, row);
        }
        tc::fence_proxy_async();

        // ---- X = V - aprev o (K S0)  (warps 0-1, token rows) ----
        if (wait_all(bar_acc2, par)) { failed = true; break; }
        if (warp < 2) {
            const int i = 32 * warp + lane;
            float d1[64];
            ld_row64(tq + Ly::ACC2, d1);
            const float ap = s_aprev[i];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
                const uint4 v = *reinterpret_cast<const uint4*>(vr + tc::sw128(i, cc));
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = unpack_h2(w4[e]);
                    d1[8 * cc + 2 * e] = f.x - ap * d1[8 * cc + 2 * e];
                    d1[8 * cc + 2 * e + 1] = f.y - ap * d1[8 * cc + 2 * e + 1];
                }
            }
            st_row_f16(xr, i, d1);
        }
        tc::fence_proxy_async();
        tc::tc_fence_before();
        __syncthreads();

        // ---- R = T X  (ACC3 lanes 0-63) ----
        if (tid == 0) {
            tc::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                tc::mma_f16(tmem + Ly::ACC3, tc::make_desc(tc::smem_u32(tzm) + 32 * kk, 16, 1024),
                            tc::make_desc(tc::smem_u32(xr) + kk * 2048, 16384, 1024), IDESC_KM, kk != 0);
            tc::mma_commit(bar_acc3);
        }
        if (wait_all(bar_acc3, par)) { failed = true; break; }
        if (warp < 2) {
            const int i = 32 * warp + lane;
            float r[64];
            ld_row64(tq + Ly::ACC3, r);
            const int t = t0 + i;
            if (p.err_out && t < T_) {
                float4* dst = reinterpret_cast<float4*>(p.err_out + ((int64_t)lane_bh * T_ + t) * DH);
#pragma unroll
                for (int q = 0; q < 16; ++q) dst[q] = make_float4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
            }
            const float bi = s_beta[i], ae = s_aend[i];
            float rb[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                rb[j] = bi * r[j];
                r[j] = ae * rb[j];
            }
            st_row_f16(vr, i, rb);     // R * beta (V is dead)
            st_row_f16(xr, i, r);      // R' = a_end * beta * R (X is dead)
        }
        tc::fence_proxy_async();
        tc::tc_fence_before();
        __syncthreads();

        // ---- ACC4 = Mqk (R*beta) (lanes 64-127); S += K^T R' ----
        if (tid == 0) {
            tc::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                tc::mma_f16(tmem + Ly::ACC4, tc::make_desc(tc::smem_u32(tzm + 8192) + 32 * kk, 16, 1024),
                            tc::make_desc(tc::smem_u32(vr) + kk * 2048, 16384, 1024), IDESC_KM, kk != 0);
            tc::mma_commit(bar_acc4);
            for (int b = 0; b < NB; ++b)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    tc::mma_f16(tmem + 64 * b,
                                tc::make_desc(tc::smem_u32(kq + 2 * b * SLICE) + kk * 2048, SLICE, 1024),
                                tc::make_desc(tc::smem_u32(xr) + kk * 2048, 16384, 1024), IDESC_MM, 1u);
            tc::mma_commit(bar_upd);
        }

        // ---- Y = aprev o (Q S0) + Mqk R  (warps 2-3, token rows) ----
        if (wait_all(bar_acc4, par)) { failed = true; break; }
        if (warp >= 2) {
            const int i = 32 * (warp - 2) + lane;
            float y[64], m[64];
            ld_row64(tq + Ly::ACC2, y);
            ld_row64(tq + Ly::ACC4, m);
            const int t = t0 + i;
            if (t < T_) {
                const float ap = s_aprev[i];
                uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + ((int64_t)lane_bh * T_ + t) * DH);
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    float o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) o[e] = fmaf(ap, y[8 * cc + e], m[8 * cc + e]);
                    dst[cc] = make_uint4(pack_h2(o[0], o[1]), pack_h2(o[2], o[3]), pack_h2(o[4], o[5]),
                                         pack_h2(o[6], o[7]));
                }
            }
        }
    }

    if (!failed && p.nchunks > 0) failed = wait_all(bar_upd, (uint32_t)((p.nchunks - 1) & 1));
    if (!failed) {
        __half* s_fin = static_cast<__half*>(p.s_final);
        for (int b = 0; b < NB; ++b) {
            const int slot = 128 * b + 32 * warp + lane;
            float x[64];
            ld_row64(tq + 64 * b, x);
            const int64_t o = ((int64_t)lane_bh * S + slot) * DH;
            uint4* dst = reinterpret_cast<uint4*>(s_fin + o);
#pragma unroll
            for (int cc = 0; cc < 8; ++cc)
                dst[cc] = make_uint4(pack_h2(x[8 * cc], x[8 * cc + 1]), pack_h2(x[8 * cc + 2], x[8 * cc + 3]),
                                     pack_h2(x[8 * cc + 4], x[8 * cc + 5]), pack_h2(x[8 * cc + 6], x[8 * cc + 7]));
            if (p.s_final_f) {
                float4* df = reinterpret_cast<float4*>(p.s_final_f + o);
#pragma unroll
                for (int q = 0; q < 16; ++q) df[q] = make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
            }
        }
    } else if (tid == 0) {
        dg::flag_status(p.status, DG_DEVCHK_TIMEOUT);
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, Ly::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 3-D map over [lanes][T][cols] fp16 with a 64 x 64 box and 128B swizzle
bool make_map(CUtensorMap* m, const void* base, int cols, int T, int lanes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)T, (cuuint64_t)lanes};
    cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)cols * 2 * (cuuint64_t)T};
    cuuint32_t box[3] = {64, 64, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int S>
int launch_chunk(const void* v, const void* beta, const void* wk, const void* wq, const void* decay,
                 int dynamic_decay, const void* s_init, void* out, void* s_final, float* err_out,
                 float* s_final_f, int B, int H, int T, int32_t* status, cudaStream_t stream) {
    const int lanes = B * H;
    CUtensorMap mk, mq, mv;
    if (!make_map(&mk, wk, S, T, lanes) || !make_map(&mq, wq, S, T, lanes) || !make_map(&mv, v, DH, T, lanes))
        return DG_ERR_UNSUPPORTED;
    ChunkParams p{beta, decay, s_init, out, s_final, err_out, s_final_f, status,
                  H, T, (T + CH - 1) / CH, dynamic_decay};
    const size_t smem = Layout<S>::BYTES + 1024;
    auto kern = dense_chunk_kernel<S>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    kern<<<lanes, 128, smem, stream>>>(mk, mq, mv, p);
    return dg_host::check_launch();
}

}  // namespace

namespace dg_host {

bool dense_chunked_tc_supports(int dtype, int B, int H, int T, int S, int Dh) {
    (void)B; (void)H;
    return dtype == DG_DTYPE_F16 && Dh == DH && T > 0 && (S == 128 || S == 256 || S == 384 || S == 512);
}

int dense_forward_chunked_tc(int dtype, int B, int H, int T, int S, int Dh, const void* v, const void* beta,
                             const void* wk, const void* wq, const void* decay, int dynamic_decay,
                             const void* s_init, void* out, void* s_final, float* err_out, float* s_final_f,
                             cudaStream_t stream) {
    if (!dense_chunked_tc_supports(dtype, B, H, T, S, Dh)) return DG_ERR_UNSUPPORTED;
    const uintptr_t mis = (uintptr_t)v | (uintptr_t)wk | (uintptr_t)wq | (uintptr_t)out | (uintptr_t)s_final |
                          (uintptr_t)(s_init ? s_init : s_final) | (uintptr_t)(err_out ? (void*)err_out : s_final) |
                          (uintptr_t)(s_final_f ? (void*)s_final_f : s_final);
    if (mis & 15) return DG_ERR_MISALIGNED;
    int32_t* status = nullptr;
    switch (S) {
    case 128: return launch_chunk<128>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, stream);
    case 256: return launch_chunk<256>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, stream);
    case 384: return launch_chunk<384>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, stream);
    case 512: return launch_chunk<512>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, stream);
    default: return DG_ERR_UNSUPPORTED;
    }
}

}  // namespace dg_host
