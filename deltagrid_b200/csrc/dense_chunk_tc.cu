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
// Hardware mapping (one CTA per lane (b,h), two warpgroups):
//   - S (slots x 64, fp32) lives in TMEM for all T steps; it is only rounded to
//     the storage dtype as an MMA operand copy, streamed 128 slots at a time
//     TMEM -> registers -> fp16 shared memory.
//   - wk / wq / v chunks arrive by TMA (3-D maps [lane][T][cols], 128B swizzle;
//     out-of-range steps of the last chunk read as zeros, which contribute
//     nothing: beta = 0 and alpha = 1 there).  Q of the next chunk is loaded as
//     soon as [K;Q] S0 has consumed the current one; K and V of the next chunk
//     are prefetched into L2 and loaded once the state update has read K.
//   - warpgroup 0 runs the state path (S0 conversion, X, R, Y epilogues) and
//     its thread 0 issues TMA and MMAs; warpgroup 1 forms L and Mqk from the
//     Gram MMA and T = (I+L)^{-1} in fp32 (16x16 block substitution), in
//     parallel with the state path, and hands T over through an mbarrier.
//   - every mbarrier wait is bounded and turns into an error status.
//   - y is written per token row; s_final (and the fp32 copy) at the end.
//
// Inputs: fp16 (kind::f16).  Dh = 64, slots in {128, 256, 384, 512}.
#include "chunk_common.cuh"

namespace {

using namespace dgc;
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
    static constexpr uint32_t LT = VR + 8192;               // fp32 [64][68]
    static constexpr uint32_t SC1 = LT + 64 * 68 * 4;       // WG1 per-chunk scalars: aprev, beta/a, 1/a
    static constexpr uint32_t BAR = SC1 + 3 * 64 * 4;       // 12 mbarriers + tmem base
    static constexpr uint32_t BYTES = BAR + 12 * 8 + 16;
    static constexpr uint32_t ACC1 = NB * 64;               // TMEM column bases
    static constexpr uint32_t ACC2 = ACC1 + 64;
    static constexpr uint32_t ACC3 = ACC2 + 64;
    static constexpr uint32_t ACC4 = ACC3 + 64;
    static constexpr uint32_t TMEM_COLS = 512;
};

template <typename TI> constexpr uint32_t idesc_kk() { return tc::make_idesc(128, 64, Io<TI>::kBf16, 0, 0); }
template <typename TI> constexpr uint32_t idesc_km() { return tc::make_idesc(128, 64, Io<TI>::kBf16, 0, 1); }
template <typename TI> constexpr uint32_t idesc_mm() { return tc::make_idesc(128, 64, Io<TI>::kBf16, 1, 1); }
constexpr uint32_t IDESC_KM16 = tc::make_idesc(128, 64, 0, 0, 1);     // T X and Mqk (R beta), fp16
template <int S, typename TI>
__global__ void __launch_bounds__(256, 1)
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
    float* sc1 = reinterpret_cast<float*>(sm + Ly::SC1);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly::BAR);
    uint64_t* bar_kv = bars + 0;     // TMA: K slices + V of a chunk
    uint64_t* bar_q = bars + 1;      // TMA: Q slices of a chunk
    uint64_t* bar_acc1 = bars + 2;
    uint64_t* bar_acc2 = bars + 3;
    uint64_t* bar_acc3 = bars + 4;
    uint64_t* bar_acc4 = bars + 5;
    uint64_t* bar_upd = bars + 6;
    uint64_t* bar_t = bars + 7;      // WG1 -> MMA issuer: T and Mqk tiles of the chunk written
    uint64_t* bar_s0 = bars + 8;     // two S0 buffers
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 12);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q4 = warp & 3;                       // TMEM lane quarter of this warp
    const int lane_bh = blockIdx.x;
    const int h = lane_bh % p.H;
    const int T_ = p.T, NC = p.nchunks;
    const int64_t lane_base = (int64_t)lane_bh * T_;
    const TI* beta = static_cast<const TI*>(p.beta);
    const TI* decay = static_cast<const TI*>(p.decay);

    if (warp == 0) tc::tmem_alloc(tmem_holder, Ly::TMEM_COLS);
    if (tid == 0) {
        for (int i = 0; i < 10; ++i) tc::mbar_init(bars + i, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tmk);
        tc::prefetch_tmap(&tmq);
        tc::prefetch_tmap(&tmv);
    }
    for (int i = tid; i < 8192 / 16; i += 256) reinterpret_cast<uint4*>(tzm + 8192)[i] = make_uint4(0, 0, 0, 0);
    tc::fence_proxy_async();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t tq = tmem + ((uint32_t)(32 * q4) << 16);
    const float alpha_static = p.dynamic_decay ? 1.f : dg::to_f(decay[h]);

    bool failed = false;
    if (warp < 4) {
        // ================= WG0: state path; thread 0 issues TMA and MMAs =================
        {   // initial state -> TMEM (thread = slot row 128 b + 32 warp + lane)
            const TI* s_init = static_cast<const TI*>(p.s_init);
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
                            const float2 f = Io<TI>::unpack2(w4[e]);
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
            tc::tc_fence_before();
        }
        if (tid == 0 && NC > 0) {
            tc::mbar_expect_tx(bar_kv, NSL * 8192 + 8192);
            for (int s = 0; s < NSL; ++s) tc::tma_load_3d(kq + s * SLICE, &tmk, bar_kv, 64 * s, 0, lane_bh);
            tc::tma_load_3d(vr, &tmv, bar_kv, 0, 0, lane_bh);
            tc::mbar_expect_tx(bar_q, NSL * 8192);
            for (int s = 0; s < NSL; ++s) tc::tma_load_3d(kq + s * SLICE + 8192, &tmq, bar_q, 64 * s, 0, lane_bh);
        }
        tc::group_sync(BAR_WG0);
        uint32_t s0_uses[2] = {0u, 0u};
        const int row = 32 * (warp & 1) + lane;        // token row handled in the epilogues
        for (int c = 0; c < NC && !failed; ++c) {
            const int t0 = c * CH;
            const uint32_t par = (uint32_t)(c & 1);
            const ChunkScalars cs = chunk_scalars(beta, decay, p.dynamic_decay, alpha_static, lane_base, t0, T_, lane);
            const float ap_row = pick(cs.ap0, cs.ap1, row);
            const float b_row = pick(cs.b0, cs.b1, row);
            const float ae_row = cs.atot / pick(cs.a0, cs.a1, row);
            // K, V and Q of this chunk in shared memory; previous update done
            bool bad = !tc::mbar_wait(bar_kv, par) || !tc::mbar_wait(bar_q, par);
            if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
            tc::tc_fence_after();
            if (tid == 0) {
                for (int s = 0; s < NSL; ++s)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t base = tc::smem_u32(kq + s * SLICE) + 32 * kk;
                        tc::mma_f16(tmem + Ly::ACC1, tc::make_desc(base, 16, 1024), tc::make_desc(base, 16, 1024),
                                    idesc_kk<TI>(), (s | kk) != 0);
                    }
                tc::mma_commit(bar_acc1);
                if (c + 1 < NC) {          // warm L2 with the next chunk's K and V
                    for (int s = 0; s < NSL; ++s) tc::tma_prefetch_3d(&tmk, 64 * s, t0 + CH, lane_bh);
                    tc::tma_prefetch_3d(&tmv, 0, t0 + CH, lane_bh);
                }
            }
            // [K;Q] S0 over 128-slot blocks; S0 streamed TMEM -> smem in the input type (and scaled by atot in TMEM)
            for (int b = 0; b < NB; ++b) {
                const int buf = b & 1;
                bad = false;
                if (s0_uses[buf] > 0) bad = !tc::mbar_wait(bar_s0 + buf, (s0_uses[buf] - 1) & 1u);
                tc::tc_fence_after();
                float x[64];
                ld_row64(tq + 64 * b, x);
                st_row16<TI>(s0b + buf * 16384, 32 * warp + lane, x);
                if (cs.atot != 1.f) {
                    uint32_t r0[32], r1[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        r0[i] = __float_as_uint(cs.atot * x[i]);
                        r1[i] = __float_as_uint(cs.atot * x[32 + i]);
                    }
                    tc::tmem_st32(tq + 64 * b, r0);
                    tc::tmem_st32(tq + 64 * b + 32, r1);
                    tc::tmem_wait_st();
                }
                tc::fence_proxy_async();
                tc::tc_fence_before();
                if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
                if (tid == 0) {
                    tc::tc_fence_after();
#pragma unroll
                    for (int sl = 0; sl < 2; ++sl)
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint32_t a = tc::smem_u32(kq + (2 * b + sl) * SLICE) + 32 * kk;
                            const uint32_t bb = tc::smem_u32(s0b + buf * 16384) + (sl * 4 + kk) * 2048;
                            tc::mma_f16(tmem + Ly::ACC2, tc::make_desc(a, 16, 1024), tc::make_desc(bb, 16384, 1024),
                                        idesc_km<TI>(), (b | sl | kk) != 0);
                        }
                    tc::mma_commit(bar_s0 + buf);
                    if (b == NB - 1) tc::mma_commit(bar_acc2);
                }
                s0_uses[buf]++;
            }
            if (failed) break;
            // X = V - aprev o (K S0)  (warps 0-1); then the Q tiles are free for the next chunk
            bad = !tc::mbar_wait(bar_acc2, par);
            tc::tc_fence_after();
            if (tid == 0 && c + 1 < NC) {
                tc::mbar_expect_tx(bar_q, NSL * 8192);
                for (int s = 0; s < NSL; ++s)
                    tc::tma_load_3d(kq + s * SLICE + 8192, &tmq, bar_q, 64 * s, t0 + CH, lane_bh);
            }
            if (warp < 2) {
                float d1[64];
                ld_row64(tq + Ly::ACC2, d1);
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    const uint4 v = *reinterpret_cast<const uint4*>(vr + tc::sw128(row, cc));
                    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = Io<TI>::unpack2(w4[e]);
                        d1[8 * cc + 2 * e] = f.x - ap_row * d1[8 * cc + 2 * e];
                        d1[8 * cc + 2 * e + 1] = f.y - ap_row * d1[8 * cc + 2 * e + 1];
                    }
                }
                st_row16(xr, row, d1);
            }
            tc::fence_proxy_async();
            bad = bad || !tc::mbar_wait(bar_t, par);      // T and Mqk of this chunk ready
            if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
            if (tid == 0) {                                 // R = [T; 0] X
                tc::tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    tc::mma_f16(tmem + Ly::ACC3, tc::make_desc(tc::smem_u32(tzm) + 32 * kk, 16, 1024),
                                tc::make_desc(tc::smem_u32(xr) + kk * 2048, 16384, 1024), IDESC_KM16, kk != 0);
                tc::mma_commit(bar_acc3);
            }
            bad = !tc::mbar_wait(bar_acc3, par);
            tc::tc_fence_after();
            if (warp < 2) {
                float r[64];
                ld_row64(tq + Ly::ACC3, r);
                const int t = t0 + row;
                if (p.err_out && t < T_) {
                    float4* dst = reinterpret_cast<float4*>(p.err_out + (lane_base + t) * DH);
#pragma unroll
                    for (int q = 0; q < 16; ++q) dst[q] = make_float4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
                }
                float rb[64];
#pragma unroll
                for (int j = 0; j < 64; ++j) {
                    rb[j] = b_row * r[j];
                    r[j] = ae_row * rb[j];
                }
                st_row16(vr, row, rb);       // R * beta (V is dead), fp16
                st_row16<TI>(xr, row, r);    // R' = a_end * beta * R (X is dead), input type
            }
            tc::fence_proxy_async();
            tc::tc_fence_before();
            if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
            if (tid == 0) {                                 // Mqk (R*beta); S += K^T R'
                tc::tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    tc::mma_f16(tmem + Ly::ACC4, tc::make_desc(tc::smem_u32(tzm + 8192) + 32 * kk, 16, 1024),
                                tc::make_desc(tc::smem_u32(vr) + kk * 2048, 16384, 1024), IDESC_KM16, kk != 0);
                tc::mma_commit(bar_acc4);
                for (int b = 0; b < NB; ++b)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc::mma_f16(tmem + 64 * b,
                                    tc::make_desc(tc::smem_u32(kq + 2 * b * SLICE) + kk * 2048, SLICE, 1024),
                                    tc::make_desc(tc::smem_u32(xr) + kk * 2048, 16384, 1024), idesc_mm<TI>(), 1u);
                tc::mma_commit(bar_upd);
            }
            // Y = aprev o (Q S0) + Mqk R  (warps 2-3)
            bad = !tc::mbar_wait(bar_acc4, par);
            tc::tc_fence_after();
            if (warp >= 2 && !bad) {
                float y[64], m[64];
                ld_row64(tq + Ly::ACC2, y);
                ld_row64(tq + Ly::ACC4, m);
                const int t = t0 + row;
                if (t < T_) {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<TI*>(p.out) + (lane_base + t) * DH);
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) {
                        float o[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) o[e] = fmaf(ap_row, y[8 * cc + e], m[8 * cc + e]);
                        dst[cc] = make_uint4(Io<TI>::pack2(o[0], o[1]), Io<TI>::pack2(o[2], o[3]),
                                             Io<TI>::pack2(o[4], o[5]), Io<TI>::pack2(o[6], o[7]));
                    }
                }
            }
            // the update must finish before the K / V tiles and the state are reused
            bad = bad || !tc::mbar_wait(bar_upd, par);
            tc::tc_fence_after();
            if (tid == 0 && c + 1 < NC && !bad) {
                tc::mbar_expect_tx(bar_kv, NSL * 8192 + 8192);
                for (int s = 0; s < NSL; ++s) tc::tma_load_3d(kq + s * SLICE, &tmk, bar_kv, 64 * s, t0 + CH, lane_bh);
                tc::tma_load_3d(vr, &tmv, bar_kv, 0, t0 + CH, lane_bh);
            }
            if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
        }
        if (!failed) {
            TI* s_fin = static_cast<TI*>(p.s_final);
            for (int b = 0; b < NB; ++b) {
                const int slot = 128 * b + 32 * warp + lane;
                float x[64];
                ld_row64(tq + 64 * b, x);
                const int64_t o = ((int64_t)lane_bh * S + slot) * DH;
                uint4* dst = reinterpret_cast<uint4*>(s_fin + o);
#pragma unroll
                for (int cc = 0; cc < 8; ++cc)
                    dst[cc] = make_uint4(Io<TI>::pack2(x[8 * cc], x[8 * cc + 1]), Io<TI>::pack2(x[8 * cc + 2], x[8 * cc + 3]),
                                         Io<TI>::pack2(x[8 * cc + 4], x[8 * cc + 5]),
                                         Io<TI>::pack2(x[8 * cc + 6], x[8 * cc + 7]));
                if (p.s_final_f) {
                    float4* df = reinterpret_cast<float4*>(p.s_final_f + o);
#pragma unroll
                    for (int q = 0; q < 16; ++q)
                        df[q] = make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
                }
            }
        }
    } else {
        // ================= WG1: per-chunk T = (I + L)^{-1} and Mqk =================
        const int t1 = tid - 128;
        const int row = 32 * (warp & 1) + lane;         // G row (warps 4,5) or QK row (warps 6,7)
        for (int c = 0; c < NC && !failed; ++c) {
            const int t0 = c * CH;
            const uint32_t par = (uint32_t)(c & 1);
            if (warp == 4) {      // chunk scalars for the whole warpgroup
                const ChunkScalars cs = chunk_scalars(beta, decay, p.dynamic_decay, alpha_static, lane_base, t0, T_, lane);
                reinterpret_cast<float2*>(sc1)[lane] = make_float2(cs.ap0, cs.ap1);
                reinterpret_cast<float2*>(sc1 + 64)[lane] = make_float2(cs.b0 / cs.a0, cs.b1 / cs.a1);
                reinterpret_cast<float2*>(sc1 + 128)[lane] = make_float2(1.f / cs.a0, 1.f / cs.a1);
            }
            const bool bad = !tc::mbar_wait(bar_acc1, par);
            if (tc::group_sync_or(BAR_WG1, bad)) { failed = true; break; }
            tc::tc_fence_after();
            const float ap_row = sc1[row];
            const float* wsel = (warp < 6) ? (sc1 + 64) : (sc1 + 128);   // L: beta_j / a_j; Mqk: 1 / a_j
            float g[64];
            ld_row64(tq + Ly::ACC1, g);
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const float4 w4 = reinterpret_cast<const float4*>(wsel)[q];
                const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = 4 * q + e;
                    g[j] = (j < row) ? ap_row * wv[e] * g[j] : 0.f;
                }
            }
            if (warp < 6) {         // L_ij = aprev_i beta_j / a_j (k_i . k_j), j < i
                float4* dst = reinterpret_cast<float4*>(lt + row * LDT);
#pragma unroll
                for (int q = 0; q < 16; ++q) dst[q] = make_float4(g[4 * q], g[4 * q + 1], g[4 * q + 2], g[4 * q + 3]);
            } else {                // Mqk_ij = aprev_i / a_j (q_i . k_j), j < i
                st_row16(tzm + 16384, row, g);
            }
            tc::group_sync(BAR_WG1);
            invert_unit_lower(lt, t1);
            if (t1 < 64) {
                float tr[64];
                const float4* src = reinterpret_cast<const float4*>(lt + t1 * LDT);
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    const float4 v = src[q];
                    tr[4 * q] = v.x; tr[4 * q + 1] = v.y; tr[4 * q + 2] = v.z; tr[4 * q + 3] = v.w;
                }
                st_row16(tzm, t1, tr);
            }
            tc::fence_proxy_async();
            tc::group_sync(BAR_WG1);
            if (t1 == 0) {
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar_t)) : "memory");
            }
        }
    }

    if (failed && (tid == 0 || tid == 128)) dg::flag_status(p.status, DG_DEVCHK_TIMEOUT);
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
template <int S, typename TI>
int launch_chunk(const void* v, const void* beta, const void* wk, const void* wq, const void* decay,
                 int dynamic_decay, const void* s_init, void* out, void* s_final, float* err_out,
                 float* s_final_f, int B, int H, int T, int32_t* status, cudaStream_t stream) {
    const int lanes = B * H;
    CUtensorMap mk, mq, mv;
    const bool bf = Io<TI>::kBf16 != 0;
    if (!make_map(&mk, wk, S, T, lanes, bf) || !make_map(&mq, wq, S, T, lanes, bf) ||
        !make_map(&mv, v, DH, T, lanes, bf))
        return DG_ERR_UNSUPPORTED;
    ChunkParams p{beta, decay, s_init, out, s_final, err_out, s_final_f, status,
                  H, T, (T + CH - 1) / CH, dynamic_decay};
    const size_t smem = Layout<S>::BYTES + 1024;
    auto kern = dense_chunk_kernel<S, TI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    kern<<<lanes, 256, smem, stream>>>(mk, mq, mv, p);
    return dg_host::check_launch();
}

template <typename TI>
int launch_by_slots(int S, const void* v, const void* beta, const void* wk, const void* wq, const void* decay,
                    int dynamic_decay, const void* s_init, void* out, void* s_final, float* err_out, float* s_final_f,
                    int B, int H, int T, int32_t* status, cudaStream_t stream) {
    switch (S) {
    case 128: return launch_chunk<128, TI>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, stream);
    case 256: return launch_chunk<256, TI>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, stream);
    case 384: return launch_chunk<384, TI>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, stream);
    case 512: return launch_chunk<512, TI>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, stream);
    default: return DG_ERR_UNSUPPORTED;
    }
}

}  // namespace

namespace dg_host {

bool dense_chunked_tc_supports(int dtype, int B, int H, int T, int S, int Dh) {
    (void)B; (void)H;
    return (dtype == DG_DTYPE_F16 || dtype == DG_DTYPE_BF16) && Dh == DH && T > 0 &&
           (S == 128 || S == 256 || S == 384 || S == 512);
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
    if (dtype == DG_DTYPE_BF16) return launch_by_slots<__nv_bfloat16>(S, v, beta, wk, wq, decay, dynamic_decay, s_init,
                                                                     out, s_final, err_out, s_final_f, B, H, T, status,
                                                                     stream);
    return launch_by_slots<__half>(S, v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f,
                                   B, H, T, status, stream);
}

}  // namespace dg_host
