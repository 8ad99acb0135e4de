// dense_chunk_t.cu -- chunkwise (WY/UT form) dense delta-rule recurrence on tcgen05,
// with the state held transposed: S^T (Dh rows x slots) on TMEM lanes.
//
// Same recurrence and chunk algebra as dense_chunk_tc.cu (src/cpp/delta_kernel.cu:78-112,
// src/modules/memory.py:325-410); C = 64 steps per chunk, a_i = prod_{l<=i} alpha_l,
// aprev_i = a_{i-1}:
//     L  = strict_lower(aprev_i beta_j / a_j  k_i.k_j),     T = (I + L)^{-1}
//     R  = T (V - aprev o (K S0))
//     Y  = aprev o (Q S0) + strict_lower(aprev_i / a_j  q_i.k_j) (beta o R)
//     S1 = a_{C-1} S0 + K^T diag(a_{C-1} beta_j / a_j) R
//
// Why transposed: with Dh = 64 on the M side of every product, the state is an M = 64
// accumulator (rows on 16 of each 32 TMEM lanes) and its 16-bit copy is the A operand of
// [K;Q] S0 read straight from TMEM (the tcgen05 "A in tensor memory" form).  Nothing of
// the state passes through shared memory; [K;Q] (the chunk's wk / wq tiles) is the only
// shared-memory operand of the big product, and the state copy is a TMEM -> TMEM pass.
//
// Per chunk, all MMAs are M = 64 (D at TMEM lane offset 0 unless stated):
//   P2  D2 = S0^T [K;Q]^T     A: S0^T copy (TMEM)  B: [K;Q] rows (smem, K-major), N = 128
//   P3  R^T = X^T T^T         A: X^T (TMEM)        B: T rows (smem, K-major)
//   P5  S^T += R'^T K         A: R'^T (smem)       B: K (smem, MN-major), D at lane offset 16
//   P4  Yi^T = (bR)^T Mqk^T   A: (beta R)^T (TMEM) B: Mqk columns (smem, MN-major)
//   D5  K Q^T (-> Mqk)        A: K rows (smem)     B: Q rows (smem, K-major), after P2
//   G   D1 = K K^T            next chunk's K slices streamed through a four-slot ring
// Roles (320 threads):
//   - warpgroup 0: the state chain's data work: the 16-bit S0^T copy (which the MMAs
//     read as they go, 128 slots at a time), the X, R and Y epilogues; y leaves through a
//     shared-memory tile (the R'^T tile, once the update has read it) and a TMA store;
//   - warpgroup 1, one chunk ahead: L from the Gram, T = (I + L)^{-1} in fp32 (blocked
//     substitution), T handed over as an fp16 tile; then the current chunk's Mqk tile
//     from K Q^T;
//   - warp 8 (one thread): the chain's TMA loads and MMAs, in chain order;
//   - warp 9 (one thread): the ring's TMA loads and Gram MMAs for the next chunk.
// A tcgen05.mma costs its issuing thread tens of cycles whatever its size, so the two
// MMA sequences are issued by two threads, and no data warp stalls on issue.  The Gram
// and the inverse run beside the chain instead of on it.
//
// Inputs fp16 or bf16 (kind::f16: both operands of one MMA share a type, so the S0 and R'
// copies are in the input type; T, X, beta R and Mqk are formed here and are fp16).
// With bf16 inputs and slots <= 256 the S0 and R' copies are each a bf16 pair hi + lo
// (the lo half is the rounding residue of the hi half) and [K;Q] S0 and the update take
// two MMAs per step, one per half: ~16 significant bits of the state and residual reach
// the products instead of bf16's 8.  (At 384 and 512 slots the lo half of S0 does not
// fit the TMEM the copy may use; there a single bf16 copy is taken.)
// Dh = 64, slots in {128, 256, 384, 512}.  Every wait is bounded (a launch parameter);
// one that gives up flags DG_DEVCHK_TIMEOUT, and the CTA drains the copies and MMAs it
// issued, frees its TMEM and returns.
#include "chunk_common.cuh"

namespace {

using namespace dgc;

constexpr uint32_t SLICE = 16384;        // [K rows 0-63 | Q rows 0-63] of 64 slots, 16-bit, 128B swizzle
constexpr uint32_t LANE16 = 16u << 16;   // TMEM address of the upper 16 lanes of each quarter
constexpr uint32_t DRAIN_LIMIT = 1u << 22;
constexpr int NRING = 4;                 // Gram ring slots (K slices of 8 KB)
constexpr int NTHREADS = 320;            // two warpgroups and the two issuing warps

struct TParams {
    const void* v;
    const void* beta;
    const void* decay;
    const void* s_init;
    void* s_final;
    float* err_out;
    float* s_final_f;
    int32_t* status;
    int H, T, nchunks, dynamic_decay;
    uint32_t wait_limit;   // polls of a bounded wait (each at most ~1 us); 0 gives up at once
};

template <int S, bool HILO>
struct TLayout {
    static constexpr int NSL = S / 64;
    static constexpr uint32_t KQ = 0;                       // this chunk's [K;Q] slices
    static constexpr uint32_t RING = KQ + NSL * SLICE;      // next chunk's K slices
    static constexpr uint32_t TT = RING + NRING * 8192;     // T (rows i, K-major)
    static constexpr uint32_t MQ = TT + 8192;               // Mqk (rows j, MN-major)
    static constexpr uint32_t RT = MQ + 8192;               // R'^T (rows d, K-major); then the y tile (rows t)
    static constexpr uint32_t RL = RT + 8192;               // R'^T lo half (HILO)
    static constexpr uint32_t VT = RL + (HILO ? 8192 : 0);  // V (rows t, TMA)
    static constexpr uint32_t LT = VT + 8192;               // fp32 [64][68] inverse scratch
    static constexpr uint32_t SC0 = LT + 64 * 68 * 4;       // WG0: aprev, beta, a_end / a, 1 / a, atot; two chunks
    static constexpr uint32_t SC1 = SC0 + 2 * 5 * 64 * 4;   // WG1: aprev, beta / a, 1 / a; two chunks
    static constexpr uint32_t BAR = SC1 + 2 * 3 * 64 * 4;   // mbarriers, TMEM base, abort flag
    static constexpr uint32_t BYTES = BAR + 40 * 8 + 16;
    // TMEM columns (lane offset 0 unless stated)
    static constexpr uint32_t A0 = 0;          // S0^T copy, S / 2 columns (lo half after it: HILO), live during P2
    static constexpr uint32_t XA = 0;          // X^T (P3 A), 32 columns, after P2
    static constexpr uint32_t D3 = 32;         // R^T, 64
    static constexpr uint32_t BA = 96;         // (beta R)^T (P4 A), 32
    static constexpr uint32_t D4 = 128;        // Y intra-chunk part, 64
    static constexpr uint32_t D2 = 256;        // [K S0 | Q S0]^T, 128
    static constexpr uint32_t D1 = 384;        // next chunk's K K^T, 64
    static constexpr uint32_t D5 = 448;        // this chunk's K Q^T, 64
    // the state S^T: lane offset 16, columns [0, S)
};
static_assert(TLayout<512, false>::BYTES + 1024 <= 232448, "shared memory");
static_assert(TLayout<256, true>::BYTES + 1024 <= 232448, "shared memory");

enum Bars {
    B_K = 0, B_Q, B_V,                       // TMA: this chunk's K, Q, V
    B_P2, B_D5, B_P3, B_P4, B_P5,            // MMA commits
    B_CV0, B_CV1, B_CV2, B_CV3,              // WG0: S0^T copy of slot group g written (4 warps)
    B_XD, B_RD,                              // WG0: X^T ready / R'^T and (beta R)^T ready (4 warps)
    B_T, B_MD, B_LX,                         // WG1: T tile / Mqk tile written, Gram read out (1 arrival)
    B_RF0, B_RF1, B_RF2, B_RF3,              // ring slot loaded
    B_RE0, B_RE1, B_RE2, B_RE3,              // ring slot consumed by the Gram MMAs
    B_G,                                     // Gram complete
    B_DR0, B_DR1,                            // drain commits of the two issuing threads
    NBARS
};
static_assert(NBARS <= 40, "barrier area");

template <typename TI> constexpr uint32_t idesc_in(int N, int b_mn) { return tc::make_idesc(64, N, Io<TI>::kBf16, 0, b_mn); }
constexpr uint32_t IDESC_P3 = tc::make_idesc(64, 64, 0, 0, 0);
constexpr uint32_t IDESC_P4 = tc::make_idesc(64, 64, 0, 0, 1);

__device__ __forceinline__ uint32_t pack_h2(float a, float b) { return Io<__half>::pack2(a, b); }

// bounded wait of a data warp; also gives up when another role has given up
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, uint32_t limit, volatile int* abort_flag) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (tc::mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    return false;
}
// one warp's hand-over: its TMEM writes and shared-memory writes are complete and
// ordered before the issuing thread's MMAs / async copies that read them
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
    tc::fence_proxy_async();
    tc::tc_fence_before();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(bar);
}

template <int S, typename TI>
__global__ void __launch_bounds__(NTHREADS, 1)
    dense_chunk_t_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmq,
                         const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmy,
                         TParams p) {
    constexpr bool HILO = Io<TI>::kBf16 != 0 && S <= 256;
    using Ly = TLayout<S, HILO>;
    constexpr int NSL = Ly::NSL;
    constexpr int NG = NSL / 2;              // S0^T copy groups of 128 slots
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kq = sm + Ly::KQ;
    uint8_t* ring = sm + Ly::RING;
    uint8_t* tt = sm + Ly::TT;
    uint8_t* mqt = sm + Ly::MQ;
    uint8_t* rt = sm + Ly::RT;
    uint8_t* rl = sm + Ly::RL;
    uint8_t* vt = sm + Ly::VT;
    uint8_t* yt = rt;
    float* lt = reinterpret_cast<float*>(sm + Ly::LT);
    float* sc0_base = reinterpret_cast<float*>(sm + Ly::SC0);
    float* sc1 = reinterpret_cast<float*>(sm + Ly::SC1);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly::BAR);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 40);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 40) + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q4 = warp & 3;                  // TMEM lane quarter of this warp
    const int r16 = lane & 15, half = lane >> 4;
    const int lane_bh = blockIdx.x;
    const int h = lane_bh % p.H;
    const int T_ = p.T, NC = p.nchunks;
    const int64_t lane_base = (int64_t)lane_bh * T_;
    const TI* beta = static_cast<const TI*>(p.beta);
    const TI* decay = static_cast<const TI*>(p.decay);
    const uint32_t lim = p.wait_limit;

    if (warp == 0) tc::tmem_alloc(tmem_holder, 512);
    if (tid == 0) {
        for (int i = 0; i < NBARS; ++i) {
            const bool per_warp = (i >= B_CV0 && i <= B_CV3) || i == B_XD || i == B_RD;
            tc::mbar_init(bars + i, per_warp ? 4 : 1);
        }
        *abort_flag = 0;
        tc::fence_barrier_init();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t tq0 = tmem + ((uint32_t)(32 * q4) << 16);      // this warp's rows, lane offset 0
    const uint32_t tq1 = tq0 + LANE16;                              // the state's rows
    const float alpha_static = p.dynamic_decay ? 1.f : dg::to_f(decay[h]);
    const int row = 16 * q4 + r16;           // Dh row (WG0) or chunk row (WG1) of this thread
    const int cb = 32 * half;                // first chunk step / slot of this thread's half
    bool failed = false;

    if (warp < 4) {
        // ============================ WG0: the state chain's data work ============================
        {   // initial state -> S^T (lane offset 16): thread (row d, half) holds slots [64g + 32 half, +32)
            const TI* s_init = static_cast<const TI*>(p.s_init);
            for (int g = 0; g < NSL; ++g) {
                uint32_t r[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float v = 0.f;
                    if (s_init) v = dg::to_f(s_init[((int64_t)lane_bh * S + 64 * g + cb + i) * DH + row]);
                    r[i] = __float_as_uint(v);
                }
                tc::tmem_st16x2_32(tq1 + 64 * g, r);
            }
            tc::tmem_wait_st();
        }
        // chunk scalars (aprev_t, beta_t, a_end / a_t, atot), double-buffered by chunk parity: warp 0
        // forms those of chunk c + 1 while chunk c waits for [K;Q] S0, so their loads are off the chain
        auto chunk_gates = [&](int cc) {
            float* dst = sc0_base + (cc & 1) * 320;
            const ChunkScalars cs = chunk_scalars(beta, decay, p.dynamic_decay, alpha_static, lane_base, cc * CH, T_, lane);
            reinterpret_cast<float2*>(dst)[lane] = make_float2(cs.ap0, cs.ap1);
            reinterpret_cast<float2*>(dst + 64)[lane] = make_float2(cs.b0, cs.b1);
            reinterpret_cast<float2*>(dst + 128)[lane] = make_float2(cs.atot / cs.a0, cs.atot / cs.a1);
            if (lane == 0) dst[256] = cs.atot;
        };
        if (warp == 0 && NC > 0) chunk_gates(0);
        // chunk c's y (this thread's 32 steps of its row, packed in pairs) is formed once
        // P4 and P5 are done and written to the y tile while chunk c + 1 waits for its
        // [K;Q] S0 product, so the tile stores and the TMA store are off the chain
        uint32_t ypk[16];
        int ypend = -1;                          // first step of the chunk whose y awaits its store
        auto y_store = [&]() {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int t = cb + i;
                const uint32_t pr = ypk[i >> 1];
                const uint16_t hv = (i & 1) ? (uint16_t)(pr >> 16) : (uint16_t)(pr & 0xffffu);
                *reinterpret_cast<uint16_t*>(yt + t * 128 + ((((row >> 3) ^ (t & 7))) << 4) + (row & 7) * 2) = hv;
            }
            tc::fence_proxy_async();
            tc::group_sync(BAR_WG0);
            if (tid == 0) {
                tc::tma_store_3d(&tmy, yt, 0, ypend, lane_bh);
                tc::bulk_commit_group();
            }
            ypend = -1;
        };
        for (int c = 0; c < NC && !failed; ++c) {
            const int t0 = c * CH;
            const uint32_t par = (uint32_t)(c & 1);
            float* sc0 = sc0_base + (c & 1) * 320;   // this chunk's scalars; the previous chunk may still read the other half
            // the previous chunk's update is complete: the state may be read
            bool bad = (c > 0 && !wait_bar(bars + B_P5, par ^ 1u, lim, abort_flag));
            if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
            tc::tc_fence_after();
            const float atot = sc0[256];
            // S0^T (fp32, lane offset 16) -> 16-bit copy (lane offset 0), scaled by atot in place;
            // each 128-slot group is handed to the issuing thread as soon as this warp has written it
            for (int g2 = 0; g2 < NG; ++g2) {
                uint32_t r0[32], r1[32];
                tc::tmem_ld16x2_32(tq1 + 128 * g2, r0);
                tc::tmem_ld16x2_32(tq1 + 128 * g2 + 64, r1);
                tc::tmem_wait_ld();
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) pk[i] = Io<TI>::pack2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
                tc::tmem_st16x2_16(tq0 + Ly::A0 + 64 * g2, pk);
#pragma unroll
                for (int i = 0; i < 16; ++i) pk[i] = Io<TI>::pack2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
                tc::tmem_st16x2_16(tq0 + Ly::A0 + 64 * g2 + 32, pk);
                if constexpr (HILO) {
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        pk[i] = Io<TI>::pack2_lo(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
                    tc::tmem_st16x2_16(tq0 + Ly::A0 + S / 2 + 64 * g2, pk);
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        pk[i] = Io<TI>::pack2_lo(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
                    tc::tmem_st16x2_16(tq0 + Ly::A0 + S / 2 + 64 * g2 + 32, pk);
                }
                if (atot != 1.f) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        r0[i] = __float_as_uint(atot * __uint_as_float(r0[i]));
                        r1[i] = __float_as_uint(atot * __uint_as_float(r1[i]));
                    }
                    tc::tmem_st16x2_32(tq1 + 128 * g2, r0);
                    tc::tmem_st16x2_32(tq1 + 128 * g2 + 64, r1);
                }
                tc::tmem_wait_st();
                warp_arrive(bars + B_CV0 + g2, lane);
            }
            if (warp == 0 && c + 1 < NC) chunk_gates(c + 1);
            // the previous chunk's y tile (its update has read the R'^T tile it shares)
            if (ypend >= 0) y_store();
            // X^T = V^T - (K S0)^T diag(aprev) -> 16-bit P3 operand in TMEM.  This thread's V
            // values and aprev are read while [K;Q] S0 is still in the tensor pipe
            bad = !wait_bar(bars + B_V, par, lim, abort_flag);
            if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
            float xv[32], xa[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int t = cb + i;
                xv[i] = dg::to_f(*reinterpret_cast<const TI*>(vt + t * 128 + ((((row >> 3) ^ (t & 7))) << 4) + (row & 7) * 2));
                xa[i] = sc0[t];
            }
            bad = !wait_bar(bars + B_P2, par, lim, abort_flag);
            if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
            tc::tc_fence_after();
            {
                uint32_t r[32], pk[16];
                tc::tmem_ld16x2_32(tq0 + Ly::D2, r);
                tc::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    pk[i] = pack_h2(xv[2 * i] - xa[2 * i] * __uint_as_float(r[2 * i]),
                                    xv[2 * i + 1] - xa[2 * i + 1] * __uint_as_float(r[2 * i + 1]));
                tc::tmem_st16x2_16(tq0 + Ly::XA, pk);
                tc::tmem_wait_st();
            }
            warp_arrive(bars + B_XD, lane);
            // residuals: err_out, R'^T (update operand, smem), (beta R)^T (P4 operand, TMEM); the
            // chunk scalars they take are read while R^T = X^T T^T is in the tensor pipe
            float rg[32], rb[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                rg[i] = sc0[128 + cb + i] * sc0[64 + cb + i];
                rb[i] = sc0[64 + cb + i];
            }
            bad = !wait_bar(bars + B_P3, par, lim, abort_flag);
            if (tid == 0) tc::bulk_wait_read0();      // the previous chunk's y store has read the shared tile
            if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
            tc::tc_fence_after();
            {
                uint32_t r[32], pk[16];
                tc::tmem_ld16x2_32(tq0 + Ly::D3, r);
                tc::tmem_wait_ld();
                float rr[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) rr[i] = __uint_as_float(r[i]);
                if (p.err_out) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int t = t0 + cb + i;
                        if (t < T_) p.err_out[(lane_base + t) * DH + row] = rr[i];
                    }
                }
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    float rp[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) rp[e] = rg[8 * cc + e] * rr[8 * cc + e];
                    *reinterpret_cast<uint4*>(rt + tc::sw128(row, 4 * half + cc)) =
                        make_uint4(Io<TI>::pack2(rp[0], rp[1]), Io<TI>::pack2(rp[2], rp[3]),
                                   Io<TI>::pack2(rp[4], rp[5]), Io<TI>::pack2(rp[6], rp[7]));
                    if constexpr (HILO)
                        *reinterpret_cast<uint4*>(rl + tc::sw128(row, 4 * half + cc)) =
                            make_uint4(Io<TI>::pack2_lo(rp[0], rp[1]), Io<TI>::pack2_lo(rp[2], rp[3]),
                                       Io<TI>::pack2_lo(rp[4], rp[5]), Io<TI>::pack2_lo(rp[6], rp[7]));
                }
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    pk[i] = pack_h2(rb[2 * i] * rr[2 * i], rb[2 * i + 1] * rr[2 * i + 1]);
                tc::tmem_st16x2_16(tq0 + Ly::BA, pk);
                tc::tmem_wait_st();
            }
            warp_arrive(bars + B_RD, lane);
            // Y^T = (Q S0)^T diag(aprev) + Yi^T -> y tile -> TMA store
            bad = !wait_bar(bars + B_P4, par, lim, abort_flag) || !wait_bar(bars + B_P5, par, lim, abort_flag);
            if (tc::group_sync_or(BAR_WG0, bad)) { failed = true; break; }
            tc::tc_fence_after();
            {
                uint32_t yi[32], qs[32];
                tc::tmem_ld16x2_32(tq0 + Ly::D4, yi);
                tc::tmem_ld16x2_32(tq0 + Ly::D2 + 64, qs);
                tc::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int t = cb + 2 * i;
                    ypk[i] = Io<TI>::pack2(fmaf(sc0[t], __uint_as_float(qs[2 * i]), __uint_as_float(yi[2 * i])),
                                           fmaf(sc0[t + 1], __uint_as_float(qs[2 * i + 1]), __uint_as_float(yi[2 * i + 1])));
                }
            }
            ypend = t0;
        }
        if (!failed && ypend >= 0) y_store();    // the last chunk's y
        if (tid == 0) tc::bulk_wait0();
        // final state: S^T -> s_final / s_final_f through a shared-memory transpose (the K/Q tiles are free)
        if (!failed && NC > 0) {
            bool bad = !wait_bar(bars + B_P5, (uint32_t)((NC - 1) & 1), lim, abort_flag);
            if (tc::group_sync_or(BAR_WG0, bad)) failed = true;
        }
        if (!failed) {
            tc::tc_fence_after();
            float* stg = reinterpret_cast<float*>(kq);       // [64 slots][65]
            TI* s_fin = static_cast<TI*>(p.s_final);
            for (int g = 0; g < NSL; ++g) {
                uint32_t r[32];
                tc::tmem_ld16x2_32(tq1 + 64 * g, r);
                tc::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) stg[(cb + i) * 65 + row] = __uint_as_float(r[i]);
                tc::group_sync(BAR_WG0);
                const int sr = tid >> 1, d0 = 32 * (tid & 1);
                const int64_t o = ((int64_t)lane_bh * S + 64 * g + sr) * DH + d0;
                float x[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) x[i] = stg[sr * 65 + d0 + i];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                    reinterpret_cast<uint4*>(s_fin + o)[cc] =
                        make_uint4(Io<TI>::pack2(x[8 * cc], x[8 * cc + 1]), Io<TI>::pack2(x[8 * cc + 2], x[8 * cc + 3]),
                                   Io<TI>::pack2(x[8 * cc + 4], x[8 * cc + 5]), Io<TI>::pack2(x[8 * cc + 6], x[8 * cc + 7]));
                if (p.s_final_f) {
#pragma unroll
                    for (int qq = 0; qq < 8; ++qq)
                        reinterpret_cast<float4*>(p.s_final_f + o)[qq] =
                            make_float4(x[4 * qq], x[4 * qq + 1], x[4 * qq + 2], x[4 * qq + 3]);
                }
                tc::group_sync(BAR_WG0);
            }
        }
    } else if (warp < 8) {
        // ================= WG1: T = (I + L)^{-1} and Mqk, one chunk ahead =================
        const int t1 = tid - 128;
        // Mqk of chunk m from its K Q^T: Mqk[i][j] = aprev_i / a_j  q_i . k_j, i > j; this thread
        // holds column j = its row of K Q^T, one row of the tile (MN-major for P4)
        auto mqk_tile = [&](int m) -> bool {
            const uint32_t pm = (uint32_t)(m & 1);
            bool bad2 = !wait_bar(bars + B_D5, pm, lim, abort_flag) ||
                        (m > 0 && !wait_bar(bars + B_P4, pm ^ 1u, lim, abort_flag));
            if (tc::group_sync_or(BAR_WG1, bad2)) return false;
            tc::tc_fence_after();
            const float* s1 = sc1 + (m & 1) * 192;
            uint32_t g[32];
            tc::tmem_ld16x2_32(tq0 + Ly::D5, g);
            tc::tmem_wait_ld();
            const float ia_j = s1[128 + row];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int i0 = cb + 8 * cc + 2 * e;
                    const float m0 = (i0 > row) ? s1[i0] * ia_j * __uint_as_float(g[8 * cc + 2 * e]) : 0.f;
                    const float m1 = (i0 + 1 > row) ? s1[i0 + 1] * ia_j * __uint_as_float(g[8 * cc + 2 * e + 1]) : 0.f;
                    w[e] = pack_h2(m0, m1);
                }
                *reinterpret_cast<uint4*>(mqt + tc::sw128(row, 4 * half + cc)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            tc::fence_proxy_async();
            tc::tc_fence_before();
            tc::group_sync(BAR_WG1);
            if (t1 == 0) tc::mbar_arrive(bars + B_MD);
            return true;
        };
        for (int n = 0; n < NC && !failed; ++n) {
            const int t0 = n * CH;
            const uint32_t par = (uint32_t)(n & 1);
            float* sc1n = sc1 + (n & 1) * 192;       // chunk n's scalars; chunk n - 1's stay for its Mqk
            if (warp == 4) {
                const ChunkScalars cs = chunk_scalars(beta, decay, p.dynamic_decay, alpha_static, lane_base, t0, T_, lane);
                reinterpret_cast<float2*>(sc1n)[lane] = make_float2(cs.ap0, cs.ap1);
                reinterpret_cast<float2*>(sc1n + 64)[lane] = make_float2(cs.b0 / cs.a0, cs.b1 / cs.a1);
                reinterpret_cast<float2*>(sc1n + 128)[lane] = make_float2(1.f / cs.a0, 1.f / cs.a1);
            }
            bool bad = !wait_bar(bars + B_G, par, lim, abort_flag);
            if (tc::group_sync_or(BAR_WG1, bad)) { failed = true; break; }
            tc::tc_fence_after();
            {   // L_ij = aprev_i beta_j / a_j  k_i . k_j, j < i (row i = this thread's row)
                uint32_t g[32];
                tc::tmem_ld16x2_32(tq0 + Ly::D1, g);
                tc::tmem_wait_ld();
                const float ap_i = sc1n[row];
                float4* dst = reinterpret_cast<float4*>(lt + row * LDT + cb);
#pragma unroll
                for (int qq = 0; qq < 8; ++qq) {
                    float l[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = cb + 4 * qq + e;
                        l[e] = (j < row) ? ap_i * sc1n[64 + j] * __uint_as_float(g[4 * qq + e]) : 0.f;
                    }
                    dst[qq] = make_float4(l[0], l[1], l[2], l[3]);
                }
            }
            tc::tc_fence_before();
            tc::group_sync(BAR_WG1);
            if (t1 == 0) tc::mbar_arrive(bars + B_LX);      // the Gram accumulator may take the next chunk
            invert_unit_lower(lt, t1);
            // T of this chunk replaces the previous one once P3 of the previous chunk is done
            bad = (n > 0) && !wait_bar(bars + B_P3, par ^ 1u, lim, abort_flag);
            if (tc::group_sync_or(BAR_WG1, bad)) { failed = true; break; }
            if (t1 < 64) {
                float tr[64];
                const float4* src = reinterpret_cast<const float4*>(lt + t1 * LDT);
#pragma unroll
                for (int qq = 0; qq < 16; ++qq) {
                    const float4 v = src[qq];
                    tr[4 * qq] = v.x; tr[4 * qq + 1] = v.y; tr[4 * qq + 2] = v.z; tr[4 * qq + 3] = v.w;
                }
                st_row16(tt, t1, tr);
            }
            tc::fence_proxy_async();
            tc::group_sync(BAR_WG1);
            if (t1 == 0) tc::mbar_arrive(bars + B_T);
            // the previous chunk's Mqk (its K Q^T is done by now)
            if (n > 0 && !mqk_tile(n - 1)) { failed = true; break; }
        }
        if (!failed && NC > 0 && !mqk_tile(NC - 1)) failed = true;
    } else if (warp == 8 && lane == 0) {
        // ================= warp 8: the chain's loads and MMAs, in chain order =================
        tc::prefetch_tmap(&tmk);
        tc::prefetch_tmap(&tmq);
        tc::prefetch_tmap(&tmv);
        tc::prefetch_tmap(&tmy);
        bool pend_k = false, pend_q = false, pend_v = false;
        uint32_t par_k = 0, par_q = 0, par_v = 0;
        if (NC > 0) {
            tc::mbar_expect_tx(bars + B_K, NSL * 8192);
            for (int s = 0; s < NSL; ++s) tc::tma_load_3d(kq + s * SLICE, &tmk, bars + B_K, 64 * s, 0, lane_bh);
            tc::mbar_expect_tx(bars + B_Q, NSL * 8192);
            for (int s = 0; s < NSL; ++s) tc::tma_load_3d(kq + s * SLICE + 8192, &tmq, bars + B_Q, 64 * s, 0, lane_bh);
            tc::mbar_expect_tx(bars + B_V, 8192);
            tc::tma_load_3d(vt, &tmv, bars + B_V, 0, 0, lane_bh);
            pend_k = pend_q = pend_v = true;
        }
        bool ok = true;
        for (int c = 0; c < NC && ok; ++c) {
            const uint32_t par = (uint32_t)(c & 1);
            const int t0 = c * CH;
            // this chunk's K, Q landed
            ok = wait_bar(bars + B_K, par, lim, abort_flag) && wait_bar(bars + B_Q, par, lim, abort_flag);
            if (!ok) break;
            pend_k = pend_q = false;
            // [K;Q] S0, one 128-slot group at a time as the S0^T copy is written
            for (int grp = 0; grp < NG && ok; ++grp) {
                ok = wait_bar(bars + B_CV0 + grp, par, lim, abort_flag);
                if (!ok) break;
                tc::tc_fence_after();
#pragma unroll
                for (int gg = 0; gg < 2; ++gg)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const int g = 2 * grp + gg;
                        const uint64_t bd = tc::make_desc(tc::smem_u32(kq + g * SLICE) + 32 * kk, 16, 1024);
                        tc::mma_f16_ts(tmem + Ly::D2, tmem + Ly::A0 + 32 * g + 8 * kk, bd, idesc_in<TI>(128, 0),
                                       (g | kk) != 0);
                        if constexpr (HILO)
                            tc::mma_f16_ts(tmem + Ly::D2, tmem + Ly::A0 + S / 2 + 32 * g + 8 * kk, bd,
                                           idesc_in<TI>(128, 0), 1u);
                    }
            }
            if (!ok) break;
            tc::mma_commit(bars + B_P2);
            // X^T written and V read: next V; T ready: R^T = X^T T^T
            ok = wait_bar(bars + B_XD, par, lim, abort_flag);
            if (!ok) break;
            pend_v = false;
            if (c + 1 < NC) {
                tc::mbar_expect_tx(bars + B_V, 8192);
                tc::tma_load_3d(vt, &tmv, bars + B_V, 0, t0 + CH, lane_bh);
                pend_v = true; par_v = par ^ 1u;
            }
            ok = wait_bar(bars + B_T, par, lim, abort_flag);
            if (!ok) break;
            tc::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                tc::mma_f16_ts(tmem + Ly::D3, tmem + Ly::XA + 8 * kk,
                               tc::make_desc(tc::smem_u32(tt) + 32 * kk, 16, 1024), IDESC_P3, kk != 0);
            tc::mma_commit(bars + B_P3);
            // K Q^T for this chunk's Mqk (warpgroup 1 turns it into the tile), after P3 in the
            // tensor pipe so that it runs under the R epilogue
#pragma unroll 1
            for (int g = 0; g < NSL; ++g)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    tc::mma_f16(tmem + Ly::D5, tc::make_desc(tc::smem_u32(kq + g * SLICE) + 32 * kk, 16, 1024),
                                tc::make_desc(tc::smem_u32(kq + g * SLICE + 8192) + 32 * kk, 16, 1024),
                                idesc_in<TI>(64, 0), (g | kk) != 0);
            tc::mma_commit(bars + B_D5);
            // R'^T and (beta R)^T ready: the state update, then the Y intra-chunk part once Mqk is in
            ok = wait_bar(bars + B_RD, par, lim, abort_flag);
            if (!ok) break;
            tc::tc_fence_after();
#pragma unroll
            for (int nt = 0; nt < (S + 255) / 256; ++nt) {
                const int n = (S - 256 * nt) >= 256 ? 256 : S - 256 * nt;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t bd = tc::make_desc(tc::smem_u32(kq + 4 * nt * SLICE) + kk * 2048, SLICE, 1024);
                    tc::mma_f16(tmem + LANE16 + 256 * nt, tc::make_desc(tc::smem_u32(rt) + 32 * kk, 16, 1024), bd,
                                idesc_in<TI>(n, 1), 1u);
                    if constexpr (HILO)
                        tc::mma_f16(tmem + LANE16 + 256 * nt, tc::make_desc(tc::smem_u32(rl) + 32 * kk, 16, 1024), bd,
                                    idesc_in<TI>(n, 1), 1u);
                }
            }
            tc::mma_commit(bars + B_P5);
            ok = wait_bar(bars + B_MD, par, lim, abort_flag);
            if (!ok) break;
            tc::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                tc::mma_f16_ts(tmem + Ly::D4, tmem + Ly::BA + 8 * kk,
                               tc::make_desc(tc::smem_u32(mqt) + kk * 2048, 8192, 1024), IDESC_P4, kk != 0);
            tc::mma_commit(bars + B_P4);
            // P2 and K Q^T have read Q, the update has read K: next Q and K
            ok = wait_bar(bars + B_D5, par, lim, abort_flag);
            if (!ok) break;
            if (c + 1 < NC) {
                tc::mbar_expect_tx(bars + B_Q, NSL * 8192);
                for (int s = 0; s < NSL; ++s)
                    tc::tma_load_3d(kq + s * SLICE + 8192, &tmq, bars + B_Q, 64 * s, t0 + CH, lane_bh);
                pend_q = true; par_q = par ^ 1u;
            }
            ok = wait_bar(bars + B_P5, par, lim, abort_flag);
            if (!ok) break;
            if (c + 1 < NC) {
                tc::mbar_expect_tx(bars + B_K, NSL * 8192);
                for (int s = 0; s < NSL; ++s) tc::tma_load_3d(kq + s * SLICE, &tmk, bars + B_K, 64 * s, t0 + CH, lane_bh);
                pend_k = true; par_k = par ^ 1u;
            }
        }
        if (!ok) *abort_flag = 1;
        // drain: loads in flight complete, then every MMA this thread issued
        if (pend_k) tc::mbar_wait(bars + B_K, par_k, DRAIN_LIMIT);
        if (pend_q) tc::mbar_wait(bars + B_Q, par_q, DRAIN_LIMIT);
        if (pend_v) tc::mbar_wait(bars + B_V, par_v, DRAIN_LIMIT);
        tc::mma_commit(bars + B_DR0);
        tc::mbar_wait(bars + B_DR0, 0, DRAIN_LIMIT);
    } else if (warp == 9 && lane == 0) {
        // ================= warp 9: the Gram ring, one chunk ahead of the chain =================
        uint32_t pend = 0, rpar[NRING] = {0u, 0u, 0u, 0u};
        bool ok = true;
        uint32_t u_load = 0;                  // ring slices loaded so far (over all chunks)
        auto load = [&](int m, int s) -> bool {
            const uint32_t slot = u_load % NRING, use = u_load / NRING;
            if (use > 0 && !wait_bar(bars + B_RE0 + slot, (use - 1) & 1u, lim, abort_flag)) return false;
            uint8_t* dst = ring + slot * 8192;
            tc::mbar_expect_tx(bars + B_RF0 + slot, 8192);
            tc::tma_load_3d(dst, &tmk, bars + B_RF0 + slot, 64 * s, m * CH, lane_bh);
            pend |= 1u << slot;
            rpar[slot] = use & 1u;
            ++u_load;
            return true;
        };
        const int total = NC * NSL;
        for (int j = 0; j < NRING && j < total && ok; ++j) ok = load(j / NSL, j % NSL);
        // (the loop below refills slot (j - 1) % NRING after issuing slice j; the slice
        //  j - 1 + NRING of the last slot is loaded after the last MMAs)
        for (int j = 0; j < total && ok; ++j) {
            const int m = j / NSL, s = j % NSL;
            const uint32_t slot = (uint32_t)j % NRING, use = (uint32_t)j / NRING;
            if (s == 0 && m + 1 < NC) {        // warm L2 with the next chunk's K, Q and V
                for (int ss = 0; ss < NSL; ++ss) {
                    tc::tma_prefetch_3d(&tmk, 64 * ss, (m + 1) * CH, lane_bh);
                    tc::tma_prefetch_3d(&tmq, 64 * ss, (m + 1) * CH, lane_bh);
                }
                tc::tma_prefetch_3d(&tmv, 0, (m + 1) * CH, lane_bh);
            }
            ok = wait_bar(bars + B_RF0 + slot, use & 1u, lim, abort_flag);
            if (ok && s == 0 && m > 0) ok = wait_bar(bars + B_LX, (uint32_t)((m - 1) & 1), lim, abort_flag);
            if (!ok) break;
            pend &= ~(1u << slot);
            tc::tc_fence_after();
            const uint32_t base = tc::smem_u32(ring + slot * 8192);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                tc::mma_f16(tmem + Ly::D1, tc::make_desc(base + 32 * kk, 16, 1024),
                            tc::make_desc(base + 32 * kk, 16, 1024), idesc_in<TI>(64, 0), (s | kk) != 0);
            tc::mma_commit(bars + B_RE0 + slot);
            if (s == NSL - 1) tc::mma_commit(bars + B_G);
            // refill the slot of the previous slice (its MMAs were issued one slice ago)
            if (j >= 1 && j - 1 + NRING < total) ok = load((j - 1 + NRING) / NSL, (j - 1 + NRING) % NSL);
        }
        if (!ok) *abort_flag = 1;
        for (int sl = 0; sl < NRING; ++sl)
            if (pend & (1u << sl)) tc::mbar_wait(bars + B_RF0 + sl, rpar[sl], DRAIN_LIMIT);
        tc::mma_commit(bars + B_DR1);
        tc::mbar_wait(bars + B_DR1, 0, DRAIN_LIMIT);
    }
    if (warp >= 8) __syncwarp();
    if (failed) *abort_flag = 1;
    tc::tc_fence_before();
    __syncthreads();
    if (tid == 0 && *abort_flag) dg::flag_status(p.status, DG_DEVCHK_TIMEOUT);
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int S, typename TI>
int launch_t(const void* v, const void* beta, const void* wk, const void* wq, const void* decay, int dynamic_decay,
             const void* s_init, void* out, void* s_final, float* err_out, float* s_final_f, int B, int H, int T,
             int32_t* status, uint32_t wait_limit, cudaStream_t stream) {
    const int lanes = B * H;
    CUtensorMap mk, mq, mv, my;
    const bool bf = Io<TI>::kBf16 != 0;
    if (!make_map(&mk, wk, S, T, lanes, bf) || !make_map(&mq, wq, S, T, lanes, bf) ||
        !make_map(&mv, v, DH, T, lanes, bf) || !make_map(&my, out, DH, T, lanes, bf))
        return DG_ERR_UNSUPPORTED;
    TParams prm{v, beta, decay, s_init, s_final, err_out, s_final_f, status, H, T, (T + CH - 1) / CH, dynamic_decay,
                wait_limit};
    const size_t smem = TLayout<S, Io<TI>::kBf16 != 0 && S <= 256>::BYTES + 1024;
    auto kern = dense_chunk_t_kernel<S, TI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    kern<<<lanes, NTHREADS, smem, stream>>>(mk, mq, mv, my, prm);
    return dg_host::check_launch();
}

template <typename TI>
int launch_t_slots(int S, const void* v, const void* beta, const void* wk, const void* wq, const void* decay,
                   int dynamic_decay, const void* s_init, void* out, void* s_final, float* err_out, float* s_final_f,
                   int B, int H, int T, int32_t* status, uint32_t wl, cudaStream_t stream) {
    switch (S) {
    case 128: return launch_t<128, TI>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, wl, stream);
    case 256: return launch_t<256, TI>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, wl, stream);
    case 384: return launch_t<384, TI>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, wl, stream);
    case 512: return launch_t<512, TI>(v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f, B, H, T, status, wl, stream);
    default: return DG_ERR_UNSUPPORTED;
    }
}

}  // namespace

namespace dg_host {

uint32_t wait_limit();

int dense_forward_chunked_t(int dtype, int B, int H, int T, int S, int Dh, const void* v, const void* beta,
                            const void* wk, const void* wq, const void* decay, int dynamic_decay, const void* s_init,
                            void* out, void* s_final, float* err_out, float* s_final_f, int32_t* status,
                            cudaStream_t stream) {
    if (!((dtype == DG_DTYPE_F16 || dtype == DG_DTYPE_BF16) && Dh == DH && T > 0 &&
          (S == 128 || S == 256 || S == 384 || S == 512)))
        return DG_ERR_UNSUPPORTED;
    const uintptr_t mis = (uintptr_t)v | (uintptr_t)wk | (uintptr_t)wq | (uintptr_t)s_final | (uintptr_t)out |
                          (uintptr_t)(s_final_f ? (void*)s_final_f : s_final);
    if (mis & 15) return DG_ERR_MISALIGNED;
    const uint32_t wl = wait_limit();
    if (dtype == DG_DTYPE_BF16)
        return launch_t_slots<__nv_bfloat16>(S, v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out,
                                             s_final_f, B, H, T, status, wl, stream);
    return launch_t_slots<__half>(S, v, beta, wk, wq, decay, dynamic_decay, s_init, out, s_final, err_out, s_final_f,
                                  B, H, T, status, wl, stream);
}

}  // namespace dg_host
