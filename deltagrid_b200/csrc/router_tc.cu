// router_tc.cu -- two-axis product-key router with tensor-core scores (16-bit keys).
//
// Same result as router.cu (DeltaGridLayer._route_sparse_pkm, src/modules/memory.py:240-289,
// and the q_scale multiply of memory.py:453-455), for Dh = 64, top-k in {4, 8}:
//   1. scores for all router rows as a tcgen05 GEMM: 128 tokens (one per TMEM lane) x
//      up to 256 router rows per MMA block, K = 64; the two axes run side by side in
//      two warpgroups, each with its own TMEM columns and router buffer.  The fp32
//      router is split into two 16-bit parts (hi + lo), so the product is fp32-accurate
//      up to the tensor core's accumulation; blocks stream through shared memory by TMA;
//   2. each thread keeps its token's k + 4 (2k above 256 rows) best approximate scores
//      as 32-bit keys (the score's order-preserving bits with the row in the low bits,
//      so an insert is one unsigned max/min pair per entry, all entries at once): the
//      first 32 scores by a sorting network, then 32 TMEM columns at a time, skipping
//      any 32 whose maximum is below the filter -- the last listed score, or if higher
//      the (k+1)-th listed score less a margin of eight narrow-gap widths (step 3), so
//      the list holds every score above that filter's final value;
//   3. exactness: with |approx - exact| <= delta (delta = c * sum|k| * max|W|, c
//      covering the split residual, the accumulation and the sequential-sum error)
//      and the keys' truncation below eps, two rows whose listed scores differ by more
//      than 2 delta + eps rank the same way exactly.  So when every adjacent gap among
//      the approximate top k+1 is wider, the approximate top-k (set and order) is the
//      exact one and nothing is rescored -- the common case.  Otherwise only the rows
//      in a chain of narrow gaps (starting inside the top k+1) are rescored in the
//      sequential fp32 order of the CPU oracle (each product and sum rounded
//      separately) and ranked with the lower-index-first tie order
//      (src/cpp/engine/src/deltagrid_math.cpp:155-167), so indices are exact; a chain
//      that runs past the last listed candidate, or comes within one gap width of the
//      filter's final value (below which the list may lack scores), rescans every row;
//   4. u_k (the top scores, exact where rescored, else the listed ones: relative error
//      below 2^(bits of G - 23), inside the outputs' 16-bit rounding), u_q (each query
//      dot split over eight lanes, so a warp reads whole router rows), normalisation,
//      and the K x K Kronecker outputs written with 16-byte stores.
#include <cuda.h>

#include <mutex>

#include "dg_common.cuh"
#include "tc_util.cuh"

namespace {

constexpr int RT_M = 128;        // tokens per CTA
constexpr int RT_NMAX = 128;     // router rows per MMA block (256 TMEM columns per CTA: two CTAs per SM)
constexpr int RT_E = 16;         // most approximate candidates kept per token and axis (k + 4, or 2k above 256 rows)
constexpr int RT_DH = 64;

constexpr uint32_t SM_KT = 0;                              // K tile: 128 rows x 128 B, 128B swizzle
constexpr uint32_t SM_W = 16384;                           // per axis (hi, lo) x 256 rows x 128 B
constexpr uint32_t SM_WPART = RT_NMAX * 128;
constexpr uint32_t SM_AX0 = SM_W;                           // results [axis][3][8][128] (u_k, u_q, index), over the
                                                            // router buffers once every block is scored
constexpr uint32_t SM_STASH = SM_W + 4 * SM_WPART;          // [axis][16][128] scores of the chunk being merged
constexpr uint32_t SM_BAR = SM_STASH + 2 * 16 * RT_M * 4;
static_assert((2 * 3 * 8 + 2 * RT_E) * RT_M * 4 <= 4 * SM_WPART, "results and rescored lists fit over the router buffers");
constexpr uint32_t SM_BYTES = SM_BAR + 8 * 8;

struct RtParams {
    const void* k;
    const void* q;
    const float* wk[2];
    const float* wq[2];
    const float* q_scale;        // [H] or null
    const unsigned* wmax;        // [2] max |router_k| per axis (float bits)
    void* out_wk;
    void* out_wq;
    int64_t* out_idx;
    int64_t N;
    int H, T, nrows;
    int G[2];
    float delta_scale;
    int32_t* status;
    uint32_t wait_limit;         // polls of each bounded wait
};

__device__ __forceinline__ bool ranks_before(float a, int ia, float b, int ib) {
    return (a > b) | ((a == b) & (ia < ib));
}

// Candidate keys: the score's bits in an order that compares as unsigned integers the
// way the floats compare, with the low `ib` bits replaced by (imask - row).  One key
// holds score and row; a larger key ranks first, and equal truncated scores rank the
// lower row first.  Truncation lowers a score by less than 2^ib units in its last place.
__device__ __forceinline__ uint32_t cand_key(float s, int row, uint32_t imask) {
    const uint32_t u = __float_as_uint(s);
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (o & ~imask) | (imask - (uint32_t)row);
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// a[0 .. N) sorted descending by a bitonic network (compile-time compare-exchanges)
template <int N>
__device__ __forceinline__ void bitonic_sort_desc(uint32_t* a) {
#pragma unroll
    for (int k = 2; k <= N; k <<= 1)
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1)
#pragma unroll
            for (int i = 0; i < N; ++i) {
                const int l = i ^ j;
                if (l > i) {
                    const uint32_t x = a[i], y = a[l];
                    const bool desc = (i & k) == 0;
                    a[i] = desc ? max(x, y) : min(x, y);
                    a[l] = desc ? min(x, y) : max(x, y);
                }
            }
}

// the truncated score of a key (never above the score itself); keys below every finite
// score (the empty list's zeros) give -inf
__device__ __forceinline__ float key_value(uint32_t k, uint32_t imask) {
    if (k < 0x00800000u) return -INFINITY;
    const uint32_t o = k & ~imask;
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

// NC independent sequential fp32 dots over 64 (each product and sum rounded, the
// oracle's order), interleaved so their dependency chains overlap.  x: this token's
// 64 values, 16-byte chunks at xoff(c); w[j]: router rows.
template <int NC, typename LoadX>
__device__ __forceinline__ void exact_dots(LoadX load_x, const float* const (&w)[NC], float (&out)[NC]) {
#pragma unroll
    for (int j = 0; j < NC; ++j) out[j] = 0.f;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
        float xv[8];
        load_x(c, xv);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float4 wv[NC];
#pragma unroll
            for (int j = 0; j < NC; ++j) wv[j] = __ldg(reinterpret_cast<const float4*>(w[j] + 8 * c + 4 * h));
#pragma unroll
            for (int j = 0; j < NC; ++j) {
                out[j] = __fadd_rn(out[j], __fmul_rn(wv[j].x, xv[4 * h + 0]));
                out[j] = __fadd_rn(out[j], __fmul_rn(wv[j].y, xv[4 * h + 1]));
                out[j] = __fadd_rn(out[j], __fmul_rn(wv[j].z, xv[4 * h + 2]));
                out[j] = __fadd_rn(out[j], __fmul_rn(wv[j].w, xv[4 * h + 3]));
            }
        }
    }
}

// v[i] += the partner lane's v[i + CNT] (lanes with `upper` keep the upper half instead):
// after the step, v[0 .. CNT) hold CNT of the 2 CNT values, summed over the lane pair
template <int CNT, int NV>
__device__ __forceinline__ void halve_sum(float (&v)[NV], int off, bool upper) {
#pragma unroll
    for (int i = 0; i < CNT; ++i) {
        const float send = upper ? v[i] : v[i + CNT];
        const float keep = upper ? v[i + CNT] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
}

template <typename T>
__device__ __forceinline__ void unpack8(uint4 v, float (&x)[8]) {
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = dg::to_f(e[i]);
}

// 256 threads: warps 0-3 route axis 0, warps 4-7 axis 1, of the same 128 tokens
// (thread t of a group owns token t and TMEM lane t; each axis owns 256 TMEM columns).
template <typename T, int K, int E>
__global__ void __launch_bounds__(2 * RT_M, 2)
    router_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmhi,
                     const __grid_constant__ CUtensorMap tmlo, RtParams p) {
    constexpr bool BF16 = !std::is_same<T, __half>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kt = sm + SM_KT;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + SM_BAR);
    uint64_t* bar_kt = bars;           // K tile landed
    uint64_t* bar_w = bars + 1;        // [axis] router block landed
    uint64_t* bar_a = bars + 3;        // [axis] scores of a block in TMEM (router buffer read)
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 5);
    float* res = reinterpret_cast<float*>(sm + SM_AX0);         // [axis][3][8][RT_M] u_k, u_q, index
    uint32_t* stash = reinterpret_cast<uint32_t*>(sm + SM_STASH);   // [axis][16][RT_M]

    const int tid = threadIdx.x, warp = tid >> 5;
    const int ax = warp >> 2;                      // axis of this thread's group
    const int t = tid & (RT_M - 1);                // token within the tile = TMEM lane
    const int64_t n0 = (int64_t)blockIdx.x * RT_M;
    const int64_t n = n0 + t;
    const int nrows = p.nrows;
    const int G = ax ? p.G[1] : p.G[0];       // (a select: indexing the parameter array puts it on the stack)
    const int nb = G / nrows;
    const uint32_t wpart = (uint32_t)nrows * 128u;
    const uint32_t idesc = tc::make_idesc(128, nrows, BF16 ? 1 : 0, 0, 0);
    const bool issuer = t == 0;
    uint8_t* whi = sm + SM_W + (uint32_t)(2 * ax) * SM_WPART;
    uint8_t* wlo = whi + SM_WPART;
    const int wrow0 = ax ? p.G[0] : 0;

    auto load_w = [&](int j) {
        tc::mbar_expect_tx(bar_w + ax, 2 * wpart);
        tc::tma_load_2d(whi, &tmhi, bar_w + ax, 0, wrow0 + j * nrows);
        tc::tma_load_2d(wlo, &tmlo, bar_w + ax, 0, wrow0 + j * nrows);
    };

    if (warp == 0) tc::tmem_alloc(tmem_holder, 2 * RT_NMAX);
    if (tid == 0) {
        for (int i = 0; i < 5; ++i) tc::mbar_init(bars + i, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tmk);
        tc::prefetch_tmap(&tmhi);
        tc::prefetch_tmap(&tmlo);
        tc::mbar_expect_tx(bar_kt, RT_M * 128);
        tc::tma_load_2d(kt, &tmk, bar_kt, 0, (int)n0);
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (issuer) load_w(0);
    const uint32_t tmem = *tmem_holder;
    const uint32_t tacc = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)ax * RT_NMAX;

    auto issue = [&]() {
        const uint32_t d = tmem + (uint32_t)ax * RT_NMAX;
        const uint32_t a0 = tc::smem_u32(kt);
#pragma unroll
        for (int lo = 0; lo < 2; ++lo) {
            const uint32_t b0 = tc::smem_u32(lo ? wlo : whi);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                tc::mma_f16(d, tc::make_desc(a0 + 32 * kk, 16, 1024), tc::make_desc(b0 + 32 * kk, 16, 1024), idesc,
                            (lo | kk) != 0);
        }
        tc::mma_commit(bar_a + ax);
    };

    bool bad = !tc::mbar_wait(bar_kt, 0, p.wait_limit);
    const bool kt_pending = bad;
    // the issuer's copy and MMA batch in flight (parity of the phase still awaited, or -1),
    // drained before the TMEM is freed when a wait gives up
    int pend_w = issuer ? 0 : -1, pend_a = -1;
    // sum |k| of this token, for the error bound
    float kabs = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        float x[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(kt + tc::sw128(t, c)), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) kabs += fabsf(x[e]);
    }

    // running approximate top-E as descending keys (E >= k + 4: room for the narrow-gap
    // chains of the exactness step below)
    static_assert(E >= K + 4 && E <= RT_E, "candidate list length");
    const int ib = 32 - __clz(G - 1);
    const uint32_t imask = (1u << ib) - 1u;
    // every score within mg below the (k+1)-th listed one is kept: mg is eight widths of
    // the narrow gap (2 delta + the keys' truncation) at this token's largest |score|
    const float wmx = __uint_as_float(p.wmax[ax]);
    const float mg = 8.f * (2.f * p.delta_scale * kabs * wmx + ldexpf(kabs * wmx * 1.01f, ib - 22));
    uint32_t lk[E];
#pragma unroll
    for (int i = 0; i < E; ++i) lk[i] = 0u;
    float thr = -INFINITY;                         // the filter: max(E-th key, (k+1)-th key - mg)
    uint32_t* st = stash + ax * 16 * RT_M;

    for (int j = 0; j < nb; ++j) {
        const uint32_t ph = (uint32_t)j & 1u;
        if (issuer) {
            if (!bad && tc::mbar_wait(bar_w + ax, ph, p.wait_limit)) {
                pend_w = -1;
                tc::tc_fence_after();
                issue();
                pend_a = (int)ph;
            } else {
                bad = true;
            }
        }
        if (!bad && tc::mbar_wait(bar_a + ax, ph, p.wait_limit)) {
            pend_a = -1;
        } else {
            bad = true;
        }
        tc::tc_fence_after();
        if (issuer && j + 1 < nb && !bad) {
            load_w(j + 1);                                        // the MMAs have read the router buffer
            pend_w = (int)((j + 1) & 1);
        }
        // 32 scores per TMEM read; a score enters the list only if it is at least the
        // filter, which after the first columns few are
        const int gbase = j * nrows;
        for (int c0 = 0; c0 < nrows && !bad; c0 += 32) {
            uint32_t r[32];
            tc::tmem_ld32(tacc + (uint32_t)c0, r);
            tc::tmem_wait_ld();
            if (j == 0 && c0 == 0) {
                // the first 32 scores: the list is their top 16, by a sorting network
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = cand_key(__uint_as_float(r[i]), i, imask);
                bitonic_sort_desc<16>(r);
                bitonic_sort_desc<16>(r + 16);
#pragma unroll
                for (int i = 0; i < 16; ++i) r[i] = max(r[i], r[31 - i]);       // a bitonic sequence
#pragma unroll
                for (int jj = 8; jj > 0; jj >>= 1)
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        if ((i ^ jj) > i) {
                            const uint32_t x = r[i], y = r[i ^ jj];
                            r[i] = max(x, y);
                            r[i ^ jj] = min(x, y);
                        }
#pragma unroll
                for (int i = 0; i < E; ++i) lk[i] = r[i];
                thr = fmaxf(key_value(lk[E - 1], imask), key_value(lk[K], imask) - mg);
                continue;
            }
            // the 32 scores' maximum by three-input maxima (16 instead of 31)
            float mt[12];
#pragma unroll
            for (int i = 0; i < 10; ++i)
                mt[i] = fmax3(__uint_as_float(r[3 * i]), __uint_as_float(r[3 * i + 1]), __uint_as_float(r[3 * i + 2]));
            mt[10] = __uint_as_float(r[30]);
            mt[11] = __uint_as_float(r[31]);
#pragma unroll
            for (int i = 0; i < 4; ++i) mt[i] = fmax3(mt[3 * i], mt[3 * i + 1], mt[3 * i + 2]);
            const float mx = fmaxf(fmax3(mt[0], mt[1], mt[2]), mt[3]);
            if (!(mx >= thr)) continue;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t m = 0;
#pragma unroll
                for (int i = 0; i < 16; ++i) m |= (__uint_as_float(r[16 * h + i]) >= thr ? 1u : 0u) << i;
                if (m != 0u) {
                // the half's 16 scores in this thread's 64-byte stash row, 16-byte chunks
                // rotated by lane pair so that eight lanes' stores hit distinct banks
                uint8_t* srb = reinterpret_cast<uint8_t*>(st) + t * 64;
                const int sw = (t >> 1) & 3;
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    *reinterpret_cast<uint4*>(srb + 16 * (c ^ sw)) =
                        make_uint4(r[16 * h + 4 * c], r[16 * h + 4 * c + 1], r[16 * h + 4 * c + 2], r[16 * h + 4 * c + 3]);
#pragma unroll 1
                while (m != 0u) {
                    const int i = __ffs(m) - 1;
                    m &= m - 1;
                    const uint32_t sv = *reinterpret_cast<const uint32_t*>(srb + 16 * ((i >> 2) ^ sw) + 4 * (i & 3));
                    const uint32_t key = cand_key(__uint_as_float(sv), gbase + c0 + 16 * h + i, imask);
                    // sorted insert without a dependency chain: entry q becomes
                    // max(old q, min(key, old q-1))
#pragma unroll
                    for (int q = E - 1; q > 0; --q) lk[q] = max(lk[q], min(key, lk[q - 1]));
                    lk[0] = max(lk[0], key);
                }
                thr = fmaxf(key_value(lk[E - 1], imask), key_value(lk[K], imask) - mg);
                }
            }
        }
        tc::tc_fence_before();
        asm volatile("bar.sync %0, 128;" ::"r"(1 + ax) : "memory");      // accumulator free for the next block
        tc::tc_fence_after();
    }
    float lv[E];
    int li[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
        lv[i] = key_value(lk[i], imask);
        const int row = (int)(imask - (lk[i] & imask));
        li[i] = lk[i] < 0x00800000u || row >= G ? 0 : row;     // an unfilled entry (non-finite scores)
    }

    // both axes are scored: the router buffers become the result arrays below
    __syncthreads();
    // exact top-k.  Rows whose approximate scores are more than 2 delta apart rank as
    // their approximate scores do; rescore (in the oracle's order) only the chains of
    // narrower gaps that start inside the approximate top k+1.
    const float* W = ax ? p.wk[1] : p.wk[0];
    const float delta = p.delta_scale * kabs * __uint_as_float(p.wmax[ax]);
    // plus the keys' truncation (below 2^ib units in the last place of any listed score)
    const float d2 = 2.f * delta + ldexpf(fmaxf(fabsf(lv[0]), fabsf(lv[E - 1])), ib - 22) + 1e-30f;
    uint32_t need = 0;                                    // list positions to rescore
    // the list holds every score at or above ff (the scan kept all within mg of the
    // final (k+1)-th); a chain that comes within d2 of ff may miss one: every row
    const float ff = lv[K] - mg;
#pragma unroll
    for (int i = 0; i < E - 1; ++i) {
        const bool narrow = !(lv[i] - lv[i + 1] > d2);    // (also when scores are equal or not finite)
        if (i < K) {
            if (narrow) need |= 3u << i;
        } else if ((need >> i) & 1u) {
            if (!(lv[i] - d2 >= ff)) need |= 1u << (E - 1);
            else if (narrow) need |= 1u << (i + 1);
        }
    }
    float tv[K];
    int ti[K];
    auto load_k = [&](int c, float (&x)[8]) { unpack8<T>(*reinterpret_cast<const uint4*>(kt + tc::sw128(t, c)), x); };
    if (need == 0u) {                                     // the approximate order is the exact one
#pragma unroll
        for (int r = 0; r < K; ++r) { tv[r] = lv[r]; ti[r] = li[r]; }
    } else {
#pragma unroll
        for (int r = 0; r < K; ++r) { tv[r] = -INFINITY; ti[r] = 0x7fffffff; }
        auto keep = [&](float sc, int g) {
#pragma unroll
            for (int q = 0; q < K; ++q) {
                const bool sw = ranks_before(sc, g, tv[q], ti[q]);
                const float a = tv[q];
                const int b = ti[q];
                tv[q] = sw ? sc : a;
                ti[q] = sw ? g : b;
                sc = sw ? a : sc;
                g = sw ? b : g;
            }
        };
        if ((need >> (E - 1)) & 1u) {                  // the narrow chain runs past the list: every row
#pragma unroll 1
            for (int i0 = 0; i0 < G; i0 += 8) {
                const float* wr[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) wr[j] = W + (int64_t)(i0 + j < G ? i0 + j : 0) * RT_DH;
                float sc[8];
                exact_dots<8>(load_k, wr, sc);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (i0 + j < G) keep(sc[j], i0 + j);
            }
        } else {
            // exact scores for the flagged positions, four at a time; the list goes through
            // shared memory (the stash, and the free end of the router buffers) so that the
            // positions can be indexed at run time
            uint32_t* srow = st;
            float* sval = res + 2 * 3 * 8 * RT_M + ax * RT_E * RT_M;
#pragma unroll
            for (int q = 0; q < E; ++q) {
                srow[q * RT_M + t] = (uint32_t)li[q];
                sval[q * RT_M + t] = lv[q];
            }
#pragma unroll 1
            for (uint32_t m = need; m != 0u;) {
                int pos[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    pos[j] = m ? __ffs(m) - 1 : -1;
                    if (m) m &= m - 1;
                }
                const float* wr[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) wr[j] = W + (int64_t)(pos[j] >= 0 ? (int)srow[pos[j] * RT_M + t] : 0) * RT_DH;
                float sc[4];
                exact_dots<4>(load_k, wr, sc);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (pos[j] >= 0) sval[pos[j] * RT_M + t] = sc[j];
            }
#pragma unroll
            for (int q = 0; q < E; ++q) lv[q] = sval[q * RT_M + t];
            // rank: rows outside the chains keep their approximate scores, which differ from
            // every neighbour's by more than 2 delta, so the mixed comparison is exact
#pragma unroll
            for (int q = 0; q < E; ++q) keep(lv[q], li[q]);
        }
    }
    // u_k = normalize(top scores); u_q = normalize(W_q[top] q), the K query dots interleaved
    float ssk = 0.f;
#pragma unroll
    for (int r = 0; r < K; ++r) ssk += tv[r] * tv[r];
    const float nk = fmaxf(sqrtf(ssk), 1e-12f);
    float* rs = res + ax * 3 * 8 * RT_M;
#pragma unroll
    for (int r = 0; r < K; ++r) {
        rs[(0 * 8 + r) * RT_M + t] = tv[r] / nk;
        rs[(2 * 8 + r) * RT_M + t] = __int_as_float(ti[r]);
    }
    __syncwarp();
    // query dots W_q[row] . q, eight lanes per token (each 8 of the 64 columns, with
    // fused multiply-adds), four tokens of this warp at a time: the router rows are read
    // as whole 256-byte rows
    {
        const float* WQ = ax ? p.wq[1] : p.wq[0];
        const int lane = tid & 31, sub8 = lane & 7;
#pragma unroll 2
        for (int it = 0; it < 8; ++it) {
            const int tw = (warp & 3) * 32 + 4 * it + (lane >> 3);       // token of this lane's group
            const int64_t nn = n0 + tw < p.N ? n0 + tw : 0;
            float qx[8];
            unpack8<T>(__ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + nn * RT_DH) + sub8), qx);
            float v[K];
#pragma unroll
            for (int r = 0; r < K; ++r) {
                const int row = __float_as_int(rs[(2 * 8 + r) * RT_M + tw]);
                const float4* wp = reinterpret_cast<const float4*>(WQ + (int64_t)row * RT_DH + 8 * sub8);
                const float4 a = __ldg(wp), b = __ldg(wp + 1);
                float acc = a.x * qx[0];
                acc = fmaf(a.y, qx[1], acc);
                acc = fmaf(a.z, qx[2], acc);
                acc = fmaf(a.w, qx[3], acc);
                acc = fmaf(b.x, qx[4], acc);
                acc = fmaf(b.y, qx[5], acc);
                acc = fmaf(b.z, qx[6], acc);
                v[r] = fmaf(b.w, qx[7], acc);
            }
            // sum over the group's 8 lanes, halving the values each step: lane sub8 ends with
            // row sub8 (K = 8) or row sub8 / 2 (K = 4)
            if constexpr (K == 8) {
                halve_sum<4>(v, 4, (sub8 & 4) != 0);
                halve_sum<2>(v, 2, (sub8 & 2) != 0);
                halve_sum<1>(v, 1, (sub8 & 1) != 0);
                rs[(1 * 8 + sub8) * RT_M + tw] = v[0];
            } else {
                halve_sum<2>(v, 4, (sub8 & 4) != 0);
                halve_sum<1>(v, 2, (sub8 & 2) != 0);
                v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
                if ((sub8 & 1) == 0) rs[(1 * 8 + (sub8 >> 1)) * RT_M + tw] = v[0];
            }
        }
    }
    __syncwarp();
    {
        float qv[K];
        float ssq = 0.f;
#pragma unroll
        for (int r = 0; r < K; ++r) {
            qv[r] = rs[(1 * 8 + r) * RT_M + t];
            ssq += qv[r] * qv[r];
        }
        const float nq = fmaxf(sqrtf(ssq), 1e-12f);
#pragma unroll
        for (int r = 0; r < K; ++r) rs[(1 * 8 + r) * RT_M + t] = qv[r] / nq;
    }
    bad = __syncthreads_or(bad) != 0;
    if (!bad && n < p.N) {
        // Kronecker: group ax writes rows i in [ax K/2, ax K/2 + K/2) of the K x K product
        constexpr int A = K * K;
        const int h = (int)((n / p.T) % p.H);
        const float qsc = p.q_scale ? p.q_scale[h] : 1.f;
        const float* r0 = res;
        const float* r1 = res + 3 * 8 * RT_M;
        // this group's rows i of the K x K product are one contiguous run of the token's
        // A entries: written with 16-byte stores
        constexpr int NE = K / 2 * K;                     // entries per group (32 or 8)
        T* owk = static_cast<T*>(p.out_wk) + n * A + ax * NE;
        T* owq = static_cast<T*>(p.out_wq) + n * A + ax * NE;
        int64_t* oix = p.out_idx + n * A + ax * NE;
        float ukj[K], uqj[K];
        int64_t ixj[K];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            ukj[j] = r1[(0 * 8 + j) * RT_M + t];
            uqj[j] = r1[(1 * 8 + j) * RT_M + t];
            ixj[j] = __float_as_int(r1[(2 * 8 + j) * RT_M + t]);
        }
#pragma unroll
        for (int ii = 0; ii < K / 2; ++ii) {
            const int i = ax * (K / 2) + ii;
            const float uki = r0[(0 * 8 + i) * RT_M + t];
            const float uqi = r0[(1 * 8 + i) * RT_M + t];
            const int64_t xi = (int64_t)__float_as_int(r0[(2 * 8 + i) * RT_M + t]) * p.G[1];
            uint32_t wkp[K / 2], wqp[K / 2];
#pragma unroll
            for (int j = 0; j < K / 2; ++j) {
                T a = dg::from_f<T>(uki * ukj[2 * j]), b = dg::from_f<T>(uki * ukj[2 * j + 1]);
                T c = dg::from_f<T>((uqi * uqj[2 * j]) * qsc), d = dg::from_f<T>((uqi * uqj[2 * j + 1]) * qsc);
                wkp[j] = (uint32_t)(*reinterpret_cast<uint16_t*>(&a)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&b)) << 16);
                wqp[j] = (uint32_t)(*reinterpret_cast<uint16_t*>(&c)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&d)) << 16);
            }
            if constexpr (K == 8) {
                reinterpret_cast<uint4*>(owk + ii * K)[0] = make_uint4(wkp[0], wkp[1], wkp[2], wkp[3]);
                reinterpret_cast<uint4*>(owq + ii * K)[0] = make_uint4(wqp[0], wqp[1], wqp[2], wqp[3]);
            } else {
                reinterpret_cast<uint2*>(owk + ii * K)[0] = make_uint2(wkp[0], wkp[1]);
                reinterpret_cast<uint2*>(owq + ii * K)[0] = make_uint2(wqp[0], wqp[1]);
            }
#pragma unroll
            for (int j = 0; j < K; j += 2) {
                longlong2 v2;
                v2.x = xi + ixj[j];
                v2.y = xi + ixj[j + 1];
                reinterpret_cast<longlong2*>(oix + ii * K)[j / 2] = v2;
            }
        }
    }
    if (bad && n < p.N) {
        // a wait gave up: the tile's tokens get index -1 (out of range: the recurrence
        // skips such rows and flags them in its status word) and zero weights
        constexpr int A = K * K, NE = K / 2 * K;
        T* owk = static_cast<T*>(p.out_wk) + n * A + ax * NE;
        T* owq = static_cast<T*>(p.out_wq) + n * A + ax * NE;
        int64_t* oix = p.out_idx + n * A + ax * NE;
        for (int e = 0; e < NE; ++e) {
            owk[e] = dg::from_f<T>(0.f);
            owq[e] = dg::from_f<T>(0.f);
            oix[e] = -1;
        }
    }
    if (bad && tid == 0) dg::flag_status(p.status, DG_DEVCHK_TIMEOUT);
    if (bad) {
        // let the copies and MMAs this CTA issued finish before its shared memory and
        // TMEM are released (bounded too)
        constexpr uint32_t DRAIN = 1u << 22;
        if (tid == 0 && kt_pending) tc::mbar_wait(bar_kt, 0, DRAIN);
        if (pend_w >= 0) tc::mbar_wait(bar_w + ax, (uint32_t)pend_w, DRAIN);
        if (pend_a >= 0) tc::mbar_wait(bar_a + ax, (uint32_t)pend_a, DRAIN);
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 2 * RT_NMAX);
    }
}

// router weights -> 16-bit hi and lo parts (stacked axes) and max |w| per axis
template <typename T>
__global__ void router_split_kernel(const float* w0, const float* w1, int g0, int g1, T* hi, T* lo, unsigned* wmax) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n0 = (int64_t)g0 * RT_DH, nt = n0 + (int64_t)g1 * RT_DH;
    if (i >= nt) return;
    const float w = i < n0 ? w0[i] : w1[i - n0];
    const T h = dg::from_f<T>(w);
    hi[i] = h;
    lo[i] = dg::from_f<T>(w - dg::to_f(h));
    atomicMax(wmax + (i < n0 ? 0 : 1), __float_as_uint(fabsf(w)));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// 2-D map over [rows][64] 16-bit values, box 64 x box_rows, 128B swizzle
bool make_map_2d(CUtensorMap* m, const void* base, int64_t rows, int box_rows, bool bf16) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)RT_DH, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)RT_DH * 2};
    cuuint32_t box[2] = {(cuuint32_t)RT_DH, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int K, int E>
int launch_tc(const RtParams& p0, const CUtensorMap& mk, const CUtensorMap& mhi, const CUtensorMap& mlo,
              cudaStream_t s) {
    auto kern = router_tc_kernel<T, K, E>;
    const int smem = (int)SM_BYTES + 1024;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    kern<<<(unsigned)((p0.N + RT_M - 1) / RT_M), 2 * RT_M, smem, s>>>(mk, mhi, mlo, p0);
    return dg_host::check_launch();
}

// The split router (hi, lo parts and the two max|W| words) lives in a per-device buffer
// kept across calls: a stream-ordered allocation per call costs a remap of the pool
// (~0.25 ms) whenever the stream has drained in between.  `done` is recorded after each
// call's last kernel; the next call's stream waits for it, so calls on different streams
// take turns on the buffer.  Calls under stream capture allocate from the graph instead.
struct SplitWs {
    void* p = nullptr;
    size_t bytes = 0;
    cudaEvent_t done = nullptr;
};
SplitWs g_split[64];
std::mutex g_split_mu;

}  // namespace

namespace dg_host {

uint32_t wait_limit();

// Whether the tensor-core router covers the call (else the CUDA-core router runs).
bool route_tc_supports(int dtype, int dh, int g0, int g1, int top_k, const void* k, const void* q,
                       const float* rk0, const float* rk1, const float* rq0, const float* rq1, const void* wk,
                       const void* wq, const int64_t* idx) {
    if (dtype != DG_DTYPE_F16 && dtype != DG_DTYPE_BF16) return false;
    if (dh != RT_DH || (top_k != 4 && top_k != 8)) return false;
    auto rows = [](int g) { return g <= RT_NMAX ? g : RT_NMAX; };
    if (rows(g0) != rows(g1)) return false;
    const int nr = rows(g0);
    // the scan reads the scores 32 columns at a time: whole 32-row groups per block
    if (nr % 32 != 0 || g0 % nr != 0 || g1 % nr != 0) return false;
    // inputs for TMA and 16-byte loads; outputs for the 16-byte (top-8) / 8-byte stores
    const uintptr_t al = (uintptr_t)k | (uintptr_t)q | (uintptr_t)rk0 | (uintptr_t)rk1 | (uintptr_t)rq0 |
                         (uintptr_t)rq1 | (uintptr_t)wk | (uintptr_t)wq | (uintptr_t)idx;
    return (al & 15) == 0;
}

int route_tc(int dtype, int64_t N, int H, int T, int g0, int g1, int top_k, const void* k, const void* q,
             const float* rk0, const float* rk1, const float* rq0, const float* rq1, const float* q_scale, void* wk,
             void* wq, int64_t* idx, cudaStream_t s) {
    const bool bf16 = dtype == DG_DTYPE_BF16;
    const int64_t wn = (int64_t)(g0 + g1) * RT_DH;
    const size_t bytes = (size_t)wn * 2 * 2 + 64;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(s, &cs);
    if (e != cudaSuccess) return record_cuda_error(e);
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e);
    const bool cached = cs == cudaStreamCaptureStatusNone && dev >= 0 && dev < 64;
    std::unique_lock<std::mutex> lock(g_split_mu, std::defer_lock);
    void* ws = nullptr;
    if (cached) {
        lock.lock();
        SplitWs& w = g_split[dev];
        if (!w.done) {
            e = cudaEventCreateWithFlags(&w.done, cudaEventDisableTiming);
            if (e != cudaSuccess) { w.done = nullptr; return record_cuda_error(e); }
        }
        if (w.bytes < bytes) {
            if (w.p) {
                e = cudaEventSynchronize(w.done);               // the last call has finished with it
                if (e == cudaSuccess) e = cudaFree(w.p);
                w.p = nullptr;
                w.bytes = 0;
                if (e != cudaSuccess) return record_cuda_error(e);
            }
            e = cudaMalloc(&w.p, bytes);
            if (e != cudaSuccess) { w.p = nullptr; return record_cuda_error(e); }
            w.bytes = bytes;
        } else {
            e = cudaStreamWaitEvent(s, w.done, 0);
            if (e != cudaSuccess) return record_cuda_error(e);
        }
        ws = w.p;
    } else {
        e = cudaMallocAsync(&ws, bytes, s);                    // stream-ordered (a graph allocation under capture)
        if (e != cudaSuccess) return record_cuda_error(e);
    }
    uint8_t* hi = static_cast<uint8_t*>(ws);
    uint8_t* lo = hi + wn * 2;
    unsigned* wmax = reinterpret_cast<unsigned*>(lo + wn * 2);
    int rc = DG_OK;
    e = cudaMemsetAsync(wmax, 0, 2 * sizeof(unsigned), s);
    if (e != cudaSuccess) rc = record_cuda_error(e);
    if (rc == DG_OK) {
        const unsigned blocks = (unsigned)((wn + 255) / 256);
        if (bf16)
            router_split_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(rk0, rk1, g0, g1, reinterpret_cast<__nv_bfloat16*>(hi),
                                                                     reinterpret_cast<__nv_bfloat16*>(lo), wmax);
        else
            router_split_kernel<__half><<<blocks, 256, 0, s>>>(rk0, rk1, g0, g1, reinterpret_cast<__half*>(hi),
                                                              reinterpret_cast<__half*>(lo), wmax);
        rc = check_launch();
    }
    const int nr = g0 <= RT_NMAX ? g0 : RT_NMAX;
    CUtensorMap mk, mhi, mlo;
    if (rc == DG_OK && (!make_map_2d(&mk, k, N, RT_M, bf16) || !make_map_2d(&mhi, hi, g0 + g1, nr, bf16) ||
                        !make_map_2d(&mlo, lo, g0 + g1, nr, bf16)))
        rc = DG_ERR_UNSUPPORTED;
    if (rc == DG_OK) {
        // |approx - exact| <= c * sum|k| * max|w|: split residual, accumulation and the
        // sequential sum's own rounding, with a factor 2 margin (2^-15 f16, 2^-14 bf16)
        RtParams p{k, q, {rk0, rk1}, {rq0, rq1}, q_scale, wmax, wk, wq, idx, N, H, T, nr, {g0, g1},
                   bf16 ? 6.103515625e-05f : 3.0517578125e-05f, nullptr, wait_limit()};
        // list length: k + 4 for small grids; 2k above 256 rows per axis (measured faster there)
        const bool wide = g0 > 256 || g1 > 256;
        if (bf16)
            rc = top_k == 4 ? launch_tc<__nv_bfloat16, 4, 8>(p, mk, mhi, mlo, s)
                 : wide     ? launch_tc<__nv_bfloat16, 8, 16>(p, mk, mhi, mlo, s)
                            : launch_tc<__nv_bfloat16, 8, 12>(p, mk, mhi, mlo, s);
        else
            rc = top_k == 4 ? launch_tc<__half, 4, 8>(p, mk, mhi, mlo, s)
                 : wide     ? launch_tc<__half, 8, 16>(p, mk, mhi, mlo, s)
                            : launch_tc<__half, 8, 12>(p, mk, mhi, mlo, s);
    }
    e = cached ? cudaEventRecord(g_split[dev].done, s) : cudaFreeAsync(ws, s);
    if (rc != DG_OK) return rc;
    return e == cudaSuccess ? DG_OK : record_cuda_error(e);
}

}  // namespace dg_host
