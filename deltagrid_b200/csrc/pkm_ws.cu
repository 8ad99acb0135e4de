// pkm_ws.cu -- warp-specialised Sparse Delta-PKM recurrence for 16-bit state.
//
// Same math as pkm_seq.cu (src/cpp/delta_kernel.cu:885-920): per lane and step,
// gather the `active` rows S[idx_t], y = wq.s and pred = wk.s over the rows,
// r = beta (v - pred), scatter S[idx_t] = cast(alpha s + (r) wk), rows rounded to
// the storage dtype every step.
//
// Two kernels.  For a short sequence, or when the recurrence fills every SM, they run
// back to back on the caller's stream.  Otherwise the call runs in four step pieces:
// the pre-pass of piece i + 1 runs on a low-priority side stream while the
// recurrence of piece i runs on a high-priority one, on the SMs the recurrence leaves
// free, so only the first piece's pre-pass stays on the critical path.  A piece
// boundary only turns forwards into gathers (the previous piece's rows are in global
// memory by then), so the pieces give the unsplit call's results bit for bit.
//
// pkm_hazard_kernel -- index-only pre-pass over all SMs.  For every row (t, m)
//   of every lane it finds the last earlier step w in [t-D+1, t-1] that wrote
//   the same slot and writes a 16-bit code to the workspace: -1 gather the row
//   from global memory, -2 no row (m >= A, or an index out of range, which is
//   flagged), else (t - w) << 6 | position of the slot in step w.  A CTA
//   resolves 48 steps of one lane plus D-1 steps of lookback in parallel: all
//   (slot, step, position) entries are bucket-sorted in shared memory (counting
//   sort: one 32-bit atomicAdd per entry, a block prefix sum), then every row of
//   the 48 steps scans its bucket.  Exact, with no capacity to overflow.
//
// pkm_ws_kernel -- the recurrence.  One CTA per (lane, part of the row); three
//   roles run concurrently on a ring of R = 2D row slots, synchronised by
//   mbarriers:
//   loader (1 warp)  metadata (idx, wk, wq, v, beta, alpha, codes) 16 steps at a
//       time into a 3-chunk ring, each chunk reloaded once its last update is done;
//       once a chunk has landed it turns the codes into each row's shared address (own
//       ring row, the forwarding writer's row, or the zero row) and each step's
//       forwarding distances, so the step warps read one word per row.
//   gather (2 warps for 128-byte row parts, 4 for 64-byte parts)  per step t,
//       D steps ahead of the update: row-coalesced
//       cp.async (8 lanes per 128 bytes) of the rows coded "gather" into the
//       step's ring slot; other rows copy 0 bytes (zero-fill), so the issue
//       loop has no branches.
//   step warps (KPAR groups of NSL warps, the groups taking turns by step)
//       per step s, each warp of the group first takes a 16-column slice: y and
//       pred as a tensor-core GEMV, mma.sync m16n8k16 with A = the gathered rows
//       transposed (ldmatrix.trans, one row address per lane, so forwarded rows need
//       no copy; columns are the M dimension) and B = [wq, wk] (2 of 8 N columns
//       used), four MMAs for 64 rows; r = beta (v - pred) into the step's r row in
//       shared memory.  Once every slice's r is there (an mbarrier per ring step),
//       each warp takes a block of 64 / NSL rows and forms the new rows over the whole
//       row part (fp32 math, packed f32x2, one rounding), written to the ring slot
//       (for forwarding) and to global memory with 16-byte stores, a row part per
//       group of lanes, so each store instruction writes whole rows; y is staged for
//       coalesced stores.  A step that forwards a row waits for the writer step's
//       update to finish.
//
// Ordering argument: a row gathered from global memory for step t has its last
// writer w <= t-D, and the gather is issued only after the update of step t-D
// has completed (mbarrier release/acquire; updates complete in step order); a
// row whose last writer is in the window is read from the writer's ring slot,
// which the slot's next gather (for step w+R, issued after update w+R-D >= w+D)
// cannot overwrite before every reader (steps <= w+D-1) is done.
#include <mutex>

#include "dg_common.cuh"
#include "tc_util.cuh"

namespace {

constexpr int MAXA = 64;
constexpr int CHS = 16;                 // steps per metadata chunk
constexpr int NC = 3;                   // metadata chunks resident
constexpr int NLOAD = 32;               // loader threads (one warp)
// gather threads: four warps for 64-byte row parts; two for 128-byte parts, whose
// 16 slice warps leave no registers for more
template <int PB> struct GatherCfg {
    static constexpr int NGATH = PB == 128 ? 64 : 128;
    static constexpr int ROLE_WARPS = 1 + NGATH / 32;       // loader, gather (then KPAR warps per 16-column slice)
    // warps per column slice; warp k takes the steps s with s % KPAR == k.  Three for
    // 128-byte parts (four slices: 15 warps in all measured fastest), four for 64-byte
    // parts, whose two slices need the extra steps in flight
    static constexpr int KPAR = PB == 128 ? 3 : 4;
};
constexpr int HZ_STEPS = 48;            // steps resolved per pre-pass CTA
constexpr int HZ_BUCKETS = 4096;        // pre-pass hash buckets (counting sort): ~0.9 entries per bucket
constexpr int HZ_THREADS = 512;
constexpr int HZ_MAXWIN = 16;           // largest window depth D the pre-pass covers
constexpr int HZ_KMAX = ((HZ_STEPS + HZ_MAXWIN - 1) * MAXA + HZ_THREADS - 1) / HZ_THREADS;   // entries per thread
static_assert(HZ_KMAX * HZ_THREADS >= (HZ_STEPS + HZ_MAXWIN - 1) * MAXA, "pre-pass entry slots");
constexpr int HZ_ENTRIES = (HZ_STEPS + HZ_MAXWIN - 1) * MAXA;   // most (slot, step, position) entries per block

struct WsParams {
    const void* v;
    const void* beta;
    const void* wk;
    const void* wq;
    const int64_t* idx;
    const void* decay;
    void* state;
    void* out;
    int32_t* status;
    int H, T, A, Dh, parts;
    int64_t total;
    int dynamic_decay;
    const int16_t* codes;       // [lanes, T, 64] from pkm_hazard_kernel
    void* saved;                // [lanes, T, A, Dh] rows as gathered at each step, or null
    uint64_t wait_ns;           // bound of one wait (wall time); 0 gives up without waiting
    int64_t lstride;            // steps between lanes in the per-step arrays (the whole sequence's T)
    int tbase;                  // first step of this call's piece; T counts the piece's steps
};

struct MetaLayout {
    int idx, wk, wq, v, beta, alpha, code, addr, dmask, bytes;
};

__host__ __device__ inline MetaLayout meta_layout(int A, int Dh) {
    MetaLayout L;
    int o = 0;
    L.idx = o;   o += CHS * A * 8;
    L.wk = o;    o += CHS * A * 2;
    L.wq = o;    o += CHS * A * 2;
    L.v = o;     o += CHS * Dh * 2;
    L.beta = o;  o += 32;
    L.alpha = o; o += 32;
    L.code = o;  o += CHS * 64 * 2;
    L.addr = o;  o += CHS * 64 * 4;    // per row: shared address of its data for the GEMV and update (loader-made)
    L.dmask = o; o += CHS * 4;         // per step: distances of the rows it forwards (bit d)
    L.bytes = (o + 127) / 128 * 128;
    return L;
}

// shared-memory carve-up (same arithmetic on host and device)
struct SmemLayout {
    int bars, misc, rows, zrow, rbuf, ystage, meta, total;
};
// mbarriers of the recurrence kernel: full[R], done[R], rready[R], mfull[NC], mfree[NC], mready[NC]
__host__ __device__ constexpr int ws_barriers(int PB, int D) { return 3 * (2 * D) + 3 * NC; }

__host__ __device__ inline SmemLayout smem_layout(int PB, int D, int A, int Dh) {
    SmemLayout L;
    const int R = 2 * D, RS = PB + 16;
    int o = 0;
    L.bars = o;   o += (ws_barriers(PB, D) * 8 + 127) / 128 * 128;
    L.misc = o;   o += 16;
    L.rows = o;   o += R * 64 * RS;
    L.zrow = o;   o += RS;
    L.rbuf = o;   o += R * (PB / 2) * 4;     // r of each ring step's columns (fp32)
    L.ystage = o; o += 2 * CHS * PB;     // y rows of two chunks (by chunk parity)
    o = (o + 127) / 128 * 128;
    L.meta = o;   o += NC * meta_layout(A, Dh).bytes;
    L.total = o;
    return L;
}

// home cell of a slot in the pre-pass table: a 32-bit integer mix (xor-shift /
// multiply) so that the lattice-shaped slot sets of Kronecker routing spread out
__device__ __forceinline__ uint32_t slot_home(uint32_t x) {
    x ^= x >> 16;
    x *= 0x85ebca6bu;
    x ^= x >> 13;
    x *= 0xc2b2ae35u;
    x ^= x >> 16;
    return x >> (32 - 12);                                     // HZ_BUCKETS = 4096
}

// ---------------------------------------------------------------------------
// pre-pass: row codes of steps [blockIdx.x * HZ_STEPS, +HZ_STEPS) of lane blockIdx.y (of the piece).
// The block's (slot, step, position) entries are bucket-sorted in shared memory
// (one 32-bit atomicAdd per entry gives its rank in its bucket, a block prefix sum
// the bucket starts), then every row scans its bucket for the latest earlier step
// with the same slot.  Exact: there is no capacity limit to overflow.
template <int A>
__global__ void __launch_bounds__(HZ_THREADS, 3) pkm_hazard_kernel(const int64_t* __restrict__ idx, int16_t* codes,
                                                                int32_t* status, int T, int64_t total, int D,
                                                                int64_t lstride, int tbase) {
    extern __shared__ __align__(16) uint8_t hz_smem[];
    uint32_t* cnt = reinterpret_cast<uint32_t*>(hz_smem);                 // [HZ_BUCKETS] entries per bucket
    uint32_t* start = cnt + HZ_BUCKETS;                                    // [HZ_BUCKETS] first entry of a bucket
    uint32_t* wsum = start + HZ_BUCKETS;                                   // [HZ_THREADS / 32] scan partials
    unsigned long long* ent = reinterpret_cast<unsigned long long*>(wsum + 32);   // [HZ_ENTRIES] sorted
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lid = blockIdx.y;
    const int t0 = blockIdx.x * HZ_STEPS;
    const int tb = max(0, t0 - (D - 1));
    const int te = min(T, t0 + HZ_STEPS);
    const int nE = (te - tb) * A;
    // steps [tbase, tbase + T) of a lane whose arrays hold lstride steps
    const int64_t* li = idx + ((int64_t)lid * lstride + tbase + tb) * A;
    int16_t* lc = codes + ((int64_t)lid * lstride + tbase) * 64;
    for (int i = tid; i < HZ_BUCKETS; i += HZ_THREADS) cnt[i] = 0u;
    uint32_t key[HZ_KMAX], bkt[HZ_KMAX];
#pragma unroll
    for (int k = 0; k < HZ_KMAX; ++k) {
        const int e = tid + k * HZ_THREADS;
        key[k] = 0u;
        if (e < nE) {
            const int64_t x = li[e];
            if (x >= 0 && x < total) key[k] = (uint32_t)x + 1u;
            else if (tb + e / A >= t0) dg::flag_status(status, DG_DEVCHK_INDEX_RANGE);
        }
        bkt[k] = slot_home(key[k] - 1u);
    }
    __syncthreads();
    uint32_t rank[HZ_KMAX];
#pragma unroll
    for (int k = 0; k < HZ_KMAX; ++k) rank[k] = key[k] ? atomicAdd(cnt + bkt[k], 1u) : 0u;
    __syncthreads();
    // exclusive prefix sum of the bucket counts: BPT consecutive buckets per thread
    {
        constexpr int BPT = HZ_BUCKETS / HZ_THREADS;
        uint32_t cb[BPT];
        uint32_t v = 0;
#pragma unroll
        for (int i = 0; i < BPT; ++i) { cb[i] = cnt[BPT * tid + i]; v += cb[i]; }
        const uint32_t tot = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t u = __shfl_up_sync(DG_FULL_MASK, v, o);
            if (lane >= o) v += u;
        }
        if (lane == 31) wsum[warp] = v;
        __syncthreads();
        if (warp == 0) {
            uint32_t wv = lane < HZ_THREADS / 32 ? wsum[lane] : 0u;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t u = __shfl_up_sync(DG_FULL_MASK, wv, o);
                if (lane >= o) wv += u;
            }
            if (lane < HZ_THREADS / 32) wsum[lane] = wv;          // inclusive warp totals
        }
        __syncthreads();
        uint32_t base = (warp ? wsum[warp - 1] : 0u) + v - tot;
#pragma unroll
        for (int i = 0; i < BPT; ++i) { start[BPT * tid + i] = base; base += cb[i]; }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < HZ_KMAX; ++k) {
        if (!key[k]) continue;
        const int e = tid + k * HZ_THREADS;
        const int tl = e / A, m = e - tl * A;
        ent[start[bkt[k]] + rank[k]] = (unsigned long long)key[k] | ((unsigned long long)(((uint32_t)tl << 6) | (uint32_t)m) << 32);
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < HZ_KMAX; ++k) {
        const int e = tid + k * HZ_THREADS;
        if (e >= nE) continue;
        const int tl = e / A, m = e - tl * A;
        const int t = tb + tl;
        if (t < t0) continue;                                   // lookback rows only feed the table
        int cd = -2;
        if (key[k]) {
            const uint32_t b0 = start[bkt[k]], n = cnt[bkt[k]];
            int best = -1, bpos = 0;
            for (uint32_t q = 0; q < n; ++q) {
                const unsigned long long c = ent[b0 + q];
                if ((uint32_t)c == key[k]) {
                    const uint32_t st = (uint32_t)(c >> 32);
                    const int wl = (int)(st >> 6);
                    if (wl < tl && wl > best) { best = wl; bpos = (int)(st & 63); }
                }
            }
            cd = (best >= 0 && tl - best <= D - 1) ? (((tl - best) << 6) | bpos) : -1;
        }
        lc[(int64_t)t * 64 + m] = (int16_t)cd;
    }
    if (A < 64) {                                               // positions without a row
        const int na = 64 - A;
        for (int i = tid; i < (te - t0) * na; i += HZ_THREADS)
            lc[(int64_t)(t0 + i / na) * 64 + A + i % na] = (int16_t)-2;
    }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// 16-byte copy of which only the first `src_bytes` (16 or 0) are read; the rest is zero-filled
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// one poll that lets the hardware park the warp until the phase completes (or
// ~1 ms passes), so waiting warps take no issue slots
__device__ __forceinline__ bool mbar_try_wait_long(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(tc::smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
// Bounded mbarrier wait: gives up when another role aborted or after `wait_ns` of
// wall time (2 s by default; 0 gives up at once), flagging DG_DEVCHK_TIMEOUT.
__device__ __forceinline__ bool ws_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        int32_t* status, uint64_t wait_ns) {
    if (wait_ns != 0) {
        if (mbar_try_wait_long(bar, parity)) return true;
        const uint64_t t0 = globaltimer_ns();
        while (true) {
            if (mbar_try_wait_long(bar, parity)) return true;
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > wait_ns) break;
        }
    }
    dg::flag_status(status, DG_DEVCHK_TIMEOUT);
    *abort_flag = 1;
    return false;
}

template <typename T> struct MmaOp;
template <> struct MmaOp<__half> {
    __device__ __forceinline__ static void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <> struct MmaOp<__nv_bfloat16> {
    __device__ __forceinline__ static void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// two storage values <-> two floats
__device__ __forceinline__ float2 unpack2(uint32_t u, __half) {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
__device__ __forceinline__ float2 unpack2(uint32_t u, __nv_bfloat16) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __half) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// (x0, x1) * (y0, y1) and a * (x0, x1) + (c0, c1), each element rounded once (IEEE RN)
__device__ __forceinline__ unsigned long long f2pack(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float2 f2unpack(unsigned long long r) {
    float2 f;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(r));
    return f;
}
__device__ __forceinline__ unsigned long long mul_f32x2(unsigned long long x, unsigned long long y) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(x), "l"(y));
    return d;
}
__device__ __forceinline__ unsigned long long fma_f32x2(unsigned long long a, unsigned long long b,
                                                        unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

template <typename T, int PB, int D>
__global__ void __launch_bounds__(32 * (GatherCfg<PB>::ROLE_WARPS + GatherCfg<PB>::KPAR * (PB / 32))) pkm_ws_kernel(WsParams p) {
    constexpr int NGATH = GatherCfg<PB>::NGATH;
    constexpr int ROLE_WARPS = GatherCfg<PB>::ROLE_WARPS;
    constexpr int CH = PB / 16;          // 16-byte chunks per row part
    constexpr int NSL = PB / 32;         // column slices of 16 columns; KPAR warps per slice take turns by step
    constexpr int KPAR = GatherCfg<PB>::KPAR;
    constexpr int RS = PB + 16;          // padded row stride: conflict-free ldmatrix / 16-byte accesses
    constexpr int R = 2 * D;
    constexpr int SLOT = 64 * RS;

    extern __shared__ __align__(128) uint8_t smem[];
    const SmemLayout SL = smem_layout(PB, D, p.A, p.Dh);
    const MetaLayout ML = meta_layout(p.A, p.Dh);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL.bars);   // [R] rows of step landed
    uint64_t* done = full + R;                                      // [R] every slice finished the step
    uint64_t* rready = done + R;                                    // [R] every slice's r of the step written
    uint64_t* mfull = rready + R;                                   // [NC] metadata chunk landed
    uint64_t* mfree = mfull + NC;                                   // [NC] chunk's last step done by every warp
    uint64_t* mready = mfree + NC;                                  // [NC] chunk's row-address table written
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SL.misc);
    uint8_t* rows = smem + SL.rows;
    uint8_t* zrow = smem + SL.zrow;
    float* rbuf = reinterpret_cast<float*>(smem + SL.rbuf);        // [R][PB / 2] r of the step's columns
    uint8_t* ystage = smem + SL.ystage;
    uint8_t* meta = smem + SL.meta;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lane_bh = blockIdx.y, part = blockIdx.x;
    const int A = p.A, Dh = p.Dh, T_ = p.T;
    const int64_t lt0 = (int64_t)lane_bh * p.lstride + p.tbase;   // this lane's first step of the piece
    const int64_t row_bytes = (int64_t)Dh * 2;
    const int nchunks = (T_ + CHS - 1) / CHS;
    uint8_t* gstate = reinterpret_cast<uint8_t*>(p.state) + (int64_t)lane_bh * p.total * row_bytes + (int64_t)part * PB;

    for (int i = tid; i < RS / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(zrow)[i] = 0u;
    if (tid == 0) {
        for (int i = 0; i < R; ++i) {
            tc::mbar_init(full + i, 2 * NGATH);
            tc::mbar_init(done + i, NSL * 32);
            tc::mbar_init(rready + i, NSL);
        }
        for (int i = 0; i < NC; ++i) {
            tc::mbar_init(mfull + i, NLOAD);
            tc::mbar_init(mfree + i, KPAR * NSL * 32);
            tc::mbar_init(mready + i, 1);
        }
        *abort_flag = 0;
    }
    __syncthreads();

    if (warp == 0) {
        // =============================== loader ===============================
        const T* gwk = static_cast<const T*>(p.wk);
        const T* gwq = static_cast<const T*>(p.wq);
        const T* gv = static_cast<const T*>(p.v);
        const T* gbeta = static_cast<const T*>(p.beta);
        const T* gdecay = static_cast<const T*>(p.decay);
        auto copy = [&](uint8_t* dst, const void* src, int nbytes) {
            const uint32_t d0 = tc::smem_u32(dst);
            const uint8_t* s0 = static_cast<const uint8_t*>(src);
            for (int i = lane; i < nbytes / 16; i += NLOAD) cp_async16(d0 + 16 * i, s0 + 16 * i);
        };
        auto load_chunk = [&](int c) {
            const int t0 = c * CHS;
            const int n = min(CHS, T_ - t0);              // a multiple of 8
            uint8_t* mc = meta + (c % NC) * ML.bytes;
            const int64_t bt = lt0 + t0;
            copy(mc + ML.idx, p.idx + bt * A, n * A * 8);
            copy(mc + ML.wk, gwk + bt * A, n * A * 2);
            copy(mc + ML.wq, gwq + bt * A, n * A * 2);
            copy(mc + ML.v, gv + bt * Dh, n * Dh * 2);
            copy(mc + ML.beta, gbeta + bt, n * 2);
            if (p.dynamic_decay) copy(mc + ML.alpha, gdecay + bt, n * 2);
            copy(mc + ML.code, p.codes + bt * 64, n * 128);
            cp_async_arrive_noinc(mfull + (c % NC));
        };
        // once chunk c has landed: each row's shared address for the GEMV and the update
        // (its own ring row, the forwarding writer's row, or the zero row with bit 0 set
        // when there is no row) and each step's forwarding distances, so that the step
        // warps read one word instead of decoding the code
        const uint32_t rows_u = tc::smem_u32(rows), zrow_u = tc::smem_u32(zrow);
        auto table = [&](int c) -> bool {
            const bool ok = ws_wait(mfull + (c % NC), (c / NC) & 1, abort_flag, p.status, p.wait_ns);
            if (!__all_sync(DG_FULL_MASK, ok)) return false;
            uint8_t* mc = meta + (c % NC) * ML.bytes;
            const int t0 = c * CHS, n = min(CHS, T_ - t0);
            const int16_t* code = reinterpret_cast<const int16_t*>(mc + ML.code);
            uint32_t* addr = reinterpret_cast<uint32_t*>(mc + ML.addr);
            uint32_t* dmask = reinterpret_cast<uint32_t*>(mc + ML.dmask);
            for (int ts = 0; ts < n; ++ts) {
                const int t = t0 + ts;
                uint32_t dm = 0;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int m = lane + 32 * h;
                    const int cd = code[ts * 64 + m];
                    uint32_t a;
                    if (cd >= 0) {
                        const int w = t - (cd >> 6);
                        a = rows_u + (uint32_t)((w % R) * SLOT + (cd & 63) * RS);
                        dm |= 1u << (cd >> 6);
                    } else {
                        a = cd == -1 ? rows_u + (uint32_t)((t % R) * SLOT + m * RS) : (zrow_u | 1u);
                    }
                    addr[ts * 64 + m] = a;
                }
                dm = __reduce_or_sync(DG_FULL_MASK, dm);
                if (lane == 0) dmask[ts] = dm;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(mready + (c % NC));
            return true;
        };
        load_chunk(0);
        if (nchunks > 1) load_chunk(1);
        bool tok = nchunks > 0 ? table(0) : true;
        for (int c = 0; c + 1 < nchunks && tok; ++c) {
            tok = table(c + 1);
            if (!tok) break;
            if (c + 2 < nchunks) {
                // chunk c+2 reuses the buffer of chunk c-1
                if (c >= 1) {
                    const bool ok = ws_wait(mfree + ((c - 1) % NC), ((c - 1) / NC) & 1, abort_flag, p.status, p.wait_ns);
                    if (!__all_sync(DG_FULL_MASK, ok)) break;
                }
                load_chunk(c + 2);
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp < ROLE_WARPS) {
        // =============================== gather ===============================
        const int gt = tid - 32;                          // 0 .. NGATH-1
        for (int t = 0; t < T_; ++t) {
            const int sl = t % R;
            const int c = t / CHS, ts = t % CHS;
            bool ok = true;
            if (ts == 0) ok = ws_wait(mready + (c % NC), (c / NC) & 1, abort_flag, p.status, p.wait_ns);
            if (ok && t >= D) ok = ws_wait(done + ((t - D) % R), ((t - D) / R) & 1, abort_flag, p.status, p.wait_ns);
            if (!ok) break;
            const uint8_t* mc = meta + (c % NC) * ML.bytes;
            const int64_t* midx = reinterpret_cast<const int64_t*>(mc + ML.idx) + ts * A;
            const int16_t* code = reinterpret_cast<const int16_t*>(mc + ML.code) + ts * 64;
            const uint32_t slot = tc::smem_u32(rows + sl * SLOT);
            // every (row, chunk) gets a copy; rows not coded "gather" copy 0 bytes
            // (their ring row is zero-filled and rewritten by the update before any read).
            // Addresses first, in plain code, so their shared-memory loads overlap.
            constexpr int GPT = CH * 64 / NGATH;             // copies per gather thread per step
            const uint8_t* src[GPT];
            uint32_t nb[GPT];
#pragma unroll
            for (int j = 0; j < GPT; ++j) {
                const int m = (j * NGATH + gt) / CH, cc = (j * NGATH + gt) % CH;
                const bool gath = code[m] == -1;
                const int64_t xm = midx[min(m, A - 1)];
                src[j] = gstate + (gath ? xm : 0) * row_bytes + 16 * cc;
                nb[j] = gath ? 16u : 0u;
            }
#pragma unroll
            for (int j = 0; j < GPT; ++j) {
                const int m = (j * NGATH + gt) / CH, cc = (j * NGATH + gt) % CH;
                cp_async16_zfill(slot + m * RS + 16 * cc, src[j], nb[j]);
            }
            cp_async_arrive_noinc(full + sl);
            mbar_arrive(full + sl);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
        // ============================== step warps ==============================
        // The NSL warps of a step (one par group) split it twice: the GEMV by 16-column
        // slices (warp q: columns 16q .. 16q+15 of the part, all 64 rows), then, once every
        // slice's r is in shared memory, the update by rows (warp q: rows q RW .. q RW +
        // RW - 1, whole row parts), so that each row is stored to global memory as whole
        // 16-byte chunks of one row part per lane group (LPR lanes a row).
        constexpr int LPR = CH;                                // lanes per row part (16-byte chunks)
        constexpr int RPI = 32 / LPR;                          // rows per update instruction
        constexpr int RW = 64 / NSL;                           // rows per warp in the update
        static_assert(RW == 4 * RPI, "four update iterations per warp");
        const int sw = warp - ROLE_WARPS;                      // 0 .. KPAR*NSL-1
        const int q = sw % NSL;                                // GEMV slice and update row block
        const int par = sw / NSL;                              // steps s with s % KPAR == par
        const int g = lane >> 2, tig = lane & 3;
        const int kk = ((lane >> 4) & 1) * 8 + (lane & 7);     // ldmatrix row of this lane in a K block
        const uint32_t colb = (uint32_t)(q * 32 + ((lane >> 3) & 1) * 16);
        const int ur = lane / LPR, uc = lane % LPR;            // update: rows q RW + ur + RPI i, chunk uc
        const uint32_t rows_u = tc::smem_u32(rows);
        const uint32_t zrow_u = tc::smem_u32(zrow);
        T* gout = static_cast<T*>(p.out);
        const float alpha_static = p.dynamic_decay ? 1.f : dg::to_f(static_cast<const T*>(p.decay)[lane_bh % p.H]);
        // Two copies of the step loop.  With 128-byte parts (one CTA a lane, 15 warps)
        // each step reads its GEMV's weights and row addresses before waiting for its
        // forwarding writers, and its update's operands before waiting for the other
        // slices' r.  With 64-byte parts the loop is kept as it was: the early reads, and
        // even the restructured code around them, measured slower there.
        if constexpr (PB == 128) {
            for (int s = par; s < T_; s += KPAR) {
                const int sl = s % R;
                const int cn = s / CHS, ts = s % CHS;
                const uint8_t* mc = meta + (cn % NC) * ML.bytes;
                bool ok = ws_wait(full + sl, (s / R) & 1, abort_flag, p.status, p.wait_ns);
                if (!__all_sync(DG_FULL_MASK, ok)) break;
                const uint32_t* raddr = reinterpret_cast<const uint32_t*>(mc + ML.addr) + ts * 64;
                // ---- GEMV: y and pred of the slice's 16 columns; its weights and row addresses,
                // and the step's beta and v for r, are read before any wait for a forwarding
                // writer ----
                const float bta = dg::to_f(reinterpret_cast<const T*>(mc + ML.beta)[ts]);
                const T* mv = reinterpret_cast<const T*>(mc + ML.v) + ts * Dh + part * (PB / 2);
                const float v0 = dg::to_f(mv[q * 16 + g]), v8 = dg::to_f(mv[q * 16 + g + 8]);
                const uint32_t* wsrc = reinterpret_cast<const uint32_t*>(
                    reinterpret_cast<const uint16_t*>(mc + (g == 0 ? ML.wq : ML.wk)) + ts * A);
                const bool bl = g < 2;
                const int nkb = A >> 4;
                uint32_t b[4][2], base[4];
#pragma unroll
                for (int kb = 0; kb < 4; ++kb) {
                    const int kc = min(kb, nkb - 1);                  // in-bounds for every lane; unused blocks skipped below
                    const uint32_t w0 = wsrc[kc * 8 + tig];
                    const uint32_t w1 = wsrc[kc * 8 + 4 + tig];
                    b[kb][0] = bl ? w0 : 0u;
                    b[kb][1] = bl ? w1 : 0u;
                    const int k = kc * 16 + kk;
                    base[kb] = (raddr[k] & ~15u) + colb;
                }
                // rows forwarded from an earlier step in the window: that step's update (by all
                // of its warps, whatever rows each took) must have finished
                {
                    uint32_t dm = reinterpret_cast<const uint32_t*>(mc + ML.dmask)[ts];
                    while (dm != 0u && ok) {
                        const int d = __ffs(dm) - 1;
                        dm &= dm - 1;
                        const int w = s - d;
                        ok = ws_wait(done + (w % R), (w / R) & 1, abort_flag, p.status, p.wait_ns);
                        ok = __all_sync(DG_FULL_MASK, ok);
                    }
                    if (!ok) break;
                }
                uint32_t a[4][4];
#pragma unroll
                for (int kb = 0; kb < 4; ++kb)
                    if (kb < nkb) ldsm_x4_trans(base[kb], a[kb][0], a[kb][1], a[kb][2], a[kb][3]);
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int kb = 0; kb < 4; ++kb)
                    if (kb < nkb) MmaOp<T>::run(acc, a[kb], b[kb][0], b[kb][1]);
                // lanes with tig == 0: acc = {y, pred} of column g and {y, pred} of column g + 8
                float* rstep = rbuf + sl * (PB / 2);
                if (tig == 0) {
                    const int col0 = q * 16 + g;                   // column within the part
                    // y rows are staged per chunk parity: the same row of the next chunk may
                    // belong to another warp of the slice (KPAR need not divide CHS), which can
                    // be up to D < CHS steps ahead of this warp's flush
                    T* yrow = reinterpret_cast<T*>(ystage + ((cn & 1) * CHS + ts) * PB);
                    yrow[col0] = dg::from_f<T>(acc[0]);
                    yrow[col0 + 8] = dg::from_f<T>(acc[2]);
                    rstep[col0] = bta * (v0 - acc[1]);
                    rstep[col0 + 8] = bta * (v8 - acc[3]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(rready + sl);
                // ---- update: whole row parts, new rows (fp32, one rounding) to the ring slot
                // and to global memory.  Its rows, indices and weights do not depend on the
                // barrier (which orders only r, and the row writes after every slice's GEMV
                // reads): they are read while the other slices finish ----
                const float al = p.dynamic_decay ? dg::to_f(reinterpret_cast<const T*>(mc + ML.alpha)[ts]) : alpha_static;
                const unsigned long long al2 = f2pack(al, al);
                const int64_t* midx = reinterpret_cast<const int64_t*>(mc + ML.idx) + ts * A;
                const T* mwk = reinterpret_cast<const T*>(mc + ML.wk) + ts * A;
                uint8_t* slot = rows + sl * SLOT;
                int ucd[4];
                int64_t ux[4];
                float uwk[4];
                uint4 uraw[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = q * RW + ur + RPI * i;           // rows >= A carry code -2 and are skipped
                    const int mcl = min(m, A - 1);
                    const uint32_t a = raddr[m];
                    const uint32_t src = a & ~15u;
                    ucd[i] = (a & 1u) ? -2 : 0;
                    ux[i] = midx[mcl];
                    uwk[i] = dg::to_f(mwk[mcl]);
                    uraw[i] = *reinterpret_cast<const uint4*>(rows + (src - rows_u) + uc * 16);
                }
                ok = ws_wait(rready + sl, (s / R) & 1, abort_flag, p.status, p.wait_ns);
                if (!__all_sync(DG_FULL_MASK, ok)) break;
                const float4 ra = reinterpret_cast<const float4*>(rstep + uc * 8)[0];
                const float4 rb = reinterpret_cast<const float4*>(rstep + uc * 8)[1];
                const float br[8] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = q * RW + ur + RPI * i;
                    // rows as gathered (zeros for an index out of range: its ring row was zero-filled)
                    if (p.saved != nullptr && m < A)
                        dg::st16(static_cast<uint8_t*>(p.saved) + ((lt0 + s) * A + m) * row_bytes + part * PB + uc * 16,
                                 uraw[i]);
                    if (ucd[i] == -2) continue;
                    const uint32_t in[4] = {uraw[i].x, uraw[i].y, uraw[i].z, uraw[i].w};
                    uint32_t o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 sv = unpack2(in[e], T());
                        const unsigned long long u = mul_f32x2(f2pack(br[2 * e], br[2 * e + 1]), f2pack(uwk[i], uwk[i]));
                        const float2 nv = f2unpack(fma_f32x2(al2, f2pack(sv.x, sv.y), u));
                        o[e] = pack2(nv.x, nv.y, T());
                    }
                    const uint4 nv4 = make_uint4(o[0], o[1], o[2], o[3]);
                    *reinterpret_cast<uint4*>(slot + m * RS + uc * 16) = nv4;
                    dg::st16(gstate + ux[i] * row_bytes + uc * 16, nv4);
                }
                __syncwarp();
                mbar_arrive(done + sl);
                const int t0c = s - ts;
                const int cend = min(t0c + CHS, T_);
                if (s + KPAR >= cend) {                           // this warp's last step of the chunk
                    mbar_arrive(mfree + (cn % NC));
                    // this warp's y columns of the chunk: steps s = par (mod KPAR), i.e. rows j0, j0 + KPAR, ...
                    const int j0 = ((par - t0c) % KPAR + KPAR) % KPAR;
                    const int nj = (cend - t0c - j0 + KPAR - 1) / KPAR;
                    for (int i = lane; i < 2 * nj; i += 32) {
                        const int jj = j0 + KPAR * (i >> 1), hh = i & 1;
                        const uint4 val = *reinterpret_cast<const uint4*>(ystage + ((cn & 1) * CHS + jj) * PB + q * 32 + hh * 16);
                        dg::st16(reinterpret_cast<uint8_t*>(gout + (lt0 + t0c + jj) * Dh) + part * PB + q * 32 + hh * 16,
                                 val);
                    }
                    __syncwarp();
                }
            }
        } else {
            for (int s = par; s < T_; s += KPAR) {
                const int sl = s % R;
                const int cn = s / CHS, ts = s % CHS;
                const uint8_t* mc = meta + (cn % NC) * ML.bytes;
                bool ok = ws_wait(full + sl, (s / R) & 1, abort_flag, p.status, p.wait_ns);
                if (!__all_sync(DG_FULL_MASK, ok)) break;
                const uint32_t* raddr = reinterpret_cast<const uint32_t*>(mc + ML.addr) + ts * 64;
                // rows forwarded from an earlier step in the window: that step's update (by all
                // of its warps, whatever rows each took) must have finished
                {
                    uint32_t dm = reinterpret_cast<const uint32_t*>(mc + ML.dmask)[ts];
                    while (dm != 0u && ok) {
                        const int d = __ffs(dm) - 1;
                        dm &= dm - 1;
                        const int w = s - d;
                        ok = ws_wait(done + (w % R), (w / R) & 1, abort_flag, p.status, p.wait_ns);
                        ok = __all_sync(DG_FULL_MASK, ok);
                    }
                    if (!ok) break;
                }
                // ---- GEMV: y and pred of the slice's 16 columns ----
                const uint32_t* wsrc = reinterpret_cast<const uint32_t*>(
                    reinterpret_cast<const uint16_t*>(mc + (g == 0 ? ML.wq : ML.wk)) + ts * A);
                const bool bl = g < 2;
                const int nkb = A >> 4;
                uint32_t b[4][2], base[4];
#pragma unroll
                for (int kb = 0; kb < 4; ++kb) {
                    const int kc = min(kb, nkb - 1);                  // in-bounds for every lane; unused blocks skipped below
                    const uint32_t w0 = wsrc[kc * 8 + tig];
                    const uint32_t w1 = wsrc[kc * 8 + 4 + tig];
                    b[kb][0] = bl ? w0 : 0u;
                    b[kb][1] = bl ? w1 : 0u;
                    const int k = kc * 16 + kk;
                    base[kb] = (raddr[k] & ~15u) + colb;
                }
                uint32_t a[4][4];
#pragma unroll
                for (int kb = 0; kb < 4; ++kb)
                    if (kb < nkb) ldsm_x4_trans(base[kb], a[kb][0], a[kb][1], a[kb][2], a[kb][3]);
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int kb = 0; kb < 4; ++kb)
                    if (kb < nkb) MmaOp<T>::run(acc, a[kb], b[kb][0], b[kb][1]);
                // lanes with tig == 0: acc = {y, pred} of column g and {y, pred} of column g + 8
                float* rstep = rbuf + sl * (PB / 2);
                if (tig == 0) {
                    const int col0 = q * 16 + g;                   // column within the part
                    const float bta = dg::to_f(reinterpret_cast<const T*>(mc + ML.beta)[ts]);
                    const T* mv = reinterpret_cast<const T*>(mc + ML.v) + ts * Dh + part * (PB / 2);
                    // y rows are staged per chunk parity: the same row of the next chunk may
                    // belong to another warp of the slice (KPAR need not divide CHS), which can
                    // be up to D < CHS steps ahead of this warp's flush
                    T* yrow = reinterpret_cast<T*>(ystage + ((cn & 1) * CHS + ts) * PB);
                    yrow[col0] = dg::from_f<T>(acc[0]);
                    yrow[col0 + 8] = dg::from_f<T>(acc[2]);
                    rstep[col0] = bta * (dg::to_f(mv[col0]) - acc[1]);
                    rstep[col0 + 8] = bta * (dg::to_f(mv[col0 + 8]) - acc[3]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(rready + sl);
                ok = ws_wait(rready + sl, (s / R) & 1, abort_flag, p.status, p.wait_ns);
                if (!__all_sync(DG_FULL_MASK, ok)) break;
                // ---- update: whole row parts, new rows (fp32, one rounding) to the ring slot
                // and to global memory ----
                const float4 ra = reinterpret_cast<const float4*>(rstep + uc * 8)[0];
                const float4 rb = reinterpret_cast<const float4*>(rstep + uc * 8)[1];
                const float br[8] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
                const float al = p.dynamic_decay ? dg::to_f(reinterpret_cast<const T*>(mc + ML.alpha)[ts]) : alpha_static;
                const unsigned long long al2 = f2pack(al, al);
                const int64_t* midx = reinterpret_cast<const int64_t*>(mc + ML.idx) + ts * A;
                const T* mwk = reinterpret_cast<const T*>(mc + ML.wk) + ts * A;
                uint8_t* slot = rows + sl * SLOT;
                int ucd[4];
                int64_t ux[4];
                float uwk[4];
                uint4 uraw[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = q * RW + ur + RPI * i;           // rows >= A carry code -2 and are skipped
                    const int mcl = min(m, A - 1);
                    const uint32_t a = raddr[m];
                    const uint32_t src = a & ~15u;
                    ucd[i] = (a & 1u) ? -2 : 0;
                    ux[i] = midx[mcl];
                    uwk[i] = dg::to_f(mwk[mcl]);
                    uraw[i] = *reinterpret_cast<const uint4*>(rows + (src - rows_u) + uc * 16);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = q * RW + ur + RPI * i;
                    // rows as gathered (zeros for an index out of range: its ring row was zero-filled)
                    if (p.saved != nullptr && m < A)
                        dg::st16(static_cast<uint8_t*>(p.saved) + ((lt0 + s) * A + m) * row_bytes + part * PB + uc * 16,
                                 uraw[i]);
                    if (ucd[i] == -2) continue;
                    const uint32_t in[4] = {uraw[i].x, uraw[i].y, uraw[i].z, uraw[i].w};
                    uint32_t o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 sv = unpack2(in[e], T());
                        const unsigned long long u = mul_f32x2(f2pack(br[2 * e], br[2 * e + 1]), f2pack(uwk[i], uwk[i]));
                        const float2 nv = f2unpack(fma_f32x2(al2, f2pack(sv.x, sv.y), u));
                        o[e] = pack2(nv.x, nv.y, T());
                    }
                    const uint4 nv4 = make_uint4(o[0], o[1], o[2], o[3]);
                    *reinterpret_cast<uint4*>(slot + m * RS + uc * 16) = nv4;
                    dg::st16(gstate + ux[i] * row_bytes + uc * 16, nv4);
                }
                __syncwarp();
                mbar_arrive(done + sl);
                const int t0c = s - ts;
                const int cend = min(t0c + CHS, T_);
                if (s + KPAR >= cend) {                           // this warp's last step of the chunk
                    mbar_arrive(mfree + (cn % NC));
                    // this warp's y columns of the chunk: steps s = par (mod KPAR), i.e. rows j0, j0 + KPAR, ...
                    const int j0 = ((par - t0c) % KPAR + KPAR) % KPAR;
                    const int nj = (cend - t0c - j0 + KPAR - 1) / KPAR;
                    for (int i = lane; i < 2 * nj; i += 32) {
                        const int jj = j0 + KPAR * (i >> 1), hh = i & 1;
                        const uint4 val = *reinterpret_cast<const uint4*>(ystage + ((cn & 1) * CHS + jj) * PB + q * 32 + hh * 16);
                        dg::st16(reinterpret_cast<uint8_t*>(gout + (lt0 + t0c + jj) * Dh) + part * PB + q * 32 + hh * 16,
                                 val);
                    }
                    __syncwarp();
                }
            }
        }
    }
}

constexpr int kDepthFull = 8;     // window depth for 128-byte row parts (ring of 16 slots)
constexpr int kDepthHalf = 12;    // for 64-byte row parts (ring of 24 slots)
static_assert(kDepthFull <= HZ_MAXWIN && kDepthHalf <= HZ_MAXWIN, "window depth covered by the pre-pass");
// y staging by chunk parity: a row of chunk c+2 is written no earlier than D steps after
// step t0(c)+32-D finished, which is after the owning warp flushed chunk c when D + KPAR <= CHS + 1
static_assert(kDepthFull + GatherCfg<128>::KPAR <= CHS + 1 && kDepthHalf + GatherCfg<64>::KPAR <= CHS + 1,
              "y staging depth");

// row part bytes for a call: 128 (full 64-column fp16 rows), or 64 (two CTAs per lane)
int ws_part_bytes(int B, int H, int Dh) {
    const int rb = Dh * 2;
    const int lanes = B * H;
    if (rb == 128) return lanes < 120 ? 64 : 128;
    if (rb == 64) return 64;
    if (rb == 256) return 128;
    return 0;
}

template <typename T, int PB, int D>
int launch_ws(const WsParams& p, int lanes, cudaStream_t stream) {
    const SmemLayout SL = smem_layout(PB, D, p.A, p.Dh);
    auto kern = pkm_ws_kernel<T, PB, D>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SL.total);
    if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    dim3 grid(p.parts, lanes);
    kern<<<grid, 32 * (GatherCfg<PB>::ROLE_WARPS + GatherCfg<PB>::KPAR * (PB / 32)), SL.total, stream>>>(p);
    return dg_host::check_launch();
}

}  // namespace

namespace dg_host {

uint32_t wait_limit();

size_t pkm_ws_workspace_bytes(int B, int H, int T) { return (size_t)B * H * T * 64 * sizeof(int16_t); }

bool pkm_ws_supports(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v, const void* beta,
                     const void* wk, const void* wq, const void* idx, const void* decay, int dynamic_decay,
                     const void* state, const void* saved) {
    if (dtype != DG_DTYPE_F16 && dtype != DG_DTYPE_BF16) return false;
    if (A < 16 || A > MAXA || A % 16 != 0 || T < 1 || T % 8 != 0) return false;   // whole 16-row MMA blocks
    if (total >= (int64_t)0x7fffffff - 1 || T >= (1 << 25)) return false;
    const int PB = ws_part_bytes(B, H, Dh);
    if (PB == 0) return false;
    const int D = PB == 128 ? kDepthFull : kDepthHalf;
    if (smem_layout(PB, D, A, Dh).total > 232448) return false;
    const uintptr_t al = (uintptr_t)v | (uintptr_t)beta | (uintptr_t)wk | (uintptr_t)wq | (uintptr_t)idx |
                         (uintptr_t)state | (dynamic_decay ? (uintptr_t)decay : 0) | (uintptr_t)saved;
    return (al & 15) == 0;
}

namespace {

// the pipelined call's streams and events, one set per device, created on first use
struct SideStreams {
    cudaStream_t pre = nullptr, rec = nullptr;   // pre-pass (lowest priority), recurrence (highest)
    cudaEvent_t fork = nullptr, join = nullptr, ready[4] = {};
};
SideStreams g_side[64];
std::mutex g_side_mu;

int side_streams(int dev, SideStreams** out) {
    SideStreams& ss = g_side[dev];
    if (!ss.pre) {
        int least = 0, greatest = 0;
        cudaError_t e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
        if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&ss.pre, cudaStreamNonBlocking, least);
        if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&ss.rec, cudaStreamNonBlocking, greatest);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming);
        for (int i = 0; i < 4 && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&ss.ready[i], cudaEventDisableTiming);
        if (e != cudaSuccess) {
            ss = SideStreams{};            // (a partial set is not reused; its handles are dropped)
            return dg_host::record_cuda_error(e);
        }
    }
    *out = &ss;
    return DG_OK;
}

}  // namespace

// workspace: pkm_ws_workspace_bytes(B, H, T) bytes, 16-byte aligned
int pkm_forward_ws(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v, const void* beta,
                   const void* wk, const void* wq, const int64_t* idx, const void* decay, int dynamic_decay,
                   void* state, void* out, void* saved, int32_t* status, void* workspace, cudaStream_t stream) {
    const int PB = ws_part_bytes(B, H, Dh);
    const int parts = Dh * 2 / PB;
    const int D = PB == 128 ? kDepthFull : kDepthHalf;
    const int lanes = B * H;
    int16_t* codes = static_cast<int16_t*>(workspace);
    const int hz_smem = (2 * HZ_BUCKETS + 32) * 4 + HZ_ENTRIES * 8;
    auto hz = A == 16 ? pkm_hazard_kernel<16> : A == 32 ? pkm_hazard_kernel<32> : A == 48 ? pkm_hazard_kernel<48>
                                                                                         : pkm_hazard_kernel<64>;
    cudaError_t e = cudaFuncSetAttribute(hz, cudaFuncAttributeMaxDynamicSharedMemorySize, hz_smem);
    if (e != cudaSuccess) return record_cuda_error(e);
    // the default poll budget (2^22) maps to 2 s of waiting; 0 gives up at once
    const uint64_t wait_ns = (uint64_t)wait_limit() * 2000000000ull / (1ull << 22);
    auto prepass = [&](int t0, int n, cudaStream_t s) -> int {
        const dim3 hz_grid((n + HZ_STEPS - 1) / HZ_STEPS, lanes);
        hz<<<hz_grid, HZ_THREADS, hz_smem, s>>>(idx, codes, status, n, total, D, (int64_t)T, t0);
        return check_launch();
    };
    auto recurrence = [&](int t0, int n, cudaStream_t s) -> int {
        WsParams p{v, beta, wk, wq, idx, decay, state, out, status, H, n, A, Dh, parts, total, dynamic_decay, codes,
                   saved, wait_ns, (int64_t)T, t0};
        if (dtype == DG_DTYPE_F16)
            return PB == 128 ? launch_ws<__half, 128, kDepthFull>(p, lanes, s)
                             : launch_ws<__half, 64, kDepthHalf>(p, lanes, s);
        if (dtype == DG_DTYPE_BF16)
            return PB == 128 ? launch_ws<__nv_bfloat16, 128, kDepthFull>(p, lanes, s)
                             : launch_ws<__nv_bfloat16, 64, kDepthHalf>(p, lanes, s);
        return DG_ERR_UNSUPPORTED;
    };
    // pipelined when the sequence is long and the recurrence leaves SMs free for the
    // pre-pass (its CTAs and the recurrence's do not share an SM)
    int dev = 0, sms = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e);
    int rc = sm_count(dev, &sms);
    if (rc != DG_OK) return rc;
    constexpr int NP = 4;
    const bool pipelined = T >= 1024 && T % (NP * 8) == 0 && lanes * parts + 8 <= sms && dev >= 0 && dev < 64;
    std::unique_lock<std::mutex> lock(g_side_mu, std::defer_lock);   // the device's events are reused call after call
    SideStreams* ss = nullptr;
    if (pipelined) {
        lock.lock();
        // the side streams are made on the device's first pipelined call; a first call
        // made while the caller's stream is capturing runs unpipelined instead
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        e = cudaStreamIsCapturing(stream, &cs);
        if (e != cudaSuccess) return record_cuda_error(e);
        if (g_side[dev].pre || cs == cudaStreamCaptureStatusNone) {
            rc = side_streams(dev, &ss);
            if (rc != DG_OK) return rc;
        }
    }
    if (!ss) {
        rc = prepass(0, T, stream);
        return rc != DG_OK ? rc : recurrence(0, T, stream);
    }
    const int L = T / NP;                             // a multiple of 8
    // fork: both side streams follow the work already on the caller's stream
    e = cudaEventRecord(ss->fork, stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ss->pre, ss->fork, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ss->rec, ss->fork, 0);
    if (e != cudaSuccess) return record_cuda_error(e);
    for (int i = 0; i < NP && rc == DG_OK; ++i) {
        rc = prepass(i * L, L, ss->pre);
        if (rc != DG_OK) break;
        e = cudaEventRecord(ss->ready[i], ss->pre);
        if (e != cudaSuccess) { rc = record_cuda_error(e); break; }
    }
    for (int i = 0; i < NP && rc == DG_OK; ++i) {
        e = cudaStreamWaitEvent(ss->rec, ss->ready[i], 0);
        if (e != cudaSuccess) { rc = record_cuda_error(e); break; }
        rc = recurrence(i * L, L, ss->rec);
    }
    // join: the caller's stream follows both side streams, whatever happened above
    e = cudaEventRecord(ss->fork, ss->pre);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, ss->fork, 0);
    if (e == cudaSuccess) e = cudaEventRecord(ss->join, ss->rec);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, ss->join, 0);
    if (rc != DG_OK) return rc;
    return e == cudaSuccess ? DG_OK : record_cuda_error(e);
}

}  // namespace dg_host
