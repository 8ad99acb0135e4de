// pkm_pipe.cu -- pipelined Sparse Delta-PKM recurrence with exact hazard forwarding.
//
// Same math as pkm_seq.cu (src/cpp/delta_kernel.cu:885-920): per lane and step,
// gather the `active` rows S[idx_t], y = wq.s, r = v - wk.s, scatter
// S[idx_t] = cast(alpha s + (beta r) wk), rows rounded to the storage dtype
// every step.
//
// Steps depend on each other only through shared rows, and every step's slot
// indices are inputs (state-independent), so rows can be fetched D steps ahead:
//   - one CTA per (lane, part of the row); CW column-slice warps own 16-byte
//     column slices as in pkm_seq.cu, plus two scheduler warps;
//   - at iteration s the column warps consume step s from a shared-memory row
//     ring (filled by cp.async issued at iteration s - D) and issue the copies
//     for step s + D after the iteration barrier, which orders all stores of
//     steps <= s before those copies;
//   - the scheduler fetches per-step metadata (idx, wk, wq, v, beta, alpha)
//     2D steps ahead and, for step s + D, finds for every row the most recent
//     earlier step in the window [s+1, s+D-1] that wrote the same slot (whose
//     store the copy cannot see).  Such rows are not fetched; the consumer takes
//     them from the writer's ring slot, which holds the rounded values it stored.
//     The lookup uses a shared 8-way set-associative table slot -> (step,
//     position) whose entries expire by step stamp; inserts use 64-bit CAS.  If
//     a bucket holds 8 live other slots the table overflows: the next D steps
//     then reload their rows synchronously from global memory (exact, slower).
// The per-step dependency chain is the warp reduction; memory latency is
// hidden by the D steps in flight.
#include "dg_common.cuh"

namespace {

constexpr int MAXA = 64;                 // active rows per step handled here
constexpr int WAYS = 8;                  // hash table: 512 buckets x 8 cells (one 64-byte bucket per key)
constexpr int NBUCKET = 512;
constexpr int HSIZE = NBUCKET * WAYS;

struct PipeParams {
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
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t slot_bucket(uint32_t x) { return (x * 2654435761u) >> 23; }   // 9 bits

template <int NV>
struct Log2v { static constexpr int v = (NV <= 1) ? 0 : 1 + Log2v<NV / 2>::v; };

// Sums vals[] over the warp; returns on each lane the total of value (lane >> (5 - log2 NV)).
template <int NV>
__device__ __forceinline__ float reduce_scatter(float (&vals)[NV], int lane) {
    constexpr int LOG = Log2v<NV>::v;
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

// per-step metadata slot: idx int64[64] | wk T[64] | wq T[64] | v (one row) | fwd int16[64]
__host__ __device__ constexpr int meta_bytes(int esz, int row_bytes) {
    return ((512 + 2 * MAXA * esz + row_bytes + 2 * MAXA) + 15) / 16 * 16;
}

template <typename T, int D>
__global__ void __launch_bounds__(576) pkm_pipe_kernel(PipeParams p) {
    using V = dg::Vec16<T>;
    constexpr int CPW = V::N;
    constexpr int NV = 2 * CPW;
    constexpr int DUP = 5 - Log2v<NV>::v;
    constexpr int RR = 2 * D;            // row ring: steps [s-D+1, s+D]
    constexpr int MR = 2 * D + 1;        // meta ring: steps [s, s+2D]
    constexpr int BR = 4 * D + 16;       // beta/alpha ring (steps), filled 16 bytes at a time
    constexpr int EPB = 16 / sizeof(T);  // beta values per 16-byte block

    extern __shared__ __align__(16) uint8_t smem[];
    const int CW = blockDim.x / 32 - 2;               // column-slice warps
    const int part_bytes = p.Dh * (int)sizeof(T) / p.parts;
    const int row_stride = part_bytes + 16;           // padded: conflict-free 16-byte slices
    const int slot_bytes = MAXA * row_stride;
    const int META = meta_bytes((int)sizeof(T), p.Dh * (int)sizeof(T));
    uint8_t* rows = smem;                              // [RR][MAXA][row_stride]
    uint8_t* meta = rows + RR * slot_bytes;            // [MR][META]
    T* bring = reinterpret_cast<T*>(meta + MR * META); // beta ring [BR]
    T* aring = bring + BR;                             // alpha ring [BR]
    unsigned long long* tbl = reinterpret_cast<unsigned long long*>(
        (reinterpret_cast<uintptr_t>(aring + BR) + 15) & ~uintptr_t(15));
    int* sync_until = reinterpret_cast<int*>(tbl + HSIZE);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lane_bh = blockIdx.y, part = blockIdx.x;
    const int h = lane_bh % p.H;
    const int A = p.A, Dh = p.Dh, T_ = p.T;
    const int64_t total = p.total;
    const int64_t lt0 = (int64_t)lane_bh * T_;
    const T* __restrict__ gv = static_cast<const T*>(p.v);
    const T* __restrict__ gbeta = static_cast<const T*>(p.beta);
    const T* __restrict__ gwk = static_cast<const T*>(p.wk);
    const T* __restrict__ gwq = static_cast<const T*>(p.wq);
    const T* __restrict__ gdecay = static_cast<const T*>(p.decay);
    uint8_t* gstate = reinterpret_cast<uint8_t*>(p.state) + ((int64_t)lane_bh * total * Dh) * (int64_t)sizeof(T) +
                      (int64_t)part * part_bytes;
    const int64_t row_bytes = (int64_t)Dh * sizeof(T);
    const bool is_sched = warp >= CW;              // two scheduler warps

    for (int i = tid; i < HSIZE; i += blockDim.x) tbl[i] = 0ull;
    if (tid == 0) *sync_until = -1;
    __syncthreads();

    auto meta_slot = [&](int step) { return meta + (step % MR) * META; };
    const int off_wk = 512, off_wq = 512 + MAXA * (int)sizeof(T), off_v = off_wq + MAXA * (int)sizeof(T);
    const int off_fwd = off_v + (int)row_bytes;

    // scheduler: metadata copies for one step (one commit group per step, also when empty)
    auto issue_meta = [&](int step) {
        if (step < T_) {
            uint8_t* ms = meta_slot(step);
            const int64_t bt = lt0 + step;
            const int nidx = (A * 8) / 16, nw = (A * (int)sizeof(T) + 15) / 16, nv = (int)row_bytes / 16;
            for (int i = lane; i < nidx; i += 32) cp_async16(ms + 16 * i, reinterpret_cast<const uint8_t*>(p.idx + bt * A) + 16 * i);
            for (int i = lane; i < nw; i += 32) {
                cp_async16(ms + off_wk + 16 * i, reinterpret_cast<const uint8_t*>(gwk + bt * A) + 16 * i);
                cp_async16(ms + off_wq + 16 * i, reinterpret_cast<const uint8_t*>(gwq + bt * A) + 16 * i);
            }
            for (int i = lane; i < nv; i += 32) cp_async16(ms + off_v + 16 * i, reinterpret_cast<const uint8_t*>(gv + bt * Dh) + 16 * i);
            if ((step % EPB) == 0 && lane == 0) {
                cp_async16(bring + (step % BR), gbeta + bt);
                if (p.dynamic_decay) cp_async16(aring + (step % BR), gdecay + bt);
            }
        }
        cp_commit();
    };

    const int rpl_rows = (A + 31) / 32;      // rows per lane: 1 or 2
    const float alpha_static = p.dynamic_decay ? 1.f : dg::to_f(gdecay[h]);
    const int vi = lane >> DUP;
    const bool leader = (lane & ((1 << DUP) - 1)) == 0;
    const int col_off = 16 * warp;            // this warp's slice inside the row part

    // prologue: metadata for steps 0..D-1
    if (warp == CW)
        for (int j = 0; j < D; ++j) issue_meta(j);

    for (int s = -D; s < T_; ++s) {
        // ---------------- column warps: consume step s ----------------
        if (!is_sched && s >= 0) {
            cp_wait<D - 1>();
            __syncwarp();
            uint8_t* ms = meta_slot(s);
            const int64_t* midx = reinterpret_cast<const int64_t*>(ms);
            const T* mwk = reinterpret_cast<const T*>(ms + off_wk);
            const T* mwq = reinterpret_cast<const T*>(ms + off_wq);
            const int16_t* mfwd = reinterpret_cast<const int16_t*>(ms + off_fwd);
            uint8_t* slot = rows + (s % RR) * slot_bytes;
            const bool sync_mode = s <= *sync_until;
            V rv[2];
            float wkv[2], wqv[2];
            int64_t X[2];
            bool ok[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int m = lane + 32 * i;
                ok[i] = false; wkv[i] = 0.f; wqv[i] = 0.f; X[i] = 0;
                rv[i].raw = make_uint4(0, 0, 0, 0);
                if (i < rpl_rows && m < A) {
                    const int64_t x = midx[m];
                    ok[i] = x >= 0 && x < total;
                    X[i] = ok[i] ? x : 0;
                    wkv[i] = dg::to_f(mwk[m]);
                    wqv[i] = dg::to_f(mwq[m]);
                    if (ok[i]) {
                        const int f = mfwd[m];
                        if (sync_mode) {        // L2 read: sees every earlier store of this CTA
                            rv[i].raw = __ldcg(reinterpret_cast<const uint4*>(gstate + X[i] * row_bytes + col_off));
                        } else if (f >= 0) {
                            rv[i].raw = *reinterpret_cast<const uint4*>(rows + (f >> 6) * slot_bytes +
                                                                         (f & 63) * row_stride + col_off);
                        } else {
                            rv[i].raw = *reinterpret_cast<const uint4*>(slot + m * row_stride + col_off);
                        }
                    }
                }
            }
            float vals[NV];
#pragma unroll
            for (int c = 0; c < CPW; ++c) {
                float y = 0.f, pr = 0.f;
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float sv = rv[i].get(c);
                    y = fmaf(wqv[i], sv, y);
                    pr = fmaf(wkv[i], sv, pr);
                }
                vals[c] = y;
                vals[CPW + c] = pr;
            }
            const float red = reduce_scatter<NV>(vals, lane);
            const int64_t bt = lt0 + s;
            const float al = p.dynamic_decay ? dg::to_f(aring[s % BR]) : alpha_static;
            const float bta = dg::to_f(bring[s % BR]);
            const int colg = part * (part_bytes / (int)sizeof(T)) + (col_off / (int)sizeof(T));   // first column
            const T* mv = reinterpret_cast<const T*>(ms + off_v);
            float rloc = 0.f;
            if (vi >= CPW) {
                rloc = bta * (dg::to_f(mv[colg + (vi - CPW)]) - red);
            } else if (leader) {
                static_cast<T*>(p.out)[bt * Dh + colg + vi] = dg::from_f<T>(red);
            }
            float br[CPW];
#pragma unroll
            for (int c = 0; c < CPW; ++c) br[c] = __shfl_sync(DG_FULL_MASK, rloc, (CPW + c) << DUP);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if (ok[i]) {
                    V nv;
#pragma unroll
                    for (int c = 0; c < CPW; ++c) nv.set(c, fmaf(al, rv[i].get(c), br[c] * wkv[i]));
                    const int m = lane + 32 * i;
                    *reinterpret_cast<uint4*>(slot + m * row_stride + col_off) = nv.raw;   // for forwarding
                    dg::st16(gstate + X[i] * row_bytes + col_off, nv.raw);
                }
            }
        }
        // ---------------- scheduler warps: metadata and hazards for step s + D ----------------
        // Warp CW issues the metadata copies; warps CW and CW+1 each take 32 rows.
        // A table cell holds key (slot + 1) in the low word and the writer stamp
        // (step << 6 | position) in the high word; a key's cell lives in bucket
        // slot_bucket(slot), and a cell is reusable once its writer step <= s.
        if (is_sched) {
            const int sw = warp - CW;
            if (sw == 0) {
                issue_meta(s + 2 * D);
                cp_wait<D>();             // metadata of step s + D has landed
            }
            asm volatile("bar.sync 1, 64;" ::: "memory");
            const int u = s + D;
            const int m = 32 * sw + lane;
            if (u < T_) {
                uint8_t* ms = meta_slot(u);
                const int64_t* midx = reinterpret_cast<const int64_t*>(ms);
                int16_t* mfwd = reinterpret_cast<int16_t*>(ms + off_fwd);
                bool have = false;
                uint32_t key = 0;
                unsigned long long* bk = nullptr;
                int16_t f = -1;
                if (m < A) {
                    const int64_t x = midx[m];
                    if (x >= 0 && x < total) {
                        have = true;
                        key = (uint32_t)x + 1u;
                        bk = tbl + WAYS * slot_bucket((uint32_t)x);
                        const ulonglong2* b2 = reinterpret_cast<const ulonglong2*>(bk);
                        unsigned long long c[WAYS];
#pragma unroll
                        for (int q = 0; q < WAYS / 2; ++q) { const ulonglong2 v2 = b2[q]; c[2 * q] = v2.x; c[2 * q + 1] = v2.y; }
#pragma unroll
                        for (int q = 0; q < WAYS; ++q) {
                            if ((uint32_t)c[q] == key) {
                                const uint32_t st = (uint32_t)(c[q] >> 32);
                                const int w = (int)(st >> 6);
                                if (u - w >= 1 && u - w <= D - 1) f = (int16_t)(((w % RR) << 6) | (st & 63));
                            }
                        }
                    } else {
                        dg::flag_status(p.status, DG_DEVCHK_INDEX_RANGE);
                    }
                }
                mfwd[m] = f;
                asm volatile("bar.sync 1, 64;" ::: "memory");     // all lookups of step u before its inserts
                if (have) {
                    const unsigned long long ne = (unsigned long long)key |
                                                  ((unsigned long long)(((uint32_t)u << 6) | (uint32_t)m) << 32);
                    bool placed = false;
                    for (int tries = 0; tries < 2 * WAYS && !placed; ++tries) {
                        // target: the key's own cell, else the first reusable one
                        int target = -1;
                        unsigned long long old = 0;
#pragma unroll
                        for (int q = 0; q < WAYS; ++q) {
                            const unsigned long long e = bk[q];
                            if ((uint32_t)e == key) { target = q; old = e; }
                        }
                        if (target < 0) {
#pragma unroll
                            for (int q = WAYS - 1; q >= 0; --q) {
                                const unsigned long long e = bk[q];
                                const int w = (int)((uint32_t)(e >> 32) >> 6);
                                if ((uint32_t)e == 0u || w <= s) { target = q; old = e; }
                            }
                        }
                        if (target < 0) break;
                        placed = atomicCAS(bk + target, old, ne) == old;
                    }
                    if (!placed) atomicMax(sync_until, u + D - 1);
                }
            }
        }
        __syncthreads();
        // ---------------- column warps: fetch rows of step s + D ----------------
        if (!is_sched) {
            const int u = s + D;
            if (u < T_) {
                uint8_t* ms = meta_slot(u);
                const int64_t* midx = reinterpret_cast<const int64_t*>(ms);
                const int16_t* mfwd = reinterpret_cast<const int16_t*>(ms + off_fwd);
                uint8_t* slot = rows + (u % RR) * slot_bytes;
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int m = lane + 32 * i;
                    if (i < rpl_rows && m < A) {
                        const int64_t x = midx[m];
                        if (x >= 0 && x < total && mfwd[m] < 0)
                            cp_async16(slot + m * row_stride + col_off, gstate + x * row_bytes + col_off);
                    }
                }
            }
            cp_commit();
        }
    }
    cp_wait<0>();
}

template <typename T, int D>
int launch_pipe(const PipeParams& p, int lanes, cudaStream_t stream) {
    const int part_bytes = p.Dh * (int)sizeof(T) / p.parts;
    const int cw = part_bytes / 16;
    const int threads = 32 * (cw + 2);
    const size_t smem = (size_t)(2 * D) * 64 * (part_bytes + 16) +
                        (size_t)(2 * D + 1) * meta_bytes((int)sizeof(T), p.Dh * (int)sizeof(T)) +
                        2 * (size_t)(4 * D + 16) * sizeof(T) + 16 + HSIZE * 8 + 16;
    auto kern = pkm_pipe_kernel<T, D>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    dim3 grid(p.parts, lanes);
    kern<<<grid, threads, smem, stream>>>(p);
    return dg_host::check_launch();
}

}  // namespace

namespace dg_host {

// Whether the pipelined kernel covers the call; the caller falls back otherwise.
bool pkm_pipe_supports(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v,
                       const void* beta, const void* wk, const void* wq, const void* idx, const void* decay,
                       int dynamic_decay, const void* state, const void* saved) {
    if (saved) return false;                                   // saving gathered rows: sequential kernel
    if (dtype != DG_DTYPE_F16 && dtype != DG_DTYPE_BF16 && dtype != DG_DTYPE_F32) return false;
    const int esz = dtype == DG_DTYPE_F32 ? 4 : 2;
    if (A > MAXA || A < 1 || total >= (int64_t)0x7fffffff - 1 || T < 1) return false;
    const int epb = 16 / esz;
    if (T % epb != 0) return false;                            // 16-byte beta / alpha blocks per lane
    if ((Dh * esz) % 32 != 0 || Dh * esz > (esz == 4 ? 256 : 256)) return false;
    if ((A * esz) % 16 != 0) return false;                     // 16-byte metadata copies
    const uintptr_t al = (uintptr_t)v | (uintptr_t)beta | (uintptr_t)wk | (uintptr_t)wq | (uintptr_t)idx |
                         (uintptr_t)state | (dynamic_decay ? (uintptr_t)decay : 0);
    (void)B; (void)H;
    return (al & 15) == 0;
}

int pkm_forward_pipe(int dtype, int B, int H, int T, int A, int64_t total, int Dh, const void* v, const void* beta,
                     const void* wk, const void* wq, const int64_t* idx, const void* decay, int dynamic_decay,
                     void* state, void* out, int32_t* status, cudaStream_t stream) {
    const int lanes = B * H;
    const int esz = dtype == DG_DTYPE_F32 ? 4 : 2;
    // Rows are split in two column halves (two CTAs per lane) when there are too
    // few lanes to fill the GPU, and always for fp32 so the row ring fits in
    // shared memory.  Window depth: 8 steps for full rows, 12 for halves (16-bit).
    int parts = (lanes < 120 || esz == 4) ? 2 : 1;
    if ((Dh * esz) % (32 * parts) != 0) parts = 1;
    if (esz == 4 && parts == 1 && Dh * esz > 128) return DG_ERR_UNSUPPORTED;
    PipeParams p{v, beta, wk, wq, idx, decay, state, out, status, H, T, A, Dh, parts, total, dynamic_decay};
    switch (dtype) {
    case DG_DTYPE_F16: return parts == 1 ? launch_pipe<__half, 8>(p, lanes, stream) : launch_pipe<__half, 12>(p, lanes, stream);
    case DG_DTYPE_BF16: return parts == 1 ? launch_pipe<__nv_bfloat16, 8>(p, lanes, stream) : launch_pipe<__nv_bfloat16, 12>(p, lanes, stream);
    case DG_DTYPE_F32: return launch_pipe<float, 8>(p, lanes, stream);
    default: return DG_ERR_UNSUPPORTED;
    }
}

}  // namespace dg_host
