// slot_route.cu -- dense slot routing on tcgen05: wk = L2-normalise(k P_k^T) and
// wq = (q P_q^T) * q_scale[h], for 16-bit k, q with Dh = 64 and slots a multiple of 64
// up to 512.
//
// Replaces DeltaGridLayer._route_dense's linear-projection branch
// (src/modules/memory.py:233-236: F.normalize(slot_proj_k(k)), slot_proj_q(q); the
// projections are bias-free nn.Linear, :192-193) and the q_scale multiply of
// memory.py:490-492, which the layer forms with library GEMMs and elementwise kernels
// before the recurrence.
//
// Persistent CTAs, one per SM (the accumulator takes all 512 TMEM columns), each
// taking tiles of 128 tokens in turn:
//   - warp 4, one thread: TMA loads (P_k and P_q once, 128B-swizzled; each tile's k
//     and q rows) and the MMAs: D = k P_k^T as M = 128 (a token per TMEM lane),
//     N = slots (in pieces of at most 256), K = 64, then, once the epilogue has read
//     it, D = q P_q^T into the same columns;
//   - warps 0-3 (thread t = token t of the tile = TMEM lane t): for wk, the sum of
//     squares over the row (fp32), then the row scaled by 1 / max(norm, 1e-12); for
//     wq, the row times q_scale of its head; each 64-slot slice is rounded to the
//     storage type into a 128B-swizzled shared tile and leaves by a 2-D TMA store
//     (two tiles in turn).
// The next tile's k and q load as soon as its predecessor's second product has read
// them, under the second epilogue.  Every mbarrier wait is bounded (the library's wait
// limit); a wait that gives up stops the CTA's work, flags DG_DEVCHK_TIMEOUT when a
// status word is given, and drains what the CTA issued before freeing its TMEM.
#include <cuda.h>

#include "chunk_common.cuh"

namespace {

constexpr int SR_M = 128;                 // tokens per tile
constexpr int SR_DH = 64;
constexpr int SR_SMAX = 512;
constexpr int SR_THREADS = 160;           // four epilogue warps and the issuing warp
constexpr uint32_t SR_DRAIN = 1u << 22;

// shared memory: [P_k | P_q] (S rows x 128 B each), k tile, q tile, two output tiles, barriers
constexpr uint32_t SR_PK = 0;
constexpr uint32_t SR_PQ = SR_PK + SR_SMAX * 128;
constexpr uint32_t SR_KT = SR_PQ + SR_SMAX * 128;
constexpr uint32_t SR_QT = SR_KT + SR_M * 128;
constexpr uint32_t SR_OUT = SR_QT + SR_M * 128;          // 2 x [128 rows x 128 B]
constexpr uint32_t SR_BAR = SR_OUT + 2 * SR_M * 128;
constexpr uint32_t SR_BYTES = SR_BAR + 8 * 8;

enum { B_P = 0, B_KQ, B_MK, B_MQ, B_TK, B_TQ, B_NUM };

struct SrParams {
    const float* q_scale;    // [H] or null
    int32_t* status;         // device status word or null
    int64_t N;               // tokens (B*H*T)
    int H, T, S;
    uint32_t wait_limit;
};

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
__global__ void __launch_bounds__(SR_THREADS, 1)
    slot_route_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmq,
                      const __grid_constant__ CUtensorMap tmpk, const __grid_constant__ CUtensorMap tmpq,
                      const __grid_constant__ CUtensorMap tmwk, const __grid_constant__ CUtensorMap tmwq, SrParams p) {
    constexpr bool BF16 = !std::is_same<T, __half>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + SR_BAR);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + B_NUM);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int S = p.S;
    const int64_t ntiles = (p.N + SR_M - 1) / SR_M;

    if (warp == 0) tc::tmem_alloc(tmem_holder, 512);
    if (tid == 0) {
        for (int i = 0; i < B_NUM; ++i) tc::mbar_init(bars + i, 1);
        tc::fence_barrier_init();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    bool bad = false;

    if (warp == 4) {
        // ================================ issuer ================================
        if ((tid & 31) == 0) {
            const uint32_t prows = S > 256 ? 256u : (uint32_t)S;
            auto load_tile = [&](int64_t tile) {
                tc::mbar_expect_tx(bars + B_KQ, 2 * SR_M * 128);
                tc::tma_load_2d(sm + SR_KT, &tmk, bars + B_KQ, 0, (int)(tile * SR_M));
                tc::tma_load_2d(sm + SR_QT, &tmq, bars + B_KQ, 0, (int)(tile * SR_M));
            };
            tc::prefetch_tmap(&tmk);
            tc::prefetch_tmap(&tmq);
            tc::mbar_expect_tx(bars + B_P, 2u * (uint32_t)((S + 255) / 256) * prows * 128u);
            for (int r = 0; r < S; r += 256) {
                tc::tma_load_2d(sm + SR_PK + r * 128, &tmpk, bars + B_P, 0, r);
                tc::tma_load_2d(sm + SR_PQ + r * 128, &tmpq, bars + B_P, 0, r);
            }
            int64_t tile = blockIdx.x;
            if (tile < ntiles) load_tile(tile);
            bad = !tc::mbar_wait(bars + B_P, 0, p.wait_limit);
            // in flight when a wait gives up: the load of tile i (pending_kq), the MMAs
            // of a product (pending_m: its barrier and parity)
            int pend_kq = tile < ntiles ? 0 : -1;
            int pend_mbar = -1, pend_mpar = 0;
            auto product = [&](uint32_t a_off, uint32_t b_off) {
                for (int c = 0; c < S; c += 256) {
                    const int n = S - c > 256 ? 256 : S - c;
                    const uint32_t idesc = tc::make_idesc(128, n, BF16 ? 1 : 0, 0, 0);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc::mma_f16(tmem + (uint32_t)c, tc::make_desc(tc::smem_u32(sm + a_off) + 32 * kk, 16, 1024),
                                    tc::make_desc(tc::smem_u32(sm + b_off + c * 128) + 32 * kk, 16, 1024), idesc,
                                    kk != 0);
                }
            };
            for (int64_t i = 0; tile < ntiles && !bad; ++i, tile += gridDim.x) {
                const uint32_t par = (uint32_t)(i & 1);
                if (!tc::mbar_wait(bars + B_KQ, par, p.wait_limit)) { bad = true; break; }
                pend_kq = -1;
                if (i > 0 && !tc::mbar_wait(bars + B_TQ, par ^ 1u, p.wait_limit)) { bad = true; break; }
                tc::tc_fence_after();
                product(SR_KT, SR_PK);
                tc::mma_commit(bars + B_MK);
                pend_mbar = B_MK;
                pend_mpar = (int)par;
                if (!tc::mbar_wait(bars + B_TK, par, p.wait_limit)) { bad = true; break; }
                tc::tc_fence_after();
                product(SR_QT, SR_PQ);
                tc::mma_commit(bars + B_MQ);
                pend_mbar = B_MQ;
                if (!tc::mbar_wait(bars + B_MQ, par, p.wait_limit)) { bad = true; break; }
                pend_mbar = -1;
                if (tile + gridDim.x < ntiles) {       // both products have read the k and q tiles
                    load_tile(tile + gridDim.x);
                    pend_kq = (int)(par ^ 1u);
                }
            }
            if (bad) {
                dg::flag_status(p.status, DG_DEVCHK_TIMEOUT);
                tc::mbar_wait(bars + B_P, 0, SR_DRAIN);
                if (pend_kq >= 0) tc::mbar_wait(bars + B_KQ, (uint32_t)pend_kq, SR_DRAIN);
                if (pend_mbar >= 0) tc::mbar_wait(bars + pend_mbar, (uint32_t)pend_mpar, SR_DRAIN);
            }
        }
    } else {
        // =============================== epilogue ===============================
        const int t = tid;                                       // token of the tile = TMEM lane
        const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
        uint8_t* out0 = sm + SR_OUT;
        int nstore = 0;                                          // slices stored so far (tiles alternate)
        auto emit = [&](const CUtensorMap* map, int64_t row0, float scale) {
            for (int j = 0; j < S / 64; ++j, ++nstore) {
                uint8_t* ob = out0 + (nstore & 1) * (SR_M * 128);
                // the store that last read this tile has finished reading it
                if (t == 0) tc::bulk_wait_read1();
                tc::group_sync(1);
                uint32_t ra[32], rb[32];
                tc::tmem_ld32(trow + (uint32_t)(64 * j), ra);
                tc::tmem_ld32(trow + (uint32_t)(64 * j + 32), rb);
                tc::tmem_wait_ld();
                auto put = [&](const uint32_t (&r)[32], int c0) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint4 v;
                        v.x = pack2<T>(__uint_as_float(r[8 * c + 0]) * scale, __uint_as_float(r[8 * c + 1]) * scale);
                        v.y = pack2<T>(__uint_as_float(r[8 * c + 2]) * scale, __uint_as_float(r[8 * c + 3]) * scale);
                        v.z = pack2<T>(__uint_as_float(r[8 * c + 4]) * scale, __uint_as_float(r[8 * c + 5]) * scale);
                        v.w = pack2<T>(__uint_as_float(r[8 * c + 6]) * scale, __uint_as_float(r[8 * c + 7]) * scale);
                        *reinterpret_cast<uint4*>(ob + tc::sw128((uint32_t)t, (uint32_t)(c0 + c))) = v;
                    }
                };
                put(ra, 0);
                put(rb, 4);
                tc::fence_proxy_async();
                tc::group_sync(1);
                if (t == 0) {
                    tc::tma_store_2d(map, ob, 64 * j, (int)row0);
                    tc::bulk_commit_group();
                }
            }
        };
        int64_t tile = blockIdx.x;
        for (int64_t i = 0; tile < ntiles; ++i, tile += gridDim.x) {
            const uint32_t par = (uint32_t)(i & 1);
            const int64_t row0 = tile * SR_M;
            const int64_t n = row0 + t;
            // wk: the row's norm, then the scaled row
            bad = !tc::mbar_wait(bars + B_MK, par, p.wait_limit);
            if (tc::group_sync_or(2, bad)) { bad = true; break; }
            tc::tc_fence_after();
            float ss = 0.f;
            for (int c = 0; c < S; c += 32) {
                uint32_t r[32];
                tc::tmem_ld32(trow + (uint32_t)c, r);
                tc::tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) ss = fmaf(__uint_as_float(r[e]), __uint_as_float(r[e]), ss);
            }
            emit(&tmwk, row0, 1.f / fmaxf(sqrtf(ss), 1e-12f));
            tc::tc_fence_before();
            tc::group_sync(1);
            if (t == 0) tc::mbar_arrive(bars + B_TK);
            // wq: the row times its head's q_scale
            bad = !tc::mbar_wait(bars + B_MQ, par, p.wait_limit);
            if (tc::group_sync_or(2, bad)) { bad = true; break; }
            tc::tc_fence_after();
            const float qs = (p.q_scale && n < p.N) ? p.q_scale[(n / p.T) % p.H] : 1.f;
            emit(&tmwq, row0, qs);
            tc::tc_fence_before();
            tc::group_sync(1);
            if (t == 0) tc::mbar_arrive(bars + B_TQ);
        }
        if (t == 0) tc::bulk_wait0();
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

// 2-D map over [rows][cols] 16-bit values, box 64 x box_rows, 128B swizzle
bool map_2d(CUtensorMap* m, const void* base, int64_t rows, int cols, int box_rows, bool bf16) {
    dgc::EncodeTiledFn fn = dgc::encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace dg_host {

uint32_t wait_limit();
int sm_count(int device, int* out);

bool slot_route_supports(int dtype, int dh, int slots, const void* k, const void* q, const void* pk, const void* pq,
                         const void* wk, const void* wq) {
    if (dtype != DG_DTYPE_F16 && dtype != DG_DTYPE_BF16) return false;
    if (dh != SR_DH || slots < 64 || slots > SR_SMAX || slots % 64 != 0) return false;
    const uintptr_t al = (uintptr_t)k | (uintptr_t)q | (uintptr_t)pk | (uintptr_t)pq | (uintptr_t)wk | (uintptr_t)wq;
    return (al & 15) == 0;
}

int slot_route(int dtype, int64_t N, int H, int T, int slots, const void* k, const void* q, const void* pk,
               const void* pq, const float* q_scale, void* wk, void* wq, int32_t* status, cudaStream_t s) {
    if (N == 0) return DG_OK;
    const bool bf16 = dtype == DG_DTYPE_BF16;
    CUtensorMap mk, mq, mpk, mpq, mwk, mwq;
    const int prows = slots > 256 ? 256 : slots;
    if (!map_2d(&mk, k, N, SR_DH, SR_M, bf16) || !map_2d(&mq, q, N, SR_DH, SR_M, bf16) ||
        !map_2d(&mpk, pk, slots, SR_DH, prows, bf16) || !map_2d(&mpq, pq, slots, SR_DH, prows, bf16) ||
        !map_2d(&mwk, wk, N, slots, SR_M, bf16) || !map_2d(&mwq, wq, N, slots, SR_M, bf16))
        return DG_ERR_UNSUPPORTED;
    int dev = 0, nsm = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e);
    int rc = sm_count(dev, &nsm);
    if (rc != DG_OK) return rc;
    const int64_t ntiles = (N + SR_M - 1) / SR_M;
    const unsigned grid = (unsigned)(ntiles < nsm ? ntiles : nsm);
    const int smem = (int)SR_BYTES + 1024;
    SrParams p{q_scale, status, N, H, T, slots, wait_limit()};
    if (bf16) {
        auto kern = slot_route_kernel<__nv_bfloat16>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return record_cuda_error(e);
        kern<<<grid, SR_THREADS, smem, s>>>(mk, mq, mpk, mpq, mwk, mwq, p);
    } else {
        auto kern = slot_route_kernel<__half>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return record_cuda_error(e);
        kern<<<grid, SR_THREADS, smem, s>>>(mk, mq, mpk, mpq, mwk, mwq, p);
    }
    return check_launch();
}

}  // namespace dg_host

extern "C" int dg_dense_route(int dtype, int B, int H, int T, int dh, int slots, const void* k, const void* q,
                              const void* slot_proj_k, const void* slot_proj_q, const float* q_scale, void* wk,
                              void* wq, int32_t* dev_status, void* stream) {
    if (B < 0 || H <= 0 || T < 0 || dh <= 0 || slots <= 0) return DG_ERR_INVALID_ARGUMENT;
    if (!k || !q || !slot_proj_k || !slot_proj_q || !wk || !wq) return DG_ERR_INVALID_ARGUMENT;
    if (!dg_host::slot_route_supports(dtype, dh, slots, k, q, slot_proj_k, slot_proj_q, wk, wq))
        return DG_ERR_UNSUPPORTED;
    return dg_host::slot_route(dtype, (int64_t)B * H * T, H, T, slots, k, q, slot_proj_k, slot_proj_q, q_scale, wk,
                               wq, dev_status, static_cast<cudaStream_t>(stream));
}
