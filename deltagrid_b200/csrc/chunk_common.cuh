// chunk_common.cuh -- pieces shared by the two chunkwise dense tcgen05 kernels
// (dense_chunk_tc.cu: state rows on TMEM lanes; dense_chunk_t.cu: state columns on
// TMEM lanes): 16-bit operand traits, per-chunk decay/gate scalars, the blocked
// inverse of the unit lower-triangular chunk matrix, and TMA tensor-map encoding.
#pragma once

#include "dg_common.cuh"
#include "tc_util.cuh"

#include <cuda.h>

namespace dgc {

constexpr int CH = 64;        // steps per chunk
constexpr int DH = 64;        // head dimension handled by the chunk kernels
constexpr uint32_t BAR_WG0 = 1, BAR_WG1 = 2;   // named barrier ids (0 is __syncthreads)

// Operand types.  The products with an input operand (the Gram [K;Q] K^T, [K;Q] S0 and the
// update K^T R') take the input type TI (fp16 or bf16: both operands of one kind::f16 MMA
// share a type), so the S0 and R' copies are written in TI.  T X and Mqk (R beta) have
// only operands formed here and stay fp16 for both input types.
template <typename TI> struct Io;
template <> struct Io<__half> {
    static constexpr int kBf16 = 0;
    __device__ static uint32_t pack2(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ static float2 unpack2(uint32_t u) { return __half22float2(*reinterpret_cast<__half2*>(&u)); }
};
template <> struct Io<__nv_bfloat16> {
    static constexpr int kBf16 = 1;
    __device__ static uint32_t pack2(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ static float2 unpack2(uint32_t u) { return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u)); }
    // the bf16 pair of what pack2 leaves out: a = hi + lo with both halves bf16, so a
    // product taken over hi and lo separately sees ~16 significant bits of a
    __device__ static uint32_t pack2_lo(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        const float2 hf = __bfloat1622float2(h);
        __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
        return *reinterpret_cast<uint32_t*>(&l);
    }
};
constexpr int LDT = 68;                 // fp32 row stride of the L/T scratch


// write 64 fp32 values as one 128-byte swizzled row of 16-bit type TT
template <typename TT = __half>
__device__ __forceinline__ void st_row16(uint8_t* tile, int row, const float* x) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 v;
        v.x = Io<TT>::pack2(x[8 * c + 0], x[8 * c + 1]);
        v.y = Io<TT>::pack2(x[8 * c + 2], x[8 * c + 3]);
        v.z = Io<TT>::pack2(x[8 * c + 4], x[8 * c + 5]);
        v.w = Io<TT>::pack2(x[8 * c + 6], x[8 * c + 7]);
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

// Per-chunk decay/gate scalars, computed by every warp on its own: lane l holds
// steps 2l and 2l+1.  a = inclusive product of alpha, ap = exclusive product.
struct ChunkScalars {
    float a0, a1;       // a_incl for steps 2l, 2l+1
    float ap0, ap1;     // aprev for steps 2l, 2l+1
    float b0, b1;       // beta
    float atot;         // a_{C-1}
};

// The scan of chunk_scalars on gate values already in registers (lane l: beta and alpha
// of steps 2l and 2l+1; alpha = 1 and beta = 0 beyond T).
__device__ __forceinline__ ChunkScalars gate_scalars(float b0, float b1, float al0, float al1, int lane) {
    ChunkScalars c;
    c.b0 = b0;
    c.b1 = b1;
    float incl = al0 * al1;              // inclusive scan of pair products over lanes
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(DG_FULL_MASK, incl, o);
        if (lane >= o) incl *= v;
    }
    float excl = __shfl_up_sync(DG_FULL_MASK, incl, 1);
    if (lane == 0) excl = 1.f;
    c.ap0 = excl;
    c.a0 = excl * al0;
    c.ap1 = c.a0;
    c.a1 = c.a0 * al1;
    c.atot = __shfl_sync(DG_FULL_MASK, incl, 31);
    return c;
}

template <typename TI>
__device__ __forceinline__ ChunkScalars chunk_scalars(const TI* beta, const TI* decay, int dyn,
                                                      float alpha_static, int64_t lane_base, int t0, int T_,
                                                      int lane) {
    const int t = t0 + 2 * lane;
    const bool ok0 = t < T_, ok1 = t + 1 < T_;
    const float al0 = ok0 ? (dyn ? dg::to_f(decay[lane_base + t]) : alpha_static) : 1.f;
    const float al1 = ok1 ? (dyn ? dg::to_f(decay[lane_base + t + 1]) : alpha_static) : 1.f;
    return gate_scalars(ok0 ? dg::to_f(beta[lane_base + t]) : 0.f, ok1 ? dg::to_f(beta[lane_base + t + 1]) : 0.f,
                        al0, al1, lane);
}
// value of step i from the pair registers (all lanes must call)
__device__ __forceinline__ float pick(float v0, float v1, int i) {
    const float a = __shfl_sync(DG_FULL_MASK, v0, i >> 1);
    const float b = __shfl_sync(DG_FULL_MASK, v1, i >> 1);
    return (i & 1) ? b : a;
}

// (I + L)^{-1} for strictly lower L (64x64 fp32, row stride LDT), in place, by one
// warpgroup (t = 0..127).  Two-level blocked inverse of a unit lower-triangular
// matrix, [[A, 0], [C, D]]^{-1} = [[A^-1, 0], [-D^-1 C A^-1, D^-1]]:
//   1. the four 16x16 diagonal blocks by forward substitution (one warp each);
//   2. the 32x32 halves A^-1 and D^-1: off-diagonal 16x16 block -D1^-1 L10 D0^-1;
//   3. P = C A^-1 and 4. -D^-1 P for the lower-left 32x32 quadrant.
// Products are register-tiled (each thread a 2x2 or 2x4 output tile) and every
// stage writes its results after a barrier, so reads always see the previous stage.
__device__ __forceinline__ float& lt_at(float* lt, int r, int c) { return lt[r * LDT + c]; }

static __device__ void invert_unit_lower(float* lt, int t) {
    const int warp = t >> 5, lane = t & 31;
    {   // 1. diagonal 16x16 blocks: lane = column of the block's inverse
        const int b = warp, col = lane & 15;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            float s0 = (r == col) ? 1.f : 0.f, s1 = 0.f;
#pragma unroll
            for (int j = 0; j < r; ++j) {
                const float l = lt_at(lt, 16 * b + r, 16 * b + j);
                if (j & 1) s1 = fmaf(-l, x[j], s1); else s0 = fmaf(-l, x[j], s0);
            }
            x[r] = s0 + s1;
        }
        tc::group_sync(BAR_WG1);
        if (lane < 16) {
#pragma unroll
            for (int r = 0; r < 16; ++r) lt_at(lt, 16 * b + r, 16 * b + col) = x[r];
        }
        tc::group_sync(BAR_WG1);
    }
    {   // 2. half h (64 threads): block (2h+1, 2h) = -D_{2h+1} L_{2h+1,2h} D_{2h}, 2x2 tile per thread
        const int h = t >> 6, u = t & 63, ti = u >> 3, tj = u & 7;
        const int r0 = 16 * (2 * h + 1) + 2 * ti, c0 = 16 * (2 * h) + 2 * tj;     // output rows / cols
        const int k0 = 16 * (2 * h);                                             // inner index base (D_{2h})
        float p00 = 0.f, p01 = 0.f, p10 = 0.f, p11 = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float a0 = lt_at(lt, r0, k0 + k), a1 = lt_at(lt, r0 + 1, k0 + k);
            const float2 bb = *reinterpret_cast<const float2*>(&lt_at(lt, k0 + k, c0));
            p00 = fmaf(a0, bb.x, p00); p01 = fmaf(a0, bb.y, p01);
            p10 = fmaf(a1, bb.x, p10); p11 = fmaf(a1, bb.y, p11);
        }
        tc::group_sync(BAR_WG1);
        *reinterpret_cast<float2*>(&lt_at(lt, r0, c0)) = make_float2(p00, p01);
        *reinterpret_cast<float2*>(&lt_at(lt, r0 + 1, c0)) = make_float2(p10, p11);
        tc::group_sync(BAR_WG1);
        const int d0 = 16 * (2 * h + 1);                                         // D_{2h+1} diagonal base
        float q00 = 0.f, q01 = 0.f, q10 = 0.f, q11 = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float a0 = lt_at(lt, r0, d0 + k), a1 = lt_at(lt, r0 + 1, d0 + k);
            const float2 bb = *reinterpret_cast<const float2*>(&lt_at(lt, d0 + k, c0));
            q00 = fmaf(a0, bb.x, q00); q01 = fmaf(a0, bb.y, q01);
            q10 = fmaf(a1, bb.x, q10); q11 = fmaf(a1, bb.y, q11);
        }
        tc::group_sync(BAR_WG1);
        *reinterpret_cast<float2*>(&lt_at(lt, r0, c0)) = make_float2(-q00, -q01);
        *reinterpret_cast<float2*>(&lt_at(lt, r0 + 1, c0)) = make_float2(-q10, -q11);
        tc::group_sync(BAR_WG1);
    }
    {   // 3./4. lower-left quadrant: P = C A^-1, then -D^-1 P; 2x4 tile per thread
        const int ti = t >> 3, tj = t & 7;
        const int r0 = 32 + 2 * ti, c0 = 4 * tj;
        float acc[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {           // C (rows 32..63, cols 0..31) times A^-1 (rows/cols 0..31)
            const float a0 = lt_at(lt, r0, k), a1 = lt_at(lt, r0 + 1, k);
            const float4 bb = *reinterpret_cast<const float4*>(&lt_at(lt, k, c0));
            acc[0][0] = fmaf(a0, bb.x, acc[0][0]); acc[0][1] = fmaf(a0, bb.y, acc[0][1]);
            acc[0][2] = fmaf(a0, bb.z, acc[0][2]); acc[0][3] = fmaf(a0, bb.w, acc[0][3]);
            acc[1][0] = fmaf(a1, bb.x, acc[1][0]); acc[1][1] = fmaf(a1, bb.y, acc[1][1]);
            acc[1][2] = fmaf(a1, bb.z, acc[1][2]); acc[1][3] = fmaf(a1, bb.w, acc[1][3]);
        }
        tc::group_sync(BAR_WG1);
        *reinterpret_cast<float4*>(&lt_at(lt, r0, c0)) = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
        *reinterpret_cast<float4*>(&lt_at(lt, r0 + 1, c0)) = make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]);
        tc::group_sync(BAR_WG1);
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {           // D^-1 (rows/cols 32..63) times P (rows 32..63, cols 0..31)
            const float a0 = lt_at(lt, r0, 32 + k), a1 = lt_at(lt, r0 + 1, 32 + k);
            const float4 bb = *reinterpret_cast<const float4*>(&lt_at(lt, 32 + k, c0));
            acc[0][0] = fmaf(a0, bb.x, acc[0][0]); acc[0][1] = fmaf(a0, bb.y, acc[0][1]);
            acc[0][2] = fmaf(a0, bb.z, acc[0][2]); acc[0][3] = fmaf(a0, bb.w, acc[0][3]);
            acc[1][0] = fmaf(a1, bb.x, acc[1][0]); acc[1][1] = fmaf(a1, bb.y, acc[1][1]);
            acc[1][2] = fmaf(a1, bb.z, acc[1][2]); acc[1][3] = fmaf(a1, bb.w, acc[1][3]);
        }
        tc::group_sync(BAR_WG1);
        *reinterpret_cast<float4*>(&lt_at(lt, r0, c0)) = make_float4(-acc[0][0], -acc[0][1], -acc[0][2], -acc[0][3]);
        *reinterpret_cast<float4*>(&lt_at(lt, r0 + 1, c0)) = make_float4(-acc[1][0], -acc[1][1], -acc[1][2], -acc[1][3]);
        tc::group_sync(BAR_WG1);
    }
}

// ---------------------------------------------------------------------------
// host side: tensor maps
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
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

// 3-D map over [lanes][T][cols] 16-bit elements with a 64 x 64 box and 128B swizzle
inline bool make_map(CUtensorMap* m, const void* base, int cols, int T, int lanes, bool bf16) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)T, (cuuint64_t)lanes};
    cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)cols * 2 * (cuuint64_t)T};
    cuuint32_t box[3] = {64, 64, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
              const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace dgc
