// dg_common.cuh -- shared helpers for the DeltaGrid sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/deltagrid_b200.h"

#define DG_FULL_MASK 0xffffffffu

namespace dg {

// ---- storage <-> fp32 -------------------------------------------------------
// Every kernel computes in fp32 and rounds to the storage dtype with
// round-to-nearest-even, exactly where the reference casts
// (static_cast<scalar_t>(float) in src/cpp/delta_kernel.cu).
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(double x) { return (float)x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ double from_f<double>(float x) { return (double)x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

// ---- 16-byte vectors of storage elements ------------------------------------
template <typename T>
struct Vec16 {
    static constexpr int N = 16 / sizeof(T);
    uint4 raw;
    __device__ __forceinline__ float get(int i) const {
        return to_f(reinterpret_cast<const T*>(&raw)[i]);
    }
    __device__ __forceinline__ void set(int i, float x) {
        reinterpret_cast<T*>(&raw)[i] = from_f<T>(x);
    }
};

__device__ __forceinline__ uint4 ldg16(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}
// plain (coherent, not read-only-path) 16-byte load: for data the same kernel writes
__device__ __forceinline__ uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ void st16(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

__device__ __forceinline__ void flag_status(int32_t* st, int bits) {
    if (st) atomicOr(st, bits);
}

}  // namespace dg

// host-side helpers shared by the launch files
namespace dg_host {
int record_cuda_error(cudaError_t e);   // stores e for dg_last_cuda_error, returns DG_ERR_CUDA
inline int check_launch() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DG_OK : record_cuda_error(e);
}
// multiprocessor count of a device, queried once per device and cached
int sm_count(int device, int* out);
inline size_t dtype_size(int dtype) {
    switch (dtype) {
    case DG_DTYPE_F32: return 4;
    case DG_DTYPE_F64: return 8;
    case DG_DTYPE_F16: return 2;
    case DG_DTYPE_BF16: return 2;
    default: return 0;
    }
}
}  // namespace dg_host

// dtype dispatch: calls F<T>(...) for the storage type of `dtype`
#define DG_DISPATCH(dtype, T, ...)                         \
    switch (dtype) {                                       \
    case DG_DTYPE_F32: { using T = float; __VA_ARGS__; } break;          \
    case DG_DTYPE_F64: { using T = double; __VA_ARGS__; } break;         \
    case DG_DTYPE_F16: { using T = __half; __VA_ARGS__; } break;         \
    case DG_DTYPE_BF16: { using T = __nv_bfloat16; __VA_ARGS__; } break; \
    default: return DG_ERR_INVALID_ARGUMENT;               \
    }
