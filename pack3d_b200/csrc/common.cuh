// Shared device helpers for the pack3d_b200 kernels (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pack3d_b200.h"

namespace p3d {

// ---------------------------------------------------------------- error plumbing
void set_error(const char *fmt, ...);
int fail(int status, const char *fmt, ...);

#define P3D_CHECK_ARG(cond, ...)                                  \
  do {                                                            \
    if (!(cond)) return ::p3d::fail(P3D_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

#define P3D_CUDA_TRY(expr)                                                                 \
  do {                                                                                     \
    cudaError_t err_ = (expr);                                                             \
    if (err_ != cudaSuccess)                                                               \
      return ::p3d::fail(P3D_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                    \
                         cudaGetErrorString(err_), __FILE__, __LINE__);                   \
  } while (0)

#define P3D_LAUNCH_CHECK() P3D_CUDA_TRY(cudaGetLastError())

// ---------------------------------------------------------------- element types
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
// bf16 -> fp32 is exact as a 16-bit shift of the bit pattern: integer operations only.
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __uint_as_float((uint32_t)__bfloat16_as_ushort(v) << 16);
}

// The two 16-bit values of a packed word as fp32, low half first.  bf16 -> fp32 is exact as
// a 16-bit shift of the bit pattern (two integer operations, no conversion unit); f16 uses
// the paired hardware conversion.
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Round a float through storage type T (identity for float).
template <typename T> __device__ __forceinline__ float round_to(float v) {
  return to_f32<T>(from_f32<T>(v));
}

__device__ __forceinline__ float load_any(const void *p, int dtype, int64_t i) {
  switch (dtype) {
    case P3D_F16: return __half2float(static_cast<const __half *>(p)[i]);
    case P3D_BF16: return to_f32<__nv_bfloat16>(static_cast<const __nv_bfloat16 *>(p)[i]);
    default: return static_cast<const float *>(p)[i];
  }
}

__device__ __forceinline__ void store_any(void *p, int dtype, int64_t i, float v) {
  switch (dtype) {
    case P3D_F16: static_cast<__half *>(p)[i] = __float2half_rn(v); break;
    case P3D_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v); break;
    default: static_cast<float *>(p)[i] = v;
  }
}

// ---------------------------------------------------------------- warp reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

inline int dtype_size(int dtype) { return dtype == P3D_F32 ? 4 : 2; }
inline bool dtype_ok(int dtype) { return dtype == P3D_F32 || dtype == P3D_F16 || dtype == P3D_BF16; }

// Host launch helpers implemented in the .cu files ------------------------------------
struct DeviceInfo {
  int sm_count;
  int major, minor;
  size_t smem_optin;
};
int device_info(DeviceInfo *info);

// Dynamic shared memory above the 48 KB default needs a per-kernel opt-in, and that setting
// belongs to the current device's context: a process that launches on several GPUs must set
// it on each.  `seen` (one per kernel) records the size opted in per device ordinal; the
// attribute is set again only when a launch needs more than before on that device.
constexpr int kMaxDevices = 64;
template <typename K>
inline int smem_optin(K kernel, size_t bytes, size_t (&seen)[kMaxDevices]) {
  int dev = 0;
  P3D_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(P3D_ERR_DEVICE, "device ordinal %d out of range", dev);
  if (bytes > seen[dev]) {
    P3D_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    seen[dev] = bytes;
  }
  return P3D_OK;
}

}  // namespace p3d

namespace p3d {
// Dot of a global-memory row of T with a shared-memory fp32 vector.  vec: the row is
// 16-byte aligned and d is a multiple of 8 (16-bit types) -- use 16-byte loads.
template <typename T>
__device__ __forceinline__ float dot_row(const T *row, const float *v, int d, bool vec) {
  float acc = 0.f;
  if constexpr (sizeof(T) == 2) {
    if (vec) {
      for (int c = 0; c < d; c += 8) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(row + c);
        const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = fmaf(to_f32<T>(e[i]), v[c + i], acc);
      }
      return acc;
    }
  }
  for (int c = 0; c < d; ++c) acc = fmaf(to_f32<T>(row[c]), v[c], acc);
  return acc;
}

// Warp-cooperative copy of a row of T into shared memory as fp32.
template <typename T>
__device__ __forceinline__ void row_to_smem(const T *row, float *dst, int d) {
  for (int c = threadIdx.x & 31; c < d; c += 32) dst[c] = to_f32<T>(row[c]);
  __syncwarp();
}
}  // namespace p3d
