// Shared helpers for the DDPM sm_100a kernels: element conversion, error
// reporting and launch checks. Every kernel accumulates in FP32 and converts
// at the load/store boundary, like the reference's Triton kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/ddpm_b200.h"

namespace ddpm {

// ---------------------------------------------------------------- errors ---
// Records a message for ddpm_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();
// Counts one kernel launch (read back through ddpm_launch_count()).
void note_launch();

#define DDPM_CHECK_ARG(cond, ...)                                   \
  do {                                                              \
    if (!(cond)) return ::ddpm::set_error(DDPM_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

#define DDPM_CHECK_LAUNCH(what)                                     \
  do {                                                              \
    ::ddpm::note_launch();                                          \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess)                                          \
      return ::ddpm::set_error(DDPM_ERR_CUDA, "%s: %s", what,       \
                               cudaGetErrorString(_e));             \
  } while (0)

#define DDPM_CUDA_TRY(call)                                         \
  do {                                                              \
    cudaError_t _e = (call);                                        \
    if (_e != cudaSuccess)                                          \
      return ::ddpm::set_error(DDPM_ERR_CUDA, "%s: %s", #call,      \
                               cudaGetErrorString(_e));             \
  } while (0)

// ------------------------------------------------------------ conversion ---
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}

// Read-only load through the non-coherent path (data read once per launch).
template <typename T> __device__ __forceinline__ float ldg_f32(const T* p) {
  return to_f32<T>(__ldg(p));
}
// Streaming load: evict-first, for tensors touched exactly once (the taps).
template <typename T> __device__ __forceinline__ float ldcs_f32(const T* p);
template <> __device__ __forceinline__ float ldcs_f32<float>(const float* p) { return __ldcs(p); }
template <> __device__ __forceinline__ float ldcs_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  unsigned short u = __ldcs(reinterpret_cast<const unsigned short*>(p));
  return __uint_as_float(static_cast<uint32_t>(u) << 16);
}
template <> __device__ __forceinline__ float ldcs_f32<__half>(const __half* p) {
  unsigned short u = __ldcs(reinterpret_cast<const unsigned short*>(p));
  return __half2float(__ushort_as_half(u));
}
// Streaming store.
template <typename T> __device__ __forceinline__ void stcs_f32(T* p, float v);
template <> __device__ __forceinline__ void stcs_f32<float>(float* p, float v) { __stcs(p, v); }
template <> __device__ __forceinline__ void stcs_f32<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  __nv_bfloat16 b = __float2bfloat16_rn(v);
  __stcs(reinterpret_cast<unsigned short*>(p), __bfloat16_as_ushort(b));
}
template <> __device__ __forceinline__ void stcs_f32<__half>(__half* p, float v) {
  __half h = __float2half_rn(v);
  __stcs(reinterpret_cast<unsigned short*>(p), __half_as_ushort(h));
}

// Host-side dtype code -> element size in bytes (0 if unknown).
inline int dtype_size(int dt) {
  switch (dt) {
    case DDPM_F32: return 4;
    case DDPM_BF16: return 2;
    case DDPM_F16: return 2;
    default: return 0;
  }
}

inline int max3(int a, int b, int c) { return a > b ? (a > c ? a : c) : (b > c ? b : c); }

}  // namespace ddpm
