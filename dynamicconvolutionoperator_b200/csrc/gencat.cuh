// Shared definitions of the fused generator kernels (forward and backward):
// I/O traits, tile geometry, operand staging helpers, bounded-wait helpers.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace ddpm {
namespace gencat {

// 128 output pixels per MMA tile, as an 8 x 16 block of one image.
constexpr int kTileM = 128;
constexpr int kTileH = 8;
constexpr int kTileW = 16;
constexpr int kMaxChannels = 64;
// Upper bound for any single mbarrier wait before the kernel gives up, records
// an error and unwinds (no legitimate wait in these kernels lasts this long).
constexpr uint64_t kWaitNs = 2000000000ull;

// I/O element type -> tensor-core operand type and rounding of generated taps.
template <typename T> struct IoTraits;
template <> struct IoTraits<__nv_bfloat16> {
  using Op = __nv_bfloat16;
  static constexpr bool kSplit = false;
  static constexpr bool kBf16 = true;
  // The reference rounds generated taps to the I/O dtype before use
  // (`_triton_kernels.py:332-335`), as PyTorch's bf16 generator output would be.
  __device__ static __forceinline__ float round_io(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
};
template <> struct IoTraits<__half> {
  using Op = __half;
  static constexpr bool kSplit = false;
  static constexpr bool kBf16 = false;
  __device__ static __forceinline__ float round_io(float v) {
    return __half2float(__float2half_rn(v));
  }
};
template <> struct IoTraits<float> {
  // FP32 operands are carried as bf16 hi + lo pairs (3 MMAs per step).
  using Op = __nv_bfloat16;
  static constexpr bool kSplit = true;
  static constexpr bool kBf16 = true;
  __device__ static __forceinline__ float round_io(float v) { return v; }
};

inline int padded_channels(int c) { return (c + 15) / 16 * 16; }

__device__ __forceinline__ void tile_origin(int tile, int tiles_w, int tiles_h, int& n, int& h0,
                                            int& w0) {
  const int per_img = tiles_w * tiles_h;
  n = tile / per_img;
  const int t = tile - n * per_img;
  const int th = t / tiles_w;
  h0 = th * kTileH;
  w0 = (t - th * tiles_w) * kTileW;
}

__device__ __forceinline__ void fail(volatile int* abort_flag, int* status, int code) {
  *abort_flag = 1;
  atomicCAS(status, 0, code);
}

// Warp-uniform bounded wait (all lanes see the same outcome).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag) {
  const bool ok = tc::mbar_wait(bar, parity, abort_flag, kWaitNs);
  return __all_sync(0xffffffffu, ok);
}

// Load 8 consecutive pixels y[n, c, h, w0 .. w0+7] as floats, zero outside
// the image / channel range. Vector path when the run is in range and 16-byte
// aligned.
template <typename T>
__device__ __forceinline__ void load8(const T* __restrict__ base, int n, int c, int C, int H,
                                      int W, int h, int w0, float (&v)[8]) {
  if (c >= C || h >= H || w0 >= W) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    return;
  }
  const T* src = base + ((size_t)(n * C + c) * H + h) * W + w0;
  const bool full = (w0 + 8 <= W) &&
                    ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
  if constexpr (sizeof(T) == 2) {
    if (full) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = to_f32<T>(e[i]);
      return;
    }
  } else {
    if (full) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src));
      const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = (w0 + i < W) ? to_f32<T>(__ldg(src + i)) : 0.f;
}

template <typename Op> __device__ __forceinline__ Op op_from(float v);
template <> __device__ __forceinline__ __nv_bfloat16 op_from<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half op_from<__half>(float v) {
  return __float2half_rn(v);
}
template <typename Op> __device__ __forceinline__ float op_to(Op v);
template <> __device__ __forceinline__ float op_to<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <> __device__ __forceinline__ float op_to<__half>(__half v) { return __half2float(v); }

// Store 8 floats as one 16-byte operand row; with kSplit also the residual
// (v - hi) as a second row at `dst_lo`.
template <typename Op, bool kSplit>
__device__ __forceinline__ void store8_split(uint8_t* dst_hi, uint8_t* dst_lo,
                                             const float (&v)[8]) {
  union {
    uint4 u;
    Op e[8];
  } hi, lo;
#pragma unroll
  for (int i = 0; i < 8; ++i) hi.e[i] = op_from<Op>(v[i]);
  *reinterpret_cast<uint4*>(dst_hi) = hi.u;
  if constexpr (kSplit) {
#pragma unroll
    for (int i = 0; i < 8; ++i) lo.e[i] = op_from<Op>(v[i] - op_to<Op>(hi.e[i]));
    *reinterpret_cast<uint4*>(dst_lo) = lo.u;
  }
}

// Host helpers (gencat_common.cu).
int check_shape(int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt);
int status_ptr(int** out);
int num_sms();

}  // namespace gencat
}  // namespace ddpm
