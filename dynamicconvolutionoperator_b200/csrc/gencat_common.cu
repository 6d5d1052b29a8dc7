// Host-side helpers of the fused generator kernels and the weight packer.
//
// The generator weight W [3*C*K^2, C] (a Conv2d [3CK^2, C, 1, 1] weight,
// row index (b*C + c)*K^2 + tap, reference `_triton_kernels.py:322`) is
// re-laid-out once per weight version into the exact shared-memory images the
// tensor-core kernels consume, so the kernels stream it with plain 1-D bulk
// copies. Forward image, per chunk q = (cg*3 + b)*K + ki:
//   [part (hi, lo for fp32)][Cp/8 input-channel groups][16*K rows][8]
// with row kj*16 + cl <-> weight row (b*C + cg*16 + cl)*K^2 + ki*K + kj.
// Rows/columns past C are zero (channel padding to a multiple of 16).
#include <mutex>

#include "common.cuh"
#include "gencat.cuh"

namespace ddpm {
namespace gencat {

namespace {
__device__ int g_gencat_status;
}

int check_shape(int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt) {
  DDPM_CHECK_ARG(n >= 1 && c >= 1 && h >= 1 && w >= 1, "sizes must be positive");
  DDPM_CHECK_ARG(ks >= 1 && ks % 2 == 1, "kernel_size must be a positive odd integer, got %d", ks);
  DDPM_CHECK_ARG(d0 >= 1 && d1 >= 1 && d2 >= 1, "dilations must be >= 1");
  DDPM_CHECK_ARG(dtype_size(dt) > 0, "unknown dtype code %d", dt);
  if (c > kMaxChannels)
    return set_error(DDPM_ERR_UNSUPPORTED, "fused generator supports C <= %d (got %d)",
                     kMaxChannels, c);
  if (ks != 1 && ks != 3)
    return set_error(DDPM_ERR_UNSUPPORTED, "fused generator supports K in {1, 3} (got %d)", ks);
  DDPM_CHECK_ARG((long long)n * ((h + kTileH - 1) / kTileH) * ((w + kTileW - 1) / kTileW) <
                     (1LL << 31),
                 "too many tiles");
  return DDPM_OK;
}

int status_ptr(int** out) {
  DDPM_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void**>(out), g_gencat_status));
  return DDPM_OK;
}

int num_sms() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

}  // namespace gencat

namespace {

using gencat::IoTraits;

// One thread writes one 16-byte row (8 input channels) of the forward image.
template <typename T>
__global__ void pack_fwd_kernel(const T* __restrict__ W, typename IoTraits<T>::Op* __restrict__ out,
                                int C, int Cp, int KS) {
  using Op = typename IoTraits<T>::Op;
  constexpr int kParts = IoTraits<T>::kSplit ? 2 : 1;
  const int KK = KS * KS;
  const int kN = 16 * KS;
  const int kg_n = Cp / 8;
  const long long rows_per_chunk = (long long)kParts * kg_n * kN;
  const long long total = (long long)(Cp / 16) * 3 * KS * rows_per_chunk;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int q = (int)(idx / rows_per_chunk);
    int rem = (int)(idx - (long long)q * rows_per_chunk);
    const int part = rem / (kg_n * kN);
    rem -= part * kg_n * kN;
    const int kg = rem / kN;
    const int nrow = rem - kg * kN;
    const int cg = q / (3 * KS);
    const int b = (q / KS) % 3;
    const int ki = q % KS;
    const int kj = nrow / 16;
    const int c = cg * 16 + (nrow % 16);
    const long long m = (long long)(b * C + c) * KK + ki * KS + kj;
    union {
      uint4 u;
      Op e[8];
    } row;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = kg * 8 + e;
      const float w = (c < C && i < C) ? to_f32<T>(W[m * C + i]) : 0.f;
      const Op hi = gencat::op_from<Op>(w);
      row.e[e] = part == 0 ? hi : gencat::op_from<Op>(w - gencat::op_to<Op>(hi));
    }
    reinterpret_cast<uint4*>(out)[idx] = row.u;
  }
}

template <typename T>
int launch_pack(const void* w, void* packed, int c, int ks, cudaStream_t st) {
  const int Cp = gencat::padded_channels(c);
  const int parts = IoTraits<T>::kSplit ? 2 : 1;
  const long long rows = (long long)(Cp / 16) * 3 * ks * parts * (Cp / 8) * 16 * ks;
  const int threads = 256;
  const int blocks = (int)((rows + threads - 1) / threads);
  pack_fwd_kernel<T><<<blocks, threads, 0, st>>>(
      static_cast<const T*>(w), static_cast<typename IoTraits<T>::Op*>(packed), c, Cp, ks);
  DDPM_CHECK_LAUNCH("pack_fwd_kernel");
  return DDPM_OK;
}

}  // namespace

size_t gencat_pack_bytes(int c, int ks, int dt) {
  if (c < 1 || ks < 1 || dtype_size(dt) == 0) return 0;
  const size_t Cp = gencat::padded_channels(c);
  const size_t parts = dt == DDPM_F32 ? 2 : 1;
  return (Cp / 16) * 3 * ks * parts * Cp * 16 * ks * 2;
}

int gencat_pack(const void* w, int c, int ks, int dt, void* packed, size_t packed_bytes,
                cudaStream_t st) {
  int rc = gencat::check_shape(1, c, 1, 1, ks, 1, 1, 1, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG(w && packed, "null pointer");
  DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(packed) & 15u) == 0,
                 "packed weight buffer must be 16-byte aligned");
  if (packed_bytes < gencat_pack_bytes(c, ks, dt))
    return set_error(DDPM_ERR_WORKSPACE, "packed weight buffer too small (%zu < %zu)",
                     packed_bytes, gencat_pack_bytes(c, ks, dt));
  switch (dt) {
    case DDPM_BF16: return launch_pack<__nv_bfloat16>(w, packed, c, ks, st);
    case DDPM_F16: return launch_pack<__half>(w, packed, c, ks, st);
    case DDPM_F32: return launch_pack<float>(w, packed, c, ks, st);
  }
  return set_error(DDPM_ERR_INVALID_ARG, "unknown dtype %d", dt);
}

}  // namespace ddpm
