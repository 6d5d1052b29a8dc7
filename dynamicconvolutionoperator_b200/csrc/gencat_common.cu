// Host-side helpers of the fused generator kernels and the weight packer.
//
// The generator weight W [3*C*K^2, C] (a Conv2d [3CK^2, C, 1, 1] weight,
// row index (b*C + c)*K^2 + tap, reference `_triton_kernels.py:322`) and its
// bias are re-laid-out once per weight version into the exact shared-memory
// operand images the tensor-core kernels consume, so the kernels stream them
// with plain 1-D bulk copies. Three images, back to back (see gencat.cuh,
// PackLayout): forward chunks, dX chunks and the transposed dY groups. Each
// 16-byte row holds 8 consecutive K-dimension values; fp32 weights are stored
// as a bf16 hi image followed by a bf16 lo (residual) image.
#include <mutex>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "gencat.cuh"
#include "tmap.cuh"

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
  if (ks != 1 && ks != 3 && ks != 5)
    return set_error(DDPM_ERR_UNSUPPORTED, "fused generator supports K in {1, 3, 5} (got %d)",
                     ks);
  if ((ks / 2) * max3(d0, d1, d2) > fwd_max_halo(ks))
    return set_error(DDPM_ERR_UNSUPPORTED,
                     "fused generator supports dilation halos <= %d at K = %d", fwd_max_halo(ks),
                     ks);
  DDPM_CHECK_ARG((long long)n * h * ((w + 127) / 128) < (1LL << 31), "too many tiles");
  return DDPM_OK;
}

int check_shape_bwd(int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt) {
  const int rc = check_shape(n, c, h, w, ks, d0, d1, d2, dt);
  if (rc) return rc;
  if (ks > 3)
    return set_error(DDPM_ERR_UNSUPPORTED, "fused dY + dW supports K in {1, 3} (got %d)", ks);
  return DDPM_OK;
}

int status_ptr(int** out) {
  DDPM_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void**>(out), g_gencat_status));
  return DDPM_OK;
}

// Reads (and with `reset` clears) the device-side failure code of the current
// device: 0, or the code of the first bounded wait that gave up. Synchronises
// the device; meant for tests and error paths, not for the step loop.
int read_status(int reset, int* code) {
  DDPM_CHECK_ARG(code != nullptr, "null pointer");
  DDPM_CUDA_TRY(cudaDeviceSynchronize());
  DDPM_CUDA_TRY(cudaMemcpyFromSymbol(code, g_gencat_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    DDPM_CUDA_TRY(cudaMemcpyToSymbol(g_gencat_status, &zero, sizeof(int)));
  }
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

int max_smem_optin() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 232448;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        v <= 0)
      v = 232448;
    cache[dev] = v;
  }
  return cache[dev];
}

}  // namespace gencat

namespace {

using gencat::IoTraits;
using gencat::PackLayout;

// One thread writes one 16-byte row (8 K-dimension values) of one image.
template <typename T>
__global__ void pack_kernel(const T* __restrict__ W, const T* __restrict__ bias,
                            typename IoTraits<T>::Op* __restrict__ out, PackLayout L) {
  using Op = typename IoTraits<T>::Op;
  const int C = L.C, KS = L.KS, KK = KS * KS;
  const long long total = L.fwd_rows + L.bx_rows + L.by_rows;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    long long m = -1;   // weight row
    int k0 = 0;         // first K-dimension index of this 16-byte row
    int part = 0;
    bool kdim_is_row = false;  // dY image: the K dimension runs over weight rows
    int i_col = 0;             // dY image: the weight column (input channel)
    if (idx < L.fwd_rows) {
      // [cg][part][Ck/8][3*BC][8]; row = b*BC + tap*G + cl (zero past K^2*G)
      const int G = gencat::fwd_cg(KS, L.parts == 2);
      const int BC = gencat::fwd_branch_cols(KS, L.parts == 2);
      const int nrow = 3 * BC;
      const long long per_cg = (long long)L.parts * (L.Ck / 8) * nrow;
      const int cg = (int)(idx / per_cg);
      int rem = (int)(idx - cg * per_cg);
      part = rem / ((L.Ck / 8) * nrow);
      rem -= part * (L.Ck / 8) * nrow;
      const int kg = rem / nrow;
      const int row = rem - kg * nrow;
      const int b = row / BC, tap = (row % BC) / G, c = cg * G + row % G;
      if (c < C && tap < KK) m = (long long)(b * C + c) * KK + tap;
      k0 = kg * 8;
    } else if (idx < L.fwd_rows + L.bx_rows) {
      // [q][part][Ck/8][Cp][8]; q = b*K^2 + tap; row = c
      const long long j = idx - L.fwd_rows;
      const long long per_chunk = (long long)L.parts * (L.Ck / 8) * L.Cp;
      const int q = (int)(j / per_chunk);
      int rem = (int)(j - q * per_chunk);
      part = rem / ((L.Ck / 8) * L.Cp);
      rem -= part * (L.Ck / 8) * L.Cp;
      const int kg = rem / L.Cp;
      const int c = rem - kg * L.Cp;
      const int b = q / KK, tap = q % KK;
      if (c < C) m = (long long)(b * C + c) * KK + tap;
      k0 = kg * 8;
    } else {
      // [g][part][16 row groups][Cp][8 rows]; g = cg16*octets + octet,
      // group row = j*16 + cl with slot = octet*8 + j
      const long long j = idx - L.fwd_rows - L.bx_rows;
      const long long per_group = (long long)L.parts * 16 * L.Cp;
      const int g = (int)(j / per_group);
      int rem = (int)(j - g * per_group);
      part = rem / (16 * L.Cp);
      rem -= part * 16 * L.Cp;
      const int rg = rem / L.Cp;
      i_col = rem - rg * L.Cp;
      k0 = rg * 8;
      kdim_is_row = true;
      m = g;  // group index, resolved per element below
    }
    union {
      uint4 u;
      Op e[8];
    } row;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float w = 0.f;
      if (!kdim_is_row) {
        const int i = k0 + e;
        if (m >= 0) {
          if (i < C) w = to_f32<T>(W[m * C + i]);
          else if (i == L.bias_col) w = to_f32<T>(bias[m]);
        }
      } else {
        const int grow = k0 + e;                 // row within the 128-row group
        const int octets = (3 * KK + 7) / 8;
        const int slot = ((int)m % octets) * 8 + grow / 16;
        const int c = ((int)m / octets) * 16 + grow % 16;
        if (slot < 3 * KK && c < C && i_col < C) {
          const int b = slot / KK, tap = slot % KK;
          w = to_f32<T>(W[((long long)(b * C + c) * KK + tap) * C + i_col]);
        }
      }
      const Op hi = gencat::op_from<Op>(w);
      row.e[e] = part == 0 ? hi : gencat::op_from<Op>(w - gencat::op_to<Op>(hi));
    }
    reinterpret_cast<uint4*>(out)[idx] = row.u;
  }
}

template <typename T>
int launch_pack(const void* w, const void* bias, void* packed, const PackLayout& L,
                cudaStream_t st) {
  const long long rows = L.fwd_rows + L.bx_rows + L.by_rows;
  const int threads = 256;
  const long long want = (rows + threads - 1) / threads;
  const int blocks = (int)(want < 4096 ? want : 4096);
  pack_kernel<T><<<blocks, threads, 0, st>>>(static_cast<const T*>(w), static_cast<const T*>(bias),
                                            static_cast<typename IoTraits<T>::Op*>(packed), L);
  DDPM_CHECK_LAUNCH("pack_kernel");
  return DDPM_OK;
}

}  // namespace

size_t gencat_pack_bytes(int c, int ks, int dt) {
  if (c < 1 || c > gencat::kMaxChannels || ks < 1 || dtype_size(dt) == 0) return 0;
  return gencat::PackLayout::make(c, ks, dt).total_bytes();
}

int gencat_pack(const void* w, const void* bias, int c, int ks, int dt, void* packed,
                size_t packed_bytes, cudaStream_t st) {
  int rc = gencat::check_shape(1, c, 1, 1, ks, 1, 1, 1, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG(w && bias && packed, "null pointer");
  DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(packed) & 15u) == 0,
                 "packed weight buffer must be 16-byte aligned");
  const PackLayout L = PackLayout::make(c, ks, dt);
  if (packed_bytes < L.total_bytes())
    return set_error(DDPM_ERR_WORKSPACE, "packed weight buffer too small (%zu < %zu)",
                     packed_bytes, L.total_bytes());
  switch (dt) {
    case DDPM_BF16: return launch_pack<__nv_bfloat16>(w, bias, packed, L, st);
    case DDPM_F16: return launch_pack<__half>(w, bias, packed, L, st);
    case DDPM_F32: return launch_pack<float>(w, bias, packed, L, st);
  }
  return set_error(DDPM_ERR_INVALID_ARG, "unknown dtype %d", dt);
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                CUtensorMapSwizzle swizzle) {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (encode == nullptr)
    return set_error(DDPM_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides[i];
  }
  const CUresult r = encode(map, type, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DDPM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DDPM_OK;
}

}  // namespace ddpm
