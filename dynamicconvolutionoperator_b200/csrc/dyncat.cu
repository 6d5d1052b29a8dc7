// Materialised dynamic dilated filter ("dynamic cat"), forward and backward.
//
// Forward (reference `_triton_kernels.py:21-101`):
//   out[n, 0:C]        = x
//   out[n, (b+1)C + c] = sum_tap x[c, p + off(tap)*d_b] * K[n, b, c, tap, p]
// Backward (reference `_triton_kernels.py:104-254`):
//   dK[n, b, c, tap, p] = x[c, p + off*d_b] * g[n, (b+1)C + c, p]
//   dX[n, c, q] = g[n, c, q] + sum_{b,tap} K[n,b,c,tap,q-off*d_b] * g[n,(b+1)C+c,q-off*d_b]
//
// Both are HBM-bound: the taps tensor K / dK (3*K*K planes per channel) is
// streamed exactly once, everything else is staged on chip. One CTA owns a
// 16-row x 128-column tile of one (n, c) plane; the x (and for the backward
// the three branch-gradient) planes of that tile plus the dilation halo sit in
// shared memory as FP32 with zero padding, so every shifted neighbour read is
// a bank-conflict-free LDS and no per-tap bounds check touches global memory.
// Each thread owns 8 pixels (4 columns 32 apart x 2 rows 8 apart), so every
// warp-wide tap load/store is one contiguous 32-pixel run.
#include "common.cuh"

namespace ddpm {
namespace {

constexpr int kThreadsX = 32;
constexpr int kThreadsY = 8;
constexpr int kPixX = 4;                       // columns per thread
constexpr int kPixY = 2;                       // rows per thread
constexpr int kTileW = kThreadsX * kPixX;      // 128
constexpr int kTileH = kThreadsY * kPixY;      // 16

struct Dil {
  int d[3];
};

// Stage plane[h0-R : h0+TH+R, w0-R : w0+TW+R] into smem as FP32, zero padded.
template <typename T>
__device__ __forceinline__ void stage_tile(float* __restrict__ s, const T* __restrict__ plane,
                                           int H, int W, int h0, int w0, int R, int pitch,
                                           int rows) {
  const int tid = threadIdx.y * kThreadsX + threadIdx.x;
  const int total = rows * pitch;
  for (int i = tid; i < total; i += kThreadsX * kThreadsY) {
    const int rr = i / pitch;
    const int cc = i - rr * pitch;
    const int gh = h0 - R + rr;
    const int gw = w0 - R + cc;
    float v = 0.f;
    if (gh >= 0 && gh < H && gw >= 0 && gw < W) v = ldg_f32<T>(plane + (size_t)gh * W + gw);
    s[i] = v;
  }
}

template <typename TX, typename TK, int KS>
__global__ void __launch_bounds__(kThreadsX * kThreadsY)
dyncat_fwd_kernel(const TX* __restrict__ x, const TK* __restrict__ kern, TK* __restrict__ out,
                  int C, int H, int W, Dil dil, int R) {
  extern __shared__ float smem[];
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  const int nc = blockIdx.z;
  const int n = nc / C;
  const int c = nc - n * C;
  const int h0 = blockIdx.y * kTileH;
  const int w0 = blockIdx.x * kTileW;
  const int pitch = kTileW + 2 * R;
  const int rows = kTileH + 2 * R;
  const size_t P = (size_t)H * W;

  const TX* xplane = x + (size_t)nc * P;
  stage_tile<TX>(smem, xplane, H, W, h0, w0, R, pitch, rows);
  __syncthreads();

  const size_t kbase = (size_t)n * 3 * C * KK * P + (size_t)c * KK * P;  // branch 0, tap 0
  const size_t kbranch = (size_t)C * KK * P;
  TK* obase = out + (size_t)n * 4 * C * P + (size_t)c * P;
  const size_t obranch = (size_t)C * P;

#pragma unroll 1
  for (int j = 0; j < kPixY; ++j) {
    const int ly = threadIdx.y + j * kThreadsY;
    const int h = h0 + ly;
    if (h >= H) break;
#pragma unroll 1
    for (int i = 0; i < kPixX; ++i) {
      const int lx = threadIdx.x + i * kThreadsX;
      const int w = w0 + lx;
      if (w >= W) break;
      const size_t p = (size_t)h * W + w;
      const float* srow = smem + (size_t)(ly + R) * pitch + (lx + R);
      stcs_f32<TK>(obase + p, srow[0]);
#pragma unroll
      for (int b = 0; b < 3; ++b) {
        const int d = dil.d[b];
        const TK* kp = kern + kbase + b * kbranch + p;
        float acc = 0.f;
#pragma unroll
        for (int ki = 0; ki < KS; ++ki) {
#pragma unroll
          for (int kj = 0; kj < KS; ++kj) {
            const int tap = ki * KS + kj;
            const float kv = ldcs_f32<TK>(kp + (size_t)tap * P);
            acc = fmaf(srow[(ki - r) * d * pitch + (kj - r) * d], kv, acc);
          }
        }
        stcs_f32<TK>(obase + (b + 1) * obranch + p, acc);
      }
    }
  }
}

// One launch produces dK (aligned, streaming stores) and dX (gather of the
// shifted taps). smem holds x and the three branch gradients with halo.
template <typename TX, typename TK, int KS>
__global__ void __launch_bounds__(kThreadsX * kThreadsY)
dyncat_bwd_kernel(const TX* __restrict__ x, const TK* __restrict__ kern,
                  const TK* __restrict__ gout, TX* __restrict__ gx, TK* __restrict__ gk,
                  int C, int H, int W, Dil dil, int R) {
  extern __shared__ float smem[];
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  const int nc = blockIdx.z;
  const int n = nc / C;
  const int c = nc - n * C;
  const int h0 = blockIdx.y * kTileH;
  const int w0 = blockIdx.x * kTileW;
  const int pitch = kTileW + 2 * R;
  const int rows = kTileH + 2 * R;
  const int plane_sz = pitch * rows;
  const size_t P = (size_t)H * W;

  float* xs = smem;                 // x tile
  float* gs = smem + plane_sz;      // 3 branch-gradient tiles
  const TK* gbase = gout + (size_t)n * 4 * C * P + (size_t)c * P;
  const size_t gbranch = (size_t)C * P;
  if (gk != nullptr) stage_tile<TX>(xs, x + (size_t)nc * P, H, W, h0, w0, R, pitch, rows);
#pragma unroll
  for (int b = 0; b < 3; ++b)
    stage_tile<TK>(gs + b * plane_sz, gbase + (b + 1) * gbranch, H, W, h0, w0, R, pitch, rows);
  __syncthreads();

  const size_t kbase = (size_t)n * 3 * C * KK * P + (size_t)c * KK * P;
  const size_t kbranch = (size_t)C * KK * P;

#pragma unroll 1
  for (int j = 0; j < kPixY; ++j) {
    const int ly = threadIdx.y + j * kThreadsY;
    const int h = h0 + ly;
    if (h >= H) break;
#pragma unroll 1
    for (int i = 0; i < kPixX; ++i) {
      const int lx = threadIdx.x + i * kThreadsX;
      const int w = w0 + lx;
      if (w >= W) break;
      const size_t p = (size_t)h * W + w;
      const int sidx = (ly + R) * pitch + (lx + R);
      if (gk != nullptr) {
#pragma unroll
        for (int b = 0; b < 3; ++b) {
          const int d = dil.d[b];
          const float g = gs[b * plane_sz + sidx];
          TK* kp = gk + kbase + b * kbranch + p;
#pragma unroll
          for (int ki = 0; ki < KS; ++ki) {
#pragma unroll
            for (int kj = 0; kj < KS; ++kj) {
              const int tap = ki * KS + kj;
              const float xv = xs[sidx + (ki - r) * d * pitch + (kj - r) * d];
              stcs_f32<TK>(kp + (size_t)tap * P, xv * g);
            }
          }
        }
      }
      if (gx != nullptr) {
        float acc = to_f32<TK>(gbase[p]);
#pragma unroll
        for (int b = 0; b < 3; ++b) {
          const int d = dil.d[b];
          const TK* kp = kern + kbase + b * kbranch;
#pragma unroll
          for (int ki = 0; ki < KS; ++ki) {
            const int dy = (ki - r) * d;
            const int hs = h - dy;
#pragma unroll
            for (int kj = 0; kj < KS; ++kj) {
              const int dx = (kj - r) * d;
              const int ws = w - dx;
              const int tap = ki * KS + kj;
              // Source pixel q - off must lie inside the image (zero padding).
              if (hs >= 0 && hs < H && ws >= 0 && ws < W) {
                const float kv = ldcs_f32<TK>(kp + (size_t)tap * P + (size_t)hs * W + ws);
                acc = fmaf(kv, gs[b * plane_sz + sidx - dy * pitch - dx], acc);
              }
            }
          }
        }
        gx[(size_t)nc * P + p] = from_f32<TX>(acc);
      }
    }
  }
}

template <typename TX, typename TK, int KS>
int launch_fwd(const void* x, const void* k, void* out, int n, int c, int h, int w,
               Dil dil, int R, cudaStream_t st) {
  const size_t smem = sizeof(float) * (size_t)(kTileW + 2 * R) * (kTileH + 2 * R);
  auto fn = dyncat_fwd_kernel<TX, TK, KS>;
  if (smem > 48 * 1024)
    DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((w + kTileW - 1) / kTileW, (h + kTileH - 1) / kTileH, n * c);
  dim3 block(kThreadsX, kThreadsY);
  fn<<<grid, block, smem, st>>>(static_cast<const TX*>(x), static_cast<const TK*>(k),
                                static_cast<TK*>(out), c, h, w, dil, R);
  DDPM_CHECK_LAUNCH("dyncat_fwd_kernel");
  return DDPM_OK;
}

template <typename TX, typename TK, int KS>
int launch_bwd(const void* x, const void* k, const void* g, void* gx, void* gk, int n, int c,
               int h, int w, Dil dil, int R, cudaStream_t st) {
  const size_t smem = sizeof(float) * 4 * (size_t)(kTileW + 2 * R) * (kTileH + 2 * R);
  auto fn = dyncat_bwd_kernel<TX, TK, KS>;
  if (smem > 48 * 1024)
    DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((w + kTileW - 1) / kTileW, (h + kTileH - 1) / kTileH, n * c);
  dim3 block(kThreadsX, kThreadsY);
  fn<<<grid, block, smem, st>>>(static_cast<const TX*>(x), static_cast<const TK*>(k),
                                static_cast<const TK*>(g), static_cast<TX*>(gx),
                                static_cast<TK*>(gk), c, h, w, dil, R);
  DDPM_CHECK_LAUNCH("dyncat_bwd_kernel");
  return DDPM_OK;
}

template <typename TX, typename TK>
int dispatch_fwd(int ks, const void* x, const void* k, void* out, int n, int c, int h, int w,
                 Dil dil, int R, cudaStream_t st) {
  switch (ks) {
    case 1: return launch_fwd<TX, TK, 1>(x, k, out, n, c, h, w, dil, R, st);
    case 3: return launch_fwd<TX, TK, 3>(x, k, out, n, c, h, w, dil, R, st);
    case 5: return launch_fwd<TX, TK, 5>(x, k, out, n, c, h, w, dil, R, st);
    case 7: return launch_fwd<TX, TK, 7>(x, k, out, n, c, h, w, dil, R, st);
  }
  return set_error(DDPM_ERR_UNSUPPORTED, "kernel_size %d not supported (1, 3, 5, 7)", ks);
}

template <typename TX, typename TK>
int dispatch_bwd(int ks, const void* x, const void* k, const void* g, void* gx, void* gk, int n,
                 int c, int h, int w, Dil dil, int R, cudaStream_t st) {
  switch (ks) {
    case 1: return launch_bwd<TX, TK, 1>(x, k, g, gx, gk, n, c, h, w, dil, R, st);
    case 3: return launch_bwd<TX, TK, 3>(x, k, g, gx, gk, n, c, h, w, dil, R, st);
    case 5: return launch_bwd<TX, TK, 5>(x, k, g, gx, gk, n, c, h, w, dil, R, st);
    case 7: return launch_bwd<TX, TK, 7>(x, k, g, gx, gk, n, c, h, w, dil, R, st);
  }
  return set_error(DDPM_ERR_UNSUPPORTED, "kernel_size %d not supported (1, 3, 5, 7)", ks);
}

int check_common(const void* x, int xdt, const void* k, int kdt, int n, int c, int h, int w,
                 int ks, int d0, int d1, int d2) {
  DDPM_CHECK_ARG(x != nullptr && k != nullptr, "null input pointer");
  DDPM_CHECK_ARG(dtype_size(xdt) > 0 && dtype_size(kdt) > 0, "unknown dtype code (%d, %d)", xdt,
                 kdt);
  DDPM_CHECK_ARG(n >= 1 && c >= 1 && h >= 1 && w >= 1, "sizes must be positive (n=%d c=%d h=%d w=%d)",
                 n, c, h, w);
  DDPM_CHECK_ARG(ks >= 1 && (ks % 2) == 1, "kernel_size must be a positive odd integer, got %d", ks);
  DDPM_CHECK_ARG(d0 >= 1 && d1 >= 1 && d2 >= 1, "dilations must be >= 1");
  DDPM_CHECK_ARG((long long)n * c <= 2147483647LL && h <= 65535 * kTileH,
                 "grid too large (n*c=%lld, h=%d)", (long long)n * c, h);
  DDPM_CHECK_ARG((ks / 2) * max3(d0, d1, d2) <= 64, "dilation halo too large");
  return DDPM_OK;
}

}  // namespace

// Pairs supported: identical dtypes, or fp32 x with a half-precision kernel
// tensor (the autocast case: the generator ran in bf16/fp16, x stayed fp32).
#define DDPM_DYNCAT_DISPATCH(FN, ...)                                                        \
  if (xdt == kdt && xdt == DDPM_F32) return FN<float, float>(__VA_ARGS__);                    \
  if (xdt == kdt && xdt == DDPM_BF16) return FN<__nv_bfloat16, __nv_bfloat16>(__VA_ARGS__);   \
  if (xdt == kdt && xdt == DDPM_F16) return FN<__half, __half>(__VA_ARGS__);                  \
  if (xdt == DDPM_F32 && kdt == DDPM_BF16) return FN<float, __nv_bfloat16>(__VA_ARGS__);      \
  if (xdt == DDPM_F32 && kdt == DDPM_F16) return FN<float, __half>(__VA_ARGS__);              \
  return set_error(DDPM_ERR_UNSUPPORTED, "dtype pair (x=%d, kernels=%d) not supported", xdt, kdt);

int dyncat_fwd(const void* x, int xdt, const void* k, int kdt, void* out, int n, int c, int h,
               int w, int ks, int d0, int d1, int d2, cudaStream_t st) {
  int rc = check_common(x, xdt, k, kdt, n, c, h, w, ks, d0, d1, d2);
  if (rc) return rc;
  DDPM_CHECK_ARG(out != nullptr, "null output pointer");
  Dil dil{{d0, d1, d2}};
  const int R = (ks / 2) * max3(d0, d1, d2);
  DDPM_DYNCAT_DISPATCH(dispatch_fwd, ks, x, k, out, n, c, h, w, dil, R, st)
}

int dyncat_bwd(const void* x, int xdt, const void* k, const void* g, int kdt, void* gx, void* gk,
               int n, int c, int h, int w, int ks, int d0, int d1, int d2, cudaStream_t st) {
  int rc = check_common(x, xdt, k, kdt, n, c, h, w, ks, d0, d1, d2);
  if (rc) return rc;
  DDPM_CHECK_ARG(g != nullptr, "null grad_out pointer");
  if (gx == nullptr && gk == nullptr) return DDPM_OK;
  Dil dil{{d0, d1, d2}};
  const int R = (ks / 2) * max3(d0, d1, d2);
  DDPM_DYNCAT_DISPATCH(dispatch_bwd, ks, x, k, g, gx, gk, n, c, h, w, dil, R, st)
}

}  // namespace ddpm
