// Materialised dynamic dilated filter ("dynamic cat"), forward and backward.
//
// Forward (reference `_triton_kernels.py:21-101`):
//   out[n, 0:C]        = x
//   out[n, (b+1)C + c] = sum_tap x[c, p + off(tap)*d_b] * K[n, b, c, tap, p]
// Backward (reference `_triton_kernels.py:104-254`):
//   dK[n, b, c, tap, p] = x[c, p + off*d_b] * g[n, (b+1)C + c, p]
//   dX[n, c, q] = g[n, c, q] + sum_{b,tap} K[n,b,c,tap,q-off*d_b] * g[n,(b+1)C+c,q-off*d_b]
//
// All three kernels are HBM-bound: the taps tensor K / dK (3*K*K planes per
// channel) is streamed exactly once and dominates the traffic. A CTA owns a
// 16-row tile of one (n, c) plane, 32*VEC columns wide; the x plane (forward,
// dK) or the three branch-gradient planes (dX) of that tile plus the dilation
// halo are staged in shared memory as FP32 with zero padding, so shifted
// neighbour reads never touch global memory or need bounds checks.
//
// Forward and dK: each thread owns VEC consecutive pixels (VEC*elt = 16 bytes)
// so every tap plane moves with one 128-bit streaming load/store per thread.
// The staged plane is "column-interleaved" (column cc of a row is stored at
// (cc % VEC) * (row_words / VEC) + cc / VEC): for any tap shift the 32 lanes of
// a warp then read 32 consecutive words, i.e. no bank conflicts.
// dX gathers K at shifted (unaligned) positions, so it keeps one pixel per
// thread per step, with a small register footprint for high occupancy.
#include <initializer_list>

#include "common.cuh"

namespace ddpm {
namespace {

constexpr int kThreadsX = 32;
constexpr int kThreadsY = 8;
constexpr int kRowsPerThread = 2;
constexpr int kTileH = kThreadsY * kRowsPerThread;  // 16
constexpr int kThreads = kThreadsX * kThreadsY;     // 256

struct Dil {
  int d[3];
};

// ---------------------------------------------------------- vector I/O ------
template <typename T, int VEC> struct Vec;
template <> struct Vec<float, 4> {
  using U = float4;
  __device__ static void unpack(const U& u, float (&v)[4]) { v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w; }
  __device__ static U pack(const float (&v)[4]) { return make_float4(v[0], v[1], v[2], v[3]); }
};
template <typename H> struct Vec16 {
  using U = uint4;
  __device__ static void unpack(const U& u, float (&v)[8]) {
    const H* e = reinterpret_cast<const H*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = to_f32<H>(e[i]);
  }
  __device__ static U pack(const float (&v)[8]) {
    union { U u; H e[8]; } r;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.e[i] = from_f32<H>(v[i]);
    return r.u;
  }
};
template <> struct Vec<__nv_bfloat16, 8> : Vec16<__nv_bfloat16> {};
template <> struct Vec<__half, 8> : Vec16<__half> {};

template <typename T, int VEC>
__device__ __forceinline__ void vload_cs(const T* p, float (&v)[VEC]) {
  if constexpr (VEC == 1) {
    v[0] = ldcs_f32<T>(p);
  } else {
    using V = Vec<T, VEC>;
    V::unpack(__ldcs(reinterpret_cast<const typename V::U*>(p)), v);
  }
}
template <typename T, int VEC>
__device__ __forceinline__ void vload(const T* p, float (&v)[VEC]) {
  if constexpr (VEC == 1) {
    v[0] = to_f32<T>(__ldg(p));
  } else {
    using V = Vec<T, VEC>;
    V::unpack(__ldg(reinterpret_cast<const typename V::U*>(p)), v);
  }
}
template <typename T, int VEC>
__device__ __forceinline__ void vstore_cs(T* p, const float (&v)[VEC]) {
  if constexpr (VEC == 1) {
    stcs_f32<T>(p, v[0]);
  } else {
    using V = Vec<T, VEC>;
    __stcs(reinterpret_cast<typename V::U*>(p), V::pack(v));
  }
}

// ------------------------------------------------------- staged planes ------
// Geometry of a staged, zero-padded, column-interleaved plane tile.
template <int VEC>
struct Stage {
  int R;          // halo
  int sub;        // words per interleave sub-row
  int row_words;  // = VEC * sub
  __device__ __forceinline__ int idx(int row, int cc) const {
    return row * row_words + (cc % VEC) * sub + cc / VEC;
  }
};

template <int VEC>
__host__ __device__ __forceinline__ int stage_sub(int R) {
  return (kThreadsX * VEC + 2 * R + VEC - 1) / VEC;
}

template <typename T, int VEC>
__device__ __forceinline__ void stage_plane(float* __restrict__ s, const Stage<VEC>& st,
                                            const T* __restrict__ plane, int H, int W, int h0,
                                            int w0) {
  const int rows = kTileH + 2 * st.R;
  const int cols = st.row_words;
  const int tid = threadIdx.y * kThreadsX + threadIdx.x;
  for (int i = tid; i < rows * cols; i += kThreads) {
    const int rr = i / cols;
    const int cc = i - rr * cols;
    const int gh = h0 - st.R + rr;
    const int gw = w0 - st.R + cc;
    float v = 0.f;
    if (gh >= 0 && gh < H && gw >= 0 && gw < W) v = ldg_f32<T>(plane + (size_t)gh * W + gw);
    s[st.idx(rr, cc)] = v;
  }
}

// ------------------------------------------------------------- forward ------
template <typename TX, typename TK, int KS, int VEC>
__global__ void __launch_bounds__(kThreads, 2)
dyncat_fwd_kernel(const TX* __restrict__ x, const TK* __restrict__ kern, TK* __restrict__ out,
                  int C, int H, int W, Dil dil, int R) {
  extern __shared__ float smem[];
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  const int nc = blockIdx.x;
  const int n = nc / C;
  const int c = nc - n * C;
  const int h0 = blockIdx.y * kTileH;
  const int w0 = blockIdx.z * (kThreadsX * VEC);
  const size_t P = (size_t)H * W;
  const Stage<VEC> st{R, stage_sub<VEC>(R), VEC * stage_sub<VEC>(R)};

  stage_plane<TX, VEC>(smem, st, x + (size_t)nc * P, H, W, h0, w0);
  __syncthreads();

  const size_t kbase = ((size_t)n * 3 * C + c) * KK * P;
  const size_t kbranch = (size_t)C * KK * P;
  TK* obase = out + ((size_t)n * 4 * C + c) * P;
  const size_t obranch = (size_t)C * P;
  const int lx = threadIdx.x * VEC;
  const int w = w0 + lx;
  if (w >= W) return;

#pragma unroll 1
  for (int j = 0; j < kRowsPerThread; ++j) {
    const int ly = threadIdx.y + j * kThreadsY;
    const int h = h0 + ly;
    if (h >= H) break;
    const size_t p = (size_t)h * W + w;
    float center[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) center[v] = smem[st.idx(ly + R, lx + R + v)];
    vstore_cs<TK, VEC>(obase + p, center);
#pragma unroll 1
    for (int b = 0; b < 3; ++b) {
      const int d = dil.d[b];
      const TK* kp = kern + kbase + b * kbranch + p;
      float acc[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
      // All taps of a branch in flight at once for K <= 3; one kernel row at
      // a time for larger K (register budget).
      constexpr int RG = KS <= 3 ? KS : 1;
#pragma unroll
      for (int k0 = 0; k0 < KS; k0 += RG) {
        float kv[RG * KS][VEC];
#pragma unroll
        for (int t = 0; t < RG * KS; ++t)
          vload_cs<TK, VEC>(kp + (size_t)(k0 * KS + t) * P, kv[t]);
#pragma unroll
        for (int ki = k0; ki < k0 + RG; ++ki) {
          const int row = ly + R + (ki - r) * d;
#pragma unroll
          for (int kj = 0; kj < KS; ++kj) {
            const int col = lx + R + (kj - r) * d;
#pragma unroll
            for (int v = 0; v < VEC; ++v)
              acc[v] = fmaf(smem[st.idx(row, col + v)], kv[(ki - k0) * KS + kj][v], acc[v]);
          }
        }
      }
      vstore_cs<TK, VEC>(obase + (b + 1) * obranch + p, acc);
    }
  }
}

// ---------------------------------------------------------------- dK --------
template <typename TX, typename TK, int KS, int VEC>
__global__ void __launch_bounds__(kThreads, 2)
dyncat_bwd_k_kernel(const TX* __restrict__ x, const TK* __restrict__ gout, TK* __restrict__ gk,
                    int C, int H, int W, Dil dil, int R) {
  extern __shared__ float smem[];
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  const int nc = blockIdx.x;
  const int n = nc / C;
  const int c = nc - n * C;
  const int h0 = blockIdx.y * kTileH;
  const int w0 = blockIdx.z * (kThreadsX * VEC);
  const size_t P = (size_t)H * W;
  const Stage<VEC> st{R, stage_sub<VEC>(R), VEC * stage_sub<VEC>(R)};

  stage_plane<TX, VEC>(smem, st, x + (size_t)nc * P, H, W, h0, w0);
  __syncthreads();

  const TK* gbase = gout + ((size_t)n * 4 * C + c) * P;
  const size_t gbranch = (size_t)C * P;
  const size_t kbase = ((size_t)n * 3 * C + c) * KK * P;
  const size_t kbranch = (size_t)C * KK * P;
  const int lx = threadIdx.x * VEC;
  const int w = w0 + lx;
  if (w >= W) return;

#pragma unroll 1
  for (int j = 0; j < kRowsPerThread; ++j) {
    const int ly = threadIdx.y + j * kThreadsY;
    const int h = h0 + ly;
    if (h >= H) break;
    const size_t p = (size_t)h * W + w;
#pragma unroll 1
    for (int b = 0; b < 3; ++b) {
      const int d = dil.d[b];
      float g[VEC];
      vload<TK, VEC>(gbase + (b + 1) * gbranch + p, g);
      TK* kp = gk + kbase + b * kbranch + p;
#pragma unroll
      for (int ki = 0; ki < KS; ++ki) {
        const int row = ly + R + (ki - r) * d;
#pragma unroll
        for (int kj = 0; kj < KS; ++kj) {
          const int col = lx + R + (kj - r) * d;
          float o[VEC];
#pragma unroll
          for (int v = 0; v < VEC; ++v) o[v] = smem[st.idx(row, col + v)] * g[v];
          vstore_cs<TK, VEC>(kp + (size_t)(ki * KS + kj) * P, o);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- dX --------
// One pixel per thread per step (gather at unaligned shifts); the three branch
// gradients of the tile + halo are staged in smem (plain row-major, VEC = 1).
constexpr int kDxTileW = kThreadsX * 4;  // 4 pixel columns per thread, 32 apart

template <typename TX, typename TK, int KS>
__global__ void __launch_bounds__(kThreads, 3)
dyncat_bwd_x_kernel(const TK* __restrict__ kern, const TK* __restrict__ gout, TX* __restrict__ gx,
                    int C, int H, int W, Dil dil, int R) {
  extern __shared__ float smem[];
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  const int nc = blockIdx.x;
  const int n = nc / C;
  const int c = nc - n * C;
  const int h0 = blockIdx.y * kTileH;
  const int w0 = blockIdx.z * kDxTileW;
  const size_t P = (size_t)H * W;
  const int pitch = kDxTileW + 2 * R;
  const int rows = kTileH + 2 * R;
  const int plane_sz = pitch * rows;

  const TK* gbase = gout + ((size_t)n * 4 * C + c) * P;
  const size_t gbranch = (size_t)C * P;
  {
    const int tid = threadIdx.y * kThreadsX + threadIdx.x;
    for (int i = tid; i < 3 * plane_sz; i += kThreads) {
      const int b = i / plane_sz;
      const int k = i - b * plane_sz;
      const int rr = k / pitch;
      const int cc = k - rr * pitch;
      const int gh = h0 - R + rr;
      const int gw = w0 - R + cc;
      float v = 0.f;
      if (gh >= 0 && gh < H && gw >= 0 && gw < W)
        v = ldg_f32<TK>(gbase + (b + 1) * gbranch + (size_t)gh * W + gw);
      smem[i] = v;
    }
  }
  __syncthreads();

  const size_t kbase = ((size_t)n * 3 * C + c) * KK * P;
  const size_t kbranch = (size_t)C * KK * P;
#pragma unroll 1
  for (int j = 0; j < kRowsPerThread; ++j) {
    const int ly = threadIdx.y + j * kThreadsY;
    const int h = h0 + ly;
    if (h >= H) break;
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      const int lx = threadIdx.x + i * kThreadsX;
      const int w = w0 + lx;
      if (w >= W) break;
      const size_t p = (size_t)h * W + w;
      const int sidx = (ly + R) * pitch + (lx + R);
      float acc = to_f32<TK>(gbase[p]);
#pragma unroll
      for (int b = 0; b < 3; ++b) {
        const int d = dil.d[b];
        const TK* kp = kern + kbase + b * kbranch;
        const float* gs = smem + b * plane_sz + sidx;
#pragma unroll
        for (int ki = 0; ki < KS; ++ki) {
          const int dy = (ki - r) * d;
          const bool row_ok = (unsigned)(h - dy) < (unsigned)H;
#pragma unroll
          for (int kj = 0; kj < KS; ++kj) {
            const int dx = (kj - r) * d;
            // Source pixel q - off must lie inside the image (zero padding).
            if (row_ok && (unsigned)(w - dx) < (unsigned)W) {
              const float kv = ldcs_f32<TK>(kp + (size_t)(ki * KS + kj) * P + (p - (ptrdiff_t)dy * W - dx));
              acc = fmaf(kv, gs[-dy * pitch - dx], acc);
            }
          }
        }
      }
      gx[(size_t)nc * P + p] = from_f32<TX>(acc);
    }
  }
}

// ------------------------------------------------------------- launchers ----
template <int VEC>
size_t stage_bytes(int R) {
  return sizeof(float) * (size_t)VEC * stage_sub<VEC>(R) * (kTileH + 2 * R);
}

template <typename F>
int set_smem(F fn, size_t smem) {
  if (smem > 48 * 1024)
    DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  return DDPM_OK;
}

template <typename TX, typename TK, int KS, int VEC>
int launch_fwd(const void* x, const void* k, void* out, int n, int c, int h, int w, Dil dil, int R,
               cudaStream_t st) {
  const size_t smem = stage_bytes<VEC>(R);
  auto fn = dyncat_fwd_kernel<TX, TK, KS, VEC>;
  if (int rc = set_smem(fn, smem)) return rc;
  dim3 grid(n * c, (h + kTileH - 1) / kTileH, (w + kThreadsX * VEC - 1) / (kThreadsX * VEC));
  fn<<<grid, dim3(kThreadsX, kThreadsY), smem, st>>>(static_cast<const TX*>(x),
                                                       static_cast<const TK*>(k),
                                                       static_cast<TK*>(out), c, h, w, dil, R);
  DDPM_CHECK_LAUNCH("dyncat_fwd_kernel");
  return DDPM_OK;
}

template <typename TX, typename TK, int KS, int VEC>
int launch_bwd_k(const void* x, const void* g, void* gk, int n, int c, int h, int w, Dil dil,
                 int R, cudaStream_t st) {
  const size_t smem = stage_bytes<VEC>(R);
  auto fn = dyncat_bwd_k_kernel<TX, TK, KS, VEC>;
  if (int rc = set_smem(fn, smem)) return rc;
  dim3 grid(n * c, (h + kTileH - 1) / kTileH, (w + kThreadsX * VEC - 1) / (kThreadsX * VEC));
  fn<<<grid, dim3(kThreadsX, kThreadsY), smem, st>>>(static_cast<const TX*>(x),
                                                       static_cast<const TK*>(g),
                                                       static_cast<TK*>(gk), c, h, w, dil, R);
  DDPM_CHECK_LAUNCH("dyncat_bwd_k_kernel");
  return DDPM_OK;
}

template <typename TX, typename TK, int KS>
int launch_bwd_x(const void* k, const void* g, void* gx, int n, int c, int h, int w, Dil dil,
                 int R, cudaStream_t st) {
  const size_t smem = sizeof(float) * 3 * (size_t)(kDxTileW + 2 * R) * (kTileH + 2 * R);
  auto fn = dyncat_bwd_x_kernel<TX, TK, KS>;
  if (int rc = set_smem(fn, smem)) return rc;
  dim3 grid(n * c, (h + kTileH - 1) / kTileH, (w + kDxTileW - 1) / kDxTileW);
  fn<<<grid, dim3(kThreadsX, kThreadsY), smem, st>>>(static_cast<const TK*>(k),
                                                       static_cast<const TK*>(g),
                                                       static_cast<TX*>(gx), c, h, w, dil, R);
  DDPM_CHECK_LAUNCH("dyncat_bwd_x_kernel");
  return DDPM_OK;
}

// 16-byte vectors need every row start aligned: W a multiple of VEC and
// 16-byte aligned base pointers.
inline bool vec_ok(int w, int vec, std::initializer_list<const void*> ptrs) {
  if (w % vec) return false;
  for (const void* p : ptrs)
    if (p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15u)) return false;
  return true;
}

template <typename TX, typename TK, int KS>
int fwd_ks(const void* x, const void* k, void* out, int n, int c, int h, int w, Dil dil, int R,
           cudaStream_t st) {
  constexpr int V = 16 / sizeof(TK);
  if (sizeof(TX) == sizeof(TK) && vec_ok(w, V, {x, k, out}))
    return launch_fwd<TX, TK, KS, V>(x, k, out, n, c, h, w, dil, R, st);
  if (sizeof(TX) != sizeof(TK) && vec_ok(w, V, {k, out}))
    return launch_fwd<TX, TK, KS, V>(x, k, out, n, c, h, w, dil, R, st);
  return launch_fwd<TX, TK, KS, 1>(x, k, out, n, c, h, w, dil, R, st);
}

template <typename TX, typename TK>
int dispatch_fwd(int ks, const void* x, const void* k, void* out, int n, int c, int h, int w,
                 Dil dil, int R, cudaStream_t st) {
  switch (ks) {
    case 1: return fwd_ks<TX, TK, 1>(x, k, out, n, c, h, w, dil, R, st);
    case 3: return fwd_ks<TX, TK, 3>(x, k, out, n, c, h, w, dil, R, st);
    case 5: return fwd_ks<TX, TK, 5>(x, k, out, n, c, h, w, dil, R, st);
    case 7: return fwd_ks<TX, TK, 7>(x, k, out, n, c, h, w, dil, R, st);
  }
  return set_error(DDPM_ERR_UNSUPPORTED, "kernel_size %d not supported (1, 3, 5, 7)", ks);
}

template <typename TX, typename TK, int KS>
int bwd_ks(const void* x, const void* k, const void* g, void* gx, void* gk, int n, int c, int h,
           int w, Dil dil, int R, cudaStream_t st) {
  constexpr int V = 16 / sizeof(TK);
  if (gk != nullptr) {
    const int rc = vec_ok(w, V, {g, gk})
                       ? launch_bwd_k<TX, TK, KS, V>(x, g, gk, n, c, h, w, dil, R, st)
                       : launch_bwd_k<TX, TK, KS, 1>(x, g, gk, n, c, h, w, dil, R, st);
    if (rc) return rc;
  }
  if (gx != nullptr) return launch_bwd_x<TX, TK, KS>(k, g, gx, n, c, h, w, dil, R, st);
  return DDPM_OK;
}

template <typename TX, typename TK>
int dispatch_bwd(int ks, const void* x, const void* k, const void* g, void* gx, void* gk, int n,
                 int c, int h, int w, Dil dil, int R, cudaStream_t st) {
  switch (ks) {
    case 1: return bwd_ks<TX, TK, 1>(x, k, g, gx, gk, n, c, h, w, dil, R, st);
    case 3: return bwd_ks<TX, TK, 3>(x, k, g, gx, gk, n, c, h, w, dil, R, st);
    case 5: return bwd_ks<TX, TK, 5>(x, k, g, gx, gk, n, c, h, w, dil, R, st);
    case 7: return bwd_ks<TX, TK, 7>(x, k, g, gx, gk, n, c, h, w, dil, R, st);
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
  DDPM_CHECK_ARG((long long)n * c <= 2147483647LL && h <= 65535 * kTileH && w <= 65535 * 32,
                 "grid too large (n*c=%lld, h=%d, w=%d)", (long long)n * c, h, w);
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
