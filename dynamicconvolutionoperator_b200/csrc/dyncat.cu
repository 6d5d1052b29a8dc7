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
// dX gathers K at shifted (unaligned) positions. Its vector kernel keeps the
// same layout and builds each shifted VEC-window from the two aligned 16-byte
// chunks that cover it; the scalar kernel (one pixel per thread per step)
// serves rows that are not 16-byte aligned and very large halos.
#include <initializer_list>
#include <type_traits>

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

// Staging issues kStageBatch independent loads per thread before the first
// shared-memory store: a load-then-store loop would leave one global load in
// flight per thread and make the staging phase latency-bound. Every load reads
// a clamped in-image address and is zeroed afterwards when the staged position
// lies in the padding, so no load is predicated away.
constexpr int kStageBatch = 8;

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return min(max(v, lo), hi); }

template <typename T, int VEC>
__device__ __forceinline__ void stage_plane(float* __restrict__ s, const Stage<VEC>& st,
                                            const T* __restrict__ plane, int H, int W, int h0,
                                            int w0) {
  const int rows = kTileH + 2 * st.R;
  const int cols = st.row_words;
  const int total = rows * cols;
  const int tid = threadIdx.y * kThreadsX + threadIdx.x;
  for (int base = tid; base < total; base += kThreads * kStageBatch) {
    float v[kStageBatch];
    int dst[kStageBatch];
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = min(base + u * kThreads, total - 1);
      const int rr = i / cols;
      const int cc = i - rr * cols;
      const int gh = h0 - st.R + rr;
      const int gw = w0 - st.R + cc;
      const float t = ldg_f32<T>(plane + (size_t)clampi(gh, 0, H - 1) * W + clampi(gw, 0, W - 1));
      v[u] = (gh >= 0 && gh < H && gw >= 0 && gw < W) ? t : 0.f;
      dst[u] = st.idx(rr, cc);
    }
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u)
      if (base + u * kThreads < total) s[dst[u]] = v[u];
  }
}

// NPL planes (plane i at plane0 + i * plane_stride) staged with 16-byte loads,
// for rows that are a whole number of aligned VEC-chunks (W % VEC == 0, 16-byte
// aligned base): a chunk then lies wholly inside or wholly outside the image,
// and a tile needs about VEC times fewer loads, so all of a thread's loads
// fit in one or two batches. For a fixed element of the chunk the lanes of a
// warp store consecutive words of one interleave sub-row: no bank conflicts.
template <typename T, int VEC, int NPL>
__device__ __forceinline__ void stage_planes_vec(float* __restrict__ s, int plane_words,
                                                 const Stage<VEC>& st, const T* __restrict__ plane0,
                                                 size_t plane_stride, int H, int W, int h0,
                                                 int w0) {
  using U = typename Vec<T, VEC>::U;
  const int rows = kTileH + 2 * st.R;
  const int x0 = w0 - st.R;  // global column of staged column 0
  const int k0 = x0 >= 0 ? x0 / VEC : -((VEC - 1 - x0) / VEC);  // floor(x0 / VEC)
  const int nk = (x0 + st.row_words - 1) / VEC - k0 + 1;        // chunks per staged row
  const int nchunk = W / VEC;
  const int per_plane = rows * nk;
  const int total = NPL * per_plane;
  const int tid = threadIdx.y * kThreadsX + threadIdx.x;
  for (int base = tid; base < total; base += kThreads * kStageBatch) {
    U u[kStageBatch];
    bool ok[kStageBatch];
#pragma unroll
    for (int q = 0; q < kStageBatch; ++q) {
      const int i = min(base + q * kThreads, total - 1);
      const int pl = i / per_plane;
      const int rem = i - pl * per_plane;
      const int rr = rem / nk;
      const int kc = k0 + rem - rr * nk;
      const int gh = h0 - st.R + rr;
      ok[q] = gh >= 0 && gh < H && kc >= 0 && kc < nchunk;
      const U* row = reinterpret_cast<const U*>(plane0 + pl * plane_stride +
                                                (size_t)clampi(gh, 0, H - 1) * W);
      u[q] = __ldg(row + clampi(kc, 0, nchunk - 1));
    }
#pragma unroll
    for (int q = 0; q < kStageBatch; ++q) {
      const int i = base + q * kThreads;
      if (i >= total) break;
      const int pl = i / per_plane;
      const int rem = i - pl * per_plane;
      const int rr = rem / nk;
      const int cc0 = (k0 + rem - rr * nk) * VEC - x0;
      float v[VEC];
      Vec<T, VEC>::unpack(u[q], v);
      float* dst = s + pl * plane_words;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int cc = cc0 + e;
        if (cc >= 0 && cc < st.row_words) dst[st.idx(rr, cc)] = ok[q] ? v[e] : 0.f;
      }
    }
  }
}

// ------------------------------------------------------------- forward ------
// Forward, dK and dX each have a compile-time instance for the dilations the
// module uses, (1, 3, 5) (template arguments D0 > 0): every tap shift, the halo
// and every shared-memory offset are then constants, and the per-tap work is
// the load or store, the reads and the arithmetic. D0 == 0 takes the
// dilations and the halo from the arguments at run time.
#define DDPM_DIL_CONSTANTS                                                      \
  constexpr bool kFixed = D0 > 0;                                              \
  constexpr int kDil[3] = {D0, D1, D2};                                        \
  constexpr int kR = (KS / 2) * (D0 > D1 ? (D0 > D2 ? D0 : D2) : (D1 > D2 ? D1 : D2)); \
  const int R = kFixed ? kR : R_rt;

// Staged word of (row ly + R + dy, column VEC*tx + e), e = R + dx + v >= 0:
// ly*row_words + tx + [(R + dy)*row_words + (e % VEC)*sub + e / VEC].
template <int VEC>
__device__ __forceinline__ int stage_off(const Stage<VEC>& st, int row, int e) {
  return row * st.row_words + (e % VEC) * st.sub + e / VEC;
}

template <typename TX, typename TK, int KS, int VEC, int D0, int D1, int D2>
__global__ void __launch_bounds__(kThreads, 2)
dyncat_fwd_kernel(const TX* __restrict__ x, const TK* __restrict__ kern, TK* __restrict__ out,
                  int C, int H, int W, Dil dil, int R_rt) {
  extern __shared__ float smem[];
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  DDPM_DIL_CONSTANTS
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
  const int tx = threadIdx.x;
  const int w = w0 + tx * VEC;
  if (w >= W) return;

#pragma unroll 1
  for (int j = 0; j < kRowsPerThread; ++j) {
    const int ly = threadIdx.y + j * kThreadsY;
    const int h = h0 + ly;
    if (h >= H) break;
    const size_t p = (size_t)h * W + w;
    const float* sthr = smem + ly * st.row_words + tx;
    float center[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) center[v] = sthr[stage_off(st, R, R + v)];
    vstore_cs<TK, VEC>(obase + p, center);
    auto branch = [&](int b, int d) {
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
          const int row = R + (ki - r) * d;
#pragma unroll
          for (int kj = 0; kj < KS; ++kj) {
#pragma unroll
            for (int v = 0; v < VEC; ++v)
              acc[v] = fmaf(sthr[stage_off(st, row, R + (kj - r) * d + v)],
                            kv[(ki - k0) * KS + kj][v], acc[v]);
          }
        }
      }
      vstore_cs<TK, VEC>(obase + (b + 1) * obranch + p, acc);
    };
    if constexpr (kFixed) {
      branch(0, kDil[0]);
      branch(1, kDil[1]);
      branch(2, kDil[2]);
    } else {
#pragma unroll 1
      for (int b = 0; b < 3; ++b) branch(b, dil.d[b]);
    }
  }
}

// ---------------------------------------------------------------- dK --------
template <typename TX, typename TK, int KS, int VEC, int D0, int D1, int D2>
__global__ void __launch_bounds__(kThreads, 2)
dyncat_bwd_k_kernel(const TX* __restrict__ x, const TK* __restrict__ gout, TK* __restrict__ gk,
                    int C, int H, int W, Dil dil, int R_rt) {
  extern __shared__ float smem[];
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  DDPM_DIL_CONSTANTS
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
  const int tx = threadIdx.x;
  const int w = w0 + tx * VEC;
  if (w >= W) return;

#pragma unroll 1
  for (int j = 0; j < kRowsPerThread; ++j) {
    const int ly = threadIdx.y + j * kThreadsY;
    const int h = h0 + ly;
    if (h >= H) break;
    const size_t p = (size_t)h * W + w;
    const float* sthr = smem + ly * st.row_words + tx;
    auto branch = [&](int b, int d) {
      float g[VEC];
      vload<TK, VEC>(gbase + (b + 1) * gbranch + p, g);
      TK* kp = gk + kbase + b * kbranch + p;
#pragma unroll
      for (int ki = 0; ki < KS; ++ki) {
        const int row = R + (ki - r) * d;
#pragma unroll
        for (int kj = 0; kj < KS; ++kj) {
          float o[VEC];
#pragma unroll
          for (int v = 0; v < VEC; ++v) o[v] = sthr[stage_off(st, row, R + (kj - r) * d + v)] * g[v];
          vstore_cs<TK, VEC>(kp + (size_t)(ki * KS + kj) * P, o);
        }
      }
    };
    if constexpr (kFixed) {
      branch(0, kDil[0]);
      branch(1, kDil[1]);
      branch(2, kDil[2]);
    } else {
#pragma unroll 1
      for (int b = 0; b < 3; ++b) branch(b, dil.d[b]);
    }
  }
}

// ---------------------------------------------------------------- dX --------
// One pixel per thread per step (gather at unaligned shifts); the three branch
// gradients of the tile + halo are staged in smem (plain row-major, VEC = 1).
constexpr int kDxTileW = kThreadsX * 4;  // 4 pixel columns per thread, 32 apart

// D0 > 0 fixes the dilations (D0, D1, D2) at compile time, as for the vector
// kernel below: tap shifts, the halo and every shared-memory offset are then
// constants. D0 == 0 takes them from `dil` and `R_rt` at run time.
template <typename TX, typename TK, int KS, int D0, int D1, int D2>
__global__ void __launch_bounds__(kThreads, 3)
dyncat_bwd_x_kernel(const TK* __restrict__ kern, const TK* __restrict__ gout, TX* __restrict__ gx,
                    int C, int H, int W, Dil dil, int R_rt) {
  extern __shared__ float smem[];
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  constexpr bool kFixed = D0 > 0;
  constexpr int kDil[3] = {D0, D1, D2};
  constexpr int kR = r * (D0 > D1 ? (D0 > D2 ? D0 : D2) : (D1 > D2 ? D1 : D2));
  const int R = kFixed ? kR : R_rt;
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
    const int total = 3 * plane_sz;
    for (int base = tid; base < total; base += kThreads * kStageBatch) {
      float v[kStageBatch];
#pragma unroll
      for (int u = 0; u < kStageBatch; ++u) {
        const int i = min(base + u * kThreads, total - 1);
        const int b = i / plane_sz;
        const int k = i - b * plane_sz;
        const int rr = k / pitch;
        const int cc = k - rr * pitch;
        const int gh = h0 - R + rr;
        const int gw = w0 - R + cc;
        const float t = ldg_f32<TK>(gbase + (b + 1) * gbranch +
                                    (size_t)clampi(gh, 0, H - 1) * W + clampi(gw, 0, W - 1));
        v[u] = (gh >= 0 && gh < H && gw >= 0 && gw < W) ? t : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kStageBatch; ++u)
        if (base + u * kThreads < total) smem[base + u * kThreads] = v[u];
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
        const int d = kFixed ? kDil[b] : dil.d[b];
        const TK* kp = kern + kbase + b * kbranch;
        const float* gs = smem + b * plane_sz + sidx;
        // A tap whose source pixel q - off lies outside the image (zero
        // padding) contributes nothing. Its load still goes out, from a
        // clamped in-image address, so that a group's loads are all issued
        // before the first FMA; the value is zeroed (a non-finite tap there
        // never reaches the sum) and meets the staged zero of the padding.
        constexpr int RG = KS <= 3 ? KS : 1;
#pragma unroll
        for (int k0 = 0; k0 < KS; k0 += RG) {
          float kv[RG * KS];
#pragma unroll
          for (int ki = k0; ki < k0 + RG; ++ki) {
            const int dy = (ki - r) * d;
            const bool row_ok = (unsigned)(h - dy) < (unsigned)H;
            const size_t srow = (size_t)clampi(h - dy, 0, H - 1) * W;
#pragma unroll
            for (int kj = 0; kj < KS; ++kj) {
              const int dx = (kj - r) * d;
              const float t =
                  ldcs_f32<TK>(kp + (size_t)(ki * KS + kj) * P + srow + clampi(w - dx, 0, W - 1));
              kv[(ki - k0) * KS + kj] = (row_ok && (unsigned)(w - dx) < (unsigned)W) ? t : 0.f;
            }
          }
#pragma unroll
          for (int ki = k0; ki < k0 + RG; ++ki) {
            const int dy = (ki - r) * d;
#pragma unroll
            for (int kj = 0; kj < KS; ++kj)
              acc = fmaf(kv[(ki - k0) * KS + kj], gs[-dy * pitch - (kj - r) * d], acc);
          }
        }
      }
      gx[(size_t)nc * P + p] = from_f32<TX>(acc);
    }
  }
}

// ------------------------------------------------------- dX (vector) --------
// The same sum as dyncat_bwd_x_kernel, in the same order, with the forward's
// thread layout: a thread owns VEC consecutive pixels, so a warp reads each
// tap plane as one contiguous 32 x 16-byte row segment instead of VEC
// separate 4- or 2-byte gathers spread over time. The tap a pixel q needs
// sits at q - off, which is not VEC-aligned for odd shifts: the thread loads
// the two aligned 16-byte chunks that cover its shifted window (the second
// one is mostly an L1 hit on the neighbour's first) and picks the window out
// of them. The window offset m = (-dx) mod VEC is the same for every thread of
// the CTA, so the pick is a uniform branch over compile-time cases.
template <int VEC, int M = 0, typename F>
__device__ __forceinline__ void with_window(int m, F&& f) {
  if constexpr (M < VEC) {
    if (m == M)
      f(std::integral_constant<int, M>{});
    else
      with_window<VEC, M + 1>(m, f);
  }
}

// D0 > 0 fixes the dilations (D0, D1, D2) at compile time (the module's
// (1, 3, 5)): every tap shift, window offset and shared-memory offset is then a
// constant, and the per-tap work is the loads, the reads and the FMAs.
// D0 == 0 takes them from `dil` at run time.
template <typename TX, typename TK, int KS, int VEC, int D0, int D1, int D2>
__global__ void __launch_bounds__(kThreads, 2)
dyncat_bwd_x_vec_kernel(const TK* __restrict__ kern, const TK* __restrict__ gout,
                        TX* __restrict__ gx, int C, int H, int W, Dil dil, int R_rt) {
  extern __shared__ float smem[];
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  constexpr bool kFixed = D0 > 0;
  constexpr int kDil[3] = {D0, D1, D2};
  constexpr int kR = r * (D0 > D1 ? (D0 > D2 ? D0 : D2) : (D1 > D2 ? D1 : D2));
  using U = typename Vec<TK, VEC>::U;
  const int R = kFixed ? kR : R_rt;
  const int nc = blockIdx.x;
  const int n = nc / C;
  const int c = nc - n * C;
  const int h0 = blockIdx.y * kTileH;
  const int w0 = blockIdx.z * (kThreadsX * VEC);
  const size_t P = (size_t)H * W;
  const Stage<VEC> st{R, stage_sub<VEC>(R), VEC * stage_sub<VEC>(R)};
  const int plane_words = st.row_words * (kTileH + 2 * R);

  const TK* gbase = gout + ((size_t)n * 4 * C + c) * P;
  const size_t gbranch = (size_t)C * P;
  stage_planes_vec<TK, VEC, 3>(smem, plane_words, st, gbase + gbranch, gbranch, H, W, h0, w0);
  __syncthreads();

  const int tx = threadIdx.x;
  const int w = w0 + tx * VEC;
  if (w >= W) return;
  const int nchunk = W / VEC;
  const size_t kbase = ((size_t)n * 3 * C + c) * KK * P;
  const size_t kbranch = (size_t)C * KK * P;

#pragma unroll 1
  for (int j = 0; j < kRowsPerThread; ++j) {
    const int ly = threadIdx.y + j * kThreadsY;
    const int h = h0 + ly;
    if (h >= H) break;
    const size_t p = (size_t)h * W + w;
    // Staged word of (row ly + R - dy, column VEC*tx + R + v - dx): with
    // e = R + v - dx >= 0 it is ly*row_words + tx + [(R - dy)*row_words +
    // (e % VEC)*sub + e / VEC], the bracket being a constant per tap and v.
    const float* gthr = smem + ly * st.row_words + tx;
    float acc[VEC];
    vload<TK, VEC>(gbase + p, acc);  // the x passthrough's gradient g[n, c, q]
    auto branch = [&](int b, int d) {
      const TK* kp = kern + kbase + b * kbranch;
      const float* gs = gthr + b * plane_words;
      // With fixed dilations the second chunk is only loaded for the shifted
      // taps (known at compile time), and a K = 3 branch's chunks all fit in
      // registers: all nine taps' loads go out before the first FMA.
      constexpr int RG = (kFixed && KS <= 3) ? KS : 1;
#pragma unroll
      for (int k0 = 0; k0 < KS; k0 += RG) {
        U ua[RG][KS], ub[RG][KS];
#pragma unroll
        for (int ki = k0; ki < k0 + RG; ++ki) {
          const int dy = (ki - r) * d;
          const TK* krow = kp + (size_t)clampi(h - dy, 0, H - 1) * W;
#pragma unroll
          for (int kj = 0; kj < KS; ++kj) {
            const int dx = (kj - r) * d;
            const int m = ((-dx) % VEC + VEC) % VEC;
            const int c0 = w / VEC + (-dx - m) / VEC;  // exact: -dx - m is a multiple of VEC
            const U* tp = reinterpret_cast<const U*>(krow + (size_t)(ki * KS + kj) * P);
            // Chunks outside the row are clamped; every element they supply
            // has its source outside the image and is zeroed below.
            ua[ki - k0][kj] = __ldg(tp + clampi(c0, 0, nchunk - 1));
            if (m != 0) ub[ki - k0][kj] = __ldg(tp + clampi(c0 + 1, 0, nchunk - 1));
          }
        }
#pragma unroll
      for (int ki = k0; ki < k0 + RG; ++ki) {
        const int dy = (ki - r) * d;
        const bool row_ok = (unsigned)(h - dy) < (unsigned)H;
        const float* grow = gs + (R - dy) * st.row_words;
#pragma unroll
        for (int kj = 0; kj < KS; ++kj) {
          const int dx = (kj - r) * d;
          const int m = ((-dx) % VEC + VEC) % VEC;
          const bool inside = row_ok && w - dx >= 0 && w + VEC - 1 - dx < W;
          float za[VEC], zb[VEC];
          Vec<TK, VEC>::unpack(ua[ki - k0][kj], za);
          if (m != 0) Vec<TK, VEC>::unpack(ub[ki - k0][kj], zb);
          with_window<VEC>(m, [&](auto mc) {
            constexpr int M = decltype(mc)::value;
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
              float t = (M + v < VEC) ? za[(M + v) % VEC] : zb[(M + v) % VEC];
              // A source pixel outside the image contributes nothing (and a
              // non-finite tap there never reaches the sum).
              if (!inside) t = (row_ok && (unsigned)(w + v - dx) < (unsigned)W) ? t : 0.f;
              const int e = R + v - dx;
              acc[v] = fmaf(t, grow[(e % VEC) * st.sub + e / VEC], acc[v]);
            }
          });
        }
      }
      }
    };
    if constexpr (kFixed) {  // constant shifts and offsets after inlining
      branch(0, kDil[0]);
      branch(1, kDil[1]);
      branch(2, kDil[2]);
    } else {
#pragma unroll 1
      for (int b = 0; b < 3; ++b) branch(b, dil.d[b]);
    }
    if constexpr (sizeof(TX) == sizeof(TK)) {
      vstore_cs<TX, VEC>(gx + (size_t)nc * P + p, acc);
    } else {  // FP32 x with a 16-bit taps tensor: VEC = 8 floats, two 16-byte stores
      float4* o = reinterpret_cast<float4*>(gx + (size_t)nc * P + p);
      __stcs(o, make_float4(acc[0], acc[1], acc[2], acc[3]));
      __stcs(o + 1, make_float4(acc[4], acc[5], acc[6], acc[7]));
    }
  }
}

// ------------------------------------------------------------- launchers ----
template <int VEC>
size_t stage_bytes(int R) {
  return sizeof(float) * (size_t)VEC * stage_sub<VEC>(R) * (kTileH + 2 * R);
}

// The dilations with compile-time kernel instances (the module's default).
inline bool is_default_dil(const Dil& dil) {
  return dil.d[0] == 1 && dil.d[1] == 3 && dil.d[2] == 5;
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
  auto fn = is_default_dil(dil) ? dyncat_fwd_kernel<TX, TK, KS, VEC, 1, 3, 5>
                                : dyncat_fwd_kernel<TX, TK, KS, VEC, 0, 0, 0>;
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
  auto fn = is_default_dil(dil) ? dyncat_bwd_k_kernel<TX, TK, KS, VEC, 1, 3, 5>
                                : dyncat_bwd_k_kernel<TX, TK, KS, VEC, 0, 0, 0>;
  if (int rc = set_smem(fn, smem)) return rc;
  dim3 grid(n * c, (h + kTileH - 1) / kTileH, (w + kThreadsX * VEC - 1) / (kThreadsX * VEC));
  fn<<<grid, dim3(kThreadsX, kThreadsY), smem, st>>>(static_cast<const TX*>(x),
                                                       static_cast<const TK*>(g),
                                                       static_cast<TK*>(gk), c, h, w, dil, R);
  DDPM_CHECK_LAUNCH("dyncat_bwd_k_kernel");
  return DDPM_OK;
}

// Shared memory of the scalar dX kernel: the three branch-gradient planes of
// its tile with the halo. The largest halo that fits the 227 KB a CTA may opt
// into is 39 ((128 + 78) x (16 + 78) x 3 x 4 bytes = 232,368).
constexpr size_t kMaxSmemPerCta = 227 * 1024;
constexpr size_t dx_stage_bytes(int R) {
  return sizeof(float) * 3 * (size_t)(kDxTileW + 2 * R) * (kTileH + 2 * R);
}
constexpr int kMaxDxHalo = 39;
static_assert(dx_stage_bytes(kMaxDxHalo) <= kMaxSmemPerCta &&
                  dx_stage_bytes(kMaxDxHalo + 1) > kMaxSmemPerCta,
              "kMaxDxHalo out of step with the dX tile");

template <typename TX, typename TK, int KS, int D0, int D1, int D2>
int launch_bwd_x(const void* k, const void* g, void* gx, int n, int c, int h, int w, Dil dil,
                 int R, cudaStream_t st) {
  const size_t smem = dx_stage_bytes(R);
  auto fn = dyncat_bwd_x_kernel<TX, TK, KS, D0, D1, D2>;
  if (int rc = set_smem(fn, smem)) return rc;
  dim3 grid(n * c, (h + kTileH - 1) / kTileH, (w + kDxTileW - 1) / kDxTileW);
  fn<<<grid, dim3(kThreadsX, kThreadsY), smem, st>>>(static_cast<const TK*>(k),
                                                       static_cast<const TK*>(g),
                                                       static_cast<TX*>(gx), c, h, w, dil, R);
  DDPM_CHECK_LAUNCH("dyncat_bwd_x_kernel");
  return DDPM_OK;
}

// The vector dX kernel stages the three branch planes at the wider vector
// tile; beyond this size (large K x dilation halos) two CTAs no longer fit on
// an SM and the scalar kernel is used.
constexpr size_t kDxVecSmemMax = 113 * 1024;

template <typename TX, typename TK, int KS, int VEC, int D0, int D1, int D2>
int launch_bwd_x_vec(const void* k, const void* g, void* gx, int n, int c, int h, int w, Dil dil,
                     int R, cudaStream_t st) {
  const size_t smem = 3 * stage_bytes<VEC>(R);
  auto fn = dyncat_bwd_x_vec_kernel<TX, TK, KS, VEC, D0, D1, D2>;
  if (int rc = set_smem(fn, smem)) return rc;
  dim3 grid(n * c, (h + kTileH - 1) / kTileH, (w + kThreadsX * VEC - 1) / (kThreadsX * VEC));
  fn<<<grid, dim3(kThreadsX, kThreadsY), smem, st>>>(static_cast<const TK*>(k),
                                                       static_cast<const TK*>(g),
                                                       static_cast<TX*>(gx), c, h, w, dil, R);
  DDPM_CHECK_LAUNCH("dyncat_bwd_x_vec_kernel");
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
  if (gx != nullptr) {
    // The vector dX kernel serves 16-bit taps with K <= 3 (its chunk pairs fit
    // in registers without spilling). For FP32 taps the scalar kernel, at
    // three CTAs per SM, is the faster one (162 against 184 us at B1 C64 256^2
    // K3 on B200).
    if constexpr (V == 8 && KS <= 3) {
      if (vec_ok(w, V, {k, g, gx}) && 3 * stage_bytes<V>(R) <= kDxVecSmemMax) {
        if (is_default_dil(dil))
          return launch_bwd_x_vec<TX, TK, KS, V, 1, 3, 5>(k, g, gx, n, c, h, w, dil, R, st);
        return launch_bwd_x_vec<TX, TK, KS, V, 0, 0, 0>(k, g, gx, n, c, h, w, dil, R, st);
      }
    }
    if (is_default_dil(dil))
      return launch_bwd_x<TX, TK, KS, 1, 3, 5>(k, g, gx, n, c, h, w, dil, R, st);
    return launch_bwd_x<TX, TK, KS, 0, 0, 0>(k, g, gx, n, c, h, w, dil, R, st);
  }
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

// `need_k`: the taps are read (the forward and the data gradient; the tap
// gradient alone does not read them).
int check_common(const void* x, int xdt, const void* k, int kdt, int n, int c, int h, int w,
                 int ks, int d0, int d1, int d2, bool need_k = true) {
  DDPM_CHECK_ARG(x != nullptr && (k != nullptr || !need_k), "null input pointer");
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

// TMA-fed kernels (dyncat_tma.cu) for K = 3, dilations (1, 3, 5), one dtype
// and 16-byte aligned rows; the kernels above serve every other case.
bool dyncat_tma_eligible(int xdt, int kdt, int w, int ks, int d0, int d1, int d2,
                         std::initializer_list<const void*> ptrs);
int dyncat_fwd_tma(const void* x, const void* k, void* out, int n, int c, int h, int w, int dt,
                   cudaStream_t st);
int dyncat_bwdk_tma(const void* x, const void* g, void* gk, int n, int c, int h, int w, int dt,
                    cudaStream_t st);
int dyncat_bwdx_tma(const void* k, const void* g, void* gx, int n, int c, int h, int w, int dt,
                    cudaStream_t st);

namespace {
bool g_tma_disabled = false;  // test hook: ddpm_test_disable_tma
}

int dyncat_set_tma_disabled(int disabled) {
  g_tma_disabled = disabled != 0;
  return DDPM_OK;
}

int dyncat_fwd(const void* x, int xdt, const void* k, int kdt, void* out, int n, int c, int h,
               int w, int ks, int d0, int d1, int d2, cudaStream_t st) {
  int rc = check_common(x, xdt, k, kdt, n, c, h, w, ks, d0, d1, d2);
  if (rc) return rc;
  DDPM_CHECK_ARG(out != nullptr, "null output pointer");
  if (!g_tma_disabled && dyncat_tma_eligible(xdt, kdt, w, ks, d0, d1, d2, {x, k, out})) {
    rc = dyncat_fwd_tma(x, k, out, n, c, h, w, xdt, st);
    if (rc != DDPM_ERR_UNSUPPORTED) return rc;
    clear_error();  // a tensor map the driver rejected: the kernels above
  }
  Dil dil{{d0, d1, d2}};
  const int R = (ks / 2) * max3(d0, d1, d2);
  DDPM_DYNCAT_DISPATCH(dispatch_fwd, ks, x, k, out, n, c, h, w, dil, R, st)
}

int dyncat_bwd(const void* x, int xdt, const void* k, const void* g, int kdt, void* gx, void* gk,
               int n, int c, int h, int w, int ks, int d0, int d1, int d2, cudaStream_t st) {
  int rc = check_common(x, xdt, k, kdt, n, c, h, w, ks, d0, d1, d2, gx != nullptr);
  if (rc) return rc;
  DDPM_CHECK_ARG(g != nullptr, "null grad_out pointer");
  if (gx == nullptr && gk == nullptr) return DDPM_OK;
  Dil dil{{d0, d1, d2}};
  const int R = (ks / 2) * max3(d0, d1, d2);
  // The data gradient stages three zero-padded gradient planes of its tile:
  // (128 + 2R) x (16 + 2R) floats each must fit one CTA's shared memory.
  if (gx != nullptr && dx_stage_bytes(R) > kMaxSmemPerCta)
    return set_error(DDPM_ERR_UNSUPPORTED,
                     "dilation halo %d too large for the data gradient (at most %d)", R,
                     kMaxDxHalo);
  if (!g_tma_disabled && dyncat_tma_eligible(xdt, kdt, w, ks, d0, d1, d2, {x, k, g, gx, gk})) {
    if (gk != nullptr) {
      rc = dyncat_bwdk_tma(x, g, gk, n, c, h, w, xdt, st);
      if (rc == DDPM_OK)
        gk = nullptr;  // done
      else if (rc != DDPM_ERR_UNSUPPORTED)
        return rc;
      clear_error();
    }
    if (gx != nullptr) {
      rc = dyncat_bwdx_tma(k, g, gx, n, c, h, w, xdt, st);
      if (rc == DDPM_OK)
        gx = nullptr;
      else if (rc != DDPM_ERR_UNSUPPORTED)
        return rc;
      clear_error();
    }
    if (gx == nullptr && gk == nullptr) return DDPM_OK;
  }
  DDPM_DYNCAT_DISPATCH(dispatch_bwd, ks, x, k, g, gx, gk, n, c, h, w, dil, R, st)
}

}  // namespace ddpm
