// Shared definitions of the fused generator kernels (forward and backward):
// I/O traits, tile geometry, operand staging helpers, bounded-wait helpers.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "tc.cuh"
#include "tmap.cuh"

namespace ddpm {
namespace gencat {

// 128 output pixels per MMA tile, as an 8 x 16 block of one image.
constexpr int kTileM = 128;
constexpr int kTileH = 8;
constexpr int kTileW = 16;
constexpr int kMaxChannels = 64;
// Width (pixels) of the staged x halo tile: the 16 tile columns plus 8 on each
// side, so dilation halos up to 8 pixels are covered and 8-pixel loads stay
// aligned with the tile origin.
constexpr int kHaloCols = 32;
constexpr int kMaxHalo = 8;
// K = 5 (forward only): dilation halos up to 16, a 48-column halo tile whose
// first column is 16 left of the tile origin.
constexpr int kMaxHalo5 = 16;

// Forward geometry per kernel size. A CTA owns `fwd_cg` output channels:
// 16 for K <= 3; for K = 5 the group's resident weights (3 * 25 taps per
// channel) would not fit shared memory at 16, so 8 (bf16 / fp16) or 4 (FP32,
// hi + lo images). One branch's accumulator columns (taps x channels, tap
// major) are padded to the MMA's N step of 16: 25 x 8 = 200 -> 208.
__host__ __device__ constexpr int fwd_cg(int ks, bool split) {
  return ks <= 3 ? 16 : (split ? 4 : 8);
}
__host__ __device__ constexpr int fwd_branch_cols(int ks, bool split) {
  return (ks * ks * fwd_cg(ks, split) + 15) / 16 * 16;
}
__host__ __device__ constexpr int fwd_halo_cols(int ks) { return ks <= 3 ? kHaloCols : 48; }
__host__ __device__ constexpr int fwd_halo_off(int ks) { return ks <= 3 ? 8 : 16; }
__host__ __device__ constexpr int fwd_max_halo(int ks) { return ks <= 3 ? kMaxHalo : kMaxHalo5; }
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
// GEMM K extent of the generator: C input channels + one constant-one channel
// carrying the bias, padded to the MMA K step of 16.
inline int augmented_channels(int c) { return (c + 1 + 15) / 16 * 16; }

// Layout of the packed generator weight (three operand images back to back).
//   fwd : per channel group cg of G = fwd_cg(K) channels, [part][Ck/8][3*BC
//         rows][8] with BC = fwd_branch_cols(K); row b*BC + tap*G + cl <->
//         weight row (b*C + cg*G + cl)*K^2 + tap (rows past K^2*G of a branch
//         are zero), K dimension = augmented input channels (bias at index C).
//   bx  : chunks q = b*K^2 + tap, each [part][Ck/8][Cp rows (c)][8].
//   by  : groups g = (cg16, slot octet) of 128 weight rows, row j*16 + cl <->
//         slot s = octet*8 + j = b*K^2 + tap, channel cg16*16 + cl; each group
//         [part][16 row groups][Cp (input channel i)][8 rows]: the transposed
//         weight, K dimension = weight rows.
// All sizes in 16-byte rows; `parts` = 2 for fp32 (bf16 hi + lo images).
struct PackLayout {
  int C, KS, Cp, Ck, Cq, spg, NG, parts;
  int bias_col;  // K index carrying the bias (bf16/fp16), -1 if the bias is added later
  long long fwd_rows, bx_rows, by_rows;
  __host__ __device__ size_t bx_offset() const { return (size_t)fwd_rows * 16; }
  __host__ __device__ size_t by_offset() const { return (size_t)(fwd_rows + bx_rows) * 16; }
  __host__ __device__ size_t total_bytes() const {
    return (size_t)(fwd_rows + bx_rows + by_rows) * 16;
  }
  static PackLayout make(int c, int ks, int dt) {
    PackLayout L;
    L.C = c;
    L.KS = ks;
    L.Cp = padded_channels(c);
    L.parts = dt == DDPM_F32 ? 2 : 1;
    // fp32 keeps K = Cp (shared memory budget) and adds the bias in the epilogue
    L.Ck = dt == DDPM_F32 ? L.Cp : augmented_channels(c);
    L.bias_col = dt == DDPM_F32 ? -1 : c;
    // dY / dW groups: 8 (branch, tap) slots x 16 channels = 128 weight rows
    L.Cq = 16;
    L.spg = 8;
    L.NG = (L.Cp / 16) * ((3 * ks * ks + 7) / 8);
    L.fwd_rows = (long long)(L.Cp / fwd_cg(ks, L.parts == 2)) * L.parts * (L.Ck / 8) * 3 *
                 fwd_branch_cols(ks, L.parts == 2);
    L.bx_rows = (long long)3 * ks * ks * L.parts * (L.Ck / 8) * L.Cp;
    L.by_rows = (long long)L.NG * L.parts * 16 * L.Cp;
    return L;
  }
};

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

// Warp-uniform bounded wait (all lanes see the same outcome); `hint_ns` as in
// tc::mbar_wait.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag, uint32_t hint_ns = 0) {
  const bool ok = tc::mbar_wait(bar, parity, abort_flag, kWaitNs, hint_ns);
  return __all_sync(0xffffffffu, ok);
}

// Load plane[h, w0 .. w0+7] (row-major H x W plane) as floats, zero outside
// the plane. Vector path when the whole run is inside and 16-byte aligned.
template <typename T>
__device__ __forceinline__ void load8(const T* __restrict__ plane, int H, int W, int h, int w0,
                                      float (&v)[8]) {
  if (h < 0 || h >= H || w0 >= W || w0 + 8 <= 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    return;
  }
  const T* src = plane + (ptrdiff_t)h * W + w0;
  const bool full = (w0 >= 0) && (w0 + 8 <= W) && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
  if (full) {
    if constexpr (sizeof(T) == 2) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = to_f32<T>(e[i]);
    } else {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src));
      const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int w = w0 + i;
    v[i] = (w >= 0 && w < W) ? to_f32<T>(__ldg(src + i)) : 0.f;
  }
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

// Eight consecutive elements of a row, kept in their storage format until
// they are written to shared memory (no float round trip for 16-bit data).
template <typename T> struct Raw8 {
  uint4 u;  // 8 x 16-bit
  __device__ __forceinline__ void zero() { u = make_uint4(0u, 0u, 0u, 0u); }
  __device__ __forceinline__ void ones() {
    const uint32_t one2 = std::is_same<T, __half>::value ? 0x3C003C00u : 0x3F803F80u;
    u = make_uint4(one2, one2, one2, one2);
  }
  __device__ __forceinline__ float get(int i) const {
    return to_f32<T>(reinterpret_cast<const T*>(&u)[i]);
  }
};
template <> struct Raw8<float> {
  float4 a, b;
  __device__ __forceinline__ void zero() { a = b = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void ones() { a = b = make_float4(1.f, 1.f, 1.f, 1.f); }
  __device__ __forceinline__ float get(int i) const {
    const float e[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    return e[i];
  }
};

// plane[h, w0 .. w0+7] of a row-major H x W plane, zero outside the plane.
template <typename T>
__device__ __forceinline__ Raw8<T> load_raw8(const T* __restrict__ plane, int H, int W, int h,
                                             int w0) {
  Raw8<T> r;
  r.zero();
  if (h < 0 || h >= H || w0 >= W || w0 + 8 <= 0) return r;
  const T* src = plane + (ptrdiff_t)h * W + w0;
  if (w0 >= 0 && w0 + 8 <= W && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    if constexpr (sizeof(T) == 2) {
      r.u = __ldg(reinterpret_cast<const uint4*>(src));
    } else {
      r.a = __ldg(reinterpret_cast<const float4*>(src));
      r.b = __ldg(reinterpret_cast<const float4*>(src) + 1);
    }
    return r;
  }
  T* e = reinterpret_cast<T*>(&r);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int w = w0 + i;
    if (w >= 0 && w < W) e[i] = __ldg(src + i);
  }
  return r;
}

// Eight elements at a 16-byte aligned address, no bounds logic: callers
// pass a safe address for items they will zero afterwards (so every load of
// a batch is issued before the first one is waited on).
template <typename T>
__device__ __forceinline__ Raw8<T> ldg_raw8(const T* src) {
  Raw8<T> r;
  if constexpr (sizeof(T) == 2) {
    r.u = __ldg(reinterpret_cast<const uint4*>(src));
  } else {
    r.a = __ldg(reinterpret_cast<const float4*>(src));
    r.b = __ldg(reinterpret_cast<const float4*>(src) + 1);
  }
  return r;
}

// Write 8 elements as one 16-byte MMA operand row (bf16/fp16 copy through;
// fp32 split into a bf16 hi row at `hi` and a bf16 residual row at `lo`).
template <typename T, typename Op, bool kSplit>
__device__ __forceinline__ void store_raw8(uint8_t* hi, uint8_t* lo, const Raw8<T>& r) {
  if constexpr (!kSplit) {
    *reinterpret_cast<uint4*>(hi) = r.u;
  } else {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = r.get(i);
    store8_split<Op, true>(hi, lo, v);
  }
}

// Stage the y tile of an 8 x 16 pixel tile as the MN-major MMA operand:
// 16 eight-pixel groups (row g/2, half g%2) x Ck augmented channels, one
// 16-byte row per (group, channel) at g*Ck*16 + c*16. Channel `ones_c` is the
// constant one (bias; -1 = none), others past C zero. With kSplit, the bf16
// residual goes to the same offset in `lo`.
// The item -> (channel, group) mapping is the same for every tile, so each
// thread computes it once (YPlan) and only adds the tile origin per tile.
template <int N>
struct YPlan {
  int c[N];  // channel, or -1 when the item is past the end
  int g[N];  // 8-pixel group
};

template <int N>
__device__ __forceinline__ YPlan<N> make_yplan(int Ck, int tid, int nthreads) {
  YPlan<N> pl;
#pragma unroll
  for (int u = 0; u < N; ++u) {
    const int item = tid + u * nthreads;
    pl.c[u] = item < 16 * Ck ? item % Ck : -1;
    pl.g[u] = item / Ck;
  }
  return pl;
}

template <typename T, typename Op, bool kSplit, int N>
__device__ __forceinline__ void stage_y_mn(const YPlan<N>& pl, const T* __restrict__ y,
                                           uint8_t* hi, uint8_t* lo, int n, int C, int Ck,
                                           int ones_c, int H, int W, int h0, int w0) {
  const size_t P = (size_t)H * W;
  const T* ybase = y + (size_t)n * C * P;
  // interior tile: every 8-pixel run is in the image and 16-byte aligned
  const bool interior = (h0 + kTileH <= H) && (w0 + kTileW <= W) &&
                        (((size_t)W * sizeof(T)) % 16 == 0) && (P * sizeof(T)) % 16 == 0 &&
                        ((reinterpret_cast<uintptr_t>(ybase + (size_t)h0 * W + w0) & 15u) == 0);
  Raw8<T> v[N];
#pragma unroll
  for (int u = 0; u < N; ++u) {
    const int c = pl.c[u];
    if (c >= 0 && c < C) {
      const int g = pl.g[u];
      if (interior) {
        const T* src = ybase + (size_t)c * P + (size_t)(h0 + (g >> 1)) * W + w0 + (g & 1) * 8;
        if constexpr (sizeof(T) == 2) {
          v[u].u = __ldg(reinterpret_cast<const uint4*>(src));
        } else {
          v[u].a = __ldg(reinterpret_cast<const float4*>(src));
          v[u].b = __ldg(reinterpret_cast<const float4*>(src) + 1);
        }
      } else {
        v[u] = load_raw8<T>(ybase + (size_t)c * P, H, W, h0 + (g >> 1), w0 + (g & 1) * 8);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < N; ++u) {
    const int c = pl.c[u];
    if (c < 0) continue;
    const uint32_t off = pl.g[u] * Ck * 16 + c * 16;
    if (c < C) {
      store_raw8<T, Op, kSplit>(hi + off, lo + off, v[u]);
    } else {
      float f[8];
      const float one = (c == ones_c) ? 1.f : 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = one;
      store8_split<Op, kSplit>(hi + off, lo + off, f);
    }
  }
}

// Stage the x halo of one group of 4*Q channels (Q = 4 unless given): rows
// hs .. hs+rows-1, columns ws .. ws+8*CB-1 of channels c0 .. c0+4Q-1, as FP32
// float4 cells holding four consecutive channels: cell (q4, row, col) =
// xr[(q4*rows + row)*8*CB + col]. Zero outside the image and for channels
// >= C. Items = (q4, row, 8-column block); the mapping is precomputed per
// thread (XPlan).
template <int N>
struct XPlan {
  int q4[N];   // 4-channel group, or -1
  int row[N];
  int blk[N];
};

template <int N, int Q = 4, int CB = kHaloCols / 8>
__device__ __forceinline__ XPlan<N> make_xplan(int rows, int tid, int nthreads) {
  XPlan<N> pl;
#pragma unroll
  for (int u = 0; u < N; ++u) {
    const int item = tid + u * nthreads;
    pl.blk[u] = item % CB;
    pl.row[u] = (item / CB) % rows;
    pl.q4[u] = item < Q * CB * rows ? (item / CB) / rows : -1;
  }
  return pl;
}

template <typename T, int N, int Q = 4, int CB = kHaloCols / 8>
__device__ __forceinline__ void stage_halo(const XPlan<N>& pl, const T* __restrict__ x, float4* xr,
                                           int n, int C, int H, int W, int c0, int hs, int ws,
                                           int rows) {
  const size_t P = (size_t)H * W;
  const T* xbase = x + ((size_t)n * C + c0) * P;
  const bool interior = hs >= 0 && hs + rows <= H && ws >= 0 && ws + 8 * CB <= W &&
                        c0 + 4 * Q <= C && (((size_t)W * sizeof(T)) % 16 == 0) &&
                        (P * sizeof(T)) % 16 == 0 &&
                        ((reinterpret_cast<uintptr_t>(xbase + (size_t)hs * W + ws) & 15u) == 0);
  Raw8<T> v[N][4];
#pragma unroll
  for (int u = 0; u < N; ++u) {
    const int q4 = pl.q4[u];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[u][k].zero();
      if (q4 < 0) continue;
      const int c = q4 * 4 + k;
      if (interior) {
        const T* src = xbase + (size_t)c * P + (size_t)(hs + pl.row[u]) * W + ws + pl.blk[u] * 8;
        if constexpr (sizeof(T) == 2) {
          v[u][k].u = __ldg(reinterpret_cast<const uint4*>(src));
        } else {
          v[u][k].a = __ldg(reinterpret_cast<const float4*>(src));
          v[u][k].b = __ldg(reinterpret_cast<const float4*>(src) + 1);
        }
      } else if (c0 + c < C) {
        v[u][k] = load_raw8<T>(xbase + (size_t)c * P, H, W, hs + pl.row[u], ws + pl.blk[u] * 8);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < N; ++u) {
    if (pl.q4[u] < 0) continue;
    float4* dst = xr + (pl.q4[u] * rows + pl.row[u]) * (8 * CB) + pl.blk[u] * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      dst[i] = make_float4(v[u][0].get(i), v[u][1].get(i), v[u][2].get(i), v[u][3].get(i));
  }
}

// ------------------------------------------------------ packed FP32 math ---
// sm_100 executes two FP32 FMAs per instruction on register pairs.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Two FP32 values rounded to bf16 (round to nearest even) and back, packed.
__device__ __forceinline__ unsigned long long f2_round_bf16(float lo, float hi) {
  uint32_t p;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
  return f2_pack(__uint_as_float(p << 16), __uint_as_float(p & 0xFFFF0000u));
}
__device__ __forceinline__ unsigned long long f2_round_f16(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  const float2 f = __half22float2(h);
  return f2_pack(f.x, f.y);
}
// Two floats -> one 32-bit word of two Op values (first value in bits 0-15),
// round to nearest even; and back.
template <typename Op> __device__ __forceinline__ uint32_t cvt2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t cvt2<__nv_bfloat16>(float lo, float hi) {
  uint32_t p;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
  return p;
}
template <> __device__ __forceinline__ uint32_t cvt2<__half>(float lo, float hi) {
  uint32_t p;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
  return p;
}
template <typename Op> __device__ __forceinline__ unsigned long long uncvt2(uint32_t p);
template <> __device__ __forceinline__ unsigned long long uncvt2<__nv_bfloat16>(uint32_t p) {
  return f2_pack(__uint_as_float(p << 16), __uint_as_float(p & 0xFFFF0000u));
}
template <> __device__ __forceinline__ unsigned long long uncvt2<__half>(uint32_t p) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&p));
  return f2_pack(f.x, f.y);
}

// acc (two FP32 lanes) += a * b per lane, where a and b each hold two Op
// values (first value in bits 0-15): one mixed-precision FMA per lane
// (`fma.rn.f32.bf16` / `.f16`, 16-bit multiplicands, FP32 addend and result),
// so no conversion of a or b to FP32 is issued. Fused with one rounding, like
// fmaf(float(a), float(b), acc): the same result bit for bit.
template <typename Op>
__device__ __forceinline__ unsigned long long fma_io2(uint32_t a, uint32_t b,
                                                      unsigned long long acc);
template <>
__device__ __forceinline__ unsigned long long fma_io2<__nv_bfloat16>(uint32_t a, uint32_t b,
                                                                     unsigned long long acc) {
  float lo, hi;
  f2_unpack(acc, lo, hi);
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %2;\n\t"
      "mov.b32 {bl, bh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, al, bl, %0;\n\t"
      "fma.rn.f32.bf16 %1, ah, bh, %1;\n\t}"
      : "+f"(lo), "+f"(hi)
      : "r"(a), "r"(b));
  return f2_pack(lo, hi);
}
template <>
__device__ __forceinline__ unsigned long long fma_io2<__half>(uint32_t a, uint32_t b,
                                                              unsigned long long acc) {
  float lo, hi;
  f2_unpack(acc, lo, hi);
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %2;\n\t"
      "mov.b32 {bl, bh}, %3;\n\t"
      "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
      "fma.rn.f32.f16 %1, ah, bh, %1;\n\t}"
      : "+f"(lo), "+f"(hi)
      : "r"(a), "r"(b));
  return f2_pack(lo, hi);
}

// Two 16-bit values as one word, the first in bits 0-15.
template <typename T>
__device__ __forceinline__ uint32_t pack_raw2(T lo, T hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
  else
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// a * b per 16-bit lane, rounded once to Op (round to nearest even): the
// exact product of two 16-bit values rounded to the type, the same value as
// the FP32 product (exact) converted with cvt2.
template <typename Op> __device__ __forceinline__ uint32_t mul_io2(uint32_t a, uint32_t b);
template <> __device__ __forceinline__ uint32_t mul_io2<__nv_bfloat16>(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <> __device__ __forceinline__ uint32_t mul_io2<__half>(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Eight floats, held as four packed pairs, stored as one 16-byte operand row;
// with kSplit also the residual (v - hi) row at dst_lo (exact subtraction).
template <typename Op, bool kSplit>
__device__ __forceinline__ void store8x2_split(uint8_t* dst_hi, uint8_t* dst_lo,
                                               const unsigned long long (&v)[4]) {
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float a, b;
    f2_unpack(v[i], a, b);
    h[i] = cvt2<Op>(a, b);
  }
  *reinterpret_cast<uint4*>(dst_hi) = make_uint4(h[0], h[1], h[2], h[3]);
  if constexpr (kSplit) {
    const unsigned long long neg1 = f2_pack(-1.f, -1.f);
    uint32_t l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a, b;
      f2_unpack(f2_fma(uncvt2<Op>(h[i]), neg1, v[i]), a, b);
      l[i] = cvt2<Op>(a, b);
    }
    *reinterpret_cast<uint4*>(dst_lo) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// Four channels (two f32x2 pairs) as one 8-byte cell half: the 4-channel
// counterpart of store8x2_split.
template <typename Op, bool kSplit>
__device__ __forceinline__ void store4x2_split(uint8_t* dst_hi, uint8_t* dst_lo,
                                               const unsigned long long (&v)[2]) {
  uint32_t h[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float a, b;
    f2_unpack(v[i], a, b);
    h[i] = cvt2<Op>(a, b);
  }
  *reinterpret_cast<uint2*>(dst_hi) = make_uint2(h[0], h[1]);
  if constexpr (kSplit) {
    const unsigned long long neg1 = f2_pack(-1.f, -1.f);
    uint32_t l[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float a, b;
      f2_unpack(f2_fma(uncvt2<Op>(h[i]), neg1, v[i]), a, b);
      l[i] = cvt2<Op>(a, b);
    }
    *reinterpret_cast<uint2*>(dst_lo) = make_uint2(l[0], l[1]);
  }
}

// Eight elements as four 32-bit words of two operand values (element 2i in
// the low half of word i); with kSplit (FP32) the bf16 hi words and the
// bf16 residual words (v - hi, exact subtraction).
template <typename T, typename Op, bool kSplit>
__device__ __forceinline__ void raw8_words(const Raw8<T>& r, uint32_t (&hi)[4], uint32_t (&lo)[4]) {
  if constexpr (!kSplit) {
    hi[0] = r.u.x;
    hi[1] = r.u.y;
    hi[2] = r.u.z;
    hi[3] = r.u.w;
  } else {
    const unsigned long long neg1 = f2_pack(-1.f, -1.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = r.get(2 * i), b = r.get(2 * i + 1);
      hi[i] = cvt2<Op>(a, b);
      float ra, rb;
      f2_unpack(f2_fma(uncvt2<Op>(hi[i]), neg1, f2_pack(a, b)), ra, rb);
      lo[i] = cvt2<Op>(ra, rb);
    }
  }
}

// Transpose 8 channels x 8 pixels (one Raw8 per channel) into 8 K-major
// operand rows of 8 channels each at dst + px*16 (the bf16 residual rows at
// dst + lo_off + px*16 when kSplit). 16-bit data is permuted without a float
// round trip; FP32 data is split with packed bf16x2 conversions.
template <typename T, typename Op, bool kSplit>
__device__ __forceinline__ void store_transposed(uint8_t* dst, uint32_t lo_off,
                                                 const Raw8<T> (&v)[8]) {
  if constexpr (sizeof(T) == 2 && !kSplit) {
    const uint32_t* w[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) w[e] = reinterpret_cast<const uint32_t*>(&v[e].u);
#pragma unroll
    for (int px = 0; px < 8; ++px) {
      const uint32_t sel = (px & 1) ? 0x7632u : 0x5410u;
      uint4 row;
      row.x = __byte_perm(w[0][px >> 1], w[1][px >> 1], sel);
      row.y = __byte_perm(w[2][px >> 1], w[3][px >> 1], sel);
      row.z = __byte_perm(w[4][px >> 1], w[5][px >> 1], sel);
      row.w = __byte_perm(w[6][px >> 1], w[7][px >> 1], sel);
      *reinterpret_cast<uint4*>(dst + px * 16) = row;
    }
  } else {
#pragma unroll
    for (int px = 0; px < 8; ++px) {
      unsigned long long pr[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) pr[e] = f2_pack(v[2 * e].get(px), v[2 * e + 1].get(px));
      store8x2_split<Op, kSplit>(dst + px * 16, dst + lo_off + px * 16, pr);
    }
  }
}

// Tap pair (lo, hi) as used by the filter: rounded to the I/O dtype (bf16/fp16
// taps are rounded like the reference, `_triton_kernels.py:332-335`).
template <typename T>
__device__ __forceinline__ unsigned long long tap_pair(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return f2_round_bf16(lo, hi);
  else if constexpr (std::is_same<T, __half>::value) return f2_round_f16(lo, hi);
  else return f2_pack(lo, hi);
}

// Round generated taps to the I/O precision (bf16 / fp16), as the reference
// does before using them (`_triton_kernels.py:332-335`); identity for fp32.
// bf16 uses integer round-to-nearest-even on the bit pattern (full-rate ALU
// ops instead of conversion instructions); taps are finite by construction.
template <typename T>
__device__ __forceinline__ void round_taps(float (&v)[16]) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      uint32_t u = __float_as_uint(v[i]);
      u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
      v[i] = __uint_as_float(u);
    }
  } else if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = IoTraits<T>::round_io(v[i]);
  }
}

// Host helpers (gencat_common.cu).
int check_shape(int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt);
// check_shape plus the dY + dW kernels' limit K <= 3.
int check_shape_bwd(int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt);
int status_ptr(int** out);
int read_status(int reset, int* code);
int num_sms();
// Dynamic shared memory a block may opt in to on the current device (bytes).
int max_smem_optin();

// Staged operands of the fused backward (gencat_stage.cu), written once per
// backward so the kernels stage tiles with bulk / TMA copies instead of
// per-thread loads and register transposes.
//
// y plane: y channel-last, zero padded, in the MMA operand type; layout
// [part][n][G][Hp][Wp][8]: 16-byte rows of 8 channels, G = round16(C+1)/8
// groups; channel C is the constant one of the bias / db column (1 at every
// position), channels above it are zero. Plane row i holds image row i - ph
// (ph = (K/2) * max dilation), plane column j holds image column j - pw (pw =
// 8 for K <= 3, 16 for K = 5), and Wp = 128 * ceil(W / 128) + 2 pw, so a
// (128 + 2 pw)-pixel segment starting pw columns left of any 128-pixel row
// tile, at any row within the dilation halo, is in range.
// FP32 stores a bf16 hi part and a bf16 residual part.
//
// x plane (after the y plane, 256-byte aligned): 16-byte cells
// [n][Cq][H][W][cell] with Cq = ceil(C / xcell) (channels >= C zero); FP32
// data as FP32 cells of xcell = 4 channels, 16-bit data in its own type,
// xcell = 8 channels per cell (half the bytes; the consumers multiply the
// 16-bit values directly). Not padded: it is read by TMA, which zero-fills
// outside the image.
struct StageLayout {
  int N, C, H, W, G, ph, pw, Hp, Wp, parts, Cq, xcell;
  size_t part_bytes, x_offset, x_bytes;
  __host__ __device__ size_t y_bytes() const { return part_bytes * parts; }
  __host__ __device__ size_t total_bytes() const { return x_offset + x_bytes; }
  // byte offset of the y-plane row (part, n, group g, plane row i, plane column j)
  __host__ __device__ size_t row_offset(int part, int n, int i, int g, int j) const {
    return (size_t)part * part_bytes + ((((size_t)n * G + g) * Hp + i) * Wp + j) * 16;
  }
  static StageLayout make(int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt) {
    StageLayout L;
    L.N = n;
    L.C = c;
    L.H = h;
    L.W = w;
    L.G = (c + 1 + 15) / 16 * 2;
    L.ph = (ks / 2) * max3(d0, d1, d2);
    // columns: 8 (K <= 3) or 16 (K = 5) zero columns before image column 0,
    // the dX kernels' row segment offset, so a segment starts at a 16-pixel block
    L.pw = ks <= 3 ? 8 : 16;
    L.Hp = h + 2 * L.ph;
    L.Wp = (w + kTileM - 1) / kTileM * kTileM + 2 * L.pw;
    L.parts = dt == DDPM_F32 ? 2 : 1;
    L.part_bytes = (size_t)n * L.G * L.Hp * L.Wp * 16;
    L.xcell = dt == DDPM_F32 ? 4 : 8;
    L.Cq = (c + L.xcell - 1) / L.xcell;
    L.x_offset = (L.y_bytes() + 255) / 256 * 256;
    L.x_bytes = (size_t)n * L.Cq * h * w * 16;
    return L;
  }
};
size_t stage_bytes(int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt);
// x may be null: only the y plane is written (enough for dX).
int stage(const void* x, const void* y, void* staged, size_t staged_bytes, int n, int c, int h,
          int w, int ks, int d0, int d1, int d2, int dt, cudaStream_t st);
// TMA descriptors of the staged planes for 8 x 16 pixel tiles (64-bit element
// views): x halo box {halo_cols px, 8 + 2R rows, `cells` x cells}, coordinates
// ((w0 - off) * 2, h0 - R, first cell, n); y tile box {16 px, 8 rows, ygroups
// channel groups}, coordinates ((w0 + pw) * 2, h0 + ph, 0, part * N + n).
// False when the driver rejects one (callers then stage from x and y).
// `cells` = the channels a CTA stages / sl.xcell.
bool encode_stage_maps(CUtensorMap* xmap, CUtensorMap* ymap, int R, int ygroups,
                       const uint8_t* staged, const StageLayout& sl, int halo_cols, int cells);
// Tensor map reading a (16 * blocks)-pixel row segment of the y plane
// ([group][pixel][8 channels], all `ngroups` channel groups of one part) as one
// 5-D box: coordinates (0, first plane column / 16, plane row, 0, part * N + n).
bool encode_stage_segment_map(CUtensorMap* map, int ngroups, const uint8_t* staged,
                              const StageLayout& sl, int blocks = 9);

}  // namespace gencat
}  // namespace ddpm
