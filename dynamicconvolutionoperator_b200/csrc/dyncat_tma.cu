// Materialised dynamic filter ("dynamic cat") fed by TMA: forward, tap
// gradient (dK) and data gradient (dX) for K = 3 and the module's dilations
// (1, 3, 5), 16-byte aligned rows (W % 8 == 0). Same sums, in the same order,
// as the kernels of dyncat.cu (bit-identical results); those serve every other
// case.
//
// All three are HBM-bound: the taps tensor K (dK) of 27 planes per channel
// dominates the traffic. In dyncat.cu each thread loads its taps into
// registers, so the bytes in flight per SM are capped by the register file and
// the CTA's staging phase leaves the memory system idle. Here one producer
// thread per CTA streams the tiles with TMA copies into a ring of shared-memory
// stages, a full kernel row of taps per stage, several stages ahead, while the
// 256 consumer threads compute from shared memory:
//
//   tile     = 16 rows x 128 columns of one (n, c) plane; persistent CTAs walk
//              the tiles (tile t, t + grid, ...);
//   x / g    = the tile's x (forward, dK) or branch gradients (dX) with the
//              dilation halo: one box per tile, columns w0 - 8 .. w0 + 135 and
//              rows h0 - R .. h0 + 15 + R, zero filled outside the image (the
//              zero padding of the reference's unfold), double buffered;
//   stage    = forward: the three taps of one kernel row, one box {128, 16, 3};
//              dX: the same taps at the shifted source positions q - off, one
//              box {136, 16} per tap starting at the 16-byte aligned column
//              at or left of w0 - dx (the window is picked out of it at an
//              offset below one vector);
//   consumer = a thread owns VEC = 16 / sizeof(T) consecutive pixels (one
//              16-byte vector) of RPT rows; it reads x or g windows and taps
//              from shared memory with 16-byte loads (conflict free: eight
//              consecutive threads read eight consecutive vectors of a row)
//              and writes its outputs with 16-byte streaming stores.
//
// Every TMA copy starts at a 16-byte aligned innermost coordinate (w0, w0 - 8
// or w0 + floor_VEC(-dx), all multiples of VEC elements). Waits are bounded:
// a wait that runs out records a status code (ddpm_device_status), every role
// stops, and the producer waits for its copies in flight before the CTA exits.
#include <cstdint>
#include <initializer_list>
#include <type_traits>

#include "common.cuh"
#include "gencat.cuh"
#include "tc.cuh"
#include "tmap.cuh"

namespace ddpm {
namespace {

constexpr int kTW = 128;            // tile columns
constexpr int kTH = 16;             // tile rows
constexpr int kHaloCols = kTW + 16; // x / g box columns: [w0 - 8, w0 + 136)
constexpr int kWinCols = kTW + 8;   // dX tap box columns
constexpr int kConsumers = 256;
constexpr int kThreads = kConsumers + 32;  // + the producer warp
constexpr int kKS = 3;
constexpr uint64_t kWaitNs = 2000000000ull;

template <typename T>
struct Geo {
  static constexpr int VEC = 16 / (int)sizeof(T);  // elements per 16-byte vector
  static constexpr int TPR = kTW / VEC;            // threads per tile row
  static constexpr int ROWSTEP = kConsumers / TPR; // rows between a thread's rows
  static constexpr int RPT = kTH / ROWSTEP;        // rows per thread
};

// ------------------------------------------------------------ conversion ---
template <typename T>
__device__ __forceinline__ void unpack_words(const uint32_t (&w)[4], float (&v)[8]);
template <>
__device__ __forceinline__ void unpack_words<__nv_bfloat16>(const uint32_t (&w)[4], float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <>
__device__ __forceinline__ void unpack_words<__half>(const uint32_t (&w)[4], float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// VEC elements of a 16-byte aligned shared-memory vector, as floats.
template <typename T>
__device__ __forceinline__ void lds_vec(const T* p, float (&v)[Geo<T>::VEC]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  if constexpr (sizeof(T) == 4) {
    v[0] = __uint_as_float(u.x);
    v[1] = __uint_as_float(u.y);
    v[2] = __uint_as_float(u.z);
    v[3] = __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    unpack_words<T>(w, v);
  }
}

// VEC elements starting O elements into the aligned vector at p (0 <= O <
// VEC): picked out of the two aligned vectors that cover them.
template <typename T, int O>
__device__ __forceinline__ void lds_window(const T* p, float (&v)[Geo<T>::VEC]) {
  constexpr int VEC = Geo<T>::VEC;
  if constexpr (O == 0) {
    lds_vec<T>(p, v);
  } else {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    const uint4 b = *reinterpret_cast<const uint4*>(p + VEC);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(w[O + i]);
    } else {
      uint32_t s[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (O % 2 == 0)
          s[i] = w[O / 2 + i];
        else  // the high half of word k and the low half of word k + 1
          s[i] = __byte_perm(w[O / 2 + i], w[O / 2 + i + 1], 0x5432);
      }
      unpack_words<T>(s, v);
    }
  }
}

template <typename T>
__device__ __forceinline__ void stg_vec(T* p, const float (&v)[Geo<T>::VEC]) {
  if constexpr (sizeof(T) == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
  } else {
    union {
      uint4 u;
      T e[8];
    } r;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.e[i] = from_f32<T>(v[i]);
    __stcs(reinterpret_cast<uint4*>(p), r.u);
  }
}

// ------------------------------------------------------------ params -------
struct TmaParams {
  CUtensorMap src;   // forward / dK: x {W, H, N*C}; dX: grad_out {W, H, C, 4, N}
  CUtensorMap aux;   // forward / dX: taps {W, H, N*3*C*9}; dK: grad_out {W, H, C, 4, N}
  void* out;         // forward: out [N, 4C, H, W]; dK: grad taps; dX: grad x [N, C, H, W]
  int N, C, H, W;
  int tiles_w, tiles_h, num_tiles;
  int* status;
};

__device__ __forceinline__ void tile_coords(const TmaParams& p, int tile, int& n, int& c,
                                            int& h0, int& w0) {
  const int wb = tile % p.tiles_w;
  int t = tile / p.tiles_w;
  const int hb = t % p.tiles_h;
  t /= p.tiles_h;
  c = t % p.C;
  n = t / p.C;
  h0 = hb * kTH;
  w0 = wb * kTW;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(tc::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2),
      "r"(tc::smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fail(volatile int* abort_flag, int* status, int code) {
  *abort_flag = 1;
  atomicCAS(status, 0, code);
}

// Consumer-side bounded wait, uniform over the warp.
__device__ __forceinline__ bool cwait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const bool ok = tc::mbar_wait(bar, parity, abort_flag, kWaitNs);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) tc::mbar_arrive(bar);
}

// The producer's drain: wait (bounded) until the last `n` phases armed on the
// ring `bars` (stages s - n .. s - 1 of a ring of `depth`) have completed, so
// no copy is in flight when the CTA exits.
__device__ __forceinline__ void drain(uint64_t* bars, int depth, uint32_t s, volatile int* abort_flag) {
  const uint32_t n = s < (uint32_t)depth ? s : (uint32_t)depth;
  for (uint32_t k = s - n; k < s; ++k)
    tc::mbar_wait(&bars[k % depth], (k / depth) & 1, nullptr, kWaitNs);
}

// Shared-memory carve-up: `nx` halo buffers of `xbytes`, `ns` stages of
// `sbytes`, then the mbarriers; every buffer 128-byte aligned.
struct Smem {
  uint32_t x, stage, bars, total;
};
__host__ __device__ constexpr uint32_t align128(uint32_t v) { return (v + 127u) & ~127u; }
__host__ __device__ inline Smem carve(uint32_t xbytes, int nx, uint32_t sbytes, int ns) {
  Smem L{};
  L.x = 0;
  L.stage = align128(L.x + nx * align128(xbytes));
  L.bars = align128(L.stage + ns * align128(sbytes));
  L.total = L.bars + 8 * (4 + 2 * ns);
  return L;
}

// ------------------------------------------------------------- forward ------
template <typename T, int D>
__device__ __forceinline__ void fwd_branch(const T* xs, const T* stage_base, uint32_t sstride,
                                           int ns, uint64_t* full, uint64_t* empty, uint32_t& s,
                                           int col, int r0, volatile int* abort_flag,
                                           float (&acc)[Geo<T>::RPT][Geo<T>::VEC], bool& ok) {
  using Gm = Geo<T>;
  constexpr int VEC = Gm::VEC;
  constexpr int R = 5;  // (K/2) * max dilation for (1, 3, 5)
#pragma unroll
  for (int j = 0; j < Gm::RPT; ++j)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[j][v] = 0.f;
#pragma unroll
  for (int ki = 0; ki < kKS; ++ki, ++s) {
    const int slot = s % ns;
    if (!cwait(&full[slot], (s / ns) & 1, abort_flag)) {
      ok = false;
      return;
    }
    const T* taps = stage_base + slot * sstride;
    const int dy = (ki - 1) * D;
#pragma unroll
    for (int j = 0; j < Gm::RPT; ++j) {
      const int row = r0 + j * Gm::ROWSTEP;
      // x at columns w - 8 .. w + VEC + 7 of source row (row + dy)
      const T* xrow = xs + (R + row + dy) * kHaloCols + VEC * col;
      float xv[VEC + 16];
#pragma unroll
      for (int q = 0; q < (VEC + 16) / VEC; ++q) {
        float t[VEC];
        lds_vec<T>(xrow + q * VEC, t);
#pragma unroll
        for (int v = 0; v < VEC; ++v) xv[q * VEC + v] = t[v];
      }
#pragma unroll
      for (int kj = 0; kj < kKS; ++kj) {
        float kv[VEC];
        lds_vec<T>(taps + (kj * kTH + row) * kTW + VEC * col, kv);
        const int dx = (kj - 1) * D;
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[j][v] = fmaf(xv[8 + v + dx], kv[v], acc[j][v]);
      }
    }
    warp_arrive(&empty[slot]);
  }
}

template <typename T, int NS>
__global__ void __launch_bounds__(kThreads) fwd_tma_kernel(const __grid_constant__ TmaParams p) {
  using Gm = Geo<T>;
  constexpr int VEC = Gm::VEC;
  constexpr int R = 5;
  constexpr uint32_t XBYTES = (kTH + 2 * R) * kHaloCols * sizeof(T);
  constexpr uint32_t SBYTES = kKS * kTH * kTW * sizeof(T);
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ int abort_s;
  const Smem L = carve(XBYTES, 2, SBYTES, NS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* x_full = bars;         // [2]
  uint64_t* x_empty = bars + 2;    // [2]
  uint64_t* full = bars + 4;       // [NS]
  uint64_t* empty = full + NS;     // [NS]
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&x_full[i], 1);
      tc::mbar_init(&x_empty[i], kConsumers / 32);
    }
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], kConsumers / 32);
    }
    tc::fence_mbar_init();
    abort_s = 0;
  }
  __syncthreads();
  volatile int* abort_flag = &abort_s;
  const int C = p.C, H = p.H, W = p.W;
  const size_t P = (size_t)H * W;

  if (threadIdx.x >= kConsumers) {
    // ---- producer --------------------------------------------------------
    if (threadIdx.x == kConsumers) {
      uint32_t s = 0, it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int n, c, h0, w0;
        tile_coords(p, tile, n, c, h0, w0);
        const int xb = it & 1;
        if (!tc::mbar_wait(&x_empty[xb], ((it >> 1) & 1) ^ 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 40);
          break;
        }
        tc::mbar_arrive_expect_tx(&x_full[xb], XBYTES);
        tma_load_3d(smem + L.x + xb * align128(XBYTES), &p.src, w0 - 8, h0 - R, n * C + c,
                    &x_full[xb]);
        bool stop = false;
        for (int b = 0; b < 3 && !stop; ++b) {
          for (int ki = 0; ki < kKS; ++ki, ++s) {
            const int slot = s % NS;
            if (!tc::mbar_wait(&empty[slot], ((s / NS) & 1) ^ 1, abort_flag, kWaitNs)) {
              fail(abort_flag, p.status, 41);
              stop = true;
              break;
            }
            tc::mbar_arrive_expect_tx(&full[slot], SBYTES);
            tma_load_3d(smem + L.stage + slot * align128(SBYTES), &p.aux, w0, h0,
                        ((n * 3 + b) * C + c) * 9 + ki * kKS, &full[slot]);
          }
        }
        if (stop) {
          ++it;
          break;
        }
      }
      drain(full, NS, s, abort_flag);
      drain(x_full, 2, it, abort_flag);
    }
  } else {
    // ---- consumers ---------------------------------------------------------
    const int col = threadIdx.x % Gm::TPR;
    const int r0 = threadIdx.x / Gm::TPR;
    T* out = static_cast<T*>(p.out);
    const T* stage_base = reinterpret_cast<const T*>(smem + L.stage);
    const uint32_t sstride = align128(SBYTES) / sizeof(T);
    uint32_t s = 0, it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int n, c, h0, w0;
      tile_coords(p, tile, n, c, h0, w0);
      const int xb = it & 1;
      if (!cwait(&x_full[xb], (it >> 1) & 1, abort_flag)) {
        fail(abort_flag, p.status, 42);
        break;
      }
      const T* xs = reinterpret_cast<const T*>(smem + L.x + xb * align128(XBYTES));
      const int w = w0 + VEC * col;
      T* on = out + ((size_t)n * 4 * C + c) * P;
      // passthrough out[:, c] = x, straight from the halo box
#pragma unroll
      for (int j = 0; j < Gm::RPT; ++j) {
        const int h = h0 + r0 + j * Gm::ROWSTEP;
        if (h < H && w < W)
          __stcs(reinterpret_cast<uint4*>(on + (size_t)h * W + w),
                 *reinterpret_cast<const uint4*>(xs + (R + r0 + j * Gm::ROWSTEP) * kHaloCols +
                                                 8 + VEC * col));
      }
      float acc[Gm::RPT][VEC];
      bool ok = true;
#pragma unroll
      for (int b = 0; b < 3; ++b) {
        if (b == 0)
          fwd_branch<T, 1>(xs, stage_base, sstride, NS, full, empty, s, col, r0, abort_flag, acc, ok);
        else if (b == 1)
          fwd_branch<T, 3>(xs, stage_base, sstride, NS, full, empty, s, col, r0, abort_flag, acc, ok);
        else
          fwd_branch<T, 5>(xs, stage_base, sstride, NS, full, empty, s, col, r0, abort_flag, acc, ok);
        if (!ok) break;
        T* ob = on + (size_t)(b + 1) * C * P;
#pragma unroll
        for (int j = 0; j < Gm::RPT; ++j) {
          const int h = h0 + r0 + j * Gm::ROWSTEP;
          if (h < H && w < W) stg_vec<T>(ob + (size_t)h * W + w, acc[j]);
        }
      }
      if (!ok) {
        fail(abort_flag, p.status, 43);
        break;
      }
      warp_arrive(&x_empty[xb]);
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------- dK --------
// dK[b, tap, p] = x[p + off] * g_b[p]: per tile the x halo box and the three
// branch-gradient tiles (one box {128, 16, 1, 3, 1}), double buffered; the
// consumers only compute and store the 27 tap planes.
template <typename T, int D>
__device__ __forceinline__ void bwdk_branch(const T* xs, const T* gs, T* gk_branch, size_t P,
                                            int H, int W, int h0, int w, int col, int r0) {
  using Gm = Geo<T>;
  constexpr int VEC = Gm::VEC;
  constexpr int R = 5;
#pragma unroll
  for (int j = 0; j < Gm::RPT; ++j) {
    const int row = r0 + j * Gm::ROWSTEP;
    const int h = h0 + row;
    float g[VEC];
    lds_vec<T>(gs + row * kTW + VEC * col, g);
#pragma unroll
    for (int ki = 0; ki < kKS; ++ki) {
      const int dy = (ki - 1) * D;
      const T* xrow = xs + (R + row + dy) * kHaloCols + VEC * col;
      float xv[VEC + 16];
#pragma unroll
      for (int q = 0; q < (VEC + 16) / VEC; ++q) {
        float t[VEC];
        lds_vec<T>(xrow + q * VEC, t);
#pragma unroll
        for (int v = 0; v < VEC; ++v) xv[q * VEC + v] = t[v];
      }
      if (h < H && w < W) {
#pragma unroll
        for (int kj = 0; kj < kKS; ++kj) {
          const int dx = (kj - 1) * D;
          float o[VEC];
#pragma unroll
          for (int v = 0; v < VEC; ++v) o[v] = xv[8 + v + dx] * g[v];
          stg_vec<T>(gk_branch + (size_t)(ki * kKS + kj) * P + (size_t)h * W + w, o);
        }
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) bwdk_tma_kernel(const __grid_constant__ TmaParams p) {
  using Gm = Geo<T>;
  constexpr int VEC = Gm::VEC;
  constexpr int R = 5;
  constexpr uint32_t XBYTES = (kTH + 2 * R) * kHaloCols * sizeof(T);
  constexpr uint32_t GBYTES = 3 * kTH * kTW * sizeof(T);
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ int abort_s;
  // two buffers, each the x halo box followed by the three gradient tiles
  const uint32_t buf = align128(XBYTES) + align128(GBYTES);
  const Smem L = carve(buf, 2, 0, 0);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* x_full = bars;
  uint64_t* x_empty = bars + 2;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&x_full[i], 1);
      tc::mbar_init(&x_empty[i], kConsumers / 32);
    }
    tc::fence_mbar_init();
    abort_s = 0;
  }
  __syncthreads();
  volatile int* abort_flag = &abort_s;
  const int C = p.C, H = p.H, W = p.W;
  const size_t P = (size_t)H * W;

  if (threadIdx.x >= kConsumers) {
    if (threadIdx.x == kConsumers) {
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int n, c, h0, w0;
        tile_coords(p, tile, n, c, h0, w0);
        const int xb = it & 1;
        if (!tc::mbar_wait(&x_empty[xb], ((it >> 1) & 1) ^ 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 44);
          break;
        }
        uint8_t* dst = smem + L.x + xb * align128(buf);
        tc::mbar_arrive_expect_tx(&x_full[xb], XBYTES + GBYTES);
        tma_load_3d(dst, &p.src, w0 - 8, h0 - R, n * C + c, &x_full[xb]);
        tc::tma_load_5d(dst + align128(XBYTES), &p.aux, w0, h0, c, 1, n, &x_full[xb]);
      }
      drain(x_full, 2, it, abort_flag);
    }
  } else {
    const int col = threadIdx.x % Gm::TPR;
    const int r0 = threadIdx.x / Gm::TPR;
    T* gk = static_cast<T*>(p.out);
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int n, c, h0, w0;
      tile_coords(p, tile, n, c, h0, w0);
      const int xb = it & 1;
      if (!cwait(&x_full[xb], (it >> 1) & 1, abort_flag)) {
        fail(abort_flag, p.status, 45);
        break;
      }
      const T* xs = reinterpret_cast<const T*>(smem + L.x + xb * align128(buf));
      const T* gs = reinterpret_cast<const T*>(smem + L.x + xb * align128(buf) + align128(XBYTES));
      const int w = w0 + VEC * col;
      const size_t kb = ((size_t)n * 3 * C + c) * 9 * P;
      const size_t kbr = (size_t)C * 9 * P;
      bwdk_branch<T, 1>(xs, gs, gk + kb, P, H, W, h0, w, col, r0);
      bwdk_branch<T, 3>(xs, gs + kTH * kTW, gk + kb + kbr, P, H, W, h0, w, col, r0);
      bwdk_branch<T, 5>(xs, gs + 2 * kTH * kTW, gk + kb + 2 * kbr, P, H, W, h0, w, col, r0);
      warp_arrive(&x_empty[xb]);
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------- dX --------
// dX[q] = g0[q] + sum_{b, tap} K[b, tap, q - off] * g_b[q - off]: per tile the
// four gradient planes (g0 and the three branches) with the halo, one box
// {144, 16 + 2R, 1, 4, 1}, double buffered; per (branch, kernel row) a stage
// of the three taps at their shifted source windows.

// floor(v / VEC) * VEC for small |v|
template <int VEC>
__host__ __device__ constexpr int floor_vec(int v) {
  return v >= 0 ? v / VEC * VEC : -((-v + VEC - 1) / VEC) * VEC;
}

template <typename T, int D>
__device__ __forceinline__ void bwdx_branch(const T* gbr, const T* stage_base, uint32_t sstride,
                                            int ns, uint64_t* full, uint64_t* empty, uint32_t& s,
                                            int col, int r0, volatile int* abort_flag,
                                            float (&acc)[Geo<T>::RPT][Geo<T>::VEC], bool& ok) {
  using Gm = Geo<T>;
  constexpr int VEC = Gm::VEC;
  constexpr int R = 5;
#pragma unroll
  for (int ki = 0; ki < kKS; ++ki, ++s) {
    const int slot = s % ns;
    if (!cwait(&full[slot], (s / ns) & 1, abort_flag)) {
      ok = false;
      return;
    }
    const T* taps = stage_base + slot * sstride;
    const int dy = (ki - 1) * D;
#pragma unroll
    for (int j = 0; j < Gm::RPT; ++j) {
      const int row = r0 + j * Gm::ROWSTEP;
      // g_b at source row (row - dy), columns from (w - dx): halo box row
      // R + row - dy, box column 8 - dx + VEC * col
      const T* grow = gbr + (R + row - dy) * kHaloCols + VEC * col;
#pragma unroll
      for (int kj = 0; kj < kKS; ++kj) {
        // the tap window at source columns w - dx .. : its box starts at
        // column w0 + floor_VEC(-dx), so the window sits O = -dx - floor_VEC(-dx)
        // elements into the thread's vector
        float kv[VEC], gv[VEC];
        const T* trow = taps + (kj * kTH + row) * kWinCols + VEC * col;
        if (kj == 0) {
          constexpr int DX = -D;
          constexpr int O = -DX - floor_vec<VEC>(-DX);
          lds_window<T, O>(trow, kv);
          constexpr int G = 8 - DX;
          lds_window<T, G % VEC>(grow + G / VEC * VEC, gv);
        } else if (kj == 1) {
          lds_vec<T>(trow, kv);
          lds_vec<T>(grow + 8, gv);
        } else {
          constexpr int DX = D;
          constexpr int O = -DX - floor_vec<VEC>(-DX);
          lds_window<T, O>(trow, kv);
          constexpr int G = 8 - DX;
          lds_window<T, G % VEC>(grow + G / VEC * VEC, gv);
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[j][v] = fmaf(kv[v], gv[v], acc[j][v]);
      }
    }
    warp_arrive(&empty[slot]);
  }
}

template <typename T, int NS>
__global__ void __launch_bounds__(kThreads) bwdx_tma_kernel(const __grid_constant__ TmaParams p) {
  using Gm = Geo<T>;
  constexpr int VEC = Gm::VEC;
  constexpr int R = 5;
  constexpr uint32_t GBYTES = 4 * (kTH + 2 * R) * kHaloCols * sizeof(T);
  constexpr uint32_t TAPBYTES = kTH * kWinCols * sizeof(T);
  constexpr uint32_t SBYTES = kKS * TAPBYTES;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ int abort_s;
  const Smem L = carve(GBYTES, 2, SBYTES, NS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* g_full = bars;
  uint64_t* g_empty = bars + 2;
  uint64_t* full = bars + 4;
  uint64_t* empty = full + NS;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&g_full[i], 1);
      tc::mbar_init(&g_empty[i], kConsumers / 32);
    }
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], kConsumers / 32);
    }
    tc::fence_mbar_init();
    abort_s = 0;
  }
  __syncthreads();
  volatile int* abort_flag = &abort_s;
  const int C = p.C, H = p.H, W = p.W;
  const size_t P = (size_t)H * W;
  constexpr int kDil[3] = {1, 3, 5};

  if (threadIdx.x >= kConsumers) {
    if (threadIdx.x == kConsumers) {
      uint32_t s = 0, it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int n, c, h0, w0;
        tile_coords(p, tile, n, c, h0, w0);
        const int gb = it & 1;
        if (!tc::mbar_wait(&g_empty[gb], ((it >> 1) & 1) ^ 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 46);
          break;
        }
        tc::mbar_arrive_expect_tx(&g_full[gb], GBYTES);
        tc::tma_load_5d(smem + L.x + gb * align128(GBYTES), &p.src, w0 - 8, h0 - R, c, 0, n,
                        &g_full[gb]);
        bool stop = false;
        for (int b = 0; b < 3 && !stop; ++b) {
          const int d = kDil[b];
          for (int ki = 0; ki < kKS; ++ki, ++s) {
            const int slot = s % NS;
            if (!tc::mbar_wait(&empty[slot], ((s / NS) & 1) ^ 1, abort_flag, kWaitNs)) {
              fail(abort_flag, p.status, 47);
              stop = true;
              break;
            }
            tc::mbar_arrive_expect_tx(&full[slot], SBYTES);
            const int dy = (ki - 1) * d;
            uint8_t* dst = smem + L.stage + slot * align128(SBYTES);
            const int plane = ((n * 3 + b) * C + c) * 9 + ki * kKS;
            for (int kj = 0; kj < kKS; ++kj) {
              const int dx = (kj - 1) * d;
              tma_load_3d(dst + kj * TAPBYTES, &p.aux, w0 + floor_vec<VEC>(-dx), h0 - dy,
                          plane + kj, &full[slot]);
            }
          }
        }
        if (stop) {
          ++it;
          break;
        }
      }
      drain(full, NS, s, abort_flag);
      drain(g_full, 2, it, abort_flag);
    }
  } else {
    const int col = threadIdx.x % Gm::TPR;
    const int r0 = threadIdx.x / Gm::TPR;
    T* gx = static_cast<T*>(p.out);
    const T* stage_base = reinterpret_cast<const T*>(smem + L.stage);
    const uint32_t sstride = align128(SBYTES) / sizeof(T);
    constexpr uint32_t plane = (kTH + 2 * R) * kHaloCols;  // elements per g plane
    uint32_t s = 0, it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int n, c, h0, w0;
      tile_coords(p, tile, n, c, h0, w0);
      const int gb = it & 1;
      if (!cwait(&g_full[gb], (it >> 1) & 1, abort_flag)) {
        fail(abort_flag, p.status, 48);
        break;
      }
      const T* gs = reinterpret_cast<const T*>(smem + L.x + gb * align128(GBYTES));
      const int w = w0 + VEC * col;
      float acc[Gm::RPT][VEC];
      // the passthrough's gradient g0[q]
#pragma unroll
      for (int j = 0; j < Gm::RPT; ++j)
        lds_vec<T>(gs + (R + r0 + j * Gm::ROWSTEP) * kHaloCols + 8 + VEC * col, acc[j]);
      bool ok = true;
      bwdx_branch<T, 1>(gs + plane, stage_base, sstride, NS, full, empty, s, col, r0, abort_flag,
                        acc, ok);
      if (ok)
        bwdx_branch<T, 3>(gs + 2 * plane, stage_base, sstride, NS, full, empty, s, col, r0,
                          abort_flag, acc, ok);
      if (ok)
        bwdx_branch<T, 5>(gs + 3 * plane, stage_base, sstride, NS, full, empty, s, col, r0,
                          abort_flag, acc, ok);
      if (!ok) {
        fail(abort_flag, p.status, 49);
        break;
      }
      T* gxn = gx + ((size_t)n * C + c) * P;
#pragma unroll
      for (int j = 0; j < Gm::RPT; ++j) {
        const int h = h0 + r0 + j * Gm::ROWSTEP;
        if (h < H && w < W) stg_vec<T>(gxn + (size_t)h * W + w, acc[j]);
      }
      warp_arrive(&g_empty[gb]);
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------- host ---------
template <typename T>
CUtensorMapDataType tmap_type() {
  if constexpr (sizeof(T) == 4) return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if constexpr (std::is_same<T, __half>::value) return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// 3-D view {W, H, planes} of contiguous [planes, H, W] data.
template <typename T>
int map_planes(CUtensorMap* m, const void* base, int w, int h, long long planes, uint32_t bw,
               uint32_t bh, uint32_t bp) {
  const uint64_t dims[3] = {(uint64_t)w, (uint64_t)h, (uint64_t)planes};
  const uint64_t strides[2] = {(uint64_t)w * sizeof(T), (uint64_t)w * h * sizeof(T)};
  const uint32_t box[3] = {bw, bh, bp};
  return encode_tmap(m, tmap_type<T>(), 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// 5-D view {W, H, C, 4, N} of grad_out [N, 4C, H, W].
template <typename T>
int map_gout(CUtensorMap* m, const void* base, int n, int c, int w, int h, uint32_t bw,
             uint32_t bh, uint32_t bb) {
  const uint64_t e = sizeof(T);
  const uint64_t dims[5] = {(uint64_t)w, (uint64_t)h, (uint64_t)c, 4, (uint64_t)n};
  const uint64_t strides[4] = {(uint64_t)w * e, (uint64_t)w * h * e, (uint64_t)c * w * h * e,
                               (uint64_t)4 * c * w * h * e};
  const uint32_t box[5] = {bw, bh, 1, bb, 1};
  return encode_tmap(m, tmap_type<T>(), 5, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <typename K>
int grid_for(K kernel, uint32_t smem, int num_tiles, int* grid) {
  if (smem > 48 * 1024)
    DDPM_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
  int per_sm = 0;
  DDPM_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem));
  if (per_sm < 1) return set_error(DDPM_ERR_UNSUPPORTED, "TMA filter kernel does not fit an SM");
  const int want = gencat::num_sms() * per_sm;
  *grid = num_tiles < want ? num_tiles : want;
  return DDPM_OK;
}

TmaParams base_params(void* out, int n, int c, int h, int w) {
  TmaParams q{};
  q.out = out;
  q.N = n;
  q.C = c;
  q.H = h;
  q.W = w;
  q.tiles_w = (w + kTW - 1) / kTW;
  q.tiles_h = (h + kTH - 1) / kTH;
  q.num_tiles = n * c * q.tiles_w * q.tiles_h;
  return q;
}

// Stage depths: enough stages in flight for HBM latency, two CTAs per SM
// where they fit.
template <typename T> constexpr int fwd_stages() { return sizeof(T) == 4 ? 3 : 6; }
template <typename T> constexpr int bwdx_stages() { return sizeof(T) == 4 ? 3 : 3; }

template <typename T>
int fwd_tma(const void* x, const void* k, void* out, int n, int c, int h, int w, cudaStream_t st) {
  TmaParams q = base_params(out, n, c, h, w);
  if (int rc = gencat::status_ptr(&q.status)) return rc;
  if (map_planes<T>(&q.src, x, w, h, (long long)n * c, kHaloCols, kTH + 10, 1) ||
      map_planes<T>(&q.aux, k, w, h, (long long)n * 3 * c * 9, kTW, kTH, kKS))
    return DDPM_ERR_UNSUPPORTED;
  constexpr int NS = fwd_stages<T>();
  const Smem L = carve((kTH + 10) * kHaloCols * sizeof(T), 2, kKS * kTH * kTW * sizeof(T), NS);
  auto fn = fwd_tma_kernel<T, NS>;
  int grid = 0;
  if (int rc = grid_for(fn, L.total, q.num_tiles, &grid)) return rc;
  fn<<<grid, kThreads, L.total, st>>>(q);
  DDPM_CHECK_LAUNCH("dyncat_fwd_tma_kernel");
  return DDPM_OK;
}

template <typename T>
int bwdk_tma(const void* x, const void* g, void* gk, int n, int c, int h, int w, cudaStream_t st) {
  TmaParams q = base_params(gk, n, c, h, w);
  if (int rc = gencat::status_ptr(&q.status)) return rc;
  if (map_planes<T>(&q.src, x, w, h, (long long)n * c, kHaloCols, kTH + 10, 1) ||
      map_gout<T>(&q.aux, g, n, c, w, h, kTW, kTH, 3))
    return DDPM_ERR_UNSUPPORTED;
  const uint32_t buf = align128((kTH + 10) * kHaloCols * sizeof(T)) +
                       align128(3 * kTH * kTW * sizeof(T));
  const Smem L = carve(buf, 2, 0, 0);
  auto fn = bwdk_tma_kernel<T>;
  int grid = 0;
  if (int rc = grid_for(fn, L.total, q.num_tiles, &grid)) return rc;
  fn<<<grid, kThreads, L.total, st>>>(q);
  DDPM_CHECK_LAUNCH("dyncat_bwdk_tma_kernel");
  return DDPM_OK;
}

template <typename T>
int bwdx_tma(const void* k, const void* g, void* gx, int n, int c, int h, int w, cudaStream_t st) {
  TmaParams q = base_params(gx, n, c, h, w);
  if (int rc = gencat::status_ptr(&q.status)) return rc;
  if (map_gout<T>(&q.src, g, n, c, w, h, kHaloCols, kTH + 10, 4) ||
      map_planes<T>(&q.aux, k, w, h, (long long)n * 3 * c * 9, kWinCols, kTH, 1))
    return DDPM_ERR_UNSUPPORTED;
  constexpr int NS = bwdx_stages<T>();
  const Smem L = carve(4 * (kTH + 10) * kHaloCols * sizeof(T), 2,
                       kKS * kTH * kWinCols * sizeof(T), NS);
  auto fn = bwdx_tma_kernel<T, NS>;
  int grid = 0;
  if (int rc = grid_for(fn, L.total, q.num_tiles, &grid)) return rc;
  fn<<<grid, kThreads, L.total, st>>>(q);
  DDPM_CHECK_LAUNCH("dyncat_bwdx_tma_kernel");
  return DDPM_OK;
}

bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Whether the TMA kernels serve this call: K = 3, dilations (1, 3, 5), one
// dtype for x and the taps, rows of whole 16-byte vectors (W % 8 == 0) and
// 16-byte aligned tensors.
bool dyncat_tma_eligible(int xdt, int kdt, int w, int ks, int d0, int d1, int d2,
                         std::initializer_list<const void*> ptrs) {
  if (xdt != kdt || ks != 3 || d0 != 1 || d1 != 3 || d2 != 5 || w % 8 != 0) return false;
  if (dtype_size(xdt) == 0) return false;
  for (const void* p : ptrs)
    if (!aligned16(p)) return false;
  return true;
}

// The TMA kernels; DDPM_ERR_UNSUPPORTED (with nothing launched) when a tensor
// map cannot be encoded, so the caller takes the kernels of dyncat.cu.
int dyncat_fwd_tma(const void* x, const void* k, void* out, int n, int c, int h, int w, int dt,
                   cudaStream_t st) {
  switch (dt) {
    case DDPM_BF16: return fwd_tma<__nv_bfloat16>(x, k, out, n, c, h, w, st);
    case DDPM_F16: return fwd_tma<__half>(x, k, out, n, c, h, w, st);
    case DDPM_F32: return fwd_tma<float>(x, k, out, n, c, h, w, st);
  }
  return DDPM_ERR_UNSUPPORTED;
}

int dyncat_bwdk_tma(const void* x, const void* g, void* gk, int n, int c, int h, int w, int dt,
                    cudaStream_t st) {
  switch (dt) {
    case DDPM_BF16: return bwdk_tma<__nv_bfloat16>(x, g, gk, n, c, h, w, st);
    case DDPM_F16: return bwdk_tma<__half>(x, g, gk, n, c, h, w, st);
    case DDPM_F32: return bwdk_tma<float>(x, g, gk, n, c, h, w, st);
  }
  return DDPM_ERR_UNSUPPORTED;
}

int dyncat_bwdx_tma(const void* k, const void* g, void* gx, int n, int c, int h, int w, int dt,
                    cudaStream_t st) {
  switch (dt) {
    case DDPM_BF16: return bwdx_tma<__nv_bfloat16>(k, g, gx, n, c, h, w, st);
    case DDPM_F16: return bwdx_tma<__half>(k, g, gx, n, c, h, w, st);
    case DDPM_F32: return bwdx_tma<float>(k, g, gx, n, c, h, w, st);
  }
  return DDPM_ERR_UNSUPPORTED;
}

}  // namespace ddpm
