// Fused generator backward: dY, and dW / db, with dK formed on chip.
// Replaces `_generator_dynamic_cat_bwd_y` (reference `_triton_kernels.py:534-623`),
// `_generator_dynamic_cat_bwd_weight_partial` (`:626-751`) and
// `_generator_dynamic_cat_bwd_weight_reduce` (`:754-811`):
//
//   dK[(b,c,tap), p] = x[c, p + o] * g_b[c, p]            (never stored to HBM)
//   dY[i, p]         = sum_{(b,c,tap)} W[(b,c,tap), i] * dK[(b,c,tap), p]
//   dW[(b,c,tap), i] = sum_p dK[(b,c,tap), p] * y[i, p]
//   db[(b,c,tap)]    = sum_p dK[(b,c,tap), p]
//
// Both GEMMs take dK as their A operand. Weight rows are processed in groups
// of 128 = 8 (branch, tap) "slots" x 16 channels (one x-halo channel group).
// A group's dK tile is built in shared memory by CUDA-core builder warps,
// thread = pixel: for each slot one 16-channel x neighbour (four LDS.128 from
// the staged FP32 halo, as in the forward) times the 16 g_b values of the
// pixel, written as two 16-byte rows. The tile layout
//   (pixel m, row) at (m/8)*2048 + (row/8)*128 + (m%8)*16 + (row%8)*2
// is at once the K-major operand [pixels x rows] of the dY GEMM and the
// MN-major operand [rows x pixels] of the dW GEMM (same core matrices).
//
// dY kernel: persistent over 8x16 pixel tiles; D_y (128 pixels x Cp) sits in
// TMEM for the whole tile while the transposed-weight groups (packed "by"
// image) stream through a ring; builders drain D_y to dY at the end of a tile.
// dW kernel: grid = (group batch, spatial split); D_w of up to 6 groups
// (128 rows x Nw each, Nw = round16(C + 1): the y tile carries a constant-one
// channel at index C so column C of D_w is db) accumulates over all tiles of
// the split; partials go to a workspace and a short kernel reduces them into
// the Conv2d weight layout.
#include <mutex>

#include "common.cuh"
#include "tc.cuh"
#include "gencat.cuh"
#include "tmap.cuh"

namespace ddpm {
namespace {

using namespace gencat;

constexpr int kDkBytes = kTileM * 128 * 2;  // one dK tile part (bf16 / fp16)

// ----------------------------------------------------------- dK builder -----
// Slots of octet OCT: s = OCT*8 + j -> (b, tap) = (s / K^2, s % K^2); s >= 3K^2
// is padding (zero rows). gv[b][i] = the pair (g_b[2i], g_b[2i+1]) of this
// pixel's 16-channel group, packed; products and conversions run on f32x2 /
// bf16x2 pairs.
// `cols`: cells per halo row (kHaloCols, or 16 + 2R for K = 5).
template <typename T, typename Op, bool kSplit, int KS, int OCT, int J0 = 0, int JN = 8>
__device__ __forceinline__ void build_octet(uint8_t* dk, const float4* xc, int xr_plane,
                                            const unsigned long long (&gv)[3][8],
                                            const int (&dil)[3], int m,
                                            uint32_t lo_off = kDkBytes, int cols = kHaloCols) {
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  const uint32_t base = (m >> 3) * 2048 + (m & 7) * 16;
  const unsigned long long zero2 = 0ull;
#pragma unroll
  for (int j = J0; j < J0 + JN; ++j) {
    const int s = OCT * 8 + j;
    unsigned long long prod[8];
    if (s < 3 * KK) {
      const int b = s / KK, tap = s % KK;
      const int dy = (tap / KS - r) * dil[b], dx = (tap % KS - r) * dil[b];
      const float4* cell = xc + dy * cols + dx;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const float4 v = cell[q4 * xr_plane];
        prod[q4 * 2 + 0] = f2_fma(f2_pack(v.x, v.y), gv[b][q4 * 2 + 0], zero2);
        prod[q4 * 2 + 1] = f2_fma(f2_pack(v.z, v.w), gv[b][q4 * 2 + 1], zero2);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) prod[i] = zero2;
    }
    const unsigned long long lo8[4] = {prod[0], prod[1], prod[2], prod[3]};
    const unsigned long long hi8[4] = {prod[4], prod[5], prod[6], prod[7]};
    const uint32_t off = base + (j * 2) * 128;
    store8x2_split<Op, kSplit>(dk + off, dk + lo_off + off, lo8);
    store8x2_split<Op, kSplit>(dk + off + 128, dk + lo_off + off + 128, hi8);
  }
}

template <typename T, typename Op, bool kSplit, int KS>
__device__ __forceinline__ void build_dk(uint8_t* dk, int octet, const float4* xc, int xr_plane,
                                         const unsigned long long (&gv)[3][8],
                                         const int (&dil)[3], int m) {
  switch (octet) {
    case 0: build_octet<T, Op, kSplit, KS, 0>(dk, xc, xr_plane, gv, dil, m); break;
    case 1: build_octet<T, Op, kSplit, KS, 1>(dk, xc, xr_plane, gv, dil, m); break;
    case 2: build_octet<T, Op, kSplit, KS, 2>(dk, xc, xr_plane, gv, dil, m); break;
    default: build_octet<T, Op, kSplit, KS, 3>(dk, xc, xr_plane, gv, dil, m); break;
  }
}

// Half of an octet (slots 4*half .. 4*half+3): two builder threads per pixel.
// lo_off: bytes from a slot's hi part to its lo part (FP32).
template <typename T, typename Op, bool kSplit, int KS, int O = 0>
__device__ __forceinline__ void build_dk_half(uint8_t* dk, int octet, int half, const float4* xc,
                                              int xr_plane, const unsigned long long (&gv)[3][8],
                                              const int (&dil)[3], int m,
                                              uint32_t lo_off = kDkBytes, int cols = kHaloCols) {
  constexpr int kOct = (3 * KS * KS + 7) / 8;
  if constexpr (O < kOct) {
    if (octet == O || O == kOct - 1) {
      if (half == 0)
        build_octet<T, Op, kSplit, KS, O, 0, 4>(dk, xc, xr_plane, gv, dil, m, lo_off, cols);
      else
        build_octet<T, Op, kSplit, KS, O, 4, 4>(dk, xc, xr_plane, gv, dil, m, lo_off, cols);
      return;
    }
    build_dk_half<T, Op, kSplit, KS, O + 1>(dk, octet, half, xc, xr_plane, gv, dil, m, lo_off,
                                            cols);
  }
}

// The same octet half from an x halo of 8-channel 16-bit cells (staged 16-bit
// data): gw[b][i] = the raw pair (g_b[2i], g_b[2i+1]) of the pixel's 16
// channels; each dK pair is one packed 16-bit multiply of an x word and a g
// word, rounded once (the value the FP32 product and conversion give).
template <typename T, typename Op, int KS, int OCT, int J0>
__device__ __forceinline__ void build_octet_io(uint8_t* dk, const uint4* xc, int xr_plane,
                                               const uint32_t (&gw)[3][8], const int (&dil)[3],
                                               int m, int cols) {
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  const uint32_t base = (m >> 3) * 2048 + (m & 7) * 16;
#pragma unroll
  for (int j = J0; j < J0 + 4; ++j) {
    const int s = OCT * 8 + j;
    uint32_t pw[8];
    if (s < 3 * KK) {
      const int b = s / KK, tap = s % KK;
      const int dy = (tap / KS - r) * dil[b], dx = (tap % KS - r) * dil[b];
      const uint4* cell = xc + dy * cols + dx;
#pragma unroll
      for (int c8 = 0; c8 < 2; ++c8) {
        const uint4 v = cell[c8 * xr_plane];
        pw[c8 * 4 + 0] = mul_io2<Op>(v.x, gw[b][c8 * 4 + 0]);
        pw[c8 * 4 + 1] = mul_io2<Op>(v.y, gw[b][c8 * 4 + 1]);
        pw[c8 * 4 + 2] = mul_io2<Op>(v.z, gw[b][c8 * 4 + 2]);
        pw[c8 * 4 + 3] = mul_io2<Op>(v.w, gw[b][c8 * 4 + 3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) pw[i] = 0u;
    }
    const uint32_t off = base + (j * 2) * 128;
    *reinterpret_cast<uint4*>(dk + off) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
    *reinterpret_cast<uint4*>(dk + off + 128) = make_uint4(pw[4], pw[5], pw[6], pw[7]);
  }
}

template <typename T, typename Op, int KS, int O = 0>
__device__ __forceinline__ void build_dk_half_io(uint8_t* dk, int octet, int half, const uint4* xc,
                                                 int xr_plane, const uint32_t (&gw)[3][8],
                                                 const int (&dil)[3], int m, int cols) {
  constexpr int kOct = (3 * KS * KS + 7) / 8;
  if constexpr (O < kOct) {
    if (octet == O || O == kOct - 1) {
      if (half == 0)
        build_octet_io<T, Op, KS, O, 0>(dk, xc, xr_plane, gw, dil, m, cols);
      else
        build_octet_io<T, Op, KS, O, 4>(dk, xc, xr_plane, gw, dil, m, cols);
      return;
    }
    build_dk_half_io<T, Op, KS, O + 1>(dk, octet, half, xc, xr_plane, gw, dil, m, cols);
  }
}

// g_b[cg16*16 + cl, pixel] for the three branches (zero off-image / c >= C).
template <typename T>
__device__ __forceinline__ void load_gv(unsigned long long (&gv)[3][8], const T* gn, int C,
                                        size_t P, int cg16, size_t pix, bool px_ok) {
  float v[3][16];
#pragma unroll
  for (int b = 0; b < 3; ++b)
#pragma unroll
    for (int cl = 0; cl < 16; ++cl) {
      const int c = cg16 * 16 + cl;
      v[b][cl] = (px_ok && c < C) ? to_f32<T>(__ldg(gn + (size_t)((b + 1) * C + c) * P + pix))
                                  : 0.f;
    }
#pragma unroll
  for (int b = 0; b < 3; ++b)
#pragma unroll
    for (int i = 0; i < 8; ++i) gv[b][i] = f2_pack(v[b][2 * i], v[b][2 * i + 1]);
}

// The same from a channel-last grad_out [N][H][W][4C]: per branch the 16
// channels are one contiguous run (16-byte vector loads).
template <typename T>
__device__ __forceinline__ void load_gv_nhwc(unsigned long long (&gv)[3][8], const T* gout, int n,
                                             int H, int W, int C, int cg16, int h, int w,
                                             bool px_ok) {
  constexpr int kVecs = 16 * (int)sizeof(T) / 16;  // vectors per 16 channels
  constexpr int kPer = 16 / (int)sizeof(T);        // elements per vector
#pragma unroll
  for (int b = 0; b < 3; ++b) {
    float v[16];
    const uint4* src = reinterpret_cast<const uint4*>(
        gout + (((size_t)n * H + h) * W + w) * 4 * C + (b + 1) * C + cg16 * 16);
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
      uint4 u = make_uint4(0u, 0u, 0u, 0u);
      if (px_ok) u = __ldg(src + k);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < kPer; ++i) v[k * kPer + i] = to_f32<T>(e[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) gv[b][i] = f2_pack(v[2 * i], v[2 * i + 1]);
  }
}

// =============================================================== dY =========
template <typename T, int KS>
struct ByCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  static constexpr int kParts = kSplit ? 2 : 1;
  static constexpr int kDkSlots = kSplit ? 1 : 2;
  static constexpr int kWStages = kSplit ? 2 : 3;
  static constexpr int kProducers = 128;
  static constexpr int kXItems = (16 * (kTileH + 2 * kMaxHalo) + kProducers - 1) / kProducers;
  static constexpr int kThreads = 32 * (2 + 4 + 4);
  static constexpr int kOct = (3 * KS * KS + 7) / 8;
};

struct BySmem {
  uint32_t xr, dk, w, bars, total, xr_bytes, dk_bytes, w_bytes;
};

template <typename T, int KS>
__host__ __device__ inline BySmem by_smem_layout(int Cp, int R) {
  using Cfg = ByCfg<T, KS>;
  BySmem L;
  L.xr_bytes = (uint32_t)16 * (kTileH + 2 * R) * kHaloCols * 4;
  L.dk_bytes = (uint32_t)Cfg::kParts * kDkBytes;
  L.w_bytes = (uint32_t)Cfg::kParts * 128 * Cp * 2;
  L.xr = 0;
  L.dk = L.xr + 2 * L.xr_bytes;
  L.w = L.dk + Cfg::kDkSlots * L.dk_bytes;
  L.bars = L.w + Cfg::kWStages * L.w_bytes;
  L.total = L.bars + 8 * (4 + 2 * Cfg::kDkSlots + 2 * Cfg::kWStages + 4);
  return L;
}

struct ByParams {
  const void* x;
  const void* wpack;  // "by" image
  const void* gout;
  void* gy;
  int N, C, H, W, Cp, R;
  int d[3];
  int tiles_w, tiles_h, num_tiles;
  int* status;
};

template <typename T, int KS>
__global__ void __launch_bounds__(ByCfg<T, KS>::kThreads, 1)
gencat_bwd_y_kernel(const ByParams p) {
  using Cfg = ByCfg<T, KS>;
  using Op = typename IoTraits<T>::Op;
  constexpr int NS = Cfg::kDkSlots;
  constexpr int S = Cfg::kWStages;
  constexpr int NOCT = Cfg::kOct;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int C = p.C, Cp = p.Cp, H = p.H, W = p.W, R = p.R;
  const size_t P = (size_t)H * W;
  const BySmem L = by_smem_layout<T, KS>(Cp, R);
  const int ncg = Cp / 16;
  const int ngroups = ncg * NOCT;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* x_full = bars;             // [2]
  uint64_t* x_empty = bars + 2;        // [2]
  uint64_t* k_full = bars + 4;         // [NS]
  uint64_t* k_empty = k_full + NS;     // [NS]
  uint64_t* w_full = k_empty + NS;     // [S]
  uint64_t* w_empty = w_full + S;      // [S]
  uint64_t* d_full = w_empty + S;      // [2]
  uint64_t* d_empty = d_full + 2;      // [2]
  const int xr_rows = kTileH + 2 * R;
  const int xr_plane = xr_rows * kHaloCols;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 128);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&x_full[i], Cfg::kProducers);
      tc::mbar_init(&x_empty[i], 128);
      tc::mbar_init(&d_full[i], 1);
      tc::mbar_init(&d_empty[i], 128);
    }
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&k_full[i], 128);
      tc::mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&w_full[i], 1);
      tc::mbar_init(&w_empty[i], 1);
    }
    tc::fence_mbar_init();
    abort_s = 0;
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  volatile int* abort_flag = &abort_s;

  if (warp == 0) {
    // ---- transposed-weight groups through the ring -------------------------
    if (lane == 0) {
      const uint8_t* wsrc = static_cast<const uint8_t*>(p.wpack);
      uint32_t wq = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        for (int g = 0; g < ngroups; ++g, ++wq) {
          const int s = wq % S;
          if (!tc::mbar_wait(&w_empty[s], ((wq / S) & 1) ^ 1, abort_flag, kWaitNs)) {
            fail(abort_flag, p.status, 30);
            goto done;
          }
          tc::mbar_arrive_expect_tx(&w_full[s], L.w_bytes);
          tc::bulk_g2s(smem + L.w + s * L.w_bytes, wsrc + (size_t)g * L.w_bytes, L.w_bytes,
                       &w_full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA: D_y[tile] += dK . W^T, over all groups -----------------------
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(kTileM, Cp, IoTraits<T>::kBf16, false, false);
      const uint32_t b_lbo = Cp * 16;
      const uint64_t b_step = (2 * b_lbo) >> 4;      // descriptor advance per K step
      const uint64_t b_lo = (128 * Cp * 2) >> 4;     // hi -> lo part of a weight group
      uint32_t wq = 0, kq = 0, it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        const int tb = it & 1;
        if (!tc::mbar_wait(&d_empty[tb], ((it >> 1) & 1) ^ 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 31);
          goto done;
        }
        tc::tc_fence_after();
        const uint32_t dt = tmem_base + tb * Cp;
        for (int g = 0; g < ngroups; ++g, ++wq, ++kq) {
          const int s = wq % S, ks_ = kq % NS;
          if (!tc::mbar_wait(&k_full[ks_], (kq / NS) & 1, abort_flag, kWaitNs) ||
              !tc::mbar_wait(&w_full[s], (wq / S) & 1, abort_flag, kWaitNs)) {
            fail(abort_flag, p.status, 32);
            goto done;
          }
          tc::tc_fence_after();
          // A: dK, K-major (rows are K): row-group stride 128, pixel-group stride 2048
          const uint64_t ad =
              tc::smem_desc(tc::smem_u32(smem + L.dk + ks_ * L.dk_bytes), 128, 2048);
          const uint64_t bd = tc::smem_desc(tc::smem_u32(smem + L.w + s * L.w_bytes), b_lbo, 128);
          const uint32_t acc0 = g > 0 ? 1u : 0u;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t a_k = ad + ks * (256 >> 4);
            const uint64_t b_k = bd + ks * b_step;
            tc::mma_f16(dt, a_k, b_k, idesc, ks > 0 ? 1u : acc0);
            if constexpr (Cfg::kSplit) {
              tc::mma_f16(dt, a_k + (kDkBytes >> 4), b_k, idesc, 1u);
              tc::mma_f16(dt, a_k, b_k + b_lo, idesc, 1u);
            }
          }
          tc::mma_commit(&k_empty[ks_]);
          tc::mma_commit(&w_empty[s]);
        }
        tc::mma_commit(&d_full[tb]);
      }
    }
  } else if (warp < 6) {
    // ---- x-halo producers (per tile and 16-channel group) ------------------
    const int pt = threadIdx.x - 64;
    const XPlan<Cfg::kXItems> plan = make_xplan<Cfg::kXItems>(xr_rows, pt, Cfg::kProducers);
    uint32_t xq = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      for (int cg = 0; cg < ncg; ++cg, ++xq) {
        const int xb = xq & 1;
        if (!warp_wait(&x_empty[xb], ((xq >> 1) & 1) ^ 1, abort_flag)) {
          fail(abort_flag, p.status, 33);
          break;
        }
        float4* xr = reinterpret_cast<float4*>(smem + L.xr + xb * L.xr_bytes);
        stage_halo<T, Cfg::kXItems>(plan, static_cast<const T*>(p.x), xr, n, C, H, W, cg * 16,
                                    h0 - R, w0 - 8, xr_rows);
        tc::mbar_arrive(&x_full[xb]);
      }
    }
  } else {
    // ---- builders (thread = pixel = TMEM lane) + D_y drain ----------------
    const int quad = warp & 3;
    const int m = quad * 32 + lane;
    const int mr = m >> 4, mc = m & 15;
    const T* gout = static_cast<const T*>(p.gout);
    T* gy = static_cast<T*>(p.gy);
    const int dil[3] = {p.d[0], p.d[1], p.d[2]};
    uint32_t xq = 0, kq = 0, it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      const int h = h0 + mr, w = w0 + mc;
      const bool px_ok = (h < H) && (w < W);
      const size_t pix = px_ok ? (size_t)h * W + w : 0;
      const T* gn = gout + (size_t)n * 4 * C * P;
      bool failed = false;
      for (int cg = 0; cg < ncg && !failed; ++cg, ++xq) {
        unsigned long long gv[3][16 / 2];
        load_gv<T>(gv, gn, C, P, cg, pix, px_ok);
        const int xb = xq & 1;
        if (!warp_wait(&x_full[xb], (xq >> 1) & 1, abort_flag)) {
          fail(abort_flag, p.status, 34);
          failed = true;
          break;
        }
        const float4* xc = reinterpret_cast<const float4*>(smem + L.xr + xb * L.xr_bytes) +
                           (mr + R) * kHaloCols + (mc + 8);
        for (int oct = 0; oct < NOCT; ++oct, ++kq) {
          const int ks_ = kq % NS;
          if (!warp_wait(&k_empty[ks_], ((kq / NS) & 1) ^ 1, abort_flag)) {
            fail(abort_flag, p.status, 35);
            failed = true;
            break;
          }
          build_dk<T, Op, Cfg::kSplit, KS>(smem + L.dk + ks_ * L.dk_bytes, oct, xc, xr_plane, gv,
                                           dil, m);
          tc::fence_proxy_async_smem();
          tc::mbar_arrive(&k_full[ks_]);
        }
        tc::mbar_arrive(&x_empty[xb]);
      }
      if (failed) break;
      // drain D_y of this tile
      const int tb = it & 1;
      if (!warp_wait(&d_full[tb], (it >> 1) & 1, abort_flag)) {
        fail(abort_flag, p.status, 36);
        break;
      }
      tc::tc_fence_after();
      for (int i0 = 0; i0 < Cp; i0 += 16) {
        float dv[16];
        tc::tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + tb * Cp + i0, dv);
        tc::tmem_ld_wait();
        if (px_ok) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int i = i0 + k;
            if (i < C) gy[((size_t)n * C + i) * P + pix] = from_f32<T>(dv[k]);
          }
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&d_empty[tb]);
    }
  }
done:
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 128);
  }
}

// =============================================================== dW =========
template <typename T, int KS>
struct BwCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  static constexpr int kParts = kSplit ? 2 : 1;
  static constexpr int kDkSlots = kSplit ? 1 : 2;
  static constexpr int kYBufs = kSplit ? 1 : 2;
  static constexpr int kProducers = 128;
  static constexpr int kXItems = (16 * (kTileH + 2 * kMaxHalo) + kProducers - 1) / kProducers;
  static constexpr int kYItems = (16 * 80 + kProducers - 1) / kProducers;
  static constexpr int kThreads = 32 * (2 + 4 + 4 + 4);
  static constexpr int kOct = (3 * KS * KS + 7) / 8;
};

struct BwSmem {
  uint32_t xr, y, dk, bars, total, xr_bytes, y_bytes, dk_bytes;
};

template <typename T, int KS>
__host__ __device__ inline BwSmem bw_smem_layout(int Nw, int R) {
  using Cfg = BwCfg<T, KS>;
  BwSmem L;
  L.xr_bytes = (uint32_t)16 * (kTileH + 2 * R) * kHaloCols * 4;
  L.y_bytes = (uint32_t)Cfg::kParts * kTileM * Nw * 2;
  L.dk_bytes = (uint32_t)Cfg::kParts * kDkBytes;
  L.xr = 0;
  L.y = L.xr + 2 * L.xr_bytes;
  L.dk = L.y + Cfg::kYBufs * L.y_bytes;
  L.bars = L.dk + Cfg::kDkSlots * L.dk_bytes;
  L.total = L.bars + 8 * (8 + 2 * Cfg::kDkSlots + 1);
  return L;
}

struct BwParams {
  const void* x;
  const void* y;
  const void* gout;
  float* partial;  // [splits][NG][128][Nw]
  int N, C, H, W, Cp, Nw, R;
  int d[3];
  int tiles_w, tiles_h, num_tiles;
  int ngroups, gb;    // groups; groups per batch
  int splits;
  int* status;
};

template <typename T, int KS>
__global__ void __launch_bounds__(BwCfg<T, KS>::kThreads, 1)
gencat_bwd_w_kernel(const BwParams p) {
  using Cfg = BwCfg<T, KS>;
  using Op = typename IoTraits<T>::Op;
  constexpr int NS = Cfg::kDkSlots;
  constexpr int NY = Cfg::kYBufs;
  constexpr int NOCT = Cfg::kOct;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int C = p.C, H = p.H, W = p.W, R = p.R, Nw = p.Nw;
  const size_t P = (size_t)H * W;
  const BwSmem L = bw_smem_layout<T, KS>(Nw, R);
  const int batch = blockIdx.x % ((p.ngroups + p.gb - 1) / p.gb);
  const int split = blockIdx.x / ((p.ngroups + p.gb - 1) / p.gb);
  const int g0 = batch * p.gb;
  const int g1 = min(p.ngroups, g0 + p.gb);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* x_full = bars;          // [2]
  uint64_t* x_empty = bars + 2;     // [2]
  uint64_t* y_full = bars + 4;      // [2]
  uint64_t* y_empty = bars + 6;     // [2]
  uint64_t* k_full = bars + 8;      // [NS]
  uint64_t* k_empty = k_full + NS;  // [NS]
  uint64_t* d_full = k_empty + NS;  // [1]
  const int xr_rows = kTileH + 2 * R;
  const int xr_plane = xr_rows * kHaloCols;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&x_full[i], Cfg::kProducers);
      tc::mbar_init(&x_empty[i], 128);
      tc::mbar_init(&y_full[i], Cfg::kProducers);
      tc::mbar_init(&y_empty[i], 1);
    }
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&k_full[i], 128);
      tc::mbar_init(&k_empty[i], 1);
    }
    tc::mbar_init(d_full, 1);
    tc::fence_mbar_init();
    abort_s = 0;
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  volatile int* abort_flag = &abort_s;

  if (warp == 0) {
    // idle after TMEM allocation
  } else if (warp == 1) {
    // ---- MMA: D_w[g] += dK^T . y_tile, over the split's tiles --------------
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(kTileM, Nw, IoTraits<T>::kBf16, true, false);
      const uint32_t b_lbo = Nw * 16;          // pixel-group stride of the y tile
      const uint64_t b_step = (2 * b_lbo) >> 4;  // descriptor advance per K step
      const uint64_t y_lo = (kTileM * Nw * 2) >> 4;  // hi -> lo part of the y tile
      uint32_t kq = 0, it = 0;
      bool first = true;
      for (int tile = split; tile < p.num_tiles; tile += p.splits, ++it) {
        const int yb = it % NY;
        if (!tc::mbar_wait(&y_full[yb], (it / NY) & 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 40);
          goto done;
        }
        tc::tc_fence_after();
        const uint64_t yd = tc::smem_desc(tc::smem_u32(smem + L.y + yb * L.y_bytes), b_lbo, 128);
        for (int g = g0; g < g1; ++g, ++kq) {
          const int ks_ = kq % NS;
          if (!tc::mbar_wait(&k_full[ks_], (kq / NS) & 1, abort_flag, kWaitNs)) {
            fail(abort_flag, p.status, 41);
            goto done;
          }
          tc::tc_fence_after();
          // A: dK, MN-major (rows are M, pixels are K): K-group stride 2048, M-group 128
          const uint64_t ad =
              tc::smem_desc(tc::smem_u32(smem + L.dk + ks_ * L.dk_bytes), 2048, 128);
          const uint32_t dt = tmem_base + (g - g0) * Nw;
          const uint32_t acc0 = first ? 0u : 1u;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t a_k = ad + ks * ((2 * 2048) >> 4);
            const uint64_t b_k = yd + ks * b_step;
            tc::mma_f16(dt, a_k, b_k, idesc, ks > 0 ? 1u : acc0);
            if constexpr (Cfg::kSplit) {
              tc::mma_f16(dt, a_k + (kDkBytes >> 4), b_k, idesc, 1u);
              tc::mma_f16(dt, a_k, b_k + y_lo, idesc, 1u);
            }
          }
          tc::mma_commit(&k_empty[ks_]);
        }
        tc::mma_commit(&y_empty[yb]);
        first = false;
      }
      tc::mma_commit(d_full);
    }
  } else if (warp < 6) {
    // ---- x-halo producers ----------------------------------------------------
    const int pt = threadIdx.x - 64;
    const XPlan<Cfg::kXItems> plan = make_xplan<Cfg::kXItems>(xr_rows, pt, Cfg::kProducers);
    uint32_t xq = 0;
    for (int tile = split; tile < p.num_tiles && !*abort_flag; tile += p.splits) {
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      int cur = -1;
      for (int g = g0; g < g1; ++g) {
        const int cg = g / NOCT;
        if (cg == cur) continue;
        cur = cg;
        const int xb = xq & 1;
        if (!warp_wait(&x_empty[xb], ((xq >> 1) & 1) ^ 1, abort_flag)) {
          fail(abort_flag, p.status, 42);
          break;
        }
        float4* xr = reinterpret_cast<float4*>(smem + L.xr + xb * L.xr_bytes);
        stage_halo<T, Cfg::kXItems>(plan, static_cast<const T*>(p.x), xr, n, C, H, W, cg * 16,
                                    h0 - R, w0 - 8, xr_rows);
        tc::mbar_arrive(&x_full[xb]);
        ++xq;
      }
    }
  } else if (warp < 10) {
    // ---- y-tile producers (B operand, ones channel at C for db) -----------
    const int pt = threadIdx.x - 192;
    const YPlan<Cfg::kYItems> plan = make_yplan<Cfg::kYItems>(Nw, pt, Cfg::kProducers);
    uint32_t it = 0;
    for (int tile = split; tile < p.num_tiles; tile += p.splits, ++it) {
      const int yb = it % NY;
      if (!warp_wait(&y_empty[yb], ((it / NY) & 1) ^ 1, abort_flag)) {
        fail(abort_flag, p.status, 43);
        break;
      }
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      uint8_t* ys = smem + L.y + yb * L.y_bytes;
      stage_y_mn<T, Op, Cfg::kSplit, Cfg::kYItems>(plan, static_cast<const T*>(p.y), ys,
                                                   ys + kTileM * Nw * 2, n, C, Nw, C, H, W, h0,
                                                   w0);
      tc::fence_proxy_async_smem();
      tc::mbar_arrive(&y_full[yb]);
    }
  } else {
    // ---- builders (thread = pixel) then the D_w drain (thread = row) -------
    const int quad = warp & 3;
    const int m = quad * 32 + lane;
    const int mr = m >> 4, mc = m & 15;
    const T* gout = static_cast<const T*>(p.gout);
    const int dil[3] = {p.d[0], p.d[1], p.d[2]};
    uint32_t xq = 0, kq = 0;
    bool failed = false;
    for (int tile = split; tile < p.num_tiles && !failed; tile += p.splits) {
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      const int h = h0 + mr, w = w0 + mc;
      const bool px_ok = (h < H) && (w < W);
      const size_t pix = px_ok ? (size_t)h * W + w : 0;
      const T* gn = gout + (size_t)n * 4 * C * P;
      int cur = -1;
      unsigned long long gv[3][16 / 2];
      const float4* xc = nullptr;
      int xb = 0;
      for (int g = g0; g < g1; ++g, ++kq) {
        const int cg = g / NOCT;
        if (cg != cur) {
          if (cur >= 0) {
            tc::mbar_arrive(&x_empty[xb]);
            ++xq;
          }
          cur = cg;
          load_gv<T>(gv, gn, C, P, cg, pix, px_ok);
          xb = xq & 1;
          if (!warp_wait(&x_full[xb], (xq >> 1) & 1, abort_flag)) {
            fail(abort_flag, p.status, 44);
            failed = true;
            break;
          }
          xc = reinterpret_cast<const float4*>(smem + L.xr + xb * L.xr_bytes) +
               (mr + R) * kHaloCols + (mc + 8);
        }
        const int ks_ = kq % NS;
        if (!warp_wait(&k_empty[ks_], ((kq / NS) & 1) ^ 1, abort_flag)) {
          fail(abort_flag, p.status, 45);
          failed = true;
          break;
        }
        build_dk<T, Op, Cfg::kSplit, KS>(smem + L.dk + ks_ * L.dk_bytes, g % NOCT, xc, xr_plane,
                                         gv, dil, m);
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&k_full[ks_]);
      }
      if (!failed && cur >= 0) {
        tc::mbar_arrive(&x_empty[xb]);
        ++xq;
      }
    }
    // drain: lane = weight row of the group, columns = Nw
    if (!failed && warp_wait(d_full, 0, abort_flag)) {
      tc::tc_fence_after();
      for (int g = g0; g < g1; ++g) {
        float* dst = p.partial + (((size_t)split * p.ngroups + g) * 128 + m) * Nw;
        for (int c0 = 0; c0 < Nw; c0 += 16) {
          float dv[16];
          tc::tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + (g - g0) * Nw + c0, dv);
          tc::tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 16; k += 4)
            *reinterpret_cast<float4*>(dst + c0 + k) =
                make_float4(dv[k], dv[k + 1], dv[k + 2], dv[k + 3]);
        }
      }
    } else if (!failed) {
      fail(abort_flag, p.status, 46);
    }
  }
done:
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 512);
  }
}

// Sum the split partials into the Conv2d layout: gw[(b*C + c)*K^2 + tap, i],
// gb[(b*C + c)*K^2 + tap] (column C of the partials is the bias gradient).
template <typename T>
__global__ void gencat_wreduce_kernel(const float* __restrict__ partial, T* __restrict__ gw,
                                      T* __restrict__ gb, int C, int KS, int ngroups, int Nw,
                                      int splits) {
  const int KK = KS * KS;
  const int noct = (3 * KK + 7) / 8;
  const long long total = (long long)ngroups * 128 * (C + 1);
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(idx % (C + 1));
    const int row = (int)((idx / (C + 1)) % 128);
    const int g = (int)(idx / ((long long)(C + 1) * 128));
    const int slot = (g % noct) * 8 + row / 16;
    const int c = (g / noct) * 16 + row % 16;
    if (slot >= 3 * KK || c >= C) continue;
    float acc = 0.f;
    const float* src = partial + ((size_t)g * 128 + row) * Nw + i;
    for (int s = 0; s < splits; ++s) acc += src[(size_t)s * ngroups * 128 * Nw];
    const int b = slot / KK, tap = slot % KK;
    const long long mrow = (long long)(b * C + c) * KK + tap;
    if (i < C) gw[mrow * C + i] = from_f32<T>(acc);
    else gb[mrow] = from_f32<T>(acc);
  }
}

// ========================================================== dY + dW ==========
// One pass builds every dK tile once and feeds both GEMMs (the separate dY and
// dW kernels above each build all of dK). CTA = (16-channel group cg, spatial
// split; at K = 5 also an octet set: the cg's 10 octets in sets of <= 4): D_w
// of the CTA's octets (<= 4 x Nw TMEM columns) accumulates over the split's
// tiles; per tile, D_y (128 pixels x Cp, double buffered at columns
// 384 / 448) holds the cg's share of dY and is added into an FP32 dY
// accumulator with reductions to global memory (the other channel groups'
// CTAs add theirs); the x-halo producer warps do that drain for the previous
// tile while the builders work on the next (with staged operands the
// y-tile producer warps do it, so that the x-halo copies never wait behind a
// drain). Builders run two threads per pixel (four slots each); one issuer
// warp per GEMM. With staged operands
// (gencat_stage.cu) one thread per producer group issues one TMA copy per tile
// instead: the x halo from the FP32 cell plane (box 32 px x halo rows x 4
// channel quads, zero filled outside the image) and the y tile from the y
// plane (box 16 px x 8 rows x all channel groups), which makes the dW GEMM's B
// operand MN-major ([channel group][pixel][8 channels]). With kGTma (16-bit,
// staged) the gradient values of the cg's 16 channels x 3 branches also come
// by one TMA copy per tile, one tile ahead, into a single buffer the builders
// release as soon as they hold the values in registers; otherwise each builder
// loads its pixel's 48 values from global memory at the start of the tile.
//
// FP32 with kLoRing: the dK hi part is double buffered and the lo part single
// buffered; both issuers run an octet's MMAs with the lo operand first and
// release the lo buffer then, so the next octet's build starts after a third
// of the current octet's MMAs instead of after all of them (with one 64 KB
// slot, build and MMAs alternated). The weight ring holds one part (16 KB)
// per stage, 3 stages, to pay for the extra 32 KB.
template <typename T, int KS, bool kStaged = false, bool kGTmaArg = false,
          bool kLoRingArg = false>
struct DywCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  static constexpr bool kGTma = kGTmaArg;
  static constexpr bool kLoRing = kLoRingArg;
  static_assert(!kLoRing || kSplit, "the lo ring is for the FP32 split operands");
  static constexpr int kParts = kSplit ? 2 : 1;
  // dK stages between builders and MMAs (lo ring: the hi slots); staged 16-bit
  // data at K <= 3 has the room for a third beside its 16-bit x halos
  static constexpr int kDkSlots = kSplit ? (kLoRing ? 2 : 1) : ((kStaged && KS <= 3) ? 3 : 2);
  static constexpr int kXBufs = kSplit ? 1 : 2;  // at most; DywParams::nx is the count used
  static constexpr int kYBufs = kSplit ? 1 : 2;
  static constexpr int kWStages = kLoRing ? 3 : 2;
  static constexpr int kProducers = 128;
  static constexpr int kXItems = (16 * (kTileH + 2 * kMaxHalo) + kProducers - 1) / kProducers;
  static constexpr int kYItems = (16 * 80 + kProducers - 1) / kProducers;
  static constexpr int kOct = (3 * KS * KS + 7) / 8;
  static constexpr int kFirstXWarp = 3, kFirstYWarp = 7, kFirstBuilderWarp = 11;
  static constexpr int kThreads = 32 * (kFirstBuilderWarp + 8);
  static constexpr uint32_t kDyCol = 384;
  // x halo cells: staged 16-bit data as 8-channel cells in the I/O type (kXIo:
  // one packed multiply per dK pair), otherwise FP32 cells of 4 channels
  static constexpr bool kXIo = kStaged && !kSplit;
  static constexpr int kXCells = kXIo ? 2 : 4;  // cells per pixel (16 channels)
};

struct DywSmem {
  uint32_t xr, y, dk, w, g, dyb, bars, total, xr_bytes, y_bytes, dk_bytes, w_bytes, g_bytes;
};

// x halo of the dY+dW kernel: `dyw_halo_cols` cells per row starting
// `dyw_halo_off` columns left of the tile: 32 from w0 - 8 for K <= 3 (halos up
// to 8); for K = 5 exactly the 16 + 2R columns its halo R needs (16-bit cells:
// two x buffers up to R = 11, one up to R = 16).
__host__ __device__ inline int dyw_halo_cols(int ks, int R) {
  return ks <= 3 ? kHaloCols : 16 + 2 * R;
}
__host__ __device__ inline int dyw_halo_off(int ks, int R) { return ks <= 3 ? 8 : R; }
// K = 5: a channel group's 10 octets of slots do not fit as D_w accumulators
// (80 columns each) beside D_y in TMEM, so CTAs take sets of at most 4.
constexpr int kDywSetOct = 4;

// Every wait of the merged dY + dW kernel lets a waiting thread stay suspended
// (not issuing) for up to this long, woken by the phase's completion.
constexpr uint32_t kHintNs = 100000;

// D_y drain buffers: one per TMEM lane quadrant (the drain warp's 32 pixels =
// 2 rows x 16 columns), 8 channels at a time: [8 ch][2 rows][16 px] FP32.
constexpr uint32_t kDyChunkBytes = 8 * 2 * 16 * 4;

// `nx` x-halo buffers (2, or 1 where two do not fit), then y, dK, weight ring,
// (kGTma) the gradient tile [branch][channel][8 rows][16 px] and the four
// D_y drain buffers (4 KB).
// C=64, K=3, halo 5: fp32 36 + 40 + 64 + 2x32 + 4 KB = 208 KB;
// bf16 2x36 + 2x20 + 2x32 + 2x16 (+ 12) + 4 KB = 212 (224) KB; staged bf16
// (16-bit x cells, three dK stages) 2x18 + 2x20 + 3x32 + 2x16 (+ 12) + 4 KB =
// 208 (220) KB.
template <typename T, int KS, bool kGTma = false, bool kLoRing = false, bool kStaged = false>
__host__ __device__ inline DywSmem dyw_smem_layout(int Cp, int Nw, int R, int nx) {
  using Cfg = DywCfg<T, KS, kStaged, kGTma, kLoRing>;
  DywSmem L;
  L.xr_bytes = (uint32_t)Cfg::kXCells * (kTileH + 2 * R) * dyw_halo_cols(KS, R) * 16;
  L.y_bytes = (uint32_t)Cfg::kParts * kTileM * Nw * 2;
  // lo ring: dk_bytes / w_bytes are one part; the lo buffer follows the hi slots
  L.dk_bytes = (uint32_t)(kLoRing ? 1 : Cfg::kParts) * kDkBytes;
  L.w_bytes = (uint32_t)(kLoRing ? 1 : Cfg::kParts) * 128 * Cp * 2;
  L.g_bytes = kGTma ? (uint32_t)(3 * 16 * kTileM * sizeof(T)) : 0u;
  L.xr = 0;
  L.y = L.xr + nx * L.xr_bytes;
  L.dk = L.y + Cfg::kYBufs * L.y_bytes;
  L.w = L.dk + (Cfg::kDkSlots + (kLoRing ? 1 : 0)) * L.dk_bytes;
  L.g = L.w + Cfg::kWStages * L.w_bytes;
  L.dyb = L.g + L.g_bytes;
  L.bars = L.dyb + 4 * kDyChunkBytes;
  L.total = L.bars + 8 * (4 + 2 * Cfg::kYBufs + 2 * Cfg::kDkSlots + 2 * Cfg::kWStages + 9);
  return L;
}

struct DywParams {
  const void* x;
  const void* y;
  const void* wpack;  // "by" image
  const void* gout;
  float* gy_acc;      // FP32 dY accumulator, zeroed before the launch
  float* partial;     // [splits][NG][128][Nw]
  int N, C, H, W, Cp, Nw, R;
  int d[3];
  int tiles_w, tiles_h, num_tiles;
  int ngroups, ncg, splits;
  int nsets;          // octet sets per channel group (K = 5: 3 sets of <= 4 octets)
  int nx;             // x-halo buffers (1 or 2)
  // grad_out channel-last [N][H][W][4C] (kGTma only): gmap {C, 4, W, H, N}, box
  // {16, 3, 16, 8, 1}, landing as [8 rows][16 px][3 branches][16 channels]
  int g_nhwc;
  int* status;
};

// Tensor maps of the staged operands (a separate grid-constant parameter so the
// non-staged kernel's parameter block keeps its register allocation).
struct DywMaps {
  CUtensorMap xmap;  // staged x plane (64-bit view) {W*2, H, Cq, N}, box {64, 8+2R, 4, 1}
  CUtensorMap ymap;  // staged y plane (64-bit view) {Wp*2, Hp, G, parts*N}, box {32, 8, G, 1}
  CUtensorMap gmap;  // grad_out {W, H, C, 4, N}, box {16, 8, 16, 3, 1} (kGTma only)
  CUtensorMap dymap; // FP32 dY accumulator {W, H, C, N}, box {16, 2, 8, 1} (dy_tma)
  int ph, pw;        // y-plane row / column offsets
  int dy_tma;        // dymap is valid: D_y drains by TMA reductions, not atomics
};

// D_y of the it-th tile of a split (64 columns at `dy_col`, double buffered)
// into the FP32 dY accumulator: the calling warp reads TMEM lane quadrant
// `quad`, thread = pixel m of the tile. With a dY tensor map, eight channels at
// a time go through the warp's 1 KB buffer `buf` and one TMA reduction
// (cp.reduce.async.bulk.tensor .add, [8 ch][2 rows][16 px]) per chunk, issued
// by lane 0 after it has waited until the previous one read its source; the
// 64 scalar atomics per thread this replaces cost ~19 % of the bf16 kernel
// time at B=8. False when the bounded wait gives up.
__device__ __forceinline__ bool drain_dy(const DywParams& p, const DywMaps& maps, uint32_t it,
                                         int split, int quad, int lane, uint32_t tmem_base,
                                         uint32_t dy_col, uint64_t* d_full, uint64_t* d_empty,
                                         volatile int* abort_flag, float* buf) {
  const int tb = it & 1;
  if (!warp_wait(&d_full[tb], (it >> 1) & 1, abort_flag, kHintNs)) return false;
  tc::tc_fence_after();
  float dv[4][16];
  const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + dy_col + tb * 64;
#pragma unroll
  for (int q = 0; q < 4; ++q) tc::tmem_ld16(taddr + q * 16, dv[q]);
  tc::tmem_ld_wait();
  tc::tc_fence_before();
  tc::mbar_arrive(&d_empty[tb]);
  int n, h0, w0;
  tile_origin(split + (int)it * p.splits, p.tiles_w, p.tiles_h, n, h0, w0);
  if (maps.dy_tma) {
    // rows h0 + 2 quad, +1 (boxes reaching past H or W are clipped by the
    // TMA unit; a box starting past them is not issued)
    const int hq = h0 + 2 * quad;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (hq >= p.H || q * 8 >= p.C) break;  // warp-uniform
      if (lane == 0) tc::bulk_wait_read_all();
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 8; ++c) buf[c * 32 + lane] = dv[(q * 8 + c) >> 4][(q * 8 + c) & 15];
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tc::tma_reduce_add_4d(&maps.dymap, buf, w0, hq, q * 8, n);
        tc::bulk_commit();
      }
    }
    return true;
  }
  const int m = quad * 32 + lane;
  const int h = h0 + (m >> 4), w = w0 + (m & 15);
  if (h < p.H && w < p.W) {
    const size_t P = (size_t)p.H * p.W;
    float* acc = p.gy_acc + (size_t)n * p.C * P + (size_t)h * p.W + w;
#pragma unroll
    for (int k = 0; k < 64; ++k)
      if (k < p.C) atomicAdd(acc + (size_t)k * P, dv[k >> 4][k & 15]);
  }
  return true;
}

template <typename T, int KS, bool kStaged, bool kGTma, bool kLoRing>
__global__ void __launch_bounds__(DywCfg<T, KS, kStaged, kGTma, kLoRing>::kThreads, 1)
gencat_bwd_dyw_kernel(const DywParams p, const __grid_constant__ DywMaps maps) {
  using Cfg = DywCfg<T, KS, kStaged, kGTma, kLoRing>;
  using Op = typename IoTraits<T>::Op;
  constexpr int NS = Cfg::kDkSlots;
  const int NX = Cfg::kXBufs == 1 ? 1 : p.nx;  // 1 or 2: index = xq & (NX-1), lap = xq >> (NX-1)
  const int nx_sh = NX - 1;
  constexpr int NY = Cfg::kYBufs;
  constexpr int S = Cfg::kWStages;
  constexpr int NOCT = Cfg::kOct;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int C = p.C, Cp = p.Cp, H = p.H, W = p.W, R = p.R, Nw = p.Nw;
  const size_t P = (size_t)H * W;
  const DywSmem L = dyw_smem_layout<T, KS, kGTma, kLoRing, kStaged>(Cp, Nw, R, NX);
  const int cg = blockIdx.x % p.ncg;
  const int oset = (blockIdx.x / p.ncg) % p.nsets;
  const int split = blockIdx.x / (p.ncg * p.nsets);
  // this CTA's octets of the channel group (all of them for K <= 3)
  const int oct0 = p.nsets == 1 ? 0 : oset * kDywSetOct;
  const int oct1 = p.nsets == 1 ? NOCT : min(oct0 + kDywSetOct, NOCT);
  const int xcols = dyw_halo_cols(KS, R), xoff = dyw_halo_off(KS, R);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* x_full = bars;             // [2] (NX used)
  uint64_t* x_empty = x_full + 2;      // [2]
  uint64_t* y_full = x_empty + 2;      // [NY]
  uint64_t* y_empty = y_full + NY;     // [NY]
  uint64_t* k_full = y_empty + NY;     // [NS]
  uint64_t* k_empty = k_full + NS;     // [NS]
  uint64_t* w_full = k_empty + NS;     // [S]
  uint64_t* w_empty = w_full + S;      // [S]
  uint64_t* d_full = w_empty + S;      // [2]
  uint64_t* d_empty = d_full + 2;      // [2]
  uint64_t* w_done = d_empty + 2;      // [1]
  uint64_t* g_full = w_done + 1;       // [1] (kGTma)
  uint64_t* g_empty = g_full + 1;      // [1] (kGTma)
  uint64_t* lo_full = g_empty + 1;     // [1] (kLoRing: the lo buffer)
  uint64_t* lo_empty = lo_full + 1;    // [1]
  const int xr_rows = kTileH + 2 * R;
  const int xr_plane = xr_rows * xcols;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&x_full[i], Cfg::kProducers);
      tc::mbar_init(&x_empty[i], 256);
    }
    for (int i = 0; i < NY; ++i) {
      tc::mbar_init(&y_full[i], Cfg::kProducers);
      tc::mbar_init(&y_empty[i], 1);
    }
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&k_full[i], 256);
      tc::mbar_init(&k_empty[i], 2);
    }
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&w_full[i], 1);
      tc::mbar_init(&w_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&d_full[i], 1);
      tc::mbar_init(&d_empty[i], Cfg::kProducers);
    }
    tc::mbar_init(w_done, 1);
    tc::mbar_init(g_full, 1);
    tc::mbar_init(g_empty, 256);
    tc::mbar_init(lo_full, 256);
    tc::mbar_init(lo_empty, 2);
    tc::fence_mbar_init();
    abort_s = 0;
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  volatile int* abort_flag = &abort_s;

  if (warp == 0) {
    // ---- the cg's transposed-weight groups, once per tile ---------------------
    if (lane == 0) {
      const uint8_t* wsrc = static_cast<const uint8_t*>(p.wpack);
      uint32_t wq = 0;
      // a group's image is both parts back to back; the lo ring streams them
      // as separate stages (hi, then lo)
      constexpr int kLoads = kLoRing ? 2 : 1;
      const size_t w_group = (size_t)Cfg::kParts * 128 * Cp * 2;
      for (int tile = split; tile < p.num_tiles; tile += p.splits) {
        for (int oct = oct0; oct < oct1; ++oct) {
          for (int part = 0; part < kLoads; ++part, ++wq) {
            const int s = wq % S;
            if (!tc::mbar_wait(&w_empty[s], ((wq / S) & 1) ^ 1, abort_flag, kWaitNs, kHintNs)) {
              fail(abort_flag, p.status, 50);
              goto done;
            }
            tc::mbar_arrive_expect_tx(&w_full[s], L.w_bytes);
            tc::bulk_g2s(smem + L.w + s * L.w_bytes,
                         wsrc + (size_t)(cg * NOCT + oct) * w_group + (size_t)part * L.w_bytes,
                         L.w_bytes, &w_full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---- dY issuer: D_y[tile] = sum over the cg's octets of dK . W -----------
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(kTileM, Cp, IoTraits<T>::kBf16, false, false);
      const uint32_t b_lbo = Cp * 16;
      const uint64_t b_step = (2 * b_lbo) >> 4;
      const uint64_t b_lo = (128 * Cp * 2) >> 4;
      uint32_t wq = 0, kq = 0, it = 0;
      for (int tile = split; tile < p.num_tiles; tile += p.splits, ++it) {
        const int tb = it & 1;
        if (!tc::mbar_wait(&d_empty[tb], ((it >> 1) & 1) ^ 1, abort_flag, kWaitNs, kHintNs)) {
          fail(abort_flag, p.status, 51);
          goto done;
        }
        tc::tc_fence_after();
        const uint32_t dt = tmem_base + Cfg::kDyCol + tb * 64;
        if constexpr (kLoRing) {
          // per octet: lo * W_hi, release lo; hi * W_hi; hi * W_lo
          const uint64_t lo_d =
              tc::smem_desc(tc::smem_u32(smem + L.dk + 2 * kDkBytes), 128, 2048);
          for (int oct = oct0; oct < oct1; ++oct, ++kq) {
            const int hb = kq & 1;
            const int s_hi = wq % S;
            if (!tc::mbar_wait(&k_full[hb], (kq >> 1) & 1, abort_flag, kWaitNs, kHintNs) ||
                !tc::mbar_wait(lo_full, kq & 1, abort_flag, kWaitNs, kHintNs) ||
                !tc::mbar_wait(&w_full[s_hi], (wq / S) & 1, abort_flag, kWaitNs, kHintNs)) {
              fail(abort_flag, p.status, 52);
              goto done;
            }
            tc::tc_fence_after();
            const uint64_t hi_d =
                tc::smem_desc(tc::smem_u32(smem + L.dk + hb * kDkBytes), 128, 2048);
            const uint64_t bh = tc::smem_desc(tc::smem_u32(smem + L.w + s_hi * L.w_bytes), b_lbo, 128);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              tc::mma_f16(dt, lo_d + ks * (256 >> 4), bh + ks * b_step, idesc,
                          (oct > oct0 || ks > 0) ? 1u : 0u);
            tc::mma_commit(lo_empty);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              tc::mma_f16(dt, hi_d + ks * (256 >> 4), bh + ks * b_step, idesc, 1u);
            tc::mma_commit(&w_empty[s_hi]);
            ++wq;
            const int s_lo = wq % S;
            if (!tc::mbar_wait(&w_full[s_lo], (wq / S) & 1, abort_flag, kWaitNs, kHintNs)) {
              fail(abort_flag, p.status, 52);
              goto done;
            }
            tc::tc_fence_after();
            const uint64_t bl = tc::smem_desc(tc::smem_u32(smem + L.w + s_lo * L.w_bytes), b_lbo, 128);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              tc::mma_f16(dt, hi_d + ks * (256 >> 4), bl + ks * b_step, idesc, 1u);
            tc::mma_commit(&w_empty[s_lo]);
            ++wq;
            tc::mma_commit(&k_empty[hb]);
          }
          tc::mma_commit(&d_full[tb]);
          continue;
        }
        for (int oct = oct0; oct < oct1; ++oct, ++wq, ++kq) {
          const int s = wq % S, ks_ = kq % NS;
          if (!tc::mbar_wait(&k_full[ks_], (kq / NS) & 1, abort_flag, kWaitNs, kHintNs) ||
              !tc::mbar_wait(&w_full[s], (wq / S) & 1, abort_flag, kWaitNs, kHintNs)) {
            fail(abort_flag, p.status, 52);
            goto done;
          }
          tc::tc_fence_after();
          // A: dK, K-major (rows are K): row-group stride 128, pixel-group stride 2048
          const uint64_t ad =
              tc::smem_desc(tc::smem_u32(smem + L.dk + ks_ * L.dk_bytes), 128, 2048);
          const uint64_t bd = tc::smem_desc(tc::smem_u32(smem + L.w + s * L.w_bytes), b_lbo, 128);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t a_k = ad + ks * (256 >> 4);
            const uint64_t b_k = bd + ks * b_step;
            tc::mma_f16(dt, a_k, b_k, idesc, (oct > oct0 || ks > 0) ? 1u : 0u);
            if constexpr (Cfg::kSplit) {
              tc::mma_f16(dt, a_k + (kDkBytes >> 4), b_k, idesc, 1u);
              tc::mma_f16(dt, a_k, b_k + b_lo, idesc, 1u);
            }
          }
          tc::mma_commit(&k_empty[ks_]);
          tc::mma_commit(&w_empty[s]);
        }
        tc::mma_commit(&d_full[tb]);
      }
    }
  } else if (warp == 2) {
    // ---- dW issuer: D_w[octet] += dK . y over the split's tiles ---------------
    if (lane == 0) {
      // y tile: K-major [pixel group][channel][8 px] (staged from y), or MN-major
      // [channel group][pixel][8 ch] (copied from the y plane)
      const uint32_t idesc = tc::idesc_f16(kTileM, Nw, IoTraits<T>::kBf16, true, kStaged);
      const uint32_t b_lbo = kStaged ? 128u : (uint32_t)Nw * 16;
      const uint32_t b_sbo = kStaged ? (uint32_t)kTileM * 16 : 128u;
      const uint64_t b_step = kStaged ? (uint64_t)(256 >> 4) : (uint64_t)((2 * b_lbo) >> 4);
      const uint64_t y_lo = (kTileM * Nw * 2) >> 4;
      uint32_t kq = 0, it = 0;
      bool first = true;
      for (int tile = split; tile < p.num_tiles; tile += p.splits, ++it) {
        const int yb = it % NY;
        if (!tc::mbar_wait(&y_full[yb], (it / NY) & 1, abort_flag, kWaitNs, kHintNs)) {
          fail(abort_flag, p.status, 53);
          goto done;
        }
        tc::tc_fence_after();
        const uint64_t yd =
            tc::smem_desc(tc::smem_u32(smem + L.y + yb * L.y_bytes), b_lbo, b_sbo);
        if constexpr (kLoRing) {
          // per octet: lo * y_hi, release lo; hi * y_hi + hi * y_lo
          const uint64_t lo_d =
              tc::smem_desc(tc::smem_u32(smem + L.dk + 2 * kDkBytes), 2048, 128);
          for (int oct = oct0; oct < oct1; ++oct, ++kq) {
            const int hb = kq & 1;
            if (!tc::mbar_wait(&k_full[hb], (kq >> 1) & 1, abort_flag, kWaitNs, kHintNs) ||
                !tc::mbar_wait(lo_full, kq & 1, abort_flag, kWaitNs, kHintNs)) {
              fail(abort_flag, p.status, 54);
              goto done;
            }
            tc::tc_fence_after();
            const uint64_t hi_d =
                tc::smem_desc(tc::smem_u32(smem + L.dk + hb * kDkBytes), 2048, 128);
            const uint32_t dt = tmem_base + (oct - oct0) * Nw;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              tc::mma_f16(dt, lo_d + ks * ((2 * 2048) >> 4), yd + ks * b_step, idesc,
                          (!first || ks > 0) ? 1u : 0u);
            tc::mma_commit(lo_empty);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint64_t a_k = hi_d + ks * ((2 * 2048) >> 4);
              const uint64_t b_k = yd + ks * b_step;
              tc::mma_f16(dt, a_k, b_k, idesc, 1u);
              tc::mma_f16(dt, a_k, b_k + y_lo, idesc, 1u);
            }
            tc::mma_commit(&k_empty[hb]);
          }
          tc::mma_commit(&y_empty[yb]);
          first = false;
          continue;
        }
        for (int oct = oct0; oct < oct1; ++oct, ++kq) {
          const int ks_ = kq % NS;
          if (!tc::mbar_wait(&k_full[ks_], (kq / NS) & 1, abort_flag, kWaitNs, kHintNs)) {
            fail(abort_flag, p.status, 54);
            goto done;
          }
          tc::tc_fence_after();
          // A: dK, MN-major (rows are M, pixels are K): K-group stride 2048, M-group 128
          const uint64_t ad =
              tc::smem_desc(tc::smem_u32(smem + L.dk + ks_ * L.dk_bytes), 2048, 128);
          const uint32_t dt = tmem_base + (oct - oct0) * Nw;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t a_k = ad + ks * ((2 * 2048) >> 4);
            const uint64_t b_k = yd + ks * b_step;
            tc::mma_f16(dt, a_k, b_k, idesc, (!first || ks > 0) ? 1u : 0u);
            if constexpr (Cfg::kSplit) {
              tc::mma_f16(dt, a_k + (kDkBytes >> 4), b_k, idesc, 1u);
              tc::mma_f16(dt, a_k, b_k + y_lo, idesc, 1u);
            }
          }
          tc::mma_commit(&k_empty[ks_]);
        }
        tc::mma_commit(&y_empty[yb]);
        first = false;
      }
      tc::mma_commit(w_done);
    }
  } else if (warp < Cfg::kFirstYWarp) {
    // ---- x-halo producers (the cg's 16 channels, once per tile); without
    //      staged operands they also drain the previous tile's D_y ------------
    const int pt = threadIdx.x - 32 * Cfg::kFirstXWarp;
    const int quad = warp & 3;               // TMEM lane quadrant
    const XPlan<Cfg::kXItems> plan = make_xplan<Cfg::kXItems>(xr_rows, pt, Cfg::kProducers);
    float* dybuf = reinterpret_cast<float*>(smem + L.dyb + quad * kDyChunkBytes);
    auto drain = [&](uint32_t it) -> bool {
      return drain_dy(p, maps, it, split, quad, lane, tmem_base, Cfg::kDyCol, d_full, d_empty,
                      abort_flag, dybuf);
    };
    uint32_t xq = 0;
    bool failed = false;
    for (int tile = split; tile < p.num_tiles && !*abort_flag; tile += p.splits, ++xq) {
      const int xb = xq & nx_sh;
      if (!warp_wait(&x_empty[xb], ((xq >> nx_sh) & 1) ^ 1, abort_flag, kHintNs)) {
        fail(abort_flag, p.status, 55);
        failed = true;
        break;
      }
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      float4* xr = reinterpret_cast<float4*>(smem + L.xr + xb * L.xr_bytes);
      if constexpr (kStaged) {
        // columns w0-8 .. w0+23 (x in 8-byte units), rows h0-R .., quads 4cg .. 4cg+3
        if (pt == 0) {
          tc::mbar_arrive_expect_tx(&x_full[xb], L.xr_bytes);
          tc::tma_load_4d(xr, &maps.xmap, (w0 - xoff) * 2, h0 - R, cg * Cfg::kXCells, n,
                          &x_full[xb]);
        } else {
          tc::mbar_arrive(&x_full[xb]);
        }
        if constexpr (kGTma) {
          // gradient tile (branches 1..3, the cg's 16 channels) once the builders
          // hold the previous one in registers; zero filled outside the image
          if (warp == Cfg::kFirstXWarp + 1) {
            bool ok = true;
            if (lane == 0) {
              ok = tc::mbar_wait(g_empty, (xq & 1) ^ 1, abort_flag, kWaitNs, kHintNs);
              if (ok) {
                tc::mbar_arrive_expect_tx(g_full, L.g_bytes);
                if (p.g_nhwc)
                  tc::tma_load_5d(smem + L.g, &maps.gmap, cg * 16, 1, w0, h0, n, g_full);
                else
                  tc::tma_load_5d(smem + L.g, &maps.gmap, w0, h0, cg * 16, 1, n, g_full);
              }
            }
            if (!__all_sync(0xffffffffu, ok)) {
              fail(abort_flag, p.status, 48);
              failed = true;
              break;
            }
          }
        }
      } else {
        stage_halo<T, Cfg::kXItems>(plan, static_cast<const T*>(p.x), xr, n, C, H, W, cg * 16,
                                    h0 - R, w0 - 8, xr_rows);
        tc::mbar_arrive(&x_full[xb]);
      }
      if (!kStaged && xq > 0 && !drain(xq - 1)) {
        fail(abort_flag, p.status, 59);
        failed = true;
        break;
      }
    }
    if (!kStaged && !failed && xq > 0 && !drain(xq - 1)) fail(abort_flag, p.status, 59);
    if constexpr (!kStaged) {
      // the drain's TMA reductions complete before the CTA exits
      if (lane == 0) tc::bulk_wait_all();
      __syncwarp();
    }
  } else if (warp < Cfg::kFirstBuilderWarp) {
    // ---- y-tile producers (B operand of dW, ones channel at C for db) ---------
    const int pt = threadIdx.x - 32 * Cfg::kFirstYWarp;
    const YPlan<Cfg::kYItems> plan = make_yplan<Cfg::kYItems>(Nw, pt, Cfg::kProducers);
    const int quad = warp & 3;  // TMEM lane quadrant (staged: these warps drain D_y)
    float* dybuf = reinterpret_cast<float*>(smem + L.dyb + quad * kDyChunkBytes);
    uint32_t it = 0;
    bool failed = false;
    for (int tile = split; tile < p.num_tiles && !*abort_flag; tile += p.splits, ++it) {
      const int yb = it % NY;
      if (!warp_wait(&y_empty[yb], ((it / NY) & 1) ^ 1, abort_flag, kHintNs)) {
        fail(abort_flag, p.status, 56);
        failed = true;
        break;
      }
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      uint8_t* ys = smem + L.y + yb * L.y_bytes;
      if constexpr (kStaged) {
        // y plane rows h0+ph .. +7, columns w0+pw .. w0+pw+15, every channel group
        if (pt == 0) {
          tc::mbar_arrive_expect_tx(&y_full[yb], L.y_bytes);
          tc::tma_load_4d(ys, &maps.ymap, (w0 + maps.pw) * 2, h0 + maps.ph, 0, n, &y_full[yb]);
          if constexpr (Cfg::kSplit)
            tc::tma_load_4d(ys + kTileM * Nw * 2, &maps.ymap, (w0 + maps.pw) * 2, h0 + maps.ph, 0,
                            p.N + n, &y_full[yb]);
        } else {
          tc::mbar_arrive(&y_full[yb]);
        }
      } else {
        stage_y_mn<T, Op, Cfg::kSplit, Cfg::kYItems>(plan, static_cast<const T*>(p.y), ys,
                                                     ys + kTileM * Nw * 2, n, C, Nw, C, H, W, h0,
                                                     w0);
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&y_full[yb]);
      }
      if (kStaged && it > 0 &&
          !drain_dy(p, maps, it - 1, split, quad, lane, tmem_base, Cfg::kDyCol, d_full, d_empty,
                    abort_flag, dybuf)) {
        fail(abort_flag, p.status, 59);
        failed = true;
        break;
      }
    }
    if (kStaged && !failed && it > 0 &&
        !drain_dy(p, maps, it - 1, split, quad, lane, tmem_base, Cfg::kDyCol, d_full, d_empty,
                  abort_flag, dybuf))
      fail(abort_flag, p.status, 59);
    if constexpr (kStaged) {
      // the drain's TMA reductions complete before the CTA exits
      if (lane == 0) tc::bulk_wait_all();
      __syncwarp();
    }
  } else {
    // ---- builders (two threads per pixel), D_y and D_w drains ------------------
    const int half = (warp - Cfg::kFirstBuilderWarp) >> 2;
    const int quad = warp & 3;               // TMEM lane quadrant
    const int m = quad * 32 + lane;          // pixel of the tile / weight row of a group
    const int mr = m >> 4, mc = m & 15;
    const T* gout = static_cast<const T*>(p.gout);
    const int dil[3] = {p.d[0], p.d[1], p.d[2]};
    uint32_t xq = 0, kq = 0;
    bool failed = false;
    for (int tile = split; tile < p.num_tiles && !failed; tile += p.splits, ++xq) {
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      const int h = h0 + mr, w = w0 + mc;
      const bool px_ok = (h < H) && (w < W);
      const size_t pix = px_ok ? (size_t)h * W + w : 0;
      const T* gn = gout + (size_t)n * 4 * C * P;
      // gradient pairs of the pixel's 16 channels per branch: as f32x2 (gv) for
      // the FP32-cell builders, as raw 16-bit pairs (gw) for kXIo
      unsigned long long gv[3][8];
      uint32_t gw[3][8];
      if constexpr (kGTma) {
        static_assert(!kGTma || Cfg::kXIo, "the gradient tile by TMA implies staged 16-bit x cells");
        if (!warp_wait(g_full, xq & 1, abort_flag, kHintNs)) {
          fail(abort_flag, p.status, 47);
          failed = true;
          break;
        }
        if (p.g_nhwc) {
          // [pixel][branch][16 channels]: two 16-byte vectors per branch
          const uint4* gq = reinterpret_cast<const uint4*>(smem + L.g) + m * 6;
#pragma unroll
          for (int b = 0; b < 3; ++b) {
            const uint4 v0 = gq[2 * b], v1 = gq[2 * b + 1];
            gw[b][0] = v0.x; gw[b][1] = v0.y; gw[b][2] = v0.z; gw[b][3] = v0.w;
            gw[b][4] = v1.x; gw[b][5] = v1.y; gw[b][6] = v1.z; gw[b][7] = v1.w;
          }
        } else {
          const T* gs = reinterpret_cast<const T*>(smem + L.g) + m;
#pragma unroll
          for (int b = 0; b < 3; ++b)
#pragma unroll
            for (int i = 0; i < 8; ++i)
              gw[b][i] = pack_raw2<T>(gs[(b * 16 + 2 * i) * kTileM], gs[(b * 16 + 2 * i + 1) * kTileM]);
        }
        // The next tile's gradient arrives by TMA into this buffer once the
        // arrivals below are in: every thread first waits for its own loads (a
        // use of every loaded value here; the compiler may otherwise place the
        // uses after the arrival) and orders them before the async proxy's
        // writes. With one leader arrival after __syncwarp, and the values
        // consumed later, the TMA overwrote words still being loaded.
        {
          uint32_t dep = 0;
#pragma unroll
          for (int b = 0; b < 3; ++b)
#pragma unroll
            for (int i = 0; i < 8; ++i) dep ^= gw[b][i];
          asm volatile("" ::"r"(dep));
        }
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(g_empty);
      } else {
        if (p.g_nhwc)
          load_gv_nhwc<T>(gv, gout, n, H, W, C, cg, h, w, px_ok);
        else
          load_gv<T>(gv, gn, C, P, cg, pix, px_ok);
        if constexpr (Cfg::kXIo) {
          // exact: the values came from the 16-bit gradient
#pragma unroll
          for (int b = 0; b < 3; ++b)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float lo, hi;
              f2_unpack(gv[b][i], lo, hi);
              gw[b][i] = cvt2<Op>(lo, hi);
            }
        }
      }
      const int xb = xq & nx_sh;
      if (!warp_wait(&x_full[xb], (xq >> nx_sh) & 1, abort_flag, kHintNs)) {
        fail(abort_flag, p.status, 57);
        failed = true;
        break;
      }
      const int xcell0 = (mr + R) * xcols + (mc + xoff);
      const float4* xc = reinterpret_cast<const float4*>(smem + L.xr + xb * L.xr_bytes) + xcell0;
      const uint4* xci = reinterpret_cast<const uint4*>(smem + L.xr + xb * L.xr_bytes) + xcell0;
      for (int oct = oct0; oct < oct1; ++oct, ++kq) {
        const int ks_ = kq % NS;
        if (!warp_wait(&k_empty[ks_], ((kq / NS) & 1) ^ 1, abort_flag, kHintNs) ||
            (kLoRing && !warp_wait(lo_empty, (kq & 1) ^ 1, abort_flag, kHintNs))) {
          fail(abort_flag, p.status, 58);
          failed = true;
          break;
        }
        // lo ring: hi part in slot ks_, lo part in the buffer after both slots
        const uint32_t lo_off = kLoRing ? (uint32_t)(2 - ks_) * kDkBytes : (uint32_t)kDkBytes;
        if constexpr (Cfg::kXIo)
          build_dk_half_io<T, Op, KS>(smem + L.dk + ks_ * L.dk_bytes, oct, half, xci, xr_plane,
                                      gw, dil, m, xcols);
        else
          build_dk_half<T, Op, Cfg::kSplit, KS>(smem + L.dk + ks_ * L.dk_bytes, oct, half, xc,
                                                xr_plane, gv, dil, m, lo_off, xcols);
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&k_full[ks_]);
        if constexpr (kLoRing) tc::mbar_arrive(lo_full);
      }
      if (failed) break;
      tc::mbar_arrive(&x_empty[xb]);
    }
    // D_w of this CTA's split: lane = weight row, half h drains octets 2h, 2h+1
    if (!failed && warp_wait(w_done, 0, abort_flag, kHintNs)) {
      tc::tc_fence_after();
      for (int lo = 2 * half; lo < 2 * half + 2 && oct0 + lo < oct1; ++lo) {
        const int g = cg * NOCT + oct0 + lo;
        float* dst = p.partial + (((size_t)split * p.ngroups + g) * 128 + m) * Nw;
        for (int c0 = 0; c0 < Nw; c0 += 16) {
          float dv[16];
          tc::tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + lo * Nw + c0, dv);
          tc::tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 16; k += 4)
            *reinterpret_cast<float4*>(dst + c0 + k) =
                make_float4(dv[k], dv[k + 1], dv[k + 2], dv[k + 3]);
        }
      }
    } else if (!failed) {
      fail(abort_flag, p.status, 49);
    }
  }
done:
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 512);
  }
}

// dY (16-bit) = the FP32 accumulator rounded once.
template <typename T>
__global__ void gy_convert_kernel(const float* __restrict__ acc, T* __restrict__ gy, size_t n) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t i0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t done = 0;
  if ((reinterpret_cast<uintptr_t>(gy) & 7u) == 0) {
    // four elements per step: one 16-byte load, one 8-byte store
    const size_t n4 = n / 4;
    const float4* a4 = reinterpret_cast<const float4*>(acc);
    uint2* g4 = reinterpret_cast<uint2*>(gy);
    for (size_t i = i0; i < n4; i += stride) {
      const float4 v = a4[i];
      union {
        uint2 u;
        T e[4];
      } o;
      o.e[0] = from_f32<T>(v.x);
      o.e[1] = from_f32<T>(v.y);
      o.e[2] = from_f32<T>(v.z);
      o.e[3] = from_f32<T>(v.w);
      g4[i] = o.u;
    }
    done = n4 * 4;
  }
  for (size_t i = done + i0; i < n; i += stride) gy[i] = from_f32<T>(acc[i]);
}

// ------------------------------------------------------------- launchers ----
template <typename T, int KS>
int launch_y(const ByParams& prm, cudaStream_t st) {
  using Cfg = ByCfg<T, KS>;
  const BySmem L = by_smem_layout<T, KS>(prm.Cp, prm.R);
  auto fn = gencat_bwd_y_kernel<T, KS>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  const int grid = prm.num_tiles < num_sms() ? prm.num_tiles : num_sms();
  fn<<<grid, Cfg::kThreads, L.total, st>>>(prm);
  DDPM_CHECK_LAUNCH("gencat_bwd_y_kernel");
  return DDPM_OK;
}

template <typename T, int KS>
int launch_w(BwParams prm, int nbatches, cudaStream_t st) {
  using Cfg = BwCfg<T, KS>;
  const BwSmem L = bw_smem_layout<T, KS>(prm.Nw, prm.R);
  auto fn = gencat_bwd_w_kernel<T, KS>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  fn<<<nbatches * prm.splits, Cfg::kThreads, L.total, st>>>(prm);
  DDPM_CHECK_LAUNCH("gencat_bwd_w_kernel");
  return DDPM_OK;
}

template <typename T>
int launch_reduce(const float* partial, void* gw, void* gb, int C, int KS, int ngroups, int Nw,
                  int splits, cudaStream_t st) {
  const long long total = (long long)ngroups * 128 * (C + 1);
  const int threads = 256;
  const long long want = (total + threads - 1) / threads;
  gencat_wreduce_kernel<T><<<(int)(want < 2048 ? want : 2048), threads, 0, st>>>(
      partial, static_cast<T*>(gw), static_cast<T*>(gb), C, KS, ngroups, Nw, splits);
  DDPM_CHECK_LAUNCH("gencat_wreduce_kernel");
  return DDPM_OK;
}

struct WPlan {
  int Nw, gb, nbatches, splits;
  size_t ws_bytes;
};

WPlan plan_w(int n, int c, int h, int w, int ks) {
  const gencat::PackLayout pl = gencat::PackLayout::make(c, ks, DDPM_BF16);
  WPlan q;
  q.Nw = gencat::augmented_channels(c);  // input channels + the constant-one (db) column
  q.gb = 512 / q.Nw;
  if (q.gb > pl.NG) q.gb = pl.NG;
  q.nbatches = (pl.NG + q.gb - 1) / q.gb;
  const int tiles = n * ((h + gencat::kTileH - 1) / gencat::kTileH) *
                    ((w + gencat::kTileW - 1) / gencat::kTileW);
  int sp = num_sms() / q.nbatches;
  if (sp < 1) sp = 1;
  if (sp > tiles) sp = tiles;
  q.splits = sp;
  q.ws_bytes = (size_t)sp * pl.NG * 128 * q.Nw * sizeof(float);
  return q;
}

// Merged dY + dW pass: CTAs = channel groups x splits; workspace = D_w partials,
// then (16-bit dY only) the FP32 dY accumulator at a 256-byte aligned offset.
struct DywPlan {
  int Nw, ncg, nsets, splits;  // CTAs = ncg x nsets x splits
  size_t partial_bytes, acc_offset, ws_bytes;  // ws_bytes includes the accumulator
};

DywPlan plan_dyw(int n, int c, int h, int w, int ks) {
  const gencat::PackLayout pl = gencat::PackLayout::make(c, ks, DDPM_BF16);
  DywPlan q;
  q.Nw = gencat::augmented_channels(c);
  q.ncg = pl.Cp / 16;
  const int noct = (3 * ks * ks + 7) / 8;
  q.nsets = ks <= 3 ? 1 : (noct + kDywSetOct - 1) / kDywSetOct;
  const int tiles = n * ((h + gencat::kTileH - 1) / gencat::kTileH) *
                    ((w + gencat::kTileW - 1) / gencat::kTileW);
  int sp = num_sms() / (q.ncg * q.nsets);
  if (sp < 1) sp = 1;
  if (sp > tiles) sp = tiles;
  q.splits = sp;
  q.partial_bytes = (size_t)sp * pl.NG * 128 * q.Nw * sizeof(float);
  q.acc_offset = (q.partial_bytes + 255) / 256 * 256;
  q.ws_bytes = q.acc_offset + (size_t)n * c * h * w * sizeof(float);
  return q;
}

template <typename T, int KS, bool kStaged, bool kGTma, bool kLoRing = false>
int launch_dyw_k(const DywParams& prm, const DywMaps& maps, cudaStream_t st) {
  using Cfg = DywCfg<T, KS, kStaged, kGTma, kLoRing>;
  const DywSmem L =
      dyw_smem_layout<T, KS, kGTma, kLoRing, kStaged>(prm.Cp, prm.Nw, prm.R, prm.nx);
  auto fn = gencat_bwd_dyw_kernel<T, KS, kStaged, kGTma, kLoRing>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  fn<<<prm.ncg * prm.nsets * prm.splits, Cfg::kThreads, L.total, st>>>(prm, maps);
  DDPM_CHECK_LAUNCH("gencat_bwd_dyw_kernel");
  return DDPM_OK;
}

// Picks the variant and the x-buffer count: the gradient tile by TMA where the
// caller could encode its map (16-bit, staged), two x buffers where they fit.
template <typename T, int KS>
int launch_dyw(DywParams prm, const DywMaps& maps, bool staged, bool g_tma, cudaStream_t st) {
  const int lim = max_smem_optin();
  constexpr int kMaxX = DywCfg<T, KS>::kXBufs;
  if constexpr (!IoTraits<T>::kSplit) {
    if (staged && g_tma)
      for (int nx = kMaxX; nx >= 1; --nx)
        if ((int)dyw_smem_layout<T, KS, true, false, true>(prm.Cp, prm.Nw, prm.R, nx).total <=
            lim) {
          prm.nx = nx;
          return launch_dyw_k<T, KS, true, true>(prm, maps, st);
        }
  } else {
    // FP32: the lo ring where it fits (halos up to 5 at C = 64)
    if (staged &&
        (int)dyw_smem_layout<T, KS, false, true, true>(prm.Cp, prm.Nw, prm.R, 1).total <= lim) {
      prm.nx = 1;
      return launch_dyw_k<T, KS, true, false, true>(prm, maps, st);
    }
  }
  if constexpr (KS <= 3) {
    for (int nx = kMaxX; nx >= 1; --nx) {
      const uint32_t need =
          staged ? dyw_smem_layout<T, KS, false, false, true>(prm.Cp, prm.Nw, prm.R, nx).total
                 : dyw_smem_layout<T, KS>(prm.Cp, prm.Nw, prm.R, nx).total;
      if ((int)need <= lim) {
        prm.nx = nx;
        return staged ? launch_dyw_k<T, KS, true, false>(prm, maps, st)
                      : launch_dyw_k<T, KS, false, false>(prm, maps, st);
      }
    }
  }
  // K = 5 runs only with staged operands and the gradient tile by TMA
  return set_error(DDPM_ERR_UNSUPPORTED, "dY+dW tile does not fit in shared memory");
}

template <typename T>
int finish_dyw(const DywParams& prm, void* gy, void* gw, void* gb, int c, int ks, int ngroups,
               cudaStream_t st) {
  int rc = launch_reduce<T>(prm.partial, gw, gb, c, ks, ngroups, prm.Nw, prm.splits, st);
  if (rc) return rc;
  if constexpr (!std::is_same<T, float>::value) {
    const size_t nel = (size_t)prm.N * c * prm.H * prm.W;
    const size_t want = (nel / 4 + 255) / 256 + 1;
    gy_convert_kernel<T><<<(int)(want < 4096 ? want : 4096), 256, 0, st>>>(
        prm.gy_acc, static_cast<T*>(gy), nel);
    DDPM_CHECK_LAUNCH("gy_convert_kernel");
  }
  return DDPM_OK;
}

}  // namespace

size_t gencat_bwd_workspace_bytes(int n, int c, int h, int w, int ks) {
  if (n < 1 || c < 1 || c > gencat::kMaxChannels || h < 1 || w < 1 ||
      (ks != 1 && ks != 3 && ks != 5))
    return 0;
  if (ks == 5) return plan_dyw(n, c, h, w, ks).ws_bytes;  // the merged pass only
  const size_t a = plan_w(n, c, h, w, ks).ws_bytes;
  const size_t b = plan_dyw(n, c, h, w, ks).ws_bytes;
  return a > b ? a : b;
}

// `staged`: staged operands (gencat::stage with x) for the merged pass, or null
// to stage tiles from x and y.
int gencat_bwd_yw(const void* x, const void* y, const void* staged, size_t staged_bytes,
                  const void* wpack, const void* gout, void* gy, void* gw, void* gb,
                  void* workspace, size_t ws_bytes, int n, int c, int h, int w, int ks, int d0,
                  int d1, int d2, int dt, cudaStream_t st, int g_nhwc) {
  // K = 5: the merged pass with staged operands, 16-bit data (the gradient tile
  // by TMA; FP32's hi / lo operand rings leave no room for its wider halo)
  int rc = ks == 5 ? gencat::check_shape(n, c, h, w, ks, d0, d1, d2, dt)
                   : gencat::check_shape_bwd(n, c, h, w, ks, d0, d1, d2, dt);
  if (rc) return rc;
  if (ks == 5 && (dt == DDPM_F32 || staged == nullptr || gy == nullptr || gw == nullptr ||
                  gb == nullptr || workspace == nullptr))
    return set_error(DDPM_ERR_UNSUPPORTED,
                     "fused dY + dW at K = 5 needs 16-bit data, staged operands, all three "
                     "gradients and the workspace");
  DDPM_CHECK_ARG(((x && y) || staged) && wpack && gout, "null pointer");
  if (g_nhwc && (c != 64 || staged == nullptr))
    return set_error(DDPM_ERR_UNSUPPORTED,
                     "a channel-last grad_out needs C == 64 and staged operands");
  if (staged != nullptr) {
    const gencat::StageLayout sl = gencat::StageLayout::make(n, c, h, w, ks, d0, d1, d2, dt);
    if (staged_bytes < sl.total_bytes())
      return set_error(DDPM_ERR_WORKSPACE, "staged operands too small (%zu < %zu)", staged_bytes,
                       sl.total_bytes());
    DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(staged) & 255u) == 0,
                   "staged operands must be 256-byte aligned");
    DDPM_CHECK_ARG(gy && gw && gb && workspace,
                   "the staged pass computes grad_y, grad_weight and grad_bias together");
  }
  const gencat::PackLayout pl = gencat::PackLayout::make(c, ks, dt);
  const int R = (ks / 2) * max3(d0, d1, d2);
  const int tiles_w = (w + gencat::kTileW - 1) / gencat::kTileW;
  const int tiles_h = (h + gencat::kTileH - 1) / gencat::kTileH;
  int* status = nullptr;
  rc = gencat::status_ptr(&status);
  if (rc) return rc;

  if (gy != nullptr && gw != nullptr && gb != nullptr && workspace != nullptr &&
      (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0) {
    // merged pass: dK built once for dY and dW
    const DywPlan q = plan_dyw(n, c, h, w, ks);
    const size_t need = dt == DDPM_F32 ? q.partial_bytes : q.ws_bytes;
    if (ws_bytes >= need) {
      DywParams dp{};
      dp.x = x;
      dp.y = y;
      dp.wpack = static_cast<const uint8_t*>(wpack) + pl.by_offset();
      dp.gout = gout;
      dp.partial = static_cast<float*>(workspace);
      dp.gy_acc = dt == DDPM_F32 ? static_cast<float*>(gy)
                                 : reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                                            q.acc_offset);
      dp.N = n;
      dp.C = c;
      dp.H = h;
      dp.W = w;
      dp.Cp = pl.Cp;
      dp.Nw = q.Nw;
      dp.R = R;
      dp.d[0] = d0;
      dp.d[1] = d1;
      dp.d[2] = d2;
      dp.tiles_w = tiles_w;
      dp.tiles_h = tiles_h;
      dp.num_tiles = n * tiles_w * tiles_h;
      dp.ngroups = pl.NG;
      dp.ncg = q.ncg;
      dp.splits = q.splits;
      dp.nsets = q.nsets;
      dp.status = status;
      bool use_staged = false, g_tma = false;
      DywMaps maps{};
      if (staged != nullptr) {
        const gencat::StageLayout sl = gencat::StageLayout::make(n, c, h, w, ks, d0, d1, d2, dt);
        use_staged = gencat::encode_stage_maps(&maps.xmap, &maps.ymap, R, sl.G,
                                               static_cast<const uint8_t*>(staged), sl,
                                               dyw_halo_cols(ks, R), 16 / sl.xcell);
        maps.ph = sl.ph;
        maps.pw = sl.pw;
        // gradient tiles by TMA (16-bit) when the row pitch and base allow a map
        const size_t es = (size_t)dtype_size(dt);
        if (g_nhwc && dt == DDPM_F32) {
          // FP32 builders load their gradient values themselves (channel-last)
          DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(gout) & 15u) == 0,
                         "grad_out must be 16-byte aligned");
          dp.g_nhwc = 1;
        } else if (g_nhwc) {
          const uint64_t gd[5] = {(uint64_t)c, 4, (uint64_t)w, (uint64_t)h, (uint64_t)n};
          const uint64_t gs[4] = {(uint64_t)c * es, (uint64_t)4 * c * es,
                                  (uint64_t)4 * c * w * es, (uint64_t)4 * c * w * h * es};
          const uint32_t gb_[5] = {16, 3, (uint32_t)gencat::kTileW, (uint32_t)gencat::kTileH, 1};
          const CUtensorMapDataType ty = dt == DDPM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
          if (!use_staged || (reinterpret_cast<uintptr_t>(gout) & 15u) != 0 ||
              encode_tmap(&maps.gmap, ty, 5, gout, gd, gs, gb_, CU_TENSOR_MAP_SWIZZLE_NONE) !=
                  DDPM_OK)
            return set_error(DDPM_ERR_UNSUPPORTED,
                             "channel-last grad_out: the gradient tensor map is unavailable");
          g_tma = true;
          dp.g_nhwc = 1;
        } else if (use_staged && dt != DDPM_F32 && ((size_t)w * es) % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(gout) & 15u) == 0) {
          const uint64_t gd[5] = {(uint64_t)w, (uint64_t)h, (uint64_t)c, 4, (uint64_t)n};
          const uint64_t gs[4] = {w * es, (uint64_t)h * w * es, (uint64_t)c * h * w * es,
                                  (uint64_t)4 * c * h * w * es};
          const uint32_t gb_[5] = {(uint32_t)gencat::kTileW, (uint32_t)gencat::kTileH, 16, 3, 1};
          const CUtensorMapDataType ty = dt == DDPM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
          if (encode_tmap(&maps.gmap, ty, 5, gout, gd, gs, gb_, CU_TENSOR_MAP_SWIZZLE_NONE) ==
              DDPM_OK)
            g_tma = true;
          else
            clear_error();
        }
      }
      DDPM_CHECK_ARG(use_staged || (x && y), "tensor maps unavailable: x and y are needed");
      // D_y drains by TMA reductions into the FP32 accumulator where its row
      // pitch and base allow a tensor map (else by atomics)
      if (((size_t)w * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(dp.gy_acc) & 15u) == 0) {
        const uint64_t dd[4] = {(uint64_t)w, (uint64_t)h, (uint64_t)c, (uint64_t)n};
        const uint64_t ds[3] = {(uint64_t)w * 4, (uint64_t)h * w * 4, (uint64_t)c * h * w * 4};
        const uint32_t db[4] = {16, 2, 8, 1};
        if (encode_tmap(&maps.dymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dp.gy_acc, dd, ds, db,
                        CU_TENSOR_MAP_SWIZZLE_NONE) == DDPM_OK)
          maps.dy_tma = 1;
        else
          clear_error();
      }
      if (ks == 5 && !(use_staged && g_tma))
        return set_error(DDPM_ERR_UNSUPPORTED,
                         "fused dY + dW at K = 5 needs the gradient tile by TMA (16-byte aligned "
                         "rows)");
      DDPM_CUDA_TRY(cudaMemsetAsync(dp.gy_acc, 0, (size_t)n * c * h * w * sizeof(float), st));
      switch (dt * 10 + ks) {
        case DDPM_BF16 * 10 + 1: rc = launch_dyw<__nv_bfloat16, 1>(dp, maps, use_staged, g_tma, st); break;
        case DDPM_BF16 * 10 + 3: rc = launch_dyw<__nv_bfloat16, 3>(dp, maps, use_staged, g_tma, st); break;
        case DDPM_F16 * 10 + 1: rc = launch_dyw<__half, 1>(dp, maps, use_staged, g_tma, st); break;
        case DDPM_F16 * 10 + 3: rc = launch_dyw<__half, 3>(dp, maps, use_staged, g_tma, st); break;
        case DDPM_F32 * 10 + 1: rc = launch_dyw<float, 1>(dp, maps, use_staged, g_tma, st); break;
        case DDPM_F32 * 10 + 3: rc = launch_dyw<float, 3>(dp, maps, use_staged, g_tma, st); break;
        case DDPM_BF16 * 10 + 5: rc = launch_dyw<__nv_bfloat16, 5>(dp, maps, true, true, st); break;
        case DDPM_F16 * 10 + 5: rc = launch_dyw<__half, 5>(dp, maps, true, true, st); break;
        default: rc = set_error(DDPM_ERR_UNSUPPORTED, "unsupported dtype/kernel size");
      }
      if (rc) return rc;
      switch (dt) {
        case DDPM_BF16: return finish_dyw<__nv_bfloat16>(dp, gy, gw, gb, c, ks, pl.NG, st);
        case DDPM_F16: return finish_dyw<__half>(dp, gy, gw, gb, c, ks, pl.NG, st);
        default: return finish_dyw<float>(dp, gy, gw, gb, c, ks, pl.NG, st);
      }
    }
  }
  // separate dY and dW passes (no merged-pass workspace): they stage from x and y
  if (g_nhwc)
    return set_error(DDPM_ERR_UNSUPPORTED,
                     "a channel-last grad_out needs the merged pass (grad_y, grad_weight, "
                     "grad_bias and the workspace)");
  DDPM_CHECK_ARG(x && y, "x and y are needed without a merged-pass workspace");
  if (gy != nullptr) {
    ByParams bp{};
    bp.x = x;
    bp.wpack = static_cast<const uint8_t*>(wpack) + pl.by_offset();
    bp.gout = gout;
    bp.gy = gy;
    bp.N = n;
    bp.C = c;
    bp.H = h;
    bp.W = w;
    bp.Cp = pl.Cp;
    bp.R = R;
    bp.d[0] = d0;
    bp.d[1] = d1;
    bp.d[2] = d2;
    bp.tiles_w = tiles_w;
    bp.tiles_h = tiles_h;
    bp.num_tiles = n * tiles_w * tiles_h;
    bp.status = status;
    switch (dt * 10 + ks) {
      case DDPM_BF16 * 10 + 1: rc = launch_y<__nv_bfloat16, 1>(bp, st); break;
      case DDPM_BF16 * 10 + 3: rc = launch_y<__nv_bfloat16, 3>(bp, st); break;
      case DDPM_F16 * 10 + 1: rc = launch_y<__half, 1>(bp, st); break;
      case DDPM_F16 * 10 + 3: rc = launch_y<__half, 3>(bp, st); break;
      case DDPM_F32 * 10 + 1: rc = launch_y<float, 1>(bp, st); break;
      case DDPM_F32 * 10 + 3: rc = launch_y<float, 3>(bp, st); break;
      default: rc = set_error(DDPM_ERR_UNSUPPORTED, "unsupported dtype/kernel size");
    }
    if (rc) return rc;
  }
  if (gw != nullptr || gb != nullptr) {
    DDPM_CHECK_ARG(gw && gb, "grad_weight and grad_bias must both be given");
    const WPlan q = plan_w(n, c, h, w, ks);
    if (workspace == nullptr || ws_bytes < q.ws_bytes)
      return set_error(DDPM_ERR_WORKSPACE, "workspace too small (%zu < %zu)", ws_bytes, q.ws_bytes);
    DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 15u) == 0,
                   "workspace must be 16-byte aligned");
    BwParams wp{};
    wp.x = x;
    wp.y = y;
    wp.gout = gout;
    wp.partial = static_cast<float*>(workspace);
    wp.N = n;
    wp.C = c;
    wp.H = h;
    wp.W = w;
    wp.Cp = pl.Cp;
    wp.Nw = q.Nw;
    wp.R = R;
    wp.d[0] = d0;
    wp.d[1] = d1;
    wp.d[2] = d2;
    wp.tiles_w = tiles_w;
    wp.tiles_h = tiles_h;
    wp.num_tiles = n * tiles_w * tiles_h;
    wp.ngroups = pl.NG;
    wp.gb = q.gb;
    wp.splits = q.splits;
    wp.status = status;
    switch (dt * 10 + ks) {
      case DDPM_BF16 * 10 + 1: rc = launch_w<__nv_bfloat16, 1>(wp, q.nbatches, st); break;
      case DDPM_BF16 * 10 + 3: rc = launch_w<__nv_bfloat16, 3>(wp, q.nbatches, st); break;
      case DDPM_F16 * 10 + 1: rc = launch_w<__half, 1>(wp, q.nbatches, st); break;
      case DDPM_F16 * 10 + 3: rc = launch_w<__half, 3>(wp, q.nbatches, st); break;
      case DDPM_F32 * 10 + 1: rc = launch_w<float, 1>(wp, q.nbatches, st); break;
      case DDPM_F32 * 10 + 3: rc = launch_w<float, 3>(wp, q.nbatches, st); break;
      default: rc = set_error(DDPM_ERR_UNSUPPORTED, "unsupported dtype/kernel size");
    }
    if (rc) return rc;
    switch (dt) {
      case DDPM_BF16:
        return launch_reduce<__nv_bfloat16>(wp.partial, gw, gb, c, ks, pl.NG, q.Nw, q.splits, st);
      case DDPM_F16:
        return launch_reduce<__half>(wp.partial, gw, gb, c, ks, pl.NG, q.Nw, q.splits, st);
      case DDPM_F32:
        return launch_reduce<float>(wp.partial, gw, gb, c, ks, pl.NG, q.Nw, q.splits, st);
    }
  }
  return DDPM_OK;
}

// --------------------------------------------- no-allocation variant -----
// gencat_bwd_yw_static computes the same dY, dW and db as gencat_bwd_yw but
// keeps the FP32 weight-gradient partials in a fixed file-scope device array
// instead of a caller-provided workspace, so the call itself allocates no
// device memory. It serves hosts that cannot hand us a workspace: a plain C
// caller that only owns the tensors of the step (no allocator of its own), or
// a step loop that must not call cudaMalloc because that call can synchronise
// the whole device and stall work queued on other streams.
//
// Limits and contract:
//  * the scratch is kStaticScratchBytes (8 MiB) per device. The spatial split
//    count of the weight-gradient reduction is capped so that
//    splits * groups * 128 * Nw FP32 partials fit; a shape whose single split
//    would not fit is rejected with DDPM_ERR_WORKSPACE (cannot happen within
//    the fused kernels' C <= 64, K <= 3 limits: one split is at most 640 KiB).
//    Fewer splits than the workspace path means fewer CTAs on the dW kernel,
//    so this variant is slower on large images; the summation order differs
//    from gencat_bwd_yw's, so dW / db agree to FP32 rounding, not bit for bit.
//  * nothing in the scratch needs to start at zero: every partial the reduce
//    kernel reads is written by the dW kernel earlier in the same call.
//  * the scratch is shared by every call on a device. Two calls whose kernels
//    can overlap (different streams without ordering, or several host
//    threads) race on it and corrupt each other's dW / db; callers must
//    order them, e.g. by issuing them on one stream.
//  * the device address of the scratch is looked up once per device, on the
//    first call made while that device is current, with
//    cudaGetSymbolAddress; that first call should therefore come before any
//    stream capture is begun on the device.
namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;
constexpr int kMaxScratchDevices = 64;

__device__ __align__(256) unsigned char g_bwd_static_scratch[kStaticScratchBytes];

std::mutex g_static_scratch_mu;
void* g_static_scratch_addr[kMaxScratchDevices] = {};

// Device address of this device's scratch, looked up on first use.
int static_scratch(void** out) {
  int dev = -1;
  DDPM_CUDA_TRY(cudaGetDevice(&dev));
  DDPM_CHECK_ARG(dev >= 0 && dev < kMaxScratchDevices, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (g_static_scratch_addr[dev] == nullptr) {
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_bwd_static_scratch);
    if (e != cudaSuccess || addr == nullptr)
      return set_error(DDPM_ERR_CUDA, "cudaGetSymbolAddress(static scratch) failed: %s",
                       cudaGetErrorString(e));
    g_static_scratch_addr[dev] = addr;
  }
  *out = g_static_scratch_addr[dev];
  return DDPM_OK;
}

}  // namespace

int gencat_bwd_yw_static(const void* x, const void* y, const void* wpack, const void* gout,
                         void* gy, void* gw, void* gb, int n, int c, int h, int w, int ks, int d0,
                         int d1, int d2, int dt, cudaStream_t st) {
  int rc = gencat::check_shape_bwd(n, c, h, w, ks, d0, d1, d2, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG(x && y && wpack && gout, "null pointer");
  DDPM_CHECK_ARG((gw == nullptr) == (gb == nullptr),
                 "grad_weight and grad_bias must both be given");
  void* scratch = nullptr;
  rc = static_scratch(&scratch);
  if (rc) return rc;
  // dY needs no scratch: the workspace path's dY launch is used as is.
  if (gy != nullptr) {
    rc = gencat_bwd_yw(x, y, nullptr, 0, wpack, gout, gy, nullptr, nullptr, nullptr, 0, n, c, h,
                       w, ks, d0, d1, d2, dt, st, 0);
    if (rc) return rc;
  }
  if (gw == nullptr) return DDPM_OK;

  const gencat::PackLayout pl = gencat::PackLayout::make(c, ks, dt);
  WPlan q = plan_w(n, c, h, w, ks);
  const size_t split_bytes = (size_t)pl.NG * 128 * q.Nw * sizeof(float);
  if (split_bytes > kStaticScratchBytes)
    return set_error(DDPM_ERR_WORKSPACE,
                     "shape needs %zu bytes of static scratch, the limit is %zu bytes",
                     split_bytes, kStaticScratchBytes);
  const int max_splits = (int)(kStaticScratchBytes / split_bytes);
  if (q.splits > max_splits) q.splits = max_splits;
  int* status = nullptr;
  rc = gencat::status_ptr(&status);
  if (rc) return rc;

  BwParams wp{};
  wp.x = x;
  wp.y = y;
  wp.gout = gout;
  wp.partial = static_cast<float*>(scratch);
  wp.N = n;
  wp.C = c;
  wp.H = h;
  wp.W = w;
  wp.Cp = pl.Cp;
  wp.Nw = q.Nw;
  wp.R = (ks / 2) * max3(d0, d1, d2);
  wp.d[0] = d0;
  wp.d[1] = d1;
  wp.d[2] = d2;
  wp.tiles_w = (w + gencat::kTileW - 1) / gencat::kTileW;
  wp.tiles_h = (h + gencat::kTileH - 1) / gencat::kTileH;
  wp.num_tiles = n * wp.tiles_w * wp.tiles_h;
  wp.ngroups = pl.NG;
  wp.gb = q.gb;
  wp.splits = q.splits;
  wp.status = status;
  switch (dt * 10 + ks) {
    case DDPM_BF16 * 10 + 1: rc = launch_w<__nv_bfloat16, 1>(wp, q.nbatches, st); break;
    case DDPM_BF16 * 10 + 3: rc = launch_w<__nv_bfloat16, 3>(wp, q.nbatches, st); break;
    case DDPM_F16 * 10 + 1: rc = launch_w<__half, 1>(wp, q.nbatches, st); break;
    case DDPM_F16 * 10 + 3: rc = launch_w<__half, 3>(wp, q.nbatches, st); break;
    case DDPM_F32 * 10 + 1: rc = launch_w<float, 1>(wp, q.nbatches, st); break;
    case DDPM_F32 * 10 + 3: rc = launch_w<float, 3>(wp, q.nbatches, st); break;
    default: rc = set_error(DDPM_ERR_UNSUPPORTED, "unsupported dtype/kernel size");
  }
  if (rc) return rc;
  switch (dt) {
    case DDPM_BF16:
      return launch_reduce<__nv_bfloat16>(wp.partial, gw, gb, c, ks, pl.NG, q.Nw, q.splits, st);
    case DDPM_F16:
      return launch_reduce<__half>(wp.partial, gw, gb, c, ks, pl.NG, q.Nw, q.splits, st);
    default:
      return launch_reduce<float>(wp.partial, gw, gb, c, ks, pl.NG, q.Nw, q.splits, st);
  }
}

}  // namespace ddpm
