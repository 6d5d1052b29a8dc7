// Fused generator backward, input gradient dX (recompute of the taps).
// Replaces `_generator_dynamic_cat_bwd_x` (reference `_triton_kernels.py:430-531`):
//
//   dX[c, q] = g[c, q] + sum_{b, tap} gen[(b,c,tap), q - o] * g_b[c, q - o]
//   gen      = round_io(W * y + bias)      (the forward's taps, recomputed)
//   o        = ((ki - r) * d_b, (kj - r) * d_b), zero outside the image.
//
// The taps needed at q are the generator outputs at the SHIFTED pixel q - o.
// Tile = 128 consecutive pixels of one image row (TMEM lane m <-> column
// w0 + m). Work advances in units = (tile, branch b, kernel row ki): the y row
// h - (ki - r) d_b, columns w0-8 .. w0+135 (w0-16 .. w0+143 at K = 5, whose
// halos reach 16), is staged once per unit in the
// K-major interleaved operand layout ([channel group][pixel][8]); pixel rows
// are 16 bytes apart, so the operand of tap (ki, kj) is the staged segment
// with the descriptor start moved by (8 - dx) pixels, and each (b, tap) chunk
// is one M=128 x N=Cp GEMM whose rows are already the shifted taps. Instead
// of 27 reloads of shifted y tiles (the reference's approach) a tile stages
// 3K row segments.
//
// The same unit also stages the upstream-gradient row g_b[:, h - dy, w0-8 ..
// w0+135] (all Cp channels, I/O dtype) with 1-D bulk copies that complete on
// the unit's barrier, so the epilogue reads g_b at q - o from shared memory
// instead of gathering it through L1 (27 x 64 scalar loads per pixel and tile
// bounded the earlier version by memory latency). Units are double buffered.
//
// Warp roles: w0 = TMEM allocator + weight producer, w1-w2 = MMA issuers
// (even / odd chunks: one thread issuing N=Cp MMAs back to back leaves the
// tensor pipe idle ~half the time), then the unit producers, then two epilogue
// warpgroups owning the 16-channel blocks {0, 2} and {1, 3} of every chunk.
// Producers: from y itself, 8 warps load 8-pixel vectors and transpose them
// into the operand (each thread issues its global loads before waiting for a
// free buffer) and the gradient rows arrive by one bulk copy per channel; from
// staged y (gencat_stage.cu, a channel-last operand copy of y), one thread
// issues one 1-D bulk copy per (part, channel group) and, when the row pitch
// allows a tensor map, the whole [Cp][144] gradient segment as one TMA copy
// (zero filled outside the image) — per-channel copies issued by a warp
// against one mbarrier cost ~3 us per unit.
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "tc.cuh"
#include "gencat.cuh"
#include "tmap.cuh"

namespace ddpm {
namespace {

using namespace gencat;

// Every wait of this kernel lets a waiting thread stay suspended (not issuing)
// for up to this long, woken by the phase's completion: the epilogue warps
// that wait on the MMAs then leave their issue slots to the others (2.6 %
// faster at B=64 bf16 than the spinning waits, same results).
constexpr uint32_t kHintNs = 100000;

// Staged pixels per row segment: 128 plus seg_off(K) on each side (8 for K <= 3,
// whose dilation halos reach 8 pixels; 16 for K = 5, halos up to 16).
__host__ __device__ constexpr int seg_off(int ks) { return ks <= 3 ? 8 : 16; }
__host__ __device__ constexpr int seg_px(int ks) { return kTileM + 2 * seg_off(ks); }

template <typename T, int KS, bool kStaged = false>
struct BxCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  static constexpr int kParts = kSplit ? 2 : 1;
  // units in flight (16-bit staged: a third unit buffer fits and keeps one
  // more unit's copies outstanding)
  static constexpr int kUnitBufs = (kStaged && !kSplit) ? 3 : 2;
  // FP32 at K = 5: 160-pixel segments and 75 bias rows leave room for two
  static constexpr int kWStages = kSplit ? (KS >= 5 ? 2 : 4) : 6;
  static constexpr int kSeg = seg_px(KS);
  static constexpr int kOff = seg_off(KS);
  static constexpr bool kBiasInGemm = !kSplit;
  static constexpr int kIssuers = 2;        // MMA issuer warps (alternate chunks)
  static constexpr int kFirstProducerWarp = 1 + kIssuers;
  static constexpr int kProducers = kStaged ? 32 : 256;
  static constexpr int kFirstEpiWarp = kFirstProducerWarp + kProducers / 32;
  // epilogue warpgroups: the staged variant (one light producer warp) has the
  // registers for four, one 16-channel block each, which hides twice the TMEM
  // and shared-memory load latency of two warpgroups with two blocks each
  static constexpr int kEpiWG = kStaged ? 4 : 2;
  static constexpr int kBlkPerWG = 4 / kEpiWG;
  static constexpr int kThreads = 32 * (kFirstEpiWarp + 4 * kEpiWG);
};

struct BxSmem {
  uint32_t reg, gs, w, bias, bars, total;
  uint32_t reg_part, reg_bytes, g_bytes, w_bytes;
};

// One unit buffer = the y row segment (both parts) + the gradient row segment.
// C=64: fp32 2x36 + 2x36 + 4x16 + 7 KB = 215 KB; bf16 2x23 + 2x18 + 6x10 KB = 143 KB
// (3 unit buffers when staged: 184 KB). K = 5: fp32 2x40 + 2x40 + 2x16 + 19 KB
// = 211 KB; bf16 staged 3x25 + 3x20 + 6x10 KB = 196 KB.
template <typename T, int KS, bool kStaged>
__host__ __device__ inline BxSmem bx_smem_layout(int Cp, int Ck, int C) {
  using Cfg = BxCfg<T, KS, kStaged>;
  constexpr int kSeg = Cfg::kSeg;
  BxSmem L;
  L.reg_part = (uint32_t)Ck * kSeg * 2;
  L.reg_bytes = Cfg::kParts * L.reg_part;
  L.g_bytes = (uint32_t)Cp * kSeg * sizeof(T);
  L.w_bytes = (uint32_t)Cfg::kParts * Cp * Ck * 2;
  L.reg = 0;
  // 1024-byte aligned: a 128-byte-swizzled TMA destination (channel-last grad_out)
  L.gs = (L.reg + Cfg::kUnitBufs * L.reg_bytes + 1023u) / 1024u * 1024u;
  L.w = L.gs + Cfg::kUnitBufs * L.g_bytes;
  L.bias = L.w + Cfg::kWStages * L.w_bytes;
  L.bars = L.bias + (Cfg::kBiasInGemm ? 0u : (uint32_t)(3 * KS * KS * Cp * 4));
  L.total = L.bars + 8 * (3 * Cfg::kUnitBufs + 2 * Cfg::kWStages + 2 * 8);
  return L;
}

struct BxParams {
  const void* y;
  const void* wpack;  // "bx" image
  const void* bias;
  const void* gout;
  void* gx;
  int N, C, H, W, Cp, Ck;
  int d[3];
  int tiles_w, num_tiles;
  const uint8_t* staged;  // staged y, or null (stage from y)
  StageLayout sl;
  CUtensorMap gmap;       // grad_out {W, H, 4C, N}, box {kSeg, 1, Cp, 1} (staged path)
  CUtensorMap ymap;       // y-plane row segment, box of kSeg/16 16-px blocks x Ck/8 groups
  int g_tma;              // gmap is valid
  int y_tma;              // ymap is valid
  // grad_out channel-last [N][H][W][4C] (16-bit, C == 64, staged): gmap is then
  // {C, 4, W, H, N}, box {64, 1, kSeg, 1, 1} with 128-byte swizzle, landing as
  // [kSeg px][64 channels], 16-byte chunk j of pixel row r at chunk j ^ (r & 7)
  int g_nhwc;
  int* status;
};

// Gradient row segment g_b[:, hr, w0-OFF .. w0-OFF+SEG-1] of one unit into
// `gs` ([Cp][SEG], I/O dtype): one channel per thread (threads tid, tid + nthr,
// ...), 1-D bulk copies counted on `bar` when every row start is 16-byte
// aligned, zero outside the image.
template <typename T, int SEG, int OFF>
__device__ __forceinline__ void stage_grad_rows(T* gs, const T* gout, uint64_t* bar, int tid,
                                                int nthr, int n, int b, int hr, int w0, int C,
                                                int Cp, int H, int W, size_t P, uint32_t g_bytes,
                                                bool g_bulk) {
  constexpr int kSeg = SEG;
  const int lo = w0 - OFF < 0 ? 0 : w0 - OFF;
  const int hi = w0 + kSeg - OFF > W ? W : w0 + kSeg - OFF;
  const bool row_ok = hr >= 0 && hr < H;
  if (!row_ok) {
    // the whole segment is outside the image: vector zero stores over all threads
    uint4* z = reinterpret_cast<uint4*>(gs);
    for (int i = tid; i < (int)(g_bytes / 16); i += nthr) z[i] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  for (int c = tid; c < Cp; c += nthr) {
    T* dst = gs + (size_t)c * kSeg;
    const T* src = gout + ((size_t)n * 4 * C + (size_t)(b + 1) * C + c) * P + (size_t)hr * W;
    if (c < C && g_bulk) {
      for (int x = 0; x < lo - (w0 - OFF); ++x) dst[x] = T(0.f);
      for (int x = hi - (w0 - OFF); x < kSeg; ++x) dst[x] = T(0.f);
      const uint32_t bytes = (uint32_t)(hi - lo) * sizeof(T);
      tc::mbar_expect_tx(bar, bytes);  // before the copy can complete
      tc::bulk_g2s(dst + (lo - (w0 - OFF)), src + lo, bytes, bar);
    } else {
      for (int x = 0; x < kSeg; ++x) {
        const int col = w0 - OFF + x;
        dst[x] = (c < C && col >= 0 && col < W) ? src[col] : T(0.f);
      }
    }
  }
}

template <typename T, int KS, bool kStaged, bool kNhwc = false>
__global__ void __launch_bounds__(BxCfg<T, KS, kStaged>::kThreads, 1)
gencat_bwd_x_kernel(const __grid_constant__ BxParams p) {
  using Cfg = BxCfg<T, KS, kStaged>;
  using Op = typename IoTraits<T>::Op;
  constexpr int S = Cfg::kWStages;
  constexpr int NU = Cfg::kUnitBufs;
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  constexpr int kSeg = Cfg::kSeg;
  constexpr int kOff = Cfg::kOff;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int C = p.C, Cp = p.Cp, Ck = p.Ck, H = p.H, W = p.W;
  const size_t P = (size_t)H * W;
  const BxSmem L = bx_smem_layout<T, KS, kStaged>(Cp, Ck, C);
  constexpr int NB = 8;  // TMEM chunk accumulators: 512 / Cp >= 8 for every Cp <= 64
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* u_full = bars;              // [NU] producers (128 arrivals) + gradient bytes
  uint64_t* r_empty = bars + NU;        // [NU] MMAs done with the y segment
  uint64_t* g_empty = bars + 2 * NU;    // [NU] epilogue done with the gradient segment
  uint64_t* w_full = bars + 3 * NU;     // [S]
  uint64_t* w_empty = w_full + S;       // [S]
  uint64_t* t_full = w_empty + S;       // [NB]
  uint64_t* t_empty = t_full + NB;      // [NB]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < NU; ++i) {
      tc::mbar_init(&u_full[i], Cfg::kProducers);
      tc::mbar_init(&r_empty[i], Cfg::kIssuers);
      tc::mbar_init(&g_empty[i], 128 * Cfg::kEpiWG);
    }
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&w_full[i], 1);
      tc::mbar_init(&w_empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      tc::mbar_init(&t_full[i], 1);
      tc::mbar_init(&t_empty[i], 128 * Cfg::kEpiWG);
    }
    tc::fence_mbar_init();
    abort_s = 0;
  }
  if constexpr (!Cfg::kBiasInGemm) {
    float* bias_s = reinterpret_cast<float*>(smem + L.bias);
    const T* bias = static_cast<const T*>(p.bias);
    // bias_s[(b*K^2 + tap)*Cp + c]
    for (int i = threadIdx.x; i < 3 * KK * Cp; i += blockDim.x) {
      const int q = i / Cp, c = i % Cp;
      const int b = q / KK, tap = q % KK;
      bias_s[i] = c < C ? to_f32<T>(bias[(b * C + c) * KK + tap]) : 0.f;
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  volatile int* abort_flag = &abort_s;
  constexpr int kUnits = 3 * KS;  // (branch, kernel row) units per tile

  if (warp == 0) {
    // ---- weight producer: 3*K^2 chunks per tile, in (b, ki, kj) order -----
    if (lane == 0) {
      const uint8_t* wsrc = static_cast<const uint8_t*>(p.wpack);
      uint32_t wq = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        for (int q = 0; q < 3 * KK; ++q, ++wq) {
          const int s = wq % S;
          if (!tc::mbar_wait(&w_empty[s], ((wq / S) & 1) ^ 1, abort_flag, kWaitNs, kHintNs)) {
            fail(abort_flag, p.status, 20);
            goto done;
          }
          tc::mbar_arrive_expect_tx(&w_full[s], L.w_bytes);
          tc::bulk_g2s(smem + L.w + s * L.w_bytes, wsrc + (size_t)q * L.w_bytes, L.w_bytes,
                       &w_full[s]);
        }
      }
    }
  } else if (warp < Cfg::kFirstProducerWarp) {
    // ---- MMA issuers: warp 1 + i issues the chunks with index % 2 == i ------
    if (lane == 0) {
      const uint32_t me = warp - 1;
      const uint32_t idesc = tc::idesc_f16(kTileM, Cp, IoTraits<T>::kBf16, false, false);
      constexpr uint32_t a_lbo = kSeg * 16;     // channel-group stride of a y segment
      const uint32_t b_lbo = Cp * 16;           // channel-group stride of a weight chunk
      constexpr uint64_t a_step = (2 * a_lbo) >> 4;  // descriptor advance per K step
      const uint64_t b_step = (2 * b_lbo) >> 4;
      const uint64_t a_lo = L.reg_part >> 4;     // hi -> lo part offsets
      const uint64_t b_lo = (Cp * Ck * 2) >> 4;
      const int nks = Ck / 16;
      uint32_t wq = 0, uq = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        for (int u = 0; u < kUnits; ++u, ++uq) {
          const int b = u / KS;
          const int ub = uq % NU;
          if (!tc::mbar_wait(&u_full[ub], (uq / NU) & 1, abort_flag, kWaitNs, kHintNs)) {
            fail(abort_flag, p.status, 21);
            goto done;
          }
          tc::tc_fence_after();
          const uint64_t a_base =
              tc::smem_desc(tc::smem_u32(smem + L.reg + ub * L.reg_bytes), a_lbo, 128);
          const int d = p.d[b];
          for (int kj = 0; kj < KS; ++kj, ++wq) {
            if ((wq & 1u) != me) continue;
            const int s = wq % S;
            const int j = wq % NB;  // chunk counter == weight counter
            if (!tc::mbar_wait(&w_full[s], (wq / S) & 1, abort_flag, kWaitNs, kHintNs) ||
                !tc::mbar_wait(&t_empty[j], ((wq / NB) & 1) ^ 1, abort_flag, kWaitNs, kHintNs)) {
              fail(abort_flag, p.status, 22);
              goto done;
            }
            tc::tc_fence_after();
            const int dx = (kj - r) * d;
            // window: pixels (kOff - dx) .. (kOff - dx) + 127 of the staged segment
            const uint64_t ad = a_base + (uint64_t)(kOff - dx);
            const uint64_t bd =
                tc::smem_desc(tc::smem_u32(smem + L.w + s * L.w_bytes), b_lbo, 128);
            const uint32_t dt = tmem_base + j * Cp;
            for (int ks = 0; ks < nks; ++ks) {
              tc::mma_f16(dt, ad + ks * a_step, bd + ks * b_step, idesc, ks > 0 ? 1u : 0u);
              if constexpr (Cfg::kSplit) {
                tc::mma_f16(dt, ad + a_lo + ks * a_step, bd + ks * b_step, idesc, 1u);
                tc::mma_f16(dt, ad + ks * a_step, bd + b_lo + ks * b_step, idesc, 1u);
              }
            }
            tc::mma_commit(&w_empty[s]);
            tc::mma_commit(&t_full[j]);
          }
          tc::mma_commit(&r_empty[ub]);
        }
      }
      // teardown frees TMEM: wait for this thread's last MMAs
      tc::mma_commit(&r_empty[uq % NU]);
      if (!tc::mbar_wait(&r_empty[uq % NU], (uq / NU) & 1, abort_flag, kWaitNs, kHintNs))
        fail(abort_flag, p.status, 27);
    }
  } else if (warp < Cfg::kFirstEpiWarp) {
    // ---- unit producers ---------------------------------------------------------
    const int pt = threadIdx.x - 32 * Cfg::kFirstProducerWarp;
    const T* y = static_cast<const T*>(p.y);
    const T* gout = static_cast<const T*>(p.gout);
    const int ones_c = Cfg::kBiasInGemm ? C : -1;
    // gradient rows can be bulk-copied when every row start is 16-byte aligned
    const bool g_bulk = ((size_t)W * sizeof(T)) % 16 == 0 &&
                        (reinterpret_cast<uintptr_t>(gout) & 15u) == 0;
    const int items = (Ck / 8) * (kSeg / 8);  // (channel group, 8-pixel block)
    uint32_t uq = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
      const int per_img = H * p.tiles_w;
      const int n = tile / per_img;
      const int h = (tile % per_img) / p.tiles_w;
      const int w0 = (tile % p.tiles_w) * kTileM;
      bool failed = false;
      for (int u = 0; u < kUnits; ++u, ++uq) {
        const int b = u / KS, ki = u % KS;
        const int d = p.d[b];
        const int hr = h - (ki - r) * d;  // image row of this unit
        const int ub = uq % NU;
        uint8_t* reg = smem + L.reg + ub * L.reg_bytes;
        T* gs = reinterpret_cast<T*>(smem + L.gs + ub * L.g_bytes);
        if constexpr (kStaged) {
          // staged y: one bulk copy per (part, channel group); plane row hr + ph,
          // plane columns w0 .. w0+kSeg-1 = image columns w0-kOff .. (the
          // plane's column padding equals kOff)
          if (!warp_wait(&r_empty[ub], ((uq / NU) & 1) ^ 1, abort_flag, kHintNs) ||
              !warp_wait(&g_empty[ub], ((uq / NU) & 1) ^ 1, abort_flag, kHintNs)) {
            fail(abort_flag, p.status, 23);
            failed = true;
            break;
          }
          const int ng = Ck / 8;
          if (pt == 0) {
            // one arrival carries the unit's whole byte count, then the copies
            const uint32_t ybytes = (uint32_t)(ng * Cfg::kParts) * kSeg * 16;
            tc::mbar_arrive_expect_tx(&u_full[ub], ybytes + (p.g_tma ? L.g_bytes : 0u));
            if (p.y_tma) {
              // one box per part (the 1-D copies below cost ~60 ns each to issue)
#pragma unroll
              for (int part = 0; part < Cfg::kParts; ++part)
                tc::tma_load_5d(reg + part * L.reg_part, &p.ymap, 0, w0 / 16, hr + p.sl.ph, 0,
                                part * p.N + n, &u_full[ub]);
            } else {
              for (int k = 0; k < ng * Cfg::kParts; ++k) {
                const int part = k / ng, kg = k - part * ng;
                const uint8_t* src = p.staged + p.sl.row_offset(part, n, hr + p.sl.ph, kg, w0);
                tc::bulk_g2s(reg + part * L.reg_part + kg * kSeg * 16, src, kSeg * 16,
                             &u_full[ub]);
              }
            }
            if (p.g_tma) {
              if constexpr (kNhwc) {
                // one 128-byte-wide box per 128 bytes of channels (FP32: two)
                constexpr int kBoxes = (int)sizeof(T) / 2;
#pragma unroll
                for (int bx = 0; bx < kBoxes; ++bx)
                  tc::tma_load_5d(reinterpret_cast<uint8_t*>(gs) + bx * kSeg * 128, &p.gmap,
                                  bx * (64 / kBoxes), b + 1, w0 - kOff, hr, n, &u_full[ub]);
              } else {
                tc::tma_load_4d(gs, &p.gmap, w0 - kOff, hr, (b + 1) * C, n, &u_full[ub]);
              }
            }
          }
          if (!p.g_tma)
            stage_grad_rows<T, kSeg, kOff>(gs, gout, &u_full[ub], pt, Cfg::kProducers, n, b, hr,
                                           w0, C, Cp, H, W, P, L.g_bytes, g_bulk);
          __syncwarp();
          if (pt != 0) tc::mbar_arrive(&u_full[ub]);
        } else {
          bool waited = false;
          for (int base = 0; base < items; base += Cfg::kProducers) {
            // (1) this thread's y item: 8 channels x 8 pixels, loaded before any wait
            const int item = base + pt;
            const int jb = item % (kSeg / 8);
            const int kg = item / (kSeg / 8);
            Raw8<T> v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int c = kg * 8 + e;
              if (item < items && c < C)
                v[e] = load_raw8<T>(y + ((size_t)n * C + c) * P, H, W, hr, w0 - kOff + jb * 8);
              else if (c == ones_c)
                v[e].ones();
              else
                v[e].zero();
            }
            if (!waited) {
              if (!warp_wait(&r_empty[ub], ((uq / NU) & 1) ^ 1, abort_flag, kHintNs) ||
                  !warp_wait(&g_empty[ub], ((uq / NU) & 1) ^ 1, abort_flag, kHintNs)) {
                fail(abort_flag, p.status, 23);
                failed = true;
                break;
              }
              waited = true;
              // (2) gradient row segment, one channel per thread: columns w0-kOff ..
              stage_grad_rows<T, kSeg, kOff>(gs, gout, &u_full[ub], pt, Cfg::kProducers, n, b,
                                             hr, w0, C, Cp, H, W, P, L.g_bytes, g_bulk);
            }
            if (item < items)
              store_transposed<T, Op, Cfg::kSplit>(reg + (kg * kSeg + jb * 8) * 16, L.reg_part, v);
          }
          if (failed) break;
          tc::fence_proxy_async_smem();
        }
        if (failed) break;
        if constexpr (!kStaged) tc::mbar_arrive(&u_full[ub]);
      }
      if (failed) break;
    }
  } else {
    // ---- epilogue: warpgroup wg owns channel blocks wg, wg + kEpiWG --------
    const int ew = warp - Cfg::kFirstEpiWarp;
    const int wg = ew >> 2;
    const int quad = warp & 3;
    const int m = quad * 32 + lane;
    const T* gout = static_cast<const T*>(p.gout);
    T* gx = static_cast<T*>(p.gx);
    const float* bias_s = reinterpret_cast<const float*>(smem + L.bias);
    const int nblk = Cp / 16;
    uint32_t tq = 0, uq = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int per_img = H * p.tiles_w;
      const int n = tile / per_img;
      const int h = (tile % per_img) / p.tiles_w;
      const int w = (tile % p.tiles_w) * kTileM + m;
      const bool px_ok = w < W;
      const T* gn = gout + (size_t)n * 4 * C * P;
      float acc[Cfg::kBlkPerWG][16];
      unsigned long long acc2[8];    // staged path: channel pairs (2c, 2c+1) of acc[0]
#pragma unroll
      for (int i = 0; i < 8; ++i) acc2[i] = 0ull;
      float g0[Cfg::kBlkPerWG][16];  // x-branch gradient
      T g0raw[16];  // staged: loaded during the last unit, converted at the tile end
#pragma unroll
      for (int bi = 0; bi < Cfg::kBlkPerWG; ++bi)
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[bi][i] = 0.f;
      bool failed = false;
      for (int u = 0; u < kUnits && !failed; ++u, ++uq) {
        const int b = u / KS, ki = u % KS;
        const int d = p.d[b];
        const int ub = uq % NU;
        if constexpr (kStaged) {
          // global loads issued here land while the last unit is computed (at
          // the tile end they took ~3 us under the kernel's own copy traffic)
          // (kept in the I/O type: a conversion right after the load waited for it)
          if (u == kUnits - 1) {
            if constexpr (kNhwc) {
              // channel-last: the pixel's 16 channels are 16-byte vectors
              constexpr int kVecs = 16 * (int)sizeof(T) / 16;
              const uint4* g0v = reinterpret_cast<const uint4*>(
                  gout + (((size_t)n * H + h) * W + w) * 4 * C + wg * 16);
#pragma unroll
              for (int k = 0; k < kVecs; ++k) {
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                if (px_ok && wg < nblk) v = __ldg(g0v + k);
                memcpy(reinterpret_cast<uint8_t*>(g0raw) + 16 * k, &v, 16);
              }
            } else {
              const T* g0p = gn + (size_t)(wg * 16) * P + (size_t)h * W + w;
#pragma unroll
              for (int cl = 0; cl < 16; ++cl)
                g0raw[cl] =
                    (px_ok && wg < nblk && wg * 16 + cl < C) ? __ldg(g0p + cl * P) : T(0.f);
            }
          }
        }
        if (!warp_wait(&u_full[ub], (uq / NU) & 1, abort_flag, kHintNs)) {
          fail(abort_flag, p.status, 25);
          failed = true;
          break;
        }
        const T* gs = reinterpret_cast<const T*>(smem + L.gs + ub * L.g_bytes);
        if constexpr (kStaged) {
          // One channel block per warpgroup. The next chunk's wait and TMEM load
          // are issued before the current chunk is computed, so each chunk's
          // wait / load latency overlaps the previous chunk's math. The staged
          // gradient segment is zero outside the image.
          static_assert(Cfg::kBlkPerWG == 1, "staged epilogue: one block per warpgroup");
          const bool blk_ok = wg < nblk;
          const T* gcol = gs + (size_t)(wg * 16) * kSeg + (m + kOff);
          const uint32_t tcol = tmem_base + ((uint32_t)(quad * 32) << 16) + wg * 16;
          float dv[2][16];
          if (!warp_wait(&t_full[tq % NB], (tq / NB) & 1, abort_flag, kHintNs)) {
            fail(abort_flag, p.status, 24);
            failed = true;
            break;
          }
          tc::tc_fence_after();
          if (blk_ok) tc::tmem_ld16(tcol + (tq % NB) * Cp, dv[0]);
#pragma unroll
          for (int kj = 0; kj < KS; ++kj, ++tq) {
            const int cur = kj & 1;
            tc::tmem_ld_wait();
            if (kj + 1 < KS) {
              const uint32_t tn = tq + 1;
              if (!warp_wait(&t_full[tn % NB], (tn / NB) & 1, abort_flag, kHintNs)) {
                fail(abort_flag, p.status, 24);
                failed = true;
                break;
              }
              tc::tc_fence_after();
              if (blk_ok) tc::tmem_ld16(tcol + (tn % NB) * Cp, dv[cur ^ 1]);
            }
            if constexpr (sizeof(T) == 2) {
              if (blk_ok) {
                // 16-bit: each word of two gradient values meets the matching
                // pair of rounded taps in two mixed-precision FMAs (no
                // conversion of either to FP32)
                uint32_t gw[8];
                if constexpr (kNhwc) {
                  // channel-last: the block's channels are chunks 2wg and 2wg+1
                  // (8 each) of swizzled pixel row m + kOff - dx (chunk j of
                  // row r at j ^ (r & 7))
                  const int pr = m + kOff - (kj - r) * d;
                  const uint8_t* row = reinterpret_cast<const uint8_t*>(gs) + pr * 128;
                  const uint4 v0 =
                      *reinterpret_cast<const uint4*>(row + (((2 * wg) ^ (pr & 7)) * 16));
                  const uint4 v1 =
                      *reinterpret_cast<const uint4*>(row + (((2 * wg + 1) ^ (pr & 7)) * 16));
                  gw[0] = v0.x; gw[1] = v0.y; gw[2] = v0.z; gw[3] = v0.w;
                  gw[4] = v1.x; gw[5] = v1.y; gw[6] = v1.z; gw[7] = v1.w;
                } else {
                  // [Cp][kSeg] segment: channel pairs of column m + kOff - dx
                  const int dx = (kj - r) * d;
#pragma unroll
                  for (int i = 0; i < 8; ++i)
                    gw[i] = pack_raw2<T>(gcol[(2 * i) * kSeg - dx], gcol[(2 * i + 1) * kSeg - dx]);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  acc2[i] = fma_io2<Op>(cvt2<Op>(dv[cur][2 * i], dv[cur][2 * i + 1]), gw[i], acc2[i]);
              }
            } else if (blk_ok) {
              const int dx = (kj - r) * d;
              float gv[16];
              // FP32 (16-bit takes the branch above)
              if constexpr (kNhwc) {
                // pixel row m + kOff - dx
                // of the swizzled [kSeg][128 bytes] segments; box wg / 2 holds
                // channels 32 (wg / 2) .. +31, the block's 16 channels are its
                // chunks 4 (wg % 2) .. +3, chunk j of row r at j ^ (r & 7)
                const int pr = m + kOff - dx;
                const uint8_t* row = reinterpret_cast<const uint8_t*>(gs) +
                                     (wg >> 1) * kSeg * 128 + pr * 128;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const float4 v = *reinterpret_cast<const float4*>(
                      row + ((((wg & 1) * 4 + k) ^ (pr & 7)) * 16));
                  gv[4 * k] = v.x;
                  gv[4 * k + 1] = v.y;
                  gv[4 * k + 2] = v.z;
                  gv[4 * k + 3] = v.w;
                }
              } else {
#pragma unroll
                for (int cl = 0; cl < 16; ++cl) gv[cl] = to_f32<T>(gcol[cl * kSeg - dx]);
              }
              if constexpr (!Cfg::kBiasInGemm) {
                const float* bs = bias_s + (b * KK + ki * KS + kj) * Cp + wg * 16;
#pragma unroll
                for (int cl = 0; cl < 16; ++cl) dv[cur][cl] += bs[cl];
              }
              // taps rounded to the I/O type a pair per conversion, then two
              // FMAs per instruction (same products and sums as fmaf per value)
#pragma unroll
              for (int i = 0; i < 8; ++i)
                acc2[i] = f2_fma(tap_pair<T>(dv[cur][2 * i], dv[cur][2 * i + 1]),
                                 f2_pack(gv[2 * i], gv[2 * i + 1]), acc2[i]);
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&t_empty[tq % NB]);
          }
        } else {
          for (int kj = 0; kj < KS; ++kj, ++tq) {
            const int tap = ki * KS + kj;
            const int dx = (kj - r) * d;
            // g_b at (h - dy, w - dx): staged column m + kOff - dx (zero off-image)
            const bool ok = px_ok && (unsigned)(w - dx) < (unsigned)W;
            const int j = tq % NB;
            if (!warp_wait(&t_full[j], (tq / NB) & 1, abort_flag, kHintNs)) {
              fail(abort_flag, p.status, 24);
              failed = true;
              break;
            }
            tc::tc_fence_after();
            // 96-register budget: one channel block at a time
#pragma unroll
            for (int bi = 0; bi < Cfg::kBlkPerWG; ++bi) {
              const int blk = wg + Cfg::kEpiWG * bi;
              if (blk >= nblk) break;
              float dv1[16];
              tc::tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + j * Cp + blk * 16, dv1);
              float gv1[16];
              const T* gcol = gs + (size_t)(blk * 16) * kSeg + (m + kOff - dx);
#pragma unroll
              for (int cl = 0; cl < 16; ++cl) gv1[cl] = ok ? to_f32<T>(gcol[cl * kSeg]) : 0.f;
              tc::tmem_ld_wait();
              if constexpr (!Cfg::kBiasInGemm) {
                const float* bs = bias_s + (b * KK + tap) * Cp + blk * 16;
#pragma unroll
                for (int cl = 0; cl < 16; ++cl) dv1[cl] += bs[cl];
              }
              round_taps<T>(dv1);
#pragma unroll
              for (int cl = 0; cl < 16; ++cl) acc[bi][cl] = fmaf(dv1[cl], gv1[cl], acc[bi][cl]);
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&t_empty[j]);
          }
        }
        if (!failed) tc::mbar_arrive(&g_empty[ub]);
      }
      if (failed) break;
      if (px_ok) {
        // all loads of the x-branch gradient before the first store (gx may
        // alias nothing, but the compiler cannot know; interleaved, every load
        // waited for the previous store: 32 serial load latencies per tile)
        const size_t q = (size_t)h * W + w;
        if constexpr (kStaged) {
#pragma unroll
          for (int cl = 0; cl < 16; ++cl) g0[0][cl] = to_f32<T>(g0raw[cl]);
#pragma unroll
          for (int i = 0; i < 8; ++i) f2_unpack(acc2[i], acc[0][2 * i], acc[0][2 * i + 1]);
        } else {
#pragma unroll
          for (int bi = 0; bi < Cfg::kBlkPerWG; ++bi) {
            const int blk = wg + Cfg::kEpiWG * bi;
#pragma unroll
            for (int cl = 0; cl < 16; ++cl) {
              const int c = blk * 16 + cl;
              g0[bi][cl] = (blk < nblk && c < C) ? to_f32<T>(__ldg(gn + (size_t)c * P + q)) : 0.f;
            }
          }
        }
#pragma unroll
        for (int bi = 0; bi < Cfg::kBlkPerWG; ++bi) {
          const int blk = wg + Cfg::kEpiWG * bi;
          if (blk >= nblk) break;
#pragma unroll
          for (int cl = 0; cl < 16; ++cl) {
            const int c = blk * 16 + cl;
            if (c < C) gx[((size_t)n * C + c) * P + q] = from_f32<T>(acc[bi][cl] + g0[bi][cl]);
          }
        }
      }
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

template <typename T, int KS, bool kStaged, bool kNhwc = false>
int launch_k(const BxParams& prm, cudaStream_t st) {
  using Cfg = BxCfg<T, KS, kStaged>;
  const BxSmem L = bx_smem_layout<T, KS, kStaged>(prm.Cp, prm.Ck, prm.C);
  auto fn = gencat_bwd_x_kernel<T, KS, kStaged, kNhwc>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  const int grid = prm.num_tiles < num_sms() ? prm.num_tiles : num_sms();
  fn<<<grid, Cfg::kThreads, L.total, st>>>(prm);
  DDPM_CHECK_LAUNCH("gencat_bwd_x_kernel");
  return DDPM_OK;
}

template <typename T, int KS>
int launch(const BxParams& prm, cudaStream_t st) {
  if (prm.g_nhwc) return launch_k<T, KS, true, true>(prm, st);
  if (prm.staged != nullptr) return launch_k<T, KS, true>(prm, st);
  return launch_k<T, KS, false>(prm, st);
}

template <typename T>
int dispatch(int ks, const BxParams& prm, cudaStream_t st) {
  switch (ks) {
    case 1: return launch<T, 1>(prm, st);
    case 3: return launch<T, 3>(prm, st);
    case 5: return launch<T, 5>(prm, st);
  }
  return set_error(DDPM_ERR_UNSUPPORTED, "fused generator: kernel_size %d not supported", ks);
}

}  // namespace

// `staged`: staged operands (gencat::stage; the y plane is used) or null to
// stage the operand from y itself.
int gencat_bwd_x(const void* y, const void* staged, size_t staged_bytes, const void* wpack,
                 const void* bias, const void* gout, void* gx, int n, int c, int h, int w, int ks,
                 int d0, int d1, int d2, int dt, cudaStream_t st, int g_nhwc) {
  int rc = gencat::check_shape(n, c, h, w, ks, d0, d1, d2, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG((y || staged) && wpack && bias && gout && gx, "null pointer");
  if (g_nhwc && (c != 64 || staged == nullptr))
    return set_error(DDPM_ERR_UNSUPPORTED,
                     "a channel-last grad_out needs C == 64 and staged operands");
  const gencat::PackLayout pl = gencat::PackLayout::make(c, ks, dt);
  const int kSegPx = seg_px(ks);
  BxParams prm{};
  prm.y = y;
  prm.wpack = static_cast<const uint8_t*>(wpack) + pl.bx_offset();
  prm.bias = bias;
  prm.gout = gout;
  prm.gx = gx;
  prm.N = n;
  prm.C = c;
  prm.H = h;
  prm.W = w;
  prm.Cp = pl.Cp;
  prm.Ck = pl.Ck;
  prm.d[0] = d0;
  prm.d[1] = d1;
  prm.d[2] = d2;
  prm.tiles_w = (w + gencat::kTileM - 1) / gencat::kTileM;
  prm.num_tiles = n * h * prm.tiles_w;
  prm.staged = static_cast<const uint8_t*>(staged);
  prm.sl = gencat::StageLayout::make(n, c, h, w, ks, d0, d1, d2, dt);
  if (staged != nullptr) {
    if (staged_bytes < prm.sl.y_bytes())
      return set_error(DDPM_ERR_WORKSPACE, "staged y too small (%zu < %zu)", staged_bytes,
                       prm.sl.y_bytes());
    DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(staged) & 15u) == 0,
                   "staged y must be 16-byte aligned");
    prm.y_tma = gencat::encode_stage_segment_map(&prm.ymap, pl.Ck / 8, prm.staged, prm.sl,
                                                 kSegPx / 16)
                    ? 1
                    : 0;
    // gradient segments by TMA when the row pitch and base allow a tensor map
    const int es = dtype_size(dt);
    if (g_nhwc) {
      DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(gout) & 15u) == 0,
                     "grad_out must be 16-byte aligned");
      const CUtensorMapDataType ty = dt == DDPM_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                     : dt == DDPM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
      const uint64_t dims[5] = {(uint64_t)c, 4, (uint64_t)w, (uint64_t)h, (uint64_t)n};
      const uint64_t strides[4] = {(uint64_t)c * es, (uint64_t)4 * c * es,
                                   (uint64_t)4 * c * w * es, (uint64_t)4 * c * w * h * es};
      // 128 bytes of channels per box (the 128-byte swizzle span): 64 16-bit
      // or 32 FP32 channels; FP32 takes two boxes per unit
      const uint32_t box[5] = {(uint32_t)(128 / es), 1, (uint32_t)kSegPx, 1, 1};
      if (encode_tmap(&prm.gmap, ty, 5, gout, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) !=
          DDPM_OK)
        return DDPM_ERR_CUDA;  // the message is set
      prm.g_tma = 1;
      prm.g_nhwc = 1;
    } else if (((size_t)w * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(gout) & 15u) == 0) {
      const CUtensorMapDataType ty = dt == DDPM_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                     : dt == DDPM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
      const uint64_t dims[4] = {(uint64_t)w, (uint64_t)h, (uint64_t)4 * c, (uint64_t)n};
      const uint64_t strides[3] = {(uint64_t)w * es, (uint64_t)h * w * es,
                                   (uint64_t)4 * c * h * w * es};
      const uint32_t box[4] = {(uint32_t)kSegPx, 1, (uint32_t)pl.Cp, 1};
      if (encode_tmap(&prm.gmap, ty, 4, gout, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE) ==
          DDPM_OK)
        prm.g_tma = 1;
      else
        clear_error();
    }
  }
  rc = gencat::status_ptr(&prm.status);
  if (rc) return rc;
  switch (dt) {
    case DDPM_BF16: return dispatch<__nv_bfloat16>(ks, prm, st);
    case DDPM_F16: return dispatch<__half>(ks, prm, st);
    case DDPM_F32: return dispatch<float>(ks, prm, st);
  }
  return set_error(DDPM_ERR_INVALID_ARG, "unknown dtype %d", dt);
}

}  // namespace ddpm
