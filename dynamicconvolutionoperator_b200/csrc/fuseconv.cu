// Native 3x3 "fuse" convolution of the DDPM (4C -> C, stride 1, zero pad 1).
// Replaces the cuDNN call `self.fuse(cat_out)` (reference `triton_impl.py:294,
// 392`) and its backward (cuDNN dgrad + wgrad):
//
//   out[o, p]   = bias[o] + sum_{t, i} W[o, i, t] * cat[i, p + off(t)]
//   dcat[i, p]  = sum_{t, o} W[o, i, t] * dout[o, p - off(t)]
//   dW[o, i, t] = sum_p dout[o, p] * cat[i, p + off(t)]     (fuseconv_wgrad.cu)
//   off(t) = (ky - 1, kx - 1), t = ky * 3 + kx, zero outside the image.
//
// Why native: in true FP32 (no TF32) cuDNN runs this convolution on its FFT
// and SIMT paths, ~2 ms of a ~3 ms training step at 256^2 on B200; and for
// 16-bit outputs `nn.Conv2d` adds the bias after the convolution has already
// been rounded, so the output is rounded twice. Here the convolution runs on
// the tensor cores (FP32 via bf16 hi + lo operands, 3 MMAs per step) and the
// bias is added to the FP32 accumulator before the single output rounding.
//
// Forward and data gradient are the same shifted-window GEMM (as in the fused
// generator's dX kernel): a unit is TWO consecutive output rows h0, h0 + 1 of
// 128 pixels (w0 .. w0 + 127); the 4 source rows they need (h0 - 1 .. h0 + 2)
// x 144 columns (w0 - 8 .. w0 + 135) of one channel slab are staged in the
// K-major interleaved operand layout [slab channel/8][row][pixel][8] (one
// 16-byte row = 8 channels of one pixel), so the A operand of tap t for output
// row h0 + mh is a descriptor whose start moves by whole pixel rows. Each tap
// and slab is one M=128 x N x K=slab GEMM per output row; the weight chunk of
// (slab, tap) is shared by both rows. Weights are pre-packed per weight
// version into the exact shared-memory B images and streamed by bulk copies.
//
// Warp roles (14 warps): w0 = TMEM allocator + weight producer, w1 = MMA
// issuer, w2-w5 = slab producers, w6-w13 = two epilogue warpgroups (one per
// output row of the unit).
#include "common.cuh"
#include "tc.cuh"
#include "gencat.cuh"
#include "fuseconv.cuh"
#include "tmap.cuh"

namespace ddpm {
namespace {

using namespace gencat;

constexpr int kSeg = fuseconv::kSeg;
constexpr int kRows = 4;           // staged source rows per unit
constexpr int kMaxRegBufs = 4;
constexpr int kMaxWStages = 16;

struct FcParams {
  const void* src;      // staged tensor: cat (forward) or dout (data gradient)
  const uint8_t* wimg;  // packed B image of this pass
  const void* bias;     // forward only (nullptr for the data gradient)
  void* dst;
  int N, H, W;
  int Csrc;             // channels of src (GEMM K before padding)
  int Cdst;             // channels of dst
  int KC, nslab;        // slab channels, slabs
  int Nn;               // MMA N = dst channels per unit (<= 128)
  int nhalf;            // dst channel blocks of Nn (data gradient: ceil(Cin / 128))
  int tiles_w, hpairs, num_units;
  int reg_bufs, w_stages;
  int row_major;        // staged slab order [row][group][px][8] (else [group][row][px][8])
  int dst_nhwc;         // dst channel-last [N][H][W][Cdst] (Cdst % 16 == 0), else NCHW
  uint32_t reg_part, reg_bytes;
  uint32_t w_chunk;     // bytes per streamed weight chunk (FcCfg::kTapsPerChunk taps)
  uint32_t w_tap;       // bytes of one (slab, tap) B image within a chunk
  int* status;
};

// Tensor map of the staged source planes (separate grid-constant parameter):
// dims {32 x 64-bit (16 px), Wp/16, Hp, G, parts*N}, box {32, 9, 4, KC/8, 1},
// which lands as the slab operand [KC/8][4 rows][144 px][8 channels].
struct FcMaps {
  CUtensorMap smap;
  // row-major slabs (FcParams::row_major): the weight gradient's grad_out
  // planes [n][h][Cout/8][w][8], one map per part (smap = hi, smap_lo = lo),
  // dims {16 x 64-bit (8 px), W/8, Cout/8, H, N}, box {16, 18, KC/8, 4, 1},
  // which lands as [4 rows][KC/8][144 px][8 channels]
  CUtensorMap smap_lo;
};

struct FcSmem {
  uint32_t reg, w, bias, bars, total;
};

__host__ __device__ inline FcSmem fc_smem_layout(const FcParams& p) {
  FcSmem L;
  L.reg = 0;
  L.w = L.reg + p.reg_bufs * p.reg_bytes;
  L.bias = L.w + p.w_stages * p.w_chunk;
  L.bars = L.bias + 128 * 4;
  L.total = L.bars + 8 * (2 * kMaxRegBufs + 2 * kMaxWStages + 4);
  return L;
}

template <typename T, bool kDgrad, bool kStaged = false>
struct FcCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  // K slab: input channels (forward) or output channels (data gradient)
  static constexpr int KC = kDgrad ? (kSplit ? 32 : 64) : (kSplit ? 16 : 32);
  static constexpr int kSteps = KC / 16;
  // staged planes: one warp (one thread issues the TMA boxes)
  static constexpr int kProducers = kStaged ? 32 : 256;
  // taps per streamed weight chunk: the forward streams a slab's 9 tap images
  // (4 KB each) as one chunk, so the issuers wait, and commit, once per slab
  // instead of once per 1-3 MMAs; the data gradient's tap images are 16-32 KB
  static constexpr int kTapsPerChunk = kDgrad ? 1 : 9;
  static constexpr int kItems = (KC / 8) * kRows * (kSeg / 8);  // 8 channels x 8 pixels each
  static constexpr int kItemsMax = sizeof(T) == 4 ? 1 : 2;      // per thread and round
  static constexpr int kRounds = (kItems + kProducers * kItemsMax - 1) / (kProducers * kItemsMax);
  static constexpr int kFirstProducerWarp = 3;
  static constexpr int kFirstEpiWarp = kFirstProducerWarp + kProducers / 32;
  // epilogue warpgroups: the staged variant has the threads for one per output
  // row (half the stores per thread); otherwise one warpgroup drains both rows
  static constexpr int kEpiWG = kStaged ? 2 : 1;
  static constexpr int kThreads = 32 * (kFirstEpiWarp + 4 * kEpiWG);
};

// kDgrad = false: forward (window of tap (ky, kx) for output row h0 + mh starts
// at source row h0 + mh + ky - 1, column + kx - 1); true: data gradient
// (source row h0 + mh - ky + 1, column - kx + 1).
//
// Two MMA issuer warps, one per output row: a tcgen05.mma costs its issuing
// thread ~55 cycles, so with N <= 128 a single issuer would leave the tensor
// pipe idle between instructions. Their inner loops are unrolled over taps
// and K steps with descriptors advanced by constants.
// Sixteen FP32 accumulators -> sixteen consecutive channel-last elements of
// dst (16-byte aligned): FP32 as four 16-byte stores, 16-bit types rounded a
// pair per conversion (round to nearest even, as from_f32) into two.
template <typename T>
__device__ __forceinline__ void store16_cl(T* dst, const float (&v)[16]) {
  if constexpr (sizeof(T) == 4) {
    float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = cvt2<T>(v[2 * i], v[2 * i + 1]);
    uint4* d = reinterpret_cast<uint4*>(dst);
    d[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

template <typename T, bool kDgrad, bool kStaged>
__global__ void __launch_bounds__(FcCfg<T, kDgrad, kStaged>::kThreads, 1)
fuseconv_kernel(const FcParams p, const __grid_constant__ FcMaps maps) {
  using Cfg = FcCfg<T, kDgrad, kStaged>;
  using Op = typename IoTraits<T>::Op;
  constexpr bool kSplit = Cfg::kSplit;
  constexpr int KC = Cfg::KC;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const FcSmem L = fc_smem_layout(p);
  const int NR = p.reg_bufs, S = p.w_stages, Nn = p.Nn;
  const int H = p.H, W = p.W;
  const size_t P = (size_t)H * W;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* r_full = bars;                    // [NR]
  uint64_t* r_empty = bars + kMaxRegBufs;     // [NR]
  uint64_t* w_full = bars + 2 * kMaxRegBufs;  // [S]
  uint64_t* w_empty = w_full + kMaxWStages;   // [S]
  uint64_t* t_full = w_empty + kMaxWStages;   // [2]
  uint64_t* t_empty = t_full + 2;             // [2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < NR; ++i) {
      tc::mbar_init(&r_full[i], Cfg::kProducers);
      tc::mbar_init(&r_empty[i], 2);
    }
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&w_full[i], 1);
      tc::mbar_init(&w_empty[i], 2);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&t_full[i], 2);
      tc::mbar_init(&t_empty[i], 128 * Cfg::kEpiWG);
    }
    tc::fence_mbar_init();
    abort_s = 0;
  }
  {
    float* bias_s = reinterpret_cast<float*>(smem + L.bias);
    const T* bias = static_cast<const T*>(p.bias);
    for (int i = threadIdx.x; i < 128; i += blockDim.x)
      bias_s[i] = (bias != nullptr && i < p.Cdst) ? to_f32<T>(bias[i]) : 0.f;
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  volatile int* abort_flag = &abort_s;
  const int chunks = p.nslab * (9 / Cfg::kTapsPerChunk);  // weight chunks per unit

  if (warp == 0) {
    // ---- weight producer ------------------------------------------------------
    if (lane == 0) {
      uint32_t wq = 0;
      for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
        const int half = u % p.nhalf;
        const uint8_t* base = p.wimg + (size_t)half * chunks * p.w_chunk;
        for (int q = 0; q < chunks; ++q, ++wq) {
          const int s = wq % S;
          if (!tc::mbar_wait(&w_empty[s], ((wq / S) & 1) ^ 1, abort_flag, kWaitNs)) {
            fail(abort_flag, p.status, 60);
            goto done;
          }
          tc::mbar_arrive_expect_tx(&w_full[s], p.w_chunk);
          tc::bulk_g2s(smem + L.w + s * p.w_chunk, base + (size_t)q * p.w_chunk, p.w_chunk,
                       &w_full[s]);
        }
      }
    }
  } else if (warp < Cfg::kFirstProducerWarp) {
    // ---- MMA issuers: warp 1 -> output row h0, warp 2 -> row h0 + 1 ----------
    if (lane == 0) {
      const int mh = warp - 1;
      const uint32_t idesc = tc::idesc_f16(128, Nn, IoTraits<T>::kBf16, false, false);
      // channel-group stride of a slab, and the row stride (16-byte units)
      const uint32_t a_lbo = p.row_major ? kSeg * 16 : kRows * kSeg * 16;
      const int a_row = p.row_major ? (KC / 8) * kSeg : kSeg;
      const uint32_t b_lbo = Nn * 16;                // channel-group stride of a weight chunk
      // descriptor increments (units of 16 bytes)
      const uint64_t a_step = (2 * a_lbo) >> 4;      // one K step (16 channels)
      const uint64_t b_step = (2 * b_lbo) >> 4;
      const uint64_t a_lo = p.reg_part >> 4;          // hi -> lo part of the slab
      const uint64_t b_lo = (Nn * KC * 2) >> 4;       // hi -> lo part of a weight chunk
      uint32_t wq = 0, rq = 0, ti = 0;
      for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++ti) {
        const int tb = ti & 1;
        if (!tc::mbar_wait(&t_empty[tb], ((ti >> 1) & 1) ^ 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 61);
          goto done;
        }
        tc::tc_fence_after();
        const uint32_t d = tmem_base + tb * 256 + mh * 128;
        for (int sl = 0; sl < p.nslab; ++sl, ++rq) {
          const int rb = rq % NR;
          if (!tc::mbar_wait(&r_full[rb], (rq / NR) & 1, abort_flag, kWaitNs)) {
            fail(abort_flag, p.status, 62);
            goto done;
          }
          tc::tc_fence_after();
          const uint64_t a_base =
              tc::smem_desc(tc::smem_u32(smem + L.reg + rb * p.reg_bytes), a_lbo, 128);
          constexpr int TPC = Cfg::kTapsPerChunk;
          const uint64_t b_tap = p.w_tap >> 4;  // descriptor advance per tap image
#pragma unroll
          for (int tcg = 0; tcg < 9 / TPC; ++tcg, ++wq) {
            const int s = wq % S;
            if (!tc::mbar_wait(&w_full[s], (wq / S) & 1, abort_flag, kWaitNs)) {
              fail(abort_flag, p.status, 63);
              goto done;
            }
            tc::tc_fence_after();
            const uint64_t bstage =
                tc::smem_desc(tc::smem_u32(smem + L.w + s * p.w_chunk), b_lbo, 128);
#pragma unroll
            for (int tt = 0; tt < TPC; ++tt) {
              const int t = tcg * TPC + tt;
              const int ky = t / 3, kx = t % 3;
              const int seg = kDgrad ? (mh - ky + 2) : (mh + ky);
              const int col = kDgrad ? (9 - kx) : (7 + kx);
              const uint64_t ad = a_base + (uint64_t)(seg * a_row + col);
              const uint64_t bd = bstage + tt * b_tap;
#pragma unroll
              for (int ks = 0; ks < Cfg::kSteps; ++ks) {
                const uint32_t acc = (sl > 0 || t > 0 || ks > 0) ? 1u : 0u;
                tc::mma_f16(d, ad + ks * a_step, bd + ks * b_step, idesc, acc);
                if constexpr (kSplit) {
                  tc::mma_f16(d, ad + a_lo + ks * a_step, bd + ks * b_step, idesc, 1u);
                  tc::mma_f16(d, ad + ks * a_step, bd + b_lo + ks * b_step, idesc, 1u);
                }
              }
            }
            tc::mma_commit(&w_empty[s]);
          }
          tc::mma_commit(&r_empty[rb]);
        }
        tc::mma_commit(&t_full[tb]);
      }
    }
  } else if (warp < Cfg::kFirstEpiWarp) {
    // ---- slab producers (256 threads) -----------------------------------------
    const int pt = threadIdx.x - 32 * Cfg::kFirstProducerWarp;
    const T* src = static_cast<const T*>(p.src);
    uint32_t rq = 0;
    for (int u = blockIdx.x; u < p.num_units && !*abort_flag; u += gridDim.x) {
      const int v_ = u / p.nhalf;
      const int wt = v_ % p.tiles_w;
      const int hp = (v_ / p.tiles_w) % p.hpairs;
      const int n = v_ / (p.tiles_w * p.hpairs);
      const int h0 = 2 * hp, w0 = wt * 128;
      const T* srcn = src + (size_t)n * p.Csrc * P;
      for (int sl = 0; sl < p.nslab; ++sl, ++rq) {
        const int rb = rq % NR;
        uint8_t* reg = smem + L.reg + rb * p.reg_bytes;
        bool failed = false;
        if constexpr (kStaged) {
          // plane rows h0 .. h0+3 = image rows h0-1 .. h0+2; plane columns
          // w0 .. w0+143 = image columns w0-8 .. w0+135; one box per part
          if (!warp_wait(&r_empty[rb], ((rq / NR) & 1) ^ 1, abort_flag)) {
            fail(abort_flag, p.status, 64);
            break;
          }
          if (pt == 0) {
            tc::mbar_arrive_expect_tx(&r_full[rb], p.reg_bytes);
#pragma unroll
            for (int part = 0; part < (kSplit ? 2 : 1); ++part) {
              if (p.row_major)  // 8-px blocks from w0-8, rows from h0-1 (zero outside)
                tc::tma_load_5d(reg + part * p.reg_part, part ? &maps.smap_lo : &maps.smap, 0,
                                w0 / 8 - 1, sl * (KC / 8), h0 - 1, n, &r_full[rb]);
              else
                tc::tma_load_5d(reg + part * p.reg_part, &maps.smap, 0, w0 / 16, h0,
                                sl * (KC / 8), part * p.N + n, &r_full[rb]);
            }
          } else {
            tc::mbar_arrive(&r_full[rb]);
          }
          continue;
        }
#pragma unroll 1
        for (int round = 0; round < Cfg::kRounds; ++round) {
          const int base = round * Cfg::kProducers * Cfg::kItemsMax;
          // loads first: they do not depend on the buffer being free
          Raw8<T> v[Cfg::kItemsMax][8];
#pragma unroll
          for (int k = 0; k < Cfg::kItemsMax; ++k) {
            const int item = base + k * Cfg::kProducers + pt;
            const int jb = item % (kSeg / 8);
            const int seg = (item / (kSeg / 8)) % kRows;
            const int kg = item / ((kSeg / 8) * kRows);
            const int hr = h0 - 1 + seg;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int c = sl * KC + kg * 8 + e;
              if (item < Cfg::kItems && c < p.Csrc)
                v[k][e] = load_raw8<T>(srcn + (size_t)c * P, H, W, hr, w0 - 8 + jb * 8);
              else
                v[k][e].zero();
            }
          }
          if (round == 0 && !warp_wait(&r_empty[rb], ((rq / NR) & 1) ^ 1, abort_flag)) {
            fail(abort_flag, p.status, 64);
            failed = true;
            break;
          }
#pragma unroll
          for (int k = 0; k < Cfg::kItemsMax; ++k) {
            const int item = base + k * Cfg::kProducers + pt;
            if (item >= Cfg::kItems) continue;
            const int jb = item % (kSeg / 8);
            const int seg = (item / (kSeg / 8)) % kRows;
            const int kg = item / ((kSeg / 8) * kRows);
            const uint32_t off = ((kg * kRows + seg) * kSeg + jb * 8) * 16;
            store_transposed<T, Op, kSplit>(reg + off, p.reg_part, v[k]);
          }
        }
        if (failed) break;
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&r_full[rb]);
      }
    }
  } else {
    // ---- epilogue: warpgroup ewg drains output rows ewg, ewg + kEpiWG ---------
    const int ewg = (warp - Cfg::kFirstEpiWarp) >> 2;
    const int quad = warp & 3;
    const int m = quad * 32 + lane;
    const float* bias_s = reinterpret_cast<const float*>(smem + L.bias);
    T* dst = static_cast<T*>(p.dst);
    uint32_t ti = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++ti) {
      const int half = u % p.nhalf;
      const int v_ = u / p.nhalf;
      const int wt = v_ % p.tiles_w;
      const int hp = (v_ / p.tiles_w) % p.hpairs;
      const int n = v_ / (p.tiles_w * p.hpairs);
      const int w = wt * 128 + m;
      const int tb = ti & 1;
      if (!warp_wait(&t_full[tb], (ti >> 1) & 1, abort_flag)) {
        fail(abort_flag, p.status, 65);
        break;
      }
      tc::tc_fence_after();
      const int c0 = half * Nn;
#pragma unroll 1
      for (int mh = ewg; mh < 2; mh += Cfg::kEpiWG) {
        const int h = 2 * hp + mh;
        const bool ok = h < H && w < W;
        const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + tb * 256 + mh * 128;
        T* out = dst + ((size_t)n * p.Cdst + c0) * P + (size_t)h * W + w;
        // channel-last: the pixel's channels are contiguous, 16 per vector store
        T* out_cl = dst + (((size_t)n * H + h) * W + w) * p.Cdst + c0;
        for (int blk = 0; blk < Nn; blk += 32) {
          float a[2][16];
          tc::tmem_ld16(taddr + blk, a[0]);
          tc::tmem_ld16(taddr + blk + 16, a[1]);
          tc::tmem_ld_wait();
          if (ok && p.dst_nhwc) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int cb = blk + hh * 16;
              if (c0 + cb >= p.Cdst) break;
              if constexpr (!kDgrad) {
#pragma unroll
                for (int e = 0; e < 16; ++e) a[hh][e] += bias_s[cb + e];
              }
              store16_cl<T>(out_cl + cb, a[hh]);
            }
          } else if (ok) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const int c = blk + hh * 16 + e;
                const float bv = kDgrad ? 0.f : bias_s[c];
                if (c0 + c < p.Cdst) out[(size_t)c * P] = from_f32<T>(a[hh][e] + bv);
              }
          }
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&t_empty[tb]);
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

// ------------------------------------------------------------- weight pack ----
// One thread per 16-byte B-operand row (8 K-dimension values).
template <typename T>
__global__ void fuseconv_pack_kernel(const T* __restrict__ w, typename IoTraits<T>::Op* out,
                                     fuseconv::Layout L) {
  using Op = typename IoTraits<T>::Op;
  const long long fwd_rows = (long long)L.fwd_bytes / 16;
  const long long total = (long long)(L.fwd_bytes + L.dg_bytes) / 16;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    int o0, i0, t, part;  // first element; the 8 values run over i (forward) or o (dgrad)
    bool run_i;
    if (idx < fwd_rows) {
      // chunk (slab, tap): [part][KC/8][Np][8]
      const long long per_chunk = (long long)L.parts * (L.KC / 8) * L.Np;
      const long long ch = idx / per_chunk;
      long long r = idx % per_chunk;
      part = (int)(r / ((L.KC / 8) * L.Np));
      r %= (L.KC / 8) * L.Np;
      const int kg = (int)(r / L.Np);
      o0 = (int)(r % L.Np);
      const int slab = (int)(ch / 9);
      t = (int)(ch % 9);
      i0 = slab * L.KC + kg * 8;
      run_i = true;
    } else {
      // chunk (half, slab, tap): [part][KD/8][128][8]
      const long long j = idx - fwd_rows;
      const long long per_chunk = (long long)L.parts * (L.KD / 8) * 128;
      const long long ch = j / per_chunk;
      long long r = j % per_chunk;
      part = (int)(r / ((L.KD / 8) * 128));
      r %= (L.KD / 8) * 128;
      const int kg = (int)(r / 128);
      const int il = (int)(r % 128);
      const int half = (int)(ch / (L.nslabD * 9));
      const int slab = (int)((ch / 9) % L.nslabD);
      t = (int)(ch % 9);
      i0 = half * 128 + il;
      o0 = slab * L.KD + kg * 8;
      run_i = false;
    }
    union {
      uint4 u;
      Op e[8];
    } row;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int o = run_i ? o0 : o0 + e;
      const int i = run_i ? i0 + e : i0;
      float v = 0.f;
      if (o < L.Cout && i < L.Cin) v = to_f32<T>(w[((size_t)o * L.Cin + i) * 9 + t]);
      const Op hi = op_from<Op>(v);
      row.e[e] = part == 0 ? hi : op_from<Op>(v - op_to<Op>(hi));
    }
    reinterpret_cast<uint4*>(out)[idx] = row.u;
  }
}

template <typename T, bool kDgrad, bool kStaged>
int launch_conv(FcParams prm, const FcMaps& maps, cudaStream_t st) {
  const FcSmem L = fc_smem_layout(prm);
  auto fn = fuseconv_kernel<T, kDgrad, kStaged>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  const int grid = prm.num_units < num_sms() ? prm.num_units : num_sms();
  fn<<<grid, FcCfg<T, kDgrad, kStaged>::kThreads, L.total, st>>>(prm, maps);
  DDPM_CHECK_LAUNCH(kDgrad ? "fuseconv_dgrad_kernel" : "fuseconv_fwd_kernel");
  return DDPM_OK;
}

template <typename T>
int dispatch_conv(bool dgrad, bool staged, const FcParams& prm, const FcMaps& maps,
                  cudaStream_t st) {
  if (staged)
    return dgrad ? launch_conv<T, true, true>(prm, maps, st)
                 : launch_conv<T, false, true>(prm, maps, st);
  return dgrad ? launch_conv<T, true, false>(prm, maps, st)
               : launch_conv<T, false, false>(prm, maps, st);
}

// ------------------------------------------------------------ plane staging ----
constexpr int kPlaneCols = 64;   // plane columns per block
constexpr int kPlaneChans = 64;  // channels per block

// Block = (n, plane row, 64-column strip, 64-channel chunk): 8-pixel vector
// loads of one channel, a shared tile (68-float rows: 16-byte aligned vector
// stores, conflict-free column reads) transposes, each thread writes 16-byte
// rows of 8 channels (consecutive threads = consecutive columns).
template <typename T>
__global__ void __launch_bounds__(256) stage_planes_kernel(const T* __restrict__ src,
                                                           uint4* __restrict__ hi,
                                                           uint4* __restrict__ lo,
                                                           const fuseconv::PlaneLayout L) {
  using Op = typename IoTraits<T>::Op;
  constexpr bool kSplit = IoTraits<T>::kSplit;
  __shared__ __align__(16) float tile[kPlaneChans][kPlaneCols + 4];
  const int ni = blockIdx.x, n = ni / L.Hp, i = ni - n * L.Hp;
  const int hr = i - 1;                      // image row (may be outside the image)
  const int j0 = blockIdx.y * kPlaneCols;    // first plane column
  const int c0 = blockIdx.z * kPlaneChans;   // first channel
  const size_t P = (size_t)L.H * L.W;
  for (int item = threadIdx.x; item < kPlaneChans * (kPlaneCols / 8); item += blockDim.x) {
    const int g = item & 7, cl = item >> 3, c = c0 + cl;
    Raw8<T> v;
    if (c < L.C)
      v = load_raw8<T>(src + ((size_t)n * L.C + c) * P, L.H, L.W, hr, j0 - 8 + g * 8);
    else
      v.zero();
    float4* row = reinterpret_cast<float4*>(&tile[cl][g * 8]);
    row[0] = make_float4(v.get(0), v.get(1), v.get(2), v.get(3));
    row[1] = make_float4(v.get(4), v.get(5), v.get(6), v.get(7));
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < (kPlaneChans / 8) * kPlaneCols; idx += blockDim.x) {
    const int kg = idx / kPlaneCols, x = idx - kg * kPlaneCols;
    const int g = c0 / 8 + kg;
    if (j0 + x >= L.Wp || g >= L.G) continue;
    unsigned long long pr[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[e] = f2_pack(tile[kg * 8 + 2 * e][x], tile[kg * 8 + 2 * e + 1][x]);
    const size_t dst = (((size_t)n * L.G + g) * L.Hp + i) * L.Wp + j0 + x;
    uint4 vh, vl;
    store8x2_split<Op, kSplit>(reinterpret_cast<uint8_t*>(&vh), reinterpret_cast<uint8_t*>(&vl), pr);
    hi[dst] = vh;
    if constexpr (kSplit) lo[dst] = vl;
  }
}

template <typename T>
int launch_stage_planes(const T* src, uint8_t* planes, const fuseconv::PlaneLayout& L,
                        cudaStream_t st) {
  uint4* hi = reinterpret_cast<uint4*>(planes);
  uint4* lo = L.parts > 1 ? reinterpret_cast<uint4*>(planes + L.part_bytes) : nullptr;
  const dim3 grid((unsigned)(L.N * L.Hp), (unsigned)((L.Wp + kPlaneCols - 1) / kPlaneCols),
                  (unsigned)((L.G * 8 + kPlaneChans - 1) / kPlaneChans));
  stage_planes_kernel<T><<<grid, 256, 0, st>>>(src, hi, lo, L);
  DDPM_CHECK_LAUNCH("fuseconv_stage_planes_kernel");
  return DDPM_OK;
}

bool encode_plane_map(CUtensorMap* map, const uint8_t* planes, const fuseconv::PlaneLayout& L,
                      int KC) {
  const uint64_t d[5] = {32, (uint64_t)L.Wp / 16, (uint64_t)L.Hp, (uint64_t)L.G,
                         (uint64_t)L.parts * L.N};
  const uint64_t s4[4] = {256, (uint64_t)L.Wp * 16, (uint64_t)L.Hp * L.Wp * 16,
                          (uint64_t)L.G * L.Hp * L.Wp * 16};
  const uint32_t box[5] = {32, 9, (uint32_t)kRows, (uint32_t)(KC / 8), 1};
  if (encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 5, planes, d, s4, box,
                  CU_TENSOR_MAP_SWIZZLE_NONE) != DDPM_OK) {
    clear_error();
    return false;
  }
  return true;
}

int check_conv(int n, int cin, int cout, int h, int w, int dt) {
  DDPM_CHECK_ARG(n >= 1 && h >= 1 && w >= 1 && cin >= 1 && cout >= 1, "sizes must be positive");
  DDPM_CHECK_ARG(dtype_size(dt) > 0, "unknown dtype code %d", dt);
  if (cin > fuseconv::kMaxCin || cout > fuseconv::kMaxCout)
    return set_error(DDPM_ERR_UNSUPPORTED, "native fuse conv supports Cin <= %d, Cout <= %d",
                     fuseconv::kMaxCin, fuseconv::kMaxCout);
  DDPM_CHECK_ARG((long long)n * ((h + 1) / 2) * ((w + 127) / 128) * 2 < (1LL << 31),
                 "too many tiles");
  return DDPM_OK;
}

FcParams common_params(int n, int h, int w, int nhalf, int* status) {
  FcParams q{};
  q.N = n;
  q.H = h;
  q.W = w;
  q.tiles_w = (w + 127) / 128;
  q.hpairs = (h + 1) / 2;
  q.nhalf = nhalf;
  q.num_units = n * q.hpairs * q.tiles_w * nhalf;
  q.status = status;
  return q;
}

int dispatch_dt(int dt, bool dgrad, bool staged, const FcParams& prm, const FcMaps& maps,
                cudaStream_t st) {
  switch (dt) {
    case DDPM_BF16: return dispatch_conv<__nv_bfloat16>(dgrad, staged, prm, maps, st);
    case DDPM_F16: return dispatch_conv<__half>(dgrad, staged, prm, maps, st);
    case DDPM_F32: return dispatch_conv<float>(dgrad, staged, prm, maps, st);
  }
  return set_error(DDPM_ERR_INVALID_ARG, "unknown dtype %d", dt);
}

// Staged planes argument check and tensor map (KC = the pass's K slab).
int plane_map(FcMaps* maps, const void* planes, size_t bytes, int n, int c, int h, int w,
              int dt, int KC) {
  const fuseconv::PlaneLayout L = fuseconv::PlaneLayout::make(n, c, h, w, dt);
  if (bytes < L.bytes())
    return set_error(DDPM_ERR_WORKSPACE, "staged planes too small (%zu < %zu)", bytes, L.bytes());
  DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(planes) & 255u) == 0,
                 "staged planes must be 256-byte aligned");
  if (!encode_plane_map(&maps->smap, static_cast<const uint8_t*>(planes), L, KC))
    return set_error(DDPM_ERR_CUDA, "tensor map of the staged planes could not be encoded");
  return DDPM_OK;
}

}  // namespace

namespace fuseconv {

PlaneLayout PlaneLayout::make(int n, int c, int h, int w, int dt) {
  PlaneLayout L{};
  L.N = n;
  L.C = c;
  L.H = h;
  L.W = w;
  L.G = (c + 63) / 64 * 8;
  L.Hp = h + 2;
  L.Wp = (w + 127) / 128 * 128 + 16;
  L.parts = dt == DDPM_F32 ? 2 : 1;
  L.part_bytes = (size_t)n * L.G * L.Hp * L.Wp * 16;
  return L;
}

Layout Layout::make(int cin, int cout, int dt) {
  Layout L{};
  const bool split = dt == DDPM_F32;
  L.Cin = cin;
  L.Cout = cout;
  L.parts = split ? 2 : 1;
  L.Np = (cout + 15) / 16 * 16;
  L.KC = split ? 16 : 32;
  L.nslab = (cin + L.KC - 1) / L.KC;
  L.KD = split ? 32 : 64;
  L.nslabD = (cout + L.KD - 1) / L.KD;
  L.nhalf = (cin + 127) / 128;
  L.fwd_chunk = (size_t)L.parts * L.KC * L.Np * 2;
  L.dg_chunk = (size_t)L.parts * L.KD * 128 * 2;
  L.fwd_bytes = (size_t)L.nslab * 9 * L.fwd_chunk;
  L.dg_bytes = (size_t)L.nhalf * L.nslabD * 9 * L.dg_chunk;
  return L;
}

}  // namespace fuseconv

size_t fuseconv_pack_bytes(int cin, int cout, int dt) {
  if (cin < 1 || cout < 1 || cin > fuseconv::kMaxCin || cout > fuseconv::kMaxCout ||
      dtype_size(dt) == 0)
    return 0;
  const fuseconv::Layout L = fuseconv::Layout::make(cin, cout, dt);
  return L.fwd_bytes + L.dg_bytes;
}

int fuseconv_pack(const void* w, int cin, int cout, int dt, void* packed, size_t bytes,
                  cudaStream_t st) {
  int rc = check_conv(1, cin, cout, 1, 1, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG(w && packed, "null pointer");
  DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(packed) & 15u) == 0,
                 "packed weight buffer must be 16-byte aligned");
  const fuseconv::Layout L = fuseconv::Layout::make(cin, cout, dt);
  if (bytes < L.fwd_bytes + L.dg_bytes)
    return set_error(DDPM_ERR_WORKSPACE, "packed weight buffer too small (%zu < %zu)", bytes,
                     L.fwd_bytes + L.dg_bytes);
  const long long rows = (long long)(L.fwd_bytes + L.dg_bytes) / 16;
  const int threads = 256;
  const long long want = (rows + threads - 1) / threads;
  const int blocks = (int)(want < 4096 ? want : 4096);
  switch (dt) {
    case DDPM_BF16:
      fuseconv_pack_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(
          static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(packed), L);
      break;
    case DDPM_F16:
      fuseconv_pack_kernel<__half><<<blocks, threads, 0, st>>>(
          static_cast<const __half*>(w), static_cast<__half*>(packed), L);
      break;
    default:
      fuseconv_pack_kernel<float><<<blocks, threads, 0, st>>>(
          static_cast<const float*>(w), static_cast<__nv_bfloat16*>(packed), L);
  }
  DDPM_CHECK_LAUNCH("fuseconv_pack_kernel");
  return DDPM_OK;
}

size_t fuseconv_stage_bytes(int n, int c, int h, int w, int dt) {
  if (n < 1 || c < 1 || h < 1 || w < 1 || c > fuseconv::kMaxCin || dtype_size(dt) == 0) return 0;
  return fuseconv::PlaneLayout::make(n, c, h, w, dt).bytes();
}

int fuseconv_stage(const void* src, void* planes, size_t bytes, int n, int c, int h, int w, int dt,
                   cudaStream_t st) {
  DDPM_CHECK_ARG(n >= 1 && c >= 1 && h >= 1 && w >= 1, "sizes must be positive");
  DDPM_CHECK_ARG(dtype_size(dt) > 0, "unknown dtype code %d", dt);
  if (c > fuseconv::kMaxCin)
    return set_error(DDPM_ERR_UNSUPPORTED, "staged planes support C <= %d", fuseconv::kMaxCin);
  DDPM_CHECK_ARG(src && planes, "null pointer");
  const fuseconv::PlaneLayout L = fuseconv::PlaneLayout::make(n, c, h, w, dt);
  if (bytes < L.bytes())
    return set_error(DDPM_ERR_WORKSPACE, "staged planes too small (%zu < %zu)", bytes, L.bytes());
  DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(planes) & 255u) == 0,
                 "staged planes must be 256-byte aligned");
  uint8_t* pl = static_cast<uint8_t*>(planes);
  switch (dt) {
    case DDPM_BF16: return launch_stage_planes(static_cast<const __nv_bfloat16*>(src), pl, L, st);
    case DDPM_F16: return launch_stage_planes(static_cast<const __half*>(src), pl, L, st);
    default: return launch_stage_planes(static_cast<const float*>(src), pl, L, st);
  }
}

// `cat` (NCHW) or, when `planes` is set, its staged planes (fuseconv_stage).
int fuseconv_fwd_any(const void* cat, const void* planes, size_t planes_bytes, const void* packed,
                     const void* bias, void* out, int n, int cin, int cout, int h, int w, int dt,
                     cudaStream_t st) {
  int rc = check_conv(n, cin, cout, h, w, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG((cat || planes) && packed && out, "null pointer");
  int* status = nullptr;
  rc = gencat::status_ptr(&status);
  if (rc) return rc;
  const fuseconv::Layout L = fuseconv::Layout::make(cin, cout, dt);
  FcParams q = common_params(n, h, w, 1, status);
  q.src = cat;
  q.wimg = static_cast<const uint8_t*>(packed);
  q.bias = bias;
  q.dst = out;
  q.Csrc = cin;
  q.Cdst = cout;
  q.KC = L.KC;
  q.nslab = L.nslab;
  q.Nn = L.Np;
  q.reg_part = (uint32_t)L.KC * kRows * kSeg * 2;
  q.reg_bytes = q.reg_part * L.parts;
  q.reg_bufs = 3;
  q.w_chunk = (uint32_t)(9 * L.fwd_chunk);  // a slab's 9 tap images per chunk
  q.w_tap = (uint32_t)L.fwd_chunk;
  q.w_stages = 3;
  FcMaps maps{};
  if (planes != nullptr) {
    rc = plane_map(&maps, planes, planes_bytes, n, cin, h, w, dt, L.KC);
    if (rc) return rc;
  }
  return dispatch_dt(dt, false, planes != nullptr, q, maps, st);
}

int fuseconv_fwd(const void* cat, const void* packed, const void* bias, void* out, int n, int cin,
                 int cout, int h, int w, int dt, cudaStream_t st) {
  return fuseconv_fwd_any(cat, nullptr, 0, packed, bias, out, n, cin, cout, h, w, dt, st);
}

int fuseconv_fwd_staged(const void* planes, size_t planes_bytes, const void* packed,
                        const void* bias, void* out, int n, int cin, int cout, int h, int w, int dt,
                        cudaStream_t st) {
  DDPM_CHECK_ARG(planes, "null pointer");
  return fuseconv_fwd_any(nullptr, planes, planes_bytes, packed, bias, out, n, cin, cout, h, w, dt,
                          st);
}

// `gout` (NCHW) or, when `planes` is set, its staged planes (fuseconv_stage).
int fuseconv_dgrad_any(const void* gout, const void* planes, size_t planes_bytes,
                       const void* packed, void* gcat, int n, int cin, int cout, int h, int w,
                       int dt, cudaStream_t st, int gcat_nhwc = 0) {
  int rc = check_conv(n, cin, cout, h, w, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG((gout || planes) && packed && gcat, "null pointer");
  DDPM_CHECK_ARG(!gcat_nhwc || (cin % 16 == 0 && (reinterpret_cast<uintptr_t>(gcat) & 15u) == 0),
                 "a channel-last gradient needs Cin %% 16 == 0 and a 16-byte aligned buffer");
  int* status = nullptr;
  rc = gencat::status_ptr(&status);
  if (rc) return rc;
  const fuseconv::Layout L = fuseconv::Layout::make(cin, cout, dt);
  FcParams q = common_params(n, h, w, L.nhalf, status);
  q.src = gout;
  q.wimg = static_cast<const uint8_t*>(packed) + L.fwd_bytes;
  q.bias = nullptr;
  q.dst = gcat;
  q.dst_nhwc = gcat_nhwc;
  q.Csrc = cout;
  q.Cdst = cin;
  q.KC = L.KD;
  q.nslab = L.nslabD;
  q.Nn = 128;
  q.reg_part = (uint32_t)L.KD * kRows * kSeg * 2;
  q.reg_bytes = q.reg_part * L.parts;
  q.reg_bufs = 2;
  q.w_chunk = (uint32_t)L.dg_chunk;
  q.w_tap = (uint32_t)L.dg_chunk;
  q.w_stages = 4;
  FcMaps maps{};
  if (planes != nullptr) {
    rc = plane_map(&maps, planes, planes_bytes, n, cout, h, w, dt, L.KD);
    if (rc) return rc;
  }
  return dispatch_dt(dt, true, planes != nullptr, q, maps, st);
}

int fuseconv_dgrad(const void* gout, const void* packed, void* gcat, int n, int cin, int cout,
                   int h, int w, int dt, cudaStream_t st, int gcat_nhwc) {
  return fuseconv_dgrad_any(gout, nullptr, 0, packed, gcat, n, cin, cout, h, w, dt, st,
                            gcat_nhwc);
}

// Data gradient reading grad_out from the weight gradient's channel-last
// planes [n][h][Np/8][w][8] (hi, and lo for FP32; W % 8 == 0, 16-byte aligned):
// one box per slab and part over those planes, so grad_out is not staged a
// second time. Returns DDPM_ERR_UNSUPPORTED, nothing launched, if a tensor map
// is rejected.
int fuseconv_dgrad_rowmajor(const void* hi, const void* lo, const void* packed, void* gcat, int n,
                            int cin, int cout, int h, int w, int dt, cudaStream_t st,
                            int gcat_nhwc) {
  int rc = check_conv(n, cin, cout, h, w, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG(!gcat_nhwc || (cin % 16 == 0 && (reinterpret_cast<uintptr_t>(gcat) & 15u) == 0),
                 "a channel-last gradient needs Cin %% 16 == 0 and a 16-byte aligned buffer");
  DDPM_CHECK_ARG(hi && packed && gcat && (dt != DDPM_F32 || lo), "null pointer");
  DDPM_CHECK_ARG(w % 8 == 0, "row-major grad_out planes need W %% 8 == 0");
  int* status = nullptr;
  rc = gencat::status_ptr(&status);
  if (rc) return rc;
  const fuseconv::Layout L = fuseconv::Layout::make(cin, cout, dt);
  FcParams q = common_params(n, h, w, L.nhalf, status);
  q.wimg = static_cast<const uint8_t*>(packed) + L.fwd_bytes;
  q.dst = gcat;
  q.dst_nhwc = gcat_nhwc;
  q.Csrc = cout;
  q.Cdst = cin;
  q.KC = L.KD;
  q.nslab = L.nslabD;
  q.Nn = 128;
  q.reg_part = (uint32_t)L.KD * kRows * kSeg * 2;
  q.reg_bytes = q.reg_part * L.parts;
  q.reg_bufs = 2;
  q.w_chunk = (uint32_t)L.dg_chunk;
  q.w_tap = (uint32_t)L.dg_chunk;
  q.w_stages = 4;
  q.row_major = 1;
  const uint64_t ng = (uint64_t)L.Np / 8;
  const uint64_t d[5] = {16, (uint64_t)w / 8, ng, (uint64_t)h, (uint64_t)n};
  const uint64_t s4[4] = {128, (uint64_t)w * 16, ng * w * 16, (uint64_t)h * ng * w * 16};
  const uint32_t box[5] = {16, 18, (uint32_t)(L.KD / 8), (uint32_t)kRows, 1};
  FcMaps maps{};
  for (int part = 0; part < L.parts; ++part) {
    if (encode_tmap(part ? &maps.smap_lo : &maps.smap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 5,
                    part ? lo : hi, d, s4, box, CU_TENSOR_MAP_SWIZZLE_NONE) != DDPM_OK) {
      clear_error();
      return DDPM_ERR_UNSUPPORTED;
    }
  }
  return dispatch_dt(dt, true, true, q, maps, st);
}

int fuseconv_dgrad_staged(const void* planes, size_t planes_bytes, const void* packed, void* gcat,
                          int n, int cin, int cout, int h, int w, int dt, cudaStream_t st) {
  DDPM_CHECK_ARG(planes, "null pointer");
  return fuseconv_dgrad_any(nullptr, planes, planes_bytes, packed, gcat, n, cin, cout, h, w, dt,
                            st);
}

}  // namespace ddpm
