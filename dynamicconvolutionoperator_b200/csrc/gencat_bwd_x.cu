// Fused generator backward, input gradient dX (recompute of the taps).
// Replaces `_generator_dynamic_cat_bwd_x` (reference `_triton_kernels.py:430-531`):
//
//   dX[c, q] = g[c, q] + sum_{b, tap} gen[(b,c,tap), q - o] * g_b[c, q - o]
//   gen      = round_io(W * y + bias)      (the forward's taps, recomputed)
//   o        = ((ki - r) * d_b, (kj - r) * d_b), zero outside the image.
//
// The taps needed at q are the generator outputs at the SHIFTED pixel q - o.
// Instead of 27 reloads of shifted y tiles (the reference's approach), one
// shared-memory copy of the y rows a tile needs is staged per branch in the
// K-major interleaved operand layout ([channel group][row segment][pixel][8]):
// pixel rows are 16 bytes apart, so the MMA operand for tap (ki, kj) is just
// a descriptor whose start address is moved by (8 - dx) pixels inside row
// segment ki. Each (branch, tap) chunk is one M=128 x N=Cp GEMM whose rows
// are already the shifted taps of the tile's pixels.
//
// Tile = 128 consecutive pixels of one image row (TMEM lane m <-> column
// w0 + m). Per branch the staged region is K rows x 144 pixels (columns
// w0-8 .. w0+135) x Ck channels. The weight chunk of (b, tap) is the packed
// "bx" image row block [Ck/8][Cp][8], streamed through a ring of bulk copies.
// Epilogue warpgroup h owns the 16-channel blocks h, h+2 of every chunk and
// multiplies with g_b at q - o read through L1.
//
// Warp roles (15 warps): w0 = TMEM allocator + weight producer, w1-w2 = MMA
// issuers (even / odd chunks: one thread issuing N=Cp MMAs back to back
// leaves the tensor pipe idle ~half the time), w3-w6 = region producers,
// w7-w14 = two epilogue warpgroups.
#include "common.cuh"
#include "tc.cuh"
#include "gencat.cuh"

namespace ddpm {
namespace {

using namespace gencat;

constexpr int kSeg = 144;  // staged pixels per row segment (128 + 8 on each side)

template <typename T, int KS>
struct BxCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  static constexpr int kParts = kSplit ? 2 : 1;
  static constexpr int kRegBufs = kSplit ? 1 : 2;
  static constexpr int kWStages = 6;
  static constexpr bool kBiasInGemm = !kSplit;
  static constexpr int kIssuers = 2;        // MMA issuer warps (alternate chunks)
  static constexpr int kFirstProducerWarp = 1 + kIssuers;
  static constexpr int kFirstEpiWarp = kFirstProducerWarp + 4;
  static constexpr int kThreads = 32 * (kFirstEpiWarp + 8);
};

struct BxSmem {
  uint32_t reg, w, bias, bars, total;
  uint32_t reg_part, reg_bytes, w_bytes;
};

template <typename T, int KS>
__host__ __device__ inline BxSmem bx_smem_layout(int Cp, int Ck, int C) {
  using Cfg = BxCfg<T, KS>;
  BxSmem L;
  L.reg_part = (uint32_t)Ck * KS * kSeg * 2;
  L.reg_bytes = Cfg::kParts * L.reg_part;
  L.w_bytes = (uint32_t)Cfg::kParts * Cp * Ck * 2;
  L.reg = 0;
  L.w = L.reg + Cfg::kRegBufs * L.reg_bytes;
  L.bias = L.w + Cfg::kWStages * L.w_bytes;
  L.bars = L.bias + (Cfg::kBiasInGemm ? 0u : (uint32_t)(3 * KS * KS * Cp * 4));
  const int nb = 512 / Cp > 8 ? 8 : 512 / Cp;
  L.total = L.bars + 8 * (4 + 2 * Cfg::kWStages + 2 * nb);
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
  int* status;
};

template <typename T, int KS>
__global__ void __launch_bounds__(BxCfg<T, KS>::kThreads, 1)
gencat_bwd_x_kernel(const BxParams p) {
  using Cfg = BxCfg<T, KS>;
  using Op = typename IoTraits<T>::Op;
  constexpr int S = Cfg::kWStages;
  constexpr int NR = Cfg::kRegBufs;
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int C = p.C, Cp = p.Cp, Ck = p.Ck, H = p.H, W = p.W;
  const size_t P = (size_t)H * W;
  const BxSmem L = bx_smem_layout<T, KS>(Cp, Ck, C);
  const int NB = 512 / Cp > 8 ? 8 : 512 / Cp;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* r_full = bars;           // [2]
  uint64_t* r_empty = bars + 2;      // [2]
  uint64_t* w_full = bars + 4;       // [S]
  uint64_t* w_empty = w_full + S;    // [S]
  uint64_t* t_full = w_empty + S;    // [NB]
  uint64_t* t_empty = t_full + NB;   // [NB]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&r_full[i], 128);
      tc::mbar_init(&r_empty[i], Cfg::kIssuers);
    }
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&w_full[i], 1);
      tc::mbar_init(&w_empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      tc::mbar_init(&t_full[i], 1);
      tc::mbar_init(&t_empty[i], 256);
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

  if (warp == 0) {
    // ---- weight producer: 3*K^2 chunks per tile ---------------------------
    if (lane == 0) {
      const uint8_t* wsrc = static_cast<const uint8_t*>(p.wpack);
      uint32_t wq = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        for (int q = 0; q < 3 * KK; ++q, ++wq) {
          const int s = wq % S;
          if (!tc::mbar_wait(&w_empty[s], ((wq / S) & 1) ^ 1, abort_flag, kWaitNs)) {
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
    // ---- MMA issuers: warp 1 + i issues the chunks q with q % 2 == i --------
    if (lane == 0) {
      const uint32_t me = warp - 1;
      const uint32_t idesc = tc::idesc_f16(kTileM, Cp, IoTraits<T>::kBf16, false, false);
      const uint32_t a_lbo = KS * kSeg * 16;    // channel-group stride of the region
      const uint32_t b_lbo = Cp * 16;           // channel-group stride of a weight chunk
      const uint64_t a_step = (2 * a_lbo) >> 4;  // descriptor advance per K step
      const uint64_t b_step = (2 * b_lbo) >> 4;
      const uint64_t a_lo = L.reg_part >> 4;     // hi -> lo part offsets
      const uint64_t b_lo = (Cp * Ck * 2) >> 4;
      const int nks = Ck / 16;
      uint32_t wq = 0, tq = 0, rq = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        for (int b = 0; b < 3; ++b, ++rq) {
          const int rb = rq % NR;
          if (!tc::mbar_wait(&r_full[rb], (rq / NR) & 1, abort_flag, kWaitNs)) {
            fail(abort_flag, p.status, 21);
            goto done;
          }
          tc::tc_fence_after();
          const uint64_t a_base =
              tc::smem_desc(tc::smem_u32(smem + L.reg + rb * L.reg_bytes), a_lbo, 128);
          const int d = p.d[b];
          for (int tap = 0; tap < KK; ++tap, ++wq, ++tq) {
            if ((wq & 1u) != me) continue;
            const int s = wq % S;
            const int j = tq % NB;
            if (!tc::mbar_wait(&w_full[s], (wq / S) & 1, abort_flag, kWaitNs) ||
                !tc::mbar_wait(&t_empty[j], ((tq / NB) & 1) ^ 1, abort_flag, kWaitNs)) {
              fail(abort_flag, p.status, 22);
              goto done;
            }
            tc::tc_fence_after();
            const int ki = tap / KS, kj = tap % KS;
            const int dx = (kj - r) * d;
            // window: row segment ki, pixels (8 - dx) .. (8 - dx) + 127
            const uint64_t ad = a_base + (uint64_t)(ki * kSeg + 8 - dx);
            const uint64_t bd =
                tc::smem_desc(tc::smem_u32(smem + L.w + s * L.w_bytes), b_lbo, 128);
            const uint32_t dt = tmem_base + j * Cp;
            // plain runtime loop (no MMA under a per-step condition in an unrolled loop)
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
          tc::mma_commit(&r_empty[rb]);
        }
      }
    }
  } else if (warp < Cfg::kFirstEpiWarp) {
    // ---- region producers (128 threads) ------------------------------------
    const int pt = threadIdx.x - 32 * Cfg::kFirstProducerWarp;
    const T* y = static_cast<const T*>(p.y);
    const int ones_c = Cfg::kBiasInGemm ? C : -1;
    uint32_t rq = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
      const int per_img = H * p.tiles_w;
      const int n = tile / per_img;
      const int h = (tile % per_img) / p.tiles_w;
      const int w0 = (tile % p.tiles_w) * kTileM;
      for (int b = 0; b < 3; ++b, ++rq) {
        const int rb = rq % NR;
        if (!warp_wait(&r_empty[rb], ((rq / NR) & 1) ^ 1, abort_flag)) {
          fail(abort_flag, p.status, 23);
          break;
        }
        uint8_t* reg = smem + L.reg + rb * L.reg_bytes;
        const int d = p.d[b];
        // item = (channel group kg, segment s, 8-pixel block jb)
        const int items = (Ck / 8) * KS * (kSeg / 8);
        for (int item = pt; item < items; item += 128) {
          const int jb = item % (kSeg / 8);
          const int s = (item / (kSeg / 8)) % KS;
          const int kg = item / ((kSeg / 8) * KS);
          const int hr = h - (s - r) * d;  // image row of segment s
          Raw8<T> v[8];                    // [channel] x 8 pixels
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int c = kg * 8 + e;
            if (c < C)
              v[e] = load_raw8<T>(y + ((size_t)n * C + c) * P, H, W, hr, w0 - 8 + jb * 8);
            else
              v[e].zero();
          }
#pragma unroll
          for (int px = 0; px < 8; ++px) {
            float col[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int c = kg * 8 + e;
              col[e] = c < C ? v[e].get(px) : (c == ones_c ? 1.f : 0.f);
            }
            const uint32_t off = ((kg * KS + s) * kSeg + jb * 8 + px) * 16;
            store8_split<Op, Cfg::kSplit>(reg + off, reg + L.reg_part + off, col);
          }
        }
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&r_full[rb]);
      }
    }
  } else {
    // ---- epilogue: warpgroup wg owns channel blocks wg, wg + 2 ------------
    const int ew = warp - Cfg::kFirstEpiWarp;
    const int wg = ew >> 2;
    const int quad = warp & 3;
    const int m = quad * 32 + lane;
    const T* gout = static_cast<const T*>(p.gout);
    T* gx = static_cast<T*>(p.gx);
    const float* bias_s = reinterpret_cast<const float*>(smem + L.bias);
    const int nblk = Cp / 16;
    uint32_t tq = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int per_img = H * p.tiles_w;
      const int n = tile / per_img;
      const int h = (tile % per_img) / p.tiles_w;
      const int w = (tile % p.tiles_w) * kTileM + m;
      const bool px_ok = w < W;
      const T* gn = gout + (size_t)n * 4 * C * P;
      float acc[2][16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[0][i] = acc[1][i] = 0.f;
      bool failed = false;
      for (int b = 0; b < 3 && !failed; ++b) {
        const int d = p.d[b];
        for (int tap = 0; tap < KK; ++tap, ++tq) {
          const int ki = tap / KS, kj = tap % KS;
          const int dy = (ki - r) * d, dx = (kj - r) * d;
          const bool ok = px_ok && (unsigned)(h - dy) < (unsigned)H && (unsigned)(w - dx) < (unsigned)W;
          const size_t src = (size_t)(h - dy) * W + (w - dx);
          const int j = tq % NB;
          if (!warp_wait(&t_full[j], (tq / NB) & 1, abort_flag)) {
            fail(abort_flag, p.status, 24);
            failed = true;
            break;
          }
          tc::tc_fence_after();
#pragma unroll
          for (int bi = 0; bi < 2; ++bi) {
            const int blk = wg + 2 * bi;
            if (blk >= nblk) break;
            float dv[16];
            tc::tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + j * Cp + blk * 16, dv);
            float gv[16];
#pragma unroll
            for (int cl = 0; cl < 16; ++cl) {
              const int c = blk * 16 + cl;
              gv[cl] = (ok && c < C) ? to_f32<T>(__ldg(gn + (size_t)((b + 1) * C + c) * P + src))
                                     : 0.f;
            }
            tc::tmem_ld_wait();
            if constexpr (!Cfg::kBiasInGemm) {
              const float* bs = bias_s + (b * KK + tap) * Cp + blk * 16;
#pragma unroll
              for (int cl = 0; cl < 16; ++cl) dv[cl] += bs[cl];
            }
            round_taps<T>(dv);
#pragma unroll
            for (int cl = 0; cl < 16; ++cl) acc[bi][cl] = fmaf(dv[cl], gv[cl], acc[bi][cl]);
          }
          tc::tc_fence_before();
          tc::mbar_arrive(&t_empty[j]);
        }
      }
      if (failed) break;
      if (px_ok) {
        const size_t q = (size_t)h * W + w;
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const int blk = wg + 2 * bi;
          if (blk >= nblk) break;
#pragma unroll
          for (int cl = 0; cl < 16; ++cl) {
            const int c = blk * 16 + cl;
            if (c < C) {
              const float g0 = to_f32<T>(gn[(size_t)c * P + q]);
              gx[((size_t)n * C + c) * P + q] = from_f32<T>(acc[bi][cl] + g0);
            }
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

template <typename T, int KS>
int launch(const BxParams& prm, cudaStream_t st) {
  using Cfg = BxCfg<T, KS>;
  const BxSmem L = bx_smem_layout<T, KS>(prm.Cp, prm.Ck, prm.C);
  auto fn = gencat_bwd_x_kernel<T, KS>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  const int grid = prm.num_tiles < num_sms() ? prm.num_tiles : num_sms();
  fn<<<grid, Cfg::kThreads, L.total, st>>>(prm);
  DDPM_CHECK_LAUNCH("gencat_bwd_x_kernel");
  return DDPM_OK;
}

template <typename T>
int dispatch(int ks, const BxParams& prm, cudaStream_t st) {
  switch (ks) {
    case 1: return launch<T, 1>(prm, st);
    case 3: return launch<T, 3>(prm, st);
  }
  return set_error(DDPM_ERR_UNSUPPORTED, "fused generator: kernel_size %d not supported", ks);
}

}  // namespace

int gencat_bwd_x(const void* y, const void* wpack, const void* bias, const void* gout, void* gx,
                 int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt,
                 cudaStream_t st) {
  int rc = gencat::check_shape(n, c, h, w, ks, d0, d1, d2, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG(y && wpack && bias && gout && gx, "null pointer");
  const gencat::PackLayout pl = gencat::PackLayout::make(c, ks, dt);
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
