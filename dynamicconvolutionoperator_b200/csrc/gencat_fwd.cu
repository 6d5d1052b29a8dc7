// Fused 1x1 generator + dilated dynamic filter, forward ("gencat").
// Replaces `_generator_dynamic_cat_fwd` / `_launch_generator_dynamic_cat`
// (reference `_triton_kernels.py:268-420`, `:873-908`).
//
//   gen[(b*C+c)*K^2 + tap, p] = sum_i W[(b*C+c)*K^2 + tap, i] * y[i, p] + bias[...]
//   out[0:C]          = x
//   out[(b+1)C + c]   = sum_tap round_io(gen[(b,c,tap), p]) * x[c, p + off(tap)*d_b]
//
// The generated taps (3*C*K^2 per pixel) never leave the SM: the generator
// GEMM runs on the tensor cores (tcgen05.mma, kind::f16, FP32 accumulator in
// TMEM) and the epilogue warps consume the taps straight out of TMEM.
//
// Work decomposition (persistent CTAs, one per SM, 512 TMEM columns):
//   * tile  = 8 x 16 output pixels of one image = the 128 rows of the MMA's
//             M dimension = the 128 TMEM lanes (lane m <-> pixel (m/16, m%16));
//   * chunk = (channel group cg of 16, branch b, kernel row ki): N = 16*K
//             accumulator columns, column kj*16 + cl <-> tap (ki, kj) of
//             channel cg*16 + cl. A tile is (Cp/16) * 3 * K chunks.
//   * operands: A = the y tile, MN-major in shared memory ([8-pixel group]
//             [channel][8 pixels], so each 16-byte row is one contiguous global
//             segment of 8 pixels of one channel); B = the chunk's weight rows,
//             pre-packed in global memory in the exact K-major smem image and
//             streamed through a 4-stage ring with 1-D bulk async copies.
//   * FP32 I/O: y and W are split into bf16 hi + lo parts and each MMA step
//             is hi*hi + lo*hi + hi*lo (relative error ~2^-16 per product).
//
// Warp roles (12 warps): w0 = TMEM allocator + weight producer, w1 = MMA
// issuer, w2-w3 = y-tile producers, w4-w11 = two epilogue warpgroups. Output
// group (cg, b) belongs to warpgroup (cg*3+b) % 2, which consumes its K chunks
// in order from a ring of TMEM accumulator buffers.
#include "common.cuh"
#include "tc.cuh"
#include "gencat.cuh"

namespace ddpm {
namespace {

using namespace gencat;

template <typename T, int KS>
struct FwdCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  static constexpr int kParts = kSplit ? 2 : 1;
  static constexpr int kN = 16 * KS;                         // accumulator columns per chunk
  static constexpr int kNumBuf = (512 / kN) > 8 ? 8 : (512 / kN);
  static constexpr int kWStages = 4;
  static constexpr int kEpiWG = 2;
  static constexpr int kThreads = 32 * (4 + 4 * kEpiWG);
};

struct FwdSmem {
  // byte offsets into dynamic shared memory
  uint32_t y, w, bias, bars, total;
  uint32_t y_bytes, w_bytes;
};

template <typename T, int KS>
__host__ __device__ inline FwdSmem fwd_smem_layout(int C, int Cp) {
  using Cfg = FwdCfg<T, KS>;
  FwdSmem L;
  L.y_bytes = (uint32_t)Cfg::kParts * kTileM * Cp * 2;
  L.w_bytes = (uint32_t)Cfg::kParts * Cfg::kN * Cp * 2;
  L.y = 0;
  L.w = L.y + 2 * L.y_bytes;
  L.bias = L.w + Cfg::kWStages * L.w_bytes;
  uint32_t bias_bytes = (uint32_t)(3 * C * KS * KS) * 4;
  L.bars = (L.bias + bias_bytes + 15) & ~15u;
  L.total = L.bars + 8 * (4 + 2 * Cfg::kWStages + 2 * Cfg::kNumBuf) + 16;
  return L;
}

struct FwdParams {
  const void* x;
  const void* y;
  const void* wpack;
  const void* bias;
  void* out;
  int N, C, H, W, Cp;
  int d[3];
  int tiles_w, tiles_h, num_tiles;
  int* status;
};

template <typename T, int KS>
__global__ void __launch_bounds__(FwdCfg<T, KS>::kThreads, 1)
gencat_fwd_kernel(const FwdParams p) {
  using Cfg = FwdCfg<T, KS>;
  using Op = typename IoTraits<T>::Op;
  constexpr int kN = Cfg::kN;
  constexpr int NB = Cfg::kNumBuf;
  constexpr int S = Cfg::kWStages;
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int C = p.C, Cp = p.Cp, H = p.H, W = p.W;
  const size_t P = (size_t)H * W;
  const FwdSmem L = fwd_smem_layout<T, KS>(C, Cp);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* y_full = bars;           // [2]
  uint64_t* y_empty = bars + 2;      // [2]
  uint64_t* w_full = bars + 4;       // [S]
  uint64_t* w_empty = w_full + S;    // [S]
  uint64_t* t_full = w_empty + S;    // [NB]
  uint64_t* t_empty = t_full + NB;   // [NB]
  float* bias_s = reinterpret_cast<float*>(smem + L.bias);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nchunks = (Cp / 16) * 3 * KS;
  const uint32_t chunk_bytes = L.w_bytes;

  // ---- setup --------------------------------------------------------------
  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&y_full[i], 64);
      tc::mbar_init(&y_empty[i], 1);
    }
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&w_full[i], 1);
      tc::mbar_init(&w_empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      tc::mbar_init(&t_full[i], 1);
      tc::mbar_init(&t_empty[i], 128);
    }
    tc::fence_mbar_init();
    abort_s = 0;
  }
  {
    const T* bias = static_cast<const T*>(p.bias);
    for (int i = threadIdx.x; i < 3 * C * KK; i += blockDim.x) bias_s[i] = to_f32<T>(bias[i]);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  volatile int* abort_flag = &abort_s;

  if (warp == 0) {
    // ---- weight producer: stream packed chunks through the ring ----------
    if (lane == 0) {
      const uint8_t* wsrc = static_cast<const uint8_t*>(p.wpack);
      uint32_t wq = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        for (int q = 0; q < nchunks; ++q, ++wq) {
          const int s = wq % S;
          if (!tc::mbar_wait(&w_empty[s], ((wq / S) & 1) ^ 1, abort_flag, kWaitNs)) {
            fail(abort_flag, p.status, 10);
            goto done;
          }
          tc::mbar_arrive_expect_tx(&w_full[s], chunk_bytes);
          tc::bulk_g2s(smem + L.w + s * chunk_bytes, wsrc + (size_t)q * chunk_bytes, chunk_bytes,
                       &w_full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer --------------------------------------------------------
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(kTileM, kN, IoTraits<T>::kBf16, true, false);
      const uint32_t a_sbo = Cp * 16;           // 8-pixel groups
      const uint32_t b_lbo = kN * 16;           // 8-channel groups of the weight chunk
      const uint32_t ypart = kTileM * Cp * 2;   // hi -> lo offset of the y tile
      const uint32_t wpart = kN * Cp * 2;       // hi -> lo offset of a weight chunk
      uint32_t wq = 0, tq = 0, it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        const int yb = it & 1;
        if (!tc::mbar_wait(&y_full[yb], (it >> 1) & 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 11);
          goto done;
        }
        tc::tc_fence_after();
        const uint32_t ya = tc::smem_u32(smem + L.y + yb * L.y_bytes);
        for (int q = 0; q < nchunks; ++q, ++wq, ++tq) {
          const int s = wq % S;
          const int j = tq % NB;
          if (!tc::mbar_wait(&w_full[s], (wq / S) & 1, abort_flag, kWaitNs) ||
              !tc::mbar_wait(&t_empty[j], ((tq / NB) & 1) ^ 1, abort_flag, kWaitNs)) {
            fail(abort_flag, p.status, 12);
            goto done;
          }
          tc::tc_fence_after();
          const uint32_t wb = tc::smem_u32(smem + L.w + s * chunk_bytes);
          const uint32_t d = tmem_base + j * kN;
          for (int ks = 0; ks < Cp / 16; ++ks) {
            const uint64_t a_hi = tc::smem_desc(ya + ks * 256, 128, a_sbo);
            const uint64_t b_hi = tc::smem_desc(wb + ks * 2 * b_lbo, b_lbo, 128);
            tc::mma_f16(d, a_hi, b_hi, idesc, ks > 0 ? 1u : 0u);
            if constexpr (Cfg::kSplit) {
              const uint64_t a_lo = tc::smem_desc(ya + ypart + ks * 256, 128, a_sbo);
              const uint64_t b_lo = tc::smem_desc(wb + wpart + ks * 2 * b_lbo, b_lbo, 128);
              tc::mma_f16(d, a_lo, b_hi, idesc, 1u);
              tc::mma_f16(d, a_hi, b_lo, idesc, 1u);
            }
          }
          tc::mma_commit(&w_empty[s]);
          tc::mma_commit(&t_full[j]);
        }
        tc::mma_commit(&y_empty[yb]);
      }
    }
  } else if (warp < 4) {
    // ---- y-tile producers (64 threads) -------------------------------------
    const int pt = threadIdx.x - 64;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const int yb = it & 1;
      if (!warp_wait(&y_empty[yb], ((it >> 1) & 1) ^ 1, abort_flag)) {
        fail(abort_flag, p.status, 13);
        break;
      }
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      uint8_t* ys = smem + L.y + yb * L.y_bytes;
      // 16 eight-pixel groups x Cp channels; one 16-byte smem row each.
      // Loads are issued in batches of 8 independent rows per thread so the
      // global latency is paid once per batch, not once per row.
      constexpr int kBatch = 8;
      for (int base = pt; base < 16 * Cp; base += 64 * kBatch) {
        float v[kBatch][8];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int item = base + u * 64;
          const int c = item % Cp;
          const int g = item / Cp;             // 8-pixel group: row g/2, half g%2
          if (item < 16 * Cp)
            load8<T>(static_cast<const T*>(p.y), n, c, C, H, W, h0 + (g >> 1), w0 + (g & 1) * 8,
                     v[u]);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int item = base + u * 64;
          if (item >= 16 * Cp) break;
          const int c = item % Cp;
          const int g = item / Cp;
          // MN-major interleaved: group g at g*Cp*16, channel c at (c/8)*128 + (c%8)*16
          const uint32_t off = g * Cp * 16 + (c >> 3) * 128 + (c & 7) * 16;
          store8_split<Op, Cfg::kSplit>(ys + off, ys + kTileM * Cp * 2 + off, v[u]);
        }
      }
      tc::fence_proxy_async_smem();
      tc::mbar_arrive(&y_full[yb]);
    }
  } else {
    // ---- epilogue warpgroups -----------------------------------------------
    const int ew = warp - 4;
    const int wg = ew >> 2;
    const int quad = warp & 3;               // TMEM lane quadrant of this warp
    const int m = quad * 32 + lane;          // pixel row of the MMA tile
    const T* x = static_cast<const T*>(p.x);
    T* out = static_cast<T*>(p.out);
    uint32_t tq = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      const int h = h0 + (m >> 4);
      const int w = w0 + (m & 15);
      const bool px_ok = (h < H) && (w < W);
      const size_t pix = (size_t)h * W + w;
      const T* xn = x + (size_t)n * C * P;
      T* on = out + (size_t)n * 4 * C * P;
      bool failed = false;
      for (int cg = 0; cg < Cp / 16 && !failed; ++cg) {
        for (int b = 0; b < 3; ++b) {
          const bool mine = ((cg * 3 + b) % Cfg::kEpiWG) == wg;
          if (!mine) {
            tq += KS;
            continue;
          }
          const int d = p.d[b];
          float acc[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
          for (int ki = 0; ki < KS; ++ki, ++tq) {
            const int dy = (ki - r) * d;
            const bool row_ok = px_ok && (unsigned)(h + dy) < (unsigned)H;
            const T* xrow = xn + (size_t)(cg * 16) * P + (ptrdiff_t)(pix + (ptrdiff_t)dy * W);
            // x neighbours of tap (ki, kj) for the 16 channels of the group;
            // independent of the MMA result, so the first batch is issued
            // before waiting for the accumulator.
            auto load_x = [&](int kj, float (&xv)[16]) {
              const int dx = (kj - r) * d;
              const bool ok = row_ok && (unsigned)(w + dx) < (unsigned)W;
#pragma unroll
              for (int cl = 0; cl < 16; ++cl) {
                const bool okc = ok && (cg * 16 + cl < C);
                xv[cl] = okc ? to_f32<T>(__ldg(xrow + (size_t)cl * P + dx)) : 0.f;
              }
            };
            float xv[16];
            load_x(0, xv);
            const int j = tq % NB;
            if (!warp_wait(&t_full[j], (tq / NB) & 1, abort_flag)) {
              fail(abort_flag, p.status, 14);
              failed = true;
              break;
            }
            tc::tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + j * kN;
#pragma unroll
            for (int kj = 0; kj < KS; ++kj) {
              float dv[16];
              tc::tmem_ld16(taddr + kj * 16, dv);
              float xnext[16];
              if (kj + 1 < KS) load_x(kj + 1, xnext);
              tc::tmem_ld_wait();
              const float* bs = bias_s + (size_t)(b * C + cg * 16) * KK + ki * KS + kj;
#pragma unroll
              for (int cl = 0; cl < 16; ++cl) {
                const float bv = (cg * 16 + cl < C) ? bs[cl * KK] : 0.f;
                const float g = IoTraits<T>::round_io(dv[cl] + bv);
                acc[cl] = fmaf(g, xv[cl], acc[cl]);
              }
              if (kj + 1 < KS) {
#pragma unroll
                for (int cl = 0; cl < 16; ++cl) xv[cl] = xnext[cl];
              }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&t_empty[j]);
          }
          if (failed) break;
          if (px_ok) {
#pragma unroll
            for (int cl = 0; cl < 16; ++cl) {
              const int c = cg * 16 + cl;
              if (c < C) on[(size_t)((b + 1) * C + c) * P + pix] = from_f32<T>(acc[cl]);
            }
          }
        }
      }
      if (failed) break;
      // passthrough out[:, 0:C] = x, channels split across the warpgroups
      if (px_ok) {
        for (int c = wg; c < C; c += Cfg::kEpiWG) on[(size_t)c * P + pix] = xn[(size_t)c * P + pix];
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
int launch(const FwdParams& prm, cudaStream_t st) {
  using Cfg = FwdCfg<T, KS>;
  const FwdSmem L = fwd_smem_layout<T, KS>(prm.C, prm.Cp);
  auto fn = gencat_fwd_kernel<T, KS>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  const int grid = prm.num_tiles < num_sms() ? prm.num_tiles : num_sms();
  fn<<<grid, Cfg::kThreads, L.total, st>>>(prm);
  DDPM_CHECK_LAUNCH("gencat_fwd_kernel");
  return DDPM_OK;
}

template <typename T>
int dispatch(int ks, const FwdParams& prm, cudaStream_t st) {
  switch (ks) {
    case 1: return launch<T, 1>(prm, st);
    case 3: return launch<T, 3>(prm, st);
  }
  return set_error(DDPM_ERR_UNSUPPORTED, "fused generator: kernel_size %d not supported", ks);
}

}  // namespace

int gencat_fwd(const void* x, const void* y, const void* wpack, const void* bias, void* out,
               int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt,
               cudaStream_t st) {
  int rc = gencat::check_shape(n, c, h, w, ks, d0, d1, d2, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG(x && y && wpack && bias && out, "null pointer");
  FwdParams prm{};
  prm.x = x;
  prm.y = y;
  prm.wpack = wpack;
  prm.bias = bias;
  prm.out = out;
  prm.N = n;
  prm.C = c;
  prm.H = h;
  prm.W = w;
  prm.Cp = gencat::padded_channels(c);
  prm.d[0] = d0;
  prm.d[1] = d1;
  prm.d[2] = d2;
  prm.tiles_w = (w + gencat::kTileW - 1) / gencat::kTileW;
  prm.tiles_h = (h + gencat::kTileH - 1) / gencat::kTileH;
  prm.num_tiles = n * prm.tiles_w * prm.tiles_h;
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
