// Native weight and bias gradient of the 3x3 fuse convolution (the cuDNN
// wgrad of `self.fuse`, reference `triton_impl.py:294, 392`):
//
//   dW[o, i, ky, kx] = sum_q cat[i, q] * dout[o, q - (ky - 1, kx - 1)]   (dout zero-padded)
//   db[o]            = sum_p dout[o, p]
//
// CTA = (128-channel input chunk ic, kernel row ky) x spatial split. For each
// row tile q (row h, columns w0 .. w0+TW-1; TW = 128, or 64 for FP32 whose
// operands are twice as large) of its split, one MMA per 16-pixel K step:
//   A = cat[ic*128 .. +127, h, w0 .. w0+TW-1], K-major [pixel group][channel]
//       [8 pixels]: every 16-byte operand row is 8 consecutive pixels of one
//       channel, read straight from NCHW (no transpose);
//   B = dout row h - ky + 1 as three MN-major copies, N = (kx, o): copy kx
//       holds dout[o, h - ky + 1, w0 + q + 1 - kx] at row q, so the three kx
//       taps share one N = 3*Np instruction (full tensor rate; three N = Np
//       instructions run at about half of it). The copies are written with
//       stmatrix.trans from 8-pixel vector loads of 8 channels;
//   D (128 input channels x 3*Np columns in TMEM) += A . B over the tile.
// D accumulates over the split's tiles and is written as FP32 partials
// [split][ic][ky][128][3*Np]; a second kernel sums the splits into dW. While
// the tiles stream, the drain warps of the (ic 0, ky 1) CTA of every split sum
// its dout rows per channel into db partials [split][Np].
#include "common.cuh"
#include "tc.cuh"
#include "gencat.cuh"
#include "fuseconv.cuh"

namespace ddpm {
namespace {

using namespace gencat;

template <typename T>
struct WgCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  static constexpr int kTW = kSplit ? 64 : 128;     // tile width (pixels = GEMM K per tile)
  static constexpr int kKSteps = kTW / 16;
  static constexpr int kStages = 2;
  static constexpr int kProducers = 256;
  static constexpr int kProducerWarps = kProducers / 32;
  static constexpr int kAItems = 128 * (kTW / 8) / kProducers;  // 16-byte A rows per thread
  // staged dout columns: w0 - 8 .. w0 - 8 + 32 * kBChunks - 1 (covers w0 - 1 .. w0 + TW)
  static constexpr int kBChunks = (kTW + 9 + 31) / 32;
  static constexpr int kFirstProducerWarp = 2;
  static constexpr int kFirstDrainWarp = kFirstProducerWarp + kProducerWarps;
  static constexpr int kThreads = 32 * (kFirstDrainWarp + 4);
};

struct WgParams {
  const void* cat;   // [N, Cin, H, W]
  const void* dout;  // [N, Cout, H, W]
  float* partial;    // [splits][nic][3][128][3*Np]
  float* db_partial; // [splits][Np] or null
  int N, H, W, Cin, Cout, Np, nic;
  int tiles_w, num_tiles, splits;
  int vec;  // W % 8 == 0 and 16-byte aligned tensors: branch-free vector loads
  uint32_t a_part, a_bytes, b_part, b_bytes;
  int* status;
};

struct WgSmem {
  uint32_t a, b, junk, bars, total;
};

__host__ __device__ inline WgSmem wg_smem_layout(const WgParams& p, int stages) {
  WgSmem L;
  L.a = 0;
  L.b = L.a + stages * p.a_bytes;
  L.junk = L.b + stages * p.b_bytes;  // 32 x 16 B sink for B rows outside every window
  L.bars = L.junk + 512;
  L.total = L.bars + 8 * (2 * stages + 1);
  return L;
}

template <typename T>
__device__ __forceinline__ void wg_tile_coords(const WgParams& p, int tile, int& n, int& h, int& w0) {
  const int per_img = p.H * p.tiles_w;
  n = tile / per_img;
  h = (tile % per_img) / p.tiles_w;
  w0 = (tile % p.tiles_w) * WgCfg<T>::kTW;
}

template <typename T>
__global__ void __launch_bounds__(WgCfg<T>::kThreads, 1) fuseconv_wgrad_kernel(const WgParams p) {
  using Cfg = WgCfg<T>;
  using Op = typename IoTraits<T>::Op;
  constexpr int S = Cfg::kStages;
  constexpr int TW = Cfg::kTW;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const WgSmem L = wg_smem_layout(p, S);
  const int H = p.H, W = p.W, Np = p.Np;
  const size_t P = (size_t)H * W;
  const int unit = blockIdx.x % (p.nic * 3);
  const int split = blockIdx.x / (p.nic * 3);
  const int ic = unit / 3, ky = unit % 3;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* s_full = bars;        // [S] producers
  uint64_t* s_empty = bars + S;   // [S] MMA commit
  uint64_t* d_done = bars + 2 * S;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 256);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&s_full[i], Cfg::kProducers);
      tc::mbar_init(&s_empty[i], 1);
    }
    tc::mbar_init(d_done, 1);
    tc::fence_mbar_init();
    abort_s = 0;
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  volatile int* abort_flag = &abort_s;

  if (warp == 1) {
    // ---- MMA issuer -----------------------------------------------------------
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(128, 3 * Np, IoTraits<T>::kBf16, false, true);
      constexpr uint64_t a_step = (2 * 128 * 16) >> 4;  // one K step = 2 pixel groups of A
      constexpr uint64_t b_step = (16 * 16) >> 4;       // 16 pixel rows of B
      const uint64_t a_lo = p.a_part >> 4, b_lo = p.b_part >> 4;
      uint32_t sq = 0;
      bool first = true;
      for (int tile = split; tile < p.num_tiles; tile += p.splits, ++sq) {
        const int sb = sq % S;
        if (!tc::mbar_wait(&s_full[sb], (sq / S) & 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 70);
          goto done;
        }
        tc::tc_fence_after();
        const uint64_t ad = tc::smem_desc(tc::smem_u32(smem + L.a + sb * p.a_bytes), 128 * 16, 128);
        const uint64_t bd = tc::smem_desc(tc::smem_u32(smem + L.b + sb * p.b_bytes), 128, TW * 16);
        for (int ks = 0; ks < Cfg::kKSteps; ++ks) {
          const uint64_t a_k = ad + ks * a_step, b_k = bd + ks * b_step;
          tc::mma_f16(tmem_base, a_k, b_k, idesc, (!first || ks > 0) ? 1u : 0u);
          if constexpr (Cfg::kSplit) {
            tc::mma_f16(tmem_base, a_k + a_lo, b_k, idesc, 1u);
            tc::mma_f16(tmem_base, a_k, b_k + b_lo, idesc, 1u);
          }
        }
        tc::mma_commit(&s_empty[sb]);
        first = false;
      }
      tc::mma_commit(d_done);
    }
  } else if (warp >= Cfg::kFirstProducerWarp && warp < Cfg::kFirstDrainWarp) {
    // ---- producers (256 threads) ---------------------------------------------
    const int pt = threadIdx.x - 32 * Cfg::kFirstProducerWarp;
    const int pw = pt >> 5;
    const T* cat = static_cast<const T*>(p.cat);
    const T* dout = static_cast<const T*>(p.dout);
    const int ngroups_o = Np / 8;
    const int b_tasks = ngroups_o * Cfg::kBChunks;  // (og, 32-column chunk)
    // stmatrix row address: lane 8i + r writes column r of matrix i, which is
    // the staged pixel 8 * (r / 2) + 2 * i + r % 2 of the lane group's chunk.
    const int pofs = 8 * ((lane & 7) >> 1) + 2 * (lane >> 3) + (lane & 1);
    const uint32_t junk = tc::smem_u32(smem + L.junk) + lane * 16;
    uint32_t sq = 0;
    for (int tile = split; tile < p.num_tiles && !*abort_flag; tile += p.splits, ++sq) {
      int n, h, w0;
      wg_tile_coords<T>(p, tile, n, h, w0);
      const int sb = sq % S;
      if (!warp_wait(&s_empty[sb], ((sq / S) & 1) ^ 1, abort_flag)) {
        fail(abort_flag, p.status, 71);
        break;
      }
      uint8_t* a = smem + L.a + sb * p.a_bytes;
      const uint32_t b = tc::smem_u32(smem + L.b + sb * p.b_bytes);
      // A: item = (input channel il, pixel group g), one 16-byte operand row. A
      // quarter-warp covers 8 consecutive channels of one pixel group (8
      // consecutive smem rows: no bank conflict).
      const T* cat_n = cat + (size_t)n * p.Cin * P;
      const int hr = h - ky + 1;
      const T* dout_n = dout + (size_t)n * p.Cout * P;
      Raw8<T> va[Cfg::kAItems];
      Raw8<T> vb[Cfg::kBChunks];
      if (p.vec) {
        // W % 8 == 0 and aligned tensors: every 8-pixel vector is wholly inside
        // or wholly outside the image. All loads are issued unconditionally
        // (invalid items from the plane base) and masked afterwards.
        bool oka[Cfg::kAItems], okb[Cfg::kBChunks];
#pragma unroll
        for (int k = 0; k < Cfg::kAItems; ++k) {
          const int combo = pw * Cfg::kAItems + k;
          const int il = (combo & 15) * 8 + (lane & 7);
          const int g = (combo >> 4) * 4 + (lane >> 3);
          const int c = ic * 128 + il;
          oka[k] = c < p.Cin && w0 + g * 8 < W;
          const T* src = cat_n + (size_t)c * P + (size_t)h * W + w0 + g * 8;
          va[k] = ldg_raw8<T>(oka[k] ? src : cat);
        }
#pragma unroll
        for (int k = 0; k < Cfg::kBChunks; ++k) {
          const int task = pw + k * Cfg::kProducerWarps;
          const int og = task / Cfg::kBChunks, c = task - og * Cfg::kBChunks;
          const int o = og * 8 + (lane >> 2);
          const int col = w0 - 8 + 32 * c + 8 * (lane & 3);
          okb[k] = task < b_tasks && o < p.Cout && hr >= 0 && hr < H && col >= 0 && col < W;
          const T* src = dout_n + (size_t)o * P + (size_t)hr * W + col;
          vb[k] = ldg_raw8<T>(okb[k] ? src : dout);
        }
#pragma unroll
        for (int k = 0; k < Cfg::kAItems; ++k)
          if (!oka[k]) va[k].zero();
#pragma unroll
        for (int k = 0; k < Cfg::kBChunks; ++k)
          if (!okb[k]) vb[k].zero();
      } else {
#pragma unroll
        for (int k = 0; k < Cfg::kAItems; ++k) {
          const int combo = pw * Cfg::kAItems + k;
          const int il = (combo & 15) * 8 + (lane & 7);
          const int g = (combo >> 4) * 4 + (lane >> 3);
          const int c = ic * 128 + il;
          if (c < p.Cin)
            va[k] = load_raw8<T>(cat_n + (size_t)c * P, H, W, h, w0 + g * 8);
          else
            va[k].zero();
        }
        // B: warp task = (output-channel group og, chunk of 32 staged columns);
        // lane = (channel og*8 + lane/4, 8 columns from 8 * (lane % 4)).
#pragma unroll
        for (int k = 0; k < Cfg::kBChunks; ++k) {
          const int task = pw + k * Cfg::kProducerWarps;
          const int og = task / Cfg::kBChunks, c = task - og * Cfg::kBChunks;
          const int o = og * 8 + (lane >> 2);
          if (task < b_tasks && o < p.Cout)
            vb[k] = load_raw8<T>(dout_n + (size_t)o * P, H, W, hr, w0 - 8 + 32 * c + 8 * (lane & 3));
          else
            vb[k].zero();
        }
      }
#pragma unroll
      for (int k = 0; k < Cfg::kAItems; ++k) {
        const int combo = pw * Cfg::kAItems + k;
        const int il = (combo & 15) * 8 + (lane & 7);
        const int g = (combo >> 4) * 4 + (lane >> 3);
        const uint32_t off = (g * 128 + il) * 16;
        store_raw8<T, Op, Cfg::kSplit>(a + off, a + p.a_part + off, va[k]);
      }
#pragma unroll
      for (int k = 0; k < Cfg::kBChunks; ++k) {
        const int task = pw + k * Cfg::kProducerWarps;
        if (task < b_tasks) {  // warp-uniform
          const int og = task / Cfg::kBChunks, c = task - og * Cfg::kBChunks;
          uint32_t hi[4], lo[4];
          raw8_words<T, Op, Cfg::kSplit>(vb[k], hi, lo);
          // staged column j = 32c + pofs is dout column w0 - 8 + j; copy kx
          // keeps it at row q = j - 9 + kx when 0 <= q < TW.
#pragma unroll
          for (int kx = 0; kx < 3; ++kx) {
            const int q = 32 * c + pofs - 9 + kx;
            const bool in = q >= 0 && q < TW;
            const uint32_t row = b + ((kx * ngroups_o + og) * TW + q) * 16;
            tc::stmatrix_x4_trans(in ? row : junk, hi[0], hi[1], hi[2], hi[3]);
            if constexpr (Cfg::kSplit)
              tc::stmatrix_x4_trans(in ? row + p.b_part : junk, lo[0], lo[1], lo[2], lo[3]);
          }
        }
      }
      tc::fence_proxy_async_smem();
      tc::mbar_arrive(&s_full[sb]);
    }
  } else if (warp >= Cfg::kFirstDrainWarp) {
    // ---- drain (128 threads, lane = input channel of the chunk) -------------------
    const int quad = warp & 3;
    const int dt = (warp - Cfg::kFirstDrainWarp) * 32 + lane;
    if (p.db_partial != nullptr && ic == 0 && ky == 1) {
      // db partial of this split: thread = (channel dt/2, half of each tile row)
      const T* dout = static_cast<const T*>(p.dout);
      const int o = dt >> 1, half = dt & 1;
      float acc = 0.f;
      if (o < p.Cout) {
        for (int tile = split; tile < p.num_tiles && !*abort_flag; tile += p.splits) {
          int n, h, w0;
          wg_tile_coords<T>(p, tile, n, h, w0);
          const T* plane = dout + ((size_t)n * p.Cout + o) * P;
          Raw8<T> v[TW / 16];
          if (p.vec) {
            bool ok[TW / 16];
#pragma unroll
            for (int j = 0; j < TW / 16; ++j) {
              const int col = w0 + half * (TW / 2) + 8 * j;
              ok[j] = col < W;
              v[j] = ldg_raw8<T>(ok[j] ? plane + (size_t)h * W + col : plane);
            }
#pragma unroll
            for (int j = 0; j < TW / 16; ++j)
              if (!ok[j]) v[j].zero();
          } else {
#pragma unroll
            for (int j = 0; j < TW / 16; ++j)
              v[j] = load_raw8<T>(plane, H, W, h, w0 + half * (TW / 2) + 8 * j);
          }
#pragma unroll
          for (int j = 0; j < TW / 16; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc += v[j].get(e);
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (half == 0 && o < p.Cout) p.db_partial[(size_t)split * Np + o] = acc;
    }
    const int il = quad * 32 + lane;
    if (warp_wait(d_done, 0, abort_flag)) {
      tc::tc_fence_after();
      float* dst = p.partial + ((((size_t)split * p.nic + ic) * 3 + ky) * 128 + il) * (3 * Np);
      for (int c0 = 0; c0 < 3 * Np; c0 += 16) {
        float v[16];
        tc::tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + c0, v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 16; k += 4)
          *reinterpret_cast<float4*>(dst + c0 + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
      }
    } else {
      fail(abort_flag, p.status, 72);
    }
  }
done:
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 256);
  }
}

// dW[o, i, ky, kx] = sum over splits of the partials (threads walk the
// partials' own layout, output channel fastest, so the split-strided reads
// coalesce; the dW writes scatter), and db[o] = sum over splits of the db
// partials (items past the dW part).
template <typename T>
__global__ void fuseconv_wgrad_reduce_kernel(const float* __restrict__ partial,
                                             const float* __restrict__ db_partial,
                                             T* __restrict__ dw, T* __restrict__ db, int Cin,
                                             int Cout, int Np, int nic, int splits) {
  const long long stride = (long long)nic * 3 * 128 * 3 * Np;
  const long long total = stride + (db != nullptr ? Cout : 0);
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    if (idx >= stride) {
      const int o = (int)(idx - stride);
      float acc = 0.f;
      for (int s = 0; s < splits; ++s) acc += db_partial[(size_t)s * Np + o];
      db[o] = from_f32<T>(acc);
      continue;
    }
    const int col = (int)(idx % (3 * Np));
    const long long r = idx / (3 * Np);  // (ic * 3 + ky) * 128 + il
    const int il = (int)(r % 128);
    const int ky = (int)((r / 128) % 3);
    const int ic = (int)(r / (3 * 128));
    const int kx = col / Np, o = col - kx * Np;
    const int i = ic * 128 + il;
    if (o >= Cout || i >= Cin) continue;
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += partial[idx + s * stride];
    dw[(((size_t)o * Cin + i) * 3 + ky) * 3 + kx] = from_f32<T>(acc);
  }
}

struct WgPlan {
  int Np, nic, splits, tiles_w, num_tiles;
  size_t partial_bytes, ws_bytes;
};

WgPlan plan_wgrad(int n, int cin, int cout, int h, int w, int tw) {
  WgPlan q;
  q.Np = (cout + 15) / 16 * 16;
  q.nic = (cin + 127) / 128;
  q.tiles_w = (w + tw - 1) / tw;
  q.num_tiles = n * h * q.tiles_w;
  int sp = num_sms() / (q.nic * 3);
  if (sp < 1) sp = 1;
  if (sp > q.num_tiles) sp = q.num_tiles;
  q.splits = sp;
  q.partial_bytes = (size_t)sp * q.nic * 3 * 128 * 3 * q.Np * sizeof(float);
  q.ws_bytes = q.partial_bytes + (size_t)sp * q.Np * sizeof(float);
  return q;
}

int wgrad_tile_width(int dt) { return dt == DDPM_F32 ? WgCfg<float>::kTW : WgCfg<__half>::kTW; }

template <typename T>
int run_wgrad(const WgParams& prm, void* dw, void* db, cudaStream_t st) {
  using Cfg = WgCfg<T>;
  const WgSmem L = wg_smem_layout(prm, Cfg::kStages);
  auto fn = fuseconv_wgrad_kernel<T>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  fn<<<prm.nic * 3 * prm.splits, Cfg::kThreads, L.total, st>>>(prm);
  DDPM_CHECK_LAUNCH("fuseconv_wgrad_kernel");
  const long long total = (long long)prm.nic * 3 * 128 * 3 * prm.Np + prm.Cout;
  const long long want = (total + 255) / 256;
  fuseconv_wgrad_reduce_kernel<T><<<(int)(want < 2048 ? want : 2048), 256, 0, st>>>(
      prm.partial, prm.db_partial, static_cast<T*>(dw), static_cast<T*>(db), prm.Cin, prm.Cout,
      prm.Np, prm.nic, prm.splits);
  DDPM_CHECK_LAUNCH("fuseconv_wgrad_reduce_kernel");
  return DDPM_OK;
}

}  // namespace

size_t fuseconv_wgrad_workspace_bytes(int n, int cin, int cout, int h, int w) {
  if (n < 1 || h < 1 || w < 1 || cin < 1 || cout < 1 || cin > fuseconv::kMaxCin ||
      cout > fuseconv::kMaxCout)
    return 0;
  // the larger of the FP32 and 16-bit plans (the split count is shared)
  const WgPlan a = plan_wgrad(n, cin, cout, h, w, WgCfg<float>::kTW);
  const WgPlan b = plan_wgrad(n, cin, cout, h, w, WgCfg<__half>::kTW);
  return a.ws_bytes > b.ws_bytes ? a.ws_bytes : b.ws_bytes;
}

int fuseconv_wgrad(const void* cat, const void* gout, void* gw, void* gb, void* ws, size_t ws_bytes,
                   int n, int cin, int cout, int h, int w, int dt, cudaStream_t st) {
  DDPM_CHECK_ARG(n >= 1 && h >= 1 && w >= 1 && cin >= 1 && cout >= 1, "sizes must be positive");
  DDPM_CHECK_ARG(dtype_size(dt) > 0, "unknown dtype code %d", dt);
  if (cin > fuseconv::kMaxCin || cout > fuseconv::kMaxCout)
    return set_error(DDPM_ERR_UNSUPPORTED, "native fuse conv supports Cin <= %d, Cout <= %d",
                     fuseconv::kMaxCin, fuseconv::kMaxCout);
  DDPM_CHECK_ARG(cat && gout && gw, "null pointer");
  const WgPlan q = plan_wgrad(n, cin, cout, h, w, wgrad_tile_width(dt));
  if (ws == nullptr || ws_bytes < q.ws_bytes)
    return set_error(DDPM_ERR_WORKSPACE, "workspace too small (%zu < %zu)", ws_bytes, q.ws_bytes);
  DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(ws) & 15u) == 0, "workspace must be 16-byte aligned");
  int* status = nullptr;
  int rc = gencat::status_ptr(&status);
  if (rc) return rc;
  const bool split = dt == DDPM_F32;
  const int tw = wgrad_tile_width(dt);
  WgParams prm{};
  prm.cat = cat;
  prm.dout = gout;
  prm.partial = static_cast<float*>(ws);
  prm.db_partial = gb != nullptr
                       ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + q.partial_bytes)
                       : nullptr;
  prm.N = n;
  prm.H = h;
  prm.W = w;
  prm.Cin = cin;
  prm.Cout = cout;
  prm.Np = q.Np;
  prm.nic = q.nic;
  prm.tiles_w = q.tiles_w;
  prm.num_tiles = q.num_tiles;
  prm.splits = q.splits;
  prm.vec = (w % 8) == 0 &&
            ((reinterpret_cast<uintptr_t>(cat) | reinterpret_cast<uintptr_t>(gout)) & 15u) == 0;
  prm.a_part = (uint32_t)(tw / 8) * 128 * 16;            // pixel groups x 128 channels x 16 B
  prm.a_bytes = prm.a_part * (split ? 2 : 1);
  prm.b_part = (uint32_t)(3 * (q.Np / 8)) * tw * 16;     // [kx][o/8][TW rows][8]
  prm.b_bytes = prm.b_part * (split ? 2 : 1);
  prm.status = status;
  switch (dt) {
    case DDPM_BF16: return run_wgrad<__nv_bfloat16>(prm, gw, gb, st);
    case DDPM_F16: return run_wgrad<__half>(prm, gw, gb, st);
    default: return run_wgrad<float>(prm, gw, gb, st);
  }
}

}  // namespace ddpm
