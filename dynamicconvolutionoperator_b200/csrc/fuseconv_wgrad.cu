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
//
// TMA path (W % 8 == 0, 16-byte aligned tensors): a pre-pass writes dout
// channel-last as operand planes [n][h][o/8][w][8] (bf16 hi + lo planes for
// FP32) and per-(row, 32-column strip) db partials. The main kernel then has
// no load warps: one thread issues, per tile and several tiles ahead, the A
// copy (16-bit: box 64 px x 128 channels, 128-byte swizzle = the canonical
// K-major SW128 operand) and three B copies, one per kx (box TW px x Np
// channels of one staged row, x coordinate w0 + 1 - kx px, zero fill outside
// the image), so the three taps stay one N = 3*Np instruction. (One B copy
// read through three shifted N = Np windows moves fewer bytes from L2 but
// re-reads A from shared memory once per tap, and measured slower.) All A
// stages sit in one shared-memory region and all B stages in another, far
// apart. FP32 A
// arrives raw (128-byte swizzled rows of 32 px) in a separate ring and four
// converter warps split it into the bf16 hi / lo operand.
#include "common.cuh"
#include "tc.cuh"
#include "gencat.cuh"
#include "fuseconv.cuh"
#include "tmap.cuh"

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
  float* db_mid;     // level-2 rows of the db reduction
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

// dW[o, i, ky, kx] = sum over splits of the partials. Blocks below `dw_blocks`
// walk the partials' own layout four columns (output channels) per thread, so
// the split-strided float4 reads coalesce; the dW writes scatter. The
// `db_blocks` blocks after them reduce the db partials [parts][Np] in two
// levels: block j sums a contiguous range of parts for every output channel
// (64 consecutive threads read one 64-channel row, so the reads coalesce; four
// row lanes are combined in a fixed order) into db_mid[j][Np]; the final
// kernel sums db_mid over j in order. Deterministic, like the dW sum.
constexpr int kDbMidBlocks = 128;  // most level-1 db blocks (db_mid rows)

template <typename T>
__global__ void __launch_bounds__(256) fuseconv_wgrad_reduce_kernel(
    const float* __restrict__ partial, const float* __restrict__ db_part,
    float* __restrict__ db_mid, T* __restrict__ dw, int Cin, int Cout, int Np, int nic,
    int splits, int db_parts, int dw_blocks, int db_blocks) {
  if ((int)blockIdx.x >= dw_blocks) {
    const int j = blockIdx.x - dw_blocks;
    const int per = (db_parts + db_blocks - 1) / db_blocks;
    const int k0 = j * per, k1 = min(db_parts, k0 + per);
    const int o = threadIdx.x & 63, lane4 = threadIdx.x >> 6;  // Np <= 64
    float acc = 0.f;
    if (o < Np)
      for (int k = k0 + lane4; k < k1; k += 4) acc += db_part[(size_t)k * Np + o];
    __shared__ float red[4][64];
    red[lane4][o] = acc;
    __syncthreads();
    if (threadIdx.x < Np)
      db_mid[(size_t)j * Np + threadIdx.x] =
          ((red[0][threadIdx.x] + red[1][threadIdx.x]) + red[2][threadIdx.x]) + red[3][threadIdx.x];
    return;
  }
  const long long stride = (long long)nic * 3 * 128 * 3 * Np;  // floats per split
  const long long quads = stride / 4;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < quads;
       q += (long long)dw_blocks * blockDim.x) {
    const long long idx = q * 4;
    const int col = (int)(idx % (3 * Np));
    const long long r = idx / (3 * Np);  // (ic * 3 + ky) * 128 + il
    const int il = (int)(r % 128);
    const int ky = (int)((r / 128) % 3);
    const int ic = (int)(r / (3 * 128));
    const int i = ic * 128 + il;
    if (i >= Cin) continue;
    const float4* src = reinterpret_cast<const float4*>(partial + idx);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int s = 0; s < splits; ++s) {
      const float4 v = src[(size_t)s * (stride / 4)];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int kx = (col + e) / Np, o = (col + e) - kx * Np;
      if (o < Cout) dw[(((size_t)o * Cin + i) * 3 + ky) * 3 + kx] = from_f32<T>(a4[e]);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(64) fuseconv_db_final_kernel(const float* __restrict__ db_mid,
                                                               T* __restrict__ db, int Cout,
                                                               int Np, int rows) {
  const int o = threadIdx.x;
  if (o >= Cout) return;
  float acc = 0.f;
  for (int j = 0; j < rows; ++j) acc += db_mid[(size_t)j * Np + o];
  db[o] = from_f32<T>(acc);
}

template <typename T>
int launch_wgrad_reduce(const float* partial, const float* db_part, float* db_mid, void* dw,
                        void* db, int cin, int cout, int Np, int nic, int splits, int db_parts,
                        cudaStream_t st) {
  const long long quads = (long long)nic * 3 * 128 * 3 * Np / 4;
  long long blocks = (quads + 255) / 256;
  if (blocks > 1024) blocks = 1024;
  const int dw_blocks = (int)blocks;
  int db_blocks = 0;
  if (db != nullptr) {
    db_blocks = (db_parts + 255) / 256;
    if (db_blocks > kDbMidBlocks) db_blocks = kDbMidBlocks;
  }
  fuseconv_wgrad_reduce_kernel<T><<<dw_blocks + db_blocks, 256, 0, st>>>(
      partial, db_part, db_mid, static_cast<T*>(dw), cin, cout, Np, nic, splits, db_parts,
      dw_blocks, db_blocks);
  DDPM_CHECK_LAUNCH("fuseconv_wgrad_reduce_kernel");
  if (db != nullptr) {
    fuseconv_db_final_kernel<T><<<1, 64, 0, st>>>(db_mid, static_cast<T*>(db), cout, Np,
                                                  db_blocks);
    DDPM_CHECK_LAUNCH("fuseconv_db_final_kernel");
  }
  return DDPM_OK;
}

// ------------------------------------------------------------- TMA path ----
// Pre-pass: dout [N, Cout, H, W] -> operand planes [N][H][Np/8][W][8] of the
// MMA type (FP32: bf16 hi plane and residual plane), channels >= Cout zero;
// db partial of the block's 64 columns per channel ->
// dbp[(n*H + h)*strips + strip][Np]. Block = (image row, 64-column strip):
// 8 lanes read 8-pixel vectors covering 64 contiguous pixels of one channel,
// a padded shared tile transposes, and each thread writes 16-byte rows of 8
// channels (consecutive lanes = consecutive pixels).
constexpr int kPackCols = 64;

template <typename T>
__global__ void __launch_bounds__(256) fuseconv_dout_pack_kernel(const T* __restrict__ dout,
                                                                 uint4* __restrict__ hi,
                                                                 uint4* __restrict__ lo,
                                                                 float* __restrict__ dbp, int H,
                                                                 int W, int Cout, int Np) {
  using Op = typename IoTraits<T>::Op;
  constexpr bool kSplit = IoTraits<T>::kSplit;
  __shared__ float tile[fuseconv::kMaxCout][kPackCols + 1];
  const int nh = blockIdx.x, n = nh / H, h = nh - n * H;
  const int w0 = blockIdx.y * kPackCols;
  const size_t P = (size_t)H * W;
  const T* src = dout + (size_t)n * Cout * P;
  // load: item = (channel c, 8-pixel group g)
  for (int item = threadIdx.x; item < Np * (kPackCols / 8); item += blockDim.x) {
    const int g = item & 7, c = item >> 3;
    Raw8<T> v;
    if (c < Cout)
      v = load_raw8<T>(src + (size_t)c * P, H, W, h, w0 + g * 8);
    else
      v.zero();
#pragma unroll
    for (int e = 0; e < 8; ++e) tile[c][g * 8 + e] = v.get(e);
  }
  __syncthreads();
  // db partial: 4 threads per channel, 16 columns each
  {
    const int c = threadIdx.x >> 2, q = threadIdx.x & 3;
    float acc = 0.f;
    if (c < Np) {
#pragma unroll
      for (int x = 0; x < 16; ++x) acc += tile[c][q * 16 + x];
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (c < Np && q == 0) dbp[((size_t)nh * gridDim.y + blockIdx.y) * Np + c] = acc;
  }
  const int ng = Np / 8;
  for (int idx = threadIdx.x; idx < ng * kPackCols; idx += blockDim.x) {
    const int og = idx / kPackCols, x = idx - og * kPackCols;
    if (w0 + x >= W) continue;
    unsigned long long pr[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[e] = f2_pack(tile[og * 8 + 2 * e][x], tile[og * 8 + 2 * e + 1][x]);
    const size_t dst = ((size_t)nh * ng + og) * W + w0 + x;
    uint4 vh, vl;
    store8x2_split<Op, kSplit>(reinterpret_cast<uint8_t*>(&vh), reinterpret_cast<uint8_t*>(&vl), pr);
    hi[dst] = vh;
    if constexpr (kSplit) lo[dst] = vl;
  }
}

// The same pre-pass for 16-bit dout, transposed in its own type (no FP32
// round trip): a [channel][64 + 8 px] tile of 16-bit values (144-byte rows,
// 16-byte aligned), each thread's two 16-byte loads issued before its first
// shared store; the db partial sums the same FP32 values in the same order.
template <typename T>
__global__ void __launch_bounds__(256) fuseconv_dout_pack16_kernel(const T* __restrict__ dout,
                                                                   uint4* __restrict__ hi,
                                                                   float* __restrict__ dbp,
                                                                   int H, int W, int Cout, int Np) {
  constexpr int kGroups = kPackCols / 8;
  constexpr int kItems = (fuseconv::kMaxCout * kGroups + 255) / 256;
  __shared__ __align__(16) uint16_t tile[fuseconv::kMaxCout][kPackCols + 8];
  const int nh = blockIdx.x, n = nh / H, h = nh - n * H;
  const int w0 = blockIdx.y * kPackCols;
  const size_t P = (size_t)H * W;
  const T* src = dout + (size_t)n * Cout * P;
  const int items = Np * kGroups;
  Raw8<T> v[kItems];
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const int item = threadIdx.x + u * 256;
    const int g = item % kGroups, c = item / kGroups;
    if (item < items && c < Cout)
      v[u] = load_raw8<T>(src + (size_t)c * P, H, W, h, w0 + g * 8);
    else
      v[u].zero();
  }
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const int item = threadIdx.x + u * 256;
    if (item < items)
      *reinterpret_cast<uint4*>(&tile[item / kGroups][(item % kGroups) * 8]) = v[u].u;
  }
  __syncthreads();
  // db partial: 4 threads per channel, 16 columns each
  {
    const int c = threadIdx.x >> 2, q = threadIdx.x & 3;
    float acc = 0.f;
    if (c < Np) {
#pragma unroll
      for (int x = 0; x < 16; ++x) {
        const uint16_t b = tile[c][q * 16 + x];
        if constexpr (std::is_same<T, __nv_bfloat16>::value)
          acc += __uint_as_float((uint32_t)b << 16);
        else
          acc += __half2float(__ushort_as_half(b));
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (c < Np && q == 0) dbp[((size_t)nh * gridDim.y + blockIdx.y) * Np + c] = acc;
  }
  const int ng = Np / 8;
  for (int idx = threadIdx.x; idx < ng * kPackCols; idx += blockDim.x) {
    const int og = idx / kPackCols, x = idx - og * kPackCols;
    if (w0 + x >= W) continue;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      w[e] = (uint32_t)tile[og * 8 + 2 * e][x] | ((uint32_t)tile[og * 8 + 2 * e + 1][x] << 16);
    hi[((size_t)nh * ng + og) * W + w0 + x] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <typename T>
struct WtCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  static constexpr int kTW = kSplit ? 32 : 64;  // A row = 128 bytes either way
  static constexpr int kKSteps = kTW / 16;
  static constexpr int kStages = kSplit ? 4 : 5;
  static constexpr int kRaw = 3;                // FP32 raw A ring
  static constexpr int kConvWarp = 2;           // FP32 converters, then drain: warps 2-5
  static constexpr int kRawWarp = 6;            // FP32 raw-A copy issuer
  static constexpr int kThreads = 32 * (kSplit ? 7 : 6);
  static constexpr uint32_t kAPart = 128 * kTW * 2;            // one bf16/fp16 A image
  static constexpr uint32_t kABytes = kAPart * (kSplit ? 2 : 1);
  static constexpr uint32_t kRawBytes = 128 * kTW * 4;         // FP32 raw A tile
};

struct WtParams {
  CUtensorMap a;     // cat (16-bit: operand; FP32: raw), box {TW, 1, 128, 1}, SWIZZLE_128B
  CUtensorMap b_hi;  // dout plane (32-bit view), box {TW*4, Np/8, 1, 1}
  CUtensorMap b_lo;  // FP32 residual plane
  float* partial;    // [splits][nic][3][128][3*Np]
  int H, Np, nic, tiles_w, num_tiles, splits;
  uint32_t b_copy;       // bytes of one kx copy of B: (Np/8) * TW * 16
  uint32_t b_stage;      // B images of one stage (3 copies, x2 for FP32), 1024-byte multiple
  int* status;
};

template <typename T>
__global__ void __launch_bounds__(WtCfg<T>::kThreads, 1)
    fuseconv_wgrad_tma_kernel(const __grid_constant__ WtParams p) {
  using Cfg = WtCfg<T>;
  using Op = typename IoTraits<T>::Op;
  constexpr int S = Cfg::kStages, R = Cfg::kRaw, TW = Cfg::kTW;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;
  __shared__ __align__(8) uint64_t bars[2 * S + 2 * R + 1];
  // 1024-byte aligned operand area (SWIZZLE_128B atoms)
  uint8_t* base = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* bbase = base + S * Cfg::kABytes;  // B stages
  uint8_t* raw = bbase + S * p.b_stage;
  uint64_t* s_full = bars;            // [S] copies (+ FP32 converters)
  uint64_t* s_empty = bars + S;       // [S] MMA commit
  uint64_t* r_full = bars + 2 * S;    // [R] raw A copy (FP32)
  uint64_t* r_empty = r_full + R;     // [R] converters (FP32)
  uint64_t* d_done = r_empty + R;

  // Loop-invariant parameters in registers: the parameter block's address is
  // taken (tensor maps), so after every "memory"-clobbering asm statement the
  // compiler would otherwise reload these through generic loads.
  const int num_tiles = p.num_tiles, splits = p.splits, H = p.H, tiles_w = p.tiles_w;
  const uint32_t b_stage = p.b_stage, b_copy = p.b_copy;
  const int unit = blockIdx.x % (p.nic * 3);
  const int split = blockIdx.x / (p.nic * 3);
  const int ic = unit / 3, ky = unit % 3;
  const int Np = p.Np;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 256);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&s_full[i], Cfg::kSplit ? 1 + 128 : 1);
      tc::mbar_init(&s_empty[i], 1);
    }
    for (int i = 0; i < R; ++i) {
      tc::mbar_init(&r_full[i], 1);
      tc::mbar_init(&r_empty[i], 128);
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

  if (warp == 0) {
    // ---- stage copy issuer ------------------------------------------------------
    if (lane == 0) {
      const uint32_t tx = (Cfg::kSplit ? 0u : Cfg::kAPart) + (Cfg::kSplit ? 6u : 3u) * b_copy;
      uint32_t sq = 0;
      for (int tile = split; tile < num_tiles; tile += splits, ++sq) {
        const int per_img = H * tiles_w;
        const int n = tile / per_img, h = (tile % per_img) / tiles_w;
        const int w0 = (tile % tiles_w) * TW;
        const int sb = sq % S;
        if (!tc::mbar_wait(&s_empty[sb], ((sq / S) & 1) ^ 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 73);
          break;
        }
        uint8_t* st = base + sb * Cfg::kABytes;
        tc::mbar_arrive_expect_tx(&s_full[sb], tx);
        if constexpr (!Cfg::kSplit) tc::tma_load_4d(st, &p.a, w0, h, ic * 128, n, &s_full[sb]);
        // B copy kx: dout row h - ky + 1, columns w0 + 1 - kx .. +TW-1 (x in 4-byte units)
        uint8_t* bst = bbase + sb * b_stage;
        const int hr = h - ky + 1;
        for (int kx = 0; kx < 3; ++kx) {
          tc::tma_load_4d(bst + kx * b_copy, &p.b_hi, (w0 + 1 - kx) * 4, 0, hr, n, &s_full[sb]);
          if constexpr (Cfg::kSplit)
            tc::tma_load_4d(bst + (3 + kx) * b_copy, &p.b_lo, (w0 + 1 - kx) * 4, 0, hr, n,
                            &s_full[sb]);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer -------------------------------------------------------------
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(128, 3 * Np, IoTraits<T>::kBf16, false, true);
      constexpr uint64_t b_step = (16 * 16) >> 4;  // 16 pixel rows of B
      const uint64_t b_lo = (3 * b_copy) >> 4;
      uint32_t sq = 0;
      bool first = true;
      for (int tile = split; tile < num_tiles; tile += splits, ++sq) {
        const int sb = sq % S;
        if (!tc::mbar_wait(&s_full[sb], (sq / S) & 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 74);
          goto done;
        }
        tc::tc_fence_after();
        const uint32_t st = tc::smem_u32(base + sb * Cfg::kABytes);
        const uint64_t bd = tc::smem_desc(tc::smem_u32(bbase + sb * b_stage), 128, TW * 16);
        if constexpr (!Cfg::kSplit) {
          const uint64_t ad = tc::smem_desc_sw128(st);
          for (int ks = 0; ks < Cfg::kKSteps; ++ks)
            tc::mma_f16(tmem_base, ad + ks * 2, bd + ks * b_step, idesc, (!first || ks > 0) ? 1u : 0u);
        } else {
          const uint64_t ad = tc::smem_desc(st, 128 * 16, 128);
          constexpr uint64_t a_step = (2 * 128 * 16) >> 4;
          constexpr uint64_t a_lo = Cfg::kAPart >> 4;
          for (int ks = 0; ks < Cfg::kKSteps; ++ks) {
            const uint64_t a_k = ad + ks * a_step, b_k = bd + ks * b_step;
            tc::mma_f16(tmem_base, a_k, b_k, idesc, (!first || ks > 0) ? 1u : 0u);
            tc::mma_f16(tmem_base, a_k + a_lo, b_k, idesc, 1u);
            tc::mma_f16(tmem_base, a_k, b_k + b_lo, idesc, 1u);
          }
        }
        tc::mma_commit(&s_empty[sb]);
        first = false;
      }
      tc::mma_commit(d_done);
    }
  } else if (Cfg::kSplit && warp == Cfg::kRawWarp) {
    // ---- FP32 raw A copy issuer ---------------------------------------------------
    if (lane == 0) {
      uint32_t sq = 0;
      for (int tile = split; tile < num_tiles; tile += splits, ++sq) {
        const int per_img = H * tiles_w;
        const int n = tile / per_img, h = (tile % per_img) / tiles_w;
        const int w0 = (tile % tiles_w) * TW;
        const int rb = sq % R;
        if (!tc::mbar_wait(&r_empty[rb], ((sq / R) & 1) ^ 1, abort_flag, kWaitNs)) {
          fail(abort_flag, p.status, 75);
          break;
        }
        tc::mbar_arrive_expect_tx(&r_full[rb], Cfg::kRawBytes);
        tc::tma_load_4d(raw + rb * Cfg::kRawBytes, &p.a, w0, h, ic * 128, n, &r_full[rb]);
      }
    }
  } else if (warp >= Cfg::kConvWarp && warp < Cfg::kConvWarp + 4) {
    const int il = (warp - Cfg::kConvWarp) * 32 + lane;  // input channel of the chunk
    bool ok = true;
    if constexpr (Cfg::kSplit) {
      // ---- FP32 converters: raw row il (32 px, 128-byte swizzled) -> A hi / lo ---
      uint32_t sq = 0;
      for (int tile = split; tile < num_tiles; tile += splits, ++sq) {
        const int sb = sq % S, rb = sq % R;
        if (!warp_wait(&r_full[rb], (sq / R) & 1, abort_flag) ||
            !warp_wait(&s_empty[sb], ((sq / S) & 1) ^ 1, abort_flag)) {
          fail(abort_flag, p.status, 76);
          ok = false;
          break;
        }
        const uint8_t* row = raw + rb * Cfg::kRawBytes + il * 128;
        uint8_t* a = base + sb * Cfg::kABytes;
#pragma unroll
        for (int g = 0; g < TW / 8; ++g) {
          const float4 u = *reinterpret_cast<const float4*>(row + (((2 * g) ^ (il & 7)) * 16));
          const float4 v = *reinterpret_cast<const float4*>(row + (((2 * g + 1) ^ (il & 7)) * 16));
          const unsigned long long pr[4] = {f2_pack(u.x, u.y), f2_pack(u.z, u.w),
                                            f2_pack(v.x, v.y), f2_pack(v.z, v.w)};
          const uint32_t off = (g * 128 + il) * 16;
          store8x2_split<Op, true>(a + off, a + Cfg::kAPart + off, pr);
        }
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&s_full[sb]);
        tc::mbar_arrive(&r_empty[rb]);
      }
    }
    // ---- drain: a warp reads TMEM lanes 32 * (warp % 4) .. +31 (channels) ------------
    const int quad = warp & 3;
    const int dl = quad * 32 + lane;
    if (ok && warp_wait(d_done, 0, abort_flag)) {
      tc::tc_fence_after();
      float* dst = p.partial + ((((size_t)split * p.nic + ic) * 3 + ky) * 128 + dl) * (3 * Np);
      for (int c0 = 0; c0 < 3 * Np; c0 += 16) {
        float v[16];
        tc::tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + c0, v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 16; k += 4)
          *reinterpret_cast<float4*>(dst + c0 + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
      }
    } else if (ok) {
      fail(abort_flag, p.status, 77);
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

struct WgPlan {
  int Np, nic, splits, tiles_w, num_tiles;
  size_t partial_bytes, mid_off, ws_bytes;  // mid_off: the db reduction's level-2 rows
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
  q.mid_off = (q.partial_bytes + (size_t)sp * q.Np * sizeof(float) + 255) / 256 * 256;
  q.ws_bytes = q.mid_off + (size_t)kDbMidBlocks * q.Np * sizeof(float);
  return q;
}

// TMA path workspace: [partials][db partials][dout plane hi][dout plane lo].
struct WtPlan {
  WgPlan g;
  int strips;  // 64-column pre-pass strips per row (db partials per row)
  size_t dbp_off, hi_off, lo_off, mid_off, ws_bytes;
};

inline size_t round256(size_t v) { return (v + 255) / 256 * 256; }

WtPlan plan_wgrad_tma(int n, int cin, int cout, int h, int w, int tw, bool split) {
  WtPlan t;
  t.g = plan_wgrad(n, cin, cout, h, w, tw);
  t.strips = (w + kPackCols - 1) / kPackCols;
  const size_t plane = (size_t)n * h * (t.g.Np / 8) * w * 16;
  t.dbp_off = round256(t.g.partial_bytes);
  t.hi_off = round256(t.dbp_off + (size_t)n * h * t.strips * t.g.Np * sizeof(float));
  t.lo_off = round256(t.hi_off + plane);
  t.mid_off = round256(split ? t.lo_off + plane : t.lo_off);
  t.ws_bytes = t.mid_off + (size_t)kDbMidBlocks * t.g.Np * sizeof(float);
  return t;
}

bool wgrad_tma_shape(int w) { return w % 8 == 0; }

template <typename T>
int run_wgrad_reg(const WgParams& prm, void* dw, void* db, cudaStream_t st) {
  using Cfg = WgCfg<T>;
  const WgSmem L = wg_smem_layout(prm, Cfg::kStages);
  auto fn = fuseconv_wgrad_kernel<T>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  fn<<<prm.nic * 3 * prm.splits, Cfg::kThreads, L.total, st>>>(prm);
  DDPM_CHECK_LAUNCH("fuseconv_wgrad_kernel");
  return launch_wgrad_reduce<T>(prm.partial, prm.db_partial, prm.db_mid, dw, db, prm.Cin,
                                prm.Cout, prm.Np,
                                prm.nic, prm.splits, prm.splits, st);
}

// Returns DDPM_ERR_UNSUPPORTED (nothing launched) when the driver rejects a
// tensor map, so the caller can take the register path.
// With `gcat` set, the data gradient runs between the pre-pass and the main
// kernel, reading grad_out from the pre-pass's planes (fuseconv_dgrad_rowmajor).
template <typename T>
int run_wgrad_tma(const void* cat, const void* gout, void* gw, void* gb, uint8_t* ws,
                  const WtPlan& t, int n, int cin, int cout, int h, int w, int dt, int* status,
                  cudaStream_t st, const void* packed = nullptr, void* gcat = nullptr,
                  int gcat_nhwc = 0) {
  using Cfg = WtCfg<T>;
  constexpr int TW = Cfg::kTW;
  const int Np = t.g.Np, ng = Np / 8;
  const int es = dtype_size(dt);
  uint4* hi = reinterpret_cast<uint4*>(ws + t.hi_off);
  uint4* lo = Cfg::kSplit ? reinterpret_cast<uint4*>(ws + t.lo_off) : nullptr;
  float* dbp = reinterpret_cast<float*>(ws + t.dbp_off);
  WtParams prm{};
  const CUtensorMapDataType at = dt == DDPM_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dt == DDPM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t adims[4] = {(uint64_t)w, (uint64_t)h, (uint64_t)cin, (uint64_t)n};
  const uint64_t astr[3] = {(uint64_t)w * es, (uint64_t)h * w * es, (uint64_t)cin * h * w * es};
  const uint32_t abox[4] = {(uint32_t)TW, 1, 128, 1};
  const uint64_t bdims[4] = {(uint64_t)w * 4, (uint64_t)ng, (uint64_t)h, (uint64_t)n};
  const uint64_t bstr[3] = {(uint64_t)w * 16, (uint64_t)ng * w * 16, (uint64_t)h * ng * w * 16};
  const uint32_t bbox[4] = {(uint32_t)TW * 4, (uint32_t)ng, 1, 1};
  if (encode_tmap(&prm.a, at, 4, cat, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B) != DDPM_OK ||
      encode_tmap(&prm.b_hi, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, hi, bdims, bstr, bbox,
                  CU_TENSOR_MAP_SWIZZLE_NONE) != DDPM_OK ||
      (Cfg::kSplit && encode_tmap(&prm.b_lo, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, lo, bdims, bstr,
                                  bbox, CU_TENSOR_MAP_SWIZZLE_NONE) != DDPM_OK)) {
    clear_error();
    return DDPM_ERR_UNSUPPORTED;
  }
  if (!Cfg::kSplit) prm.b_lo = prm.b_hi;
  prm.partial = reinterpret_cast<float*>(ws);
  prm.H = h;
  prm.Np = Np;
  prm.nic = t.g.nic;
  prm.tiles_w = t.g.tiles_w;
  prm.num_tiles = t.g.num_tiles;
  prm.splits = t.g.splits;
  prm.b_copy = (uint32_t)ng * TW * 16;
  prm.b_stage = ((Cfg::kSplit ? 6u : 3u) * prm.b_copy + 1023u) / 1024u * 1024u;
  prm.status = status;

  if constexpr (sizeof(T) == 2) {
    fuseconv_dout_pack16_kernel<T><<<dim3(n * h, t.strips), 256, 0, st>>>(
        static_cast<const T*>(gout), hi, dbp, h, w, cout, Np);
    DDPM_CHECK_LAUNCH("fuseconv_dout_pack16_kernel");
  } else {
    fuseconv_dout_pack_kernel<T><<<dim3(n * h, t.strips), 256, 0, st>>>(
        static_cast<const T*>(gout), hi, lo, dbp, h, w, cout, Np);
    DDPM_CHECK_LAUNCH("fuseconv_dout_pack_kernel");
  }
  if (gcat != nullptr) {
    int rc = fuseconv_dgrad_rowmajor(hi, lo, packed, gcat, n, cin, cout, h, w, dt, st, gcat_nhwc);
    if (rc == DDPM_ERR_UNSUPPORTED) rc = fuseconv_dgrad(gout, packed, gcat, n, cin, cout, h, w,
                                                        dt, st, gcat_nhwc);
    if (rc) return rc;
  }
  const size_t smem = (size_t)Cfg::kStages * (Cfg::kABytes + prm.b_stage) +
                      (Cfg::kSplit ? (size_t)Cfg::kRaw * Cfg::kRawBytes : 0) + 1024;
  auto fn = fuseconv_wgrad_tma_kernel<T>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  fn<<<prm.nic * 3 * prm.splits, Cfg::kThreads, smem, st>>>(prm);
  DDPM_CHECK_LAUNCH("fuseconv_wgrad_tma_kernel");
  return launch_wgrad_reduce<T>(prm.partial, dbp, reinterpret_cast<float*>(ws + t.mid_off), gw,
                                gb, cin, cout, Np, prm.nic, prm.splits, n * h * t.strips, st);
}

}  // namespace

size_t fuseconv_wgrad_workspace_bytes(int n, int cin, int cout, int h, int w) {
  if (n < 1 || h < 1 || w < 1 || cin < 1 || cout < 1 || cin > fuseconv::kMaxCin ||
      cout > fuseconv::kMaxCout)
    return 0;
  // the largest of the FP32 and 16-bit plans of both paths
  size_t best = plan_wgrad(n, cin, cout, h, w, WgCfg<float>::kTW).ws_bytes;
  const size_t b = plan_wgrad(n, cin, cout, h, w, WgCfg<__half>::kTW).ws_bytes;
  if (b > best) best = b;
  if (wgrad_tma_shape(w)) {
    const size_t c = plan_wgrad_tma(n, cin, cout, h, w, WtCfg<float>::kTW, true).ws_bytes;
    const size_t d = plan_wgrad_tma(n, cin, cout, h, w, WtCfg<__half>::kTW, false).ws_bytes;
    if (c > best) best = c;
    if (d > best) best = d;
  }
  return best;
}

int fuseconv_wgrad(const void* cat, const void* gout, void* gw, void* gb, void* ws, size_t ws_bytes,
                   int n, int cin, int cout, int h, int w, int dt, cudaStream_t st);

// Data and weight / bias gradient together: with the TMA weight-gradient path
// the data gradient reads grad_out from the planes the weight gradient's
// pre-pass writes anyway, instead of staging it separately.
int fuseconv_bwd(const void* cat, const void* gout, const void* packed, void* gcat, void* gw,
                 void* gb, void* ws, size_t ws_bytes, int n, int cin, int cout, int h, int w,
                 int dt, cudaStream_t st, int gcat_nhwc) {
  DDPM_CHECK_ARG(n >= 1 && h >= 1 && w >= 1 && cin >= 1 && cout >= 1, "sizes must be positive");
  DDPM_CHECK_ARG(dtype_size(dt) > 0, "unknown dtype code %d", dt);
  if (cin > fuseconv::kMaxCin || cout > fuseconv::kMaxCout)
    return set_error(DDPM_ERR_UNSUPPORTED, "native fuse conv supports Cin <= %d, Cout <= %d",
                     fuseconv::kMaxCin, fuseconv::kMaxCout);
  DDPM_CHECK_ARG(cat && gout && packed && gcat && gw, "null pointer");
  const size_t need = fuseconv_wgrad_workspace_bytes(n, cin, cout, h, w);
  if (ws == nullptr || ws_bytes < need)
    return set_error(DDPM_ERR_WORKSPACE, "workspace too small (%zu < %zu)", ws_bytes, need);
  DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(ws) & 255u) == 0, "workspace must be 256-byte aligned");
  int* status = nullptr;
  int rc = gencat::status_ptr(&status);
  if (rc) return rc;
  const bool aligned =
      ((reinterpret_cast<uintptr_t>(cat) | reinterpret_cast<uintptr_t>(gout)) & 15u) == 0;
  if (aligned && wgrad_tma_shape(w)) {
    uint8_t* wsb = static_cast<uint8_t*>(ws);
    switch (dt) {
      case DDPM_BF16:
        rc = run_wgrad_tma<__nv_bfloat16>(cat, gout, gw, gb, wsb,
                                          plan_wgrad_tma(n, cin, cout, h, w, 64, false), n, cin,
                                          cout, h, w, dt, status, st, packed, gcat, gcat_nhwc);
        break;
      case DDPM_F16:
        rc = run_wgrad_tma<__half>(cat, gout, gw, gb, wsb,
                                   plan_wgrad_tma(n, cin, cout, h, w, 64, false), n, cin, cout, h,
                                   w, dt, status, st, packed, gcat, gcat_nhwc);
        break;
      default:
        rc = run_wgrad_tma<float>(cat, gout, gw, gb, wsb,
                                  plan_wgrad_tma(n, cin, cout, h, w, 32, true), n, cin, cout, h, w,
                                  dt, status, st, packed, gcat, gcat_nhwc);
    }
    if (rc != DDPM_ERR_UNSUPPORTED) return rc;
  }
  rc = fuseconv_dgrad(gout, packed, gcat, n, cin, cout, h, w, dt, st, gcat_nhwc);
  if (rc) return rc;
  return fuseconv_wgrad(cat, gout, gw, gb, ws, ws_bytes, n, cin, cout, h, w, dt, st);
}

int fuseconv_wgrad(const void* cat, const void* gout, void* gw, void* gb, void* ws, size_t ws_bytes,
                   int n, int cin, int cout, int h, int w, int dt, cudaStream_t st) {
  DDPM_CHECK_ARG(n >= 1 && h >= 1 && w >= 1 && cin >= 1 && cout >= 1, "sizes must be positive");
  DDPM_CHECK_ARG(dtype_size(dt) > 0, "unknown dtype code %d", dt);
  if (cin > fuseconv::kMaxCin || cout > fuseconv::kMaxCout)
    return set_error(DDPM_ERR_UNSUPPORTED, "native fuse conv supports Cin <= %d, Cout <= %d",
                     fuseconv::kMaxCin, fuseconv::kMaxCout);
  DDPM_CHECK_ARG(cat && gout && gw, "null pointer");
  const size_t need = fuseconv_wgrad_workspace_bytes(n, cin, cout, h, w);
  if (ws == nullptr || ws_bytes < need)
    return set_error(DDPM_ERR_WORKSPACE, "workspace too small (%zu < %zu)", ws_bytes, need);
  DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(ws) & 255u) == 0, "workspace must be 256-byte aligned");
  int* status = nullptr;
  int rc = gencat::status_ptr(&status);
  if (rc) return rc;
  const bool split = dt == DDPM_F32;
  const bool aligned =
      ((reinterpret_cast<uintptr_t>(cat) | reinterpret_cast<uintptr_t>(gout)) & 15u) == 0;
  if (aligned && wgrad_tma_shape(w)) {
    uint8_t* wsb = static_cast<uint8_t*>(ws);
    switch (dt) {
      case DDPM_BF16:
        rc = run_wgrad_tma<__nv_bfloat16>(cat, gout, gw, gb, wsb,
                                          plan_wgrad_tma(n, cin, cout, h, w, 64, false), n, cin,
                                          cout, h, w, dt, status, st);
        break;
      case DDPM_F16:
        rc = run_wgrad_tma<__half>(cat, gout, gw, gb, wsb,
                                   plan_wgrad_tma(n, cin, cout, h, w, 64, false), n, cin, cout, h,
                                   w, dt, status, st);
        break;
      default:
        rc = run_wgrad_tma<float>(cat, gout, gw, gb, wsb,
                                  plan_wgrad_tma(n, cin, cout, h, w, 32, true), n, cin, cout, h, w,
                                  dt, status, st);
    }
    if (rc != DDPM_ERR_UNSUPPORTED) return rc;
  }
  const int tw = split ? WgCfg<float>::kTW : WgCfg<__half>::kTW;
  const WgPlan q = plan_wgrad(n, cin, cout, h, w, tw);
  WgParams prm{};
  prm.cat = cat;
  prm.dout = gout;
  prm.partial = static_cast<float*>(ws);
  prm.db_partial = gb != nullptr
                       ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + q.partial_bytes)
                       : nullptr;
  prm.db_mid = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + q.mid_off);
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
  prm.vec = (w % 8) == 0 && aligned;
  prm.a_part = (uint32_t)(tw / 8) * 128 * 16;            // pixel groups x 128 channels x 16 B
  prm.a_bytes = prm.a_part * (split ? 2 : 1);
  prm.b_part = (uint32_t)(3 * (q.Np / 8)) * tw * 16;     // [kx][o/8][TW rows][8]
  prm.b_bytes = prm.b_part * (split ? 2 : 1);
  prm.status = status;
  switch (dt) {
    case DDPM_BF16: return run_wgrad_reg<__nv_bfloat16>(prm, gw, gb, st);
    case DDPM_F16: return run_wgrad_reg<__half>(prm, gw, gb, st);
    default: return run_wgrad_reg<float>(prm, gw, gb, st);
  }
}

}  // namespace ddpm
