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
//   * every CTA owns ONE output channel group cg of 16 channels; the weight
//             rows of that group (3 branches x K^2 taps x 16 channels, i.e.
//             3*K chunks) are loaded into shared memory once and stay resident,
//             so no weight traffic recurs per tile (re-streaming the full
//             weight per 128-pixel tile would need ~18 TB/s of L2 bandwidth);
//   * tile  = 8 x 16 output pixels of one image = the 128 rows of the MMA's
//             M dimension = the 128 TMEM lanes (lane m <-> pixel (m/16, m%16));
//             CTAs of the same cg split the tiles between them;
//   * slot  = one branch b (K = 3) or all three branches (K = 1) of the
//             CTA's group: ONE MMA per K step with N = branches * K^2 * 16
//             accumulator columns (144 or 48), column (b', tap)*16 + cl <->
//             branch b0 + b', tap, channel cg*16 + cl. A tcgen05.mma costs
//             its issuing thread ~55 cycles whatever its N, so the widest N
//             the weight layout allows keeps the tensor pipe busy.
//   * GEMM K dimension = the Ck "augmented" input channels. For bf16/fp16:
//             y's C channels, then a constant-one channel whose weight column
//             is the bias, then zeros (Ck = round_up(C + 1, 16)) - the bias add
//             is part of the MMA. For fp32 (shared memory is tighter there) Ck
//             = Cp and the epilogue adds the bias.
//   * operands: A = the y tile, MN-major in shared memory ([8-pixel group]
//             [channel][8 pixels]); B = the group's resident weight chunks,
//             pre-packed in global memory in the exact K-major smem image
//             [Ck/8][3*K^2*16 rows][8] (any branch's rows are a contiguous
//             N range) and fetched with one 1-D bulk async copy.
//   * FP32 I/O: y and W are split into bf16 hi + lo parts and each MMA step
//             is hi*hi + lo*hi + hi*lo (relative error ~2^-16 per product).
//   * x halo: for each channel group the (8+2R) x 32 pixel neighbourhood of the
//             tile is staged in shared memory as FP32, four channels per
//             16-byte cell ([4-channel group][row][32 cols][4]), zero outside the
//             image. An epilogue thread reads the 16 channels of one tap with
//             four LDS.128 and needs no bounds checks.
//
// Warp roles (18 warps): w0 = TMEM allocator + weight loader, w1 = MMA
// issuer, w2-w5 = y-tile producers, w6-w9 = x-halo producers, w10-w17 = two
// epilogue warpgroups; slot number s (counted over the CTA's tiles) belongs
// to warpgroup s % 2, which consumes its slots in order from its own ring of
// TMEM buffers. With staged operands (16 warps): one warp per producer role
// and three epilogue warpgroups (slot s -> warpgroup s % 3). Each producer thread issues all of its loads for a tile before
// its first shared-memory store, so a tile costs one memory latency, not
// several; each epilogue thread issues the three TMEM loads of a chunk before
// a single wait. With staged operands (gencat_stage.cu) one thread per
// producer role issues one TMA copy per tile instead: the y tile from the y
// plane (then a K-major A operand, [channel group][pixel][8 channels]) and the
// x halo from the FP32 cell plane, both zero filled outside the image.
#include "common.cuh"
#include "tc.cuh"
#include "gencat.cuh"
#include "fuseconv.cuh"

namespace ddpm {
namespace {

using namespace gencat;

// Test hook (ddpm_test_skip_arrive): when set, one y-tile producer thread of
// CTA 0 withholds its arrival for the CTA's first tile, so that CTA's MMA
// issuer waits on a phase that never completes. The bounded wait gives up
// after kWaitNs, records its code in the device status word, and every role
// unwinds (TMEM is freed): the failure path of the kernels, exercised without
// a fault. Zero in normal operation.
__device__ int g_test_skip_arrive;

// Every wait of the forward kernel lets a waiting thread stay suspended (not
// issuing) for up to this long, woken by the phase's completion.
constexpr uint32_t kHintNs = 100000;

template <typename T, int KS, bool kStaged = false>
struct FwdCfg {
  static constexpr bool kSplit = IoTraits<T>::kSplit;
  static constexpr int kParts = kSplit ? 2 : 1;
  static constexpr int kCG = fwd_cg(KS, kSplit);              // output channels of a CTA
  static constexpr int kQ4 = kCG / 4;                         // 4-channel x cells per pixel
  static constexpr int kBrN = fwd_branch_cols(KS, kSplit);    // accumulator columns per branch
  static constexpr int kBr = KS == 1 ? 3 : 1;                 // branches per slot
  static constexpr int kSlots = 3 / kBr;                      // slots per tile
  static constexpr int kN = kBr * kBrN;                       // accumulator columns per slot
  static constexpr int kRows = 3 * kBrN;                      // weight rows of a channel group
  static constexpr int kNumBuf = (512 / kN) > 8 ? 8 : (512 / kN);
  // Epilogue warpgroups: slot s belongs to warpgroup s % kEpiWG. With staged
  // operands each producer role is one warp, which leaves the threads for a
  // third warpgroup: the epilogue (the bound of this kernel) then drains three
  // slots at once (where TMEM holds a buffer for each: not at K = 5 bf16, whose
  // 208-column slots fit twice). Each warpgroup owns kNumBuf / kEpiWG TMEM
  // buffers: every buffer has a single consumer that sees all of its phases in
  // order.
  static constexpr int kEpiWG = (kStaged && kNumBuf >= 3) ? 3 : 2;
  static constexpr int kBufPerWG = kNumBuf / kEpiWG;
  static_assert(kBufPerWG >= 1, "a TMEM slot per epilogue warpgroup must fit");
  static constexpr int kYBufs = kSplit ? 1 : 2;               // smem budget (see layout)
  static constexpr bool kBiasInGemm = !kSplit;
  static constexpr int kProducers = kStaged ? 32 : 128;       // threads per producer role
  static constexpr int kFirstEpiWarp = 2 + 2 * (kProducers / 32);
  static constexpr int kThreads = 32 * (kFirstEpiWarp + 4 * kEpiWG);
  // x halo tile: kHaloW columns from w0 - kHaloOff, up to kMaxR rows above and below
  static constexpr int kHaloW = fwd_halo_cols(KS);
  static constexpr int kHaloOff = fwd_halo_off(KS);
  static constexpr int kMaxR = fwd_max_halo(KS);
  // loads per producer thread and tile (whole tile in one batch)
  // y items per thread: 16 pixel groups x Ck (<= 80 for bf16/fp16, = Cp <= 64 for fp32)
  static constexpr int kYItems = (16 * (kSplit ? 64 : 80) + kProducers - 1) / kProducers;
  static constexpr int kXItems =
      (kQ4 * (kHaloW / 8) * (kTileH + 2 * kMaxR) + kProducers - 1) / kProducers;
  // x halo cells in shared memory: with staged operands 16-bit data arrives as
  // 8-channel cells in the I/O type (kXIo: the epilogue multiplies the 16-bit
  // values directly), otherwise as FP32 cells of 4 channels
  static constexpr bool kXIo = kStaged && !kSplit;
  static constexpr int kXCells = kXIo ? kCG / 8 : kQ4;  // cells per pixel
};

struct FwdSmem {
  // byte offsets into dynamic shared memory
  uint32_t y, w, xr, bias, bars, total;
  uint32_t y_bytes, w_bytes, xr_bytes;
};

// Resident weights of one channel group + y tile(s) + `nxb` (2, or 1 where two
// do not fit: FP32 with halos >= 7) x-halo buffers.
// C=64, K=3, halo 5: bf16 69 + 2x20 + 2x36 KB = 181 KB (staged 16-bit x: 2x18,
// 145 KB); fp32 108 + 32 + 72 KB = 214 KB.
// C=64, K=5, halo 10 (8 / 4 channels): bf16 97.5 + 2x20 + 2x42 KB = 221.5 KB
// (staged: 2x21, 179.5 KB); fp32 84 + 32 + 2x21 KB + 1.2 KB bias = 159 KB.
template <typename T, int KS, bool kStaged = false>
__host__ __device__ inline FwdSmem fwd_smem_layout(int Ck, int R, int nxb) {
  using Cfg = FwdCfg<T, KS, kStaged>;
  FwdSmem L;
  L.y_bytes = (uint32_t)Cfg::kParts * kTileM * Ck * 2;
  L.w_bytes = (uint32_t)Cfg::kParts * Cfg::kRows * Ck * 2;  // the group's whole image
  L.xr_bytes = (uint32_t)Cfg::kXCells * (kTileH + 2 * R) * Cfg::kHaloW * 16;
  L.y = 0;
  L.w = L.y + Cfg::kYBufs * L.y_bytes;
  L.xr = L.w + L.w_bytes;
  L.bias = L.xr + nxb * L.xr_bytes;
  L.bars = L.bias + (Cfg::kBiasInGemm ? 0u : (uint32_t)(3 * Cfg::kCG * KS * KS * 4));
  L.total = L.bars + 8 * (9 + 2 * Cfg::kNumBuf);
  return L;
}

struct FwdParams {
  const void* x;
  const void* y;
  const void* wpack;  // forward image (all channel groups)
  const void* bias;   // used by the fp32 epilogue (bias not folded into the GEMM)
  void* out;
  int N, C, H, W, Cp, Ck, R;
  int d[3];
  int tiles_w, tiles_h, num_tiles;
  int ncg, per_cg;    // channel groups; CTAs per channel group
  int nxb;            // x-halo buffers (1 or 2)
  // optional: the output also written as the fuse convolution's staged planes
  // (fuseconv::PlaneLayout of 4C channels; null = off; needs C % 8 == 0)
  uint8_t* planes;
  size_t pl_part;     // bytes per part (FP32: bf16 hi part, then lo part)
  int pl_G, pl_Hp, pl_Wp;
  int* status;
};

// One 8-channel, 16-byte plane cell (and the lo cell for FP32) of pixel (h, w).
template <typename Op, bool kSplit>
__device__ __forceinline__ void store_plane_cell(const FwdParams& p, int n, int g, int h, int w,
                                                 const unsigned long long (&pr)[4]) {
  const size_t off = ((((size_t)n * p.pl_G + g) * p.pl_Hp + (h + 1)) * p.pl_Wp + (w + 8)) * 16;
  store8x2_split<Op, kSplit>(p.planes + off, p.planes + p.pl_part + off, pr);
}
// Half `half` (channels 4*half .. +3) of that cell.
template <typename Op, bool kSplit>
__device__ __forceinline__ void store_plane_half(const FwdParams& p, int n, int g, int half, int h,
                                                 int w, const unsigned long long (&pr)[2]) {
  const size_t off =
      ((((size_t)n * p.pl_G + g) * p.pl_Hp + (h + 1)) * p.pl_Wp + (w + 8)) * 16 + half * 8;
  store4x2_split<Op, kSplit>(p.planes + off, p.planes + p.pl_part + off, pr);
}
// The group's kCG channels (pairs pr[0 .. kCG/2)) of pixel (h, w) starting at
// cat channel c0 (a multiple of kCG): whole cells, or one half cell at kCG = 4.
// `cvalid`: channels of the group below C (cells past it are not written;
// C % 8 == 0, so a valid cell is whole).
template <typename Op, bool kSplit, int kCG>
__device__ __forceinline__ void store_plane_group(const FwdParams& p, int n, int c0, int cvalid,
                                                  int h, int w, const unsigned long long* pr) {
  if constexpr (kCG == 4) {
    if (cvalid < 4) return;
    const unsigned long long q[2] = {pr[0], pr[1]};
    store_plane_half<Op, kSplit>(p, n, c0 / 8, (c0 / 4) & 1, h, w, q);
  } else {
#pragma unroll
    for (int k8 = 0; k8 < kCG / 8; ++k8) {
      if (8 * k8 + 8 > cvalid) break;
      const unsigned long long q[4] = {pr[4 * k8], pr[4 * k8 + 1], pr[4 * k8 + 2],
                                       pr[4 * k8 + 3]};
      store_plane_cell<Op, kSplit>(p, n, c0 / 8 + k8, h, w, q);
    }
  }
}

// Tensor maps of the staged operands (separate grid-constant parameter).
struct FwdMaps {
  CUtensorMap xmap, ymap;  // see gencat::encode_stage_maps
  int ph, pw;              // y-plane row / column offsets
};

template <typename T, int KS, bool kStaged>
__global__ void __launch_bounds__(FwdCfg<T, KS, kStaged>::kThreads, 1)
gencat_fwd_kernel(const FwdParams p, const __grid_constant__ FwdMaps maps) {
  using Cfg = FwdCfg<T, KS, kStaged>;
  using Op = typename IoTraits<T>::Op;
  constexpr int kN = Cfg::kN;
  constexpr int NB = Cfg::kNumBuf;
  constexpr int NY = Cfg::kYBufs;
  constexpr int KK = KS * KS;
  constexpr int r = KS / 2;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int C = p.C, Ck = p.Ck, H = p.H, W = p.W, R = p.R;
  const size_t P = (size_t)H * W;
  const FwdSmem L = fwd_smem_layout<T, KS, kStaged>(Ck, R, p.nxb);
  const int nx_sh = p.nxb - 1;  // 1 or 2 buffers: index = it & nx_sh, lap = it >> nx_sh
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* y_full = bars;           // [2]
  uint64_t* y_empty = bars + 2;      // [2]
  uint64_t* x_full = bars + 4;       // [2]
  uint64_t* x_empty = bars + 6;      // [2]
  uint64_t* w_full = bars + 8;       // [1]
  uint64_t* t_full = bars + 9;       // [NB]
  uint64_t* t_empty = t_full + NB;   // [NB]
  constexpr int kCG = Cfg::kCG;
  constexpr int kQ4 = Cfg::kQ4;
  constexpr int kHW = Cfg::kHaloW;
  const int xr_rows = kTileH + 2 * R;
  const int xr_plane = xr_rows * kHW;  // 16-byte cells per 4-channel group

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cg = blockIdx.x % p.ncg;           // this CTA's output channel group
  const int first_tile = blockIdx.x / p.ncg;
  const int tile_step = p.per_cg;

  // ---- setup --------------------------------------------------------------
  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_s, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&y_full[i], Cfg::kProducers);
      tc::mbar_init(&y_empty[i], 1);
      tc::mbar_init(&x_full[i], Cfg::kProducers);
      tc::mbar_init(&x_empty[i], 128 * Cfg::kEpiWG);
    }
    tc::mbar_init(w_full, 1);
    for (int i = 0; i < NB; ++i) {
      tc::mbar_init(&t_full[i], 1);
      tc::mbar_init(&t_empty[i], 128);
    }
    tc::fence_mbar_init();
    abort_s = 0;
  }
  if constexpr (!Cfg::kBiasInGemm) {
    float* bias_s = reinterpret_cast<float*>(smem + L.bias);
    const T* bias = static_cast<const T*>(p.bias);
    for (int i = threadIdx.x; i < 3 * kCG * KK; i += blockDim.x) {
      const int b = i / (kCG * KK), cl = (i / KK) % kCG, tap = i % KK;
      const int c = cg * kCG + cl;
      bias_s[i] = c < C ? to_f32<T>(bias[(b * C + c) * KK + tap]) : 0.f;
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  volatile int* abort_flag = &abort_s;

  if (warp == 0) {
    // ---- weight loader: the group's chunks, once, resident afterwards -----
    if (lane == 0) {
      const uint32_t bytes = L.w_bytes;
      const uint8_t* src = static_cast<const uint8_t*>(p.wpack) + (size_t)cg * bytes;
      tc::mbar_arrive_expect_tx(w_full, bytes);
      for (uint32_t off = 0; off < bytes; off += 32768) {
        const uint32_t len = bytes - off < 32768 ? bytes - off : 32768;
        tc::bulk_g2s(smem + L.w + off, src + off, len, w_full);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer --------------------------------------------------------
    if (lane == 0) {
      // y tile: MN-major [pixel group][channel][8 px] (staged from y) or K-major
      // [channel group][pixel][8 channels] (copied from the y plane)
      const uint32_t idesc = tc::idesc_f16(kTileM, kN, IoTraits<T>::kBf16, !kStaged, false);
      const uint32_t b_lbo = Cfg::kRows * 16;   // 8-channel groups of the weight image
      const uint64_t a_step = kStaged ? (uint64_t)(2 * kTileM * 16 >> 4) : (uint64_t)(256 >> 4);
      const uint64_t b_step = (2 * b_lbo) >> 4;
      const uint64_t a_lo = (kTileM * Ck * 2) >> 4;        // hi -> lo part of the y tile
      const uint64_t b_lo = (Cfg::kRows * Ck * 2) >> 4;    // hi -> lo part of the weights
      const int nks = Ck / 16;
      if (!tc::mbar_wait(w_full, 0, abort_flag, kWaitNs, kHintNs)) {
        fail(abort_flag, p.status, 10);
        goto done;
      }
      const uint64_t w_desc = tc::smem_desc(tc::smem_u32(smem + L.w), b_lbo, 128);
      uint32_t tq = 0, it = 0;
      for (int tile = first_tile; tile < p.num_tiles; tile += tile_step, ++it) {
        const int yb = it % NY;
        if (!tc::mbar_wait(&y_full[yb], (it / NY) & 1, abort_flag, kWaitNs, kHintNs)) {
          fail(abort_flag, p.status, 11);
          goto done;
        }
        tc::tc_fence_after();
        const uint64_t y_desc =
            kStaged ? tc::smem_desc(tc::smem_u32(smem + L.y + yb * L.y_bytes), kTileM * 16, 128)
                    : tc::smem_desc(tc::smem_u32(smem + L.y + yb * L.y_bytes), 128, Ck * 16);
        for (int q = 0; q < Cfg::kSlots; ++q, ++tq) {
          // slot tq belongs to epilogue warpgroup tq % kEpiWG (its own-th slot)
          const uint32_t own = tq / Cfg::kEpiWG;
          const int j = (int)(tq % Cfg::kEpiWG) * Cfg::kBufPerWG + own % Cfg::kBufPerWG;
          if (!tc::mbar_wait(&t_empty[j], ((own / Cfg::kBufPerWG) & 1) ^ 1, abort_flag,
                             kWaitNs, kHintNs)) {
            fail(abort_flag, p.status, 12);
            goto done;
          }
          tc::tc_fence_after();
          // rows of branch q (K = 3, 5) or of all branches (K = 1): (q * kN) * 16 bytes in
          const uint64_t bd = w_desc + (uint64_t)(q * kN);
          const uint32_t d = tmem_base + j * kN;
          // A plain runtime loop: an MMA under a per-step condition inside an
          // unrolled loop was compiled into wrong issue (results corrupted).
          for (int ks = 0; ks < nks; ++ks) {
            const uint64_t a_k = y_desc + ks * a_step;
            const uint64_t b_k = bd + ks * b_step;
            tc::mma_f16(d, a_k, b_k, idesc, ks > 0 ? 1u : 0u);
            if constexpr (Cfg::kSplit) {
              tc::mma_f16(d, a_k + a_lo, b_k, idesc, 1u);
              tc::mma_f16(d, a_k, b_k + b_lo, idesc, 1u);
            }
          }
          tc::mma_commit(&t_full[j]);
        }
        tc::mma_commit(&y_empty[yb]);
      }
      // Teardown frees TMEM: wait until every issued MMA has completed
      // (w_full's phase 1, after the weight load's phase 0).
      tc::mma_commit(w_full);
      if (!tc::mbar_wait(w_full, 1, abort_flag, kWaitNs, kHintNs)) fail(abort_flag, p.status, 17);
    }
  } else if (warp < 2 + Cfg::kProducers / 32) {
    // ---- y-tile producers ----------------------------------------------------
    const int pt = threadIdx.x - 64;
    const YPlan<Cfg::kYItems> plan = make_yplan<Cfg::kYItems>(Ck, pt, Cfg::kProducers);
    // the test hook: this thread withholds its first arrival (see g_test_skip_arrive)
    const bool withhold = pt == 1 && blockIdx.x == 0 && *(volatile int*)&g_test_skip_arrive;
    uint32_t it = 0;
    for (int tile = first_tile; tile < p.num_tiles; tile += tile_step, ++it) {
      const int yb = it % NY;
      if (!warp_wait(&y_empty[yb], ((it / NY) & 1) ^ 1, abort_flag, kHintNs)) {
        fail(abort_flag, p.status, 13);
        break;
      }
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      uint8_t* ys = smem + L.y + yb * L.y_bytes;
      if constexpr (kStaged) {
        // y plane rows h0+ph .. +7, columns w0+pw .. w0+pw+15, channel groups 0 .. Ck/8-1
        if (pt == 0) {
          tc::mbar_arrive_expect_tx(&y_full[yb], L.y_bytes);
          tc::tma_load_4d(ys, &maps.ymap, (w0 + maps.pw) * 2, h0 + maps.ph, 0, n, &y_full[yb]);
          if constexpr (Cfg::kSplit)
            tc::tma_load_4d(ys + kTileM * Ck * 2, &maps.ymap, (w0 + maps.pw) * 2, h0 + maps.ph, 0,
                            p.N + n, &y_full[yb]);
        } else if (!(withhold && it == 0)) {
          tc::mbar_arrive(&y_full[yb]);
        }
      } else {
        // 16 eight-pixel groups x Ck channels; one 16-byte smem row each.
        // MN-major interleaved: group g at g*Ck*16, channel c at (c/8)*128 + (c%8)*16.
        stage_y_mn<T, Op, Cfg::kSplit, Cfg::kYItems>(plan, static_cast<const T*>(p.y), ys,
                                                     ys + kTileM * Ck * 2, n, C, Ck,
                                                     Cfg::kBiasInGemm ? C : -1, H, W, h0, w0);
        tc::fence_proxy_async_smem();
        if (!(withhold && it == 0)) tc::mbar_arrive(&y_full[yb]);
      }
    }
  } else if (warp < Cfg::kFirstEpiWarp) {
    // ---- x-halo producers ----------------------------------------------------
    const int pt = threadIdx.x - 64 - Cfg::kProducers;
    const XPlan<Cfg::kXItems> plan =
        make_xplan<Cfg::kXItems, kQ4, kHW / 8>(xr_rows, pt, Cfg::kProducers);
    uint32_t it = 0;
    for (int tile = first_tile; tile < p.num_tiles; tile += tile_step, ++it) {
      const int xb = it & nx_sh;
      if (!warp_wait(&x_empty[xb], ((it >> nx_sh) & 1) ^ 1, abort_flag, kHintNs)) {
        fail(abort_flag, p.status, 15);
        break;
      }
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      float4* xr = reinterpret_cast<float4*>(smem + L.xr + xb * L.xr_bytes);
      if constexpr (kStaged) {
        if (pt == 0) {
          tc::mbar_arrive_expect_tx(&x_full[xb], L.xr_bytes);
          tc::tma_load_4d(xr, &maps.xmap, (w0 - Cfg::kHaloOff) * 2, h0 - R, cg * Cfg::kXCells,
                          n, &x_full[xb]);
        } else {
          tc::mbar_arrive(&x_full[xb]);
        }
      } else {
        stage_halo<T, Cfg::kXItems, kQ4, kHW / 8>(plan, static_cast<const T*>(p.x), xr, n, C, H,
                                                  W, cg * kCG, h0 - R, w0 - Cfg::kHaloOff,
                                                  xr_rows);
        tc::mbar_arrive(&x_full[xb]);
      }
    }
  } else {
    // ---- epilogue warpgroups -----------------------------------------------
    const int ew = warp - Cfg::kFirstEpiWarp;
    const int wg = ew >> 2;
    const int quad = warp & 3;               // TMEM lane quadrant of this warp
    const int m = quad * 32 + lane;          // pixel row of the MMA tile
    const int mr = m >> 4, mc = m & 15;
    const float* bias_s = reinterpret_cast<const float*>(smem + L.bias);
    T* out = static_cast<T*>(p.out);
    uint32_t tq = 0, it = 0;
    for (int tile = first_tile; tile < p.num_tiles; tile += tile_step, ++it) {
      int n, h0, w0;
      tile_origin(tile, p.tiles_w, p.tiles_h, n, h0, w0);
      const int h = h0 + mr;
      const int w = w0 + mc;
      const bool px_ok = (h < H) && (w < W);
      const size_t pix = (size_t)h * W + w;
      T* on = out + (size_t)n * 4 * C * P;
      const int xb = it & nx_sh;
      if (!warp_wait(&x_full[xb], (it >> nx_sh) & 1, abort_flag, kHintNs)) {
        fail(abort_flag, p.status, 16);
        break;
      }
      // this pixel's cell in the halo tile; a tap shifts it by (dy, dx)
      const int xcell0 = (mr + R) * kHW + (mc + Cfg::kHaloOff);
      const float4* xc = reinterpret_cast<const float4*>(smem + L.xr + xb * L.xr_bytes) + xcell0;
      const uint4* xci = reinterpret_cast<const uint4*>(smem + L.xr + xb * L.xr_bytes) + xcell0;
      bool failed = false;
      for (int q = 0; q < Cfg::kSlots && !failed; ++q, ++tq) {
        if (tq % Cfg::kEpiWG != (uint32_t)wg) continue;  // another warpgroup's slot
        const uint32_t own = tq / Cfg::kEpiWG;
        const int j = wg * Cfg::kBufPerWG + own % Cfg::kBufPerWG;
        if (!warp_wait(&t_full[j], (own / Cfg::kBufPerWG) & 1, abort_flag, kHintNs)) {
          fail(abort_flag, p.status, 14);
          failed = true;
          break;
        }
        tc::tc_fence_after();
        const uint32_t slot_addr = tmem_base + ((uint32_t)(quad * 32) << 16) + j * kN;
#pragma unroll
        for (int bb = 0; bb < Cfg::kBr; ++bb) {
          const int b = q * Cfg::kBr + bb;
          const int d = p.d[b];
          unsigned long long acc[kCG / 2];
#pragma unroll
          for (int i = 0; i < kCG / 2; ++i) acc[i] = 0ull;
#pragma unroll
          for (int ki = 0; ki < KS; ++ki) {
            const uint32_t taddr = slot_addr + bb * Cfg::kBrN + ki * KS * kCG;
            const float4* xrow = xc + (ki - r) * d * kHW;
            float dv[KS][kCG];
#pragma unroll
            for (int kj = 0; kj < KS; ++kj) tc::tmem_ld_cols<kCG>(taddr + kj * kCG, dv[kj]);
            tc::tmem_ld_wait();
            if (bb == Cfg::kBr - 1 && ki == KS - 1) {
              tc::tc_fence_before();
              tc::mbar_arrive(&t_empty[j]);  // the slot's accumulators are in registers now
            }
#pragma unroll
            for (int kj = 0; kj < KS; ++kj) {
              if constexpr (Cfg::kXIo) {
                // 8-channel 16-bit cells: each word of two x values meets the
                // matching pair of rounded taps in two mixed-precision FMAs
                const uint4* cell = xci + ((ki - r) * kHW + (kj - r)) * d;
#pragma unroll
                for (int c8 = 0; c8 < Cfg::kXCells; ++c8) {
                  const uint4 v = cell[c8 * xr_plane];
                  const uint32_t xw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                  for (int i = 0; i < 4; ++i)
                    acc[c8 * 4 + i] =
                        fma_io2<Op>(cvt2<Op>(dv[kj][c8 * 8 + 2 * i], dv[kj][c8 * 8 + 2 * i + 1]),
                                    xw[i], acc[c8 * 4 + i]);
                }
                continue;
              }
              const float4* cell = xrow + (kj - r) * d;
#pragma unroll
              for (int q4 = 0; q4 < kQ4; ++q4) {
                const float4 v = cell[q4 * xr_plane];
                float g0 = dv[kj][q4 * 4 + 0], g1 = dv[kj][q4 * 4 + 1];
                float g2 = dv[kj][q4 * 4 + 2], g3 = dv[kj][q4 * 4 + 3];
                if constexpr (!Cfg::kBiasInGemm) {
                  const float* bs = bias_s + (b * kCG + q4 * 4) * KK + ki * KS + kj;
                  g0 += bs[0];
                  g1 += bs[KK];
                  g2 += bs[2 * KK];
                  g3 += bs[3 * KK];
                }
                acc[q4 * 2 + 0] = f2_fma(tap_pair<T>(g0, g1), f2_pack(v.x, v.y), acc[q4 * 2 + 0]);
                acc[q4 * 2 + 1] = f2_fma(tap_pair<T>(g2, g3), f2_pack(v.z, v.w), acc[q4 * 2 + 1]);
              }
            }
          }
          if (px_ok) {
#pragma unroll
            for (int i = 0; i < kCG / 2; ++i) {
              float a0, a1;
              f2_unpack(acc[i], a0, a1);
              const int c = cg * kCG + 2 * i;
              if (c < C) on[(size_t)((b + 1) * C + c) * P + pix] = from_f32<T>(a0);
              if (c + 1 < C) on[(size_t)((b + 1) * C + c + 1) * P + pix] = from_f32<T>(a1);
            }
            if (p.planes != nullptr)  // cat channels (b+1)C + cg*kCG .. (C % 8 == 0)
              store_plane_group<Op, Cfg::kSplit, kCG>(p, n, (b + 1) * C + cg * kCG,
                                                      C - cg * kCG, h, w, acc);
          }
        }
      }
      if (failed) break;
      // passthrough out[:, cg*kCG : (cg+1)*kCG] = x, written from the halo tile
      if (px_ok && (it % Cfg::kEpiWG) == (uint32_t)wg) {
        unsigned long long xp[kCG / 2];
        if constexpr (Cfg::kXIo) {
#pragma unroll
          for (int c8 = 0; c8 < Cfg::kXCells; ++c8) {
            const uint4 v = xci[c8 * xr_plane];
            const uint32_t xw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              xp[c8 * 4 + i] = uncvt2<Op>(xw[i]);
              float e0, e1;
              f2_unpack(xp[c8 * 4 + i], e0, e1);
              const int c = cg * kCG + c8 * 8 + 2 * i;
              if (c < C) on[(size_t)c * P + pix] = from_f32<T>(e0);
              if (c + 1 < C) on[(size_t)(c + 1) * P + pix] = from_f32<T>(e1);
            }
          }
        }
#pragma unroll
        for (int q4 = 0; q4 < (Cfg::kXIo ? 0 : kQ4); ++q4) {
          const float4 v = xc[q4 * xr_plane];
          const float e[4] = {v.x, v.y, v.z, v.w};
          xp[2 * q4] = f2_pack(v.x, v.y);
          xp[2 * q4 + 1] = f2_pack(v.z, v.w);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int c = cg * kCG + q4 * 4 + k;
            if (c < C) on[(size_t)c * P + pix] = from_f32<T>(e[k]);
          }
        }
        if (p.planes != nullptr)
          store_plane_group<Op, Cfg::kSplit, kCG>(p, n, cg * kCG, C - cg * kCG, h, w, xp);
      }
      tc::mbar_arrive(&x_empty[xb]);
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

template <typename T, int KS, bool kStaged>
int launch_k(const FwdParams& prm, const FwdMaps& maps, cudaStream_t st) {
  using Cfg = FwdCfg<T, KS, kStaged>;
  FwdParams q = prm;
  q.nxb = 2;
  if ((int)fwd_smem_layout<T, KS, kStaged>(q.Ck, q.R, 2).total > max_smem_optin()) q.nxb = 1;
  const FwdSmem L = fwd_smem_layout<T, KS, kStaged>(q.Ck, q.R, q.nxb);
  if ((int)L.total > max_smem_optin())
    return set_error(DDPM_ERR_UNSUPPORTED, "forward tile needs %u bytes of shared memory",
                     L.total);
  auto fn = gencat_fwd_kernel<T, KS, kStaged>;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  const int per_cg = num_sms() / q.ncg;
  q.per_cg = q.num_tiles < per_cg ? q.num_tiles : per_cg;
  const int grid = q.ncg * q.per_cg;
  fn<<<grid, Cfg::kThreads, L.total, st>>>(q, maps);
  DDPM_CHECK_LAUNCH("gencat_fwd_kernel");
  return DDPM_OK;
}

template <typename T, int KS>
int launch(const FwdParams& prm, const FwdMaps& maps, bool staged, cudaStream_t st) {
  return staged ? launch_k<T, KS, true>(prm, maps, st) : launch_k<T, KS, false>(prm, maps, st);
}

template <typename T>
int dispatch(int ks, const FwdParams& prm, const FwdMaps& maps, bool staged, cudaStream_t st) {
  switch (ks) {
    case 1: return launch<T, 1>(prm, maps, staged, st);
    case 3: return launch<T, 3>(prm, maps, staged, st);
    case 5: return launch<T, 5>(prm, maps, staged, st);
  }
  return set_error(DDPM_ERR_UNSUPPORTED, "fused generator: kernel_size %d not supported", ks);
}

}  // namespace

// `staged`: staged operands (gencat::stage with x and y) or null to stage
// tiles from x and y.
namespace {

// Zero frame of staged fuse planes whose interior the forward writes: plane
// rows 0 and Hp-1, plane columns 0..7 and W+8..Wp-1, and channel groups at or
// beyond `gvalid`. One warp per plane row (part, n, group, row), rows strided
// over a grid of a few blocks per SM: an interior row is two short runs of
// 16-byte cells, one store instruction each.
__global__ void __launch_bounds__(256) plane_frame_zero_kernel(uint4* __restrict__ planes,
                                                               int rows, int G, int Hp, int Wp,
                                                               int W, int gvalid) {
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int tail = Wp - (W + 8);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += nwarps) {
    const int i = r % Hp;
    const int g = (r / Hp) % G;
    uint4* row = planes + (size_t)r * Wp;
    if (i == 0 || i == Hp - 1 || g >= gvalid) {
      for (int j = lane; j < Wp; j += 32) row[j] = z;
    } else {
      for (int j = lane; j < 8 + tail; j += 32) row[j < 8 ? j : W + j] = z;
    }
  }
}

}  // namespace

// `planes`: optional fuse-conv planes of the output (see FwdParams), or null.
int gencat_fwd_ex(const void* x, const void* y, const void* staged, size_t staged_bytes,
                  const void* wpack, const void* bias, void* out, void* planes,
                  size_t planes_bytes, int n, int c, int h, int w, int ks, int d0, int d1,
                  int d2, int dt, cudaStream_t st) {
  int rc = gencat::check_shape(n, c, h, w, ks, d0, d1, d2, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG(((x && y) || staged) && wpack && bias && out, "null pointer");
  FwdParams prm{};
  if (planes != nullptr) {
    if (c % 8 != 0)
      return set_error(DDPM_ERR_UNSUPPORTED,
                       "fuse planes from the forward need C %% 8 == 0 (got %d)", c);
    const fuseconv::PlaneLayout pl4 = fuseconv::PlaneLayout::make(n, 4 * c, h, w, dt);
    if (planes_bytes < pl4.bytes())
      return set_error(DDPM_ERR_WORKSPACE, "fuse planes too small (%zu < %zu)", planes_bytes,
                       pl4.bytes());
    DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(planes) & 255u) == 0,
                   "fuse planes must be 256-byte aligned");
    prm.planes = static_cast<uint8_t*>(planes);
    prm.pl_part = pl4.part_bytes;
    prm.pl_G = pl4.G;
    prm.pl_Hp = pl4.Hp;
    prm.pl_Wp = pl4.Wp;
    const long long rows = (long long)pl4.parts * pl4.N * pl4.G * pl4.Hp;
    DDPM_CHECK_ARG(rows < (1LL << 31), "too many plane rows");
    const long long blocks = (rows + 7) / 8;
    const int grid = (int)(blocks < 8LL * gencat::num_sms() ? blocks : 8LL * gencat::num_sms());
    plane_frame_zero_kernel<<<grid, 256, 0, st>>>(static_cast<uint4*>(planes), (int)rows, pl4.G,
                                                  pl4.Hp, pl4.Wp, w, (4 * c) / 8);
    DDPM_CHECK_LAUNCH("plane_frame_zero_kernel");
  }
  prm.x = x;
  prm.y = y;
  prm.wpack = wpack;
  prm.bias = bias;
  prm.out = out;
  prm.N = n;
  prm.C = c;
  prm.H = h;
  prm.W = w;
  const gencat::PackLayout pl = gencat::PackLayout::make(c, ks, dt);
  prm.Cp = pl.Cp;
  prm.Ck = pl.Ck;
  const int cgw = gencat::fwd_cg(ks, dt == DDPM_F32);
  prm.ncg = pl.Cp / cgw;
  prm.R = (ks / 2) * max3(d0, d1, d2);
  prm.d[0] = d0;
  prm.d[1] = d1;
  prm.d[2] = d2;
  prm.tiles_w = (w + gencat::kTileW - 1) / gencat::kTileW;
  prm.tiles_h = (h + gencat::kTileH - 1) / gencat::kTileH;
  prm.num_tiles = n * prm.tiles_w * prm.tiles_h;
  rc = gencat::status_ptr(&prm.status);
  if (rc) return rc;
  FwdMaps maps{};
  bool use_staged = false;
  if (staged != nullptr) {
    const gencat::StageLayout sl = gencat::StageLayout::make(n, c, h, w, ks, d0, d1, d2, dt);
    if (staged_bytes < sl.total_bytes())
      return set_error(DDPM_ERR_WORKSPACE, "staged operands too small (%zu < %zu)", staged_bytes,
                       sl.total_bytes());
    DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(staged) & 255u) == 0,
                   "staged operands must be 256-byte aligned");
    use_staged = gencat::encode_stage_maps(&maps.xmap, &maps.ymap, prm.R, pl.Ck / 8,
                                           static_cast<const uint8_t*>(staged), sl,
                                           gencat::fwd_halo_cols(ks), cgw / sl.xcell);
    maps.ph = sl.ph;
    maps.pw = sl.pw;
  }
  DDPM_CHECK_ARG(use_staged || (x && y), "tensor maps unavailable: x and y are needed");
  switch (dt) {
    case DDPM_BF16: return dispatch<__nv_bfloat16>(ks, prm, maps, use_staged, st);
    case DDPM_F16: return dispatch<__half>(ks, prm, maps, use_staged, st);
    case DDPM_F32: return dispatch<float>(ks, prm, maps, use_staged, st);
  }
  return set_error(DDPM_ERR_INVALID_ARG, "unknown dtype %d", dt);
}

int gencat_fwd_test_skip_arrive(int enable) {
  const int v = enable ? 1 : 0;
  DDPM_CUDA_TRY(cudaMemcpyToSymbol(g_test_skip_arrive, &v, sizeof(int)));
  return DDPM_OK;
}

int gencat_fwd(const void* x, const void* y, const void* staged, size_t staged_bytes,
               const void* wpack, const void* bias, void* out, int n, int c, int h, int w,
               int ks, int d0, int d1, int d2, int dt, cudaStream_t st) {
  return gencat_fwd_ex(x, y, staged, staged_bytes, wpack, bias, out, nullptr, 0, n, c, h, w, ks,
                       d0, d1, d2, dt, st);
}

}  // namespace ddpm
