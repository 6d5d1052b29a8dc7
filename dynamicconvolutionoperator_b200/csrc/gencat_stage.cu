// Staged operands of the fused generator backward (layout: StageLayout in
// gencat.cuh). One pass over y writes it channel-last in the MMA operand type,
// zero padded and with the constant-one bias channel; one pass over x writes
// it as 16-byte cells (FP32: 4 channels; 16-bit types: 8 channels in the
// input type). The backward kernels then stage their tiles with
// 1-D bulk / TMA copies instead of per-thread loads and register transposes
// (which bounded them by load latency).
#include <cstring>

#include "common.cuh"
#include "gencat.cuh"

namespace ddpm {
namespace {

using namespace gencat;

constexpr int kStageCols = 64;               // plane columns per block
constexpr int kStageChannels = kMaxChannels + 16;  // G*8 <= round16(64 + 1)

// Block = (n, plane row, 64-column strip). Loads: 8 lanes read 8-pixel
// vectors covering 64 contiguous columns of one channel; a shared tile with a
// 68-float row pitch (16-byte aligned rows for the vector stores, column
// reads still conflict-free) transposes; each thread writes 16-byte rows of
// 8 channels (consecutive lanes = consecutive columns).
template <typename T>
__global__ void __launch_bounds__(256) stage_y_kernel(const T* __restrict__ y,
                                                      uint4* __restrict__ hi,
                                                      uint4* __restrict__ lo,
                                                      const StageLayout L) {
  using Op = typename IoTraits<T>::Op;
  constexpr bool kSplit = IoTraits<T>::kSplit;
  __shared__ __align__(16) float tile[kStageChannels][kStageCols + 4];
  const int ni = blockIdx.x, n = ni / L.Hp, i = ni - n * L.Hp;
  const int hr = i - L.ph;                // image row (may be outside the image)
  const int j0 = blockIdx.y * kStageCols;  // first plane column of the block
  const int nc = L.G * 8;
  const size_t P = (size_t)L.H * L.W;
  for (int item = threadIdx.x; item < nc * (kStageCols / 8); item += blockDim.x) {
    const int g = item & 7, c = item >> 3;
    Raw8<T> v;
    if (c < L.C)
      v = load_raw8<T>(y + ((size_t)n * L.C + c) * P, L.H, L.W, hr, j0 - L.pw + g * 8);
    else if (c == L.C)
      v.ones();
    else
      v.zero();
    float4* row = reinterpret_cast<float4*>(&tile[c][g * 8]);
    row[0] = make_float4(v.get(0), v.get(1), v.get(2), v.get(3));
    row[1] = make_float4(v.get(4), v.get(5), v.get(6), v.get(7));
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < L.G * kStageCols; idx += blockDim.x) {
    const int kg = idx / kStageCols, x = idx - kg * kStageCols;
    if (j0 + x >= L.Wp) continue;
    unsigned long long pr[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[e] = f2_pack(tile[kg * 8 + 2 * e][x], tile[kg * 8 + 2 * e + 1][x]);
    const size_t dst = L.row_offset(0, n, i, kg, j0 + x) / 16;
    uint4 vh, vl;
    store8x2_split<Op, kSplit>(reinterpret_cast<uint8_t*>(&vh), reinterpret_cast<uint8_t*>(&vl), pr);
    hi[dst] = vh;
    if constexpr (kSplit) lo[dst] = vl;
  }
}

// The y plane for 16-bit data: the same rows, transposed in the input type
// (no FP32 round trip) through a [channel][128 + 8 px] tile of 16-bit values
// (272-byte rows, 16-byte aligned); block = (n, plane row, 128-column strip).
// Each thread issues all of its 16-byte pixel-vector loads (5 at most) before
// its first shared store; the writes are 16-byte rows of 8 channels,
// consecutive threads at consecutive plane columns.
template <typename T>
__global__ void __launch_bounds__(256) stage_y16_kernel(const T* __restrict__ y,
                                                        uint4* __restrict__ out,
                                                        const StageLayout L) {
  constexpr int kCols = 128;
  constexpr int kGroups = kCols / 8;  // 8-pixel vectors per channel row
  constexpr int kItems = (kStageChannels * kGroups + 255) / 256;
  __shared__ __align__(16) uint16_t tile[kStageChannels][kCols + 8];
  const int ni = blockIdx.x, n = ni / L.Hp, i = ni - n * L.Hp;
  const int hr = i - L.ph;                 // image row (may be outside the image)
  const int j0 = blockIdx.y * kCols;       // first plane column of the block
  const int items = L.G * 8 * kGroups;
  const size_t P = (size_t)L.H * L.W;
  Raw8<T> v[kItems];
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const int item = threadIdx.x + u * 256;
    const int g = item % kGroups, c = item / kGroups;
    if (item < items && c < L.C)
      v[u] = load_raw8<T>(y + ((size_t)n * L.C + c) * P, L.H, L.W, hr, j0 - L.pw + g * 8);
    else if (c == L.C)
      v[u].ones();
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
  for (int idx = threadIdx.x; idx < L.G * kCols; idx += blockDim.x) {
    const int kg = idx / kCols, x = idx - kg * kCols;
    if (j0 + x >= L.Wp) continue;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      w[e] = (uint32_t)tile[kg * 8 + 2 * e][x] | ((uint32_t)tile[kg * 8 + 2 * e + 1][x] << 16);
    out[L.row_offset(0, n, i, kg, j0 + x) / 16] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// x plane: thread = one 16-byte cell (n, cell q, h, w) = x[n, q*xcell ..
// q*xcell + xcell-1, h, w]: FP32 cells of 4 channels, or 16-bit cells of 8
// channels in the input type (channels >= C zero); consecutive threads =
// consecutive columns.
template <typename T>
__global__ void __launch_bounds__(256) stage_x_kernel(const T* __restrict__ x,
                                                      uint4* __restrict__ xp,
                                                      const StageLayout L) {
  constexpr int kCh = sizeof(T) == 4 ? 4 : 8;  // channels per cell
  const size_t P = (size_t)L.H * L.W;
  const size_t cells = (size_t)L.N * L.Cq * P;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  // four cells per thread per round, all loads issued before the stores
  for (size_t i0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i0 < cells; i0 += 4 * stride) {
    T v[4][kCh];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const size_t i = i0 + r * stride;
      const size_t pix = i % P;
      const size_t nq = i / P;
      const int q = (int)(nq % L.Cq), n = (int)(nq / L.Cq);
#pragma unroll
      for (int k = 0; k < kCh; ++k) {
        const int c = kCh * q + k;
        v[r][k] = (i < cells && c < L.C) ? __ldg(x + ((size_t)n * L.C + c) * P + pix) : T(0.f);
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const size_t i = i0 + r * stride;
      uint32_t wv[4];
      memcpy(wv, v[r], 16);  // registers: the store below is one 16-byte store
      if (i < cells) xp[i] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
  }
}

// The same x plane from 16-byte vectors: block = (pixel range, (n, cell)),
// thread = 8 consecutive pixels of the cell's channels (one vector load per
// channel), written as 8 consecutive cells (128 contiguous bytes); no index
// division per cell. Needs H*W % 8 == 0 and a 16-byte aligned x.
template <typename T>
__global__ void __launch_bounds__(256) stage_x_vec_kernel(const T* __restrict__ x,
                                                          uint4* __restrict__ xp,
                                                          const StageLayout L) {
  const size_t P = (size_t)L.H * L.W;
  const int nq = blockIdx.y, n = nq / L.Cq, q = nq - n * L.Cq;
  const size_t p0 = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (p0 >= P) return;
  uint4* dst = xp + ((size_t)n * L.Cq + q) * P + p0;
  if constexpr (sizeof(T) == 4) {
    float v[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = 4 * q + k;
      if (c < L.C) {
        const float4* src = reinterpret_cast<const float4*>(x + ((size_t)n * L.C + c) * P + p0);
        const float4 a = __ldg(src);
        const float4 b = __ldg(src + 1);
        v[k][0] = a.x; v[k][1] = a.y; v[k][2] = a.z; v[k][3] = a.w;
        v[k][4] = b.x; v[k][5] = b.y; v[k][6] = b.z; v[k][7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[k][i] = 0.f;
      }
    }
    float4* dstf = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int e = 0; e < 8; ++e) dstf[e] = make_float4(v[0][e], v[1][e], v[2][e], v[3][e]);
  } else {
    // u[k] = channel 8q + k at pixels p0 .. p0+7 (word j = pixels 2j, 2j+1);
    // cell e, word k = channels (2k, 2k+1) at pixel p0 + e
    uint32_t u[8][4];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = 8 * q + k;
      uint4 t = make_uint4(0u, 0u, 0u, 0u);
      if (c < L.C) t = __ldg(reinterpret_cast<const uint4*>(x + ((size_t)n * L.C + c) * P + p0));
      u[k][0] = t.x; u[k][1] = t.y; u[k][2] = t.z; u[k][3] = t.w;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t sel = (e & 1) ? 0x7632u : 0x5410u;  // high or low halves
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) w[k] = __byte_perm(u[2 * k][e >> 1], u[2 * k + 1][e >> 1], sel);
      dst[e] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <typename T>
int launch_stage(const T* x, const T* y, uint8_t* staged, const StageLayout& L, cudaStream_t st) {
  uint4* hi = reinterpret_cast<uint4*>(staged);
  uint4* lo = L.parts > 1 ? reinterpret_cast<uint4*>(staged + L.part_bytes) : nullptr;
  if constexpr (sizeof(T) == 2) {
    const dim3 grid((unsigned)(L.N * L.Hp), (unsigned)((L.Wp + 127) / 128));
    stage_y16_kernel<T><<<grid, 256, 0, st>>>(y, hi, L);
    DDPM_CHECK_LAUNCH("stage_y16_kernel");
  } else {
    const dim3 grid((unsigned)(L.N * L.Hp), (unsigned)((L.Wp + kStageCols - 1) / kStageCols));
    stage_y_kernel<T><<<grid, 256, 0, st>>>(y, hi, lo, L);
    DDPM_CHECK_LAUNCH("stage_y_kernel");
  }
  const size_t P = (size_t)L.H * L.W;
  if (x != nullptr && P % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
      (size_t)L.N * L.Cq <= 65535u) {
    const dim3 grid((unsigned)((P / 8 + 255) / 256), (unsigned)(L.N * L.Cq));
    stage_x_vec_kernel<T><<<grid, 256, 0, st>>>(
        x, reinterpret_cast<uint4*>(staged + L.x_offset), L);
    DDPM_CHECK_LAUNCH("stage_x_vec_kernel");
  } else if (x != nullptr) {
    const size_t cells = (size_t)L.N * L.Cq * L.H * L.W;
    size_t blocks = (cells + 4 * 256 - 1) / (4 * 256);  // four cells per thread
    if (blocks > 65535u * 8u) blocks = 65535u * 8u;
    stage_x_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(
        x, reinterpret_cast<uint4*>(staged + L.x_offset), L);
    DDPM_CHECK_LAUNCH("stage_x_kernel");
  }
  return DDPM_OK;
}

}  // namespace

namespace gencat {

size_t stage_bytes(int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt) {
  if (check_shape(n, c, h, w, ks, d0, d1, d2, dt) != DDPM_OK) {
    clear_error();
    return 0;
  }
  return StageLayout::make(n, c, h, w, ks, d0, d1, d2, dt).total_bytes();
}

int stage(const void* x, const void* y, void* staged, size_t staged_bytes, int n, int c, int h,
          int w, int ks, int d0, int d1, int d2, int dt, cudaStream_t st) {
  int rc = check_shape(n, c, h, w, ks, d0, d1, d2, dt);
  if (rc) return rc;
  DDPM_CHECK_ARG(y && staged, "null pointer");
  const StageLayout L = StageLayout::make(n, c, h, w, ks, d0, d1, d2, dt);
  const size_t need = x != nullptr ? L.total_bytes() : L.y_bytes();
  if (staged_bytes < need)
    return set_error(DDPM_ERR_WORKSPACE, "staged buffer too small (%zu < %zu)", staged_bytes,
                     need);
  DDPM_CHECK_ARG((reinterpret_cast<uintptr_t>(staged) & 255u) == 0,
                 "staged buffer must be 256-byte aligned");
  uint8_t* s = static_cast<uint8_t*>(staged);
  switch (dt) {
    case DDPM_BF16:
      return launch_stage(static_cast<const __nv_bfloat16*>(x),
                          static_cast<const __nv_bfloat16*>(y), s, L, st);
    case DDPM_F16:
      return launch_stage(static_cast<const __half*>(x), static_cast<const __half*>(y), s, L, st);
    default:
      return launch_stage(static_cast<const float*>(x), static_cast<const float*>(y), s, L, st);
  }
}

bool encode_stage_maps(CUtensorMap* xmap, CUtensorMap* ymap, int R, int ygroups,
                       const uint8_t* staged, const StageLayout& sl, int halo_cols, int cells) {
  const uint64_t xd[4] = {(uint64_t)sl.W * 2, (uint64_t)sl.H, (uint64_t)sl.Cq, (uint64_t)sl.N};
  const uint64_t xs[3] = {(uint64_t)sl.W * 16, (uint64_t)sl.H * sl.W * 16,
                          (uint64_t)sl.Cq * sl.H * sl.W * 16};
  const uint32_t xb[4] = {(uint32_t)(2 * halo_cols), (uint32_t)(kTileH + 2 * R),
                          (uint32_t)cells, 1};
  const uint64_t yd[4] = {(uint64_t)sl.Wp * 2, (uint64_t)sl.Hp, (uint64_t)sl.G,
                          (uint64_t)sl.parts * sl.N};
  const uint64_t ys[3] = {(uint64_t)sl.Wp * 16, (uint64_t)sl.Hp * sl.Wp * 16,
                          (uint64_t)sl.G * sl.Hp * sl.Wp * 16};
  const uint32_t yb[4] = {2 * kTileW, (uint32_t)kTileH, (uint32_t)ygroups, 1};
  if (encode_tmap(xmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, staged + sl.x_offset, xd, xs, xb,
                  CU_TENSOR_MAP_SWIZZLE_NONE) != DDPM_OK ||
      encode_tmap(ymap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, staged, yd, ys, yb,
                  CU_TENSOR_MAP_SWIZZLE_NONE) != DDPM_OK) {
    clear_error();
    return false;
  }
  return true;
}

bool encode_stage_segment_map(CUtensorMap* map, int ngroups, const uint8_t* staged,
                              const StageLayout& sl, int blocks) {
  // 16-pixel blocks of 256 bytes as the two inner dimensions, so one box of
  // `blocks` blocks x ngroups lands as [group][16 * blocks px][16 B] (9 blocks:
  // group stride 2304 B)
  const uint64_t d[5] = {32, (uint64_t)sl.Wp / 16, (uint64_t)sl.Hp, (uint64_t)sl.G,
                         (uint64_t)sl.parts * sl.N};
  const uint64_t s[4] = {256, (uint64_t)sl.Wp * 16, (uint64_t)sl.Hp * sl.Wp * 16,
                         (uint64_t)sl.G * sl.Hp * sl.Wp * 16};
  const uint32_t box[5] = {32, (uint32_t)blocks, 1, (uint32_t)ngroups, 1};
  if (encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 5, staged, d, s, box,
                  CU_TENSOR_MAP_SWIZZLE_NONE) != DDPM_OK) {
    clear_error();
    return false;
  }
  return true;
}

}  // namespace gencat
}  // namespace ddpm
