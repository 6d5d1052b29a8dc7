// Diagnostic: one 128 x N x K bf16 UMMA (tcgen05.mma, accumulator in TMEM)
// on a single CTA, exercising exactly the operand layouts the fused DDPM
// kernels rely on, so a descriptor or layout mistake shows up as a plain
// numeric mismatch in a test instead of inside a fused kernel.
//   variant 0: A K-major, B K-major
//   variant 1: A MN-major, B K-major
//   variant 2: A K-major, window starting `shift` rows into the staged tile
//              (any row offset, not only multiples of 8)
//   variant 3: A K-major, B MN-major with its K window starting `shift` rows
//              into the staged tile (B given as [n, k + shift])
// D[m, n] = sum_k A[shift + m, k] * B[n, k] (variants 0-2) or
// sum_k A[m, k] * B[n, shift + k] (variant 3); A, B row-major bf16 in global,
// D row-major fp32.
#include "common.cuh"
#include "tc.cuh"

namespace ddpm {
namespace {

constexpr int kM = 128;

__global__ void __launch_bounds__(128)
umma_selftest_kernel(const __nv_bfloat16* __restrict__ A, const __nv_bfloat16* __restrict__ B,
                     float* __restrict__ D, int N, int K, int shift, int variant,
                     int* __restrict__ status) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const bool b_mn = (variant == 3);
  const int rows_a = b_mn ? kM : kM + shift;
  const int kb = b_mn ? K + shift : K;  // staged K extent of B
  uint8_t* sA = smem;
  uint8_t* sB = smem + (size_t)rows_a * K * 2;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_base, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  // Stage A in the requested layout.
  const bool a_mn = (variant == 1);
  for (int i = tid; i < rows_a * K; i += blockDim.x) {
    const int r = i / K, k = i - (i / K) * K;
    uint32_t off;
    if (!a_mn) {
      off = ((k >> 3) * rows_a + r) * 16 + (k & 7) * 2;  // LBO = rows_a*16, SBO = 128
    } else {
      off = (r >> 3) * (K * 16) + (k >> 3) * 128 + (k & 7) * 16 + (r & 7) * 2;  // SBO=K*16, LBO=128
    }
    *reinterpret_cast<__nv_bfloat16*>(sA + off) = A[i];
  }
  for (int i = tid; i < N * kb; i += blockDim.x) {
    const int r = i / kb, k = i - (i / kb) * kb;
    uint32_t off;
    if (!b_mn)
      off = ((k >> 3) * N + r) * 16 + (k & 7) * 2;  // LBO = N*16, SBO = 128
    else
      off = (r >> 3) * (kb * 16) + k * 16 + (r & 7) * 2;  // LBO = 128, SBO = kb*16
    *reinterpret_cast<__nv_bfloat16*>(sB + off) = B[i];
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (tid == 0) {
    const uint32_t a0 = tc::smem_u32(sA);
    const uint32_t b0 = tc::smem_u32(sB);
    const uint32_t idesc = tc::idesc_f16(kM, N, true, a_mn, b_mn);
    for (int ks = 0; ks < K / 16; ++ks) {
      uint64_t ad, bd;
      if (!a_mn) {
        const uint32_t lbo = rows_a * 16;
        ad = tc::smem_desc(a0 + (variant == 2 ? shift * 16 : 0) + ks * 2 * lbo, lbo, 128);
      } else {
        ad = tc::smem_desc(a0 + ks * 2 * 128, 128, K * 16);
      }
      if (!b_mn) {
        const uint32_t lbob = N * 16;
        bd = tc::smem_desc(b0 + ks * 2 * lbob, lbob, 128);
      } else {
        bd = tc::smem_desc(b0 + shift * 16 + ks * 2 * 128, 128, kb * 16);
      }
      tc::mma_f16(tmem, ad, bd, idesc, ks > 0 ? 1u : 0u);
    }
    tc::mma_commit(&bar);
  }
  __syncwarp();
  const bool ok = tc::mbar_wait(&bar, 0, &abort_flag, 2000000000ull);
  if (!ok) {
    abort_flag = 1;
    if (lane == 0) atomicExch(status, 1);
  }
  tc::tc_fence_after();
  if (ok) {
    const int row = warp * 32 + lane;
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      tc::tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
      tc::tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) D[(size_t)row * N + c0 + j] = v[j];
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 256);
}

__device__ int g_selftest_status;

}  // namespace

int umma_selftest(int variant, const void* a, const void* b, float* d, int n, int k, int shift,
                  cudaStream_t st) {
  DDPM_CHECK_ARG(a && b && d, "null pointer");
  DDPM_CHECK_ARG(variant >= 0 && variant <= 3, "variant must be 0, 1, 2 or 3");
  DDPM_CHECK_ARG(n >= 16 && n <= 256 && n % 16 == 0, "n must be a multiple of 16 in [16, 256]");
  DDPM_CHECK_ARG(k >= 16 && k <= 128 && k % 16 == 0, "k must be a multiple of 16 in [16, 128]");
  DDPM_CHECK_ARG(shift >= 0 && shift <= 32 && (variant >= 2 || shift == 0), "bad shift");
  const size_t smem = variant == 3 ? (size_t)kM * k * 2 + (size_t)n * (k + shift) * 2
                                   : (size_t)(kM + shift) * k * 2 + (size_t)n * k * 2;
  DDPM_CUDA_TRY(cudaFuncSetAttribute(umma_selftest_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int* status = nullptr;
  DDPM_CUDA_TRY(cudaGetSymbolAddress((void**)&status, g_selftest_status));
  umma_selftest_kernel<<<1, 128, smem, st>>>(static_cast<const __nv_bfloat16*>(a),
                                             static_cast<const __nv_bfloat16*>(b), d, n, k,
                                             shift, variant, status);
  DDPM_CHECK_LAUNCH("umma_selftest_kernel");
  return DDPM_OK;
}

}  // namespace ddpm
