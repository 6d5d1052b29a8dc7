// sm_100a building blocks written as inline PTX: mbarriers with bounded
// waits, bulk async copies, tcgen05 TMEM allocation, UMMA descriptors,
// tcgen05.mma (kind::f16) and tcgen05.ld.
//
// Layout used for every UMMA operand in this library: the "interleaved"
// (SWIZZLE_NONE) canonical form. A K-major operand of R rows x Kc columns is
// stored as [Kc/8][R][8] 16-byte core-matrix rows: row r, k-chunk j lives at
// byte j*LBO + r*16, with LBO = R*16 (distance between k-chunks) and SBO = 128
// (distance between 8-row groups). Because rows are 16 bytes apart, a window
// that starts at ANY row is again a valid operand (start address + s*16):
// that is what lets the dX kernel read shifted pixel windows of one staged
// tile. MN-major operands (used for the weight-gradient GEMM) reuse the same
// bytes with LBO/SBO swapped in meaning (8 K-rows x 16 bytes per core matrix).
#pragma once

#include <stdint.h>

namespace ddpm {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------- mbarrier ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps (without issuing) until
// the phase completes or about `hint_ns` pass.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with `parity` to complete, for at most `limit_ns`.
// Returns false on timeout (the caller records the failure and unwinds);
// `abort_flag` (shared) lets one role stop the others early. With `hint_ns`,
// each try_wait may keep the thread suspended (not issuing) for up to that
// long, waking when the phase completes; the abort flag and the limit are
// then checked after every try.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag, uint64_t limit_ns,
                                          uint32_t hint_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    // try_wait itself parks the thread for a short, hardware-chosen time
    if (hint_ns != 0 ? mbar_try_wait_sleep(bar, parity, hint_ns) : mbar_try_wait(bar, parity))
      return true;
    if (hint_ns != 0 || (++spins & 63u) == 0) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) return false;
    }
  }
}

// --------------------------------------------------------- async proxies ---
// Make generic-proxy shared-memory writes visible to the async proxy
// (tcgen05.mma operand reads, bulk copies).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Four 8x8 matrices of 16-bit elements stored transposed (warp-collective).
// Register i of lane t holds elements (row t/4, columns 2(t%4) and 2(t%4)+1)
// of matrix i; column r of matrix i (8 elements, 16 bytes) is written to the
// shared address that lane 8i + r supplies.
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t addr, uint32_t r0, uint32_t r1,
                                                  uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};"
               :: "r"(addr), "r"(r0), "r"(r1), "r"(r2), "r"(r3) : "memory");
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// Both addresses 16-byte aligned, size a multiple of 16.
// Add `bytes` to the barrier's expected transaction count without arriving
// (for producers that arrive separately after issuing their copies).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Tiled tensor copy global -> shared (TMA), 4-D coordinates (innermost
// first), completion counted on `bar`. `tmap` is the generic address of a
// CUtensorMap held in kernel parameter space. No cluster multicast.
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, int c0, int c1, int c2,
                                            int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}

// Element-wise add of a shared-memory box into a global tensor (TMA reduction,
// 4-D tensor map), as a bulk async-group of the calling thread; coordinates
// must not be negative.
__device__ __forceinline__ void tma_reduce_add_4d(const void* tmap, const void* src, int c0,
                                                  int c1, int c2, int c3) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group"
      " [%0, {%2, %3, %4, %5}], [%1];" ::"l"(reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until every bulk async-group of this thread has read its source.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until every bulk async-group of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// 5-D variant of tma_load_4d.
__device__ __forceinline__ void tma_load_5d(void* dst, const void* tmap, int c0, int c1, int c2,
                                            int c3, int c4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(smem_u32(bar))
      : "memory");
}

// ----------------------------------------------------------------- TMEM ----
// Allocate `ncols` (power of two >= 32) TMEM columns; the base address is
// written to `*dst_smem`. Must be executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ------------------------------------------------------------- UMMA desc ---
// Shared-memory matrix descriptor, SWIZZLE_NONE, sm_100 version bits.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  // base offset 0, lbo mode 0, layout type 0 (SWIZZLE_NONE)
  return d;
}

// Descriptor of a K-major operand in the 128-byte swizzled form written by a
// TMA copy with SWIZZLE_128B: one 128-byte row per M/N index (64 16-bit K
// elements), 16-byte chunk j of row r stored at chunk j ^ (r % 8), 8-row
// groups 1024 bytes apart (SBO). The atom base must be 1024-byte aligned; a
// K step of 16 elements advances the start address by 32 bytes.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;            // LBO (unused for swizzled K-major), 16 bytes
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO
  d |= (uint64_t)1 << 46;            // descriptor version for sm_100
  d |= (uint64_t)2 << 61;            // layout type: SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with FP32 accumulation.
// ab_bf16: operands are bf16 (else fp16). a_mn / b_mn: operand is MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool ab_bf16, bool a_mn,
                                                 bool b_mn) {
  return (1u << 4)                                   // D format: F32
         | ((ab_bf16 ? 1u : 0u) << 7)                // A format
         | ((ab_bf16 ? 1u : 0u) << 10)               // B format
         | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16)
         | ((uint32_t)(N >> 3) << 17)                // N / 8
         | ((uint32_t)(M >> 4) << 24);               // M / 16
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by a single thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Each thread of the warp loads 16 consecutive 32-bit columns of its lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 8 and 4 consecutive columns (narrower channel groups).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float* v) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
// G (16, 8 or 4) consecutive columns.
template <int G>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float* v) {
  if constexpr (G == 16) tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(v));
  else if constexpr (G == 8) tmem_ld8(taddr, v);
  else tmem_ld4(taddr, v);
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t.reg .b32 r;\n\t"
      "elect.sync r|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred;
}

}  // namespace tc
}  // namespace ddpm
