// Thin inline-PTX wrappers for the sm_100a tensor-core engine: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM allocation, MMA, commit,
// loads) and the shared-memory matrix / instruction descriptors of UMMA.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace lcb200 {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of parity `parity` to complete, for at most
// `timeout_ns`, regardless of any abort flag (draining copies in flight
// before a block exits). Returns false on timeout.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity,
                                                uint64_t timeout_ns = 2000000000ull) {
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && globaltimer() - t0 > timeout_ns) return false;
  }
}

// Wait for the phase of parity `parity` to complete, for at most
// `timeout_ns`. Gives up early when *abort is set by another thread. On
// timeout, sets *abort and returns false; every caller then winds down.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t timeout_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (*abort) return false;
      if (globaltimer() - t0 > timeout_ns) {
        *abort = 1;
        return false;
      }
    }
  }
}

// ---- async proxy / TMA --------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 16-byte cp.async with zero fill when src_bytes == 0.
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has
// landed; the arrival counts toward the barrier's expected count.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// ---- tcgen05 ------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (fp16/bf16 in, fp32 acc).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}

// n (1..4) MMAs into one accumulator, issued from one statement: MMA k reads
// descriptors a0 + k*astep and b0 + k*bstep (start-address units of 16
// bytes); the first accumulates when acc != 0, the others always. Every
// operand is a distinct input register of the one statement: a descriptor
// register that the next batch overwrites is not still waiting to be read
// by a queued MMA of this batch, so batches issue back to back (one
// descriptor per statement, rewritten per MMA, runs the MMAs at their
// latency instead of their throughput).
__device__ __forceinline__ void mma_f16_ss_n(uint32_t d_tmem, uint64_t a0, uint32_t astep,
                                             uint64_t b0, uint32_t bstep, uint32_t idesc,
                                             uint32_t acc, int n) {
  const uint64_t a1 = a0 + astep, a2 = a1 + astep, a3 = a2 + astep;
  const uint64_t b1 = b0 + bstep, b2 = b1 + bstep, b3 = b2 + bstep;
  if (n >= 4) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %10, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %5, %9, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %6, %9, 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %9, 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %9, 1;\n\t}" ::"r"(d_tmem),
        "l"(a0), "l"(a1), "l"(a2), "l"(a3), "l"(b0), "l"(b1), "l"(b2), "l"(b3), "r"(idesc),
        "r"(acc));
  } else if (n == 3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %8, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %4, %7, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %5, %7, 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %6, %7, 1;\n\t}" ::"r"(d_tmem),
        "l"(a0), "l"(a1), "l"(a2), "l"(b0), "l"(b1), "l"(b2), "r"(idesc), "r"(acc));
  } else if (n == 2) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %3, %5, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %4, %5, 1;\n\t}" ::"r"(d_tmem),
        "l"(a0), "l"(a1), "l"(b0), "l"(b1), "r"(idesc), "r"(acc));
  } else if (n == 1) {
    mma_f16_ss(d_tmem, a0, b0, idesc, acc);
  }
}

// Arrive once on `bar` when all previously issued tcgen05 ops of this thread
// have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
      "[%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 16 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- UMMA descriptors -----------------------------------------------------------
// Shared-memory matrix descriptor, SWIZZLE_128B canonical layouts:
//  * K-major: rows of 128 B (64 fp16 along K), 8-row swizzle atoms of 1024 B
//    stacked along M/N with stride `sbo` (1024 when contiguous); lbo unused (1).
//  * MN-major: rows of 128 B (64 fp16 along M/N), 8 K-rows per 1024-B atom
//    (`sbo` = stride between 8-row K groups), `lbo` = stride between 64-wide
//    M/N blocks.
// Bit layout: start>>4 [0,14), lbo>>4 [16,30), sbo>>4 [32,46), version 1 at
// [46,48), base offset 0, layout type 2 (SWIZZLE_128B) at [61,64).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: A/B fp16, D fp32, given majors, MxN.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, bool a_mn_major,
                                                     bool b_mn_major) {
  return (1u << 4)                      // D format: f32
         | (0u << 7) | (0u << 10)       // A, B: f16
         | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

}  // namespace tc
}  // namespace lcb200
