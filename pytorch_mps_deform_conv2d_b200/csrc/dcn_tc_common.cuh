// dcn_tc_common.cuh -- inline-PTX helpers for the tcgen05 kernels: mbarriers
// with bounded waits, tensor-memory allocation, TF32 UMMA issue and commit,
// tensor-memory loads, shared-memory matrix descriptors, cp.async.
//
// Shared-memory operand layout used by every tcgen05 kernel here: K-major,
// 128-byte swizzle.  A row (one M or N index) holds 32 fp32 K values = 128 B
// as eight 16-byte chunks; chunk j of row r is stored at
//     r * 128 + ((j ^ (r & 7)) << 4)
// and rows are grouped by 8 into 1024-byte atoms stacked along M/N (stride
// 1024 B).  Every stage buffer starts on a 1024-byte boundary.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace dcn {
namespace tc {

// ---- error flag set by a kernel whose wait ran out (no trap, no hang) ----
__device__ __forceinline__ void flag_timeout(int* err, int code) {
  if (err) atomicExch(err, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// One hardware-suspended wait attempt: the thread sleeps until the phase
// completes or up to ~1 ms passes (the suspend-time hint, in ns), so a
// waiting warp spends few issue slots polling; callers bound the total wait
// by their own cycle count.
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
// Waits until the phase with the given parity has completed.  Gives up after
// ~`limit_cycles` SM clocks (then returns false and raises *err).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err,
                                          long long limit_cycles = 4000000000LL) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (clock64() - t0 > limit_cycles) {
      flag_timeout(err, 1);
      return false;
    }
  }
  return true;
}

// ---- bounded waits with a CTA-wide give-up ----
// Every wait of the warp-specialised kernels goes through a Watch.  The first
// wait of a CTA that runs out of its cycle budget raises bit `code` of the
// global error word `status` and the CTA's abort flag (shared memory); from
// then on every wait of the CTA gives up at once, so each role leaves its
// loop, drains what it issued (drain_wait) and reaches the kernel's final
// barrier, where tensor memory is freed.  No wait spins unbounded, none traps.
struct Watch {
  int* abort;       // shared memory, 0 until a wait of this CTA gives up
  int* status;      // global error word
  int code;         // bit raised in *status
  long long limit;  // SM clock cycles a wait may take
};
__device__ __forceinline__ bool aborted(const Watch& w) {
  return *reinterpret_cast<volatile int*>(w.abort) != 0;
}
__device__ __forceinline__ bool wait(const Watch& w, uint64_t* bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (aborted(w)) return false;
    if (mbar_try(bar, parity)) return true;
    if (clock64() - t0 > w.limit) {
      *reinterpret_cast<volatile int*>(w.abort) = 1;
      atomicOr(w.status, w.code);
      return false;
    }
  }
}
// After an abort: waits (bounded, ignoring the abort flag) for a phase that
// only this thread's own asynchronous work completes -- its TMA copies or
// its tcgen05.commit -- so nothing is in flight when the CTA frees its
// shared and tensor memory.
__device__ __forceinline__ bool drain_wait(uint64_t* bar, uint32_t parity, long long limit) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity))
    if (clock64() - t0 > limit) return false;
  return true;
}

// ---- tensor memory ----
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
// Generic-proxy shared-memory writes -> visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- UMMA ----
// Instruction descriptor, kind::tf32: D fp32, A/B tf32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 1024-byte atom
// stride (SBO), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}
// kind::f16 with bf16 A and B (both the same type), fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
// kind::f16 with fp16 A and B, fp32 accumulation (A / B format fields 0).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// One kind::f16 UMMA (bf16 or fp16 operands, as the instruction descriptor says).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on `bar` once every previously issued tcgen05.mma of this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32-bit, 8 consecutive columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- conversions / copies ----
// fp32 -> tf32 with round-to-nearest (ties away); the tensor core would
// otherwise drop the low 13 mantissa bits.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
__device__ __forceinline__ void cp_async16(uint32_t dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

}  // namespace tc
}  // namespace dcn

// ---- TMA (bulk tensor copies) and plain mbarrier arrivals ----
#include <cuda.h>

namespace dcn {
namespace tc {

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// 2-D tiled TMA load (no multicast): box at (x = inner element index, y = row)
// into `dst` (1024-byte aligned for the 128-byte swizzle), completion counted
// in bytes on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace tc
}  // namespace dcn
