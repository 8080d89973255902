// Common device helpers for the tinyserve-b200 kernels (sm_100a).
//
// - mbarrier / bulk-copy (TMA engine, non-tensor form) wrappers with bounded
//   waits: every spin gives up after a fixed number of polls, records an error
//   code in the caller-visible error word and lets the kernel return.
// - f16 magic-number conversions used to feed quantised weights into
//   mma.sync tensor-core instructions.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tsb {

// Error word codes written by kernels (read back by tsb_check_device_error()).
enum : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,   // an mbarrier wait exceeded its poll budget
  kDevBadPlan = 2,       // routing plan inconsistent (expert id out of range)
  kDevMisaligned = 3,    // a dense expert weight pointer is not 16-byte aligned (access skipped)
};

// Poll budget for mbarrier waits (each poll may suspend up to kSuspendNs).
constexpr uint32_t kMaxPolls = 4096;  // with the 1 ms suspend hint: a few seconds at most

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait with a suspend-time hint: a waiting thread sleeps in hardware until
// the phase completes or ~kSuspendNs elapse, so waiting warps do not take issue
// slots from the warps that are working (the producer in particular).
constexpr uint32_t kSuspendNs = 1000000;  // 1 ms per poll

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}

// Bounded wait (at most ~kMaxPolls hinted polls, i.e. a few seconds).  Returns
// false (and records kDevWaitTimeout) when the budget runs out; the caller then
// skips its work and unwinds.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  if (err) atomicExch(err, kDevWaitTimeout);
  return false;
}

// Bulk global->shared copy completing on an mbarrier (16-B aligned addresses,
// size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.  A pure
// register operation: not volatile, so the compiler may interleave the MMAs
// of one step with the loads and decode of the next.
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two e2m1 codes (low nibble -> low half) to f16x2, exact.
__device__ __forceinline__ uint32_t cvt_e2m1x2(uint32_t byte) {
  uint32_t r;
  asm("{\n .reg .b8 t;\n cvt.u8.u32 t, %1;\n cvt.rn.f16x2.e2m1x2 %0, t;\n}" : "=r"(r) : "r"(byte));
  return r;
}

// Packed half-precision arithmetic on f16x2 bit patterns (round to nearest,
// subnormals kept).
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t h2mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t h2fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  return __byte_perm(a, b, sel);
}

// Little-endian 32-bit load from a 2-byte aligned shared address.
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t* p) {
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
  return static_cast<uint32_t>(q[0]) | (static_cast<uint32_t>(q[1]) << 16);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// float -> bf16 round-to-nearest-even, NaN -> 0x7FC0 (the pattern torch writes).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

__device__ __forceinline__ float half_bits_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

}  // namespace tsb
