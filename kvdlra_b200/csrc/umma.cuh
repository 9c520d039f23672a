// Thin wrappers over the sm_100a 5th-generation tensor-core instructions
// (tcgen05) and the mbarrier they complete on, as this library uses them:
// one CTA (cta_group::1), both operands in shared memory, fp32 accumulators
// in tensor memory (TMEM), TF32 operands.  Instruction and descriptor formats
// follow the PTX ISA (tcgen05 "Matrix Descriptors", "Instruction
// descriptor"); the field layouts are the ones CUTLASS 4.x spells out in
// cute/arch/mma_sm100_desc.hpp.
#pragma once

#include <cstdint>

namespace kvd {
namespace umma {

// ---------------------------------------------------------------- descriptors

// Shared-memory matrix descriptor, no swizzle ("interleaved" canonical
// layout): the operand is a grid of core matrices of 8 rows x 16 bytes, each
// stored as 128 contiguous bytes (row i at byte 16 i).  `lbo` is the byte
// distance between core matrices adjacent along K, `sbo` between core
// matrices adjacent along M (or N).  Bits: [0,14) start >> 4, [16,30) lbo >> 4,
// [32,46) sbo >> 4, [46,48) descriptor version (1 on sm_100), [49,52) base
// offset (0: no swizzle), [61,64) layout type (0: no swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptor of kind::tf32 with fp32 accumulation, both operands
// K-major, dense: [4,6) D format (1 = F32), [7,10) A format (2 = TF32),
// [10,13) B format (2 = TF32), [15] A major (0 = K), [16] B major (0 = K),
// [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// The same for kind::f16 with both operands BF16 (format 1), fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------- TMEM

// Allocate `ncols` TMEM columns (a power of two >= 32); the base address is
// written to *smem_dst.  One full warp executes it.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(smem_dst);
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(a), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread t of the warp gets lane
// (taddr's lane + t), columns [col, col + 16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Ordering of tcgen05 work around thread synchronisation.
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes made visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- MMA

// D[tmem] (+)= A[smem] x B[smem]^T, kind::tf32, M x N x 8, issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
  const uint32_t z = 0;  // disable-output-lane mask: every lane written
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate), "r"(z)
      : "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T, kind::f16 (BF16 operands), M x N x 16.
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate), "r"(z)
      : "memory");
}

// Arrive on the mbarrier once every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void commit(uint64_t* mbar) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(mbar);
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(a)
               : "memory");
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(mbar);
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* mbar, uint32_t parity) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(mbar);
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` to complete, giving up after `limit` polls (each
// try_wait itself blocks for a hardware time slice); returns false then.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* mbar, uint32_t parity, long limit) {
  for (long i = 0; i < limit; ++i)
    if (mbar_try_wait(mbar, parity)) return true;
  return false;
}

// Round an fp32 value to TF32 (round to nearest, ties away), as a float.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

}  // namespace umma
}  // namespace kvd
