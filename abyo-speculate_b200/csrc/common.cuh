// Shared device helpers for the sm_100a verify-step kernels.
//
// Everything here is inline PTX or plain CUDA; no library kernels are used on
// the hot path.  The helpers cover:
//   * mma.sync m16n8k16 (f16 and bf16 inputs, f32 accumulate),
//   * TMA bulk copies (cp.async.bulk global -> shared, completion on an
//     mbarrier) and mbarrier waits that give up after a bounded number of
//     polls, setting an error flag instead of spinning forever,
//   * programmatic dependent launch (griddepcontrol) so a kernel can start
//     streaming weights while its predecessor is still finishing.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "kernels.cuh"

#define SPEC_DEV __device__ __forceinline__

namespace specb200 {

// A wait on an mbarrier is declared hung after this much wall time (ns, from
// %globaltimer), or after kMbarMaxPolls polls, whichever comes first.
constexpr unsigned long long kMbarTimeoutNs = 2000000000ull;
constexpr unsigned kMbarMaxPolls = 1u << 30;

SPEC_DEV unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

SPEC_DEV void pdl_wait() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}

SPEC_DEV void pdl_launch_dependents() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

SPEC_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

SPEC_DEV void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

SPEC_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

SPEC_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Returns true when the phase with parity `parity` has completed.
SPEC_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Bounded wait: returns false (and raises DEV_ERR_MBAR_TIMEOUT) if the phase
// never completes.  The caller must then skip its remaining work.
SPEC_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (unsigned i = 1; i < kMbarMaxPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && global_timer_ns() - t0 > kMbarTimeoutNs) break;
  }
  if (err) atomicOr(err, DEV_ERR_MBAR_TIMEOUT);
  return false;
}

// One TMA bulk copy global -> shared (16-byte aligned, size % 16 == 0);
// completion is signalled on `bar` as transaction bytes.
SPEC_DEV void tma_bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// The same copy with an L2 cache-policy hint (e.g. evict_first for weights
// streamed once per forward, so they do not push activations, partial sums
// and norm tables out of L2).
SPEC_DEV void tma_bulk_g2s_hint(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
SPEC_DEV uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// L2 prefetch of a contiguous range (no shared memory, no registers).
SPEC_DEV void tma_prefetch_l2(const void* gmem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes) : "memory");
}

// D = A(16x16, row) * B(16x8, col) + C, f16 inputs, f32 accumulate.
SPEC_DEV void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                      uint32_t b1, float c0, float c1, float c2, float c3) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

SPEC_DEV void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                       uint32_t b1, float c0, float c1, float c2, float c3) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

// ldmatrix x4 (non-transposed / transposed) from shared memory.
SPEC_DEV void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
SPEC_DEV void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

SPEC_DEV void cp_async16(void* smem, const void* gmem, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill when invalid
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n)
               : "memory");
}
SPEC_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
SPEC_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

SPEC_DEV uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  // (a & mask) | orv
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}
SPEC_DEV uint32_t lop3_or_and(uint32_t base, uint32_t b, uint32_t mask) {
  // base | (b & mask)
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xF8;\n" : "=r"(d) : "r"(base), "r"(b), "r"(mask));
  return d;
}

SPEC_DEV uint32_t pack_half2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

SPEC_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
SPEC_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace specb200
