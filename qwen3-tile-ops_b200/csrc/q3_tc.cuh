// tcgen05 / mbarrier / TMA building blocks shared by the tensor-core kernels
// (the w8a8 GEMMs and the decode attention).  sm_100a only.
//
// Every mbarrier wait here is bounded: it gives up after about one second (or
// as soon as another thread of the CTA raised the abort word), so that a kernel
// can record an error, drain what it has in flight and return.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace q3 {
namespace tcx {

__device__ __forceinline__ uint32_t su32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long *b, unsigned c) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(c) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long *b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait for the completion of the phase with parity `par`: gives up
// (false) when *abort is set or after about one second.  `sleep_ns` > 0 lets
// each try_wait suspend the thread for up to that long while the phase is
// incomplete (it resumes when the phase completes), so warps that mostly wait
// take fewer issue slots from the others.
__device__ __forceinline__ bool mbar_wait(unsigned long long *b, uint32_t par, const int *abort,
                                          uint32_t sleep_ns = 0) {
  const uint32_t a = su32(b);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    if (sleep_ns)
      asm volatile(
          "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
          " selp.u32 %0, 1, 0, p;\n}"
          : "=r"(ok)
          : "r"(a), "r"(par), "r"(sleep_ns)
          : "memory");
    else
      asm volatile(
          "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
          " selp.u32 %0, 1, 0, p;\n}"
          : "=r"(ok)
          : "r"(a), "r"(par)
          : "memory");
    if (ok) return true;
    if ((it & 127) == 0) {
      if (abort && *reinterpret_cast<const volatile int *>(abort)) return false;
      const uint64_t t = gtime();
      if (t0 == 0) t0 = t;
      else if (t - t0 > 1000000000ull) return false;
    }
  }
}
__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *m, int x, int y,
                                       unsigned long long *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}

// Shared-memory matrix descriptors (tcgen05 format: start >> 4 in bits 0-13,
// leading byte offset >> 4 in 16-29, stride byte offset >> 4 in 32-45, version
// 1 in bit 46, layout type in 61-63).
//
// 128-byte swizzle: 8-row atoms of 128-byte rows (16-byte chunk i of row r
// stored at chunk i ^ (r & 7)), atoms `sbo` bytes apart.  Read K-major, a row
// is one M/N index and holds 128 bytes of K.  Read MN-major, a row is one K
// index and holds 128 consecutive M/N indices; with M or N = 128 there is a
// single atom across, so the leading offset is not used either way.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t sbo = 1024) {
  uint64_t d = (saddr & 0x3FFFFu) >> 4;
  d |= 1ull << 16;                                   // leading byte offset (unused)
  d |= static_cast<uint64_t>(sbo >> 4) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;                                   // 128-byte swizzle
  return d;
}
// K-major, no swizzle: core matrices of 8 rows x 16 bytes (128 contiguous
// bytes); the next 16 bytes of K are `lbo` bytes on, the next 8 rows `sbo`.
__device__ __forceinline__ uint64_t sdesc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (saddr & 0x3FFFFu) >> 4;
  d |= static_cast<uint64_t>(lbo >> 4) << 16;
  d |= static_cast<uint64_t>(sbo >> 4) << 32;
  d |= 1ull << 46;
  return d;                                          // layout type 0: no swizzle
}
// instruction descriptor, kind::i8: s32 accumulate, s8 x s8, M = 128, N = n;
// a_mn / b_mn: that operand is MN-major (otherwise K-major)
__host__ __device__ constexpr uint32_t idesc_i8(int n, bool a_mn = false, bool b_mn = false) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (a_mn ? (1u << 15) : 0u) | (b_mn ? (1u << 16) : 0u) |
         (static_cast<uint32_t>(n >> 3) << 17) | ((128u >> 4) << 24);
}
__device__ __forceinline__ void tma_3d(void *dst, const CUtensorMap *m, int x, int y, int z,
                                       unsigned long long *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void mma_i8(uint32_t dt, uint64_t ad, uint64_t bd, uint32_t id,
                                       uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(dt),
      "l"(ad), "l"(bd), "r"(id), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(unsigned long long *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes of this thread -> visible to the tensor cores
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
template <int COLS>
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem) {   // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   su32(dst_smem)),
               "n"(COLS)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
template <int COLS>
__device__ __forceinline__ void tmem_dealloc(uint32_t base) {      // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "n"(COLS)
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15},"
      " [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld2(uint32_t taddr, int &v0, int &v1) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];"
               : "=r"(v0), "=r"(v1)
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 16 columns of this warp's 32 TMEM lanes set to `v`
__device__ __forceinline__ void tmem_st16(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
          taddr),
      "r"(v)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

}  // namespace tcx
}  // namespace q3
