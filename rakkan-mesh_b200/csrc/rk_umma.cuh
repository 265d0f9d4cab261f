// rk_umma.cuh — sm_100a building blocks as inline PTX: mbarriers, 1-D bulk
// and 2-D TMA tile loads (no multicast), shared-memory matrix descriptors,
// and the tcgen05 MMA / TMEM instructions.
#pragma once
#include <cstdint>
#include <cuda.h>

#include "rk_common.cuh"

namespace rk {
namespace umma {

RK_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

RK_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

RK_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

RK_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple
// of 16), counted in bytes on `bar`; no multicast.
RK_DEV void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

RK_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of the barrier for at most ~1 s of wall time;
// false when it gave up.
RK_DEV bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > 1000000000ull) return false;
  }
}

// Brings bytes of global memory into L2 without occupying the SM (16-byte
// aligned address, size a multiple of 16).
RK_DEV void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

RK_DEV void prefetch_tmap(const CUtensorMap *m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// One 2-D tile of a tensor map into shared memory; completion is counted in
// bytes on `bar`. x is the innermost coordinate (elements).
RK_DEV void tma_load_2d(uint32_t dst, const CUtensorMap *m, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor (sm_100 format) of a tile stored with the
// 128-byte swizzle, which is what TMA's CU_TENSOR_MAP_SWIZZLE_128B writes
// when the tile's rows are 128 bytes and its base is 1024-byte aligned:
//   bits  0-13  start address >> 4
//   bits 16-29  leading-dimension byte offset >> 4
//   bits 32-45  stride-dimension byte offset >> 4
//   bits 46-47  descriptor version (1 on sm_100)
//   bits 61-63  layout (2 = 128-byte swizzle)
// K-major operand: rows are M (or N) indices, 128 bytes of K each; groups of
// 8 rows lie 1024 bytes apart (SBO); LBO is unused. MN-major operand: rows
// are K indices, 128 bytes of M each; groups of 8 K-rows lie 1024 bytes
// apart (SBO); LBO would step to the next 128 M-bytes, unused for M = 128.
RK_DEV uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;            // LBO (unused): 16 bytes
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO: 1024 bytes
  d |= (uint64_t)1 << 46;            // version
  d |= (uint64_t)2 << 61;            // 128-byte swizzle
  return d;
}

// Instruction descriptor of tcgen05.mma kind::i8: signed int8 A and B,
// int32 accumulator, M×N tile, A K-major (a_mn = 0) or MN-major (a_mn = 1),
// B K-major.
RK_HD constexpr uint32_t idesc_i8(int M, int N, int a_mn) {
  return (2u << 4)                  // accumulator format: s32
         | (1u << 7)                // A: signed 8-bit
         | (1u << 10)               // B: signed 8-bit
         | ((uint32_t)a_mn << 15)   // A major
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D(tmem) (+)= A(smem) · B(smem)ᵀ, issued by one thread.
RK_DEV void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued has completed.
RK_DEV void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// TMEM allocation by one whole warp; the base address goes to *slot.
RK_DEV void tmem_alloc(uint32_t slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

RK_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

RK_DEV void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
RK_DEV void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Eight consecutive 32-bit TMEM columns of lane (warp's quarter + lane id).
RK_DEV void tmem_ld8(uint32_t taddr, int32_t v[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
      : "r"(taddr));
}

RK_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace umma
}  // namespace rk
