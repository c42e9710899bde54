// tcgen05.cuh -- thin wrappers over the sm_100a tensor-core (tcgen05) and
// tensor-memory instructions used by the INT8 contraction kernel.
//
// Shared-memory operand descriptors follow the canonical K-major layout with
// 128-byte swizzle (what a TMA tiled load with CU_TENSOR_MAP_SWIZZLE_128B
// writes): 8-row x 128-byte atoms, 16-byte chunk c of row r stored at chunk
// c ^ (r & 7), atoms 1024 bytes apart along M/N.  Atom bases must be
// 1024-byte aligned; a K step inside the atom advances the start address.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "tma.cuh"

namespace qasr {

// Descriptor of a K-major SW128 operand starting at shared address `saddr`.
QASR_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address (16-byte units)
  d |= (uint64_t)1 << 16;                    // leading byte offset: unused for swizzled K-major
  d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset: next 8-row atom
  d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                    // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor: kind::i8, A and B signed 8-bit, K-major, S32
// accumulator, M x N tile.
constexpr uint32_t umma_idesc_s8(int M, int N) {
  return (2u << 4)                  // D format: S32
         | (1u << 7) | (1u << 10)  // A, B: signed 8-bit
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
QASR_DEV void umma_s8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
QASR_DEV void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

QASR_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
QASR_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole warp: allocate `ncols` TMEM columns (power of two >= 32); the base
// address is written to *slot in shared memory.
QASR_DEV void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Whole warp (the allocating one).
QASR_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Whole warp: 32 consecutive 32-bit columns of this warp's 32 TMEM lanes
// (lane i of the warp reads TMEM lane (taddr >> 16) + i).
QASR_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2D tiled TMA load (no multicast) of box {x .. x+bx, y .. y+by} into dst.
QASR_DEV void tma_load_2d_u8(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Named barrier over `count` threads (a multiple of 32), id 1..15.
QASR_DEV void named_bar(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }

}  // namespace qasr

// ------------------------------------------------------------ clusters --
namespace qasr {

QASR_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
QASR_DEV uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
QASR_DEV uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// All threads of every CTA of the cluster (also a CTA-wide barrier).
QASR_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared::cluster address of `local` (a shared::cta address) in CTA `rank`.
QASR_DEV uint32_t cluster_map(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// Arrive (release at cluster scope) on an mbarrier of another CTA of the cluster.
QASR_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
QASR_DEV unsigned long long ld_cluster_u64(uint32_t cluster_addr) {
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(cluster_addr) : "memory");
  return v;
}
QASR_DEV void ld_cluster_u64x2(uint32_t cluster_addr, unsigned long long &a, unsigned long long &b) {
  asm volatile("ld.shared::cluster.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(cluster_addr) : "memory");
}
// Split cluster barrier, per thread (no warp convergence needed): every
// thread of the cluster arrives once, then waits before leaving.
QASR_DEV void cluster_arrive_all() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
QASR_DEV void cluster_wait_all() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
QASR_DEV bool mbar_try_wait_cluster(uint64_t *bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (remote arrivals); false on timeout.
QASR_DEV bool mbar_wait_cluster(uint64_t *bar, unsigned parity) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait_cluster(bar, parity))
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  return true;
}

}  // namespace qasr
