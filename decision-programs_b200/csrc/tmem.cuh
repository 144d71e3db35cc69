// Tensor memory (TMEM) of a CTA on sm_100a, used as plain storage: the
// histogram kernels keep their int64 window sums there (no MMA is issued).
//
// TMEM is 128 lanes x 512 columns of 32 bits per SM.  A CTA allocates a
// power-of-two number of columns (32..512) with one warp, and frees them with
// the same warp before it exits.  Warp w of the CTA reaches only lanes
// 32 (w % 4) .. 32 (w % 4) + 31; with the 32x32b shapes its thread t reads
// or writes lane 32 (w % 4) + t, N consecutive columns into N registers.
// Loads and stores are asynchronous: tmem_wait_ld() before the loaded
// registers are used, tmem_wait_st() before the stored columns are read
// again or the CTA synchronises on them.
#pragma once
#include "kernels.h"

namespace dp {

// One warp: allocates `ncols` columns, writes their base address to
// *dst (shared memory), and gives up the CTA's right to allocate more.
__device__ __forceinline__ void tmem_alloc(u32* dst, u32 ncols) {
  const u32 d = static_cast<u32>(__cvta_generic_to_shared(dst));
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(d), "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// One warp (the allocating one): frees the columns at `taddr`.
__device__ __forceinline__ void tmem_dealloc(u32 taddr, u32 ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Orders TMEM accesses around a CTA barrier: before_sync by every thread that
// accessed TMEM before the barrier, after_sync by every thread that accesses
// it after.
__device__ __forceinline__ void tmem_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 consecutive columns of this thread's lane, from / to column address
// `taddr` (lane field = the warp's first lane).
__device__ __forceinline__ void tmem_ld16(u32 taddr, u32 (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(u32 taddr, const u32 (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 4 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_ld4(u32 taddr, u32 (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
}

__device__ __forceinline__ void tmem_st4(u32 taddr, const u32 (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// TMEM address of (lane, column) relative to an allocation's base.
__device__ __forceinline__ u32 tmem_at(u32 base, u32 lane, u32 col) { return base + (lane << 16) + col; }

}  // namespace dp
