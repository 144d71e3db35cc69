// The shared-memory update of the histogram kernels (k_hist.cu) and of the
// probe that measures its ceiling (k_probe.cu): one row's 16 bin codes added
// as (g, h) into two u32 planes with 32-bit shared atomics.
#pragma once
#include "kernels.h"

namespace dp {

__device__ __forceinline__ u32 smem_addr(const void* p) {
  return static_cast<u32>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// The update of one row's 16 codes.
//
// The u32 planes hold 32 feature columns per 128-byte bin row: the g cell of
// (bin b, column c) sits at byte  R + b * 128 + 4 c  of the shared window and
// its h cell HOFF bytes above it (R: the lane's plane region, 128-byte
// aligned).  A lane holds 16 codes, columns c0 .. c0 + 15, and a lane key x
// in [0, 16) that differs between the lanes of a warp sharing c0: atomic
// step j takes column c0 + (j XOR x), so the 32 lanes of a step address 32
// distinct columns, hence 32 distinct banks, whatever the bins.
//
// Step j = 4k + t uses byte t ^ (x & 3) of word k ^ (x >> 2).  The words are
// permuted once per row (eight selects); one byte permutation per word with
// a per-lane selector then places the codes of steps 4k and 4k + 2 (or
// 4k + 1 and 4k + 3) in the two 16-bit halves of a register, zero-extended;
// one multiply-add turns both into  low16(R) + b * 128 + 4 col  at once
// (below 2^16, so no carry crosses the halves); and one permutation per code
// moves its half into the low 16 bits under the region's high half.  The
// column constant of word k is the one of word 0 with bits 4-5 flipped by k
// (R 128-byte aligned keeps the fields of the sum disjoint).  About three
// integer instructions per (row, feature) pair besides the two atomics, and
// five registers of lane constants.
struct LaneCols {
  u32 sel_e, sel_o;  // byte selectors: codes of steps 4k, 4k+2 / 4k+1, 4k+3
  u32 ce, co;        // packed addresses of those steps for bin 0, word 0
  u32 hi;            // the region's high 16 bits
  bool swap2, swap1; // word permutation k -> k ^ (x >> 2)
};

// region: shared-window address of the lane's g plane (128-byte aligned);
// c0: the lane's first column; x: the lane key
__device__ __forceinline__ LaneCols lane_cols(u32 region, u32 c0, u32 x) {
  LaneCols L;
  const u32 xl = x & 3u, xh = x >> 2;
  L.sel_e = xl | 0x40u | ((2u ^ xl) << 8) | 0x4000u;
  L.sel_o = (1u ^ xl) | 0x40u | ((3u ^ xl) << 8) | 0x4000u;
  const u32 lo = (region & 0xffffu) + 4u * c0 + 16u * xh;
  L.ce = (lo + 4u * xl) | ((lo + 4u * (2u ^ xl)) << 16);
  L.co = (lo + 4u * (1u ^ xl)) | ((lo + 4u * (3u ^ xl)) << 16);
  L.hi = region & 0xffff0000u;
  L.swap2 = (xh & 2u) != 0;
  L.swap1 = (xh & 1u) != 0;
  return L;
}

template <u32 HOFF>
__device__ __forceinline__ void red_pair(u32 addr, u32 g, u32 h) {
  asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(addr), "r"(g) : "memory");
  asm volatile("red.shared.add.u32 [%0+%2], %1;" ::"r"(addr), "r"(h), "n"(HOFF) : "memory");
}

// One row's 16 codes into the g and h planes.  With CLAMP (planes of
// MB + 1 bin rows), codes above MB go to row MB, which is never read.
template <u32 HOFF, u32 CLAMP = 0>
__device__ __forceinline__ void add_row(uint4 v, u32 gq, u32 hq, const LaneCols& L) {
  const u32 u0 = L.swap2 ? v.z : v.x, u1 = L.swap2 ? v.w : v.y;
  const u32 u2 = L.swap2 ? v.x : v.z, u3 = L.swap2 ? v.y : v.w;
  const u32 w[4] = {L.swap1 ? u1 : u0, L.swap1 ? u0 : u1, L.swap1 ? u3 : u2, L.swap1 ? u2 : u3};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    u32 xe = __byte_perm(w[k], 0u, L.sel_e);
    u32 xo = __byte_perm(w[k], 0u, L.sel_o);
    if (CLAMP) {
      xe = __vminu2(xe, CLAMP * 0x10001u);
      xo = __vminu2(xo, CLAMP * 0x10001u);
    }
    const u32 flip = 16u * u32(k) * 0x10001u;
    const u32 ae = xe * 128u + (L.ce ^ flip);
    const u32 ao = xo * 128u + (L.co ^ flip);
    red_pair<HOFF>(__byte_perm(ae, L.hi, 0x7610u), gq, hq);
    red_pair<HOFF>(__byte_perm(ao, L.hi, 0x7610u), gq, hq);
    red_pair<HOFF>(__byte_perm(ae, L.hi, 0x7632u), gq, hq);
    red_pair<HOFF>(__byte_perm(ao, L.hi, 0x7632u), gq, hq);
  }
}

// Bytes added in front of planes placed in dynamic shared memory so that
// they start on a 128-byte boundary.
constexpr u32 kPlaneAlignPad = 128;
__device__ __forceinline__ u32 plane_pad(const void* dyn_smem) {
  return (128u - (smem_addr(dyn_smem) & 127u)) & 127u;
}

}  // namespace dp
