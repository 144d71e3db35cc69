// Quantile cuts (exact radix selection) and uint8 binning of a dense fp32 matrix.
#pragma once
#include "comm.h"
#include "kernels.h"

namespace dp {

constexpr u64 kPrefixBuckets = 65536;  // 16-bit key prefixes per feature

// First pass of the cut search over rows [0, R) of x: per (feature, 16-bit
// key prefix) counts of the non-missing values are added into
// cnt[F][kPrefixBuckets]; an infinite value that is not the missing value
// sets bad[0] (bad may be null).  Rows may arrive in several calls.
void launch_prefix_counts(const float* x, u64 R, u32 F, u64 stride, bool has_mv, float mv, u32* cnt, u32* bad,
                          cudaStream_t s);

// Cuts over the rows of every rank (comm == nullptr for one GPU); R_total is
// the row count over all ranks.  prefix_counts, when given, holds this rank's
// first-pass counts (launch_prefix_counts, F * kPrefixBuckets words): the pass
// is not repeated and the buffer is used as the search's scratch, so its
// contents are lost.  Synchronises `s` before returning.
void compute_cuts(const float* x, u64 R, u32 F, u64 stride, int max_bin, bool has_mv, float mv, u64 R_total,
                  Comm* comm, const CutsDevice& out, cudaStream_t s, u32* prefix_counts = nullptr);

// bins[r * bin_stride + f] (row-major, bin_stride >= F, padding zeroed) and,
// when bins_blk is set, the same codes in the 32-row blocked layout
// bins_blk[(r / 32) * 32 * F + f * 32 + r % 32] (ceil(R / 32) * 32 * F bytes),
// where the codes of one feature for 32 consecutive rows share a sector.
void launch_bin_matrix(const float* x, u64 R, u32 F, u64 stride, bool has_mv, float mv, const CutsDevice& cuts,
                       u8* bins, u64 bin_stride, cudaStream_t s, u8* bins_blk = nullptr);

}  // namespace dp
