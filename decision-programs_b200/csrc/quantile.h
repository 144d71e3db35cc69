// Quantile cuts (exact radix selection) and uint8 binning of a dense fp32 matrix.
#pragma once
#include "comm.h"
#include "kernels.h"

namespace dp {

// Cuts over the rows of every rank (comm == nullptr for one GPU); R_total is
// the row count over all ranks.  Synchronises `s` before returning.
void compute_cuts(const float* x, u64 R, u32 F, u64 stride, int max_bin, bool has_mv, float mv, u64 R_total,
                  Comm* comm, const CutsDevice& out, cudaStream_t s);

void launch_bin_matrix(const float* x, u64 R, u32 F, u64 stride, bool has_mv, float mv, const CutsDevice& cuts,
                       u8* bins, u64 bin_stride, cudaStream_t s);

}  // namespace dp
