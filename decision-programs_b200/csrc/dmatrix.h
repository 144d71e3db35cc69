// Training matrix: a dense fp32 device matrix (NaN = missing) plus owned
// labels, the first-pass prefix counts of the cut search (taken while the
// matrix is read for its validity check, or while it uploads), and the cached
// quantile cuts / uint8 bin matrix built at the first boosting round.
// XGDMatrixCreateFromCudaArrayInterface borrows a CUDA pointer that must stay
// valid while the DMatrix lives, as the reference uses it
// (native/class_native_training.cuh:49-53, native/class_study_oof.cu:532-534);
// XGDMatrixCreateFromDense copies a host matrix into device memory the
// DMatrix owns, in chunks that overlap the copy with the counting pass.
#pragma once
#include <memory>
#include <string>
#include <vector>

#include "comm.h"
#include "common.h"
#include "kernels.h"

namespace dp {

struct Quantized {
  std::vector<DevBuf<u8>> slabs;  // memory of the device buffers below
  int max_bin = 0;
  u64 bin_stride = 0;       // bytes per row of `bins` (multiple of 16)
  DevBuf<float> cut;        // [F][256]
  DevBuf<u16> nbins;        // [F]
  DevBuf<u8> has_missing;   // [F]
  DevBuf<u8> bins;          // [R][bin_stride]
  DevBuf<u8> bins_blk;      // [ceil(R/32)][F][32]: codes of one feature for 32 rows per sector
  std::vector<float> cut_h;
  std::vector<u16> nbins_h;
  std::vector<u8> has_missing_h;
  u64 rows_total = 0;       // over all ranks
  double host_ms_alloc = 0, host_ms_cuts = 0, host_ms_bins = 0;  // build phases (host clock)
};

class DMatrix {
 public:
  // Borrowed device matrix.
  DMatrix(const float* x, u64 rows, u32 cols, u64 stride, int device, bool has_mv, float mv);
  // Waits for the device, then hands the matrix's memory to SlabCache.
  ~DMatrix();
  DMatrix(const DMatrix&) = delete;
  DMatrix& operator=(const DMatrix&) = delete;
  // Host matrix copied to `device`.
  static std::unique_ptr<DMatrix> from_host(const float* x, u64 rows, u32 cols, u64 stride, int device, bool has_mv,
                                            float mv);

  void set_labels_device(const float* y, u64 n);
  void set_labels_host(const float* y, u64 n);

  // Cuts and bins for `max_bin` over all ranks of `comm` (built once).
  const Quantized& quantized(int max_bin, Comm* comm, cudaStream_t s);

  u64 rows() const { return rows_; }
  u32 cols() const { return cols_; }
  int device() const { return device_; }
  const float* labels() const { return labels_.get(); }
  bool has_labels() const { return labels_n_ == rows_; }

 private:
  DMatrix() = default;
  void check_bad(const u32* bad_dev);
  const float* x_ = nullptr;
  std::vector<DevBuf<u8>> slabs_;  // memory of owned_ and prefix_counts_
  DevBuf<float> owned_;        // host-sourced matrix
  DevBuf<u32> prefix_counts_;  // [cols][kPrefixBuckets] this rank's rows, then a flag word
  bool prefix_valid_ = false;  // counts present and not yet consumed by a cut search
  u64 rows_ = 0, stride_ = 0;
  u32 cols_ = 0;
  int device_ = 0;
  bool has_mv_ = false;
  float mv_ = 0.f;
  DevBuf<float> labels_;
  u64 labels_n_ = 0;
  std::unique_ptr<Quantized> q_;
};

}  // namespace dp
