#include "dmatrix.h"

#include "quantile.h"

namespace dp {

DMatrix::DMatrix(const float* x, u64 rows, u32 cols, u64 stride, int device, bool has_mv, float mv)
    : x_(x), rows_(rows), stride_(stride), cols_(cols), device_(device), has_mv_(has_mv), mv_(mv) {
  need(cols > 0, "DMatrix needs at least one column");
  need(stride >= cols, "DMatrix row stride is smaller than its column count");
  DeviceGuard g(device_);
  if (rows_ == 0) return;
  DevBuf<u32> bad(1);
  DP_CUDA(cudaMemset(bad.get(), 0, sizeof(u32)));
  launch_check_finite(x_, rows_, cols_, stride_, bad.get(), nullptr);
  u32 h = 0;
  DP_CUDA(cudaMemcpy(&h, bad.get(), sizeof h, cudaMemcpyDeviceToHost));
  need(h == 0, "Input data contains `inf` or a value too large, while `missing` is not set to `inf`");
}

void DMatrix::set_labels_device(const float* y, u64 n) {
  need(n == rows_, "label size differs from the number of rows");
  DeviceGuard g(device_);
  labels_.resize(n);
  if (n) DP_CUDA(cudaMemcpy(labels_.get(), y, n * sizeof(float), cudaMemcpyDefault));
  labels_n_ = n;
}

void DMatrix::set_labels_host(const float* y, u64 n) { set_labels_device(y, n); }

const Quantized& DMatrix::quantized(int max_bin, Comm* comm, cudaStream_t s) {
  if (q_ && q_->max_bin == max_bin) return *q_;
  DeviceGuard g(device_);
  auto q = std::make_unique<Quantized>();
  q->max_bin = max_bin;
  q->bin_stride = (u64(cols_) + 15) / 16 * 16;
  q->cut.resize(u64(cols_) * kMaxBins);
  q->nbins.resize(cols_);
  q->has_missing.resize(cols_);
  q->rows_total = comm ? comm->sum_host_u64(rows_, s) : rows_;
  CutsDevice cd{q->cut.get(), q->nbins.get(), q->has_missing.get()};
  compute_cuts(x_, rows_, cols_, stride_, max_bin, has_mv_, mv_, q->rows_total, comm, cd, s);
  q->bins.resize(std::max<u64>(rows_, 1) * q->bin_stride);
  launch_bin_matrix(x_, rows_, cols_, stride_, has_mv_, mv_, cd, q->bins.get(), q->bin_stride, s);
  q->cut_h.resize(q->cut.size());
  q->nbins_h.resize(cols_);
  q->has_missing_h.resize(cols_);
  DP_CUDA(cudaMemcpyAsync(q->cut_h.data(), q->cut.get(), q->cut.size() * sizeof(float), cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaMemcpyAsync(q->nbins_h.data(), q->nbins.get(), cols_ * sizeof(u16), cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaMemcpyAsync(q->has_missing_h.data(), q->has_missing.get(), cols_, cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaStreamSynchronize(s));
  q_ = std::move(q);
  return *q_;
}

}  // namespace dp
