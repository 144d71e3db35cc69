#include "dmatrix.h"

#include <algorithm>
#include <chrono>

#include "quantile.h"

namespace dp {

namespace {
constexpr const char* kInfMessage = "Input data contains `inf` or a value too large, while `missing` is not set to `inf`";
}

DMatrix::DMatrix(const float* x, u64 rows, u32 cols, u64 stride, int device, bool has_mv, float mv)
    : x_(x), rows_(rows), stride_(stride), cols_(cols), device_(device), has_mv_(has_mv), mv_(mv) {
  need(cols > 0, "DMatrix needs at least one column");
  need(stride >= cols, "DMatrix row stride is smaller than its column count");
  DeviceGuard g(device_);
  if (rows_ == 0) return;
  // the counts, then one flag word for infinite values
  SlabPlan plan;
  plan.want(prefix_counts_, u64(cols_) * kPrefixBuckets + 1);
  plan.commit(slabs_, device_);
  u32* bad = prefix_counts_.get() + u64(cols_) * kPrefixBuckets;
  DP_CUDA(cudaMemset(prefix_counts_.get(), 0, prefix_counts_.size() * sizeof(u32)));
  launch_prefix_counts(x_, rows_, cols_, stride_, has_mv_, mv_, prefix_counts_.get(), bad, nullptr);
  check_bad(bad);
  prefix_valid_ = true;
}

std::unique_ptr<DMatrix> DMatrix::from_host(const float* x, u64 rows, u32 cols, u64 stride, int device, bool has_mv,
                                            float mv) {
  need(cols > 0, "DMatrix needs at least one column");
  need(stride >= cols, "DMatrix row stride is smaller than its column count");
  std::unique_ptr<DMatrix> d(new DMatrix());
  d->rows_ = rows;
  d->cols_ = cols;
  d->stride_ = cols;
  d->device_ = device;
  d->has_mv_ = has_mv;
  d->mv_ = mv;
  DeviceGuard g(device);
  {
    SlabPlan plan;
    plan.want(d->owned_, std::max<u64>(rows, 1) * cols);
    if (rows > 0) plan.want(d->prefix_counts_, u64(cols) * kPrefixBuckets + 1);
    plan.commit(d->slabs_, device);
  }
  d->x_ = d->owned_.get();
  if (rows == 0) return d;
  u32* bad = d->prefix_counts_.get() + u64(cols) * kPrefixBuckets;
  cudaStream_t copy = nullptr, count = nullptr;
  cudaEvent_t landed = nullptr;
  DP_CUDA(cudaStreamCreateWithFlags(&copy, cudaStreamNonBlocking));
  DP_CUDA(cudaStreamCreateWithFlags(&count, cudaStreamNonBlocking));
  DP_CUDA(cudaEventCreateWithFlags(&landed, cudaEventDisableTiming));
  try {
    DP_CUDA(cudaMemsetAsync(d->prefix_counts_.get(), 0, d->prefix_counts_.size() * sizeof(u32), count));
    // about 32 MB per chunk: the counting pass of chunk i runs while chunk
    // i + 1 crosses the host link
    const u64 chunk = std::max<u64>(1, (u64(32) << 20) / (u64(cols) * sizeof(float)));
    for (u64 r0 = 0; r0 < rows; r0 += chunk) {
      const u64 n = std::min<u64>(chunk, rows - r0);
      float* dst = d->owned_.get() + r0 * cols;
      const float* src = x + r0 * stride;
      if (stride == cols)
        DP_CUDA(cudaMemcpyAsync(dst, src, n * cols * sizeof(float), cudaMemcpyHostToDevice, copy));
      else
        DP_CUDA(cudaMemcpy2DAsync(dst, cols * sizeof(float), src, stride * sizeof(float), cols * sizeof(float), n,
                                  cudaMemcpyHostToDevice, copy));
      DP_CUDA(cudaEventRecord(landed, copy));
      DP_CUDA(cudaStreamWaitEvent(count, landed, 0));
      launch_prefix_counts(dst, n, cols, cols, has_mv, mv, d->prefix_counts_.get(), bad, count);
    }
    DP_CUDA(cudaStreamSynchronize(copy));
    DP_CUDA(cudaStreamSynchronize(count));
  } catch (...) {
    cudaStreamSynchronize(copy);
    cudaStreamSynchronize(count);
    cudaEventDestroy(landed);
    cudaStreamDestroy(copy);
    cudaStreamDestroy(count);
    throw;
  }
  cudaEventDestroy(landed);
  cudaStreamDestroy(copy);
  cudaStreamDestroy(count);
  d->check_bad(bad);
  d->prefix_valid_ = true;
  return d;
}

DMatrix::~DMatrix() {
  if (slabs_.empty() && !q_) return;
  DeviceGuard g(device_);
  // what cudaFree would wait for: no kernel may still read the memory when a
  // later matrix or engine is given it
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    return;  // the device is in an error state: free normally
  }
  for (auto& slab : slabs_) SlabCache::give(device_, std::move(slab));
  if (q_)
    for (auto& slab : q_->slabs) SlabCache::give(device_, std::move(slab));
}

void DMatrix::check_bad(const u32* bad_dev) {
  u32 h = 0;
  DP_CUDA(cudaMemcpy(&h, bad_dev, sizeof h, cudaMemcpyDeviceToHost));
  need(h == 0, kInfMessage);
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
  NvtxRange nv("dp_gbdt: cuts and bins");
  if (q_ && q_->max_bin == max_bin) return *q_;
  DeviceGuard g(device_);
  auto q = std::make_unique<Quantized>();
  q->max_bin = max_bin;
  q->bin_stride = (u64(cols_) + 15) / 16 * 16;
  SlabPlan plan;
  plan.want(q->cut, u64(cols_) * kMaxBins);
  plan.want(q->nbins, cols_);
  plan.want(q->has_missing, cols_);
  plan.want(q->bins, std::max<u64>(rows_, 1) * q->bin_stride);
  plan.want(q->bins_blk, std::max<u64>((rows_ + 31) / 32, 1) * 32 * cols_);
  auto t0 = std::chrono::steady_clock::now();
  plan.commit(q->slabs, device_);
  const double ms_alloc = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  q->rows_total = comm ? comm->sum_host_u64(rows_, s) : rows_;
  CutsDevice cd{q->cut.get(), q->nbins.get(), q->has_missing.get()};
  // the first-pass counts taken at construction are consumed by the search
  compute_cuts(x_, rows_, cols_, stride_, max_bin, has_mv_, mv_, q->rows_total, comm, cd, s,
               prefix_valid_ ? prefix_counts_.get() : nullptr);
  prefix_valid_ = false;
  const double ms_cuts = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  launch_bin_matrix(x_, rows_, cols_, stride_, has_mv_, mv_, cd, q->bins.get(), q->bin_stride, s, q->bins_blk.get());
  q->cut_h.resize(q->cut.size());
  q->nbins_h.resize(cols_);
  q->has_missing_h.resize(cols_);
  DP_CUDA(cudaMemcpyAsync(q->cut_h.data(), q->cut.get(), q->cut.size() * sizeof(float), cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaMemcpyAsync(q->nbins_h.data(), q->nbins.get(), cols_ * sizeof(u16), cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaMemcpyAsync(q->has_missing_h.data(), q->has_missing.get(), cols_, cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaStreamSynchronize(s));
  q->host_ms_alloc = ms_alloc;
  q->host_ms_cuts = ms_cuts - ms_alloc;
  q->host_ms_bins = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count() - ms_cuts;
  q_ = std::move(q);
  return *q_;
}

}  // namespace dp
