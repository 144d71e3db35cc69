// dp_hist_build_noalloc: the histogram build of dp_hist_build for callers that
// cannot allocate device memory.
//
// dp_hist_build cudaMallocs its task list and a few small descriptors on every
// call.  Some callers cannot do that: a process that reserves the device's
// memory up front in its own pool (an extra cudaMalloc then fails, or splits
// the pool), or a caller on a latency-critical path where cudaMalloc/cudaFree
// and the device-wide synchronisation that cudaFree implies are not allowed.
// This entry point keeps the same scratch in one fixed-size file-scope
// __device__ array instead; every GPU that loads the library holds that array
// (about 1 MiB) until the process exits.  Nothing is allocated per call: the
// task list is staged through a small stack buffer and copied into the array.
#include <vector>

#include "../../include/dp_gbdt.h"
#include "kernels.h"

namespace {

// Capacity of the scratch task list.  One task covers a row range of one
// segment and one 32-feature tile; a call needs at least
// (segments with rows) x ceil(features / 32) tasks.
constexpr uint32_t kNoAllocMaxTasks = 32768;

struct NoAllocScratch {
  dp::HistTask tasks[kNoAllocMaxTasks];
  dp::TreeArrays trees[1];
  dp::Scales scales[1];
  dp::u32 counter;  // task queue of the kernel; zeroed by the launcher on every call
};

static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

// Device address of the scratch array on the current device.  The host
// symbol is only a stand-in for it, so the address is looked up on every call
// with the call's device current.  The lookup costs microseconds, nothing next
// to the call's own stream synchronisation, and a cached address could go
// stale: after cudaDeviceReset the library's device code is loaded anew and
// the array may sit elsewhere.  On a device's first call the lookup also loads
// that device code.
NoAllocScratch* scratch_here() {
  void* p = nullptr;
  dp::cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-allocation scratch)");
  return static_cast<NoAllocScratch*>(p);
}

}  // namespace

extern "C" int dp_hist_build_noalloc(const uint8_t* bins, uint64_t bin_stride, uint32_t features, int32_t num_bins,
                                     const float* gh, const uint32_t* ridx, const int64_t* seg_begin,
                                     const int64_t* seg_end, int32_t nseg, float sg, float sh, int64_t* hist,
                                     void* stream) {
  try {
    dp::need(nseg >= 0 && (nseg == 0 || (seg_begin && seg_end)), "invalid segments");
    dp::need(num_bins >= 1 && num_bins <= 256, "num_bins must be in [1, 256]");
    dp::need(bin_stride % 16 == 0 && bin_stride >= features,
             "bin_stride must cover the features and be a multiple of 16");
    const dp::u32 ftiles = (features + dp::kHistFeatureTile - 1) / dp::kHistFeatureTile;
    dp::u64 total = 0, min_tasks = 0, filled = 0;
    for (int32_t i = 0; i < nseg; ++i) {
      dp::need(seg_begin[i] >= 0 && seg_end[i] >= seg_begin[i] && seg_end[i] < (int64_t(1) << 31),
               "invalid segment bounds (positions must be below 2^31)");
      total += dp::u64(seg_end[i] - seg_begin[i]);
      min_tasks += seg_end[i] > seg_begin[i] ? ftiles : 0;
      filled += seg_end[i] > seg_begin[i] ? 1 : 0;
    }
    dp::need(nseg == 0 || hist != nullptr, "hist pointer is null");
    dp::need(total == 0 || (bins != nullptr && gh != nullptr && ridx != nullptr), "bins, gh or ridx pointer is null");
    const int64_t chunk = int64_t(dp::hist_chunk_rows(total * ftiles, dp::u64(nseg), bin_stride % 128 == 0));
    dp::u64 ntasks = 0;
    for (int32_t i = 0; i < nseg; ++i) {
      const int64_t n = seg_end[i] - seg_begin[i];
      if (n > 0) ntasks += dp::u64(ftiles) * dp::u64((n + chunk - 1) / chunk);
    }
    if (ntasks > kNoAllocMaxTasks)
      dp::fail("dp_hist_build_noalloc: these segments need " + std::to_string(ntasks) +
               " histogram tasks (at least " + std::to_string(min_tasks) +
               " = non-empty segments x feature tiles of 32), above its fixed capacity of " +
               std::to_string(kNoAllocMaxTasks) + "; use dp_hist_build for this size");
    NoAllocScratch* scratch = scratch_here();
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    const dp::TreeArrays th{const_cast<uint32_t*>(ridx), reinterpret_cast<float2*>(const_cast<float*>(gh))};
    const dp::Scales sc{sg, sh};
    dp::cuda_check(cudaMemcpyAsync(scratch->trees, &th, sizeof th, cudaMemcpyHostToDevice, s), "stage trees");
    dp::cuda_check(cudaMemcpyAsync(scratch->scales, &sc, sizeof sc, cudaMemcpyHostToDevice, s), "stage scales");
    // Tasks go through a stack buffer: a copy from pageable memory has read
    // its source when cudaMemcpyAsync returns, so the buffer can be refilled.
    constexpr int kBatch = 256;
    dp::HistTask batch[kBatch];
    int fill = 0;
    dp::u64 written = 0;
    auto flush = [&]() {
      if (!fill) return;
      dp::cuda_check(cudaMemcpyAsync(scratch->tasks + written, batch, fill * sizeof(dp::HistTask),
                                     cudaMemcpyHostToDevice, s),
                     "stage tasks");
      written += dp::u64(fill);
      fill = 0;
    };
    // Queue order: piece index, then segment, then feature tile, as the
    // allocating entry point queues them: the p-th pieces of all segments of a
    // node-grouped row list cover about the same rows, so blocks running at
    // one time read neighbouring rows of the bin matrix.
    std::vector<int64_t> piece(size_t(nseg), 0);
    int64_t max_pieces = 0;
    for (int32_t i = 0; i < nseg; ++i) {
      const int64_t n = seg_end[i] - seg_begin[i];
      if (n <= 0) continue;
      const int64_t pieces = (n + chunk - 1) / chunk;
      piece[i] = (n + pieces - 1) / pieces;
      max_pieces = std::max(max_pieces, pieces);
    }
    for (int64_t q = 0; q < max_pieces; ++q)
      for (int32_t i = 0; i < nseg; ++i) {
        if (!piece[i]) continue;
        const int64_t b = seg_begin[i] + q * piece[i];
        if (b >= seg_end[i]) continue;
        for (dp::u32 ft = 0; ft < ftiles; ++ft) {
          batch[fill++] = dp::HistTask{dp::u32(i), ft * dp::kHistFeatureTile, 0, 0, b,
                                       std::min<int64_t>(seg_end[i], b + piece[i])};
          if (fill == kBatch) flush();
        }
      }
    flush();
    const dp::u64 slot = dp::u64(features) * dp::kMaxBins * 2;
    if (nseg) dp::cuda_check(cudaMemsetAsync(hist, 0, dp::u64(nseg) * slot * sizeof(int64_t), s), "zero histograms");
    // the same kernel as dp_hist_build for these segments
    dp::launch_histograms(bins, bin_stride, features, dp::hist_kernel_bins(num_bins, filled), false,
                          scratch->trees, scratch->scales, scratch->tasks, dp::u32(written), &scratch->counter, hist,
                          s);
    dp::cuda_check(cudaStreamSynchronize(s), "histograms");
    return 0;
  } catch (const std::exception& e) {
    dp::set_last_error(e.what());  // read back with XGBGetLastError()
    return -1;
  }
}
