// dp_probe_hist_atomics: the shared-memory update ceiling of the histogram
// kernel on this GPU, measured live.
//
// The histogram build is bound by its shared-memory atomics (two 32-bit adds
// per (row, feature) pair into the g and h planes), not by HBM: its bytes per
// pair are small.  This probe runs the histogram kernel's inner loop alone --
// the same 1024-thread block per SM, the same two [bin][32-feature] u32
// planes, the same rotated lane -> column mapping (32 distinct columns, hence
// 32 distinct banks, per warp step) -- over pseudo-random bin codes generated
// in registers, with no global-memory traffic.  Its pairs per second are the
// ceiling against which the histogram kernel's pairs per second are read.
// The update itself is the kernels' add_row (hist_update.cuh).
#include "../../include/dp_gbdt.h"
#include "hist_update.cuh"
#include "kernels.h"

namespace dp {
namespace {

constexpr int kProbeThreads = 1024;
constexpr int kProbeCells = 256 * kHistFeatureTile;

__device__ __forceinline__ u32 xorshift32(u32 x) {
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  return x;
}

__global__ void __launch_bounds__(kProbeThreads) k_probe_atomics(u32 steps, u32* sink) {
  extern __shared__ __align__(16) unsigned char smem[];
  u32* planes = reinterpret_cast<u32*>(smem + plane_pad(smem));
  for (int i = threadIdx.x; i < 2 * kProbeCells; i += kProbeThreads) planes[i] = 0u;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const u32 s = u32(lane) >> 1, h16 = u32(lane & 1) * 16u;
  const LaneCols cols = lane_cols(smem_addr(planes), h16, s);
  u32 x = 0x9e3779b9u ^ (threadIdx.x * 0x85ebca6bu) ^ (blockIdx.x * 0xc2b2ae35u);
  x = x ? x : 1u;
  const u32 gq = 3u + threadIdx.x, hq = 5u;
  for (u32 step = 0; step < steps; ++step) {
    uint4 v;
    x = xorshift32(x);
    v.x = x;
    x = xorshift32(x);
    v.y = x;
    x = xorshift32(x);
    v.z = x;
    x = xorshift32(x);
    v.w = x;
    add_row<u32(kProbeCells) * 4u>(v, gq, hq, cols);
  }
  __syncthreads();
  u32 acc = 0;
  for (int i = threadIdx.x; i < 2 * kProbeCells; i += kProbeThreads) acc += planes[i];
  if (acc == 0x12345678u) sink[0] = acc;  // keeps the updates observable
}

}  // namespace
}  // namespace dp

extern "C" int dp_probe_hist_atomics(uint32_t steps, double* pairs_per_second, void* stream) {
  try {
    dp::need(steps > 0 && pairs_per_second != nullptr, "dp_probe_hist_atomics: steps > 0 and an output required");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int dev = 0, sms = 0;
    dp::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    dp::cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
    // 64 KB of planes; the request is raised above half an SM's shared
    // memory so that the grid places exactly one block on each SM
    const int smem = 120 * 1024;
    dp::cuda_check(cudaFuncSetAttribute(dp::k_probe_atomics, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                   "probe shared memory");
    dp::DevBuf<dp::u32> sink(1);
    cudaEvent_t e0, e1;
    dp::cuda_check(cudaEventCreate(&e0), "event");
    dp::cuda_check(cudaEventCreate(&e1), "event");
    // warm-up, then the timed launch; one block per SM, as the histogram kernel
    dp::k_probe_atomics<<<sms, dp::kProbeThreads, smem, s>>>(steps / 8 + 1, sink.get());
    dp::cuda_check(cudaEventRecord(e0, s), "event");
    dp::k_probe_atomics<<<sms, dp::kProbeThreads, smem, s>>>(steps, sink.get());
    dp::cuda_check(cudaEventRecord(e1, s), "event");
    dp::cuda_check(cudaEventSynchronize(e1), "probe");
    float ms = 0.f;
    dp::cuda_check(cudaEventElapsedTime(&ms, e0, e1), "event time");
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    dp::count_launch(2);
    // every thread updates 16 (row, feature) pairs per step
    const double pairs = double(sms) * dp::kProbeThreads * 16.0 * double(steps);
    *pairs_per_second = ms > 0.f ? pairs / (double(ms) * 1e-3) : 0.0;
    return 0;
  } catch (const std::exception& e) {
    dp::set_last_error(e.what());
    return -1;
  }
}
