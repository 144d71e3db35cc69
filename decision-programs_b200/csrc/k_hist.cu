// Histogram build: for every task (node slot, 32-feature tile, <= kWindowRows
// rows of the node's position segment) accumulate the quantised (g, h) of each
// row into hist[slot][f][bin] (int64 pairs).
//
// Design (HBM- and shared-atomic-bound, no tensor cores):
//  * the tile histogram lives in shared memory as one 64-bit word per
//    (bin, feature): sum_g * 2^32 + sum_h.  Window bounds (|q_g| <= 2^17,
//    q_h <= 2^18, <= 8192 rows) keep sum_h < 2^32 and |sum_g| < 2^31, so a
//    single 64-bit shared atomic per (row, feature) is exact;
//  * a warp reads 4 rows x 32 features per step: lane (s, q) loads the 32-bit
//    word holding features 4q..4q+3 of row s.  In atomic step j the lane
//    updates feature 4q + ((j + s) & 3), whose column is ((j+s)&3)*8 + q, so
//    the 32 lanes of a step address 32 distinct columns: every 16-lane half
//    warp hits 16 distinct 8-byte bank pairs whatever the bins are;
//  * rows are gathered through the node's row-index segment; (g, h) is read
//    in position order (the partition kernel moves it with the row index);
//  * at the end of the task the tile is drained with 64-bit global atomics
//    (integer, so the result does not depend on block order).
#include "kernels.h"

namespace dp {

namespace {

constexpr int kFT = kHistFeatureTile;  // 32 features per tile
constexpr int kQPR = kFT / 4;          // 32-bit words per row tile
constexpr int kRPW = 32 / kQPR;        // rows per warp step
constexpr int kUnroll = 8;             // row steps in flight per warp
constexpr int kHistThreads = 256;

__global__ void __launch_bounds__(kHistThreads) k_hist(const u8* __restrict__ bins, u64 bstride, u32 F,
                                                       const TreeArrays* __restrict__ trees,
                                                       const Scales* __restrict__ scales,
                                                       const HistTask* __restrict__ tasks, i64* __restrict__ hist) {
  extern __shared__ unsigned long long sh[];  // [kMaxBins][kFT]
  const HistTask t = tasks[blockIdx.x];
  for (int i = threadIdx.x; i < kMaxBins * kFT; i += kHistThreads) sh[i] = 0ull;
  __syncthreads();

  const TreeArrays ta = trees[t.tree];
  const Scales sc = scales[t.tree];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kWarps = kHistThreads / 32;
  const int s = lane / kQPR, q = lane % kQPR;
  // words past the row's bin_stride (last tile of a row) are never read
  const bool qvalid = u64(t.f0) + 4u * q < bstride;
  const u8* base = bins + t.f0 + 4 * q;
  constexpr i64 kStep = i64(kWarps) * kRPW;

  for (i64 i0 = t.begin + i64(warp) * kRPW + s; i0 < t.end; i0 += kStep * kUnroll) {
    u32 row[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const i64 i = i0 + u * kStep;
      row[u] = i < t.end ? __ldg(ta.ridx + i) : 0xffffffffu;
    }
    u32 word[kUnroll];
    float2 g[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (row[u] != 0xffffffffu && qvalid) {
        word[u] = __ldg(reinterpret_cast<const u32*>(base + u64(row[u]) * bstride));
        g[u] = __ldg(ta.gh + (i0 + u * kStep));
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (row[u] == 0xffffffffu || !qvalid) continue;
      const long long gq = quantize(g[u].x, sc.sg);
      const long long hq = quantize(g[u].y, sc.sh);
      const unsigned long long packed = (static_cast<unsigned long long>(gq) << 32) + static_cast<unsigned long long>(hq);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int jj = (j + s) & 3;
        const u32 b = (word[u] >> (8 * jj)) & 0xffu;
        atomicAdd(&sh[b * kFT + jj * kQPR + q], packed);
      }
    }
  }
  __syncthreads();

  i64* out = hist + u64(t.slot) * F * (2 * kMaxBins);
  for (int idx = threadIdx.x; idx < kMaxBins * kFT; idx += kHistThreads) {
    const unsigned long long v = sh[idx];
    if (!v) continue;
    const int b = idx / kFT, col = idx % kFT;
    const u32 f = t.f0 + 4 * (col % kQPR) + col / kQPR;
    if (f >= F) continue;
    const long long gs = static_cast<long long>(v) >> 32;
    const long long hs = static_cast<long long>(v & 0xffffffffull);
    unsigned long long* cell = reinterpret_cast<unsigned long long*>(out + (u64(f) * kMaxBins + b) * 2);
    atomicAdd(cell, static_cast<unsigned long long>(gs));
    atomicAdd(cell + 1, static_cast<unsigned long long>(hs));
  }
}

// hist[dst] = parent[par] - hist[src]; one block handles 2048 int64 of one triple.
__global__ void __launch_bounds__(256) k_subtract(i64* hist, const i64* __restrict__ parent, u64 slot_elems,
                                                  const u32* __restrict__ triples) {
  const u32 tr = blockIdx.y;
  const u32 par = triples[3 * tr], src = triples[3 * tr + 1], dst = triples[3 * tr + 2];
  const longlong2* a = reinterpret_cast<const longlong2*>(parent + u64(par) * slot_elems);
  const longlong2* b = reinterpret_cast<const longlong2*>(hist + u64(src) * slot_elems);
  longlong2* c = reinterpret_cast<longlong2*>(hist + u64(dst) * slot_elems);
  const u64 n2 = slot_elems / 2;
  for (u64 i = u64(blockIdx.x) * blockDim.x + threadIdx.x; i < n2; i += u64(gridDim.x) * blockDim.x) {
    const longlong2 x = a[i], y = b[i];
    c[i] = make_longlong2(x.x - y.x, x.y - y.y);
  }
}

}  // namespace

void launch_histograms(const u8* bins, u64 bin_stride, u32 F, const TreeArrays* trees, const Scales* scales,
                       const HistTask* tasks, u32 ntasks, i64* hist, cudaStream_t s) {
  if (!ntasks) return;
  constexpr int kSmem = kMaxBins * kFT * sizeof(unsigned long long);
  static thread_local int configured_device = -1;
  int dev = 0;
  DP_CUDA(cudaGetDevice(&dev));
  if (configured_device != dev) {
    DP_CUDA(cudaFuncSetAttribute(k_hist, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    configured_device = dev;
  }
  k_hist<<<ntasks, kHistThreads, kSmem, s>>>(bins, bin_stride, F, trees, scales, tasks, hist);
  after_launch("histograms");
}

void launch_subtract(i64* hist, const i64* parent_hist, u64 slot_elems, const u32* triples, u32 n, cudaStream_t s) {
  if (!n) return;
  const u64 blocks = (slot_elems / 2 + 2047) / 2048;
  dim3 grid(unsigned(blocks ? blocks : 1), n);
  k_subtract<<<grid, 256, 0, s>>>(hist, parent_hist, slot_elems, triples);
  after_launch("subtract");
}

}  // namespace dp
