// Histogram build: for every task (node slot, 32-feature tile, a range of the
// node's row positions) accumulate the quantised (g, h) of each row into
// hist[slot][f][bin] (int64 pairs).
//
// Design (HBM- and shared-atomic-bound, no tensor cores):
//  * two u32 planes in shared memory, g and h, laid out [bin][column]: one
//    32-bit shared atomic per (row, feature) and plane.  The quantiser bounds
//    (|q_g| <= 2^17, q_h <= 2^18) keep the sums of an 8192-row window inside
//    int32 / uint32, so after every window the planes are folded into int64
//    planes in shared memory; a block can therefore own an arbitrarily long
//    row range and drains to global memory once;
//  * a warp reads 4 rows x 32 features per step: lane (s, q) loads the 32-bit
//    word holding features 4q..4q+3 of row s.  In atomic step j the lane
//    updates feature 4q + ((j + s) & 3), whose column is ((j+s)&3)*8 + q, so
//    the 32 lanes of a step hit 32 distinct banks whatever the bins are;
//  * rows are gathered through the node's row-index segment; (g, h) is read
//    in position order (the partition kernel moves it with the row index);
//  * the final drain uses 64-bit global atomics (integer: order-independent).
#include "kernels.h"

namespace dp {

namespace {

constexpr int kFT = kHistFeatureTile;  // 32 features per tile
constexpr int kQPR = kFT / 4;          // 32-bit words per row tile
constexpr int kRPW = 32 / kQPR;        // rows per warp step
constexpr int kUnroll = 8;             // row steps in flight per warp

template <int MB, int THREADS>
__global__ void __launch_bounds__(THREADS) k_hist(const u8* __restrict__ bins, u64 bstride, u32 F,
                                                  const TreeArrays* __restrict__ trees,
                                                  const Scales* __restrict__ scales,
                                                  const HistTask* __restrict__ tasks, i64* __restrict__ hist) {
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr int kCells = MB * kFT;
  u32* Lg = reinterpret_cast<u32*>(smem);
  u32* Lh = Lg + kCells;
  long long* Wg = reinterpret_cast<long long*>(Lh + kCells);
  long long* Wh = Wg + kCells;
  const HistTask t = tasks[blockIdx.x];
  const bool multi = t.end - t.begin > kWindowRows;
  for (int i = threadIdx.x; i < kCells; i += THREADS) {
    Lg[i] = 0u;
    Lh[i] = 0u;
    if (multi) { Wg[i] = 0; Wh[i] = 0; }
  }
  __syncthreads();

  const TreeArrays ta = trees[t.tree];
  const Scales sc = scales[t.tree];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kWarps = THREADS / 32;
  const int s = lane / kQPR, q = lane % kQPR;
  // words past the row's bin_stride (last tile of a row) are never read
  const bool qvalid = u64(t.f0) + 4u * q < bstride;
  const u8* base = bins + t.f0 + 4 * q;
  constexpr i64 kStep = i64(kWarps) * kRPW;

  for (i64 w0 = t.begin; w0 < t.end; w0 += kWindowRows) {
    const i64 w1 = (t.end - w0) < kWindowRows ? t.end : w0 + kWindowRows;
    for (i64 i0 = w0 + i64(warp) * kRPW + s; i0 < w1; i0 += kStep * kUnroll) {
      u32 row[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const i64 i = i0 + u * kStep;
        row[u] = i < w1 ? __ldg(ta.ridx + i) : 0xffffffffu;
      }
      u32 word[kUnroll];
      float2 g[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        word[u] = 0u;
        g[u] = make_float2(0.f, 0.f);
        if (row[u] != 0xffffffffu && qvalid) {
          word[u] = __ldg(reinterpret_cast<const u32*>(base + u64(row[u]) * bstride));
          g[u] = __ldg(ta.gh + (i0 + u * kStep));
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (row[u] == 0xffffffffu || !qvalid) continue;
        const u32 gq = static_cast<u32>(quantize(g[u].x, sc.sg));
        const u32 hq = static_cast<u32>(quantize(g[u].y, sc.sh));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int jj = (j + s) & 3;
          const u32 b = (word[u] >> (8 * jj)) & 0xffu;
          if (MB < 256 && b >= u32(MB)) continue;
          const int cell = int(b) * kFT + jj * kQPR + q;
          atomicAdd(Lg + cell, gq);
          atomicAdd(Lh + cell, hq);
        }
      }
    }
    if (multi) {
      __syncthreads();
      for (int i = threadIdx.x; i < kCells; i += THREADS) {
        Wg[i] += static_cast<long long>(static_cast<int>(Lg[i]));
        Wh[i] += static_cast<long long>(Lh[i]);
        Lg[i] = 0u;
        Lh[i] = 0u;
      }
      __syncthreads();
    }
  }
  __syncthreads();

  i64* out = hist + u64(t.slot) * F * (2 * kMaxBins);
  for (int idx = threadIdx.x; idx < kCells; idx += THREADS) {
    const long long gs = multi ? Wg[idx] : static_cast<long long>(static_cast<int>(Lg[idx]));
    const long long hs = multi ? Wh[idx] : static_cast<long long>(Lh[idx]);
    if (!(gs | hs)) continue;
    const int b = idx / kFT, col = idx % kFT;
    const u32 f = t.f0 + 4 * (col % kQPR) + col / kQPR;
    if (f >= F) continue;
    unsigned long long* cell = reinterpret_cast<unsigned long long*>(out + (u64(f) * kMaxBins + b) * 2);
    atomicAdd(cell, static_cast<unsigned long long>(gs));
    atomicAdd(cell + 1, static_cast<unsigned long long>(hs));
  }
}

template <int MB, int THREADS>
void launch_hist_variant(const u8* bins, u64 bin_stride, u32 F, const TreeArrays* trees, const Scales* scales,
                         const HistTask* tasks, u32 ntasks, i64* hist, cudaStream_t s) {
  constexpr int kSmem = MB * kFT * (4 + 4 + 8 + 8);
  static thread_local int configured_device = -1;
  int dev = 0;
  DP_CUDA(cudaGetDevice(&dev));
  if (configured_device != dev) {
    DP_CUDA(cudaFuncSetAttribute(k_hist<MB, THREADS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    configured_device = dev;
  }
  k_hist<MB, THREADS><<<ntasks, THREADS, kSmem, s>>>(bins, bin_stride, F, trees, scales, tasks, hist);
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

void launch_histograms(const u8* bins, u64 bin_stride, u32 F, int max_bins, const TreeArrays* trees,
                       const Scales* scales, const HistTask* tasks, u32 ntasks, i64* hist, cudaStream_t s) {
  if (!ntasks) return;
  if (max_bins <= 64)
    launch_hist_variant<64, 512>(bins, bin_stride, F, trees, scales, tasks, ntasks, hist, s);
  else
    launch_hist_variant<256, 1024>(bins, bin_stride, F, trees, scales, tasks, ntasks, hist, s);
  after_launch("histograms");
}

u64 hist_chunk_rows(u64 total_rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const u64 target = u64(sms) * 2;  // about two blocks per SM over the launch
  u64 chunk = (total_rows + target - 1) / target;
  chunk = (chunk + kWindowRows - 1) / kWindowRows * kWindowRows;
  return chunk < u64(kWindowRows) ? u64(kWindowRows) : chunk;
}

void launch_subtract(i64* hist, const i64* parent_hist, u64 slot_elems, const u32* triples, u32 n, cudaStream_t s) {
  if (!n) return;
  const u64 blocks = (slot_elems / 2 + 2047) / 2048;
  dim3 grid(unsigned(blocks ? blocks : 1), n);
  k_subtract<<<grid, 256, 0, s>>>(hist, parent_hist, slot_elems, triples);
  after_launch("subtract");
}

}  // namespace dp
