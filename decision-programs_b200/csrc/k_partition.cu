// Row partition: stable split of every split node's position segment into
// [left rows][right rows], moving the row index and the (g, h) pair together
// so that the next histogram pass reads (g, h) contiguously.
// Routing: bin <= split bin goes left (equivalent to x < split_condition);
// the missing code follows default_left (native/class_tree_runtime_compare.cu:47,
// native/class_runtime.cu:128).
#include "kernels.h"

namespace dp {

namespace {

constexpr int kPartThreads = 256;
constexpr int kWordsPerTask = kPartChunk / 32;

__device__ __forceinline__ bool goes_left(u8 b, const PartNode& nd) {
  if (nd.missing_is_bin && b == kMissingBin) return nd.default_left != 0;
  return int(b) <= nd.bin;
}

__global__ void __launch_bounds__(kPartThreads) k_part_count(const u8* __restrict__ bins, u64 bstride,
                                                             const TreeArrays* __restrict__ trees,
                                                             const PartNode* __restrict__ nodes,
                                                             const PartTask* __restrict__ tasks, u32* __restrict__ flags,
                                                             u32* __restrict__ left) {
  __shared__ u32 wsum[kPartThreads / 32];
  const PartTask t = tasks[blockIdx.x];
  const PartNode nd = nodes[t.node];
  const u32* ridx = trees[nd.tree].ridx;
  const u8* col = bins + nd.feature;
  u32* fl = flags + u64(blockIdx.x) * kWordsPerTask;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  u32 cnt = 0;
  constexpr int kIlp = 4;  // independent row gathers in flight per thread
  for (i64 base = t.begin; base < t.end; base += kPartThreads * kIlp) {
    u32 r[kIlp];
#pragma unroll
    for (int u = 0; u < kIlp; ++u) {
      const i64 i = base + u * kPartThreads + threadIdx.x;
      r[u] = i < t.end ? __ldg(ridx + i) : 0xffffffffu;
    }
    u8 b[kIlp];
#pragma unroll
    for (int u = 0; u < kIlp; ++u) b[u] = r[u] != 0xffffffffu ? __ldg(col + u64(r[u]) * bstride) : u8(0);
#pragma unroll
    for (int u = 0; u < kIlp; ++u) {
      const bool go = r[u] != 0xffffffffu && goes_left(b[u], nd);
      const u32 ballot = __ballot_sync(0xffffffffu, go);
      const i64 w0 = base + u * kPartThreads + warp * 32;
      if (lane == 0 && w0 < t.end) fl[(w0 - t.begin) / 32] = ballot;
      cnt += go;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if (lane == 0) wsum[warp] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    u32 s = 0;
    for (int w = 0; w < kPartThreads / 32; ++w) s += wsum[w];
    left[blockIdx.x] = s;
  }
}

__global__ void __launch_bounds__(kPartThreads) k_part_scatter(const TreeArrays* __restrict__ src,
                                                               const TreeArrays* __restrict__ dst,
                                                               const PartNode* __restrict__ nodes,
                                                               const PartTask* __restrict__ tasks,
                                                               const u32* __restrict__ flags,
                                                               const i64* __restrict__ left_off,
                                                               const i64* __restrict__ right_off) {
  __shared__ u32 wl[kPartThreads / 32];
  const PartTask t = tasks[blockIdx.x];
  const PartNode nd = nodes[t.node];
  const TreeArrays s = src[nd.tree];
  const TreeArrays d = dst[nd.tree];
  const u32* fl = flags + u64(blockIdx.x) * kWordsPerTask;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  i64 lpos = nd.begin + left_off[blockIdx.x];
  i64 rpos = nd.begin + nd.nleft + right_off[blockIdx.x];
  for (i64 base = t.begin; base < t.end; base += kPartThreads) {
    const i64 w0 = base + warp * 32;
    const u32 ballot = w0 < t.end ? fl[(w0 - t.begin) / 32] : 0u;
    if (lane == 0) wl[warp] = __popc(ballot);
    __syncthreads();
    u32 lbefore = 0, ltotal = 0;
    for (int w = 0; w < kPartThreads / 32; ++w) {
      const u32 c = wl[w];
      if (w < warp) lbefore += c;
      ltotal += c;
    }
    const i64 rows_before = i64(warp) * 32;  // valid rows in earlier warps of this step
    const i64 step_rows = (t.end - base) < kPartThreads ? (t.end - base) : i64(kPartThreads);
    const i64 i = base + threadIdx.x;
    if (i < t.end) {
      const u32 lt = (1u << lane) - 1u;
      const bool go = (ballot >> lane) & 1u;
      const u32 lrank = lbefore + __popc(ballot & lt);
      const i64 dstpos = go ? lpos + lrank
                            : rpos + (rows_before + lane - i64(lrank));
      d.ridx[dstpos] = s.ridx[i];
      d.gh[dstpos] = s.gh[i];
    }
    lpos += ltotal;
    rpos += step_rows - ltotal;
    __syncthreads();
  }
}

}  // namespace

void launch_partition_count(const u8* bins, u64 bin_stride, const TreeArrays* trees, const PartNode* nodes,
                            const PartTask* tasks, u32 ntasks, u32* flags, u32* left, cudaStream_t s) {
  if (!ntasks) return;
  k_part_count<<<ntasks, kPartThreads, 0, s>>>(bins, bin_stride, trees, nodes, tasks, flags, left);
  after_launch("partition_count");
}

void launch_partition_scatter(const TreeArrays* src, const TreeArrays* dst, const PartNode* nodes,
                              const PartTask* tasks, u32 ntasks, const u32* flags, const i64* left_off,
                              const i64* right_off, cudaStream_t s) {
  if (!ntasks) return;
  k_part_scatter<<<ntasks, kPartThreads, 0, s>>>(src, dst, nodes, tasks, flags, left_off, right_off);
  after_launch("partition_scatter");
}

}  // namespace dp
