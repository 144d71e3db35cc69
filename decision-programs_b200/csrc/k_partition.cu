// Row partition: every split node's position segment becomes
// [left rows][right rows]; the row index and the quantised (g, h) pair move
// together so that the next histogram pass reads (g, h) contiguously.
// Routing: bin <= split bin goes left (equivalent to x < split_condition);
// the missing code follows default_left (native/class_tree_runtime_compare.cu:47,
// native/class_runtime.cu:128).
//
// The split feature's code of row r is read from the 32-row blocked bin
// layout (bins_blk[r / 32][f][r % 32]), so one 32-byte sector serves up to 32
// rows of a node instead of one row per 128-byte row-major line.
//
// One pass: a block decides its task's rows (decision bits kept in shared
// memory), reserves space in its node's left and right parts with one atomic
// add on each of the node's cursors, then scatters: left rows upward from the
// segment start, right rows downward from the segment end.  Row order inside a
// segment depends on block scheduling, but nothing computed from a segment
// does: histogram sums are integer and every row gets exactly one leaf.
#include "kernels.h"

namespace dp {

namespace {

constexpr int kPartThreads = 256;
// Independent row gathers in flight per thread.  Below depth 4 every row's
// code is its own 32-byte sector (a 64-byte DRAM fetch), and ncu shows DRAM
// about half busy with 21 long-scoreboard stalls per issue at five blocks per
// SM; sixteen gathers per thread (4096-row tasks, four blocks per SM) were
// slower on B200 (config 4: 4.95 against 4.85 ms per round).
#ifndef DP_PART_ILP
#define DP_PART_ILP 8
#endif
constexpr int kIlp = DP_PART_ILP;
constexpr int kScatterSteps = 4;  // 256-position steps whose (g, h) loads are in flight together
constexpr int kWordsPerTask = kPartChunk / 32;
static_assert(kPartChunk % (kPartThreads * kIlp) == 0, "task rows are whole gather rounds");
static_assert(kPartChunk % (kPartThreads * kScatterSteps) == 0, "task rows are whole scatter rounds");

__device__ __forceinline__ bool goes_left(u8 b, const PartNode& nd) {
  if (nd.missing_is_bin && b == kMissingBin) return nd.default_left != 0;
  return int(b) <= nd.bin;
}

__device__ __forceinline__ void partition_task(u32 task, const u8* __restrict__ bins_blk, u64 blk_stride,
                                               const TreeArrays* __restrict__ src,
                                               const TreeArrays* __restrict__ dst,
                                               const PartNode* __restrict__ nodes,
                                               const PartTask* __restrict__ tasks, u32* __restrict__ cursors) {
  __shared__ u32 ballots[kWordsPerTask];
  __shared__ u32 s_ridx[kPartChunk];  // the task's row indices, read once
  __shared__ u32 wsum[kPartThreads / 32];
  __shared__ u32 base_lr[2];
  const PartTask t = tasks[task];
  const PartNode nd = nodes[t.node];
  const TreeArrays s = src[nd.tree];
  const TreeArrays d = dst[nd.tree];
  const u8* col = bins_blk + u64(nd.feature) * 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const u32 n = u32(t.end - t.begin);

  // decisions
  u32 cnt = 0;
  for (u32 base = 0; base < n; base += kPartThreads * kIlp) {
    u32 r[kIlp];
#pragma unroll
    for (int u = 0; u < kIlp; ++u) {
      const u32 i = base + u * kPartThreads + threadIdx.x;
      r[u] = i < n ? __ldg(s.ridx + t.begin + i) : 0xffffffffu;
      if (i < n) s_ridx[i] = r[u];
    }
    u8 b[kIlp];
#pragma unroll
    for (int u = 0; u < kIlp; ++u)
      b[u] = r[u] != 0xffffffffu ? __ldg(col + u64(r[u] >> 5) * blk_stride + (r[u] & 31u)) : u8(0);
#pragma unroll
    for (int u = 0; u < kIlp; ++u) {
      const bool go = r[u] != 0xffffffffu && goes_left(b[u], nd);
      const u32 ballot = __ballot_sync(0xffffffffu, go);
      if (lane == 0) ballots[(base + u * kPartThreads) / 32 + warp] = ballot;
      cnt += go;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if (lane == 0) wsum[warp] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    u32 left = 0;
    for (int w = 0; w < kPartThreads / 32; ++w) left += wsum[w];
    base_lr[0] = atomicAdd(cursors + 2 * t.node, left);
    base_lr[1] = atomicAdd(cursors + 2 * t.node + 1, n - left);
  }
  __syncthreads();

  // scatter, 256 positions per step, kScatterSteps steps' (g, h) loads in
  // flight together; ranks from the stored ballots
  u32 run_left = 0;
  const i64 lbase = nd.begin + base_lr[0];
  const i64 rtop = nd.end - 1 - i64(base_lr[1]);
  for (u32 base0 = 0; base0 < n; base0 += kPartThreads * kScatterSteps) {
    float2 g[kScatterSteps];
#pragma unroll
    for (int u = 0; u < kScatterSteps; ++u) {
      const u32 i = base0 + u * kPartThreads + threadIdx.x;
      if (i < n) g[u] = __ldg(s.gh + t.begin + i);
    }
#pragma unroll
    for (int u = 0; u < kScatterSteps; ++u) {
      const u32 base = base0 + u * kPartThreads;
      const u32 wi = base / 32 + warp;
      const u32 ballot = base + warp * 32 < n ? ballots[wi] : 0u;
      u32 before = 0, step_left = 0;
#pragma unroll
      for (int w = 0; w < kPartThreads / 32; ++w) {
        const u32 c = (base + w * 32 < n) ? __popc(ballots[base / 32 + w]) : 0u;
        if (w < warp) before += c;
        step_left += c;
      }
      const u32 i = base + threadIdx.x;
      if (i < n) {
        const bool go = (ballot >> lane) & 1u;
        const u32 lrank = run_left + before + __popc(ballot & ((1u << lane) - 1u));
        const i64 to = go ? lbase + lrank : rtop - i64(i - lrank);
        d.ridx[to] = s_ridx[i];
        d.gh[to] = g[u];
      }
      run_left += step_left;
    }
  }
  __syncthreads();  // shared state is reused by the block's next task
}

__global__ void __launch_bounds__(kPartThreads) k_partition(const u8* __restrict__ bins_blk, u64 blk_stride,
                                                            const TreeArrays* __restrict__ src,
                                                            const TreeArrays* __restrict__ dst,
                                                            const PartNode* __restrict__ nodes,
                                                            const PartTask* __restrict__ tasks,
                                                            u32* __restrict__ cursors) {
  partition_task(blockIdx.x, bins_blk, blk_stride, src, dst, nodes, tasks, cursors);
}

// Task count in device memory: a fixed grid walks the tasks.
__global__ void __launch_bounds__(kPartThreads) k_partition_dev(const u8* __restrict__ bins_blk, u64 blk_stride,
                                                                const TreeArrays* __restrict__ src,
                                                                const TreeArrays* __restrict__ dst,
                                                                const PartNode* __restrict__ nodes,
                                                                const PartTask* __restrict__ tasks,
                                                                const u32* __restrict__ ntasks,
                                                                u32* __restrict__ cursors) {
  const u32 n = *ntasks;
  for (u32 t = blockIdx.x; t < n; t += gridDim.x)
    partition_task(t, bins_blk, blk_stride, src, dst, nodes, tasks, cursors);
}

// The last level of a tree: nothing is built from the children, so rows do
// not move; each row of a split node adds its child's leaf value (vals, f32
// bits [2 node + side]) to its margin, the same float addition the margin
// update makes.
__global__ void __launch_bounds__(kPartThreads) k_partition_leaves(const u8* __restrict__ bins_blk, u64 blk_stride,
                                                                   const TreeArrays* __restrict__ src,
                                                                   const PartNode* __restrict__ nodes,
                                                                   const PartTask* __restrict__ tasks,
                                                                   const u32* __restrict__ ntasks,
                                                                   const u32* __restrict__ vals, float* margin, u32 K) {
  const u32 n = *ntasks;
  for (u32 task = blockIdx.x; task < n; task += gridDim.x) {
    const PartTask t = tasks[task];
    const PartNode nd = nodes[t.node];
    const u32* ridx = src[nd.tree].ridx + t.begin;
    const float vl = __uint_as_float(vals[2 * t.node]), vr = __uint_as_float(vals[2 * t.node + 1]);
    const u8* col = bins_blk + u64(nd.feature) * 32;
    const u32 cnt = u32(t.end - t.begin);
    for (u32 base = 0; base < cnt; base += kPartThreads * kIlp) {
      u32 r[kIlp];
#pragma unroll
      for (int u = 0; u < kIlp; ++u) {
        const u32 i = base + u * kPartThreads + threadIdx.x;
        r[u] = i < cnt ? __ldg(ridx + i) : 0xffffffffu;
      }
      u8 b[kIlp];
      float m[kIlp];
#pragma unroll
      for (int u = 0; u < kIlp; ++u) {
        b[u] = 0;
        m[u] = 0.f;
        if (r[u] != 0xffffffffu) {
          b[u] = __ldg(col + u64(r[u] >> 5) * blk_stride + (r[u] & 31u));
          m[u] = margin[u64(r[u]) * K + nd.tree];
        }
      }
#pragma unroll
      for (int u = 0; u < kIlp; ++u)
        if (r[u] != 0xffffffffu) margin[u64(r[u]) * K + nd.tree] = m[u] + (goes_left(b[u], nd) ? vl : vr);
    }
  }
}

}  // namespace

void launch_partition_leaves(const u8* bins_blk, u64 blk_stride, const TreeArrays* src, const PartNode* nodes,
                             const PartTask* tasks, const u32* ntasks_dev, const u32* vals, float* margin, u32 K,
                             cudaStream_t s) {
  int dev = 0, sms = 148;
  DP_CUDA(cudaGetDevice(&dev));
  DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  k_partition_leaves<<<sms * 8, kPartThreads, 0, s>>>(bins_blk, blk_stride, src, nodes, tasks, ntasks_dev, vals,
                                                       margin, K);
  after_launch("partition_leaves");
}

void launch_partition(const u8* bins_blk, u64 blk_stride, const TreeArrays* src, const TreeArrays* dst,
                      const PartNode* nodes, const PartTask* tasks, u32 ntasks, u32* cursors, cudaStream_t s) {
  if (!ntasks) return;
  k_partition<<<ntasks, kPartThreads, 0, s>>>(bins_blk, blk_stride, src, dst, nodes, tasks, cursors);
  after_launch("partition");
}

void launch_partition_dev(const u8* bins_blk, u64 blk_stride, const TreeArrays* src, const TreeArrays* dst,
                          const PartNode* nodes, const PartTask* tasks, const u32* ntasks_dev, u32* cursors,
                          cudaStream_t s) {
  int dev = 0, sms = 148;
  DP_CUDA(cudaGetDevice(&dev));
  DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  k_partition_dev<<<sms * 8, kPartThreads, 0, s>>>(bins_blk, blk_stride, src, dst, nodes, tasks, ntasks_dev,
                                                    cursors);
  after_launch("partition");
}

}  // namespace dp
