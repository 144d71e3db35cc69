// Host launchers of the sm_100a kernels of the GBDT-training path.  All
// pointers are device pointers unless named *_host; every launcher enqueues on
// `stream` and never synchronises.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "common.h"
#include "dp_math.cuh"

namespace dp {

// One unit of histogram work: rows at positions [begin, end) of a node's
// segment, accumulated into histogram slot `slot` for features
// [f0, f0 + feature tile).
struct HistTask {
  u32 slot;
  u32 f0;
  u32 tree;   // selects the (g,h) / row-index arrays of this tree
  u32 excl;   // 1: no other task covers this (slot, tile); its sums are stored, not added
  i64 begin;
  i64 end;
};

// Per-tree position-ordered arrays used by the histogram and partition kernels.
struct TreeArrays {
  u32* ridx;    // [positions] row index
  float2* gh;   // [positions] (g, h)
};

// Quantiser scales of one tree: s_g, s_h.
struct Scales {
  float sg, sh;
};

// Best split candidate.  gain = -inf when no valid candidate exists.
struct SplitCand {
  double gain;
  i64 gl, hl;  // left quantised sums (missing bin included when default_left)
  i32 feature;
  i32 bin;
  i32 default_left;
  i32 pad;
};

constexpr u32 kNoSlot = 0xffffffffu;

// Open node handed to split evaluation.  A node whose histogram was not built
// (the larger sibling) has par != kNoSlot: its histogram is parent[par] -
// hist[small], derived while it is evaluated and stored into its slot.
struct EvalNode {
  u32 slot;   // histogram slot
  u32 tree;
  i64 gq, hq; // quantised totals
  u32 par;    // parent slot in the previous level's histograms, or kNoSlot
  u32 small;  // slot of the built sibling
};

#ifdef __CUDACC__
// Last-block pattern: every thread of a launch calls it once, after its
// block's writes that the last block reads.  True in the block that finishes
// last (the other blocks' writes are then visible to it through L2: read them
// with __ldcg); that block also returns *done to zero for the next launch.
__device__ __forceinline__ bool last_block(u32* done, u32 nblocks) {
  __shared__ bool s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    s_last = atomicAdd(done, 1u) + 1u == nblocks;
    if (s_last) atomicExch(done, 0u);  // every block has counted
  }
  __syncthreads();
  if (s_last) __threadfence();
  return s_last;
}

// Reduction by one whole block of M rows of n values each (row r at
// src[r * n], written by other blocks: read through L2) into out[r]: warp w
// takes columns [w n / W, (w + 1) n / W) of every row, with independent
// loads, then one thread per row combines the W warps' results.  sh holds
// W * M values (shared memory).
template <class T, class Op>
__device__ void reduce_rows(const T* src, u32 M, u32 n, T* sh, T* out, T init, Op op) {
  const u32 W = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const u32 c0 = u32(u64(n) * warp / W), c1 = u32(u64(n) * (warp + 1) / W);
  for (u32 r = 0; r < M; ++r) {
    const T* row = src + u64(r) * n;
    T acc = init;
    u32 c = c0 + lane;
    for (; c + 96 < c1; c += 128) {
      const T a = __ldcg(row + c), b = __ldcg(row + c + 32), d = __ldcg(row + c + 64), e = __ldcg(row + c + 96);
      acc = op(acc, op(op(a, b), op(d, e)));
    }
    for (; c < c1; c += 32) acc = op(acc, __ldcg(row + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = op(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if (lane == 0) sh[warp * M + r] = acc;
  }
  __syncthreads();
  for (u32 r = threadIdx.x; r < M; r += blockDim.x) {
    T acc = init;
    for (u32 w = 0; w < W; ++w) acc = op(acc, sh[w * M + r]);
    out[r] = acc;
  }
  __syncthreads();
}
#endif

// ---- binning (quantile cuts by exact radix selection) ---------------------
struct CutState;  // defined in k_quantile.cu
struct CutsDevice {
  float* cut = nullptr;      // [F][256] boundaries
  u16* nbins = nullptr;      // [F] value bins
  u8* has_missing = nullptr; // [F]
};

// ---- gradients --------------------------------------------------------------
enum Objective : int { kSquaredError = 0, kLogistic = 1, kSoftprob = 2, kSoftmax = 3 };

// Row sampling of one round: with rate < 1, row r of tree k is kept iff
// sample_uniform(sample_hash(seed, *round, k, kSampleRow, row0 + r, 0)) <
// rate; a dropped row's (g, h) become (0, 0) before the maxima, so it adds
// nothing to any histogram.  row0 is this rank's first global row.
struct RowSample {
  double rate = 1.0;
  long long seed = 0;
  const u32* round = nullptr;  // device counter of the current round
  u64 row0 = 0;
};
// gh[k][r] from margins [R][K] and labels; maxima of |g| and h per class are
// atomically maxed into gmax[k], hmax[k] (float bits as u32; must be zeroed).
void launch_gradients(int objective, int K, const float* margin, const float* label, u64 R, float2* gh,
                      u32* gmax_bits, u32* hmax_bits, cudaStream_t s, const RowSample& rs = RowSample());
// scales[k] from the maxima.
void launch_scales(int K, const u32* gmax_bits, const u32* hmax_bits, Scales* scales, cudaStream_t s);
// The same gradients for K <= 64 without atomics on zeroed maxima: each block
// writes its maxima to part ([2K][gradient_blocks(R)] u32), and the last
// block reduces them into gmax / hmax and, with scales set, computes the
// scales (launch_scales' formula).  *done must be zero at the first launch;
// every launch leaves it zero.  Launches one block even for R == 0.
constexpr int kMaxReducedClasses = 64;
u32 gradient_blocks(u64 R);
void launch_gradients_reduced(int objective, int K, const float* margin, const float* label, u64 R, float2* gh,
                              u32* gmax_bits, u32* hmax_bits, u32* part, u32* done, Scales* scales, cudaStream_t s,
                              const RowSample& rs = RowSample{});
// Copies n segments of 32-bit words (src[i] -> dst[i], words[i] each) in one
// launch; dst may be pinned host memory (its device address).
void launch_copy_words(const u32* const* src, u32* const* dst, const u64* words, int n, cudaStream_t s);

// ---- histograms -------------------------------------------------------------
// hist[slot][F][256][2] (int64) must be zeroed for every slot the tasks touch.
// Every bin value must be < max_bins (<= 64 selects a smaller tile).  With
// quantized_gh the (g, h) arrays hold int32 pairs (see launch_quantize_gh);
// otherwise fp32 pairs quantised with `scales`.  `counter` is one u32 of
// device scratch (the task queue), reset by the launcher unless
// counter_zeroed says a kernel before it on the stream zeroed it.  Positions
// must be below 2^31.
// With ntasks_dev set, the task count is read from device memory (ntasks is
// then ignored) and the grid covers every SM.
// Output layout (element offsets; a cell is the (g, h) pair of one bin):
// feature f of slot s lands at (f / fg) * group_stride + s * slot_stride +
// (f % fg) * 2 * kMaxBins.  The default (layout == nullptr) is fg = F,
// slot_stride = F * 2 * kMaxBins: hist[slot][F][256][2].  Feature groups of
// fg features let the sums of each group be contiguous over the built slots
// (what a reduce-scatter over feature groups needs).
struct HistLayout {
  u32 fg;
  u64 slot_stride;
  u64 group_stride;
};
void launch_histograms(const u8* bins, u64 bin_stride, u32 F, int max_bins, bool quantized_gh,
                       const TreeArrays* trees, const Scales* scales, const HistTask* tasks, u32 ntasks,
                       u32* counter, i64* hist, cudaStream_t s, const u32* ntasks_dev = nullptr,
                       const HistLayout* layout = nullptr, bool counter_zeroed = false);
constexpr u32 kHistFeatureTile = 32;
// The 256-bin build over 64-feature tasks (HistTask.f0 a multiple of 64):
// same inputs and output as launch_histograms; one block per SM, each using
// all of its SM's tensor memory for the window sums.
constexpr u32 kHistWideTile = 64;
void launch_histograms_wide(const u8* bins, u64 bin_stride, u32 F, bool quantized_gh, const TreeArrays* trees,
                            const Scales* scales, const HistTask* tasks, u32 ntasks, u32* counter, i64* hist,
                            cudaStream_t s, const u32* ntasks_dev, const HistLayout* layout,
                            bool counter_zeroed = false);
// Rows per histogram task for a launch over `total_rows` row-tiles of nseg
// segments (about four tasks per SM, sixteen for 2 to 16 segments, eight for
// 17 to 256, three when every row is whole 128-byte lines).
u64 hist_chunk_rows(u64 total_rows, u64 nseg, bool whole_lines);
// Bin budget of the 32-feature kernel that a kernel-level build launches when
// its codes are below num_bins and `segments` segments hold rows.  The 64-bin
// kernel (two 512-thread blocks per SM, int64 sums in shared memory) is the
// faster one only from 2 to 256 segments; with one segment, or 512 and more,
// the 256-bin kernel is.  Measured on B200, 100M x 32 rows, 64-bin codes
// (16-bin codes the same within 1 %), 64-bin against 256-bin kernel: 1 node
// 1.41 / 1.18 ms, 2 nodes 1.27 / 1.34, 8 nodes 1.40 / 1.50, 64 nodes 1.56 /
// 1.62, 256 nodes 1.60 / 1.74, 512 nodes 1.80 / 1.69, 1024 nodes 2.22 / 1.88.
// Both kernels give identical sums.
inline int hist_kernel_bins(int num_bins, u64 segments) {
  return (num_bins <= 64 && segments >= 2 && segments <= 256) ? num_bins : 256;
}
// gh[k][r] (fp32 pairs) -> int32 pairs rint(g * s_g), rint(h * s_h), in place.
void launch_quantize_gh(float2* gh, u64 R, int K, const Scales* scales, cudaStream_t s);

// ---- split evaluation --------------------------------------------------------
// Per (node, feature chunk) candidate into cand[node][chunk]; then the best per
// node into best[node].
void launch_eval_splits(const i64* hist, u32 F, const u16* nbins, const u8* has_missing, const EvalNode* nodes,
                        u32 nnodes, const Scales* scales, SplitParams p, SplitCand* cand, SplitCand* best,
                        cudaStream_t s);
// Features per split-evaluation work item: 8 (one per warp) gives small
// levels twice the blocks of 16 (measured: config 1 0.266 -> 0.247 ms,
// config 2 0.842 -> 0.815 ms per round, config 4 unchanged).
#ifndef DP_EVAL_CHUNK
#define DP_EVAL_CHUNK 8
#endif
constexpr u32 kEvalFeatureChunk = DP_EVAL_CHUNK;
// The same with the node count in device memory, over F features that sit
// at a stride of fstride features per slot (0: F) and whose global ids start
// at f_base (nbins / has_missing point at the first of them).  F may be 0:
// every node then gets "no candidate" (gain -inf, feature -1).
// With fmask set, feature f (global id) of the open node at index i is a
// candidate only if bit f of fmask[i * mask_words ...] is set.
// Per (node, feature chunk) candidates only, cand[node * nchunks + chunk],
// with nchunks >= ceil(F / kEvalFeatureChunk) and >= 1 (chunks past the
// features hold "no candidate"); the caller takes the best over chunks.
// Derived siblings read parent_hist; with store_derived their histograms are
// written into their slots (needed when the next level subtracts from them).
void launch_eval_candidates_dev(const i64* hist, u32 F, const u16* nbins, const u8* has_missing,
                                const EvalNode* nodes, const u32* nnodes_dev, const Scales* scales, SplitParams p,
                                SplitCand* cand, u32 nchunks, cudaStream_t s, u32 fstride, u32 f_base,
                                const u32* fmask, u32 mask_words, const i64* parent_hist, int store_derived);

// ---- partition ----------------------------------------------------------------
struct PartTask {
  u32 node;      // index into PartNode
  u32 pad;
  i64 begin;     // positions [begin, end), at most kPartChunk rows
  i64 end;
};
struct PartNode {
  u32 tree;
  i32 feature;
  i32 bin;
  i32 default_left;
  i32 missing_is_bin;  // has_missing[feature]
  i32 pad;
  i64 begin;           // segment [begin, end)
  i64 end;
};
// Splits every node's segment from `src` into `dst`: left rows fill
// [begin, begin + nleft), right rows [begin + nleft, end).  cursors[2*node]
// and cursors[2*node+1] (zeroed u32 scratch) end as the node's left and right
// row counts.  Bin codes come from the 32-row blocked layout:
// bins_blk[(r / 32) * blk_stride + f * 32 + r % 32], blk_stride = 32 * F.
void launch_partition(const u8* bins_blk, u64 blk_stride, const TreeArrays* src, const TreeArrays* dst,
                      const PartNode* nodes, const PartTask* tasks, u32 ntasks, u32* cursors, cudaStream_t s);
// Rows per partition task: 2048 gives small levels twice the tasks of 4096
// (measured with the 8-feature evaluation items: config 1 0.247 -> 0.230 ms,
// config 2 0.815 -> 0.778 ms per round, config 4 5.33 -> 5.34 ms).
#ifndef DP_PART_CHUNK
#define DP_PART_CHUNK 2048
#endif
constexpr u32 kPartChunk = DP_PART_CHUNK;
// The same with the task count in device memory.
void launch_partition_dev(const u8* bins_blk, u64 blk_stride, const TreeArrays* src, const TreeArrays* dst,
                          const PartNode* nodes, const PartTask* tasks, const u32* ntasks_dev, u32* cursors,
                          cudaStream_t s);

// ---- leaves -------------------------------------------------------------------
// The last level's split nodes: each row of the tasks adds vals[2 node] (left)
// or vals[2 node + 1] (right), f32 bits, to margin[row * K + tree]; rows do
// not move.
void launch_partition_leaves(const u8* bins_blk, u64 blk_stride, const TreeArrays* src, const PartNode* nodes,
                             const PartTask* tasks, const u32* ntasks_dev, const u32* vals, float* margin, u32 K,
                             cudaStream_t s);
struct LeafTask {
  const u32* ridx;
  i64 begin, end;
  float value;
  u32 klass;
};
void launch_leaf_update(const LeafTask* tasks, u32 ntasks, float* margin, u32 K, cudaStream_t s);
void launch_leaf_update_dev(const LeafTask* tasks, const u32* ntasks_dev, float* margin, u32 K, cudaStream_t s);

// ---- misc ---------------------------------------------------------------------
// margin[r][k] = base[k] for r < R.
void launch_init_margins(float* margin, u64 R, int K, const float* base, cudaStream_t s);
// Flags (atomicOr into bad[0]) any +-inf in x[r*stride + f].
void launch_check_finite(const float* x, u64 R, u32 F, u64 stride, u32* bad, cudaStream_t s);
// Labels: flags values that are not valid for the objective.
void launch_check_labels(const float* y, u64 R, int objective, int K, u32* bad, cudaStream_t s);

}  // namespace dp
