// Device-side bookkeeping of one boosting round: node records of the K trees,
// the open nodes of the current level, and the work lists each level's
// kernels consume.  Every count lives in device memory, so the host enqueues a
// whole round without waiting and reads the trees back once.  Every buffer a
// kernel writes carries its capacity; a write past it sets a bit of
// RoundCounters::overflow instead of touching memory, and the host turns a set
// bit into an error after the round.
#pragma once
#include "kernels.h"

namespace dp {

// One tree node; records are laid out [node id][tree] so that capacity grows
// by appending.
struct NodeRec {
  i64 gq, hq;              // quantised totals over all ranks
  i32 left, right, parent, feature;
  i32 bin, default_left;
  float cond, gain;        // split threshold (leaf value at a leaf), gain
};
static_assert(sizeof(NodeRec) == 48, "node record layout");

struct OpenRec {
  u32 tree, id, slot, pad;
  i64 begin, count;        // this rank's positions
};

struct LeafRec {
  u32 tree, id, set, pad;
  i64 begin, count;
};

struct RoundCounters {
  u32 n_open, n_build, n_split, n_hist_tasks;
  u32 n_part_tasks, n_leaves, n_leaf_tasks, n_triples;
  u32 overflow;
  u32 n_zero;              // histogram slots the next histogram launch adds into (zero_list)
  u32 pad[6];
};

// Overflow bits.
enum : u32 {
  kOvfHistTasks = 1, kOvfNodes = 2, kOvfLeaves = 4, kOvfPartTasks = 8, kOvfLeafTasks = 16,
  kOvfLostRows = 32, kOvfOpen = 64, kOvfBadCand = 256,
};

constexpr i64 kLeafChunkRows = 16384;  // rows per margin-update task

struct LevelStats {
  i64 rows_built;          // this rank's rows in directly built nodes
  u32 n_build, n_open;
};

struct RoundBuffers {
  NodeRec* nodes;          // [maxn][K]
  u32* next_id;            // [K]
  u32* tree_first;         // [K] scratch of the decision kernel
  OpenRec* open_cur;       // this level's open nodes (trees contiguous, ids ascending)
  OpenRec* open_next;      // [cap_next]
  u32* build;              // open indices of this level's directly built nodes
  const u32* triples;      // this level's (parent slot, small slot, large slot), [n_triples]
  u32* build_next;         // [cap_split]
  u32* triples_next;       // [3 * cap_split] (parent slot, small slot, large slot)
  HistTask* hist_tasks;    // [cap_hist_tasks]
  EvalNode* eval_nodes;    // [cap_split]
  // Split candidates per (rank, open node, feature chunk),
  // [nranks][cap_split][nchunks]; the decision takes the best in that order
  // (rank order and chunk order are feature order, so on equal gain the
  // lower feature stays).
  const SplitCand* cands;
  u32 nranks, nchunks;
  u32* split_idx;          // [cap_split]
  PartNode* part_nodes;    // [cap_split]
  PartTask* part_tasks;    // [cap_part_tasks]
  u32* cursors;            // [2 * cap_split]
  LeafRec* leaves;         // [cap_leaves]
  LeafTask* leaf_tasks;    // [cap_leaf_tasks]
  RoundCounters* ctr;
  LevelStats* stats;       // [max_depth + 1]
  u32* hist_counter;       // the histogram kernel's task queue; zeroed by k_hist_tasks
  u32* zero_list;          // [cap_split] slots whose sums are added by several tasks, or by none
  u32 K, maxn;
  // Which child of a split is built directly (the other is parent minus it):
  // the one with fewer rows, or, when rows are sharded (by_hess), the one
  // with the smaller hessian sum, which every rank knows without an exchange.
  // Ties go left.  The choice changes no result, only the work.
  u32 by_hess;
  u64 cap_split, cap_next, cap_hist_tasks, cap_part_tasks, cap_leaves, cap_leaf_tasks;
};

// Roots of the K trees; their totals come from gh_totals ([K][2], summed over
// all ranks).  Also zeroes the nstats level statistics.
void launch_round_init(const RoundBuffers& b, u64 R, const i64* gh_totals, u32 nstats, cudaStream_t s);
// Round start after the scales: tree k's (g, h) become int32 pairs
// (launch_quantize_gh), its row indices 0..R-1, and the quantised sums go to
// totals ([K][2]); with init set (one rank: no exchange of the totals) the
// launch then also does launch_round_init's work.  part holds
// quantize_round_blocks(R, K) * K * 2 int64; *done is zero at the first
// launch and every launch leaves it zero.
u32 quantize_round_blocks(u64 R, int K);
void launch_quantize_round(const RoundBuffers& b, float2* gh, u64 R, const Scales* scales, u32* ridx, i64* part,
                           u32* done, i64* totals, u32 nstats, bool init, cudaStream_t s);
// Histogram tasks of the build list, and the split-evaluation inputs of every
// open node.
// `tile` features per task (32, or 64 for the wide histogram kernel); ftiles
// tasks per row range; rows split into pieces of equal size for about
// target_tasks tasks in all (2048 rows at least).
void launch_hist_tasks(const RoundBuffers& b, u32 ftiles, u32 tile, int depth, u32 target_tasks, cudaStream_t s);
// Zeroes the slots k_hist_tasks listed (zero_list, n_zero): those of nodes
// cut into several pieces, whose tasks add their sums, and of nodes with no
// rows here, which no task writes; a node built by one task is stored whole.
// Slot s of group g starts at g * group_stride + s * slot_stride (groups = 1:
// group_stride unused) and holds slot_stride int64.
void launch_zero_listed(const RoundBuffers& b, i64* hist, u64 slot_stride, u64 group_stride, u32 groups,
                        cudaStream_t s);
// Splits (depth < max_depth, gain > 0) or closes every open node.
void launch_decide(const RoundBuffers& b, const float* cut, const u8* has_missing, u32 F, int depth, int max_depth,
                   int set, cudaStream_t s);
void launch_children(const RoundBuffers& b, int depth, int max_depth, cudaStream_t s);
// Column sampling of this level: for every open node, the features that may
// split it, as bits fmask[i * W + f / 32].  Nested exact-count selections
// (the candidates with the smallest sample_hash, ties to the lower feature):
// the tree keeps max(1, floor(c_tree F)) features (kind kSampleTree, index
// 0), the level that fraction c_level of the tree's (kSampleLevel, index
// depth), the node c_node of the level's (kSampleNode, index node id).  The
// round comes from *round_dev.  F must be at most 16384.
void launch_feature_masks(const RoundBuffers& b, u32 F, long long seed, const u32* round_dev, double c_tree,
                          double c_level, double c_node, int depth, u32* fmask, u32 W, cudaStream_t s);
// *round_dev += 1 (the end of a round).
void launch_bump_round(u32* round_dev, cudaStream_t s);
// ridx_sets[s] is the base of the K per-tree row-index arrays of set s
// (tree k at + k * R).  With split_leaves, also the leaf values of the
// children of this level's splits: into their node records and, as f32 bits,
// into cursors[2 s], cursors[2 s + 1] for launch_partition_leaves.
void launch_leaf_values(const RoundBuffers& b, const Scales* scales, SplitParams p, u32* const ridx_sets[2], u64 R,
                        cudaStream_t s, bool split_leaves = false);

}  // namespace dp
