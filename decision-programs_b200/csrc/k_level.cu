// Per-level bookkeeping kernels of a boosting round (see level.h).  They are
// tiny next to the histogram and partition passes; what they buy is that no
// count ever has to travel to the host inside a round.  The work lists they
// write (histogram, partition and margin-update tasks) are the ones the host
// used to build, in the same order.
#include "level.h"

namespace dp {

namespace {

constexpr int kBook = 1024;  // threads of the single-block bookkeeping kernels
constexpr i64 kLeafChunk = kLeafChunkRows;

// Exclusive block-wide scan (blockDim.x == kBook); *total gets the sum.
__device__ u64 scan_block(u64 v, u64* total) {
  __shared__ u64 ws[33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  u64 incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const u64 t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) ws[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const u64 w = ws[lane];
    u64 wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const u64 t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    ws[lane] = wi - w;
    if (lane == 31) ws[32] = wi;
  }
  __syncthreads();
  const u64 out = ws[warp] + incl - v;
  const u64 tot = ws[32];
  __syncthreads();
  *total = tot;
  return out;
}

// Expands a chunk of up to kBook items into tasks with the whole block: the
// calling thread's item owns `cnt` tasks; emit(j, q, t) runs once per task
// with j the owning thread, q the task's index within the item and t its
// global index base + (position in chunk), for t < cap only.  Returns the
// chunk's task count (all of them, including any past cap).
template <class Emit>
__device__ u64 expand(u64 cnt, u64 base, u64 cap, Emit emit) {
  __shared__ u64 s_off[kBook];
  u64 n = 0;
  s_off[threadIdx.x] = scan_block(cnt, &n);
  __syncthreads();
  for (u64 t = threadIdx.x; t < n; t += kBook) {
    int lo = 0, hi = kBook;  // s_off[lo] <= t < s_off[hi] (hi == kBook: past the end)
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_off[mid] <= t) lo = mid;
      else hi = mid;
    }
    if (base + t < cap) emit(lo, t - s_off[lo], base + t);
  }
  __syncthreads();
  return n;
}

__device__ __forceinline__ NodeRec& node_at(const RoundBuffers& b, u32 tree, u32 id) {
  return b.nodes[u64(id) * b.K + tree];
}

// One block: the K roots (open at depth 0, built directly), the counters and
// the level statistics of a new round.
__device__ void round_init_block(const RoundBuffers& b, u64 R, const i64* totals, u32 nstats) {
  for (u32 k = threadIdx.x; k < b.K; k += blockDim.x) {
    b.open_cur[k] = OpenRec{k, 0u, k, 0u, 0, i64(R)};
    b.build[k] = k;
    b.next_id[k] = 1u;
    node_at(b, k, 0) = NodeRec{totals[2 * k], totals[2 * k + 1], -1, -1, -1, -1, 0, 0, 0.f, 0.f};
  }
  for (u32 d = threadIdx.x; d < nstats; d += blockDim.x) b.stats[d] = LevelStats{};
  if (threadIdx.x == 0) {
    RoundCounters c{};
    c.n_open = b.K;
    c.n_build = b.K;
    *b.ctr = c;
  }
}

__global__ void k_round_init(RoundBuffers b, u64 R, const i64* __restrict__ totals, u32 nstats) {
  round_init_block(b, R, totals, nstats);
}

constexpr int kQuantThreads = 256;
constexpr u32 kQuantSharedSums = 128;  // classes x 2 reduced through shared memory by the last block

// grid (blocks, K); see launch_quantize_round.
__global__ void __launch_bounds__(kQuantThreads) k_quantize_round(RoundBuffers b, float2* gh, u64 R,
                                                                  const Scales* __restrict__ sc, u32* ridx, i64* part,
                                                                  u32* done, i64* totals, u32 nstats, int init) {
  const u32 k = blockIdx.y;
  const Scales s = sc[k];
  float2* g = gh + u64(k) * R;
  u32* rk = ridx + u64(k) * R;
  long long sg = 0, sh = 0;
  for (u64 i = u64(blockIdx.x) * blockDim.x + threadIdx.x; i < R; i += u64(gridDim.x) * blockDim.x) {
    const float2 v = g[i];
    const int2 q = make_int2(quantize(v.x, s.sg), quantize(v.y, s.sh));
    reinterpret_cast<int2*>(g)[i] = q;
    rk[i] = u32(i);
    sg += q.x;
    sh += q.y;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sg += __shfl_xor_sync(0xffffffffu, sg, o);
    sh += __shfl_xor_sync(0xffffffffu, sh, o);
  }
  __shared__ long long wg[kQuantThreads / 32], wh[kQuantThreads / 32];
  if (lane == 0) {
    wg[warp] = sg;
    wh[warp] = sh;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kQuantThreads / 32; ++w) {
      sg += wg[w];
      sh += wh[w];
    }
    // [K][2][blocks]: row 2k + c holds every block's sum of component c
    part[(2 * u64(k)) * gridDim.x + blockIdx.x] = sg;
    part[(2 * u64(k) + 1) * gridDim.x + blockIdx.x] = sh;
  }
  if (!last_block(done, gridDim.x * gridDim.y)) return;
  const u32 nk2 = b.K * 2;
  if (nk2 <= kQuantSharedSums) {
    __shared__ i64 s_red[(kQuantThreads / 32) * kQuantSharedSums];
    reduce_rows(part, nk2, gridDim.x, s_red, totals, i64(0), [](i64 x, i64 y) { return x + y; });
  } else {
    for (u32 kk = warp; kk < b.K; kk += kQuantThreads / 32) {
      long long a = 0, c = 0;
      const i64* pk = part + 2 * u64(kk) * gridDim.x;
      for (u32 j = lane; j < gridDim.x; j += 32) {
        a += __ldcg(pk + j);
        c += __ldcg(pk + gridDim.x + j);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        c += __shfl_xor_sync(0xffffffffu, c, o);
      }
      if (lane == 0) {
        totals[2 * kk] = a;
        totals[2 * kk + 1] = c;
      }
    }
  }
  if (!init) return;
  __syncthreads();  // the totals this block wrote
  round_init_block(b, R, totals, nstats);
}

// Pieces of a node of `count` rows: floor(count / chunk), at least one, so a
// node below two chunks stays one piece, which alone covers its histogram
// slot and stores it instead of adding to it (a partial piece's drain, 16384
// int64 reductions per 32-feature tile, costs about as much as its rows at
// a few thousand rows).
__device__ __forceinline__ u64 hist_pieces(i64 count, u64 chunk) {
  if (count <= 0) return 0;
  const u64 n = u64(count) / chunk;
  return n ? n : 1;
}

// Histogram tasks of the build list: about `target` tasks of equal row
// counts, the feature tiles of one row range adjacent in the queue so that
// blocks running at the same time read all sectors of the same rows.
__global__ void __launch_bounds__(kBook) k_hist_tasks(RoundBuffers b, u32 ftiles, u32 tile, u32 target, int depth) {
  __shared__ i64 s_begin[kBook], s_count[kBook];
  __shared__ u32 s_slot[kBook], s_tree[kBook];
  const u32 nb = b.ctr->n_build;
  if (threadIdx.x == 0) *b.hist_counter = 0u;  // the next histogram launch's queue
  u64 rows = 0, total = 0;
  for (u32 i = threadIdx.x; i < nb; i += kBook) rows += u64(b.open_cur[b.build[i]].count);
  scan_block(rows, &total);
  u64 chunk = (total * ftiles + target - 1) / target;
  if (chunk < 2048) chunk = 2048;
  u64 base = 0, zbase = 0;
  for (u32 c0 = 0; c0 < nb; c0 += kBook) {
    const u32 i = c0 + threadIdx.x;
    u64 pieces = 0;
    if (i < nb) {
      const OpenRec o = b.open_cur[b.build[i]];
      s_begin[threadIdx.x] = o.begin;
      s_count[threadIdx.x] = o.count;
      s_slot[threadIdx.x] = o.slot;
      s_tree[threadIdx.x] = o.tree;
      pieces = hist_pieces(o.count, chunk);
    }
    // slots that are not stored whole by one task are zeroed before the build
    u64 nz = 0;
    const u64 zpos = zbase + scan_block(i < nb && pieces != 1 ? 1 : 0, &nz);
    if (i < nb && pieces != 1) b.zero_list[zpos] = s_slot[threadIdx.x];
    zbase += nz;
    base += expand(pieces * ftiles, base, b.cap_hist_tasks, [&](int j, u64 q, u64 t) {
      const i64 cnt = s_count[j], beg0 = s_begin[j], end0 = beg0 + cnt;
      const i64 np = i64(hist_pieces(cnt, chunk));
      const i64 piece = (cnt + np - 1) / np;
      const i64 p = i64(q / ftiles);
      const u32 ft = u32(q % ftiles);
      const i64 beg = beg0 + p * piece < end0 ? beg0 + p * piece : end0;
      const i64 end = beg + piece < end0 ? beg + piece : end0;
      // a node covered by one row range is the only writer of its tiles
      b.hist_tasks[t] = HistTask{s_slot[j], ft * tile, s_tree[j], np == 1 ? 1u : 0u, beg, end};
    });
  }
  // split-evaluation inputs of the open nodes; a node in slot ns + j (the
  // larger sibling of triple j) is derived from its parent and slot j
  const u32 n_open = b.ctr->n_open, nt = b.ctr->n_triples;
  for (u32 i = threadIdx.x; i < n_open; i += kBook) {
    const OpenRec o = b.open_cur[i];
    const NodeRec& r = node_at(b, o.tree, o.id);
    u32 par = kNoSlot, small = 0;
    if (depth > 0 && o.slot >= nt && o.slot - nt < nt) {
      const u32 j = o.slot - nt;
      par = b.triples[3 * j];
      small = b.triples[3 * j + 1];
    }
    b.eval_nodes[i] = EvalNode{o.slot, o.tree, r.gq, r.hq, par, small};
  }
  if (threadIdx.x == 0) {
    if (base > b.cap_hist_tasks) b.ctr->overflow |= kOvfHistTasks;
    b.ctr->n_hist_tasks = u32(base < b.cap_hist_tasks ? base : b.cap_hist_tasks);
    b.ctr->n_zero = u32(zbase);
    b.stats[depth].rows_built = i64(total);
    b.stats[depth].n_build = nb;
    b.stats[depth].n_open = n_open;
  }
}

__global__ void k_zero_listed(const RoundCounters* __restrict__ ctr, const u32* __restrict__ list, i64* hist,
                              u64 slot_stride, u64 group_stride, u32 groups) {
  const u64 per = slot_stride / 2;  // 16-byte stores per slot and group
  const u64 n = u64(ctr->n_zero) * groups * per;
  longlong2* const h = reinterpret_cast<longlong2*>(hist);
  for (u64 k = u64(blockIdx.x) * blockDim.x + threadIdx.x; k < n; k += u64(gridDim.x) * blockDim.x) {
    const u64 e = k % per, sg = k / per;
    const u64 g = sg % groups, li = sg / groups;
    h[(g * group_stride + u64(list[li]) * slot_stride) / 2 + e] = make_longlong2(0, 0);
  }
}

// Splits or closes every open node, in open-list order (trees contiguous,
// node ids ascending).  Child ids follow creation order within each tree: the
// split of rank r in its tree gets left = next_id + 2r, right = left + 1.
__global__ void __launch_bounds__(kBook) k_decide(RoundBuffers b, const float* __restrict__ cut,
                                                  const u8* __restrict__ has_missing, u32 F, int depth,
                                                  int max_depth, int set) {
  __shared__ i64 s_begin[kBook], s_end[kBook];
  __shared__ u32 s_rank[kBook];
  const u32 n_open = b.ctr->n_open;
  u64 split_base = 0, part_base = 0;
  u64 leaf_base = b.ctr->n_leaves;
  for (u32 c0 = 0; c0 < n_open; c0 += kBook) {
    const u32 i = c0 + threadIdx.x;
    const bool valid = i < n_open;
    OpenRec o{};
    SplitCand bs{};
    bs.feature = -1;
    if (valid) {
      o = b.open_cur[i];
      if (depth < max_depth) {
        // the first maximum over (rank, chunk) in that order: gains are read
        // eight at a time with independent loads, then the winner whole
        const u32 nk = b.nranks * b.nchunks;
        u32 best_k = 0;
        double best_g = 0.0;
        for (u32 k0 = 0; k0 < nk; k0 += 8) {
          double g[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const u32 k = k0 + u, r = k / b.nchunks, c = k - r * b.nchunks;
            g[u] = k < nk ? b.cands[(u64(r) * b.cap_split + i) * b.nchunks + c].gain : 0.0;
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const u32 k = k0 + u;
            if (k < nk && (k == 0 || g[u] > best_g)) {
              best_g = g[u];
              best_k = k;
            }
          }
        }
        const u32 r = best_k / b.nchunks, c = best_k - r * b.nchunks;
        bs = b.cands[(u64(r) * b.cap_split + i) * b.nchunks + c];
      }
    }
    // a candidate that came through the exchange names a feature and bin
    // inside the matrix; anything else (an exchange that was aborted part way)
    // is reported instead of indexing the cut table with it
    const bool in_range = bs.feature >= 0 && u32(bs.feature) < F && bs.bin >= 0 && bs.bin < i32(kMaxBins);
    if (valid && depth < max_depth && bs.gain > 0.0 && bs.feature >= 0 && !in_range)
      atomicOr(&b.ctr->overflow, kOvfBadCand);
    const bool split = valid && depth < max_depth && in_range && bs.gain > 0.0;
    const bool leaf = valid && !split;
    // what a split reads (the node's totals, the threshold, the feature's
    // missing flag), loaded before the block scans so that the loads' latency
    // overlaps the barriers
    i64 node_gq = 0, node_hq = 0;
    float cond = 0.f;
    i32 missing_is_bin = 0;
    if (split) {
      const NodeRec& p0 = node_at(b, o.tree, o.id);
      node_gq = p0.gq;
      node_hq = p0.hq;
      cond = cut[u64(bs.feature) * kMaxBins + bs.bin];
      missing_is_bin = i32(has_missing[bs.feature]);
    }
    u64 ns = 0, nl = 0;
    const u64 rs = split_base + scan_block(split ? 1 : 0, &ns);
    const u64 rl = leaf_base + scan_block(leaf ? 1 : 0, &nl);
    const bool first_of_tree = valid && (i == 0 || b.open_cur[i - 1].tree != o.tree);
    const bool last_of_tree = valid && (i + 1 == n_open || b.open_cur[i + 1].tree != o.tree);
    if (first_of_tree) b.tree_first[o.tree] = u32(rs);
    __syncthreads();
    bool ok = false;
    if (split) {
      const u32 rank = u32(rs) - b.tree_first[o.tree];
      const u32 lid = b.next_id[o.tree] + 2 * rank, rid = lid + 1;
      ok = rid < b.maxn && rs < b.cap_split;
      if (ok) {
        NodeRec& p = node_at(b, o.tree, o.id);
        p.left = i32(lid);
        p.right = i32(rid);
        p.feature = bs.feature;
        p.bin = bs.bin;
        p.default_left = bs.default_left;
        p.cond = cond;
        p.gain = float(bs.gain);
        node_at(b, o.tree, lid) = NodeRec{bs.gl, bs.hl, -1, -1, i32(o.id), -1, 0, 0, 0.f, 0.f};
        node_at(b, o.tree, rid) = NodeRec{node_gq - bs.gl, node_hq - bs.hl, -1, -1, i32(o.id), -1, 0, 0, 0.f, 0.f};
        b.part_nodes[rs] = PartNode{o.tree, bs.feature, bs.bin, bs.default_left, missing_is_bin, 0, o.begin,
                                    o.begin + o.count};
        b.split_idx[rs] = i;
        b.cursors[2 * rs] = 0u;
        b.cursors[2 * rs + 1] = 0u;
      } else {
        atomicOr(&b.ctr->overflow, kOvfNodes);
      }
    }
    if (leaf) {
      if (rl < b.cap_leaves) b.leaves[rl] = LeafRec{o.tree, o.id, u32(set), 0u, o.begin, o.count};
      else atomicOr(&b.ctr->overflow, kOvfLeaves);
    }
    s_begin[threadIdx.x] = o.begin;
    s_end[threadIdx.x] = o.begin + o.count;
    s_rank[threadIdx.x] = u32(rs);
    __syncthreads();  // every node of this chunk has read next_id
    if (last_of_tree) b.next_id[o.tree] += 2u * (u32(rs) + (split ? 1u : 0u) - b.tree_first[o.tree]);
    const u64 ptasks = (ok && o.count > 0) ? (u64(o.count) + kPartChunk - 1) / kPartChunk : 0;
    part_base += expand(ptasks, part_base, b.cap_part_tasks, [&](int j, u64 q, u64 t) {
      const i64 beg = s_begin[j] + i64(q) * kPartChunk;
      const i64 end = beg + kPartChunk < s_end[j] ? beg + kPartChunk : s_end[j];
      b.part_tasks[t] = PartTask{s_rank[j], 0u, beg, end};
    });
    split_base += ns;
    leaf_base += nl;
  }
  if (threadIdx.x == 0) {
    b.ctr->n_split = u32(split_base < b.cap_split ? split_base : b.cap_split);
    b.ctr->n_part_tasks = u32(part_base < b.cap_part_tasks ? part_base : b.cap_part_tasks);
    if (part_base > b.cap_part_tasks) b.ctr->overflow |= kOvfPartTasks;
    b.ctr->n_leaves = u32(leaf_base < b.cap_leaves ? leaf_base : b.cap_leaves);
  }
}

// Children of every split node become the next level's open list (see
// RoundBuffers::by_hess for which child is built directly).  Block 0 also
// sets the next level's counts.
__global__ void k_children(RoundBuffers b, int depth, int max_depth) {
  const u32 ns = b.ctr->n_split;
  const bool more = depth + 1 < max_depth;
  const bool fits = 2 * u64(ns) <= b.cap_next;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    b.ctr->n_open = fits ? 2 * ns : 0u;
    b.ctr->n_build = (more && fits) ? ns : 0u;
    b.ctr->n_triples = (more && fits) ? ns : 0u;
    if (!fits) atomicOr(&b.ctr->overflow, kOvfOpen);
  }
  if (!fits) return;
  for (u32 j = blockIdx.x * blockDim.x + threadIdx.x; j < ns; j += gridDim.x * blockDim.x) {
    const OpenRec o = b.open_cur[b.split_idx[j]];
    const NodeRec& p = node_at(b, o.tree, o.id);
    const i64 nleft = i64(b.cursors[2 * j]), nright = i64(b.cursors[2 * j + 1]);
    if (nleft + nright != o.count) atomicOr(&b.ctr->overflow, kOvfLostRows);
    const bool right_small = b.by_hess ? node_at(b, o.tree, u32(p.right)).hq < node_at(b, o.tree, u32(p.left)).hq
                                       : nright < nleft;
    const u32 lslot = right_small ? ns + j : j, rslot = right_small ? j : ns + j;
    b.open_next[2 * j] = OpenRec{o.tree, u32(p.left), lslot, 0u, o.begin, nleft};
    b.open_next[2 * j + 1] = OpenRec{o.tree, u32(p.right), rslot, 0u, o.begin + nleft, o.count - nleft};
    if (more) {
      b.build_next[j] = right_small ? 2 * j + 1 : 2 * j;
      b.triples_next[3 * j] = o.slot;
      b.triples_next[3 * j + 1] = j;
      b.triples_next[3 * j + 2] = ns + j;
    }
  }
}

// Leaf values into the node records, then the margin-update tasks (chunks of
// up to kLeafChunk rows of each leaf segment).  With split_leaves, the
// children of this level's splits are leaves as well (the last level, whose
// rows do not move): their values go into their records and, as f32 bits, to
// cursors[2 s] (left) and cursors[2 s + 1] (right) of split s.
__global__ void __launch_bounds__(kBook) k_leaf_values(RoundBuffers b, const Scales* __restrict__ scales,
                                                       SplitParams p, const u32* ridx0, const u32* ridx1, u64 R,
                                                       int split_leaves) {
  if (split_leaves) {
    const u32 ns = b.ctr->n_split;
    for (u32 j = threadIdx.x; j < ns; j += kBook) {
      const OpenRec o = b.open_cur[b.split_idx[j]];
      const NodeRec& par = node_at(b, o.tree, o.id);
      const Scales sc = scales[o.tree];
      const i32 child[2] = {par.left, par.right};
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        NodeRec& n = node_at(b, o.tree, u32(child[c]));
        const float v = leaf_weight(n.gq, n.hq, sc.sg, sc.sh, p);
        n.cond = v;
        n.feature = 0;
        b.cursors[2 * j + c] = __float_as_uint(v);
      }
    }
  }
  __shared__ i64 s_begin[kBook], s_end[kBook];
  __shared__ const u32* s_ridx[kBook];
  __shared__ float s_value[kBook];
  __shared__ u32 s_tree[kBook];
  const u32 nl = b.ctr->n_leaves;
  u64 base = 0;
  for (u32 c0 = 0; c0 < nl; c0 += kBook) {
    const u32 i = c0 + threadIdx.x;
    u64 chunks = 0;
    if (i < nl) {
      const LeafRec l = b.leaves[i];
      NodeRec& n = node_at(b, l.tree, l.id);
      const Scales sc = scales[l.tree];
      const float v = leaf_weight(n.gq, n.hq, sc.sg, sc.sh, p);
      n.cond = v;
      n.feature = 0;
      s_begin[threadIdx.x] = l.begin;
      s_end[threadIdx.x] = l.begin + l.count;
      s_ridx[threadIdx.x] = (l.set ? ridx1 : ridx0) + u64(l.tree) * R;
      s_value[threadIdx.x] = v;
      s_tree[threadIdx.x] = l.tree;
      chunks = l.count > 0 ? (u64(l.count) + kLeafChunk - 1) / kLeafChunk : 0;
    }
    base += expand(chunks, base, b.cap_leaf_tasks, [&](int j, u64 q, u64 t) {
      const i64 beg = s_begin[j] + i64(q) * kLeafChunk;
      const i64 end = beg + kLeafChunk < s_end[j] ? beg + kLeafChunk : s_end[j];
      b.leaf_tasks[t] = LeafTask{s_ridx[j], beg, end, s_value[j], s_tree[j]};
    });
  }
  if (threadIdx.x == 0) {
    if (base > b.cap_leaf_tasks) b.ctr->overflow |= kOvfLeafTasks;
    b.ctr->n_leaf_tasks = u32(base < b.cap_leaf_tasks ? base : b.cap_leaf_tasks);
  }
}

constexpr u32 kMaskThreads = 256;

// One block per open node (grid-stride); shared: the hash of every feature
// and two membership flags per feature.
__global__ void __launch_bounds__(kMaskThreads) k_feature_masks(RoundBuffers b, u32 F, long long seed,
                                                                const u32* __restrict__ round_dev, double c_tree,
                                                                double c_level, double c_node, int depth,
                                                                u32* __restrict__ fmask, u32 W) {
  extern __shared__ __align__(8) unsigned char msm[];
  u64* key = reinterpret_cast<u64*>(msm);
  u8* in = msm + 8 * u64(F);
  u8* keep = in + F;
  __shared__ u32 s_count;
  const u32 n_open = b.ctr->n_open;
  const u32 round = *round_dev;
  for (u32 i = blockIdx.x; i < n_open; i += gridDim.x) {
    const OpenRec o = b.open_cur[i];
    for (u32 f = threadIdx.x; f < F; f += kMaskThreads) in[f] = 1;
    // one nested selection: the `c` fraction of the current set with the
    // smallest (hash, feature)
    auto select = [&](double c, u32 kind, u64 index) {
      if (c >= 1.0) return;
      if (threadIdx.x == 0) s_count = 0;
      __syncthreads();
      u32 mine = 0;
      for (u32 f = threadIdx.x; f < F; f += kMaskThreads) {
        key[f] = sample_hash(seed, round, o.tree, kind, f, index);
        mine += in[f];
      }
      atomicAdd(&s_count, mine);
      __syncthreads();
      const u32 want = sample_count(c, s_count);
      for (u32 f = threadIdx.x; f < F; f += kMaskThreads) {
        u32 rank = 0;
        if (in[f]) {
          const u64 kf = key[f];
          for (u32 g = 0; g < F; ++g) rank += (in[g] && (key[g] < kf || (key[g] == kf && g < f))) ? 1u : 0u;
        }
        keep[f] = in[f] && rank < want;
      }
      __syncthreads();
      for (u32 f = threadIdx.x; f < F; f += kMaskThreads) in[f] = keep[f];
      __syncthreads();
    };
    __syncthreads();
    select(c_tree, kSampleTree, 0);
    select(c_level, kSampleLevel, u64(depth));
    select(c_node, kSampleNode, u64(o.id));
    for (u32 w = threadIdx.x; w < W; w += kMaskThreads) {
      u32 bits = 0;
      for (u32 j = 0; j < 32; ++j) {
        const u32 f = w * 32 + j;
        if (f < F && in[f]) bits |= 1u << j;
      }
      fmask[u64(i) * W + w] = bits;
    }
    __syncthreads();
  }
}

__global__ void k_bump_round(u32* round_dev) { *round_dev += 1u; }

int sm_count() {
  int dev = 0, sms = 148;
  DP_CUDA(cudaGetDevice(&dev));
  DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  return sms;
}

}  // namespace

void launch_round_init(const RoundBuffers& b, u64 R, const i64* gh_totals, u32 nstats, cudaStream_t s) {
  k_round_init<<<1, 256, 0, s>>>(b, R, gh_totals, nstats);
  after_launch("round_init");
}

u32 quantize_round_blocks(u64 R, int K) {
  const u64 cap = (u64(sm_count()) * 8 + u64(K) - 1) / u64(K);  // about eight blocks per SM in all
  const u64 want = (R + kQuantThreads - 1) / kQuantThreads;
  const u64 n = want < cap ? want : cap;
  return u32(n ? n : 1);
}

void launch_quantize_round(const RoundBuffers& b, float2* gh, u64 R, const Scales* scales, u32* ridx, i64* part,
                           u32* done, i64* totals, u32 nstats, bool init, cudaStream_t s) {
  need(b.K <= 65535u, "internal error: class count exceeds the grid");
  const dim3 grid(quantize_round_blocks(R, int(b.K)), b.K);
  k_quantize_round<<<grid, kQuantThreads, 0, s>>>(b, gh, R, scales, ridx, part, done, totals, nstats, init ? 1 : 0);
  after_launch("quantize_round");
}

void launch_hist_tasks(const RoundBuffers& b, u32 ftiles, u32 tile, int depth, u32 target_tasks, cudaStream_t s) {
  k_hist_tasks<<<1, kBook, 0, s>>>(b, ftiles, tile, target_tasks ? target_tasks : 1u, depth);
  after_launch("hist_tasks");
}

void launch_zero_listed(const RoundBuffers& b, i64* hist, u64 slot_stride, u64 group_stride, u32 groups,
                        cudaStream_t s) {
  need(slot_stride % 2 == 0 && (groups <= 1 || group_stride % 2 == 0), "internal error: slot strides");
  k_zero_listed<<<sm_count() * 4, 256, 0, s>>>(b.ctr, b.zero_list, hist, slot_stride, groups > 1 ? group_stride : 0,
                                               groups ? groups : 1);
  after_launch("zero_listed");
}

void launch_decide(const RoundBuffers& b, const float* cut, const u8* has_missing, u32 F, int depth, int max_depth,
                   int set, cudaStream_t s) {
  k_decide<<<1, kBook, 0, s>>>(b, cut, has_missing, F, depth, max_depth, set);
  after_launch("decide");
}

void launch_children(const RoundBuffers& b, int depth, int max_depth, cudaStream_t s) {
  k_children<<<sm_count(), 256, 0, s>>>(b, depth, max_depth);
  after_launch("children");
}

void launch_leaf_values(const RoundBuffers& b, const Scales* scales, SplitParams p, u32* const ridx_sets[2], u64 R,
                        cudaStream_t s, bool split_leaves) {
  k_leaf_values<<<1, kBook, 0, s>>>(b, scales, p, ridx_sets[0], ridx_sets[1], R, split_leaves ? 1 : 0);
  after_launch("leaf_values");
}

void launch_feature_masks(const RoundBuffers& b, u32 F, long long seed, const u32* round_dev, double c_tree,
                          double c_level, double c_node, int depth, u32* fmask, u32 W, cudaStream_t s) {
  need(F <= 16384, "column sampling supports at most 16384 features");
  const size_t smem = 10 * size_t(F);
  static thread_local int configured_device = -1;
  int dev = 0;
  DP_CUDA(cudaGetDevice(&dev));
  if (configured_device != dev) {
    DP_CUDA(cudaFuncSetAttribute(k_feature_masks, cudaFuncAttributeMaxDynamicSharedMemorySize, 10 * 16384));
    configured_device = dev;
  }
  const u32 blocks = u32(b.cap_split < 4096 ? (b.cap_split ? b.cap_split : 1) : 4096);
  k_feature_masks<<<blocks, kMaskThreads, smem, s>>>(b, F, seed, round_dev, c_tree, c_level, c_node, depth, fmask,
                                                     W);
  after_launch("feature_masks");
}

void launch_bump_round(u32* round_dev, cudaStream_t s) {
  k_bump_round<<<1, 1, 0, s>>>(round_dev);
  after_launch("bump_round");
}

}  // namespace dp
