// Histogram build: for every task (node slot, 32-feature tile, a range of the
// node's row positions) accumulate the quantised (g, h) of each row into
// hist[slot][f][bin] (int64 pairs).
//
// Design (HBM- and shared-atomic-bound, no tensor cores):
//  * persistent blocks (one 1024-thread block per SM for 256 bins) pull tasks
//    from an atomic counter; consecutive tasks of the same (node, tile) keep
//    accumulating, so a block drains to global memory only when the node or
//    tile changes and the tail of the launch stays balanced;
//  * two u32 planes in shared memory, g and h, laid out [bin][column]: one
//    32-bit shared atomic per (row, feature) and plane.  The quantiser bounds
//    keep the sums of a kWindowRows window inside int32 / uint32, so every
//    window is folded into int64 planes in shared memory; the final drain uses
//    64-bit global atomics (integer: the result does not depend on order);
//  * a warp reads 16 rows x 32 features per step with 16-byte loads: lane
//    (s, h) holds bytes 16h..16h+15 of row s, rotated by s bytes once, so that
//    in atomic step j it updates feature 16h + ((j + s) & 15).  The 32 lanes
//    of a step then address 32 distinct feature columns -- 32 distinct banks
//    of the [bin][feature] planes whatever the bins are -- while every byte
//    extraction uses a compile-time position;
//  * rows are gathered through the node's row-index segment; (g, h) is read
//    in position order, already quantised to int32 pairs by the training
//    engine (the kernel-level entry point may pass fp32 pairs instead).
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "hist_update.cuh"
#include "tmem.cuh"
#include "kernels.h"

namespace dp {

namespace {

constexpr int kFT = kHistFeatureTile;  // 32 features per tile
constexpr int kRPW = 16;               // rows per warp step (two lanes per row)
// Row steps in flight per warp, measured on B200: 4 for the 32-feature
// 256-bin kernel (config 5, 100M x 32, 1 / 8 / 1024 nodes: 1.19 / 1.89 /
// 2.15 ms against 1.20 / 1.98 / 2.28 with 6 and 1.22 / 2.01 / 2.31 with 8);
// 4 for the 64-feature kernel (config 4: 2.79 ms of histograms per round
// against 2.81 with 6, with half the register-spill traffic around its
// folds); 4 for the 512-thread 64-bin kernel.
#ifndef DP_HIST_UNROLL
#define DP_HIST_UNROLL 4
#endif
#ifndef DP_HIST_WIDE_UNROLL
#define DP_HIST_WIDE_UNROLL 4
#endif
#ifndef DP_HIST_THREADS
#define DP_HIST_THREADS 1024
#endif
template <int MB>
__host__ __device__ constexpr int unroll_for() { return MB >= 256 ? DP_HIST_UNROLL : 4; }
constexpr u32 kNoRow = 0xffffffffu;

struct HistArgs {
  const u8* bins;
  u64 bstride;
  u32 F;
  u32 ntasks;
  const u32* ntasks_dev;  // when set, the task count is read from device memory
  const TreeArrays* trees;
  const Scales* scales;
  const HistTask* tasks;
  u32* counter;
  i64* hist;
  HistLayout layout;
};

// 16 bytes of a row's bin codes.  With `line` the load also asks L2 to fetch
// the whole 128-byte line: when rows are whole lines (row stride a multiple
// of 128 bytes) the line holds this row's other feature tiles, which the
// tasks of the same piece (queued next to this one) read at about the same
// time, so DRAM serves one line instead of four separate 32-byte sectors.
__device__ __forceinline__ uint4 load_codes(const u8* p, bool line) {
#ifndef DP_HIST_NO_LINE_FETCH
  if (line) {
    uint4 v;
    asm volatile("ld.global.nc.L2::128B.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
  }
#endif
  return __ldg(reinterpret_cast<const uint4*>(p));
}

template <bool QUANT>
__device__ __forceinline__ void load_q(const TreeArrays& ta, const Scales& sc, u32 i, u32& gq, u32& hq) {
  if (QUANT) {
    const int2 v = __ldg(reinterpret_cast<const int2*>(ta.gh) + i);
    gq = u32(v.x);
    hq = u32(v.y);
  } else {
    const float2 v = __ldg(ta.gh + i);
    gq = u32(quantize(v.x, sc.sg));
    hq = u32(quantize(v.y, sc.sh));
  }
}

// Window sums of the 32-feature kernel in tensor memory: TMEM lane 32 q + t
// holds feature t of the tile for the MB / 4 bins MB / 4 q .. (lane quarter
// q), bin b' of those in columns 4 b' .. 4 b' + 3 (g low and high word, h low
// and high word).  Warp w serves lane quarter w % 4 and NBW = MB / warps of
// its bins.
template <u32 MB, u32 NBW>
struct TilePart {
  u32 bin0, col;
  __device__ __forceinline__ explicit TilePart(u32 tmem_base) {
    const u32 w = threadIdx.x >> 5, tq = w & 3u;
    bin0 = tq * (MB / 4u) + (w >> 2) * NBW;
    col = tmem_at(tmem_base, 32u * tq, 4u * (w >> 2) * NBW);
  }
};

// The window's u32 sums of this warp's cells (planes [bin][32], the h plane
// hoff words after the g plane) into the int64 sums in TMEM; `clean`: the
// key's first fold, which copies; `clear`: zero the planes.  Out of line, as
// the 64-feature kernel's fold.
template <u32 MB, u32 NBW>
__device__ __noinline__ void tile_fold(u32* Lg, u32 hoff, u32 tmem_base, bool clean, bool clear) {
  const TilePart<MB, NBW> tp(tmem_base);
  const u32 t = threadIdx.x & 31u;
#pragma unroll 1
  for (u32 i = 0; i < NBW; ++i) {
    u32 r[4];
    if (!clean) tmem_ld4(tp.col + 4u * i, r);
    const u32 cell = (tp.bin0 + i) * 32u + t;
    const u32 g = Lg[cell], h = Lg[cell + hoff];
    if (clear) {
      Lg[cell] = 0u;
      Lg[cell + hoff] = 0u;
    }
    if (!clean) {
      tmem_wait_ld();
    } else {
      r[0] = r[1] = r[2] = r[3] = 0u;
    }
    const u64 G = ((u64(r[1]) << 32) | r[0]) + u64(i64(int(g)));
    const u64 H = ((u64(r[3]) << 32) | r[2]) + u64(h);
    r[0] = u32(G);
    r[1] = u32(G >> 32);
    r[2] = u32(H);
    r[3] = u32(H >> 32);
    tmem_st4(tp.col + 4u * i, r);
  }
  tmem_wait_st();
}

// shared memory of the 32-feature kernel: the u32 planes, or in the drain
// the [feature][bin] int64 pairs staged over them
// (256 bins: the window sums in tensor memory); with 64 bins the u32 planes
// and after them int64 planes [feature][bin + 1] of the window sums, which
// for this small kernel cost less than the tensor-memory fold (config 5, 64
// bins, 8 nodes: 1.63 against 1.87 ms)
template <int MB>
constexpr int hist_smem() {
  constexpr int rows = MB < 256 ? MB + 1 : 256;
  constexpr int planes = rows * kHistFeatureTile * 8;
  constexpr int stage = kHistFeatureTile * MB * 16;
  constexpr int wplanes = kHistFeatureTile * (MB + 1) * 16;
  return int(kPlaneAlignPad) + (MB == 256 ? (planes > stage ? planes : stage) : planes + wplanes);
}

template <int MB, int THREADS, bool QUANT>
__global__ void __launch_bounds__(THREADS, THREADS <= 512 ? 2 : 1) k_hist(HistArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ u32 s_task;
  static_assert(unroll_for<MB>() % 2 == 0, "the two lanes of a row slot split the prefetch");
  // Row-index prefetch through shared memory (the 64-bin kernel, measured
  // 10-15% faster with it); the 256-bin kernel keeps direct loads: its planes
  // already fill most of shared memory, and with the stage it ran slower.
  constexpr bool kPrefetch = MB < 256;
  // per warp, two stages of the row indices of one iteration
  __shared__ u32 s_rows[kPrefetch ? (THREADS / 32) * 2 * unroll_for<MB>() * kRPW : 1];
  // u32 planes [bin][feature]: all 256 bin rows for MB = 256; for MB < 256
  // one more row, which takes the updates of codes >= MB (clamped to MB) and
  // is never folded
  constexpr int kRows = MB < 256 ? MB + 1 : 256;
  constexpr u32 kHOff = u32(kRows) * kFT * 4;  // h plane offset in bytes
  constexpr int kPlaneCells = kRows * kFT;
  constexpr int kCells = MB * kFT;
  constexpr int kWarps = THREADS / 32;
  constexpr u32 kStep = u32(kWarps) * kRPW;
  constexpr int kUnroll = unroll_for<MB>();
  constexpr u32 kNBW = u32(MB) / u32(kWarps);               // bins of the window sums per warp
  constexpr u32 kTmemCols = u32(MB);                         // 4 columns x MB / 4 bins per lane
  static_assert(kNBW * u32(kWarps) == u32(MB) && kWarps % 4 == 0, "bins split evenly over the warps");
  // bits of a code word that are set only by codes >= MB (MB = 64)
  constexpr u32 kHighBits = MB == 64 ? 0xc0c0c0c0u : 0u;
  static_assert(MB == 64 || MB == 256, "64- or 256-bin planes");
  constexpr bool kTmem = MB == 256;  // window sums in tensor memory, else in shared int64 planes
  constexpr int kWRow = MB + 1;      // int64 planes [feature][bin], rows padded
  constexpr int kWCells = kFT * kWRow;
  __shared__ u32 s_tmem;
  u32* Lg = reinterpret_cast<u32*>(smem + plane_pad(smem));
  u32* Lh = Lg + kPlaneCells;
  long long* Wg = reinterpret_cast<long long*>(Lh + kPlaneCells);  // (64 bins only)
  long long* Wh = Wg + kWCells;
  for (int i = threadIdx.x; i < kPlaneCells; i += THREADS) {
    Lg[i] = 0u;
    Lh[i] = 0u;
  }
  if constexpr (kTmem) {
    if (threadIdx.x < 32) tmem_alloc(&s_tmem, kTmemCols);
    tmem_fence_before_sync();
    __syncthreads();
    tmem_fence_after_sync();
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const u32 s = u32(lane) >> 1, h16 = u32(lane & 1) * 16u;  // row slot, feature half
  // atomic step j updates feature 16h + (j ^ s) of the tile; the planes start
  // below 2^16 in the shared window (the system's reserved bytes and this
  // kernel's static variables come first)
  const LaneCols cols = lane_cols(smem_addr(Lg), h16, s);
  u32 key_slot = kNoRow, key_f0 = 0, key_tree = 0;  // current accumulation target (block-uniform)
  bool key_excl = false;  // the key's task is the only one writing its (slot, tile)
  u32 in_window = 0;                                // rows in the u32 planes since the last fold
  const u32 ntasks = a.ntasks_dev ? *a.ntasks_dev : a.ntasks;

  bool t_clean = true;  // the window sums hold nothing of the current key (block-uniform)
  // 64 bins: the window into the int64 planes (transposed to [feature][bin]),
  // the window cleared; the key's first fold copies
  auto wfold = [&]() {
    for (int i = threadIdx.x; i < kCells; i += THREADS) {
      const int b = i / kFT, f = i % kFT;
      const long long g = static_cast<long long>(static_cast<int>(Lg[i])), h = static_cast<long long>(Lh[i]);
      Wg[f * kWRow + b] = t_clean ? g : Wg[f * kWRow + b] + g;
      Wh[f * kWRow + b] = t_clean ? h : Wh[f * kWRow + b] + h;
      Lg[i] = 0u;
      Lh[i] = 0u;
    }
    t_clean = false;
  };

  for (;;) {
    if (threadIdx.x == 0) s_task = atomicAdd(a.counter, 1u);
    __syncthreads();  // also: every warp has finished the previous task
    const u32 ti = s_task;
    const bool done = ti >= ntasks;
    HistTask t{};
    if (!done) t = a.tasks[ti];
    const bool same = !done && t.slot == key_slot && t.f0 == key_f0 && t.tree == key_tree;
    if (!same && key_slot != kNoRow && !kTmem) {
      wfold();
      __syncthreads();
      // consecutive threads take consecutive bins of one feature
      i64* out = a.hist + u64(key_slot) * a.layout.slot_stride;
      if (key_excl) {
        for (int idx = threadIdx.x; idx < kCells; idx += THREADS) {
          const int f = idx / MB, b = idx % MB;
          const u32 gf = key_f0 + u32(f);
          if (gf >= a.F) continue;
          const u32 grp = gf / a.layout.fg, fl = gf - grp * a.layout.fg;
          i64* cell = out + grp * a.layout.group_stride + (u64(fl) * kMaxBins + b) * 2;
          *reinterpret_cast<longlong2*>(cell) = make_longlong2(Wg[f * kWRow + b], Wh[f * kWRow + b]);
        }
      } else {
        // g and h of a cell on neighbouring lanes: a warp's 32 reductions
        // cover 16 whole cells, eight 32-byte sectors
        for (int idx = threadIdx.x; idx < 2 * kCells; idx += THREADS) {
          const int c = idx >> 1, comp = idx & 1;
          const int f = c / MB, b = c % MB;
          const u32 gf = key_f0 + u32(f);
          if (gf >= a.F) continue;
          const long long v = comp ? Wh[f * kWRow + b] : Wg[f * kWRow + b];
          const u32 grp = gf / a.layout.fg, fl = gf - grp * a.layout.fg;
          i64* cell = out + grp * a.layout.group_stride + (u64(fl) * kMaxBins + b) * 2 + comp;
          if (v) atomicAdd(reinterpret_cast<unsigned long long*>(cell), static_cast<unsigned long long>(v));
        }
      }
      t_clean = true;
      key_slot = kNoRow;
      in_window = 0;
    }
    if (!same && key_slot != kNoRow && kTmem) {
      tile_fold<u32(MB), kNBW>(Lg, u32(kPlaneCells), s_tmem, t_clean, false);  // the last window joins the sums
      t_clean = false;
      __syncthreads();  // the planes are read: they become the staging area
      // [feature][bin] int64 pairs, bin index XOR feature (four wavefronts
      // per warp both when a warp writes a bin of 32 features and when it
      // reads 32 bins of one feature)
      longlong2* T = reinterpret_cast<longlong2*>(Lg);
      {
        const TilePart<u32(MB), kNBW> tp(s_tmem);
        const u32 t = u32(lane);
#pragma unroll 1
        for (u32 i = 0; i < kNBW; ++i) {
          u32 r[4];
          tmem_ld4(tp.col + 4u * i, r);
          tmem_wait_ld();
          const u32 b = tp.bin0 + i;
          T[t * u32(MB) + (b ^ t)] = make_longlong2(static_cast<long long>((u64(r[1]) << 32) | r[0]),
                                                     static_cast<long long>((u64(r[3]) << 32) | r[2]));
        }
      }
      __syncthreads();
      // consecutive threads take consecutive bins of one feature: a warp
      // covers one contiguous 512-byte run.  A task that alone covers its
      // (slot, tile) stores every cell (16-byte stores, no read of the line);
      // otherwise non-zero cells are added with 64-bit reductions.
      i64* out = a.hist + u64(key_slot) * a.layout.slot_stride;
      if (key_excl) {
        for (int idx = threadIdx.x; idx < kCells; idx += THREADS) {
          const u32 f = u32(idx) / u32(MB), b = u32(idx) % u32(MB);
          const u32 gf = key_f0 + f;
          if (gf >= a.F) continue;
          const u32 grp = gf / a.layout.fg, fl = gf - grp * a.layout.fg;
          i64* cell = out + grp * a.layout.group_stride + (u64(fl) * kMaxBins + b) * 2;
          *reinterpret_cast<longlong2*>(cell) = T[f * u32(MB) + (b ^ f)];
        }
      } else {
        // g and h of a cell on neighbouring lanes: a warp's 32 reductions
        // cover 16 whole cells, eight 32-byte sectors
        const long long* T64 = reinterpret_cast<const long long*>(T);
        for (int idx = threadIdx.x; idx < 2 * kCells; idx += THREADS) {
          const u32 c = u32(idx) >> 1, comp = u32(idx) & 1u;
          const u32 f = c / u32(MB), b = c % u32(MB);
          const u32 gf = key_f0 + f;
          if (gf >= a.F) continue;
          const long long v = T64[2u * (f * u32(MB) + (b ^ f)) + comp];
          const u32 grp = gf / a.layout.fg, fl = gf - grp * a.layout.fg;
          i64* cell = out + grp * a.layout.group_stride + (u64(fl) * kMaxBins + b) * 2 + comp;
          if (v) atomicAdd(reinterpret_cast<unsigned long long*>(cell), static_cast<unsigned long long>(v));
        }
      }
      __syncthreads();  // the staging area is read before it is cleared
      for (int i = threadIdx.x; i < kPlaneCells; i += THREADS) {
        Lg[i] = 0u;
        Lh[i] = 0u;
      }
      t_clean = true;
      key_slot = kNoRow;
      in_window = 0;
    }
    if (done) break;
    __syncthreads();  // s_task is read by all before thread 0 rewrites it
    key_slot = t.slot;
    key_f0 = t.f0;
    key_tree = t.tree;
    key_excl = t.excl != 0;
    const TreeArrays ta = a.trees[t.tree];
    Scales sc{1.f, 1.f};
    if (!QUANT) sc = a.scales[t.tree];
    // halves past the row's bin_stride (last tile of a row) are never read
    const bool qvalid = u64(t.f0) + h16 < a.bstride;
    const bool line_rows = (a.bstride & 127u) == 0;
    const u8* base = a.bins + t.f0 + h16;
    u32 pos = u32(t.begin);
    const u32 tend = u32(t.end);
    while (pos < tend) {
      const u32 room = u32(kWindowRows) - in_window;
      const u32 end = (tend - pos) < room ? tend : pos + room;
      // Warp-uniform iterations over this warp's positions w0 + s + u * kStep.
      // The row indices of the next iteration are copied into the warp's
      // shared stage with cp.async while this one runs, so an iteration waits
      // for one global round trip (the codes and (g, h)), not two.
      u32* const stage0 = s_rows + warp * (2 * kUnroll * kRPW);
      auto prefetch = [&](u32 w0, u32* st) {
        // the two lanes of a row slot split its kUnroll indices
#pragma unroll
        for (int q = 0; q < kUnroll / 2; ++q) {
          const int u = q + int(lane & 1) * (kUnroll / 2);
          const u32 i = w0 + s + u32(u) * kStep;
          u32* dst = st + u * kRPW + s;
          if (i < end) {
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(ta.ridx + i)
                         : "memory");
          } else {
            *dst = kNoRow;
          }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
      };
      int cur = 0;
      if constexpr (kPrefetch) prefetch(pos + u32(warp) * kRPW, stage0);
      for (u32 w0 = pos + u32(warp) * kRPW; w0 < end; w0 += kStep * kUnroll) {
        const u32 i0 = w0 + s;
        u32 row[kUnroll];
        if constexpr (kPrefetch) {
          const u32 w1 = w0 + kStep * kUnroll;
          u32* const st = stage0 + cur * (kUnroll * kRPW);
          if (w1 < end) {
            prefetch(w1, stage0 + (cur ^ 1) * (kUnroll * kRPW));
          } else {
            asm volatile("cp.async.commit_group;" ::: "memory");  // an empty group keeps the wait uniform
          }
          asm volatile("cp.async.wait_group 1;" ::: "memory");
          __syncwarp();
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) row[u] = qvalid ? st[u * kRPW + s] : kNoRow;
          __syncwarp();  // the stage is refilled by the iteration after next
          cur ^= 1;
        } else {
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const u32 i = i0 + u * kStep;
            row[u] = (i < end && qvalid) ? __ldg(ta.ridx + i) : kNoRow;
          }
        }
        uint4 v[kUnroll];
        u32 gq[kUnroll], hq[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          v[u] = make_uint4(0u, 0u, 0u, 0u);
          gq[u] = 0u;
          hq[u] = 0u;
          if (row[u] != kNoRow) {
            v[u] = load_codes(base + u64(row[u]) * a.bstride, line_rows);
            load_q<QUANT>(ta, sc, i0 + u * kStep, gq[u], hq[u]);
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (row[u] != kNoRow) {
            if (MB < 256 && ((v[u].x | v[u].y | v[u].z | v[u].w) & kHighBits) != 0u)
              add_row<kHOff, u32(MB)>(v[u], gq[u], hq[u], cols);  // a code >= MB: clamped to the spare row
            else
              add_row<kHOff>(v[u], gq[u], hq[u], cols);
          }
      }
      if constexpr (kPrefetch) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncwarp();
      }
      in_window += end - pos;
      pos = end;
      if (in_window == u32(kWindowRows)) {
        __syncthreads();
        if constexpr (kTmem) {
          tile_fold<u32(MB), kNBW>(Lg, u32(kPlaneCells), s_tmem, t_clean, true);
          t_clean = false;
        } else {
          wfold();
        }
        __syncthreads();
        in_window = 0;
      }
    }
  }
  if constexpr (kTmem) {
    tmem_fence_before_sync();
    __syncthreads();
    if (threadIdx.x < 32) tmem_dealloc(s_tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// 256-bin kernel over 64-feature tiles (the training path's kernel when the
// matrix has more than 32 features, on one GPU).
//
// Same task queue and output as k_hist, but a task covers 64 features: a
// warp step takes 8 rows x 64 bytes (four lanes per row, 16 bytes each), so a
// scattered row costs one cache-line lookup per 64 features instead of one per
// 32 -- the lookups share the L1/shared data path with the shared atomics.
// The u32 planes fill 128 KB of shared memory as two 64 KB regions, one per
// 32-feature half of the tile, each a g plane [bin][32] and 32 KB above it an
// h plane (the layout of k_hist, so the packed address arithmetic of add_row
// applies, with the half in the address's high 16 bits).  Lane (s, q) has
// the key s + 8 (q >> 1): in every atomic step the 16 lanes of q = 0, 2 (and
// of q = 1, 3) hit 16 distinct banks.
//
// The int64 window sums live in tensor memory (all 512 columns of the SM):
// folding a window reads the u32 planes once and clears them, with the
// read-modify-write of the int64 sums off the L1/shared data path and out of
// L2.  TMEM lane 32 q + t holds tile feature 32 (q >> 1) + t for the bins
// 128 (q & 1) .. + 127, bin b' of those in columns 4 b' .. 4 b' + 3 (g low and
// high word, h low and high word); warp w serves lane quarter q = w % 4 (the
// only lanes it can reach) and 16 of its bins.  The drain stages each
// 32-feature half through the planes' shared memory as [feature][bin] int64
// pairs (bin index XOR feature, so that both the staging writes, a feature
// per lane, and the reads, a bin per lane, stay at four wavefronts per warp)
// and writes the output with consecutive threads on consecutive bins of one
// feature: whole lines for the stores of a node built by one task, and eight
// sectors per warp for the 64-bit atomics of a node split into pieces.
constexpr int kWide = 64;
constexpr u32 kWideRegion = 65536;  // bytes of one half's g and h planes
constexpr u32 kWideH = 32768;       // h plane offset in a region, bytes
constexpr u32 kWideTmemCols = 512;

// u32 index (from the planes' start) of the g cell of (bin b, tile feature f)
// of the 64-feature kernel; its h cell is kWideH / 4 further
__device__ __forceinline__ u32 wide_cell(u32 b, u32 f) {
  return (f >> 5) * (kWideRegion / 4) + b * 32u + (f & 31u);
}

// Lane constants of the 64-feature kernel: lane (s, q) reads 16 bytes at
// feature 16 q of the tile from row slot s; its region is the half q >> 1, its
// first column 16 (q & 1) there, and its key s + 8 (q >> 1) differs from
// every other lane's of the same first column.
__device__ __forceinline__ LaneCols wide_lane(u32 lane, const u32* planes) {
  const u32 s8 = lane >> 2, q = lane & 3u;
  return lane_cols(smem_addr(planes) + (q >> 1) * kWideRegion, 16u * (q & 1u), s8 + 8u * (q >> 1));
}

// This warp's part of the 64-feature kernel's window sums: lane quarter
// w % 4, the 16 bins bin0 .. bin0 + 15 of the half w % 4 >> 1, one feature f
// (of the tile) per thread, and the TMEM address col of its first bin.
struct WidePart {
  u32 half, bin0, f, col;
};

__device__ __forceinline__ WidePart wide_part(u32 tmem_base) {
  const u32 w = threadIdx.x >> 5, tq = w & 3u;
  return WidePart{tq >> 1, 128u * (tq & 1u) + 16u * (w >> 2), 32u * (tq >> 1) + (threadIdx.x & 31u),
                  tmem_at(tmem_base, 32u * tq, 64u * (w >> 2))};
}

// The window's u32 sums of this warp's cells into the int64 sums in TMEM
// (with `clean` the first fold of a key, which copies); with `clear` the
// planes are zeroed.  Each warp touches only its own TMEM cells.  Kept out of
// line: inlined into the row loop it made the compiler spill the loop's
// registers.
__device__ __noinline__ void wide_fold(u32* L, u32 tmem_base, bool clean, bool clear) {
  constexpr u32 kH = kWideH / 4;
  const WidePart tp = wide_part(tmem_base);
#pragma unroll 1
  for (u32 i = 0; i < 16; ++i) {  // one bin (four columns) at a time
    u32 r[4];
    if (!clean) tmem_ld4(tp.col + 4u * i, r);
    const u32 cell = wide_cell(tp.bin0 + i, tp.f);
    const u32 g = L[cell], h = L[cell + kH];
    if (clear) {
      L[cell] = 0u;
      L[cell + kH] = 0u;
    }
    if (!clean) {
      tmem_wait_ld();
    } else {
      r[0] = r[1] = r[2] = r[3] = 0u;
    }
    const u64 G = ((u64(r[1]) << 32) | r[0]) + u64(i64(int(g)));
    const u64 H = ((u64(r[3]) << 32) | r[2]) + u64(h);
    r[0] = u32(G);
    r[1] = u32(G >> 32);
    r[2] = u32(H);
    r[3] = u32(H >> 32);
    tmem_st4(tp.col + 4u * i, r);
  }
  tmem_wait_st();
}

template <bool QUANT>
__global__ void __launch_bounds__(1024) k_hist_wide(HistArgs a) {
  constexpr int THREADS = 1024;
  constexpr int kCells = 256 * kWide;
  constexpr int kRows = 8;                       // rows per warp step
  constexpr u32 kStep = u32(THREADS / 32) * kRows;
  constexpr int kUnroll = DP_HIST_WIDE_UNROLL;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ u32 s_task, s_tmem;
  u32* L = reinterpret_cast<u32*>(smem + plane_pad(smem));
  for (int i = threadIdx.x; i < 2 * kCells; i += THREADS) L[i] = 0u;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == 0) tmem_alloc(&s_tmem, kWideTmemCols);
  const u32 s8 = u32(lane) >> 2;
  const u32 q16 = 16u * u32(lane & 3);
  const LaneCols wl = wide_lane(u32(lane), L);
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  u32 key_slot = kNoRow, key_f0 = 0, key_tree = 0;
  bool key_excl = false;
  u32 in_window = 0;
  bool t_clean = true;  // TMEM holds nothing of the current key (block-uniform)
  const u32 ntasks = a.ntasks_dev ? *a.ntasks_dev : a.ntasks;

  for (;;) {
    if (threadIdx.x == 0) s_task = atomicAdd(a.counter, 1u);
    __syncthreads();  // also: every warp has finished the previous task
    const u32 ti = s_task;
    const bool done = ti >= ntasks;
    HistTask t{};
    if (!done) t = a.tasks[ti];
    const bool same = !done && t.slot == key_slot && t.f0 == key_f0 && t.tree == key_tree;
    if (!same && key_slot != kNoRow) {
      wide_fold(L, s_tmem, t_clean, false);  // the last window joins the sums
      t_clean = false;
      __syncthreads();  // the planes are read: they become the staging area
      longlong2* T = reinterpret_cast<longlong2*>(L);  // [32 features][256 bins], bin index ^ feature
      i64* out = a.hist + u64(key_slot) * a.layout.slot_stride;
      const WidePart tp = wide_part(s_tmem);
      for (u32 hf = 0; hf < 2; ++hf) {
        if (tp.half == hf) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            u32 r[16];
            tmem_ld16(tp.col + 16u * u32(c), r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const u32 b = tp.bin0 + 4u * u32(c) + u32(i);
              T[u32(lane) * 256u + (b ^ u32(lane))] =
                  make_longlong2(static_cast<long long>((u64(r[4 * i + 1]) << 32) | r[4 * i]),
                                 static_cast<long long>((u64(r[4 * i + 3]) << 32) | r[4 * i + 2]));
            }
          }
        }
        __syncthreads();
        if (key_excl) {
          for (u32 i = threadIdx.x; i < 32u * 256u; i += THREADS) {
            const u32 fl32 = i >> 8, b = i & 255u;
            const u32 gf = key_f0 + 32u * hf + fl32;
            if (gf >= a.F) continue;
            const u32 grp = gf / a.layout.fg, fl = gf - grp * a.layout.fg;
            i64* cell = out + grp * a.layout.group_stride + (u64(fl) * kMaxBins + b) * 2;
            *reinterpret_cast<longlong2*>(cell) = T[fl32 * 256u + (b ^ fl32)];
          }
        } else {
          // g and h of a cell on neighbouring lanes: a warp's 32 reductions
          // cover 16 whole cells, eight 32-byte sectors
          const long long* T64 = reinterpret_cast<const long long*>(T);
          for (u32 i = threadIdx.x; i < 2u * 32u * 256u; i += THREADS) {
            const u32 c = i >> 1, comp = i & 1u;
            const u32 fl32 = c >> 8, b = c & 255u;
            const u32 gf = key_f0 + 32u * hf + fl32;
            if (gf >= a.F) continue;
            const long long v = T64[2u * (fl32 * 256u + (b ^ fl32)) + comp];
            const u32 grp = gf / a.layout.fg, fl = gf - grp * a.layout.fg;
            i64* cell = out + grp * a.layout.group_stride + (u64(fl) * kMaxBins + b) * 2 + comp;
            if (v) atomicAdd(reinterpret_cast<unsigned long long*>(cell), static_cast<unsigned long long>(v));
          }
        }
        __syncthreads();  // the staging area is read before it is refilled or cleared
      }
      for (int i = threadIdx.x; i < 2 * kCells; i += THREADS) L[i] = 0u;
      t_clean = true;
      key_slot = kNoRow;
      in_window = 0;
    }
    if (done) break;
    __syncthreads();  // s_task read by all; the planes cleared by the drain
    key_slot = t.slot;
    key_f0 = t.f0;
    key_tree = t.tree;
    key_excl = t.excl != 0;
    const TreeArrays ta = a.trees[t.tree];
    Scales sc{1.f, 1.f};
    if (!QUANT) sc = a.scales[t.tree];
    const bool qvalid = u64(t.f0) + q16 < a.bstride;
    const bool line_rows = (a.bstride & 127u) == 0;
    const u8* base = a.bins + t.f0 + q16;
    u32 pos = u32(t.begin);
    const u32 tend = u32(t.end);
    while (pos < tend) {
      const u32 room = u32(kWindowRows) - in_window;
      const u32 end = (tend - pos) < room ? tend : pos + room;
      for (u32 i0 = pos + u32(warp) * kRows + s8; i0 < end; i0 += kStep * kUnroll) {
        u32 row[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const u32 i = i0 + u * kStep;
          row[u] = (i < end && qvalid) ? __ldg(ta.ridx + i) : kNoRow;
        }
        uint4 v[kUnroll];
        u32 gq[kUnroll], hq[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          v[u] = make_uint4(0u, 0u, 0u, 0u);
          gq[u] = 0u;
          hq[u] = 0u;
          if (row[u] != kNoRow) {
            v[u] = load_codes(base + u64(row[u]) * a.bstride, line_rows);
            load_q<QUANT>(ta, sc, i0 + u * kStep, gq[u], hq[u]);
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (row[u] != kNoRow) add_row<kWideH>(v[u], gq[u], hq[u], wl);
      }
      in_window += end - pos;
      pos = end;
      if (in_window == u32(kWindowRows)) {
        __syncthreads();
        wide_fold(L, s_tmem, t_clean, true);
        t_clean = false;
        __syncthreads();
        in_window = 0;
      }
    }
  }
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(s_tmem, kWideTmemCols);
}

template <bool QUANT>
void launch_hist_wide_variant(const HistArgs& a, cudaStream_t s, bool counter_zeroed) {
  constexpr int kSmem = int(kPlaneAlignPad) + 256 * kWide * 8;
  static thread_local int configured_device = -1;
  static thread_local int grid_cap = 0;
  int dev = 0;
  DP_CUDA(cudaGetDevice(&dev));
  if (configured_device != dev) {
    DP_CUDA(cudaFuncSetAttribute(k_hist_wide<QUANT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    int sms = 0, per_sm = 0;
    DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DP_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_hist_wide<QUANT>, 1024, kSmem));
    // every block takes all of its SM's tensor memory, so there must be
    // exactly one per SM
    need(per_sm == 1, "internal error: the 64-feature histogram kernel must run one block per SM");
    grid_cap = sms;
    configured_device = dev;
  }
  const u32 grid = (a.ntasks_dev || a.ntasks >= u32(grid_cap)) ? u32(grid_cap) : a.ntasks;
  if (!counter_zeroed) DP_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(u32), s));
  k_hist_wide<QUANT><<<grid, 1024, kSmem, s>>>(a);
}

template <int MB, int THREADS, bool QUANT>
void launch_hist_variant(const HistArgs& a, cudaStream_t s, bool counter_zeroed) {
  constexpr int kSmem = hist_smem<MB>();
  static thread_local int configured_device = -1;
  static thread_local int grid_cap = 0;
  int dev = 0;
  DP_CUDA(cudaGetDevice(&dev));
  if (configured_device != dev) {
    DP_CUDA(cudaFuncSetAttribute(k_hist<MB, THREADS, QUANT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    int sms = 0, per_sm = 0;
    DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DP_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_hist<MB, THREADS, QUANT>, THREADS, kSmem));
    // every block allocates MB tensor-memory columns; the blocks one SM holds
    // must fit its 512 (an allocation beyond them would wait for a release)
    need(per_sm >= 1 && (MB < 256 || per_sm * MB <= 512),
         "internal error: histogram blocks per SM exceed the tensor memory");
    grid_cap = sms * per_sm;
    configured_device = dev;
  }
  const u32 grid = (a.ntasks_dev || a.ntasks >= u32(grid_cap)) ? u32(grid_cap) : a.ntasks;
  if (!counter_zeroed) DP_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(u32), s));
  k_hist<MB, THREADS, QUANT><<<grid, THREADS, kSmem, s>>>(a);
}

}  // namespace

void launch_histograms(const u8* bins, u64 bin_stride, u32 F, int max_bins, bool quantized_gh,
                       const TreeArrays* trees, const Scales* scales, const HistTask* tasks, u32 ntasks,
                       u32* counter, i64* hist, cudaStream_t s, const u32* ntasks_dev, const HistLayout* layout,
                       bool counter_zeroed) {
  if (!ntasks && !ntasks_dev) return;
  const HistLayout lay = layout ? *layout : HistLayout{F, u64(F) * 2 * kMaxBins, 0};
  need(lay.fg > 0, "histogram layout needs a positive feature group size");
  const HistArgs a{bins, bin_stride, F, ntasks, ntasks_dev, trees, scales, tasks, counter, hist, lay};
  if (max_bins <= 64) {
    if (quantized_gh) launch_hist_variant<64, 512, true>(a, s, counter_zeroed);
    else launch_hist_variant<64, 512, false>(a, s, counter_zeroed);
  } else {
    if (quantized_gh) launch_hist_variant<256, DP_HIST_THREADS, true>(a, s, counter_zeroed);
    else launch_hist_variant<256, DP_HIST_THREADS, false>(a, s, counter_zeroed);
  }
  after_launch("histograms");
}

void launch_histograms_wide(const u8* bins, u64 bin_stride, u32 F, bool quantized_gh, const TreeArrays* trees,
                            const Scales* scales, const HistTask* tasks, u32 ntasks, u32* counter, i64* hist,
                            cudaStream_t s, const u32* ntasks_dev, const HistLayout* layout, bool counter_zeroed) {
  if (!ntasks && !ntasks_dev) return;
  const HistLayout lay = layout ? *layout : HistLayout{F, u64(F) * 2 * kMaxBins, 0};
  need(lay.fg > 0, "histogram layout needs a positive feature group size");
  const HistArgs a{bins, bin_stride, F, ntasks, ntasks_dev, trees, scales, tasks, counter, hist, lay};
  if (quantized_gh) launch_hist_wide_variant<true>(a, s, counter_zeroed);
  else launch_hist_wide_variant<false>(a, s, counter_zeroed);
  after_launch("histograms");
}

u64 hist_chunk_rows(u64 total_rows, u64 nseg, bool whole_lines) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Tasks per SM, balanced by the task queue: about four; sixteen for 2 to 16
  // segments and eight for 17 to 256, whose rows interleave in the matrix:
  // with the queue in piece order, the pieces of one row range run together,
  // and smaller pieces keep them within what L2 holds for each range.  With
  // one segment or more than 256 the extra drains cost more than that gains.
  // Measured on B200, config 5 (100M x 32), ms at 4 / 8 / 16 tasks per SM:
  // 256 bins, 8 nodes 1.68 / 1.55 / 1.51; 64 nodes 1.63 / 1.59 / 1.64; 256
  // nodes 1.75 / 1.62 / 1.72; 1024 nodes 1.86 / 1.93 / 2.01 (1.86 at 2); 64
  // bins, 64 nodes 1.56 / 1.48 / 1.46; 256 nodes 1.59 / 1.45 / 1.46; one node
  // 0.57 of HBM at 4 against 0.56 at 16.  Rows that are whole 128-byte lines
  // share no line, so three, for fewer drains (10M x 128, one node: 0.529
  // against 0.552 ms).  DP_HIST_TASKS_PER_SM overrides.
  u64 per_sm = whole_lines ? 3 : (nseg >= 2 && nseg <= 16) ? 16 : (nseg > 16 && nseg <= 256) ? 8 : 4;
  if (const char* v = std::getenv("DP_HIST_TASKS_PER_SM"))
    if (*v) per_sm = std::max<u64>(1, std::strtoull(v, nullptr, 10));
  const u64 target = u64(sms) * per_sm;
  const u64 chunk = (total_rows + target - 1) / target;
  return chunk < 2048 ? 2048 : chunk;
}

}  // namespace dp
