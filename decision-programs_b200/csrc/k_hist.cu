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
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "hist_update.cuh"
#include "kernels.h"

namespace dp {

namespace {

constexpr int kFT = kHistFeatureTile;  // 32 features per tile
constexpr int kRPW = 16;               // rows per warp step (two lanes per row)
// Row steps in flight per warp.  Measured on B200 with the packed update
// (config 5, 100M x 32): 4 is best for the 32-feature 256-bin kernel (1, 8
// and 1024 nodes: 1.19 / 1.89 / 2.15 ms against 1.20 / 1.98 / 2.28 with 6
// and 1.22 / 2.01 / 2.31 with 8); the 64-feature kernel keeps 6 (config 4:
// 3.06 ms of histograms per round against 3.07 with 4 and 3.31 with 8); the
// 512-thread 64-bin kernel 4.
#ifndef DP_HIST_UNROLL
#define DP_HIST_UNROLL 4
#endif
#ifndef DP_HIST_WIDE_UNROLL
#define DP_HIST_WIDE_UNROLL 6
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

template <int MB, int THREADS, bool QUANT>
__global__ void __launch_bounds__(THREADS) k_hist(HistArgs a) {
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
  constexpr int kWRow = MB + 1;              // int64 planes: [feature][bin], rows padded
  constexpr int kWCells = kFT * kWRow;
  constexpr int kWarps = THREADS / 32;
  constexpr u32 kStep = u32(kWarps) * kRPW;
  constexpr int kUnroll = unroll_for<MB>();
  // bits of a code word that are set only by codes >= MB (MB = 64)
  constexpr u32 kHighBits = MB == 64 ? 0xc0c0c0c0u : 0u;
  static_assert(MB == 64 || MB == 256, "64- or 256-bin planes");
  u32* Lg = reinterpret_cast<u32*>(smem + plane_pad(smem));
  u32* Lh = Lg + kPlaneCells;
  long long* Wg = reinterpret_cast<long long*>(Lh + kPlaneCells);
  long long* Wh = Wg + kWCells;
  for (int i = threadIdx.x; i < kPlaneCells; i += THREADS) {
    Lg[i] = 0u;
    Lh[i] = 0u;
  }
  for (int i = threadIdx.x; i < kWCells; i += THREADS) {
    Wg[i] = 0;
    Wh[i] = 0;
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

  // Moves the window sums into the int64 planes (transposed to [feature][bin])
  // and clears the window.  The first fold of a key copies (the planes hold
  // the previous key's drained values), later folds add.
  bool w_clean = true;  // block-uniform
  auto fold = [&]() {
    if (w_clean) {
      for (int i = threadIdx.x; i < kCells; i += THREADS) {
        const int b = i / kFT, f = i % kFT;
        Wg[f * kWRow + b] = static_cast<long long>(static_cast<int>(Lg[i]));
        Wh[f * kWRow + b] = static_cast<long long>(Lh[i]);
        Lg[i] = 0u;
        Lh[i] = 0u;
      }
    } else {
      for (int i = threadIdx.x; i < kCells; i += THREADS) {
        const int b = i / kFT, f = i % kFT;
        Wg[f * kWRow + b] += static_cast<long long>(static_cast<int>(Lg[i]));
        Wh[f * kWRow + b] += static_cast<long long>(Lh[i]);
        Lg[i] = 0u;
        Lh[i] = 0u;
      }
    }
    w_clean = false;
  };

  for (;;) {
    if (threadIdx.x == 0) s_task = atomicAdd(a.counter, 1u);
    __syncthreads();  // also: every warp has finished the previous task
    const u32 ti = s_task;
    const bool done = ti >= ntasks;
    HistTask t{};
    if (!done) t = a.tasks[ti];
    const bool same = !done && t.slot == key_slot && t.f0 == key_f0 && t.tree == key_tree;
    if (!same && key_slot != kNoRow) {
      fold();
      __syncthreads();
      // consecutive threads take consecutive bins of one feature: a warp
      // covers one contiguous 512-byte run.  A task that alone covers its
      // (slot, tile) stores every cell (16-byte stores, no read of the line);
      // otherwise non-zero cells are added with 64-bit reductions.
      i64* out = a.hist + u64(key_slot) * a.layout.slot_stride;
      for (int idx = threadIdx.x; idx < kCells; idx += THREADS) {
        const int f = idx / MB, b = idx % MB;
        const long long gs = Wg[f * kWRow + b], hs = Wh[f * kWRow + b];
        const u32 gf = key_f0 + u32(f);
        if (gf >= a.F) continue;
        const u32 grp = gf / a.layout.fg, fl = gf - grp * a.layout.fg;
        i64* cell = out + grp * a.layout.group_stride + (u64(fl) * kMaxBins + b) * 2;
        if (key_excl) {
          *reinterpret_cast<longlong2*>(cell) = make_longlong2(gs, hs);
        } else if (gs | hs) {
          atomicAdd(reinterpret_cast<unsigned long long*>(cell), static_cast<unsigned long long>(gs));
          atomicAdd(reinterpret_cast<unsigned long long*>(cell) + 1, static_cast<unsigned long long>(hs));
        }
      }
      w_clean = true;
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
        fold();
        __syncthreads();
        in_window = 0;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// 256-bin kernel over 64-feature tiles (the training path's kernel when the
// matrix has more than 32 features).
//
// Same task queue and output as k_hist, but a task covers 64 features: a
// warp step takes 8 rows x 64 bytes (four lanes per row, 16 bytes each), so a
// scattered row costs one cache-line lookup per 64 features instead of one per
// 32 -- the lookups share the L1/shared data path with the shared atomics.
// The u32 planes fill 128 KB of shared memory as two 64 KB regions, one per
// 32-feature half of the tile, each a g plane [bin][32] and 32 KB above it an
// h plane (the layout of k_hist, so the packed address arithmetic of add_row
// applies, with the half in the address's high 16 bits).  The int64 window
// sums live in a block-private scratch in global memory (L2-resident, layout
// [bin][64], coalesced folds).  Lane (s, q) rotates its 16 bytes by
// s + 8 (q >> 1): in every atomic step the 16 lanes of q = 0, 2 (and of
// q = 1, 3) hit 16 distinct banks.
constexpr int kWide = 64;
constexpr u32 kWideRegion = 65536;  // bytes of one half's g and h planes

// u32 index (from the planes' start) of the g cell of (bin b, tile feature f)
// of the 64-feature kernels; its h cell is kWideH / 4 further
__device__ __forceinline__ u32 wide_cell(u32 b, u32 f) {
  return (f >> 5) * (kWideRegion / 4) + b * 32u + (f & 31u);
}

constexpr u32 kWideH = 32768;  // h plane offset of a 64-feature kernel's region, bytes

// Lane constants of the 64-feature kernels: lane (s, q) reads 16 bytes at
// feature 16 q of the tile from row slot s; its region is the half q >> 1, its
// first column 16 (q & 1) there, and its key s + 8 (q >> 1) differs from
// every other lane's of the same first column.
__device__ __forceinline__ LaneCols wide_lane(u32 lane, const u32* planes) {
  const u32 s8 = lane >> 2, q = lane & 3u;
  return lane_cols(smem_addr(planes) + (q >> 1) * kWideRegion, 16u * (q & 1u), s8 + 8u * (q >> 1));
}

template <bool QUANT>
__global__ void __launch_bounds__(1024) k_hist_wide(HistArgs a, long long* __restrict__ wscr) {
  constexpr int MB = 256, THREADS = 1024;
  constexpr int kCells = MB * kWide;
  constexpr int kRows = 8;                       // rows per warp step
  constexpr u32 kStep = u32(THREADS / 32) * kRows;
  constexpr int kUnroll = DP_HIST_WIDE_UNROLL;
  constexpr u32 kH = kWideH / 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ u32 s_task;
  u32* L = reinterpret_cast<u32*>(smem + plane_pad(smem));
  long long* Sg = wscr + u64(blockIdx.x) * 2 * kCells;
  long long* Sh = Sg + kCells;
  for (int i = threadIdx.x; i < 2 * kCells; i += THREADS) L[i] = 0u;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const u32 s8 = u32(lane) >> 2;
  const LaneCols wl = wide_lane(u32(lane), L);
  const u32 q16 = 16u * u32(lane & 3);
  u32 key_slot = kNoRow, key_f0 = 0, key_tree = 0;
  bool key_excl = false;
  u32 in_window = 0;
  bool s_clean = true;  // the scratch holds nothing of the current key (block-uniform)
  const u32 ntasks = a.ntasks_dev ? *a.ntasks_dev : a.ntasks;

  // the window's sums into the scratch ([bin][64], cell i = b * 64 + f), the
  // planes cleared; consecutive threads read consecutive columns of a half
  auto fold = [&]() {
    for (int i = threadIdx.x; i < kCells; i += THREADS) {
      const u32 c = wide_cell(u32(i) / kWide, u32(i) % kWide);
      const long long g = static_cast<long long>(static_cast<int>(L[c]));
      const long long h = static_cast<long long>(L[c + kH]);
      Sg[i] = s_clean ? g : Sg[i] + g;
      Sh[i] = s_clean ? h : Sh[i] + h;
      L[c] = 0u;
      L[c + kH] = 0u;
    }
    s_clean = false;
  };

  for (;;) {
    if (threadIdx.x == 0) s_task = atomicAdd(a.counter, 1u);
    __syncthreads();
    const u32 ti = s_task;
    const bool done = ti >= ntasks;
    HistTask t{};
    if (!done) t = a.tasks[ti];
    const bool same = !done && t.slot == key_slot && t.f0 == key_f0 && t.tree == key_tree;
    if (!same && key_slot != kNoRow) {
      // scratch + last window straight to the output; each thread keeps the
      // cells it folded, so no barrier is needed between the two
      i64* out = a.hist + u64(key_slot) * a.layout.slot_stride;
      for (int i = threadIdx.x; i < kCells; i += THREADS) {
        const u32 b = u32(i) / kWide, f = u32(i) % kWide;
        const u32 c = wide_cell(b, f);
        long long gs = static_cast<long long>(static_cast<int>(L[c]));
        long long hs = static_cast<long long>(L[c + kH]);
        if (!s_clean) {
          gs += Sg[i];
          hs += Sh[i];
        }
        L[c] = 0u;
        L[c + kH] = 0u;
        const u32 gf = key_f0 + f;
        if (gf >= a.F) continue;
        const u32 grp = gf / a.layout.fg, fl = gf - grp * a.layout.fg;
        i64* cell = out + grp * a.layout.group_stride + (u64(fl) * kMaxBins + b) * 2;
        if (key_excl) {
          *reinterpret_cast<longlong2*>(cell) = make_longlong2(gs, hs);
        } else if (gs | hs) {
          atomicAdd(reinterpret_cast<unsigned long long*>(cell), static_cast<unsigned long long>(gs));
          atomicAdd(reinterpret_cast<unsigned long long*>(cell) + 1, static_cast<unsigned long long>(hs));
        }
      }
      s_clean = true;
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
        fold();
        __syncthreads();
        in_window = 0;
      }
    }
  }
}

template <bool QUANT>
void launch_hist_wide_variant(const HistArgs& a, i64* scratch, u64 scratch_elems, cudaStream_t s) {
  constexpr int kSmem = int(kPlaneAlignPad) + 256 * kWide * 8;
  static thread_local int configured_device = -1;
  static thread_local int grid_cap = 0;
  int dev = 0;
  DP_CUDA(cudaGetDevice(&dev));
  if (configured_device != dev) {
    DP_CUDA(cudaFuncSetAttribute(k_hist_wide<QUANT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    // shared-memory carve-out in percent (testing knob: how L1 size matters)
    if (const char* c = std::getenv("DP_HIST_CARVEOUT"))
      DP_CUDA(cudaFuncSetAttribute(k_hist_wide<QUANT>, cudaFuncAttributePreferredSharedMemoryCarveout, std::atoi(c)));
    int sms = 0, per_sm = 0;
    DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DP_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_hist_wide<QUANT>, 1024, kSmem));
    grid_cap = sms * (per_sm > 0 ? per_sm : 1);
    configured_device = dev;
  }
  const u32 grid = (a.ntasks_dev || a.ntasks >= u32(grid_cap)) ? u32(grid_cap) : a.ntasks;
  need(scratch_elems >= u64(grid) * 2 * 256 * kWide, "internal error: histogram window scratch too small for the grid");
  DP_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(u32), s));
  k_hist_wide<QUANT><<<grid, 1024, kSmem, s>>>(a, reinterpret_cast<long long*>(scratch));
}

// ---------------------------------------------------------------------------
// The 64-feature kernel with the row codes brought into shared memory by the
// tensor memory accelerator instead of per-lane global loads: one untiled
// bulk copy per row (cp.async.bulk), or with GATHER one tiled gather of four
// rows per instruction (cp.async.bulk.tensor tile::gather4 over a tensor map
// of the bin matrix: box `pitch` bytes x 1 row).
//
// Each warp owns two stages of 24 rows x 64 bytes and one mbarrier per stage,
// and takes chunks of 24 consecutive row positions of the window (chunk c
// goes to warp c mod 32).  Lanes 0..23 read the chunk's row indices; lanes
// issue the chunk's copies (24 row copies, or 6 gathers of four rows whose
// indices come by shuffles) and lane 0 arms the stage's barrier with the
// chunk's byte count.  While the atomics of one chunk run, the copies of
// the warp's next two chunks are in flight, and the scattered row reads use
// the copy engine rather than the L1 load path that the shared atomics also
// occupy.  The atomics, planes, window folds and drain are k_hist_wide's.
//
// Every barrier wait is bounded (about a second of global timer): a wait that
// runs out ORs the status bit, the warp stops issuing, and the blocks leave
// at their next task fetch after a bounded wait for their copies in flight.
constexpr int kBulkStages = 2;
// planes, 128 bytes of alignment room, stages of ROWS rows (128-byte
// aligned), barriers
template <int ROWS>
constexpr int bulk_smem() { return int(kPlaneAlignPad) + 256 * kWide * 8 + 32 * kBulkStages * ROWS * kWide + 32 * kBulkStages * 8; }
constexpr u64 kBulkWaitNs = 1000000000ull;

__device__ __forceinline__ void mbar_init(u32 bar, u32 count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect(u32 bar, u32 bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(u32 bar, u32 parity) {
  u32 ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ u64 global_ns() {
  u64 t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// true when the barrier's phase of this parity completed, false after about
// kBulkWaitNs without completion
__device__ __forceinline__ bool mbar_wait_bounded(u32 bar, u32 parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const u64 t0 = global_ns();
  for (u32 it = 1; it < (1u << 28); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && global_ns() - t0 > kBulkWaitNs) return false;
  }
  return false;
}

// global -> this CTA's shared memory, completion counted on `bar` in bytes;
// dst, src and bytes multiples of 16
__device__ __forceinline__ void bulk_copy_g2s(u32 dst, const void* src, u32 bytes, u32 bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// four rows (r0..r3) x the box width from column x of the tensor map's bin
// matrix, one after the other into shared memory at dst (128-byte aligned)
__device__ __forceinline__ void gather4_g2s(u32 dst, const CUtensorMap* map, int x, u32 r0, u32 r1, u32 r2, u32 r3,
                                            u32 bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<u64>(map)), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(bar)
      : "memory");
}

template <bool QUANT, bool GATHER, int kBulkRows>
__global__ void __launch_bounds__(1024) k_hist_bulk(HistArgs a, long long* __restrict__ wscr, u32* __restrict__ status,
                                                    u32 status_bit, u32 pitch, u32 copy_warps,
                                                    const __grid_constant__ CUtensorMap map) {
  constexpr int MB = 256, THREADS = 1024, kWarps = THREADS / 32;
  constexpr int kCells = MB * kWide;
  constexpr int kSteps = kBulkRows / 8;  // 8-row steps per chunk
  constexpr int kBulkStageBytes = kBulkRows * kWide;
  constexpr int kDirect = 6 / kSteps;    // chunks per iteration of the direct-load warps
  static_assert(kBulkRows % 8 == 0 && 6 % kSteps == 0, "chunks of 8, 16 or 24 rows");
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ u32 s_task;
  __shared__ u32 s_abort;
  constexpr u32 kH = kWideH / 4;
  u32* L = reinterpret_cast<u32*>(smem + plane_pad(smem));  // the planes of k_hist_wide
  // planes end 128-byte aligned (they start so and hold 128 KB)
  unsigned char* stages = reinterpret_cast<unsigned char*>(L) + 2 * kCells * 4;
  unsigned long long* bars =
      reinterpret_cast<unsigned long long*>(stages + kWarps * kBulkStages * kBulkStageBytes);
  long long* Sg = wscr + u64(blockIdx.x) * 2 * kCells;
  long long* Sh = Sg + kCells;
  for (int i = threadIdx.x; i < 2 * kCells; i += THREADS) L[i] = 0u;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned char* my_stages = stages + warp * kBulkStages * kBulkStageBytes;
  const u32 stage_s = smem_addr(my_stages);
  const u32 bar = smem_addr(bars + warp * kBulkStages);  // stage k's barrier at bar + 8 k
  if (lane < kBulkStages) mbar_init(bar + 8u * u32(lane), 1u);
  if (threadIdx.x == 0) s_abort = 0;
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  const u32 s8 = u32(lane) >> 2;
  const LaneCols wl = wide_lane(u32(lane), L);
  const u32 q16 = 16u * u32(lane & 3);
  u32 key_slot = kNoRow, key_f0 = 0, key_tree = 0;
  bool key_excl = false;
  u32 in_window = 0;
  bool s_clean = true;
  u32 parity = 0;     // bit k: the phase parity that stage k's next wait expects
  u32 pending = 0;    // bit k: stage k has copies issued and not yet waited for
  bool stop = false;  // this warp's wait ran out
  const u32 ntasks = a.ntasks_dev ? *a.ntasks_dev : a.ntasks;
  __syncthreads();

  auto fold = [&]() {
    for (int i = threadIdx.x; i < kCells; i += THREADS) {
      const u32 c = wide_cell(u32(i) / kWide, u32(i) % kWide);
      const long long g = static_cast<long long>(static_cast<int>(L[c]));
      const long long h = static_cast<long long>(L[c + kH]);
      Sg[i] = s_clean ? g : Sg[i] + g;
      Sh[i] = s_clean ? h : Sh[i] + h;
      L[c] = 0u;
      L[c + kH] = 0u;
    }
    s_clean = false;
  };

  for (;;) {
    if (threadIdx.x == 0) s_task = *reinterpret_cast<volatile u32*>(&s_abort) ? 0xffffffffu : atomicAdd(a.counter, 1u);
    __syncthreads();
    const u32 ti = s_task;
    const bool done = ti >= ntasks;
    HistTask t{};
    if (!done) t = a.tasks[ti];
    const bool same = !done && t.slot == key_slot && t.f0 == key_f0 && t.tree == key_tree;
    if (!same && key_slot != kNoRow) {
      i64* out = a.hist + u64(key_slot) * a.layout.slot_stride;
      for (int i = threadIdx.x; i < kCells; i += THREADS) {
        const int b = i / kWide, f = i % kWide;
        const u32 c = wide_cell(u32(b), u32(f));
        long long gs = static_cast<long long>(static_cast<int>(L[c]));
        long long hs = static_cast<long long>(L[c + kH]);
        if (!s_clean) {
          gs += Sg[i];
          hs += Sh[i];
        }
        L[c] = 0u;
        L[c + kH] = 0u;
        const u32 gf = key_f0 + u32(f);
        if (gf >= a.F) continue;
        const u32 grp = gf / a.layout.fg, fl = gf - grp * a.layout.fg;
        i64* cell = out + grp * a.layout.group_stride + (u64(fl) * kMaxBins + b) * 2;
        if (key_excl) {
          *reinterpret_cast<longlong2*>(cell) = make_longlong2(gs, hs);
        } else if (gs | hs) {
          atomicAdd(reinterpret_cast<unsigned long long*>(cell), static_cast<unsigned long long>(gs));
          atomicAdd(reinterpret_cast<unsigned long long*>(cell) + 1, static_cast<unsigned long long>(hs));
        }
      }
      s_clean = true;
      key_slot = kNoRow;
      in_window = 0;
    }
    if (done) break;
    __syncthreads();
    key_slot = t.slot;
    key_f0 = t.f0;
    key_tree = t.tree;
    key_excl = t.excl != 0;
    const TreeArrays ta = a.trees[t.tree];
    Scales sc{1.f, 1.f};
    if (!QUANT) sc = a.scales[t.tree];
    // bytes of each row's copy: the tile's codes inside the row stride (a
    // multiple of 16); lanes past them hold no feature of the matrix
    const u32 cbytes = u32(min(u64(kWide), a.bstride - t.f0));
    const bool qvalid = q16 < cbytes;
    const u8* src = a.bins + t.f0;
    u32 pos = u32(t.begin);
    const u32 tend = u32(t.end);
    while (pos < tend) {
      const u32 room = u32(kWindowRows) - in_window;
      const u32 end = (tend - pos) < room ? tend : pos + room;
      const u32 nchunks = (end - pos + kBulkRows - 1) / kBulkRows;
      auto chunk_rows = [&](u32 cc) { return cc < nchunks ? min(u32(kBulkRows), end - pos - cc * kBulkRows) : 0u; };
      // lane l < n: the row index of the chunk's l-th position
      auto load_row = [&](u32 cc) {
        return u32(lane) < chunk_rows(cc) ? __ldg(ta.ridx + pos + cc * kBulkRows + lane) : 0u;
      };
      // the raw (g, h) words of the lane's three rows of the chunk
      auto load_gh = [&](u32 cc, u32* g, u32* h) {
        const u32 n = chunk_rows(cc);
#pragma unroll
        for (int u = 0; u < kSteps; ++u) {
          const u32 r = u32(u) * 8u + s8;
          g[u] = h[u] = 0u;
          if (r < n && qvalid) {
            const uint2 w = __ldg(reinterpret_cast<const uint2*>(ta.gh) + pos + cc * kBulkRows + r);
            g[u] = w.x;
            h[u] = w.y;
          }
        }
      };
      auto issue = [&](u32 cc, u32 st, u32 row) {
        const u32 n = chunk_rows(cc);
        if constexpr (GATHER) {
          // gather l takes the rows of lanes 4l..4l+3; the chunk's last
          // gather repeats its first row where the chunk ends
          const u32 ng = (n + 3u) / 4u;
          u32 rr[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) rr[j] = __shfl_sync(0xffffffffu, row, (4 * lane + j) & 31);
#pragma unroll
          for (int j = 1; j < 4; ++j)
            if (4u * u32(lane) + u32(j) >= n) rr[j] = rr[0];
          if (lane == 0) mbar_arrive_expect(bar + 8u * st, ng * 4u * pitch);
          if (u32(lane) < ng)
            gather4_g2s(stage_s + st * kBulkStageBytes + u32(lane) * 256u, &map, int(t.f0), rr[0], rr[1], rr[2], rr[3],
                        bar + 8u * st);
        } else {
          if (lane == 0) mbar_arrive_expect(bar + 8u * st, n * cbytes);
          if (u32(lane) < n)
            bulk_copy_g2s(stage_s + st * kBulkStageBytes + u32(lane) * kWide, src + u64(row) * a.bstride, cbytes,
                          bar + 8u * st);
        }
        pending |= 1u << st;
      };
      // Register pipeline: while chunk k is counted, the copies of chunks
      // k+1 and k+2 are in flight, and so are the (g, h) of chunk k+1 and the
      // row indices of chunk k+3, so no global load latency stands between
      // two chunks.
      if (u32(warp) >= copy_warps) {
        // the other warps count their chunks from direct loads, six row
        // steps in flight at a time
        const u8* base = a.bins + t.f0 + q16;
        const bool line_rows = (a.bstride & 127u) == 0;
        for (u32 c = u32(warp); c < nchunks; c += u32(kDirect) * kWarps) {
          u32 row[kDirect * kSteps], at[kDirect * kSteps];
#pragma unroll
          for (int u = 0; u < kDirect * kSteps; ++u) {
            const u32 cc = c + u32(u / kSteps) * kWarps, r = u32(u % kSteps) * 8u + s8;
            at[u] = pos + cc * kBulkRows + r;
            row[u] = (r < chunk_rows(cc) && qvalid) ? __ldg(ta.ridx + at[u]) : kNoRow;
          }
          uint4 v[kDirect * kSteps];
          u32 gq[kDirect * kSteps], hq[kDirect * kSteps];
#pragma unroll
          for (int u = 0; u < kDirect * kSteps; ++u) {
            v[u] = make_uint4(0u, 0u, 0u, 0u);
            gq[u] = hq[u] = 0u;
            if (row[u] != kNoRow) {
              v[u] = load_codes(base + u64(row[u]) * a.bstride, line_rows);
              load_q<QUANT>(ta, sc, at[u], gq[u], hq[u]);
            }
          }
#pragma unroll
          for (int u = 0; u < kDirect * kSteps; ++u)
            if (row[u] != kNoRow) add_row<kWideH>(v[u], gq[u], hq[u], wl);
        }
      }
      u32 c = u32(warp);
      if (u32(warp) < copy_warps && !stop) {
        const u32 r0 = load_row(c), r1 = load_row(c + kWarps);
        if (c < nchunks) issue(c, 0, r0);
        if (c + kWarps < nchunks) issue(c + kWarps, 1, r1);
      }
      const bool copies = u32(warp) < copy_warps;
      u32 row_ahead = copies ? load_row(c + 2u * kWarps) : 0u;
      u32 gn[kSteps], hn[kSteps];
      load_gh(copies ? c : nchunks, gn, hn);
      for (u32 k = 0; copies && !stop && c < nchunks; ++k, c += kWarps) {
        const u32 st = k & 1u;
        // one decision for the warp, so that it stays converged
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar + 8u * st, (parity >> st) & 1u))) {
          stop = true;
          if (lane == 0) {
            atomicOr(status, status_bit);
            *reinterpret_cast<volatile u32*>(&s_abort) = 1u;
          }
          break;
        }
        parity ^= 1u << st;
        pending &= ~(1u << st);
        const u32 n = chunk_rows(c);
        const unsigned char* sb = my_stages + st * kBulkStageBytes;
        uint4 v[kSteps];
        u32 gq[kSteps], hq[kSteps];
        bool ok[kSteps];
#pragma unroll
        for (int u = 0; u < kSteps; ++u) {
          const u32 r = u32(u) * 8u + s8;
          ok[u] = r < n && qvalid;
          // a gather's four rows sit at `pitch` bytes from a 256-byte slot
          const u32 at = GATHER ? (r >> 2) * 256u + (r & 3u) * pitch : r * u32(kWide);
          v[u] = ok[u] ? *reinterpret_cast<const uint4*>(sb + at + q16) : make_uint4(0u, 0u, 0u, 0u);
          if (QUANT) {
            gq[u] = gn[u];
            hq[u] = hn[u];
          } else {
            gq[u] = u32(quantize(__uint_as_float(gn[u]), sc.sg));
            hq[u] = u32(quantize(__uint_as_float(hn[u]), sc.sh));
          }
        }
        load_gh(c + kWarps, gn, hn);
        __syncwarp();
        if (c + 2u * kWarps < nchunks) {
          // the stage's reads above come before the copies that refill it
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue(c + 2u * kWarps, st, row_ahead);
        }
        row_ahead = load_row(c + 3u * kWarps);
#pragma unroll
        for (int u = 0; u < kSteps; ++u)
          if (ok[u]) add_row<kWideH>(v[u], gq[u], hq[u], wl);
      }
      in_window += end - pos;
      pos = end;
      if (in_window == u32(kWindowRows)) {
        __syncthreads();
        fold();
        __syncthreads();
        in_window = 0;
      }
    }
  }
  // only a warp whose wait ran out leaves copies in flight: give them the
  // same bounded time before the block's shared memory is released
  for (u32 st = 0; st < u32(kBulkStages); ++st)
    if ((pending >> st) & 1u) mbar_wait_bounded(bar + 8u * st, (parity >> st) & 1u);
}

template <bool QUANT, bool GATHER, int ROWS>
void launch_hist_bulk_rows(const HistArgs& a, i64* scratch, u64 scratch_elems, u32* status, u32 status_bit,
                              const HistBinsMap* map, cudaStream_t s) {
  static thread_local int configured_device = -1;
  static thread_local int grid_cap = 0;
  int dev = 0;
  DP_CUDA(cudaGetDevice(&dev));
  if (configured_device != dev) {
    DP_CUDA(cudaFuncSetAttribute(k_hist_bulk<QUANT, GATHER, ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize, bulk_smem<ROWS>()));
    int sms = 0, per_sm = 0;
    DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DP_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_hist_bulk<QUANT, GATHER, ROWS>, 1024, bulk_smem<ROWS>()));
    need(per_sm > 0, "the bulk-copy histogram kernel does not fit on this device");
    grid_cap = sms * per_sm;
    configured_device = dev;
  }
  need(status != nullptr && status_bit != 0, "internal error: the bulk-copy histogram kernel needs a status word");
  need((reinterpret_cast<uintptr_t>(a.bins) & 15u) == 0 && (a.bstride & 15u) == 0,
       "internal error: bulk copies need 16-byte aligned bin rows");
  CUtensorMap m{};
  u32 pitch = kWide;
  if (GATHER) {
    need(map != nullptr && map->bins == a.bins && map->stride == a.bstride,
         "internal error: the gather kernel needs the bin matrix's tensor map");
    static_assert(sizeof(m) == sizeof(map->desc), "tensor map size");
    std::memcpy(&m, map->desc, sizeof m);
    pitch = map->box;
  }
  const u32 grid = (a.ntasks_dev || a.ntasks >= u32(grid_cap)) ? u32(grid_cap) : a.ntasks;
  need(scratch_elems >= u64(grid) * 2 * 256 * kWide, "internal error: histogram window scratch too small for the grid");
  // warps that take their codes by copies; the rest load them directly
  const char* cw = std::getenv("DP_HIST_COPY_WARPS");
  const u32 copy_warps = cw && *cw ? u32(std::min(32l, std::max(0l, std::strtol(cw, nullptr, 10)))) : 32u;
  DP_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(u32), s));
  k_hist_bulk<QUANT, GATHER, ROWS><<<grid, 1024, bulk_smem<ROWS>(), s>>>(a, reinterpret_cast<long long*>(scratch), status, status_bit,
                                                           pitch, copy_warps, m);
}

// chunk rows per stage: DP_HIST_BULK_ROWS 8, 16 or 24 (default 24)
template <bool QUANT, bool GATHER>
void launch_hist_bulk_variant(const HistArgs& a, i64* scratch, u64 scratch_elems, u32* status, u32 status_bit,
                              const HistBinsMap* map, cudaStream_t s) {
  const char* r = std::getenv("DP_HIST_BULK_ROWS");
  const long rows = r && *r ? std::strtol(r, nullptr, 10) : 24;
  if (rows == 8) launch_hist_bulk_rows<QUANT, GATHER, 8>(a, scratch, scratch_elems, status, status_bit, map, s);
  else if (rows == 16) launch_hist_bulk_rows<QUANT, GATHER, 16>(a, scratch, scratch_elems, status, status_bit, map, s);
  else launch_hist_bulk_rows<QUANT, GATHER, 24>(a, scratch, scratch_elems, status, status_bit, map, s);
}

template <int MB, int THREADS, bool QUANT>
void launch_hist_variant(const HistArgs& a, cudaStream_t s) {
  constexpr int kRows = MB < 256 ? MB + 1 : 256;  // u32 plane rows (k_hist)
  constexpr int kSmem = int(kPlaneAlignPad) + kRows * kFT * (4 + 4) + kFT * (MB + 1) * (8 + 8);
  static thread_local int configured_device = -1;
  static thread_local int grid_cap = 0;
  int dev = 0;
  DP_CUDA(cudaGetDevice(&dev));
  if (configured_device != dev) {
    DP_CUDA(cudaFuncSetAttribute(k_hist<MB, THREADS, QUANT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    int sms = 0, per_sm = 0;
    DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DP_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_hist<MB, THREADS, QUANT>, THREADS, kSmem));
    grid_cap = sms * (per_sm > 0 ? per_sm : 1);
    configured_device = dev;
  }
  const u32 grid = (a.ntasks_dev || a.ntasks >= u32(grid_cap)) ? u32(grid_cap) : a.ntasks;
  DP_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(u32), s));
  k_hist<MB, THREADS, QUANT><<<grid, THREADS, kSmem, s>>>(a);
}

}  // namespace

void launch_histograms(const u8* bins, u64 bin_stride, u32 F, int max_bins, bool quantized_gh,
                       const TreeArrays* trees, const Scales* scales, const HistTask* tasks, u32 ntasks,
                       u32* counter, i64* hist, cudaStream_t s, const u32* ntasks_dev, const HistLayout* layout) {
  if (!ntasks && !ntasks_dev) return;
  const HistLayout lay = layout ? *layout : HistLayout{F, u64(F) * 2 * kMaxBins, 0};
  need(lay.fg > 0, "histogram layout needs a positive feature group size");
  const HistArgs a{bins, bin_stride, F, ntasks, ntasks_dev, trees, scales, tasks, counter, hist, lay};
  if (max_bins <= 64) {
    if (quantized_gh) launch_hist_variant<64, 512, true>(a, s);
    else launch_hist_variant<64, 512, false>(a, s);
  } else {
    if (quantized_gh) launch_hist_variant<256, DP_HIST_THREADS, true>(a, s);
    else launch_hist_variant<256, DP_HIST_THREADS, false>(a, s);
  }
  after_launch("histograms");
}

u64 hist_wide_scratch_elems() {
  int dev = 0, sms = 148, per_sm = 1;
  DP_CUDA(cudaGetDevice(&dev));
  DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  constexpr int kSmem = int(kPlaneAlignPad) + 256 * kWide * 8;
  DP_CUDA(cudaFuncSetAttribute(k_hist_wide<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
  DP_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_hist_wide<true>, 1024, kSmem));
  return u64(sms) * u64(per_sm > 0 ? per_sm : 1) * 2 * 256 * kWide;
}

void launch_histograms_wide(const u8* bins, u64 bin_stride, u32 F, bool quantized_gh, const TreeArrays* trees,
                            const Scales* scales, const HistTask* tasks, u32 ntasks, u32* counter, i64* hist,
                            cudaStream_t s, const u32* ntasks_dev, const HistLayout* layout, i64* scratch,
                            u64 scratch_elems, int bulk, u32* status, u32 bulk_status_bit, const HistBinsMap* map) {
  if (!ntasks && !ntasks_dev) return;
  const HistLayout lay = layout ? *layout : HistLayout{F, u64(F) * 2 * kMaxBins, 0};
  need(lay.fg > 0, "histogram layout needs a positive feature group size");
  const HistArgs a{bins, bin_stride, F, ntasks, ntasks_dev, trees, scales, tasks, counter, hist, lay};
  if (bulk == 2) {
    if (quantized_gh) launch_hist_bulk_variant<true, true>(a, scratch, scratch_elems, status, bulk_status_bit, map, s);
    else launch_hist_bulk_variant<false, true>(a, scratch, scratch_elems, status, bulk_status_bit, map, s);
  } else if (bulk == 1) {
    if (quantized_gh) launch_hist_bulk_variant<true, false>(a, scratch, scratch_elems, status, bulk_status_bit, map, s);
    else launch_hist_bulk_variant<false, false>(a, scratch, scratch_elems, status, bulk_status_bit, map, s);
  } else if (quantized_gh) {
    launch_hist_wide_variant<true>(a, scratch, scratch_elems, s);
  } else {
    launch_hist_wide_variant<false>(a, scratch, scratch_elems, s);
  }
  after_launch("histograms");
}

void encode_hist_bins_map(const u8* bins, u64 stride, u64 rows, HistBinsMap* out) {
  need((reinterpret_cast<uintptr_t>(bins) & 15u) == 0 && stride % 16 == 0 && stride > 0,
       "internal error: a tensor map needs 16-byte aligned bin rows");
  need(rows > 0 && rows <= 0x7fffffffull, "internal error: tensor map rows out of range");
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q{};
    void* fn = nullptr;
    DP_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q));
    need(q == cudaDriverEntryPointSuccess && fn, "cuTensorMapEncodeTiled is not available from the driver");
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const u32 box = u32(stride < u64(kWide) ? stride : u64(kWide));
  const cuuint64_t dims[2] = {stride, rows};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t boxdim[2] = {box, 1};
  const cuuint32_t estride[2] = {1, 1};
  CUtensorMap m{};
  const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<u8*>(bins), dims, strides, boxdim,
                            estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  need(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed for the bin matrix (" + std::to_string(int(r)) + ")");
  static_assert(sizeof(m) == sizeof(out->desc), "tensor map size");
  std::memcpy(out->desc, &m, sizeof m);
  out->bins = bins;
  out->stride = stride;
  out->box = box;
}

u64 hist_chunk_rows(u64 total_rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const u64 target = u64(sms) * 4;  // about four tasks per SM, balanced by the task queue
  const u64 chunk = (total_rows + target - 1) / target;
  return chunk < 2048 ? 2048 : chunk;
}

}  // namespace dp
