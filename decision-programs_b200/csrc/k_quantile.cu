// Quantile cuts and uint8 binning.
//
// The cut rule (per feature, over every non-missing value of every rank's
// rows, -0.0 folded into +0.0):
//   B_f = min(max_bin, 256, 255 if the column has a missing value);
//   <= B_f distinct values  -> every distinct value except the minimum is a boundary;
//   otherwise               -> boundary k (k = 1..B_f-1) is the value of rank
//                              floor(k n / B_f) in sorted order, deduplicated,
//                              the minimum excluded.
//   bin(x) = number of boundaries <= x; a missing value gets code 255.
// Splitting at bin b sends bin <= b left, i.e. x < boundary_b, matching the
// reference's routing `x < split_condition` (native/class_tree_runtime_compare.cu:47).
//
// The order statistics are found exactly, without sorting, by radix
// selection on the monotone 32-bit key of each value: a count per 16-bit
// prefix, then two 8-bit refinements restricted to at most 256 active
// prefixes per feature (the prefixes that contain a wanted rank, or all
// non-empty prefixes while the column may have <= B_f distinct values).
// Each pass streams the fp32 matrix once with coalesced loads; counts are
// integer, so sharded ranks reach identical cuts after summing them.
#include <vector>

#include "comm.h"
#include "kernels.h"
#include "quantile.h"

namespace dp {

namespace {

constexpr int kSlots = 256;
constexpr int kTile = 32;  // features per block in the counting passes

struct FeatState {
  u64 n;           // non-missing values (all ranks)
  u32 B;           // bin budget
  u32 mode;        // 1: all distinct values still tracked; 0: quantile targets only
  u32 nact;        // active prefixes
  u32 nb;          // final: boundaries + 1
  u32 prefix[kSlots];
  u64 base[kSlots];  // values below the prefix
  u64 cnt[kSlots];   // values with the prefix
};

__device__ __forceinline__ u32 fkey(float v) {
  if (v == 0.0f) v = 0.0f;
  const u32 u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float keyf(u32 k) {
  const u32 u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
__device__ __forceinline__ bool missing(float v, int has_mv, float mv) { return isnan(v) || (has_mv && v == mv); }

// Does [base, base+cnt) contain rank 0 or a target rank floor(k n / B), 1 <= k < B?
__device__ __forceinline__ bool holds_target(u64 base, u64 cnt, u64 n, u32 B) {
  if (cnt == 0) return false;
  if (base == 0) return true;
  const u64 klo = (base * B + n - 1) / n;
  u64 khi = ((base + cnt) * B + n - 1) / n - 1;
  if (khi > B - 1) khi = B - 1;
  return klo <= khi;
}

constexpr int kUnroll = 4;  // rows of loads in flight per thread

// Pass 1: count per (feature, 16-bit key prefix).  Lane = feature of a
// 32-feature tile, warp = row: each warp load is one contiguous 128-byte run.
// Infinite values (not the missing value) are flagged in bad[0].
__global__ void __launch_bounds__(256) k_count16(const float* __restrict__ x, u64 R, u32 F, u64 stride, int has_mv,
                                                 float mv, u32* __restrict__ cnt, u32* __restrict__ bad) {
  const u32 ftiles = (F + kTile - 1) / kTile;
  const u32 ft = blockIdx.y % ftiles;
  const u32 f = ft * kTile + (threadIdx.x & 31);
  const u64 step = u64(gridDim.x) * (blockDim.x / 32);
  u32* c = cnt + u64(f) * 65536;
  bool inf = false;
  if (f < F) {
    for (u64 r0 = u64(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); r0 < R; r0 += kUnroll * step) {
      float v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const u64 r = r0 + u * step;
        v[u] = r < R ? x[r * stride + f] : __int_as_float(0x7fc00000);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (missing(v[u], has_mv, mv)) continue;
        inf |= isinf(v[u]);
        atomicAdd(c + (fkey(v[u]) >> 16), 1u);
      }
    }
  }
  if (bad && __any_sync(0xffffffffu, inf) && (threadIdx.x & 31) == 0) atomicOr(bad, 1u);
}

// Block-wide exclusive scan of one value per thread (blockDim.x <= 1024);
// *total receives the block sum.  Ends with a barrier so it can be reused.
__device__ u64 block_excl_scan(u64 v, u64* total) {
  __shared__ u64 ws[33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = int(blockDim.x >> 5);
  u64 incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const u64 t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) ws[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const u64 w = lane < nwarps ? ws[lane] : 0;
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
  if (total) *total = tot;
  return out;
}

// After pass 1 (one block of 1024 threads per feature): totals, mode and the
// active 16-bit prefixes.
__global__ void __launch_bounds__(1024) k_select16(const u32* __restrict__ cnt, u64 R_total, int max_bin,
                                                   FeatState* __restrict__ st) {
  const u32 f = blockIdx.x;
  const u32* c = cnt + u64(f) * 65536;
  constexpr int kPer = 65536 / 1024;
  const int t = threadIdx.x;
  u64 my = 0;
  u32 nz = 0;
  for (int j = 0; j < kPer; ++j) {
    const u32 v = c[t * kPer + j];
    my += v;
    nz += v != 0;
  }
  u64 n = 0;
  const u64 before = block_excl_scan(my, &n);
  u64 nz_total = 0;
  block_excl_scan(nz, &nz_total);
  const bool has_missing = n < R_total;
  u32 B = u32(max_bin < 256 ? max_bin : 256);
  if (has_missing && B > 255) B = 255;
  const u32 mode = nz_total <= B ? 1u : 0u;
  // mark active buckets, then compact them in order
  u32 act = 0;
  if (n > 0) {
    u64 cum = before;
    for (int j = 0; j < kPer; ++j) {
      const u32 v = c[t * kPer + j];
      if (v && (mode ? true : holds_target(cum, v, n, B))) ++act;
      cum += v;
    }
  }
  u64 nact = 0;
  u64 slot = block_excl_scan(act, &nact);
  if (n > 0) {
    u64 cum = before;
    for (int j = 0; j < kPer; ++j) {
      const u32 v = c[t * kPer + j];
      if (v && (mode ? true : holds_target(cum, v, n, B))) {
        st[f].prefix[slot] = u32(t * kPer + j);
        st[f].base[slot] = cum;
        st[f].cnt[slot] = v;
        ++slot;
      }
      cum += v;
    }
  }
  if (t == 0) {
    st[f].n = n;
    st[f].B = B;
    st[f].mode = mode;
    st[f].nact = u32(nact);
    st[f].nb = 1;
  }
}

// Passes 2 and 3: count the next 8-bit digit of values whose prefix is active.
// shift = bits below the active prefix (16, then 8).  The active lists sit in
// shared memory with a row stride of kSlots + 1 words, so the 32 lanes of a
// warp (32 features) searching at the same index hit 32 different banks.
__global__ void __launch_bounds__(256) k_count8(const float* __restrict__ x, u64 R, u32 F, u64 stride, int has_mv,
                                                float mv, const FeatState* __restrict__ st, int shift,
                                                u32* __restrict__ cnt) {
  __shared__ u32 pre[kTile][kSlots + 1];
  __shared__ u32 nact[kTile];
  const u32 ftiles = (F + kTile - 1) / kTile;
  const u32 ft = blockIdx.y % ftiles;
  for (int i = threadIdx.x; i < kTile * kSlots; i += blockDim.x) {
    const u32 fl = i / kSlots, s = i % kSlots, f = ft * kTile + fl;
    pre[fl][s] = (f < F && s < st[f].nact) ? st[f].prefix[s] : 0xffffffffu;
  }
  if (threadIdx.x < kTile) {
    const u32 f = ft * kTile + threadIdx.x;
    nact[threadIdx.x] = f < F ? st[f].nact : 0;
  }
  __syncthreads();
  const u32 fl = threadIdx.x & 31;
  const u32 f = ft * kTile + fl;
  const u32 na = f < F ? nact[fl] : 0;
  if (na == 0) return;
  const u32* P = pre[fl];
  const u64 step = u64(gridDim.x) * (blockDim.x / 32);
  for (u64 r0 = u64(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); r0 < R; r0 += kUnroll * step) {
    float v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const u64 r = r0 + u * step;
      v[u] = r < R ? x[r * stride + f] : __int_as_float(0x7fc00000);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (missing(v[u], has_mv, mv)) continue;
      const u32 k = fkey(v[u]);
      const u32 p = k >> shift;
      // first active prefix >= p (entries past nact hold 0xffffffff)
      u32 pos = 0;
#pragma unroll
      for (u32 w = kSlots / 2; w > 0; w >>= 1)
        if (P[pos + w - 1] < p) pos += w;
      if (pos < na && P[pos] == p) atomicAdd(cnt + (u64(f) * kSlots + pos) * 256 + ((k >> (shift - 8)) & 0xffu), 1u);
    }
  }
}

// After a refinement pass (one block of 256 threads per feature; thread = slot).
__global__ void __launch_bounds__(256) k_select8(const u32* __restrict__ cnt, FeatState* __restrict__ st) {
  const u32 f = blockIdx.x;
  FeatState& S = st[f];
  const u32 s = threadIdx.x;
  const u32 na = S.nact;
  const u64 n = S.n;
  const u32 B = S.B;
  const u32* c = cnt + (u64(f) * kSlots + s) * 256;
  u32 nz = 0;
  if (s < na)
    for (int d = 0; d < 256; ++d) nz += c[d] != 0;
  __shared__ u32 new_prefix[kSlots];
  __shared__ u64 new_base[kSlots], new_cnt[kSlots];
  u64 nz_total = 0;
  block_excl_scan(nz, &nz_total);
  const u32 mode = (S.mode && nz_total <= B) ? 1u : 0u;
  u32 act = 0;
  u32 my_prefix = 0;
  u64 my_base = 0;
  if (s < na) {
    my_prefix = S.prefix[s];
    my_base = S.base[s];
    u64 cum = my_base;
    for (int d = 0; d < 256; ++d) {
      const u32 v = c[d];
      if (v && (mode ? true : holds_target(cum, v, n, B))) ++act;
      cum += v;
    }
  }
  u64 nact = 0;
  u64 slot = block_excl_scan(act, &nact);
  if (s < na) {
    u64 cum = my_base;
    for (int d = 0; d < 256; ++d) {
      const u32 v = c[d];
      if (v && (mode ? true : holds_target(cum, v, n, B))) {
        new_prefix[slot] = (my_prefix << 8) | u32(d);
        new_base[slot] = cum;
        new_cnt[slot] = v;
        ++slot;
      }
      cum += v;
    }
  }
  __syncthreads();
  if (s < nact) {
    S.prefix[s] = new_prefix[s];
    S.base[s] = new_base[s];
    S.cnt[s] = new_cnt[s];
  }
  if (s == 0) {
    S.mode = mode;
    S.nact = u32(nact);
  }
}

// Final boundaries from full 32-bit keys (one thread per feature).
__global__ void k_finalize(FeatState* __restrict__ st, u32 F, u64 R_total, float* __restrict__ cut,
                           u16* __restrict__ nbins, u8* __restrict__ has_missing) {
  const u32 f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= F) return;
  FeatState& S = st[f];
  float* cf = cut + u64(f) * 256;
  u32 nb = 0;
  if (S.n > 0 && S.nact > 0) {
    if (S.mode) {
      for (u32 i = 1; i < S.nact; ++i) cf[nb++] = keyf(S.prefix[i]);
    } else {
      const u32 min_key = S.prefix[0];
      u32 e = 0, last = 0;
      for (u32 k = 1; k < S.B; ++k) {
        const u64 rank = (u64(k) * S.n) / S.B;
        while (e + 1 < S.nact && S.base[e] + S.cnt[e] <= rank) ++e;
        const u32 key = S.prefix[e];
        if (key == min_key) continue;
        if (nb > 0 && key <= last) continue;
        cf[nb++] = keyf(key);
        last = key;
      }
    }
  }
  for (u32 i = nb; i < 256; ++i) cf[i] = 0.0f;
  S.nb = nb + 1;
  nbins[f] = u16(nb + 1);
  has_missing[f] = S.n < R_total ? 1 : 0;
}

// bins[r][f] = #boundaries <= x (255 for missing); padding columns are zero.
// Boundaries past a feature's last one read +inf, so a fixed eight-step
// search counts the boundaries <= x; rows of kSlots + 1 words keep the lanes'
// lookups in distinct banks.  A block bins 32-row tiles of a 32-feature
// slice: lane = feature, warp = rows warp + 8u.  With bins_blk set, the tile
// is also written in the 32-row blocked layout
// bins_blk[r / 32][f][r % 32] (see launch_bin_matrix) through a shared-memory
// transpose, as 4-byte stores.
__global__ void __launch_bounds__(256) k_bin(const float* __restrict__ x, u64 R, u32 F, u64 stride, int has_mv,
                                             float mv, const float* __restrict__ cut, const u16* __restrict__ nbins,
                                             u8* __restrict__ bins, u64 bstride, u8* __restrict__ bins_blk) {
  __shared__ float c[kTile][kSlots + 1];
  __shared__ __align__(4) u8 tile[kTile][36];  // [feature][row of the tile], padded
  const u32 ftiles = (u32(bstride) + kTile - 1) / kTile;
  const u32 ft = blockIdx.y % ftiles;
  for (int i = threadIdx.x; i < kTile * kSlots; i += blockDim.x) {
    const u32 fl = i / kSlots, j = i % kSlots, f = ft * kTile + fl;
    c[fl][j] = (f < F && j + 1 < nbins[f]) ? cut[u64(f) * kSlots + j] : __int_as_float(0x7f800000);
  }
  __syncthreads();
  const u32 fl = threadIdx.x & 31, f = ft * kTile + fl, warp = threadIdx.x >> 5;
  const float* C = c[fl];
  const u64 ntiles = (R + 31) / 32;
  for (u64 tb = blockIdx.x; tb < ntiles; tb += gridDim.x) {
    float v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const u64 r = tb * 32 + warp + 8 * u;
      v[u] = (r < R && f < F) ? x[r * stride + f] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const u32 rl = warp + 8 * u;
      const u64 r = tb * 32 + rl;
      u8 b = 0;
      if (r < R && f < F) {
        if (missing(v[u], has_mv, mv)) {
          b = kMissingBin;
        } else {
          u32 pos = 0;
#pragma unroll
          for (u32 w = kSlots / 2; w > 0; w >>= 1)
            if (C[pos + w - 1] <= v[u]) pos += w;
          b = u8(pos);
        }
      }
      if (r < R && f < bstride) bins[r * bstride + f] = b;
      tile[fl][rl] = b;
    }
    if (bins_blk) {
      __syncthreads();
      const u32 tf = threadIdx.x >> 3, tr = (threadIdx.x & 7) * 4, gf = ft * kTile + tf;
      if (gf < F)
        *reinterpret_cast<u32*>(bins_blk + tb * (32 * u64(F)) + u64(gf) * 32 + tr) =
            *reinterpret_cast<const u32*>(&tile[tf][tr]);
      __syncthreads();
    }
  }
}

unsigned row_blocks(u64 R, u32 rows_per_block, u32 ftiles) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  u64 want = (R + rows_per_block - 1) / rows_per_block;
  u64 cap = (u64(sms) * 16 + ftiles - 1) / ftiles;
  if (cap < 1) cap = 1;
  return unsigned(want < cap ? (want ? want : 1) : cap);
}

}  // namespace

void launch_prefix_counts(const float* x, u64 R, u32 F, u64 stride, bool has_mv, float mv, u32* cnt, u32* bad,
                          cudaStream_t s) {
  if (!R || !F) return;
  const u32 ftiles = (F + kTile - 1) / kTile;
  const dim3 grid(row_blocks(R, 8, ftiles), ftiles);
  k_count16<<<grid, 256, 0, s>>>(x, R, F, stride, int(has_mv), mv, cnt, bad);
  after_launch("cut_count16");
}

void compute_cuts(const float* x, u64 R, u32 F, u64 stride, int max_bin, bool has_mv, float mv, u64 R_total,
                  Comm* comm, const CutsDevice& out, cudaStream_t s, u32* prefix_counts) {
  need(F > 0, "cuts need at least one feature");
  need(R_total < (u64(1) << 32), "row count exceeds the 32-bit count range of the cut search");
  need(max_bin >= 2, "max_bin must be at least 2");
  const u32 ftiles = (F + kTile - 1) / kTile;
  const dim3 grid(row_blocks(R, 8, ftiles), ftiles);
  // scratch: the count words (the caller's prefix counts when given), then
  // the per-feature search state
  const u64 cnt_words = u64(F) * kPrefixBuckets;
  const u64 st_off = prefix_counts ? 0 : (cnt_words * sizeof(u32) + 255) / 256 * 256;
  DevBuf<u8> scratch(st_off + u64(F) * sizeof(FeatState));
  u32* cnt = prefix_counts ? prefix_counts : reinterpret_cast<u32*>(scratch.get());
  FeatState* st = reinterpret_cast<FeatState*>(scratch.get() + st_off);
  if (!prefix_counts) {
    DP_CUDA(cudaMemsetAsync(cnt, 0, cnt_words * sizeof(u32), s));
    launch_prefix_counts(x, R, F, stride, has_mv, mv, cnt, nullptr, s);
  }
  if (comm) comm->sum_u32(cnt, cnt_words, s);
  k_select16<<<F, 1024, 0, s>>>(cnt, R_total, max_bin, st);
  after_launch("cut_select16");
  for (int shift : {16, 8}) {
    DP_CUDA(cudaMemsetAsync(cnt, 0, u64(F) * kSlots * 256 * sizeof(u32), s));
    if (R) {
      k_count8<<<grid, 256, 0, s>>>(x, R, F, stride, int(has_mv), mv, st, shift, cnt);
      after_launch("cut_count8");
    }
    if (comm) comm->sum_u32(cnt, u64(F) * kSlots * 256, s);
    k_select8<<<F, 256, 0, s>>>(cnt, st);
    after_launch("cut_select8");
  }
  k_finalize<<<(F + 127) / 128, 128, 0, s>>>(st, F, R_total, out.cut, out.nbins, out.has_missing);
  after_launch("cut_finalize");
  // temporaries are freed after the stream drains
  DP_CUDA(cudaStreamSynchronize(s));
}

void launch_bin_matrix(const float* x, u64 R, u32 F, u64 stride, bool has_mv, float mv, const CutsDevice& cuts,
                       u8* bins, u64 bin_stride, cudaStream_t s, u8* bins_blk) {
  if (!R) return;
  const u32 ftiles = u32((bin_stride + kTile - 1) / kTile);
  const dim3 grid(row_blocks(R, 32, ftiles), ftiles);
  k_bin<<<grid, 256, 0, s>>>(x, R, F, stride, int(has_mv), mv, cuts.cut, cuts.nbins, bins, bin_stride, bins_blk);
  after_launch("bin_matrix");
}

}  // namespace dp
