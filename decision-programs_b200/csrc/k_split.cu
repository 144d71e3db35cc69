// Split evaluation: for every open node, the best (feature, bin, missing
// direction) by second-order gain (Chen & Guestrin 2016):
//   gain = 0.5 * (s(GL,HL) + s(GR,HR) - s(G,H)) - gamma,  s(G,H) = T(G)^2/(H+lambda)
// A warp scans one feature: lane l owns bins [8l, 8l+8) and the warp-level
// exclusive scan of the lanes' int64 sums gives every prefix exactly.  Ties
// resolve to the lowest (feature, bin, default_left), i.e. the first maximum
// in scan order, at every reduction level.
#include "kernels.h"

namespace dp {

namespace {

constexpr int kEvalThreads = 256;

struct Best {
  double gain;
  i64 gl, hl;
  i32 f, b, d;
};

__device__ __forceinline__ bool better(const Best& a, const Best& c) {
  if (a.gain > c.gain) return true;
  if (!(a.gain == c.gain)) return false;
  if (a.f != c.f) return a.f < c.f;
  if (a.b != c.b) return a.b < c.b;
  return a.d < c.d;
}

__device__ __forceinline__ Best shfl_best(const Best& v, int src) {
  Best o;
  o.gain = __shfl_sync(0xffffffffu, v.gain, src);
  o.gl = __shfl_sync(0xffffffffu, v.gl, src);
  o.hl = __shfl_sync(0xffffffffu, v.hl, src);
  o.f = __shfl_sync(0xffffffffu, v.f, src);
  o.b = __shfl_sync(0xffffffffu, v.b, src);
  o.d = __shfl_sync(0xffffffffu, v.d, src);
  return o;
}

// Best candidate of one (node, feature chunk) work item, written to cand[w].
__device__ __forceinline__ void eval_item(u32 w, i64* hist, u32 F, const u16* __restrict__ nbins,
                                          const u8* __restrict__ has_missing, const EvalNode* __restrict__ nodes,
                                          const Scales* __restrict__ scales, const SplitParams& p, u32 nchunks,
                                          SplitCand* __restrict__ cand, u32 fstride, u32 f_base,
                                          const u32* __restrict__ fmask, u32 mask_words,
                                          const i64* __restrict__ parent, int store_derived) {
  __shared__ Best wbest[kEvalThreads / 32];
  __shared__ longlong2 stage[kEvalThreads / 32][kMaxBins];  // one 4 KB transpose stage per warp
  const u32 node = w / nchunks, chunk = w % nchunks;
  const EvalNode nd = nodes[node];
  const Scales sc = scales[nd.tree];
  const double isg = 1.0 / double(sc.sg), ish = 1.0 / double(sc.sh);
  const double G = double(nd.gq) * isg, H = double(nd.hq) * ish;
  const double sp = node_score(G, H, p);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  Best best{-HUGE_VAL, 0, 0, -1, -1, 0};
  const u32 f_end = min(F, (chunk + 1) * kEvalFeatureChunk);
  for (u32 f = chunk * kEvalFeatureChunk + warp; f < f_end; f += kEvalThreads / 32) {
    const int nb = nbins[f];
    if (nb < 2) continue;
    // Coalesced loads (lane l takes bins 32j + l), a derived sibling formed
    // and stored in that order (parent - built sibling, stored for the next
    // level whatever this node's feature mask), then a transpose through the
    // warp's shared-memory stage so that lane l holds bins [8l, 8l + 8) for
    // the scan.  The stage is swizzled (16-byte chunk c at c ^ ((c >> 3) & 7))
    // so that both the row-wise writes and the column-wise reads of eight
    // consecutive lanes hit eight distinct bank groups.
    i64* hf = hist + (u64(nd.slot) * fstride + f) * (2 * kMaxBins);
    longlong2 x[8];
    if (nd.par != kNoSlot) {
      const longlong2* pv =
          reinterpret_cast<const longlong2*>(parent + (u64(nd.par) * fstride + f) * (2 * kMaxBins)) + lane;
      const longlong2* sv =
          reinterpret_cast<const longlong2*>(hist + (u64(nd.small) * fstride + f) * (2 * kMaxBins)) + lane;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const longlong2 a = pv[32 * j], b = sv[32 * j];
        x[j] = make_longlong2(a.x - b.x, a.y - b.y);
      }
      if (store_derived) {
        longlong2* dv = reinterpret_cast<longlong2*>(hf) + lane;
#pragma unroll
        for (int j = 0; j < 8; ++j) dv[32 * j] = x[j];
      }
    } else {
      const longlong2* v = reinterpret_cast<const longlong2*>(hf) + lane;
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = v[32 * j];
    }
    if (fmask) {
      const u32 gf = f_base + f;
      if (!((fmask[u64(node) * mask_words + (gf >> 5)] >> (gf & 31u)) & 1u)) continue;
    }
    {
      longlong2* st = stage[warp];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const u32 c = 32u * j + u32(lane);
        st[c ^ ((c >> 3) & 7u)] = x[j];
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const u32 c = 8u * u32(lane) + j;
        x[j] = st[c ^ ((c >> 3) & 7u)];
      }
      __syncwarp();  // the stage is rewritten by the warp's next feature
    }
    const bool hm = has_missing[f] != 0;
    // the missing code is bin 255: lane 31's last pair
    const i64 gm31 = __shfl_sync(0xffffffffu, x[7].x, 31), hm31 = __shfl_sync(0xffffffffu, x[7].y, 31);
    const i64 gm = hm ? gm31 : 0, hmq = hm ? hm31 : 0;
    i64 sg_l = 0, sh_l = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (8 * lane + j >= nb) x[j] = make_longlong2(0, 0);  // missing bin and empty tail excluded
      sg_l += x[j].x;
      sh_l += x[j].y;
    }
    // exclusive warp scan of the lane sums
    i64 eg = sg_l, eh = sh_l;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const i64 ug = __shfl_up_sync(0xffffffffu, eg, o), uh = __shfl_up_sync(0xffffffffu, eh, o);
      if (lane >= o) { eg += ug; eh += uh; }
    }
    eg -= sg_l;
    eh -= sh_l;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      eg += x[j].x;
      eh += x[j].y;
      const int b = 8 * lane + j;
      if (b > nb - 2) continue;
#pragma unroll
      for (int d = 0; d < 2; ++d) {
        if (d == 1 && !hm) break;
        const i64 glq = eg + (d ? gm : 0), hlq = eh + (d ? hmq : 0);
        const i64 grq = nd.gq - glq, hrq = nd.hq - hlq;
        const double gain = split_gain(double(glq) * isg, double(hlq) * ish, double(grq) * isg,
                                       double(hrq) * ish, sp, p);
        const Best c{gain, glq, hlq, i32(f_base + f), b, d};
        if (better(c, best)) best = c;
      }
    }
  }
  // warp reduction, then block reduction; `better` breaks ties by index
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const Best other = shfl_best(best, lane ^ o);
    if (better(other, best)) best = other;
  }
  if (lane == 0) wbest[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    Best b = wbest[0];
    for (int wi = 1; wi < kEvalThreads / 32; ++wi)
      if (better(wbest[wi], b)) b = wbest[wi];
    SplitCand out;
    out.gain = b.gain;
    out.gl = b.gl;
    out.hl = b.hl;
    out.feature = b.f;
    out.bin = b.b;
    out.default_left = b.d;
    out.pad = 0;
    cand[w] = out;
  }
  __syncthreads();  // wbest is reused by the next work item of this block
}

__global__ void __launch_bounds__(kEvalThreads) k_eval(i64* hist, u32 F,
                                                       const u16* __restrict__ nbins,
                                                       const u8* __restrict__ has_missing,
                                                       const EvalNode* __restrict__ nodes,
                                                       const Scales* __restrict__ scales, SplitParams p, u32 nchunks,
                                                       SplitCand* __restrict__ cand) {
  eval_item(blockIdx.x, hist, F, nbins, has_missing, nodes, scales, p, nchunks, cand, F, 0, nullptr, 0, nullptr, 0);
}

// Node count in device memory: a fixed grid walks the work items.
__global__ void __launch_bounds__(kEvalThreads, 4) k_eval_dev(i64* hist, u32 F,
                                                           const u16* __restrict__ nbins,
                                                           const u8* __restrict__ has_missing,
                                                           const EvalNode* __restrict__ nodes,
                                                           const Scales* __restrict__ scales, SplitParams p,
                                                           u32 nchunks, const u32* __restrict__ nnodes,
                                                           SplitCand* __restrict__ cand, u32 fstride, u32 f_base,
                                                           const u32* __restrict__ fmask, u32 mask_words,
                                                           const i64* __restrict__ parent, int store_derived) {
  const u32 items = *nnodes * nchunks;
  for (u32 w = blockIdx.x; w < items; w += gridDim.x)
    eval_item(w, hist, F, nbins, has_missing, nodes, scales, p, nchunks, cand, fstride, f_base, fmask, mask_words,
              parent, store_derived);
}

__global__ void k_reduce_cands(const SplitCand* __restrict__ cand, u32 nnodes_host, const u32* __restrict__ nnodes_dev,
                               u32 nchunks, SplitCand* __restrict__ best) {
  const u32 nnodes = nnodes_dev ? *nnodes_dev : nnodes_host;
  for (u32 n = blockIdx.x * blockDim.x + threadIdx.x; n < nnodes; n += gridDim.x * blockDim.x) {
  SplitCand b = cand[u64(n) * nchunks];
  for (u32 c = 1; c < nchunks; ++c) {
    const SplitCand x = cand[u64(n) * nchunks + c];
    // chunks hold increasing features, so on equal gain the earlier one wins
    if (x.gain > b.gain) b = x;
  }
  best[n] = b;
  }
}

}  // namespace

void launch_eval_splits(const i64* hist, u32 F, const u16* nbins, const u8* has_missing, const EvalNode* nodes,
                        u32 nnodes, const Scales* scales, SplitParams p, SplitCand* cand, SplitCand* best,
                        cudaStream_t s) {
  if (!nnodes) return;
  const u32 nchunks = (F + kEvalFeatureChunk - 1) / kEvalFeatureChunk;
  k_eval<<<nnodes * nchunks, kEvalThreads, 0, s>>>(const_cast<i64*>(hist), F, nbins, has_missing, nodes, scales, p,
                                                   nchunks, cand);
  after_launch("eval_splits");
  k_reduce_cands<<<(nnodes + 127) / 128, 128, 0, s>>>(cand, nnodes, nullptr, nchunks, best);
  after_launch("reduce_splits");
}

void launch_eval_candidates_dev(const i64* hist, u32 F, const u16* nbins, const u8* has_missing,
                                const EvalNode* nodes, const u32* nnodes_dev, const Scales* scales, SplitParams p,
                                SplitCand* cand, u32 nchunks, cudaStream_t s, u32 fstride, u32 f_base,
                                const u32* fmask, u32 mask_words, const i64* parent_hist, int store_derived) {
  need(nchunks >= 1 && nchunks * kEvalFeatureChunk >= F, "candidate chunks do not cover the features");
  int dev = 0, sms = 148;
  DP_CUDA(cudaGetDevice(&dev));
  DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  k_eval_dev<<<sms * 8, kEvalThreads, 0, s>>>(const_cast<i64*>(hist), F, nbins, has_missing, nodes, scales, p,
                                               nchunks, nnodes_dev, cand, fstride ? fstride : F, f_base, fmask,
                                               mask_words, parent_hist, store_derived);
  after_launch("eval_splits");
}

}  // namespace dp
