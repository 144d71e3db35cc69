// Tree-ensemble prediction (see predict.h).  One thread per (row, class);
// consecutive threads take consecutive rows of one class, so a warp walks the
// same trees.  The rows a warp reads stay in L1 while it walks.
#include "predict.h"

namespace dp {

namespace {

__global__ void __launch_bounds__(256) k_predict(const float* __restrict__ x, u64 R, u64 stride, int has_mv, float mv,
                                                 const PredNode* __restrict__ nodes, const u32* __restrict__ tree_off,
                                                 const u32* __restrict__ tree_class, u32 t_begin, u32 t_end, int K,
                                                 const float* __restrict__ base, float* __restrict__ margin,
                                                 u32* __restrict__ bad) {
  const u64 n = R * u64(K);
  for (u64 idx = u64(blockIdx.x) * blockDim.x + threadIdx.x; idx < n; idx += u64(gridDim.x) * blockDim.x) {
    const u32 k = u32(idx / R);
    const u64 r = idx - u64(k) * R;
    const float* xr = x + r * stride;
    float m = base[k];
    for (u32 t = t_begin; t < t_end; ++t) {
      if (tree_class[t] != k) continue;
      const u32 off = tree_off[t], size = tree_off[t + 1] - off;
      const PredNode* tn = nodes + off;
      PredNode nd = tn[0];
      u32 steps = 0;
      while (nd.left >= 0) {
        if (++steps > size) {  // a cycle: the model is malformed
          atomicOr(bad, 1u);
          break;
        }
        const float v = __ldg(xr + (nd.feat_dl & 0x7fffffffu));
        const bool miss = isnan(v) || (has_mv && v == mv);
        const i32 next = miss ? ((nd.feat_dl >> 31) ? nd.left : nd.right) : (v < nd.cond ? nd.left : nd.right);
        nd = tn[next];
      }
      m = m + nd.cond;
    }
    margin[r * u64(K) + k] = m;
  }
}

__global__ void __launch_bounds__(256) k_transform(int objective, int K, const float* __restrict__ margin, u64 R,
                                                   float* __restrict__ out) {
  for (u64 r = u64(blockIdx.x) * blockDim.x + threadIdx.x; r < R; r += u64(gridDim.x) * blockDim.x) {
    const float* m = margin + r * u64(K);
    if (objective == kSquaredError) {
      out[r] = m[0];
    } else if (objective == kLogistic) {
      out[r] = float(1.0 / (1.0 + dp_exp(-double(m[0]))));
    } else if (objective == kSoftprob) {
      double mx = m[0];
      for (int k = 1; k < K; ++k) mx = double(m[k]) > mx ? double(m[k]) : mx;
      double s = 0.0;
      for (int k = 0; k < K; ++k) s = s + dp_exp(double(m[k]) - mx);
      for (int k = 0; k < K; ++k) out[r * u64(K) + k] = float(dp_exp(double(m[k]) - mx) / s);
    } else {
      int best = 0;
      for (int k = 1; k < K; ++k)
        if (m[k] > m[best]) best = k;
      out[r] = float(best);
    }
  }
}

int blocks_for(u64 n) {
  int dev = 0, sms = 148;
  DP_CUDA(cudaGetDevice(&dev));
  DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const u64 want = (n + 255) / 256, cap = u64(sms) * 16;
  return int(want < cap ? (want ? want : 1) : cap);
}

}  // namespace

void launch_predict_margins(const float* x, u64 R, u64 stride, bool has_mv, float mv, const PredNode* nodes,
                            const u32* tree_off, const u32* tree_class, u32 t_begin, u32 t_end, int K,
                            const float* base, float* margin, u32* bad, cudaStream_t s) {
  if (!R) return;
  k_predict<<<blocks_for(R * u64(K)), 256, 0, s>>>(x, R, stride, int(has_mv), mv, nodes, tree_off, tree_class,
                                                    t_begin, t_end, K, base, margin, bad);
  after_launch("predict");
}

void launch_predict_transform(int objective, int K, const float* margin, u64 R, float* out, cudaStream_t s) {
  if (!R) return;
  k_transform<<<blocks_for(R), 256, 0, s>>>(objective, K, margin, R, out);
  after_launch("predict_transform");
}

}  // namespace dp
