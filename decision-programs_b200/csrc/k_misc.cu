// Objective gradients, quantiser scales, leaf/margin update and input checks.
//
// Gradients (per row, double precision, then rounded to float):
//   reg:squarederror          g = m - y,            h = 1
//   binary:logistic           p = 1/(1+e^-m),       g = p - y,  h = max(p(1-p), 1e-16)
//   multi:softprob / softmax  p_k = softmax(m)_k,   g_k = p_k - [y==k],
//                                                   h_k = max(2 p_k (1-p_k), 1e-16)
// These are the objectives the reference configures or that its drop-in
// callers need (native/class_native_training.cuh:60 hard-codes
// multi:softmax; BASELINE configs add binary:logistic and reg:squarederror).
#include "kernels.h"

namespace dp {

namespace {

constexpr int kSharedClasses = kMaxReducedClasses;

__device__ __forceinline__ u32 warp_max(u32 b) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
  return b;
}

// Maxima of |g| and h per class (float bits compare as unsigned for
// non-negative values): per-thread registers for one class, per-block shared
// counters for up to kSharedClasses classes, then either one global atomic
// per block and class (gmax / hmax zeroed before), or (part set) per-block
// maxima part[block][2K] that the last block to finish reduces into gmax /
// hmax and, with scales_out, into the scales; that block also returns *done
// to zero, so nothing has to be zeroed before the next launch.
__global__ void __launch_bounds__(256) k_gradients(int objective, int K, const float* __restrict__ margin,
                                                    const float* __restrict__ label, u64 R, float2* __restrict__ gh,
                                                    u32* gmax, u32* hmax, RowSample rs, u32* part, u32* done,
                                                    Scales* scales_out) {
  __shared__ u32 smg[kSharedClasses], smh[kSharedClasses];
  const bool sampling = rs.rate < 1.0;
  const u32 round = sampling ? *rs.round : 0u;
  auto kept = [&](u64 r, int k) {
    return !sampling || sample_uniform(sample_hash(rs.seed, round, u32(k), kSampleRow, rs.row0 + r, 0)) < rs.rate;
  };
  const bool shared_max = K <= kSharedClasses;
  for (int k = threadIdx.x; k < kSharedClasses; k += blockDim.x) { smg[k] = 0u; smh[k] = 0u; }
  __syncthreads();
  u32 lg = 0u, lh = 0u;  // this thread's maxima when K == 1
  const u64 step = u64(gridDim.x) * blockDim.x;
  for (u64 base = u64(blockIdx.x) * blockDim.x; base < R; base += step) {
    const u64 r = base + threadIdx.x;
    const bool valid = r < R;
    const double y = valid ? double(label[r]) : 0.0;
    if (objective == kSquaredError || objective == kLogistic) {
      if (valid) {
        float g, h;
        const double m = double(margin[r]);
        if (objective == kSquaredError) {
          g = float(m - y);
          h = 1.0f;
        } else {
          const double p = 1.0 / (1.0 + dp_exp(-m));
          g = float(p - y);
          h = float(fmax(p * (1.0 - p), 1e-16));
        }
        if (!kept(r, 0)) g = h = 0.f;
        gh[r] = make_float2(g, h);
        lg = max(lg, __float_as_uint(fabsf(g)));
        lh = max(lh, __float_as_uint(h));
      }
    } else {
      double mx = 0.0, s = 0.0;
      const float* m = margin + (valid ? r : 0) * u64(K);
      if (valid) {
        mx = double(m[0]);
        for (int k = 1; k < K; ++k) mx = fmax(mx, double(m[k]));
        for (int k = 0; k < K; ++k) s = s + dp_exp(double(m[k]) - mx);
      }
      for (int k = 0; k < K; ++k) {
        float g = 0.f, h = 0.f;
        if (valid) {
          const double pk = dp_exp(double(m[k]) - mx) / s;
          g = float(pk - (double(k) == y ? 1.0 : 0.0));
          h = float(fmax(2.0 * pk * (1.0 - pk), 1e-16));
          if (!kept(r, k)) g = h = 0.f;
          gh[u64(k) * R + r] = make_float2(g, h);
        }
        const u32 wg = warp_max(__float_as_uint(fabsf(g))), wh = warp_max(__float_as_uint(h));
        if ((threadIdx.x & 31) == 0 && (wg | wh)) {
          if (shared_max) { atomicMax(smg + k, wg); atomicMax(smh + k, wh); }
          else { atomicMax(gmax + k, wg); atomicMax(hmax + k, wh); }
        }
      }
    }
  }
  if (objective == kSquaredError || objective == kLogistic) {
    lg = warp_max(lg);
    lh = warp_max(lh);
    if ((threadIdx.x & 31) == 0) { atomicMax(smg, lg); atomicMax(smh, lh); }
  }
  __syncthreads();
  if (!part) {
    if (shared_max)
      for (int k = threadIdx.x; k < K; k += blockDim.x) {
        if (smg[k]) atomicMax(gmax + k, smg[k]);
        if (smh[k]) atomicMax(hmax + k, smh[k]);
      }
    return;
  }
  // per-block maxima ([2K][blocks]), then the last block reduces them
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    part[u64(k) * gridDim.x + blockIdx.x] = smg[k];
    part[u64(K + k) * gridDim.x + blockIdx.x] = smh[k];
  }
  if (!last_block(done, gridDim.x)) return;
  __shared__ u32 s_red[8 * 2 * kSharedClasses];
  __shared__ u32 s_max[2 * kSharedClasses];
  reduce_rows(part, u32(2 * K), gridDim.x, s_red, s_max, 0u, [](u32 x, u32 y) { return x > y ? x : y; });
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    smg[k] = s_max[k];
    smh[k] = s_max[K + k];
  }
  __syncthreads();
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    gmax[k] = smg[k];
    hmax[k] = smh[k];
    if (scales_out) {
      scales_out[k].sg = quant_scale(__uint_as_float(smg[k]), kGradBits);
      scales_out[k].sh = quant_scale(__uint_as_float(smh[k]), kHessBits);
    }
  }
}

__global__ void __launch_bounds__(256) k_quantize_gh(float2* gh, u64 R, int K, const Scales* __restrict__ sc) {
  const u64 n = R * u64(K);
  for (u64 i = u64(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += u64(gridDim.x) * blockDim.x) {
    const Scales s = sc[i / R];
    const float2 v = gh[i];
    reinterpret_cast<int2*>(gh)[i] = make_int2(quantize(v.x, s.sg), quantize(v.y, s.sh));
  }
}

__global__ void k_scales(int K, const u32* gmax, const u32* hmax, Scales* scales) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k < K) {
    scales[k].sg = quant_scale(__uint_as_float(gmax[k]), kGradBits);
    scales[k].sh = quant_scale(__uint_as_float(hmax[k]), kHessBits);
  }
}

// One block per leaf task; rows of a leaf are updated in place.
__global__ void __launch_bounds__(256) k_leaf_update(const LeafTask* __restrict__ tasks, u32 ntasks_host,
                                                      const u32* __restrict__ ntasks_dev, float* margin, u32 K) {
  const u32 n = ntasks_dev ? *ntasks_dev : ntasks_host;
  constexpr int kU = 4;  // rows in flight per thread
  for (u32 task = blockIdx.x; task < n; task += gridDim.x) {
    const LeafTask t = tasks[task];
    for (i64 i0 = t.begin + threadIdx.x; i0 < t.end; i0 += i64(blockDim.x) * kU) {
      u32 r[kU];
      float m[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const i64 i = i0 + i64(u) * blockDim.x;
        r[u] = i < t.end ? t.ridx[i] : 0xffffffffu;
      }
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (r[u] != 0xffffffffu) m[u] = margin[u64(r[u]) * K + t.klass];
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (r[u] != 0xffffffffu) margin[u64(r[u]) * K + t.klass] = m[u] + t.value;
    }
  }
}

__global__ void k_init_margins(float* __restrict__ margin, u64 n, int K, const float* __restrict__ base) {
  for (u64 i = u64(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += u64(gridDim.x) * blockDim.x)
    margin[i] = base[i % u64(K)];
}

__global__ void k_check_finite(const float* __restrict__ x, u64 R, u32 F, u64 stride, u32* bad) {
  const u64 n = R * F;
  bool any = false;
  for (u64 i = u64(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += u64(gridDim.x) * blockDim.x) {
    const u64 r = i / F, f = i - r * F;
    any |= isinf(x[r * stride + f]);
  }
  if (__any_sync(0xffffffffu, any) && (threadIdx.x & 31) == 0) atomicOr(bad, 1u);
}

__global__ void k_check_labels(const float* __restrict__ y, u64 R, int objective, int K, u32* bad) {
  bool any = false;
  for (u64 i = u64(blockIdx.x) * blockDim.x + threadIdx.x; i < R; i += u64(gridDim.x) * blockDim.x) {
    const float v = y[i];
    if (!isfinite(v)) any = true;
    else if (objective == kLogistic) any |= (v < 0.f || v > 1.f);
    else if (objective == kSoftprob || objective == kSoftmax) any |= (v < 0.f || v >= float(K) || v != floorf(v));
  }
  if (__any_sync(0xffffffffu, any) && (threadIdx.x & 31) == 0) atomicOr(bad, 1u);
}

constexpr int kCopySegs = 6;
struct CopySegs {
  const u32* src[kCopySegs];
  u32* dst[kCopySegs];
  u64 words[kCopySegs];
};

__global__ void __launch_bounds__(256) k_copy_words(CopySegs c) {
  const u64 step = u64(gridDim.x) * blockDim.x;
  for (int j = 0; j < kCopySegs; ++j)
    for (u64 i = u64(blockIdx.x) * blockDim.x + threadIdx.x; i < c.words[j]; i += step) c.dst[j][i] = c.src[j][i];
}

int grid_for(u64 n, int block) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const u64 want = (n + block - 1) / block;
  const u64 cap = u64(sms) * 8;
  return int(want < cap ? (want ? want : 1) : cap);
}

}  // namespace

void launch_gradients(int objective, int K, const float* margin, const float* label, u64 R, float2* gh,
                      u32* gmax_bits, u32* hmax_bits, cudaStream_t s, const RowSample& rs) {
  if (R == 0) return;
  need(rs.rate >= 1.0 || rs.round != nullptr, "row sampling needs the round counter");
  k_gradients<<<grid_for(R, 256), 256, 0, s>>>(objective, K, margin, label, R, gh, gmax_bits, hmax_bits, rs,
                                                nullptr, nullptr, nullptr);
  after_launch("gradients");
}

u32 gradient_blocks(u64 R) { return u32(grid_for(R, 256)); }

void launch_copy_words(const u32* const* src, u32* const* dst, const u64* words, int n, cudaStream_t s) {
  need(n >= 1 && n <= kCopySegs, "internal error: copy segment count");
  CopySegs c{};
  u64 most = 0;
  for (int j = 0; j < n; ++j) {
    c.src[j] = src[j];
    c.dst[j] = dst[j];
    c.words[j] = words[j];
    most = words[j] > most ? words[j] : most;
  }
  k_copy_words<<<grid_for(most, 256), 256, 0, s>>>(c);
  after_launch("copy_words");
}

void launch_gradients_reduced(int objective, int K, const float* margin, const float* label, u64 R, float2* gh,
                              u32* gmax_bits, u32* hmax_bits, u32* part, u32* done, Scales* scales, cudaStream_t s,
                              const RowSample& rs) {
  need(K <= kSharedClasses, "internal error: per-block gradient maxima hold at most 64 classes");
  need(rs.rate >= 1.0 || rs.round != nullptr, "row sampling needs the round counter");
  // one block at least (R == 0 included), so the maxima are always written
  k_gradients<<<grid_for(R, 256), 256, 0, s>>>(objective, K, margin, label, R, gh, gmax_bits, hmax_bits, rs, part,
                                                done, scales);
  after_launch("gradients");
}

void launch_scales(int K, const u32* gmax_bits, const u32* hmax_bits, Scales* scales, cudaStream_t s) {
  k_scales<<<(K + 127) / 128, 128, 0, s>>>(K, gmax_bits, hmax_bits, scales);
  after_launch("scales");
}

void launch_quantize_gh(float2* gh, u64 R, int K, const Scales* scales, cudaStream_t s) {
  if (!R) return;
  k_quantize_gh<<<grid_for(R * u64(K), 256), 256, 0, s>>>(gh, R, K, scales);
  after_launch("quantize_gh");
}

void launch_leaf_update(const LeafTask* tasks, u32 ntasks, float* margin, u32 K, cudaStream_t s) {
  if (!ntasks) return;
  k_leaf_update<<<ntasks, 256, 0, s>>>(tasks, ntasks, nullptr, margin, K);
  after_launch("leaf_update");
}

void launch_leaf_update_dev(const LeafTask* tasks, const u32* ntasks_dev, float* margin, u32 K, cudaStream_t s) {
  int dev = 0, sms = 148;
  DP_CUDA(cudaGetDevice(&dev));
  DP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  k_leaf_update<<<sms * 8, 256, 0, s>>>(tasks, 0, ntasks_dev, margin, K);
  after_launch("leaf_update");
}

void launch_init_margins(float* margin, u64 R, int K, const float* base, cudaStream_t s) {
  const u64 n = R * u64(K);
  if (!n) return;
  k_init_margins<<<grid_for(n, 256), 256, 0, s>>>(margin, n, K, base);
  after_launch("init_margins");
}

void launch_check_finite(const float* x, u64 R, u32 F, u64 stride, u32* bad, cudaStream_t s) {
  if (!R || !F) return;
  k_check_finite<<<grid_for(R * F, 256), 256, 0, s>>>(x, R, F, stride, bad);
  after_launch("check_finite");
}

void launch_check_labels(const float* y, u64 R, int objective, int K, u32* bad, cudaStream_t s) {
  if (!R) return;
  k_check_labels<<<grid_for(R, 256), 256, 0, s>>>(y, R, objective, K, bad);
  after_launch("check_labels");
}

std::atomic<u64>& launch_counter() {
  static std::atomic<u64> n{0};
  return n;
}

}  // namespace dp
