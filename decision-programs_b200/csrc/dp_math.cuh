// Arithmetic that must give the same bits on the host and on the GPU:
// exp, the gradient quantiser, split gain and leaf weight.  Every function
// uses only IEEE-754 correctly rounded operations (+ - * / fma rint ldexp) in
// a fixed order, and the library is compiled without FMA contraction, so host
// and device results are identical.
#pragma once
#include <cmath>
#include <cstdint>

#ifdef __CUDACC__
#define DP_HD __host__ __device__ __forceinline__
#else
#define DP_HD inline
#endif

namespace dp {

constexpr int kMissingBin = 255;
constexpr int kMaxBins = 256;
// Quantised gradient ranges: |q_g| <= 2^17 and 0 <= q_h <= 2^18.  With at most
// kWindowRows rows per shared-memory accumulation window, window sums satisfy
// |sum q_g| <= 16383 * 2^17 < 2^31 and sum q_h <= 16383 * 2^18 < 2^32, so
// 32-bit shared-memory counters are exact within a window.
constexpr int kGradBits = 17;
constexpr int kHessBits = 18;
constexpr int kWindowRows = 16383;

// e^x: Cody & Waite (1980) argument reduction x = k ln2 + r with ln2 split
// into a 24-bit head and a tail, the Taylor series of e^r to degree 13
// (|r| <= ln2/2) by Horner's rule with fused multiply-add, then 2^k scaling.
// Head = ln2 rounded to float; tail = ln2 - head (60-digit expansion);
// coefficients 1/n! rounded to double.
DP_HD double dp_exp(double x) {
  if (x != x) return x;
  if (x > 709.0) return HUGE_VAL;
  if (x < -745.0) return 0.0;
  const double kHead = 0.6931471824645996;
  const double kTail = -1.904654299957768e-09;
  const double kInvLn2 = 1.4426950408889634;
  const double k = rint(x * kInvLn2);
  const double hi = x - k * kHead;
  const double r = hi - k * kTail;
  double p = 1.0 / 6227020800.0;
  p = fma(p, r, 1.0 / 479001600.0);
  p = fma(p, r, 1.0 / 39916800.0);
  p = fma(p, r, 1.0 / 3628800.0);
  p = fma(p, r, 1.0 / 362880.0);
  p = fma(p, r, 1.0 / 40320.0);
  p = fma(p, r, 1.0 / 5040.0);
  p = fma(p, r, 1.0 / 720.0);
  p = fma(p, r, 1.0 / 120.0);
  p = fma(p, r, 1.0 / 24.0);
  p = fma(p, r, 1.0 / 6.0);
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  return ldexp(p, int(k));
}

// Power-of-two scale s with |v * s| < 2^bits for every |v| <= vmax.
DP_HD float quant_scale(float vmax, int bits) {
  if (!(vmax > 0.0f)) return 1.0f;
  int e = 0;
  frexpf(vmax, &e);
  e = e < -100 ? -100 : (e > 100 ? 100 : e);
  return ldexpf(1.0f, bits - e);
}

DP_HD std::int32_t quantize(float v, float s) { return std::int32_t(rintf(v * s)); }

struct SplitParams {
  double lambda = 1.0, alpha = 0.0, gamma = 0.0, min_child_weight = 1.0, eta = 0.3;
};

DP_HD double soft_threshold(double g, double alpha) {
  if (g > alpha) return g - alpha;
  if (g < -alpha) return g + alpha;
  return 0.0;
}

DP_HD double node_score(double g, double h, const SplitParams& p) {
  const double t = soft_threshold(g, p.alpha);
  return (t * t) / (h + p.lambda);
}

// Gain of one candidate, or -inf when the candidate violates a constraint.
DP_HD double split_gain(double GL, double HL, double GR, double HR, double parent_score, const SplitParams& p) {
  if (!(HL >= p.min_child_weight && HR >= p.min_child_weight && HL + p.lambda > 0.0 && HR + p.lambda > 0.0))
    return -HUGE_VAL;
  return ((node_score(GL, HL, p) + node_score(GR, HR, p)) - parent_score) * 0.5 - p.gamma;
}

// Leaf value stored in the model: float(-T(G)/(H+lambda) * eta).
DP_HD float leaf_weight(std::int64_t gq, std::int64_t hq, float sg, float sh, const SplitParams& p) {
  const double G = double(gq) * (1.0 / double(sg));
  const double H = double(hq) * (1.0 / double(sh));
  const double den = H + p.lambda;
  if (!(den > 0.0)) return 0.0f;
  const double w = -soft_threshold(G, p.alpha) / den;
  return float(w * p.eta);
}

// ---- sampling (subsample, colsample_*) -------------------------------------
// Counter-based random numbers, identical on the host and the device: the
// output function of SplitMix64 (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014) applied to a chain of key
// words (seed, round, kind and class, then two indices).
DP_HD std::uint64_t mix64(std::uint64_t z) {
  z ^= z >> 30;
  z *= 0xbf58476d1ce4e5b9ULL;
  z ^= z >> 27;
  z *= 0x94d049bb133111ebULL;
  z ^= z >> 31;
  return z;
}
enum SampleKind : std::uint32_t { kSampleRow = 1, kSampleTree = 2, kSampleLevel = 3, kSampleNode = 4 };
DP_HD std::uint64_t sample_hash(std::int64_t seed, std::uint32_t round, std::uint32_t klass, std::uint32_t kind,
                                std::uint64_t a, std::uint64_t b) {
  std::uint64_t h = mix64(std::uint64_t(seed) + 0x9e3779b97f4a7c15ULL);
  h = mix64(h ^ std::uint64_t(round));
  h = mix64(h ^ ((std::uint64_t(kind) << 32) | std::uint64_t(klass)));
  h = mix64(h ^ a);
  return mix64(h ^ b);
}
// Uniform in [0, 1) from the top 53 bits.
DP_HD double sample_uniform(std::uint64_t h) { return double(h >> 11) * (1.0 / 9007199254740992.0); }
// Features kept from n candidates at fraction c: max(1, floor(c n)), at most n.
DP_HD std::uint32_t sample_count(double c, std::uint32_t n) {
  const std::uint32_t k = std::uint32_t(c * double(n));
  return n == 0 ? 0u : (k < 1u ? 1u : (k > n ? n : k));
}

}  // namespace dp
