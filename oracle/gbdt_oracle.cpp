// TEST INFRASTRUCTURE ONLY -- CPU oracle for the GBDT-training hot path.
//
// This file is a plain C++ restatement of the training arithmetic that the
// reference trainer reaches through the XGBoost 3.4.1 C API
// (native/class_native_training.cuh:47-70: XGDMatrixCreateFromCudaArrayInterface,
// XGBoosterSetParam, XGBoosterUpdateOneIter).  XGBoost (dmlc/xgboost v3.4.1,
// CUDA `grow_gpu_hist`) is not vendored in the reference and is not installed
// here, and no reference test pins training numerics, so PARITY IS UNPINNED:
// this oracle follows the reference's parameter contract
// (native/class_native_training.cuh:16-33, :54-66), its input contract
// (dense fp32, NaN = missing, inf rejected: :42-46), its routing rule
// (`x < split_condition` goes left, missing follows default_left:
// native/class_tree_runtime_compare.cu:47, native/class_runtime.cu:128) and the
// published second-order boosting algorithm (Chen & Guestrin 2016, cited by
// docs/paper/decision-programs-paper.tex:1276) with the exact integer
// conventions written below.  It is used only by tests/, by
// __graft_entry__.smoke() and by bench.py's CPU-baseline leg; the product
// library never links or calls it.
//
// Semantics (shared bit-for-bit with the CUDA path):
//  * cuts: per feature over all non-missing values (-0.0 folded into +0.0).
//    B_f = min(max_bin, 256, 255 if the column has a missing value).  If the
//    column has <= B_f distinct values every distinct value except the minimum
//    is a boundary; otherwise boundary k (k=1..B_f-1) is the sorted value at
//    rank floor(k*n/B_f), deduplicated, minimum excluded.
//    bin(x) = #boundaries <= x; missing -> code 255.
//  * gradients in double with dp_exp (Cody-Waite reduction + degree-13 Taylor
//    polynomial by Horner's rule with fused multiply-add), rounded to float.
//  * quantiser per (round, class): s_g = 2^(17 - e) with max|g| = m*2^e,
//    m in [0.5,1); s_h = 2^(18 - e_h).  q = rint(v * s) -> |q_g| <= 2^17,
//    0 <= q_h <= 2^18.  Histograms are exact int64 sums of q.
//  * split gain (double): 0.5*((sL + sR) - sP) - gamma, s = T(G)^2/(H+lambda),
//    T = L1 soft threshold, valid iff H_L,H_R >= min_child_weight and
//    H+lambda > 0 on both sides; best = max gain, ties -> lower feature, lower
//    bin, missing-right before missing-left; a node splits iff gain > 0.
//  * leaf value = float(-T(G)/(H+lambda) * eta); margins += leaf (float).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace orc {

constexpr int kMissingBin = 255;
constexpr int kGradBits = 17;  // |q_g| <= 2^17
constexpr int kHessBits = 18;  // 0 <= q_h <= 2^18
enum Objective { kSquaredError = 0, kLogistic = 1, kSoftprob = 2, kSoftmax = 3 };

thread_local std::string last_error;

// Row-sharded runs: the only exchange steps are element-wise integer
// all-reduces (op 0 = sum, 1 = max) over every rank's buffer.  A null
// callback means a single rank.
typedef void (*AllReduceFn)(int64_t* buf, int64_t n, int op, void* ctx);
struct Comm {
  AllReduceFn fn = nullptr;
  void* ctx = nullptr;
  void sum(int64_t* b, int64_t n) const { if (fn && n) fn(b, n, 0, ctx); }
  void max(int64_t* b, int64_t n) const { if (fn && n) fn(b, n, 1, ctx); }
};

// ---------------------------------------------------------------------------
// exp(x) in double: Cody & Waite (1980) argument reduction x = k*ln2 + r with
// ln2 split into a 24-bit head (k*head is exact for |k| < 2^29) and a tail,
// then the Taylor series of e^r to degree 13 (|r| <= ln2/2 leaves a truncation
// term below 2e-16) evaluated by Horner's rule with fused multiply-add, then
// scaling by 2^k.  Constants are derived from the mathematics: the head is ln2
// rounded to float, the tail is ln2 - head from a 60-digit expansion, the
// coefficients are 1/n! rounded to double.
constexpr double kLn2Head = 0.6931471824645996;        // float(ln 2)
constexpr double kLn2Tail = -1.904654299957768e-09;    // ln 2 - head
constexpr double kInvLn2 = 1.4426950408889634;
constexpr double kInvFact[14] = {
    1.0, 1.0, 0.5, 1.0 / 6.0, 1.0 / 24.0, 1.0 / 120.0, 1.0 / 720.0, 1.0 / 5040.0,
    1.0 / 40320.0, 1.0 / 362880.0, 1.0 / 3628800.0, 1.0 / 39916800.0,
    1.0 / 479001600.0, 1.0 / 6227020800.0};

double dp_exp(double x) {
  if (std::isnan(x)) return x;
  if (x > 709.0) return std::numeric_limits<double>::infinity();
  if (x < -745.0) return 0.0;
  const double k = std::rint(x * kInvLn2);
  const double hi = x - k * kLn2Head;
  const double r = hi - k * kLn2Tail;
  double p = kInvFact[13];
  for (int n = 12; n >= 0; --n) p = std::fma(p, r, kInvFact[n]);
  return std::ldexp(p, int(k));
}

// ---------------------------------------------------------------------------
static void parallel_for(int64_t n, int threads, const std::function<void(int64_t, int64_t, int)>& fn) {
  if (n <= 0) return;
  threads = int(std::max<int64_t>(1, std::min<int64_t>(threads, n)));
  if (threads == 1) { fn(0, n, 0); return; }
  std::vector<std::thread> pool;
  int64_t chunk = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    int64_t b = t * chunk, e = std::min<int64_t>(n, b + chunk);
    if (b >= e) break;
    pool.emplace_back(fn, b, e, t);
  }
  for (auto& th : pool) th.join();
}

// Dynamic scheduling over n independent tasks.
static void parallel_tasks(int64_t n, int threads, const std::function<void(int64_t, int)>& fn) {
  if (n <= 0) return;
  threads = int(std::max<int64_t>(1, std::min<int64_t>(threads, n)));
  if (threads == 1) { for (int64_t i = 0; i < n; ++i) fn(i, 0); return; }
  std::atomic<int64_t> next{0};
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&, t] { for (int64_t i; (i = next.fetch_add(1)) < n;) fn(i, t); });
  for (auto& th : pool) th.join();
}

static inline bool is_missing(float v, bool has_mv, float mv) {
  return std::isnan(v) || (has_mv && v == mv);
}

struct Cuts {
  uint32_t F = 0;
  std::vector<float> cut;        // [F][256]; boundaries, ascending
  std::vector<uint16_t> nbins;   // value bins per feature (>= 1)
  std::vector<uint8_t> has_missing;
};

// Ascending order of non-NaN floats with -0.0 already folded into +0.0: an
// LSD radix sort over the order-preserving 32-bit key (sign bit set for
// positives, all bits flipped for negatives) in four 8-bit passes.  Equal
// values have equal keys, so the result is the array std::sort gives; short
// columns use std::sort itself.
static void sort_floats(std::vector<float>& v) {
  const size_t n = v.size();
  if (n < 4096) {
    std::sort(v.begin(), v.end());
    return;
  }
  std::vector<uint32_t> a(n), b(n);
  for (size_t i = 0; i < n; ++i) {
    uint32_t u;
    std::memcpy(&u, &v[i], 4);
    a[i] = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  for (int shift = 0; shift < 32; shift += 8) {
    size_t start[257] = {0};
    for (size_t i = 0; i < n; ++i) ++start[((a[i] >> shift) & 255u) + 1];
    for (int d = 0; d < 256; ++d) start[d + 1] += start[d];
    for (size_t i = 0; i < n; ++i) b[start[(a[i] >> shift) & 255u]++] = a[i];
    a.swap(b);
  }
  for (size_t i = 0; i < n; ++i) {
    const uint32_t u = (a[i] & 0x80000000u) ? (a[i] & 0x7fffffffu) : ~a[i];
    std::memcpy(&v[i], &u, 4);
  }
}

// Boundaries of one column from its sorted non-missing values.
static void column_cuts(std::vector<float>& v, int max_bin, bool has_missing, float* cut, uint16_t* nbins) {
  const int64_t n = int64_t(v.size());
  const int B = std::min(max_bin, has_missing ? 255 : 256);
  if (n == 0) { *nbins = 1; return; }
  sort_floats(v);
  int64_t distinct = 1;
  for (int64_t i = 1; i < n && distinct <= B; ++i) distinct += v[i] != v[i - 1];
  int nb = 0;
  if (distinct <= B) {
    for (int64_t i = 1; i < n; ++i)
      if (v[i] != v[i - 1]) cut[nb++] = v[i];
  } else {
    const float lo = v[0];
    for (int k = 1; k < B; ++k) {
      const int64_t rank = (int64_t(k) * n) / B;
      const float b = v[rank];
      if (b == lo) continue;
      if (nb > 0 && !(b > cut[nb - 1])) continue;
      cut[nb++] = b;
    }
  }
  *nbins = uint16_t(nb + 1);
}

Cuts compute_cuts(const float* x, uint64_t R, uint32_t F, uint64_t stride, int max_bin, bool has_mv, float mv,
                  int threads) {
  Cuts c;
  c.F = F;
  c.cut.assign(size_t(F) * 256, 0.f);
  c.nbins.assign(F, 1);
  c.has_missing.assign(F, 0);
  parallel_tasks(F, threads, [&](int64_t f, int) {
    std::vector<float> v;
    v.reserve(R);
    bool miss = false;
    for (uint64_t r = 0; r < R; ++r) {
      float a = x[r * stride + f];
      if (is_missing(a, has_mv, mv)) { miss = true; continue; }
      v.push_back(a == 0.0f ? 0.0f : a);  // fold -0.0 into +0.0
    }
    c.has_missing[f] = miss;
    column_cuts(v, max_bin, miss, &c.cut[size_t(f) * 256], &c.nbins[f]);
  });
  return c;
}

static inline uint8_t bin_of(float a, const float* cut, int nb, bool has_mv, float mv) {
  if (is_missing(a, has_mv, mv)) return kMissingBin;
  return uint8_t(std::upper_bound(cut, cut + (nb - 1), a) - cut);
}

// ---------------------------------------------------------------------------
// The same cut rule computed without sorting, by exact radix selection on the
// monotone 32-bit key of each value (the GPU path's algorithm): counts per
// 16-bit key prefix, then two 8-bit refinements restricted to at most 256
// active prefixes per feature (prefixes holding a wanted rank, or every
// non-empty prefix while the column may have <= B distinct values).  Counts
// are summed over ranks, so every rank reaches the same cuts.
static inline uint32_t fkey(float v) {
  if (v == 0.0f) v = 0.0f;
  uint32_t u;
  std::memcpy(&u, &v, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
static inline float keyf(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  float v;
  std::memcpy(&v, &u, 4);
  return v;
}
static inline bool holds_target(int64_t base, int64_t cnt, int64_t n, int64_t B) {
  if (cnt == 0) return false;
  if (base == 0) return true;
  const int64_t klo = (base * B + n - 1) / n;
  int64_t khi = ((base + cnt) * B + n - 1) / n - 1;
  if (khi > B - 1) khi = B - 1;
  return klo <= khi;
}

Cuts radix_cuts(const float* x, uint64_t R, uint32_t F, uint64_t stride, int max_bin, bool has_mv, float mv,
                const Comm& comm) {
  struct Entry { uint32_t prefix; int64_t base, cnt; };
  struct State { int64_t n = 0; int64_t B = 0; bool mode = false; std::vector<Entry> act; };
  int64_t rtot = int64_t(R);
  comm.sum(&rtot, 1);
  std::vector<State> st(F);
  std::vector<int64_t> cnt(size_t(F) * 65536, 0);
  for (uint64_t r = 0; r < R; ++r)
    for (uint32_t f = 0; f < F; ++f) {
      const float v = x[r * stride + f];
      if (!is_missing(v, has_mv, mv)) ++cnt[size_t(f) * 65536 + (fkey(v) >> 16)];
    }
  comm.sum(cnt.data(), int64_t(cnt.size()));
  for (uint32_t f = 0; f < F; ++f) {
    State& S = st[f];
    const int64_t* c = &cnt[size_t(f) * 65536];
    int64_t nz = 0;
    for (int b = 0; b < 65536; ++b) { S.n += c[b]; nz += c[b] != 0; }
    S.B = std::min(max_bin, 256);
    if (S.n < rtot && S.B > 255) S.B = 255;
    S.mode = nz <= S.B;
    int64_t cum = 0;
    for (int b = 0; b < 65536; ++b) {
      if (c[b] && (S.mode || holds_target(cum, c[b], S.n, S.B))) S.act.push_back({uint32_t(b), cum, c[b]});
      cum += c[b];
    }
  }
  for (int shift : {16, 8}) {
    std::vector<int64_t> c8(size_t(F) * 256 * 256, 0);
    for (uint64_t r = 0; r < R; ++r)
      for (uint32_t f = 0; f < F; ++f) {
        const float v = x[r * stride + f];
        if (is_missing(v, has_mv, mv)) continue;
        const uint32_t k = fkey(v), pfx = k >> shift;
        const auto& act = st[f].act;
        auto it = std::lower_bound(act.begin(), act.end(), pfx,
                                   [](const Entry& e, uint32_t p) { return e.prefix < p; });
        if (it != act.end() && it->prefix == pfx)
          ++c8[(size_t(f) * 256 + size_t(it - act.begin())) * 256 + ((k >> (shift - 8)) & 0xffu)];
      }
    comm.sum(c8.data(), int64_t(c8.size()));
    for (uint32_t f = 0; f < F; ++f) {
      State& S = st[f];
      int64_t nz = 0;
      for (size_t a = 0; a < S.act.size(); ++a)
        for (int d = 0; d < 256; ++d) nz += c8[(size_t(f) * 256 + a) * 256 + d] != 0;
      S.mode = S.mode && nz <= S.B;
      std::vector<Entry> next;
      for (size_t a = 0; a < S.act.size(); ++a) {
        int64_t cum = S.act[a].base;
        for (int d = 0; d < 256; ++d) {
          const int64_t v = c8[(size_t(f) * 256 + a) * 256 + d];
          if (v && (S.mode || holds_target(cum, v, S.n, S.B))) next.push_back({(S.act[a].prefix << 8) | uint32_t(d), cum, v});
          cum += v;
        }
      }
      S.act.swap(next);
    }
  }
  Cuts out;
  out.F = F;
  out.cut.assign(size_t(F) * 256, 0.f);
  out.nbins.assign(F, 1);
  out.has_missing.assign(F, 0);
  for (uint32_t f = 0; f < F; ++f) {
    const State& S = st[f];
    float* cf = &out.cut[size_t(f) * 256];
    int nb = 0;
    if (S.n > 0 && !S.act.empty()) {
      if (S.mode) {
        for (size_t i = 1; i < S.act.size(); ++i) cf[nb++] = keyf(S.act[i].prefix);
      } else {
        const uint32_t mn = S.act[0].prefix;
        size_t e = 0;
        uint32_t last = 0;
        for (int64_t k = 1; k < S.B; ++k) {
          const int64_t rank = (k * S.n) / S.B;
          while (e + 1 < S.act.size() && S.act[e].base + S.act[e].cnt <= rank) ++e;
          const uint32_t key = S.act[e].prefix;
          if (key == mn || (nb > 0 && key <= last)) continue;
          cf[nb++] = keyf(key);
          last = key;
        }
      }
    }
    out.nbins[f] = uint16_t(nb + 1);
    out.has_missing[f] = S.n < rtot;
  }
  return out;
}

void bin_matrix(const float* x, uint64_t R, uint32_t F, uint64_t stride, const Cuts& c, bool has_mv, float mv,
                uint8_t* bins, uint64_t bstride, int threads) {
  parallel_for(int64_t(R), threads, [&](int64_t b, int64_t e, int) {
    for (int64_t r = b; r < e; ++r) {
      for (uint32_t f = 0; f < F; ++f)
        bins[r * bstride + f] = bin_of(x[r * stride + f], &c.cut[size_t(f) * 256], c.nbins[f], has_mv, mv);
      for (uint64_t f = F; f < bstride; ++f) bins[r * bstride + f] = 0;
    }
  });
}

// gh layout: [K][R][2] float (g, h).
void gradients(int objective, int K, const float* margin, const float* label, uint64_t R, float* gh, int threads) {
  parallel_for(int64_t(R), threads, [&](int64_t b, int64_t e, int) {
    std::vector<double> p(K);
    for (int64_t r = b; r < e; ++r) {
      const float* m = margin + r * K;
      const double y = label[r];
      if (objective == kSquaredError) {
        double g = double(m[0]) - y;
        gh[2 * r] = float(g);
        gh[2 * r + 1] = 1.0f;
      } else if (objective == kLogistic) {
        double pr = 1.0 / (1.0 + dp_exp(-double(m[0])));
        double g = pr - y;
        double h = std::max(pr * (1.0 - pr), 1e-16);
        gh[2 * r] = float(g);
        gh[2 * r + 1] = float(h);
      } else {
        double mx = m[0];
        for (int k = 1; k < K; ++k) mx = std::max(mx, double(m[k]));
        double s = 0.0;
        for (int k = 0; k < K; ++k) { p[k] = dp_exp(double(m[k]) - mx); s = s + p[k]; }
        for (int k = 0; k < K; ++k) {
          double pk = p[k] / s;
          double g = pk - (double(k) == y ? 1.0 : 0.0);
          double h = std::max(2.0 * pk * (1.0 - pk), 1e-16);
          gh[(size_t(k) * R + r) * 2] = float(g);
          gh[(size_t(k) * R + r) * 2 + 1] = float(h);
        }
      }
    }
  });
}

// Power-of-two quantiser scale: |v*s| < 2^bits for all |v| <= vmax.
float quant_scale(float vmax, int bits) {
  if (!(vmax > 0.0f)) return 1.0f;
  int e = 0;
  std::frexp(vmax, &e);
  e = std::max(-100, std::min(100, e));
  return std::ldexp(1.0f, bits - e);
}

void quantizer(const float* gh, uint64_t R, float* sg, float* sh, const Comm& comm = Comm()) {
  float mg = 0.f, mh = 0.f;
  for (uint64_t r = 0; r < R; ++r) {
    mg = std::max(mg, std::fabs(gh[2 * r]));
    mh = std::max(mh, gh[2 * r + 1]);
  }
  // non-negative floats order like their bit patterns
  uint32_t bg, bh;
  std::memcpy(&bg, &mg, 4);
  std::memcpy(&bh, &mh, 4);
  int64_t m[2] = {int64_t(bg), int64_t(bh)};
  comm.max(m, 2);
  bg = uint32_t(m[0]);
  bh = uint32_t(m[1]);
  std::memcpy(&mg, &bg, 4);
  std::memcpy(&mh, &bh, 4);
  *sg = quant_scale(mg, kGradBits);
  *sh = quant_scale(mh, kHessBits);
}

static inline int64_t qv(float v, float s) { return int64_t(std::rint(v * s)); }

// Histogram of one row segment: hist[F][256][2] += (q_g, q_h).  `ghp` is in
// position order (ghp[i] belongs to row ridx[i]).  The rows are taken in
// blocks, and each block is added one tile of features at a time, so that the
// tile's cells (8 features x 256 bins x 16 bytes) stay in the first-level
// cache instead of every row touching all F features' cells.  The sums are
// exact integers, so the order of the additions does not change them.
static void hist_segment(const uint8_t* bins, uint64_t bstride, uint32_t F, const float* ghp, const uint32_t* ridx,
                         int64_t begin, int64_t end, float sg, float sh, int64_t* hist) {
  constexpr int64_t kRowBlock = 2048;
  constexpr uint32_t kFeatTile = 8;
  const uint8_t* rows[kRowBlock];
  int64_t q[2 * kRowBlock];
  for (int64_t b0 = begin; b0 < end; b0 += kRowBlock) {
    const int64_t n = std::min(kRowBlock, end - b0);
    for (int64_t i = 0; i < n; ++i) {
      rows[i] = bins + uint64_t(ridx[b0 + i]) * bstride;
      q[2 * i] = qv(ghp[2 * (b0 + i)], sg);
      q[2 * i + 1] = qv(ghp[2 * (b0 + i) + 1], sh);
    }
    for (uint32_t f0 = 0; f0 < F; f0 += kFeatTile) {
      const uint32_t f1 = std::min(F, f0 + kFeatTile);
      for (int64_t i = 0; i < n; ++i) {
        const uint8_t* row = rows[i];
        const int64_t g = q[2 * i], h = q[2 * i + 1];
        for (uint32_t f = f0; f < f1; ++f) {
          int64_t* cell = hist + (size_t(f) * 256 + row[f]) * 2;
          cell[0] += g;
          cell[1] += h;
        }
      }
    }
  }
}

// Histograms of several segments, threaded; outs[s] (F x 256 x 2 int64) is
// overwritten for every segment s.  A segment of at most one chunk is built by
// one task straight into its output; a longer one is split into chunks whose
// sums each thread gathers in its own buffer and adds under the segment's
// lock.  The sums are exact integers, so neither the split nor the order of
// the merges changes them.
void histograms_into(const uint8_t* bins, uint64_t bstride, uint32_t F, const float* ghp, const uint32_t* ridx,
                     const int64_t* seg_begin, const int64_t* seg_end, int64_t nseg, float sg, float sh,
                     int64_t* const* outs, int threads) {
  const size_t hsz = size_t(F) * 256 * 2;
  const int64_t kChunk = 1 << 15;
  struct Task { int64_t seg, b, e; bool whole; };
  std::vector<Task> tasks;
  std::vector<int64_t> shared_segs;  // segments of several tasks
  for (int64_t s = 0; s < nseg; ++s) {
    const bool whole = seg_end[s] - seg_begin[s] <= kChunk;
    if (!whole) shared_segs.push_back(s);
    if (whole) tasks.push_back({s, seg_begin[s], seg_end[s], true});
    else
      for (int64_t b = seg_begin[s]; b < seg_end[s]; b += kChunk)
        tasks.push_back({s, b, std::min(seg_end[s], b + kChunk), false});
  }
  parallel_tasks(int64_t(shared_segs.size()), threads,
                 [&](int64_t i, int) { std::fill(outs[shared_segs[i]], outs[shared_segs[i]] + hsz, 0); });
  threads = std::max(1, threads);
  std::vector<std::vector<int64_t>> priv(static_cast<size_t>(threads));
  std::vector<std::unique_ptr<std::atomic<int>>> lock(size_t(std::max<int64_t>(nseg, 0)));
  for (auto& l : lock) l = std::make_unique<std::atomic<int>>(0);
  parallel_tasks(int64_t(tasks.size()), threads, [&](int64_t ti, int t) {
    const Task& tk = tasks[ti];
    if (tk.whole) {
      std::fill(outs[tk.seg], outs[tk.seg] + hsz, 0);
      hist_segment(bins, bstride, F, ghp, ridx, tk.b, tk.e, sg, sh, outs[tk.seg]);
      return;
    }
    std::vector<int64_t>& local = priv[size_t(t)];
    if (local.empty()) local.assign(hsz, 0);
    hist_segment(bins, bstride, F, ghp, ridx, tk.b, tk.e, sg, sh, local.data());
    auto& l = *lock[size_t(tk.seg)];
    int expected = 0;
    while (!l.compare_exchange_weak(expected, 1)) expected = 0;
    int64_t* dst = outs[tk.seg];
    for (size_t j = 0; j < hsz; ++j) {
      dst[j] += local[j];
      local[j] = 0;
    }
    l.store(0);
  });
}

// The same with out[N][F][256][2] contiguous.
void histograms(const uint8_t* bins, uint64_t bstride, uint32_t F, const float* ghp, const uint32_t* ridx,
                const int64_t* seg_begin, const int64_t* seg_end, int64_t nseg, float sg, float sh, int64_t* out,
                int threads) {
  const size_t hsz = size_t(F) * 256 * 2;
  std::vector<int64_t*> outs(size_t(std::max<int64_t>(nseg, 0)));
  for (int64_t s = 0; s < nseg; ++s) outs[size_t(s)] = out + hsz * size_t(s);
  histograms_into(bins, bstride, F, ghp, ridx, seg_begin, seg_end, nseg, sg, sh, outs.data(), threads);
}

struct Params {
  int objective = kSquaredError;
  int K = 1;
  int max_depth = 6;
  int max_bin = 256;
  double eta = 0.3, lambda = 1.0, alpha = 0.0, gamma = 0.0, mcw = 1.0;
  float base_margin = 0.0f;
  int threads = 1;
  int subtract = 1;
  // sampling
  double subsample = 1.0, cs_tree = 1.0, cs_level = 1.0, cs_node = 1.0;
  int64_t seed = 0;
  uint64_t row0 = 0;  // first global row of this rank
};

// ---- sampling: a counter-based hash (the output function of SplitMix64,
// Steele, Lea and Flood, OOPSLA 2014) over a chain of key words.  Row r of
// tree (round, k) is kept iff uniform(hash(seed, round, k, ROW, r, 0)) <
// subsample; feature sets are nested exact-count selections of the smallest
// (hash, feature): the tree keeps max(1, floor(c_tree F)) (kind TREE, index
// 0), each level that fraction of the tree's (LEVEL, depth), each node that
// fraction of the level's (NODE, node id).
uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xbf58476d1ce4e5b9ULL;
  z ^= z >> 27;
  z *= 0x94d049bb133111ebULL;
  z ^= z >> 31;
  return z;
}
enum { kRow = 1, kTreeSet = 2, kLevelSet = 3, kNodeSet = 4 };
uint64_t sample_hash(int64_t seed, uint32_t round, uint32_t k, uint32_t kind, uint64_t a, uint64_t b) {
  uint64_t h = mix64(uint64_t(seed) + 0x9e3779b97f4a7c15ULL);
  h = mix64(h ^ uint64_t(round));
  h = mix64(h ^ ((uint64_t(kind) << 32) | uint64_t(k)));
  h = mix64(h ^ a);
  return mix64(h ^ b);
}
double sample_uniform(uint64_t h) { return double(h >> 11) * (1.0 / 9007199254740992.0); }
uint32_t sample_count(double c, uint32_t n) {
  const uint32_t k = uint32_t(c * double(n));
  return n == 0 ? 0u : std::min(n, std::max(1u, k));
}
// Features that may split node `node` at `depth` of tree (round, k).
std::vector<uint8_t> feature_set(const Params& p, uint32_t round, uint32_t k, int depth, int node, uint32_t F) {
  std::vector<uint8_t> in(F, 1);
  auto select = [&](double c, uint32_t kind, uint64_t index) {
    if (c >= 1.0) return;
    std::vector<std::pair<uint64_t, uint32_t>> v;
    for (uint32_t f = 0; f < F; ++f)
      if (in[f]) v.push_back({sample_hash(p.seed, round, k, kind, f, index), f});
    const uint32_t n = sample_count(c, uint32_t(v.size()));
    std::sort(v.begin(), v.end());
    std::fill(in.begin(), in.end(), uint8_t(0));
    for (uint32_t i = 0; i < n; ++i) in[v[i].second] = 1;
  };
  select(p.cs_tree, kTreeSet, 0);
  select(p.cs_level, kLevelSet, uint64_t(depth));
  select(p.cs_node, kNodeSet, uint64_t(node));
  return in;
}

struct Split {
  double gain = -std::numeric_limits<double>::infinity();
  int32_t feature = -1;
  int32_t bin = -1;
  int32_t default_left = 0;
  int64_t gl = 0, hl = 0;
};

static inline double soft(double g, double alpha) {
  if (g > alpha) return g - alpha;
  if (g < -alpha) return g + alpha;
  return 0.0;
}
static inline double score(double g, double h, const Params& p) {
  const double t = soft(g, p.alpha);
  return (t * t) / (h + p.lambda);
}

Split best_split(const int64_t* hist, uint32_t F, const Cuts& c, int64_t gq, int64_t hq, float sg, float sh,
                 const Params& p, const uint8_t* allowed = nullptr) {
  const double isg = 1.0 / double(sg), ish = 1.0 / double(sh);
  const double G = double(gq) * isg, H = double(hq) * ish;
  const double sp = score(G, H, p);
  Split best;
  for (uint32_t f = 0; f < F; ++f) {
    const int nb = c.nbins[f];
    if (nb < 2) continue;
    if (allowed && !allowed[f]) continue;
    const int64_t* hf = hist + size_t(f) * 256 * 2;
    const bool hm = c.has_missing[f];
    const int64_t gm = hm ? hf[2 * kMissingBin] : 0, hmq = hm ? hf[2 * kMissingBin + 1] : 0;
    int64_t gl0 = 0, hl0 = 0;
    for (int b = 0; b + 1 < nb; ++b) {
      gl0 += hf[2 * b];
      hl0 += hf[2 * b + 1];
      for (int d = 0; d < (hm ? 2 : 1); ++d) {
        const int64_t glq = gl0 + (d ? gm : 0), hlq = hl0 + (d ? hmq : 0);
        const int64_t grq = gq - glq, hrq = hq - hlq;
        const double GL = double(glq) * isg, HL = double(hlq) * ish;
        const double GR = double(grq) * isg, HR = double(hrq) * ish;
        if (!(HL >= p.mcw && HR >= p.mcw && HL + p.lambda > 0.0 && HR + p.lambda > 0.0)) continue;
        const double gain = ((score(GL, HL, p) + score(GR, HR, p)) - sp) * 0.5 - p.gamma;
        if (gain > best.gain) {
          best.gain = gain;
          best.feature = int32_t(f);
          best.bin = b;
          best.default_left = d;
          best.gl = glq;
          best.hl = hlq;
        }
      }
    }
  }
  return best;
}

float leaf_value(int64_t gq, int64_t hq, float sg, float sh, const Params& p) {
  const double G = double(gq) * (1.0 / double(sg)), H = double(hq) * (1.0 / double(sh));
  const double den = H + p.lambda;
  if (!(den > 0.0)) return 0.0f;
  const double w = -soft(G, p.alpha) / den;
  return float(w * p.eta);
}

struct Tree {
  std::vector<int32_t> left, right, feature, bin, parent;
  std::vector<float> cond, base_weight, loss_change, sum_hess;
  std::vector<uint8_t> default_left;
  std::vector<int64_t> gq, hq;
  int add(int32_t par, int64_t g, int64_t h) {
    left.push_back(-1); right.push_back(-1); feature.push_back(0); bin.push_back(-1); parent.push_back(par);
    cond.push_back(0.f); base_weight.push_back(0.f); loss_change.push_back(0.f); sum_hess.push_back(0.f);
    default_left.push_back(0); gq.push_back(g); hq.push_back(h);
    return int(left.size()) - 1;
  }
};

// Grows one tree.  ghp is the tree's (g,h) in row order; on return `leaf_of`
// holds the leaf id of every row.
Tree grow_tree(const uint8_t* bins, uint64_t bstride, uint32_t F, uint64_t R, const Cuts& c, const float* gh_rows,
               float sg, float sh, const Params& p, std::vector<int32_t>& leaf_of, const Comm& comm = Comm(),
               uint32_t round = 0, uint32_t klass = 0) {
  const bool col_sampling = p.cs_tree < 1.0 || p.cs_level < 1.0 || p.cs_node < 1.0;
  Tree t;
  std::vector<uint32_t> ridx(R), ridx2(R);
  std::vector<float> ghp(gh_rows, gh_rows + 2 * R), ghp2(2 * R);
  for (uint64_t i = 0; i < R; ++i) ridx[i] = uint32_t(i);
  const size_t hsz = size_t(F) * 256 * 2;
  struct Open { int id; int64_t begin, count; std::vector<int64_t> hist; };
  std::vector<Open> open(1);
  open[0].id = 0;
  open[0].begin = 0;
  open[0].count = int64_t(R);
  open[0].hist.resize(hsz);
  {
    int64_t b = 0, e = int64_t(R);
    histograms(bins, bstride, F, ghp.data(), ridx.data(), &b, &e, 1, sg, sh, open[0].hist.data(), p.threads);
    comm.sum(open[0].hist.data(), int64_t(hsz));
  }
  int64_t G0 = 0, H0 = 0;
  for (int b = 0; b < 256; ++b) { G0 += open[0].hist[2 * b]; H0 += open[0].hist[2 * b + 1]; }
  t.add(-1, G0, H0);
  std::vector<std::pair<int, std::pair<int64_t, int64_t>>> leaves;  // id, segment
  for (int depth = 0; depth < p.max_depth && !open.empty(); ++depth) {
    std::vector<Split> splits(open.size());
    parallel_tasks(int64_t(open.size()), p.threads, [&](int64_t i, int) {
      const int id = open[i].id;
      std::vector<uint8_t> allowed;
      if (col_sampling) allowed = feature_set(p, round, klass, depth, id, F);
      splits[i] = best_split(open[i].hist.data(), F, c, t.gq[id], t.hq[id], sg, sh, p,
                             col_sampling ? allowed.data() : nullptr);
    });
    std::vector<Open> next;
    std::vector<int> split_idx;
    for (size_t i = 0; i < open.size(); ++i) {
      const Split& s = splits[i];
      if (s.feature >= 0 && s.gain > 0.0) split_idx.push_back(int(i));
      else leaves.push_back({open[i].id, {open[i].begin, open[i].count}});
    }
    if (split_idx.empty()) { open.clear(); break; }
    // Stable partition of every split node's segment; children get ids in order.
    // Each segment is cut into chunks: the chunks count their left rows, a
    // prefix over them places each chunk's left and right rows, and the
    // chunks scatter in parallel, keeping the rows' order on each side.
    std::vector<int64_t> nleft(split_idx.size());
    {
      const int64_t kPartChunk = 1 << 16;
      struct PTask { size_t j; int64_t b, e, nl, lpos, rpos; };
      std::vector<PTask> pt;
      for (size_t j = 0; j < split_idx.size(); ++j) {
        const Open& o = open[split_idx[j]];
        for (int64_t b = o.begin; b < o.begin + o.count; b += kPartChunk)
          pt.push_back({j, b, std::min(o.begin + o.count, b + kPartChunk), 0, 0, 0});
      }
      auto goes_left = [&](size_t j, int64_t i) {
        const Split& s = splits[split_idx[j]];
        const uint8_t b = bins[uint64_t(ridx[i]) * bstride + s.feature];
        return (c.has_missing[s.feature] && b == kMissingBin) ? bool(s.default_left) : (b <= s.bin);
      };
      parallel_tasks(int64_t(pt.size()), p.threads, [&](int64_t k, int) {
        PTask& t = pt[size_t(k)];
        for (int64_t i = t.b; i < t.e; ++i) t.nl += goes_left(t.j, i) ? 1 : 0;
      });
      for (size_t k = 0; k < pt.size(); ++k) nleft[pt[k].j] += pt[k].nl;
      std::vector<int64_t> lcur(split_idx.size()), rcur(split_idx.size());
      for (size_t j = 0; j < split_idx.size(); ++j) {
        lcur[j] = open[split_idx[j]].begin;
        rcur[j] = open[split_idx[j]].begin + nleft[j];
      }
      for (auto& t : pt) {  // chunks of a segment are consecutive, in row order
        t.lpos = lcur[t.j];
        t.rpos = rcur[t.j];
        lcur[t.j] += t.nl;
        rcur[t.j] += (t.e - t.b) - t.nl;
      }
      parallel_tasks(int64_t(pt.size()), p.threads, [&](int64_t k, int) {
        const PTask& t = pt[size_t(k)];
        int64_t l = t.lpos, r = t.rpos;
        for (int64_t i = t.b; i < t.e; ++i) {
          const int64_t d = goes_left(t.j, i) ? l++ : r++;
          ridx2[d] = ridx[i];
          ghp2[2 * d] = ghp[2 * i];
          ghp2[2 * d + 1] = ghp[2 * i + 1];
        }
      });
    }
    // Copy split segments back (rows of leaves stay where they are).
    parallel_tasks(int64_t(split_idx.size()), p.threads, [&](int64_t j, int) {
      const Open& o = open[split_idx[size_t(j)]];
      std::copy(ridx2.begin() + o.begin, ridx2.begin() + o.begin + o.count, ridx.begin() + o.begin);
      std::copy(ghp2.begin() + 2 * o.begin, ghp2.begin() + 2 * (o.begin + o.count), ghp.begin() + 2 * o.begin);
    });
    // Row counts over all ranks decide which child is built directly.
    std::vector<int64_t> gcnt(2 * split_idx.size());
    for (size_t j = 0; j < split_idx.size(); ++j) {
      gcnt[2 * j] = nleft[j];
      gcnt[2 * j + 1] = open[split_idx[j]].count - nleft[j];
    }
    comm.sum(gcnt.data(), int64_t(gcnt.size()));
    // Children and their histograms.
    std::vector<int64_t> sb, se;
    std::vector<std::pair<size_t, int>> build;  // (index into next, which child)
    for (size_t j = 0; j < split_idx.size(); ++j) {
      Open& o = open[split_idx[j]];
      const Split& s = splits[split_idx[j]];
      const int id = o.id;
      t.feature[id] = s.feature;
      t.bin[id] = s.bin;
      t.cond[id] = c.cut[size_t(s.feature) * 256 + s.bin];
      t.default_left[id] = uint8_t(s.default_left);
      t.loss_change[id] = float(s.gain);
      const int lid = t.add(id, s.gl, s.hl);
      const int rid = t.add(id, t.gq[id] - s.gl, t.hq[id] - s.hl);
      t.left[id] = lid;
      t.right[id] = rid;
      Open L, Rn;
      L.id = lid; L.begin = o.begin; L.count = nleft[j];
      Rn.id = rid; Rn.begin = o.begin + nleft[j]; Rn.count = o.count - nleft[j];
      next.push_back(std::move(L));
      next.push_back(std::move(Rn));
    }
    const bool need_hist = depth + 1 < p.max_depth;
    if (need_hist) {
      // Build the smaller child (ties -> left) and subtract for the sibling.
      std::vector<size_t> small_idx;
      for (size_t j = 0; j < split_idx.size(); ++j) {
        Open& L = next[2 * j];
        Open& Rn = next[2 * j + 1];
        (void)L;
        (void)Rn;
        size_t sm = (p.subtract && gcnt[2 * j + 1] < gcnt[2 * j]) ? 2 * j + 1 : 2 * j;
        small_idx.push_back(sm);
        if (!p.subtract) small_idx.push_back(2 * j + 1);
      }
      for (size_t k = 0; k < small_idx.size(); ++k) {
        sb.push_back(next[small_idx[k]].begin);
        se.push_back(next[small_idx[k]].begin + next[small_idx[k]].count);
      }
      if (comm.fn) {
        // row-sharded: the level's built histograms go through one exchange
        std::vector<int64_t> hs(hsz * small_idx.size());
        histograms(bins, bstride, F, ghp.data(), ridx.data(), sb.data(), se.data(), int64_t(small_idx.size()), sg,
                   sh, hs.data(), p.threads);
        comm.sum(hs.data(), int64_t(hs.size()));
        for (size_t k = 0; k < small_idx.size(); ++k)
          next[small_idx[k]].hist.assign(hs.begin() + hsz * k, hs.begin() + hsz * (k + 1));
      } else {
        // built straight into the children's storage
        std::vector<int64_t*> outs(small_idx.size());
        parallel_tasks(int64_t(small_idx.size()), p.threads, [&](int64_t k, int) {
          next[small_idx[size_t(k)]].hist.resize(hsz);
          outs[size_t(k)] = next[small_idx[size_t(k)]].hist.data();
        });
        histograms_into(bins, bstride, F, ghp.data(), ridx.data(), sb.data(), se.data(), int64_t(small_idx.size()),
                        sg, sh, outs.data(), p.threads);
      }
      if (p.subtract) {
        parallel_tasks(int64_t(split_idx.size()), p.threads, [&](int64_t jj, int) {
          const size_t j = size_t(jj);
          const Open& par = open[split_idx[j]];
          const size_t sm = small_idx[j], lg = (sm == 2 * j) ? 2 * j + 1 : 2 * j;
          next[lg].hist.resize(hsz);
          for (size_t q = 0; q < hsz; ++q) next[lg].hist[q] = par.hist[q] - next[sm].hist[q];
        });
      }
    }
    open = std::move(next);
  }
  for (auto& o : open) leaves.push_back({o.id, {o.begin, o.count}});
  leaf_of.assign(R, -1);
  for (auto& lf : leaves) {
    const int id = lf.first;
    const float v = leaf_value(t.gq[id], t.hq[id], sg, sh, p);
    t.cond[id] = v;
    t.feature[id] = 0;
    for (int64_t i = lf.second.first; i < lf.second.first + lf.second.second; ++i) leaf_of[ridx[i]] = id;
  }
  for (size_t id = 0; id < t.left.size(); ++id) {
    t.base_weight[id] = leaf_value(t.gq[id], t.hq[id], sg, sh, p);
    t.sum_hess[id] = float(double(t.hq[id]) * (1.0 / double(sh)));
  }
  return t;
}

struct Model {
  Params p;
  uint64_t R = 0;
  uint32_t F = 0;
  Cuts cuts;
  std::vector<uint8_t> bins;
  uint64_t bstride = 0;
  std::vector<float> margin;  // [R][K]
  std::vector<float> label;
  std::vector<Tree> trees;
  std::vector<float> scales;  // per tree: sg, sh
  Comm comm;
};

void train_rounds(Model& m, int rounds) {
  const int K = m.p.K;
  std::vector<float> gh(size_t(K) * m.R * 2);
  for (int it = 0; it < rounds; ++it) {
    const uint32_t round = uint32_t(m.trees.size() / size_t(K));
    gradients(m.p.objective, K, m.margin.data(), m.label.data(), m.R, gh.data(), m.p.threads);
    if (m.p.subsample < 1.0)
      for (int k = 0; k < K; ++k)
        for (uint64_t r = 0; r < m.R; ++r)
          if (!(sample_uniform(sample_hash(m.p.seed, round, uint32_t(k), kRow, m.p.row0 + r, 0)) < m.p.subsample)) {
            gh[(size_t(k) * m.R + r) * 2] = 0.0f;
            gh[(size_t(k) * m.R + r) * 2 + 1] = 0.0f;
          }
    std::vector<std::vector<int32_t>> leaf_of(K);
    std::vector<Tree> round_trees(K);
    for (int k = 0; k < K; ++k) {
      const float* ghk = gh.data() + size_t(k) * m.R * 2;
      float sg, sh;
      quantizer(ghk, m.R, &sg, &sh, m.comm);
      m.scales.push_back(sg);
      m.scales.push_back(sh);
      round_trees[k] = grow_tree(m.bins.data(), m.bstride, m.F, m.R, m.cuts, ghk, sg, sh, m.p, leaf_of[k], m.comm,
                                 round, uint32_t(k));
    }
    for (int k = 0; k < K; ++k) {
      const Tree& t = round_trees[k];
      float* mg = m.margin.data();
      parallel_for(int64_t(m.R), m.p.threads, [&](int64_t b, int64_t e, int) {
        for (int64_t r = b; r < e; ++r) mg[size_t(r) * K + k] += t.cond[leaf_of[k][r]];
      });
      m.trees.push_back(t);
    }
  }
}

// Prediction with the trained ensemble.  Routing restates the reference's
// runtime: x < split_condition goes left and a missing value follows
// default_left (native/class_tree_runtime_compare.cu:47,
// native/class_runtime.cu:128); a leaf carries its value in split_conditions
// (native/class_io.hpp:187-201).  Margins add the leaves of rounds
// [it_begin, it_end) to the base margin in tree order, in float, as training
// does; the transforms use the gradients' arithmetic (double, dp_exp, rounded
// to float).  type 1: margins [R][K]; type 0: squared error -> margin,
// logistic -> probability, softprob -> K probabilities, softmax -> class index.
void predict(const Model& m, const float* x, uint64_t R, uint64_t stride, int type, int it_begin, int it_end,
             int has_mv, float mv, float* out) {
  const int K = m.p.K;
  const size_t t0 = size_t(it_begin) * K, t1 = size_t(it_end) * K;
  std::vector<float> mg(static_cast<size_t>(K));
  std::vector<double> p(static_cast<size_t>(K));
  for (uint64_t r = 0; r < R; ++r) {
    const float* xr = x + r * stride;
    for (int k = 0; k < K; ++k) mg[k] = m.p.base_margin;
    for (size_t t = t0; t < t1 && t < m.trees.size(); ++t) {
      const Tree& tr = m.trees[t];
      const int k = int(t % size_t(K));
      int id = 0;
      while (tr.left[id] >= 0) {
        const float v = xr[tr.feature[id]];
        const bool miss = std::isnan(v) || (has_mv && v == mv);
        id = miss ? (tr.default_left[id] ? tr.left[id] : tr.right[id]) : (v < tr.cond[id] ? tr.left[id] : tr.right[id]);
      }
      mg[k] = mg[k] + tr.cond[id];
    }
    if (type == 1) {
      for (int k = 0; k < K; ++k) out[r * K + k] = mg[k];
    } else if (m.p.objective == kSquaredError) {
      out[r] = mg[0];
    } else if (m.p.objective == kLogistic) {
      out[r] = float(1.0 / (1.0 + dp_exp(-double(mg[0]))));
    } else if (m.p.objective == kSoftprob) {
      double mx = mg[0];
      for (int k = 1; k < K; ++k) mx = std::max(mx, double(mg[k]));
      double sum = 0.0;
      for (int k = 0; k < K; ++k) { p[k] = dp_exp(double(mg[k]) - mx); sum = sum + p[k]; }
      for (int k = 0; k < K; ++k) out[r * K + k] = float(p[k] / sum);
    } else {
      int best = 0;
      for (int k = 1; k < K; ++k)
        if (mg[k] > mg[best]) best = k;
      out[r] = float(best);
    }
  }
}

}  // namespace orc

// ---------------------------------------------------------------------------
// C interface used through ctypes by the tests and the benchmark's CPU leg.
extern "C" {

const char* orc_last_error() { return orc::last_error.c_str(); }

double orc_exp(double x) { return orc::dp_exp(x); }

int orc_cuts(const float* x, uint64_t R, uint32_t F, uint64_t stride, int max_bin, int has_mv, float mv,
             float* cut, uint16_t* nbins, uint8_t* has_missing, int threads) {
  auto c = orc::compute_cuts(x, R, F, stride, max_bin, has_mv, mv, threads);
  std::memcpy(cut, c.cut.data(), c.cut.size() * sizeof(float));
  std::memcpy(nbins, c.nbins.data(), c.nbins.size() * sizeof(uint16_t));
  std::memcpy(has_missing, c.has_missing.data(), c.has_missing.size());
  return 0;
}

int orc_bin_matrix(const float* x, uint64_t R, uint32_t F, uint64_t stride, const float* cut, const uint16_t* nbins,
                   const uint8_t* has_missing, int has_mv, float mv, uint8_t* bins, uint64_t bstride, int threads) {
  orc::Cuts c;
  c.F = F;
  c.cut.assign(cut, cut + size_t(F) * 256);
  c.nbins.assign(nbins, nbins + F);
  c.has_missing.assign(has_missing, has_missing + F);
  orc::bin_matrix(x, R, F, stride, c, has_mv, mv, bins, bstride, threads);
  return 0;
}

int orc_gradients(int objective, int K, const float* margin, const float* label, uint64_t R, float* gh, int threads) {
  orc::gradients(objective, K, margin, label, R, gh, threads);
  return 0;
}

void orc_quantizer(const float* gh, uint64_t R, float* sg, float* sh) { orc::quantizer(gh, R, sg, sh); }

int orc_histograms(const uint8_t* bins, uint64_t bstride, uint32_t F, const float* ghp, const uint32_t* ridx,
                   const int64_t* seg_begin, const int64_t* seg_end, int64_t nseg, float sg, float sh, int64_t* out,
                   int threads) {
  orc::histograms(bins, bstride, F, ghp, ridx, seg_begin, seg_end, nseg, sg, sh, out, threads);
  return 0;
}

// Best split of each node: hist[N][F][256][2], totals[N][2];
// out_i[N][4] = feature, bin, default_left, valid; out_gain[N]; out_left[N][2].
int orc_best_splits(const int64_t* hist, int64_t N, uint32_t F, const uint16_t* nbins, const uint8_t* has_missing,
                    const int64_t* totals, float sg, float sh, double lambda, double alpha, double gamma, double mcw,
                    int32_t* out_i, double* out_gain, int64_t* out_left) {
  orc::Cuts c;
  c.F = F;
  c.nbins.assign(nbins, nbins + F);
  c.has_missing.assign(has_missing, has_missing + F);
  orc::Params p;
  p.lambda = lambda; p.alpha = alpha; p.gamma = gamma; p.mcw = mcw;
  for (int64_t n = 0; n < N; ++n) {
    auto s = orc::best_split(hist + size_t(n) * F * 512, F, c, totals[2 * n], totals[2 * n + 1], sg, sh, p);
    out_i[4 * n] = s.feature;
    out_i[4 * n + 1] = s.bin;
    out_i[4 * n + 2] = s.default_left;
    out_i[4 * n + 3] = s.feature >= 0;
    out_gain[n] = s.gain;
    out_left[2 * n] = s.gl;
    out_left[2 * n + 1] = s.hl;
  }
  return 0;
}

// Whole training run.  Returns an opaque model or NULL (see orc_last_error).
void* orc_train(const float* x, uint64_t R, uint32_t F, uint64_t stride, const float* label, int objective, int K,
                int max_depth, int max_bin, double eta, double lambda, double alpha, double gamma, double mcw,
                float base_margin, int rounds, int threads, int subtract) {
  try {
    auto m = new orc::Model;
    m->p.objective = objective;
    m->p.K = K;
    m->p.max_depth = max_depth;
    m->p.max_bin = max_bin;
    m->p.eta = eta; m->p.lambda = lambda; m->p.alpha = alpha; m->p.gamma = gamma; m->p.mcw = mcw;
    m->p.base_margin = base_margin;
    m->p.threads = std::max(1, threads);
    m->p.subtract = subtract;
    m->R = R;
    m->F = F;
    m->cuts = orc::compute_cuts(x, R, F, stride, max_bin, false, 0.f, m->p.threads);
    m->bstride = (F + 15) / 16 * 16;
    m->bins.resize(R * m->bstride);
    orc::bin_matrix(x, R, F, stride, m->cuts, false, 0.f, m->bins.data(), m->bstride, m->p.threads);
    m->label.assign(label, label + R);
    m->margin.assign(R * K, base_margin);
    orc::train_rounds(*m, rounds);
    return m;
  } catch (const std::exception& e) {
    orc::last_error = e.what();
    return nullptr;
  }
}

// The same run over this rank's rows, with `fn` summing / maxing int64 buffers
// over all ranks (null: one rank).  Cuts use the radix-selection search.
void* orc_train_sharded(const float* x, uint64_t R, uint32_t F, uint64_t stride, const float* label, int objective,
                        int K, int max_depth, int max_bin, double eta, double lambda, double alpha, double gamma,
                        double mcw, float base_margin, int rounds, int threads, orc::AllReduceFn fn, void* ctx) {
  try {
    auto m = new orc::Model;
    m->comm.fn = fn;
    m->comm.ctx = ctx;
    m->p.objective = objective;
    m->p.K = K;
    m->p.max_depth = max_depth;
    m->p.max_bin = max_bin;
    m->p.eta = eta; m->p.lambda = lambda; m->p.alpha = alpha; m->p.gamma = gamma; m->p.mcw = mcw;
    m->p.base_margin = base_margin;
    m->p.threads = std::max(1, threads);
    m->R = R;
    m->F = F;
    m->cuts = orc::radix_cuts(x, R, F, stride, max_bin, false, 0.f, m->comm);
    m->bstride = (F + 15) / 16 * 16;
    m->bins.resize(std::max<uint64_t>(R, 1) * m->bstride);
    orc::bin_matrix(x, R, F, stride, m->cuts, false, 0.f, m->bins.data(), m->bstride, m->p.threads);
    m->label.assign(label, label + R);
    m->margin.assign(R * K, base_margin);
    orc::train_rounds(*m, rounds);
    return m;
  } catch (const std::exception& e) {
    orc::last_error = e.what();
    return nullptr;
  }
}

int orc_radix_cuts(const float* x, uint64_t R, uint32_t F, uint64_t stride, int max_bin, int has_mv, float mv,
                   float* cut, uint16_t* nbins, uint8_t* has_missing, orc::AllReduceFn fn, void* ctx) {
  orc::Comm comm;
  comm.fn = fn;
  comm.ctx = ctx;
  auto c = orc::radix_cuts(x, R, F, stride, max_bin, has_mv, mv, comm);
  std::memcpy(cut, c.cut.data(), c.cut.size() * sizeof(float));
  std::memcpy(nbins, c.nbins.data(), c.nbins.size() * sizeof(uint16_t));
  std::memcpy(has_missing, c.has_missing.data(), c.has_missing.size());
  return 0;
}

void orc_set_sampling(void* h, double subsample, double cs_tree, double cs_level, double cs_node, int64_t seed,
                      uint64_t row0) {
  orc::Params& p = static_cast<orc::Model*>(h)->p;
  p.subsample = subsample;
  p.cs_tree = cs_tree;
  p.cs_level = cs_level;
  p.cs_node = cs_node;
  p.seed = seed;
  p.row0 = row0;
}

int orc_train_more(void* h, int rounds) {
  orc::train_rounds(*static_cast<orc::Model*>(h), rounds);
  return 0;
}

void orc_free(void* h) { delete static_cast<orc::Model*>(h); }
int orc_num_trees(void* h) { return int(static_cast<orc::Model*>(h)->trees.size()); }
int orc_tree_size(void* h, int t) { return int(static_cast<orc::Model*>(h)->trees[t].left.size()); }

int orc_tree(void* h, int t, int32_t* left, int32_t* right, int32_t* feature, float* cond, uint8_t* default_left,
             float* base_weight, float* loss_change, float* sum_hess, int32_t* bin) {
  const auto& tr = static_cast<orc::Model*>(h)->trees[t];
  const size_t n = tr.left.size();
  std::memcpy(left, tr.left.data(), n * 4);
  std::memcpy(right, tr.right.data(), n * 4);
  std::memcpy(feature, tr.feature.data(), n * 4);
  std::memcpy(cond, tr.cond.data(), n * 4);
  std::memcpy(default_left, tr.default_left.data(), n);
  std::memcpy(base_weight, tr.base_weight.data(), n * 4);
  std::memcpy(loss_change, tr.loss_change.data(), n * 4);
  std::memcpy(sum_hess, tr.sum_hess.data(), n * 4);
  std::memcpy(bin, tr.bin.data(), n * 4);
  return 0;
}

int orc_predict(void* h, const float* x, uint64_t R, uint64_t stride, int type, int it_begin, int it_end,
                int has_mv, float mv, float* out) {
  try {
    const orc::Model& m = *static_cast<orc::Model*>(h);
    const int rounds = int(m.trees.size()) / m.p.K;
    if (it_end == 0) it_end = rounds;
    if (it_begin < 0 || it_begin > it_end || it_end > rounds) throw std::runtime_error("iteration range");
    orc::predict(m, x, R, stride, type, it_begin, it_end, has_mv, mv, out);
    return 0;
  } catch (const std::exception& e) {
    orc::last_error = e.what();
    return -1;
  }
}

void orc_margins(void* h, float* out) {
  auto m = static_cast<orc::Model*>(h);
  std::memcpy(out, m->margin.data(), m->margin.size() * 4);
}
void orc_scales(void* h, float* out) {
  auto m = static_cast<orc::Model*>(h);
  std::memcpy(out, m->scales.data(), m->scales.size() * 4);
}
void orc_model_cuts(void* h, float* cut, uint16_t* nbins, uint8_t* has_missing) {
  auto m = static_cast<orc::Model*>(h);
  std::memcpy(cut, m->cuts.cut.data(), m->cuts.cut.size() * 4);
  std::memcpy(nbins, m->cuts.nbins.data(), m->cuts.nbins.size() * 2);
  std::memcpy(has_missing, m->cuts.has_missing.data(), m->cuts.has_missing.size());
}

}  // extern "C"
