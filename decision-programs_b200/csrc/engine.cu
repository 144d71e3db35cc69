#include "engine.h"

#include <algorithm>
#include <cstring>
#include <sstream>

namespace dp {

// ---------------------------------------------------------------- profiler
cudaEvent_t Profiler::take() {
  if (!free_.empty()) {
    cudaEvent_t e = free_.back();
    free_.pop_back();
    return e;
  }
  cudaEvent_t e;
  DP_CUDA(cudaEventCreate(&e));
  return e;
}
void Profiler::begin(cudaStream_t s, const char* name, double alg_bytes) {
  if (!on_) return;
  Pending p{take(), take(), name, alg_bytes};
  DP_CUDA(cudaEventRecord(p.a, s));
  pending_.push_back(p);
}
void Profiler::end(cudaStream_t s) {
  if (!on_) return;
  DP_CUDA(cudaEventRecord(pending_.back().b, s));
}
void Profiler::resolve() {
  for (auto& p : pending_) {
    float ms = 0.f;
    DP_CUDA(cudaEventElapsedTime(&ms, p.a, p.b));
    auto& st = stats_[p.name];
    st.launches += 1;
    st.ms += ms;
    st.bytes += p.bytes;
    free_.push_back(p.a);
    free_.push_back(p.b);
  }
  pending_.clear();
}
std::string Profiler::json() const {
  std::ostringstream o;
  o << "{";
  bool first = true;
  for (const auto& kv : stats_) {
    if (!first) o << ",";
    first = false;
    o << "\"" << kv.first << "\":{\"launches\":" << kv.second.launches << ",\"ms\":" << kv.second.ms
      << ",\"alg_bytes\":" << kv.second.bytes << "}";
  }
  o << "}";
  return o.str();
}
Profiler::~Profiler() {
  for (auto& p : pending_) { cudaEventDestroy(p.a); cudaEventDestroy(p.b); }
  for (auto e : free_) cudaEventDestroy(e);
}

// ---------------------------------------------------------------- engine
namespace {
constexpr u32 kFT = kHistFeatureTile;
constexpr i64 kLeafChunk = 16384;
}

Engine::Engine(DMatrix& d, const TrainParams& p, Comm* comm) : d_(d), p_(p), comm_(comm), device_(d.device()) {
  DeviceGuard g(device_);
  DP_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  need(d_.has_labels(), "training matrix has no labels");
  K_ = p_.K();
  need(K_ >= 1, "num_class must be set for multi-class objectives");
  R_ = d_.rows();
  F_ = d_.cols();
  need(R_ < (u64(1) << 31), "row count per device exceeds 2^31");
  q_ = &d_.quantized(p_.max_bin, comm_, stream_);
  slot_elems_ = u64(F_) * kMaxBins * 2;
  max_bins_ = 0;
  for (u32 f = 0; f < F_; ++f) {
    max_bins_ = std::max<int>(max_bins_, q_->nbins_h[f]);
    if (q_->has_missing_h[f]) max_bins_ = kMaxBins;
  }
  // label validation for the objective
  {
    DevBuf<u32> bad(1);
    DP_CUDA(cudaMemsetAsync(bad.get(), 0, 4, stream_));
    launch_check_labels(d_.labels(), R_, p_.objective_id(), K_, bad.get(), stream_);
    u32 h = 0;
    DP_CUDA(cudaMemcpyAsync(&h, bad.get(), 4, cudaMemcpyDeviceToHost, stream_));
    DP_CUDA(cudaStreamSynchronize(stream_));
    if (h) {
      if (p_.objective_id() == kLogistic) fail("label must be in [0,1] for logistic regression");
      if (p_.objective_id() == kSoftprob || p_.objective_id() == kSoftmax)
        fail("label must be an integer in [0, num_class) for multi-class objectives");
      fail("label contains NaN or infinity");
    }
  }
  const u64 RK = std::max<u64>(R_, 1) * u64(K_);
  margin_.resize(RK);
  std::vector<float> m0(RK);
  for (u64 r = 0; r < std::max<u64>(R_, 1); ++r)
    for (int k = 0; k < K_; ++k) m0[r * K_ + k] = p_.base_margin(k);
  DP_CUDA(cudaMemcpy(margin_.get(), m0.data(), RK * sizeof(float), cudaMemcpyHostToDevice));
  for (int s = 0; s < 2; ++s) {
    gh_[s].resize(RK);
    ridx_[s].resize(RK);
    std::vector<TreeArrays> ta(K_);
    for (int k = 0; k < K_; ++k) ta[k] = TreeArrays{ridx_[s].get() + u64(k) * R_, gh_[s].get() + u64(k) * R_};
    tarr_[s].resize(K_);
    DP_CUDA(cudaMemcpy(tarr_[s].get(), ta.data(), K_ * sizeof(TreeArrays), cudaMemcpyHostToDevice));
  }
  gmax_.resize(K_);
  hmax_.resize(K_);
  scales_.resize(K_);
  hist_counter_.resize(1);
  arena_.reserve(size_t(8) << 20);
}

Engine::~Engine() {
  if (stream_) {
    DeviceGuard g(device_);
    cudaStreamSynchronize(stream_);
    cudaStreamDestroy(stream_);
  }
}

void Engine::sync() {
  DP_CUDA(cudaStreamSynchronize(stream_));
  prof_.resolve();
  arena_off_ = 0;
}

template <class T>
T* Engine::stage(const std::vector<T>& v) {
  const size_t bytes = v.size() * sizeof(T);
  size_t off = (arena_off_ + 255) & ~size_t(255);
  if (off + bytes > arena_.size()) {
    // all staged copies must land before the arena is replaced
    DP_CUDA(cudaStreamSynchronize(stream_));
    prof_.resolve();
    size_t want = std::max(arena_.size() * 2, bytes + 4096);
    PinnedBuf<u8> fresh;
    fresh.reserve(want);
    arena_.swap(fresh);
    off = 0;
  }
  std::memcpy(arena_.get() + off, v.data(), bytes);
  arena_off_ = off + bytes;
  return reinterpret_cast<T*>(arena_.get() + off);
}

template <class T>
void Engine::upload(DevBuf<T>& dst, const std::vector<T>& v) {
  dst.reserve(std::max<size_t>(v.size(), 1));
  if (v.empty()) return;
  T* src = stage(v);
  DP_CUDA(cudaMemcpyAsync(dst.get(), src, v.size() * sizeof(T), cudaMemcpyHostToDevice, stream_));
}

template <class T>
const T* Engine::download(const T* src, size_t n) {
  std::vector<T> tmp(n);
  T* dst = stage(tmp);
  DP_CUDA(cudaMemcpyAsync(dst, src, n * sizeof(T), cudaMemcpyDeviceToHost, stream_));
  return dst;
}

std::vector<float> Engine::margins() const {
  DeviceGuard g(device_);
  std::vector<float> out(R_ * K_);
  DP_CUDA(cudaStreamSynchronize(stream_));
  DP_CUDA(cudaMemcpy(out.data(), margin_.get(), out.size() * sizeof(float), cudaMemcpyDeviceToHost));
  return out;
}

void Engine::boost_round(Model& m) {
  DeviceGuard g(device_);
  const int K = K_;
  const u64 R = R_;
  const u32 F = F_;
  const u32 ftiles = (F + kFT - 1) / kFT;
  const SplitParams sp = p_.split_params();
  const std::vector<float>& cut = q_->cut_h;
  const std::vector<u8>& hm = q_->has_missing_h;

  // ---- gradients and quantiser scales
  DP_CUDA(cudaMemsetAsync(gmax_.get(), 0, K * sizeof(u32), stream_));
  DP_CUDA(cudaMemsetAsync(hmax_.get(), 0, K * sizeof(u32), stream_));
  prof_.begin(stream_, "gradients", double(R) * K * (4 + 8) + double(R) * 4);
  launch_gradients(p_.objective_id(), K, margin_.get(), d_.labels(), R, gh_[0].get(), gmax_.get(), hmax_.get(),
                   stream_);
  prof_.end(stream_);
  if (comm_) {
    comm_->max_u32(gmax_.get(), K, stream_);
    comm_->max_u32(hmax_.get(), K, stream_);
  }
  launch_scales(K, gmax_.get(), hmax_.get(), scales_.get(), stream_);
  // (g, h) become exact int32 pairs once per round; every later pass reads them
  launch_quantize_gh(gh_[0].get(), R, K, scales_.get(), stream_);
  for (int k = 0; k < K; ++k) launch_iota(ridx_[0].get() + u64(k) * R, R, stream_);
  const Scales* sc_h = download(scales_.get(), K);

  std::vector<Tree> trees(K);
  std::vector<std::vector<i64>> ngq(K), nhq(K);  // quantised node totals
  std::vector<Open> open;
  for (int k = 0; k < K; ++k) {
    trees[k].klass = k;
    trees[k].add_node(-1);
    ngq[k].push_back(0);
    nhq[k].push_back(0);
    open.push_back(Open{k, 0, k, 0, i64(R), i64(q_->rows_total), 0, 0});
  }
  sync();
  std::vector<Scales> scales(sc_h, sc_h + K);

  std::vector<Leaf> leaves;
  std::vector<std::pair<int, int>> build;   // (slot, index into open) of nodes built directly
  std::vector<u32> triples;
  for (int k = 0; k < K; ++k) build.push_back({k, k});
  int set = 0, region = 0;
  for (int depth = 0; depth < p_.max_depth && !open.empty(); ++depth) {
    // ---- histograms of the build set (slots [0, nbuild) of this region)
    const u64 nslots = std::max<u64>(open.size(), 1);
    hist_[region].reserve(nslots * slot_elems_);
    i64* hist = hist_[region].get();
    const u64 nbuild = build.size();
    DP_CUDA(cudaMemsetAsync(hist, 0, nbuild * slot_elems_ * sizeof(i64), stream_));
    std::vector<HistTask> tasks;
    double rows_built = 0;
    for (auto& b : build) rows_built += double(open[b.second].count);
    const i64 chunk = i64(hist_chunk_rows(u64(rows_built) * ftiles));
    for (auto& b : build) {
      const Open& o = open[b.second];
      if (o.count == 0) continue;
      const i64 pieces = (o.count + chunk - 1) / chunk;
      const i64 piece = (o.count + pieces - 1) / pieces;
      for (u32 ft = 0; ft < ftiles; ++ft)
        for (i64 s = o.begin; s < o.begin + o.count; s += piece)
          tasks.push_back(HistTask{u32(b.first), ft * kFT, u32(o.tree), 0, s,
                                   std::min<i64>(o.begin + o.count, s + piece)});
    }
    upload(hist_tasks_, tasks);
    prof_.begin(stream_, "histograms", rows_built * (double(F) + 12.0) + double(nbuild) * slot_elems_ * 8.0);
    launch_histograms(q_->bins.get(), q_->bin_stride, F, max_bins_, true, tarr_[set].get(), scales_.get(),
                      hist_tasks_.get(), u32(tasks.size()), hist_counter_.get(), hist, stream_);
    prof_.end(stream_);
    if (comm_) comm_->sum_i64(hist, nbuild * slot_elems_, stream_);
    if (!triples.empty()) {
      upload(triples_, triples);
      prof_.begin(stream_, "subtract", double(triples.size() / 3) * slot_elems_ * 24.0);
      launch_subtract(hist, hist_[1 - region].get(), slot_elems_, triples_.get(), u32(triples.size() / 3), stream_);
      prof_.end(stream_);
    }
    if (depth == 0) {
      // root totals from feature 0 of each root histogram
      std::vector<const i64*> h0(K);
      for (int k = 0; k < K; ++k) h0[k] = download(hist + u64(k) * slot_elems_, 2 * kMaxBins);
      sync();
      for (int k = 0; k < K; ++k) {
        i64 gq = 0, hq = 0;
        for (int b = 0; b < kMaxBins; ++b) { gq += h0[k][2 * b]; hq += h0[k][2 * b + 1]; }
        open[k].gq = gq;
        open[k].hq = hq;
        ngq[k][0] = gq;
        nhq[k][0] = hq;
      }
    }
    // ---- split evaluation
    std::vector<EvalNode> en(open.size());
    for (size_t i = 0; i < open.size(); ++i)
      en[i] = EvalNode{u32(open[i].slot), u32(open[i].tree), open[i].gq, open[i].hq};
    upload(eval_nodes_, en);
    const u32 nchunks = (F + kEvalFeatureChunk - 1) / kEvalFeatureChunk;
    cand_.reserve(open.size() * nchunks);
    best_.reserve(open.size());
    prof_.begin(stream_, "eval_splits", double(open.size()) * slot_elems_ * 8.0);
    launch_eval_splits(hist, F, q_->nbins.get(), q_->has_missing.get(), eval_nodes_.get(), u32(open.size()),
                       scales_.get(), sp, cand_.get(), best_.get(), stream_);
    prof_.end(stream_);
    const SplitCand* best_h = download(best_.get(), open.size());
    sync();
    std::vector<SplitCand> best(best_h, best_h + open.size());

    std::vector<int> split;  // indices into open
    for (size_t i = 0; i < open.size(); ++i) {
      if (best[i].feature >= 0 && best[i].gain > 0.0) split.push_back(int(i));
      else leaves.push_back(Leaf{open[i].tree, open[i].id, set, open[i].begin, open[i].count});
    }
    if (split.empty()) { open.clear(); break; }

    // ---- partition
    std::vector<PartNode> pn(split.size());
    std::vector<PartTask> pt;
    for (size_t j = 0; j < split.size(); ++j) {
      const Open& o = open[split[j]];
      const SplitCand& c = best[split[j]];
      pn[j] = PartNode{u32(o.tree), c.feature, c.bin, c.default_left, i32(hm[c.feature]), 0, o.begin,
                       o.begin + o.count};
      for (i64 s = o.begin; s < o.begin + o.count; s += kPartChunk)
        pt.push_back(PartTask{u32(j), 0, s, std::min<i64>(o.begin + o.count, s + kPartChunk)});
    }
    upload(part_nodes_, pn);
    upload(part_tasks_, pt);
    cursors_.reserve(2 * split.size());
    DP_CUDA(cudaMemsetAsync(cursors_.get(), 0, 2 * split.size() * sizeof(u32), stream_));
    prof_.begin(stream_, "partition", 0.0);
    launch_partition(q_->bins.get(), q_->bin_stride, tarr_[set].get(), tarr_[1 - set].get(), part_nodes_.get(),
                     part_tasks_.get(), u32(pt.size()), cursors_.get(), stream_);
    prof_.end(stream_);
    const u32* cur_h = download(cursors_.get(), 2 * split.size());
    sync();
    std::vector<i64> nleft(split.size());
    for (size_t j = 0; j < split.size(); ++j) {
      nleft[j] = cur_h[2 * j];
      need(i64(cur_h[2 * j]) + i64(cur_h[2 * j + 1]) == open[split[j]].count, "partition lost rows");
    }
    std::vector<i64> gleft(nleft);
    if (comm_) {
      counts_.reserve(std::max<size_t>(split.size(), 1));
      upload(counts_, nleft);
      comm_->sum_i64(counts_.get(), split.size(), stream_);
      const i64* g_h = download(counts_.get(), split.size());
      sync();
      gleft.assign(g_h, g_h + split.size());
    }

    // ---- children
    std::vector<Open> next;
    const bool more = depth + 1 < p_.max_depth;
    const u32 ns = u32(split.size());
    build.clear();
    triples.clear();
    for (size_t j = 0; j < split.size(); ++j) {
      const Open& o = open[split[j]];
      const SplitCand& c = best[split[j]];
      Tree& t = trees[o.tree];
      const int lid = t.add_node(o.id);
      const int rid = t.add_node(o.id);
      t.left[o.id] = lid;
      t.right[o.id] = rid;
      ngq[o.tree].push_back(c.gl);
      nhq[o.tree].push_back(c.hl);
      ngq[o.tree].push_back(o.gq - c.gl);
      nhq[o.tree].push_back(o.hq - c.hl);
      t.feature[o.id] = c.feature;
      t.cond[o.id] = cut[u64(c.feature) * kMaxBins + c.bin];
      t.default_left[o.id] = u8(c.default_left);
      t.loss_change[o.id] = float(c.gain);
      const i64 gl_cnt = gleft[j], gr_cnt = o.gcount - gleft[j];
      const bool right_small = gr_cnt < gl_cnt;
      const int lslot = right_small ? int(ns + j) : int(j);
      const int rslot = right_small ? int(j) : int(ns + j);
      next.push_back(Open{o.tree, lid, lslot, o.begin, nleft[j], gl_cnt, c.gl, c.hl});
      next.push_back(Open{o.tree, rid, rslot, o.begin + nleft[j], o.count - nleft[j], gr_cnt, o.gq - c.gl,
                          o.hq - c.hl});
      if (more) {
        build.push_back({int(j), int(next.size()) - (right_small ? 1 : 2)});
        triples.push_back(u32(o.slot));
        triples.push_back(u32(j));
        triples.push_back(u32(ns + j));
      }
    }
    open.swap(next);
    set = 1 - set;
    region = 1 - region;
    if (!more) break;
  }
  for (const Open& o : open) leaves.push_back(Leaf{o.tree, o.id, set, o.begin, o.count});

  // ---- node statistics, leaf values and margin update
  std::vector<LeafTask> lt;
  for (const Leaf& l : leaves) {
    Tree& t = trees[l.tree];
    const float v = leaf_weight(ngq[l.tree][l.id], nhq[l.tree][l.id], scales[l.tree].sg, scales[l.tree].sh, sp);
    t.cond[l.id] = v;
    t.feature[l.id] = 0;
    const u32* ridx = ridx_[l.set].get() + u64(l.tree) * R;
    for (i64 s = l.begin; s < l.begin + l.count; s += kLeafChunk)
      lt.push_back(LeafTask{ridx, s, std::min<i64>(l.begin + l.count, s + kLeafChunk), v, u32(l.tree)});
  }
  for (int k = 0; k < K; ++k) {
    Tree& t = trees[k];
    const double ish = 1.0 / double(scales[k].sh);
    for (size_t id = 0; id < t.size(); ++id) {
      t.base_weight[id] = leaf_weight(ngq[k][id], nhq[k][id], scales[k].sg, scales[k].sh, sp);
      t.sum_hess[id] = float(double(nhq[k][id]) * ish);
    }
  }
  upload(leaf_tasks_, lt);
  prof_.begin(stream_, "leaf_update", double(R) * K * 12.0);
  launch_leaf_update(leaf_tasks_.get(), u32(lt.size()), margin_.get(), u32(K), stream_);
  prof_.end(stream_);
  sync();
  for (auto& t : trees) m.trees.push_back(std::move(t));
  m.iteration_indptr.push_back(int(m.trees.size()));
}

}  // namespace dp
