#include "engine.h"

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <locale>
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
void Profiler::record(cudaEvent_t e, cudaStream_t s) {
  // inside a stream capture an external record becomes an event node of the graph
  if (capturing_) DP_CUDA(cudaEventRecordWithFlags(e, s, cudaEventRecordExternal));
  else DP_CUDA(cudaEventRecord(e, s));
}
int Profiler::begin(cudaStream_t s, const char* name, double alg_bytes) {
  open_ = mode_ == 1 || (mode_ == 2 && std::strcmp(name, "histograms") == 0);
  if (!open_) return -1;
  Pending p{take(), take(), name, alg_bytes};
  record(p.a, s);
  pending_.push_back(p);
  return int(pending_.size()) - 1;
}
void Profiler::set_bytes(int idx, double alg_bytes) {
  std::vector<Pending>& v = graph_round_ ? graph_pending_ : pending_;
  if (idx >= 0 && size_t(idx) < v.size()) v[idx].bytes = alg_bytes;
}
void Profiler::set_units(int idx, double units) {
  std::vector<Pending>& v = graph_round_ ? graph_pending_ : pending_;
  if (idx >= 0 && size_t(idx) < v.size()) v[idx].units = units;
}
void Profiler::end(cudaStream_t s) {
  if (!open_) return;
  open_ = false;
  record(pending_.back().b, s);
}
bool Profiler::accumulate(const Pending& p) {
  float ms = 0.f;
  const cudaError_t e = cudaEventElapsedTime(&ms, p.a, p.b);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  auto& st = stats_[p.name];
  st.launches += 1;
  st.ms += ms;
  st.bytes += p.bytes;
  st.units += p.units;
  if (log_.size() >= 4096) log_.erase(log_.begin(), log_.begin() + 2048);
  log_.push_back(Entry{p.name, ms, p.bytes});
  return true;
}
void Profiler::resolve() {
  if (graph_round_) {
    for (const auto& p : graph_pending_)
      if (!accumulate(p)) graph_timing_failed_ = true;
    graph_round_ = false;
  }
  for (auto& p : pending_) {
    if (!accumulate(p)) fail("cudaEventElapsedTime failed on a profiled launch");
    free_.push_back(p.a);
    free_.push_back(p.b);
  }
  pending_.clear();
}
void Profiler::abort_capture() {
  capturing_ = false;
  for (auto& p : pending_) {
    free_.push_back(p.a);
    free_.push_back(p.b);
  }
  pending_.clear();
}
void Profiler::drop_graph() {
  for (auto& p : graph_pending_) {
    free_.push_back(p.a);
    free_.push_back(p.b);
  }
  graph_pending_.clear();
  graph_round_ = false;
}
std::string Profiler::json() const {
  std::ostringstream o;
  o.imbue(std::locale::classic());  // JSON numbers, whatever locale the caller set
  o << "{";
  bool first = true;
  for (const auto& kv : stats_) {
    if (!first) o << ",";
    first = false;
    o << "\"" << kv.first << "\":{\"launches\":" << kv.second.launches << ",\"ms\":" << kv.second.ms
      << ",\"alg_bytes\":" << kv.second.bytes << ",\"units\":" << kv.second.units << "}";
  }
  // host phases: {name: [count, ms]}
  o << (first ? "" : ",") << "\"host_ms\":{";
  bool hfirst = true;
  for (const auto& kv : host_) {
    o << (hfirst ? "" : ",") << "\"" << kv.first << "\":[" << kv.second.first << "," << kv.second.second << "]";
    hfirst = false;
  }
  o << "}";
  // the most recent launches in order: [name, ms, algorithmic bytes]
  o << ",\"log\":[";
  for (size_t i = 0; i < log_.size(); ++i)
    o << (i ? "," : "") << "[\"" << log_[i].name << "\"," << log_[i].ms << "," << log_[i].bytes << "]";
  o << "]}";
  return o.str();
}
Profiler::~Profiler() {
  for (auto& p : pending_) { cudaEventDestroy(p.a); cudaEventDestroy(p.b); }
  for (auto& p : graph_pending_) { cudaEventDestroy(p.a); cudaEventDestroy(p.b); }
  for (auto e : free_) cudaEventDestroy(e);
}

// ---------------------------------------------------------------- engine
namespace {
constexpr u32 kFT = kHistFeatureTile;

double ms_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

u64 env_u64(const char* name, u64 dflt) {
  const char* v = std::getenv(name);
  if (!v || !*v) return dflt;
  char* end = nullptr;
  const unsigned long long x = std::strtoull(v, &end, 10);
  return (end && *end == 0) ? u64(x) : dflt;
}
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
  auto t0 = std::chrono::steady_clock::now();
  q_ = &d_.quantized(p_.max_bin, comm_, stream_);
  prof_.host("quantize", ms_since(t0));
  if (q_->host_ms_alloc + q_->host_ms_cuts + q_->host_ms_bins > 0) {
    prof_.host("quantize_alloc", q_->host_ms_alloc);
    prof_.host("quantize_cuts", q_->host_ms_cuts);
    prof_.host("quantize_bins", q_->host_ms_bins);
  }
  t0 = std::chrono::steady_clock::now();
  G_ = comm_ ? comm_->size() : 1;
  rank_ = comm_ ? comm_->rank() : 0;
  fg_ = (F_ + u32(G_) - 1) / u32(G_);
  f_own0_ = u32(rank_) * fg_;
  f_own_n_ = f_own0_ < F_ ? std::min(fg_, F_ - f_own0_) : 0;
  slot_elems_ = u64(fg_) * kMaxBins * 2;
  full_slot_elems_ = u64(G_) * slot_elems_;
  nchunks_ = std::max<u32>(1, (fg_ + kEvalFeatureChunk - 1) / kEvalFeatureChunk);
  max_bins_ = 0;
  for (u32 f = 0; f < F_; ++f) {
    max_bins_ = std::max<int>(max_bins_, q_->nbins_h[f]);
    if (q_->has_missing_h[f]) max_bins_ = kMaxBins;
  }
  DP_CUDA(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, device_));
  // On one GPU, 256-bin matrices of more than two 32-feature tiles take the
  // 64-feature kernel (config 4, 128 features: histograms 2.79 against 3.13 ms
  // per round); up to 64 features the 32-feature kernel is faster (config 2:
  // 0.84 against 0.91 ms per round), and so it is with rows sharded (2 GPUs,
  // before the 64-feature kernel drained through tensor memory: 1.88 against
  // 2.16 ms).  DP_HIST_WIDE=0 / 1 overrides.
  wide_ = max_bins_ > 64 && F_ > kFT && env_u64("DP_HIST_WIDE", (G_ == 1 && F_ > 2 * kFT) ? 1 : 0) != 0;
  hist_tile_ = wide_ ? kHistWideTile : kFT;
  // Histogram tasks per SM: when the bin matrix exceeds L2 and rows share
  // 128-byte lines, about four keep the blocks running at one time on
  // neighbouring rows (L2 reuse of lines shared by several nodes' rows; one
  // per SM was 50% slower for config 5 with 8 nodes); when rows are whole
  // lines there is nothing to share and fewer pieces drain less (config 4:
  // 4.81 ms per round with three, 4.85 with two, 4.91 with four, 5.36 with
  // eight).  When it fits in
  // L2, one per SM: a quarter of the pieces' drains (config 2: 0.64 against
  // 0.73 ms per round).  DP_HIST_TASKS_PER_SM overrides.
  {
    int l2 = 0;
    DP_CUDA(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, device_));
    const bool in_l2 = u64(R_) * u64(F_) <= u64(l2) / 4 * 3;
    const bool whole_lines = q_->bin_stride % 128 == 0;  // no two rows share a 128-byte line
    const u64 per_sm = in_l2 ? 1 : (whole_lines ? 3 : 4);
    hist_target_tasks_ = u32(sms_) * u32(std::max<u64>(1, env_u64("DP_HIST_TASKS_PER_SM", per_sm)));
  }
  // testing knobs: force the exact-count path of deep levels
  async_open_limit_ = env_u64("DP_ASYNC_OPEN_LIMIT", async_open_limit_);
  async_hist_bytes_ = env_u64("DP_ASYNC_HIST_BYTES", async_hist_bytes_);
  graphs_ = env_u64("DP_CUDA_GRAPHS", 1) != 0;
  fold_last_ = env_u64("DP_FOLD_LAST_LEVEL", 1) != 0;

  // every device buffer of the engine in one allocation
  const u64 RK = std::max<u64>(R_, 1) * u64(K_);
  SlabPlan plan;
  plan.want(margin_, RK);
  for (int s = 0; s < 2; ++s) {
    plan.want(gh_[s], RK);
    plan.want(ridx_[s], RK);
    plan.want(tarr_[s], K_);
  }
  plan.want(ghmax_, 2 * size_t(K_));
  plan.want(scales_, K_);
  plan.want(hist_counter_, 1);
  plan.want(scratch_, 1 + size_t(K_));
  plan.want(gh_totals_, 2 * size_t(K_));
  if (K_ <= kMaxReducedClasses) plan.want(max_part_, size_t(gradient_blocks(R_)) * 2 * size_t(K_));
  plan.want(tot_part_, size_t(quantize_round_blocks(R_, K_)) * 2 * size_t(K_));
  plan.want(done_, 4);
  plan.want(round_dev_, 1);
  mask_words_ = (F_ + 31) / 32;
  presize(plan);
  const auto t_alloc = std::chrono::steady_clock::now();
  plan.commit(slabs_, device_);  // a freed engine's slab is reused when it fits
  prof_.host("engine_alloc", ms_since(t_alloc));
  if (G_ > 1) {
    // this rank's first global row: the rows of the lower ranks
    DevBuf<u64> rows(1 + size_t(G_));
    const u64 mine = R_;
    DP_CUDA(cudaMemcpy(rows.get(), &mine, sizeof(u64), cudaMemcpyHostToDevice));
    comm_->all_gather_bytes(rows.get(), rows.get() + 1, sizeof(u64), stream_);
    std::vector<u64> all(G_);
    DP_CUDA(cudaMemcpyAsync(all.data(), rows.get() + 1, G_ * sizeof(u64), cudaMemcpyDeviceToHost, stream_));
    sync_stream();
    for (int r = 0; r < rank_; ++r) row0_ += all[r];
  }
  arena_.reserve(size_t(1) << 20);

  // label validation, initial margins, per-tree array tables; one wait
  std::vector<float> base(K_);
  for (int k = 0; k < K_; ++k) base[k] = p_.base_margin(k);
  float* base_d = reinterpret_cast<float*>(scratch_.get() + 1);
  DP_CUDA(cudaMemsetAsync(scratch_.get(), 0, sizeof(u32), stream_));
  // the last-block counters start at zero (a reused slab holds old data)
  DP_CUDA(cudaMemsetAsync(done_.get(), 0, done_.size() * sizeof(u32), stream_));
  launch_check_labels(d_.labels(), R_, p_.objective_id(), K_, scratch_.get(), stream_);
  std::memcpy(arena_.get() + kArenaHead, base.data(), K_ * sizeof(float));
  DP_CUDA(cudaMemcpyAsync(base_d, arena_.get() + kArenaHead, K_ * sizeof(float), cudaMemcpyHostToDevice, stream_));
  launch_init_margins(margin_.get(), std::max<u64>(R_, 1), K_, base_d, stream_);
  std::vector<TreeArrays> ta(2 * size_t(K_));
  for (int s = 0; s < 2; ++s)
    for (int k = 0; k < K_; ++k) ta[s * K_ + k] = TreeArrays{ridx_[s].get() + u64(k) * R_, gh_[s].get() + u64(k) * R_};
  DP_CUDA(cudaMemcpy(tarr_[0].get(), ta.data(), K_ * sizeof(TreeArrays), cudaMemcpyHostToDevice));
  DP_CUDA(cudaMemcpy(tarr_[1].get(), ta.data() + K_, K_ * sizeof(TreeArrays), cudaMemcpyHostToDevice));
  u32 bad = 0;
  DP_CUDA(cudaMemcpyAsync(&bad, scratch_.get(), sizeof(u32), cudaMemcpyDeviceToHost, stream_));
  sync_stream();
  if (bad) {
    if (p_.objective_id() == kLogistic) fail("label must be in [0,1] for logistic regression");
    if (p_.objective_id() == kSoftprob || p_.objective_id() == kSoftmax)
      fail("label must be an integer in [0, num_class) for multi-class objectives");
    fail("label contains NaN or infinity");
  }
  prof_.host("engine_init", ms_since(t0));
}

Engine::~Engine() {
  if (stream_) {
    DeviceGuard g(device_);
    cudaStreamSynchronize(stream_);
    drop_graph();
    cudaStreamDestroy(stream_);
    // nothing is in flight: the slab goes to the cache for the next engine
    for (auto& slab : slabs_) SlabCache::give(device_, std::move(slab));
  }
}

void Engine::sync() {
  sync_stream();
  prof_.resolve();
  arena_off_ = kArenaHead;
}

template <class T>
T* Engine::stage(const std::vector<T>& v) {
  const size_t bytes = v.size() * sizeof(T);
  size_t off = (std::max(arena_off_, kArenaHead) + 255) & ~size_t(255);
  if (off + bytes > arena_.size()) {
    // all staged copies must land before the arena is replaced
    sync_stream();
    size_t want = std::max(arena_.size() * 2, bytes + 4096);
    PinnedBuf<u8> fresh;
    fresh.reserve(want);
    arena_.swap(fresh);
    off = kArenaHead;
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
void Engine::grow(DevBuf<T>& b, size_t n) {
  if (n <= b.size()) return;
  need(!capturing_, "internal error: buffer growth while capturing a round");
  drop_graph();  // the graph holds the old address
  const auto t0 = std::chrono::steady_clock::now();
  sync_stream();
  b.resize(n);
  prof_.host("grow", ms_since(t0));
}

template <class T>
void Engine::grow_keep(DevBuf<T>& b, size_t n) {
  if (n <= b.size()) return;
  need(!capturing_, "internal error: buffer growth while capturing a round");
  drop_graph();
  const auto t0 = std::chrono::steady_clock::now();
  DevBuf<T> fresh(n);
  if (b.size()) DP_CUDA(cudaMemcpyAsync(fresh.get(), b.get(), b.size() * sizeof(T), cudaMemcpyDeviceToDevice, stream_));
  sync_stream();
  b = std::move(fresh);
  prof_.host("grow", ms_since(t0));
}

void Engine::presize(SlabPlan& plan) {
  const u64 K = u64(K_), D = u64(p_.max_depth);
  const u64 Rt = std::max<u64>(q_->rows_total, 1);
  const u64 RK = std::max<u64>(R_, 1) * K;
  const u64 slot_bytes = slot_elems_ * sizeof(i64);
  // the same bounds the level loop of boost_round derives
  u64 open_hi = K, ids_hi = 1, leaves_hi = 0;
  u64 hist[2] = {0, 0}, tasks = 0, split = 0, opens[2] = {K, 0}, builds[2] = {K, 0}, send = 0;
  bool complete = true;
  for (u64 depth = 0; depth < D; ++depth) {
    if (open_hi > async_open_limit_ || open_hi * slot_bytes > async_hist_bytes_) {
      complete = false;
      break;
    }
    const u64 nbuild_hi = depth == 0 ? K : (open_hi + 1) / 2;
    const u64 next_hi = std::min<u64>(2 * open_hi, K * Rt);
    hist[depth & 1] = std::max<u64>(hist[depth & 1], std::max<u64>(open_hi, 1) * slot_elems_);
    tasks = std::max<u64>(tasks, hist_task_bound(nbuild_hi));
    if (G_ > 1) send = std::max<u64>(send, nbuild_hi * full_slot_elems_);
    split = std::max<u64>(split, open_hi);
    opens[(depth + 1) & 1] = std::max<u64>(opens[(depth + 1) & 1], next_hi);
    builds[(depth + 1) & 1] = std::max<u64>(builds[(depth + 1) & 1], open_hi);
    leaves_hi += open_hi;
    ids_hi = std::min<u64>({ids_hi + 2 * std::min<u64>(open_hi, u64(1) << depth), (u64(1) << (depth + 2)) - 1,
                            2 * Rt + 1});
    open_hi = next_hi;
  }
  if (complete) leaves_hi += open_hi;
  for (int r = 0; r < 2; ++r) {
    plan.want(hist_[r], hist[r]);
    plan.want(open_[r], opens[r]);
    plan.want(build_[r], builds[r]);
    plan.want(triples_[r], 3 * builds[r]);
  }
  plan.want(hist_tasks_, tasks);
  plan.want(eval_nodes_, split);
  plan.want(cand_, split * nchunks_);
  if (G_ > 1) {
    plan.want(send_, send);
    plan.want(gathered_, split * nchunks_ * u64(G_));
  }
  plan.want(split_idx_, split);
  plan.want(zero_list_, split);
  plan.want(part_nodes_, split);
  plan.want(cursors_, 2 * split);
  plan.want(part_tasks_, (RK + kPartChunk - 1) / kPartChunk + split);
  plan.want(leaves_, leaves_hi);
  plan.want(leaf_tasks_, (RK + kLeafChunkRows - 1) / kLeafChunkRows + leaves_hi);
  plan.want(nodes_, ids_hi * K);
  if (col_sampling()) plan.want(fmask_, split * mask_words_);
  plan.want(ctr_, 1);
  plan.want(stats_, size_t(D) + 1);
  plan.want(next_id_, K);
  plan.want(tree_first_, K);
}

RoundBuffers Engine::round_buffers(int depth, u64 cap_split, u64 cap_next) const {
  const int c = depth & 1, n = 1 - c;
  RoundBuffers b{};
  b.nodes = nodes_.get();
  b.next_id = next_id_.get();
  b.tree_first = tree_first_.get();
  b.open_cur = open_[c].get();
  b.open_next = open_[n].get();
  b.build = build_[c].get();
  b.triples = triples_[c].get();
  b.build_next = build_[n].get();
  b.triples_next = triples_[n].get();
  b.hist_tasks = hist_tasks_.get();
  b.hist_counter = hist_counter_.get();
  b.zero_list = zero_list_.get();
  b.eval_nodes = eval_nodes_.get();
  b.cands = G_ > 1 ? gathered_.get() : cand_.get();
  b.nranks = u32(G_);
  b.nchunks = nchunks_;
  b.split_idx = split_idx_.get();
  b.part_nodes = part_nodes_.get();
  b.part_tasks = part_tasks_.get();
  b.cursors = cursors_.get();
  b.leaves = leaves_.get();
  b.leaf_tasks = leaf_tasks_.get();
  b.ctr = ctr_.get();
  b.stats = stats_.get();
  b.K = u32(K_);
  b.by_hess = G_ > 1 ? 1u : 0u;
  b.maxn = u32(std::min<u64>(nodes_.size() / u64(K_), u64(1) << 31));
  b.cap_split = cap_split;
  b.cap_next = cap_next;
  b.cap_hist_tasks = hist_tasks_.size();
  b.cap_part_tasks = part_tasks_.size();
  b.cap_leaves = leaves_.size();
  b.cap_leaf_tasks = leaf_tasks_.size();
  return b;
}

Engine::ReadbackLayout Engine::readback_layout(u64 ids) const {
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  ReadbackLayout L;
  L.ctr = 0;
  L.nid = up(L.ctr + sizeof(RoundCounters));
  L.sc = up(L.nid + size_t(K_) * sizeof(u32));
  L.st = up(L.sc + size_t(K_) * sizeof(Scales));
  L.nodes = up(L.st + (size_t(p_.max_depth) + 1) * sizeof(LevelStats));
  L.bytes = L.nodes + size_t(ids) * size_t(K_) * sizeof(NodeRec);
  return L;
}

std::vector<float> Engine::margins() const {
  DeviceGuard g(device_);
  std::vector<float> out(R_ * K_);
  // margins are read after a round has ended: no collective is in flight
  DP_CUDA(cudaStreamSynchronize(stream_));
  DP_CUDA(cudaMemcpy(out.data(), margin_.get(), out.size() * sizeof(float), cudaMemcpyDeviceToHost));
  return out;
}

bool Engine::all_levels_async() const {
  const u64 K = u64(K_), Rt = std::max<u64>(q_->rows_total, 1);
  const u64 slot_bytes = slot_elems_ * sizeof(i64);
  u64 open_hi = K;
  for (int depth = 0; depth < p_.max_depth; ++depth) {
    if (open_hi > async_open_limit_ || open_hi * slot_bytes > async_hist_bytes_) return false;
    open_hi = std::min<u64>(2 * open_hi, K * Rt);
  }
  return true;
}

void Engine::drop_graph() {
  if (graph_exec_) cudaGraphExecDestroy(graph_exec_);
  if (graph_) cudaGraphDestroy(graph_);
  graph_exec_ = nullptr;
  graph_ = nullptr;
  prof_.drop_graph();
}

void Engine::boost_round(Model& m) {
  DeviceGuard g(device_);
  NvtxRange nv("dp_gbdt: boosting round");
  const auto t_round = std::chrono::steady_clock::now();
  // Rounds after the first replay one CUDA graph of the whole round when every
  // level stays within the asynchronous bounds (nothing then waits on the
  // host inside a round, and buffers no longer move).
  const bool graphable = graphs_ && rounds_ >= 1 && all_levels_async();
  const bool sampling = row_sampling() || col_sampling();
  if (sampling && dev_round_ != u64(m.rounds())) {
    // the sampling hashes read the round from device memory, so a captured
    // round stays valid from one round to the next
    u32* r_h = reinterpret_cast<u32*>(arena_.get() + 128);  // in the arena's head
    *r_h = u32(m.rounds());
    DP_CUDA(cudaMemcpyAsync(round_dev_.get(), r_h, sizeof(u32), cudaMemcpyHostToDevice, stream_));
  }
  RoundOut out;
  if (graphable && graph_exec_ && graph_prof_ == prof_.mode()) {
    DP_CUDA(cudaGraphLaunch(graph_exec_, stream_));
    count_launch(graph_launches_);
    prof_.graph_round();
    out = graph_out_;
  } else if (graphable) {
    drop_graph();
    const u64 l0 = launch_counter().load();
    prof_.start_capture();
    capturing_ = true;
    bool captured = false;
    DP_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    try {
      out = enqueue_round();
      captured = cudaStreamEndCapture(stream_, &graph_) == cudaSuccess && graph_ != nullptr;
    } catch (...) {
      cudaGraph_t partial = nullptr;
      cudaStreamEndCapture(stream_, &partial);
      if (partial) cudaGraphDestroy(partial);
    }
    capturing_ = false;
    const u64 n = launch_counter().load() - l0;
    launch_counter().fetch_sub(n);  // captured, not run
    if (captured && cudaGraphInstantiate(&graph_exec_, graph_, 0) == cudaSuccess) {
      prof_.finish_capture();
      graph_launches_ = n;
      graph_prof_ = prof_.mode();
      graph_out_ = out;
      DP_CUDA(cudaGraphLaunch(graph_exec_, stream_));
      count_launch(graph_launches_);
      prof_.graph_round();
    } else {
      // capture is unavailable here: run this and later rounds directly
      cudaGetLastError();
      prof_.abort_capture();
      drop_graph();
      graphs_ = false;
      out = enqueue_round();
    }
  } else {
    out = enqueue_round();
  }
  prof_.host("round_enqueue", ms_since(t_round));
  finish_round(m, out);
  dev_round_ = sampling ? u64(m.rounds()) : ~u64(0);  // the round's last kernel advanced it
  ++rounds_;
}

Engine::RoundOut Engine::enqueue_round() {
  const int K = K_;
  const u64 R = R_;
  const u32 F = F_;
  const int D = p_.max_depth;
  const u32 ftiles = (F + hist_tile_ - 1) / hist_tile_;
  const SplitParams sp = p_.split_params();
  const u64 Rt = std::max<u64>(q_->rows_total, 1);
  const u64 RK = std::max<u64>(R, 1) * u64(K);
  const u64 slot_bytes = slot_elems_ * sizeof(i64);

  // ---- gradients and quantiser scales
  u32* const gmax = ghmax_.get();  // [K] |g| maxima, then [K] h maxima (f32 bits)
  u32* const hmax = ghmax_.get() + K;
  const bool one_rank = !comm_ || G_ == 1;
  grow(ctr_, 1);
  grow(stats_, size_t(D) + 1);
  grow(next_id_, K);
  grow(tree_first_, K);
  grow(open_[0], K);
  grow(build_[0], K);
  grow_keep(nodes_, size_t(K));
  RoundCounters* const ctr = ctr_.get();  // allocated once; never regrown
  const RoundBuffers rb0 = round_buffers(0, 0, 0);

  // ---- gradients and quantiser scales.  Up to 64 classes the maxima are
  // reduced by the gradient launch's last block (with one rank it also
  // computes the scales); beyond, per-class atomics on zeroed maxima.
  prof_.begin(stream_, "gradients", double(R) * K * (4 + 8) + double(R) * 4);
  RowSample rs;
  if (row_sampling()) rs = RowSample{p_.subsample, p_.seed, round_dev_.get(), row0_};
  const bool reduced = K <= kMaxReducedClasses;
  if (reduced) {
    launch_gradients_reduced(p_.objective_id(), K, margin_.get(), d_.labels(), R, gh_[0].get(), gmax, hmax,
                             max_part_.get(), done_.get(), one_rank ? scales_.get() : nullptr, stream_, rs);
  } else {
    DP_CUDA(cudaMemsetAsync(gmax, 0, 2 * size_t(K) * sizeof(u32), stream_));
    launch_gradients(p_.objective_id(), K, margin_.get(), d_.labels(), R, gh_[0].get(), gmax, hmax, stream_, rs);
  }
  prof_.end(stream_);
  if (!one_rank) comm_->max_u32(gmax, 2 * size_t(K), stream_);
  if (!reduced || !one_rank) launch_scales(K, gmax, hmax, scales_.get(), stream_);
  // (g, h) become exact int32 pairs once per round (every later pass reads
  // them), the row indices the identity, and the quantised root sums are
  // reduced by the launch's last block, which with one rank also starts the
  // round: K roots, open at depth 0 and built directly
  launch_quantize_round(rb0, gh_[0].get(), R, scales_.get(), ridx_[0].get(), tot_part_.get(), done_.get() + 1,
                        gh_totals_.get(), u32(D) + 1, one_rank, stream_);
  if (!one_rank) {
    // root totals over every rank's rows
    comm_->sum_i64(gh_totals_.get(), 2 * size_t(K), stream_);
    launch_round_init(rb0, R, gh_totals_.get(), u32(D) + 1, stream_);
  }

  // Host-side upper bounds of the device counts, which size the buffers:
  // open nodes of this level, node ids per tree, closed leaves.  Every open
  // node holds at least one row over all ranks (a split with an empty side
  // has gain -gamma <= 0), so open nodes never exceed K * rows.
  u64 open_hi = u64(K), ids_hi = 1, leaves_hi = 0;
  std::vector<int> pi_hist(D, -1), pi_eval(D, -1);
  int set = 0, region = 0, depth = 0;
  bool folded = false;              // the last level routed its rows straight into the margins
  static const char* const kLevelNames[] = {"level 0", "level 1", "level 2", "level 3", "level 4", "level 5",
                                             "level 6", "level 7", "level 8", "level 9", "level 10+"};
  for (; depth < D; ++depth) {
    NvtxRange nv_level(kLevelNames[depth < 10 ? depth : 10]);
    u64 nbuild_hi = depth == 0 ? u64(K) : (open_hi + 1) / 2;
    if (open_hi > async_open_limit_ || open_hi * slot_bytes > async_hist_bytes_) {
      RoundCounters* c_h = reinterpret_cast<RoundCounters*>(arena_.get());  // the arena's head
      DP_CUDA(cudaMemcpyAsync(c_h, ctr, sizeof(RoundCounters), cudaMemcpyDeviceToHost, stream_));
      sync_stream();
      open_hi = c_h->n_open;
      nbuild_hi = c_h->n_build;
      if (open_hi == 0) break;
    }
    const u64 next_hi = std::min<u64>(2 * open_hi, u64(K) * Rt);
    const u64 ids_next = std::min<u64>({ids_hi + 2 * std::min<u64>(open_hi, u64(1) << depth),
                                        (u64(1) << (depth + 2)) - 1, 2 * Rt + 1});
    grow(hist_[region], std::max<u64>(open_hi, 1) * slot_elems_);
    grow(hist_tasks_, hist_task_bound(nbuild_hi));
    grow(eval_nodes_, open_hi);
    grow(cand_, open_hi * nchunks_);
    if (G_ > 1) {
      grow(send_, nbuild_hi * full_slot_elems_);
      grow(gathered_, open_hi * nchunks_ * u64(G_));
    }
    grow(split_idx_, open_hi);
    grow(zero_list_, open_hi);
    if (col_sampling()) grow(fmask_, open_hi * mask_words_);
    grow(part_nodes_, open_hi);
    grow(cursors_, 2 * open_hi);
    grow(part_tasks_, (RK + kPartChunk - 1) / kPartChunk + open_hi);
    grow(open_[(depth + 1) & 1], next_hi);
    grow(build_[(depth + 1) & 1], open_hi);
    grow(triples_[(depth + 1) & 1], 3 * open_hi);
    grow_keep(leaves_, leaves_hi + open_hi);
    grow_keep(nodes_, ids_next * K);
    const RoundBuffers rb = round_buffers(depth, open_hi, next_hi);
    i64* hist = hist_[region].get();

    // ---- histograms of the directly built nodes, then their siblings.  With
    // several ranks, each builds partial histograms of all features for its
    // rows (group-major), and a reduce-scatter leaves every rank the sums of
    // its own feature group.
    launch_hist_tasks(rb, ftiles, hist_tile_, depth, hist_target_tasks_, stream_);
    i64* hout = G_ > 1 ? send_.get() : hist;
    launch_zero_listed(rb, hout, slot_elems_, nbuild_hi * slot_elems_, u32(G_), stream_);
    const HistLayout lay{fg_, slot_elems_, nbuild_hi * slot_elems_};
    pi_hist[depth] = prof_.begin(stream_, "histograms", 0.0);
    // (the task kernel zeroed the queue counter)
    if (wide_)
      launch_histograms_wide(q_->bins.get(), q_->bin_stride, F, true, tarr_[set].get(), scales_.get(),
                             hist_tasks_.get(), 0, hist_counter_.get(), hout, stream_, &ctr->n_hist_tasks,
                             G_ > 1 ? &lay : nullptr, true);
    else
      launch_histograms(q_->bins.get(), q_->bin_stride, F, max_bins_, true, tarr_[set].get(), scales_.get(),
                        hist_tasks_.get(), 0, hist_counter_.get(), hout, stream_, &ctr->n_hist_tasks,
                        G_ > 1 ? &lay : nullptr, true);
    prof_.end(stream_);
    if (G_ > 1) {
      prof_.begin(stream_, "exchange_hist", double(nbuild_hi * full_slot_elems_) * sizeof(i64));
      comm_->reduce_scatter_i64(send_.get(), hist, nbuild_hi * slot_elems_, stream_);
      prof_.end(stream_);
    }
    // ---- split evaluation over this rank's feature group, then (G > 1) the
    // per-node best over all groups
    if (col_sampling())
      launch_feature_masks(rb, F, p_.seed, round_dev_.get(), p_.colsample_bytree, p_.colsample_bylevel,
                           p_.colsample_bynode, depth, fmask_.get(), mask_words_, stream_);
    pi_eval[depth] = prof_.begin(stream_, "eval_splits", 0.0);
    launch_eval_candidates_dev(hist, f_own_n_, q_->nbins.get() + f_own0_, q_->has_missing.get() + f_own0_,
                               eval_nodes_.get(), &ctr->n_open, scales_.get(), sp, cand_.get(), nchunks_, stream_,
                               fg_, f_own0_, col_sampling() ? fmask_.get() : nullptr, mask_words_,
                               hist_[1 - region].get(), depth + 1 < D ? 1 : 0);
    prof_.end(stream_);
    if (G_ > 1) {
      const u64 bytes = open_hi * nchunks_ * sizeof(SplitCand);
      prof_.begin(stream_, "exchange_cands", double(bytes * u64(G_)));
      comm_->all_gather_bytes(cand_.get(), gathered_.get(), bytes, stream_);
      prof_.end(stream_);
    }
    launch_decide(rb, q_->cut.get(), q_->has_missing.get(), F, depth, D, set, stream_);

    if (depth + 1 == D && fold_last_) {
      // ---- the last level: its children are leaves and nothing is built
      // from them, so rows do not move.  Leaf values of every closed node and
      // of the children, the closed leaves' margin update, then each split
      // node's rows add their child's value as they are routed.
      leaves_hi += open_hi;
      grow(leaf_tasks_, (RK + kLeafChunkRows - 1) / kLeafChunkRows + leaves_hi);
      const RoundBuffers rl = round_buffers(depth, open_hi, next_hi);
      u32* const sets[2] = {ridx_[0].get(), ridx_[1].get()};
      launch_leaf_values(rl, scales_.get(), sp, sets, R, stream_, true);
      prof_.begin(stream_, "leaf_update", double(R) * K * 12.0);
      launch_leaf_update_dev(leaf_tasks_.get(), &ctr->n_leaf_tasks, margin_.get(), u32(K), stream_);
      launch_partition_leaves(q_->bins_blk.get(), 32 * u64(F), tarr_[set].get(), part_nodes_.get(),
                              part_tasks_.get(), &ctr->n_part_tasks, cursors_.get(), margin_.get(), u32(K), stream_);
      prof_.end(stream_);
      ids_hi = ids_next;  // the children's ids
      folded = true;
      break;
    }

    // ---- partition and the children's segments
    prof_.begin(stream_, "partition", 0.0);
    launch_partition_dev(q_->bins_blk.get(), 32 * u64(F), tarr_[set].get(), tarr_[1 - set].get(), part_nodes_.get(),
                         part_tasks_.get(), &ctr->n_part_tasks, cursors_.get(), stream_);
    prof_.end(stream_);
    launch_children(rb, depth, D, stream_);

    leaves_hi += open_hi;
    open_hi = next_hi;
    ids_hi = ids_next;
    set = 1 - set;
    region = 1 - region;
  }

  if (!folded) {
    // ---- nodes still open close as leaves; leaf values and margin update
    grow_keep(leaves_, leaves_hi + open_hi);
    leaves_hi += open_hi;
    grow(leaf_tasks_, (RK + kLeafChunkRows - 1) / kLeafChunkRows + leaves_hi);
    const RoundBuffers rb = round_buffers(depth, open_hi, open_hi);
    launch_decide(rb, q_->cut.get(), q_->has_missing.get(), F, D, D, set, stream_);
    u32* const sets[2] = {ridx_[0].get(), ridx_[1].get()};
    launch_leaf_values(rb, scales_.get(), sp, sets, R, stream_);
    prof_.begin(stream_, "leaf_update", double(R) * K * 12.0);
    launch_leaf_update_dev(leaf_tasks_.get(), &ctr->n_leaf_tasks, margin_.get(), u32(K), stream_);
    prof_.end(stream_);
  }
  if (row_sampling() || col_sampling()) launch_bump_round(round_dev_.get(), stream_);

  // ---- the round's results straight into pinned host memory (the host
  // reads them after one wait)
  {
    const u64 ids_read = std::min<u64>(ids_hi, nodes_.size() / u64(K));
    const ReadbackLayout L = readback_layout(ids_read);
    readback_.reserve(L.bytes);
    u8* host = nullptr;
    DP_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&host), readback_.get(), 0));
    const u32* src[5] = {reinterpret_cast<const u32*>(ctr), next_id_.get(),
                         reinterpret_cast<const u32*>(scales_.get()), reinterpret_cast<const u32*>(stats_.get()),
                         reinterpret_cast<const u32*>(nodes_.get())};
    u32* dst[5] = {reinterpret_cast<u32*>(host + L.ctr), reinterpret_cast<u32*>(host + L.nid),
                   reinterpret_cast<u32*>(host + L.sc), reinterpret_cast<u32*>(host + L.st),
                   reinterpret_cast<u32*>(host + L.nodes)};
    const u64 words[5] = {sizeof(RoundCounters) / 4, u64(K), u64(K) * sizeof(Scales) / 4,
                          (u64(D) + 1) * sizeof(LevelStats) / 4, ids_read * u64(K) * sizeof(NodeRec) / 4};
    launch_copy_words(src, dst, words, 5, stream_);
  }

  RoundOut out;
  out.ids_hi = ids_hi;
  out.pi_hist = std::move(pi_hist);
  out.pi_eval = std::move(pi_eval);
  return out;
}

void Engine::finish_round(Model& m, const RoundOut& out) {
  NvtxRange nv("dp_gbdt: round read-back");
  const int K = K_;
  const u32 F = F_;
  const int D = p_.max_depth;
  const SplitParams sp = p_.split_params();
  const u64 slot_bytes = slot_elems_ * sizeof(i64);
  const u64 ids_read = std::min<u64>(out.ids_hi, nodes_.size() / u64(K));
  auto t_wait = std::chrono::steady_clock::now();
  sync_stream();
  prof_.host("round_wait", ms_since(t_wait));
  t_wait = std::chrono::steady_clock::now();
  const ReadbackLayout L = readback_layout(ids_read);
  need(readback_.size() >= L.bytes, "internal error: round read-back buffer too small");
  const u8* rbh = readback_.get();
  const RoundCounters* c_h = reinterpret_cast<const RoundCounters*>(rbh + L.ctr);
  const u32* nid_h = reinterpret_cast<const u32*>(rbh + L.nid);
  const Scales* sc_h = reinterpret_cast<const Scales*>(rbh + L.sc);
  const LevelStats* st_h = reinterpret_cast<const LevelStats*>(rbh + L.st);
  const NodeRec* nd_h = reinterpret_cast<const NodeRec*>(rbh + L.nodes);
  const u32 ovf = c_h->overflow;
  if (ovf & kOvfLostRows) fail("partition lost rows");
  if (ovf & kOvfBadCand) fail("a split candidate from the rank exchange names no feature of the matrix");
  if (ovf) fail("internal error: a per-round work list overflowed (flags " + std::to_string(ovf) + ")");
  for (int d = 0; d < D; ++d) {
    const LevelStats& st = st_h[d];
    prof_.set_bytes(out.pi_hist[d], double(st.rows_built) * (double(F) + 12.0) +
                                        double(st.n_build) * double(F) * kMaxBins * 16.0);
    prof_.set_units(out.pi_hist[d], double(st.rows_built) * double(F));
    // built nodes read once; a derived sibling reads parent and sibling and
    // (before the last level) writes itself
    const double derived = d > 0 ? double(st.n_open - st.n_build) : 0.0;
    prof_.set_bytes(out.pi_eval[d], (double(st.n_open) + derived * (d + 1 < D ? 2.0 : 1.0)) * slot_bytes);
  }
  prof_.resolve();
  if (prof_.graph_timing_failed()) {
    // this driver does not time graph event nodes: profiled rounds run directly
    graphs_ = false;
    drop_graph();
  }

  for (int k = 0; k < K; ++k) {
    const u64 n = nid_h[k];
    need(n >= 1 && n <= ids_read, "internal error: node count of a tree out of range");
    Tree t;
    t.klass = k;
    const Scales sc = sc_h[k];
    const double ish = 1.0 / double(sc.sh);
    for (u64 id = 0; id < n; ++id) {
      const NodeRec& r = nd_h[id * K + k];
      t.add_node(r.parent);
      t.left[id] = r.left;
      t.right[id] = r.right;
      t.feature[id] = r.left < 0 ? 0 : r.feature;
      t.cond[id] = r.cond;
      t.default_left[id] = u8(r.default_left);
      t.loss_change[id] = r.gain;
      t.base_weight[id] = leaf_weight(r.gq, r.hq, sc.sg, sc.sh, sp);
      t.sum_hess[id] = float(double(r.hq) * ish);
    }
    m.trees.push_back(std::move(t));
  }
  arena_off_ = kArenaHead;
  m.iteration_indptr.push_back(int(m.trees.size()));
  prof_.host("round_readback", ms_since(t_wait));
}

}  // namespace dp
