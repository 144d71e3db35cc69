// Training engine behind XGBoosterUpdateOneIter: grows the K trees of one
// boosting round level-synchronously on the GPU (one histogram, split and
// partition launch per level for all K trees), with sibling subtraction and
// row-sharded histogram sums over `comm` when several GPUs share the rows.
// Every per-level decision is taken on the device (level.h), so a round is
// enqueued without waiting and its trees are read back once at the end.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <string>
#include <vector>

#include "comm.h"
#include "common.h"
#include "dmatrix.h"
#include "kernels.h"
#include "level.h"
#include "model.h"

namespace dp {

// Per-kernel timing with CUDA events on the engine's stream.
class Profiler {
 public:
  // Mode 0: off; 1: every timed launch; 2: histogram launches only (the
  // cheapest instrumentation of a timed round).
  void enable(int mode) { mode_ = mode; }
  bool enabled() const { return mode_ != 0; }
  int mode() const { return mode_; }
  // Returns the launch's index for set_bytes (-1 when disabled).
  int begin(cudaStream_t s, const char* name, double alg_bytes);
  // Graph capture: launches timed between start_capture and finish_capture
  // are recorded as event nodes of the graph and kept; graph_round() marks
  // the current round as a replay whose times resolve() reads from them.
  void start_capture() { capturing_ = true; }
  void finish_capture() {
    capturing_ = false;
    graph_pending_ = std::move(pending_);
    pending_.clear();
  }
  void abort_capture();
  void drop_graph();
  void graph_round() { graph_round_ = true; }
  bool graph_timing_failed() const { return graph_timing_failed_; }
  // Algorithmic bytes of a launch known only after it ran (before resolve()).
  void set_bytes(int idx, double alg_bytes);
  // Work units of a launch (histograms: (row, feature) pairs), known after it ran.
  void set_units(int idx, double units);
  void end(cudaStream_t s);
  void resolve();  // after the stream has been synchronised
  std::string json() const;
  void reset() { stats_.clear(); log_.clear(); host_.clear(); }
  // Host-side time of a phase (always recorded; cheap).
  void host(const char* name, double ms) {
    auto& h = host_[name];
    h.first += 1;
    h.second += ms;
  }
  ~Profiler();

 private:
  struct Pending { cudaEvent_t a, b; std::string name; double bytes; double units = 0.0; };
  struct Stat { u64 launches = 0; double ms = 0.0; double bytes = 0.0; double units = 0.0; };
  int mode_ = 0;
  bool open_ = false;  // the last begin() recorded an event
  bool capturing_ = false, graph_round_ = false, graph_timing_failed_ = false;
  void record(cudaEvent_t e, cudaStream_t s);
  bool accumulate(const Pending& p);
  std::vector<Pending> pending_;
  std::vector<Pending> graph_pending_;
  std::vector<cudaEvent_t> free_;
  std::map<std::string, Stat> stats_;
  struct Entry { std::string name; float ms; double bytes; };
  std::vector<Entry> log_;  // the most recent launches, bounded
  std::map<std::string, std::pair<u64, double>> host_;  // phase -> (count, ms)
  cudaEvent_t take();
};

class Engine {
 public:
  Engine(DMatrix& d, const TrainParams& p, Comm* comm);
  ~Engine();
  Engine(const Engine&) = delete;
  Engine& operator=(const Engine&) = delete;

  void boost_round(Model& m);
  // Regularisation / depth / learning-rate changes between rounds.
  void update_params(const TrainParams& p) {
    p_ = p;
    drop_graph();  // parameters are baked into the captured launches
  }
  DMatrix* matrix() const { return &d_; }
  Profiler& profiler() { return prof_; }
  cudaStream_t stream() const { return stream_; }
  // Training margins [R][K] copied to host.
  std::vector<float> margins() const;

 private:
  void sync();
  // Waits for the stream; with a communicator, through its watchdog (a peer
  // that stops or fails aborts the communicator and throws instead of waiting
  // for good).  Before an abort the round's CUDA graph, which holds the
  // communicator's calls, is released (NCCL's abort waits for that), and
  // rounds are no longer captured.
  void sync_stream() {
    if (comm_ && G_ > 1) {
      comm_->wait(stream_, [this] {
        drop_graph();
        graphs_ = false;
      });
    } else {
      DP_CUDA(cudaStreamSynchronize(stream_));
    }
  }
  template <class T>
  T* stage(const std::vector<T>& v);  // copies into the pinned arena
  template <class T>
  void upload(DevBuf<T>& dst, const std::vector<T>& v);
  // Capacity growth between launches: `grow` drops the contents, `grow_keep`
  // keeps them; both wait for the stream first, since it may still use them.
  template <class T>
  void grow(DevBuf<T>& b, size_t n);
  template <class T>
  void grow_keep(DevBuf<T>& b, size_t n);
  RoundBuffers round_buffers(int depth, u64 cap_split, u64 cap_next) const;
  // What the host needs after a round's work is enqueued.
  struct RoundOut {
    u64 ids_hi = 1;                             // bound on node ids per tree
    std::vector<int> pi_hist, pi_eval;          // profiler entries per level
  };
  RoundOut enqueue_round();                       // every launch of one round
  void finish_round(Model& m, const RoundOut& out);  // one read-back, the trees
  bool all_levels_async() const;
  bool row_sampling() const { return p_.subsample < 1.0; }
  bool col_sampling() const {
    return p_.colsample_bytree < 1.0 || p_.colsample_bylevel < 1.0 || p_.colsample_bynode < 1.0;
  }
  void drop_graph();
  // Sizes every round buffer for the levels whose bounds stay within the
  // asynchronous limits, so steady rounds allocate nothing.
  void presize(SlabPlan& plan);

  DMatrix& d_;
  TrainParams p_;
  Comm* comm_;
  int device_;
  cudaStream_t stream_ = nullptr;
  const Quantized* q_ = nullptr;
  u64 R_ = 0;
  u32 F_ = 0;
  int K_ = 1;
  int max_bins_ = kMaxBins;  // bin codes are < max_bins_ (missing code 255 included)
  // Feature groups: with G ranks each owns fg_ = ceil(F / G) consecutive
  // features (the last group may be short or empty).  A rank keeps the
  // summed histograms of its own group only: slot_elems_ = fg_ * 2 * 256.
  int G_ = 1, rank_ = 0;
  u32 fg_ = 0, f_own0_ = 0, f_own_n_ = 0;
  u32 nchunks_ = 1;          // feature chunks of split evaluation per group (>= 1, equal on every rank)
  u64 slot_elems_ = 0;       // elements of one own-group histogram slot
  u64 full_slot_elems_ = 0;  // elements of one slot over all groups (G * fg_ * 2 * 256)

  std::vector<DevBuf<u8>> slabs_;  // memory of the DevBuf views below
  DevBuf<float> margin_;
  DevBuf<float2> gh_[2];
  DevBuf<u32> ridx_[2];
  DevBuf<TreeArrays> tarr_[2];
  DevBuf<u32> ghmax_;  // gradient and hessian maxima of the round, [2][K]
  // per-block partials of the round-start reductions (gradient maxima when
  // K <= 64; quantised root sums) and the last-block counters, which every
  // launch leaves zero
  DevBuf<u32> max_part_;
  DevBuf<i64> tot_part_;
  DevBuf<u32> done_;
  DevBuf<Scales> scales_;
  DevBuf<i64> hist_[2];
  DevBuf<HistTask> hist_tasks_;
  DevBuf<u32> hist_counter_;
  // 64-feature histogram tasks (k_hist_wide)
  bool wide_ = false;
  u32 hist_tile_ = kHistFeatureTile;
  u32 hist_target_tasks_ = 4 * 148;  // histogram tasks per level, about
  // Capacity of a level's histogram task list for nbuild built nodes: pieces
  // of at least total * tiles / target rows, at least one per node and tile.
  u64 hist_task_bound(u64 nbuild) const {
    return (nbuild + 1) * u64((F_ + hist_tile_ - 1) / hist_tile_) + hist_target_tasks_;
  }
  DevBuf<EvalNode> eval_nodes_;
  DevBuf<SplitCand> cand_;                 // [open][nchunks_] this rank's candidates
  DevBuf<i64> send_;                       // this rank's partial histograms, group-major (G > 1)
  DevBuf<SplitCand> gathered_;             // [G][open][nchunks_] all ranks' candidates (G > 1)
  DevBuf<i64> gh_totals_;                  // [K][2] root sums
  DevBuf<PartNode> part_nodes_;
  DevBuf<PartTask> part_tasks_;
  DevBuf<u32> cursors_;
  DevBuf<LeafTask> leaf_tasks_;
  // round state on the device (level.h)
  DevBuf<NodeRec> nodes_;
  DevBuf<u32> next_id_, tree_first_, split_idx_, zero_list_;
  DevBuf<OpenRec> open_[2];
  DevBuf<u32> build_[2], triples_[2];
  DevBuf<LeafRec> leaves_;
  DevBuf<RoundCounters> ctr_;
  DevBuf<LevelStats> stats_;
  DevBuf<u32> scratch_;  // [0]: label check flag; [1, 1 + K): initial margins (f32 bits)
  // sampling: the round counter the sampling hashes read (device), this
  // rank's first global row, per-node feature masks of a level
  DevBuf<u32> round_dev_;
  DevBuf<u32> fmask_;
  u32 mask_words_ = 0;
  u64 row0_ = 0;
  u64 dev_round_ = ~u64(0);  // value of round_dev_ when known
  int sms_ = 148;
  // CUDA graph of a whole round (replayed while the bounds and buffers hold)
  bool graphs_ = true;  // DP_CUDA_GRAPHS=0 turns capture off
  // The last level adds leaf values while routing rows instead of moving
  // them (DP_FOLD_LAST_LEVEL=0: moves them and updates margins afterwards).
  bool fold_last_ = true;
  bool capturing_ = false;
  cudaGraph_t graph_ = nullptr;
  cudaGraphExec_t graph_exec_ = nullptr;
  int graph_prof_ = 0;  // profiler mode the graph was captured with
  u64 graph_launches_ = 0;
  RoundOut graph_out_;
  u64 rounds_ = 0;
  // A level whose open-node bound exceeds either limit first reads the exact
  // counts back (one small copy) and sizes its buffers by them.
  u64 async_open_limit_ = u64(1) << 16;
  u64 async_hist_bytes_ = u64(4) << 30;

  // The round's results (counters, node counts, scales, level statistics,
  // node records), written into pinned host memory by the round's last
  // kernel; sized and laid out by readback_layout().
  struct ReadbackLayout {
    size_t ctr = 0, nid = 0, sc = 0, st = 0, nodes = 0, bytes = 0;
  };
  ReadbackLayout readback_layout(u64 ids) const;
  PinnedBuf<u8> readback_;
  // Pinned staging: the first kArenaHead bytes hold round counters read back
  // mid-round; staged copies start after them.
  static constexpr size_t kArenaHead = 256;
  PinnedBuf<u8> arena_;
  size_t arena_off_ = kArenaHead;
  Profiler prof_;
};

}  // namespace dp
