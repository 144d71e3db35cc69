// Training engine behind XGBoosterUpdateOneIter: grows the K trees of one
// boosting round level-synchronously on the GPU (one histogram, split and
// partition launch per level for all K trees), with sibling subtraction and
// row-sharded histogram sums over `comm` when several GPUs share the rows.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <string>
#include <vector>

#include "comm.h"
#include "common.h"
#include "dmatrix.h"
#include "kernels.h"
#include "model.h"

namespace dp {

// Per-kernel timing with CUDA events on the engine's stream.
class Profiler {
 public:
  void enable(bool on) { on_ = on; }
  bool enabled() const { return on_; }
  void begin(cudaStream_t s, const char* name, double alg_bytes);
  void end(cudaStream_t s);
  void resolve();  // after the stream has been synchronised
  std::string json() const;
  void reset() { stats_.clear(); }
  ~Profiler();

 private:
  struct Pending { cudaEvent_t a, b; std::string name; double bytes; };
  struct Stat { u64 launches = 0; double ms = 0.0; double bytes = 0.0; };
  bool on_ = false;
  std::vector<Pending> pending_;
  std::vector<cudaEvent_t> free_;
  std::map<std::string, Stat> stats_;
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
  void update_params(const TrainParams& p) { p_ = p; }
  DMatrix* matrix() const { return &d_; }
  Profiler& profiler() { return prof_; }
  cudaStream_t stream() const { return stream_; }
  // Training margins [R][K] copied to host.
  std::vector<float> margins() const;

 private:
  struct Open {
    int tree, id, slot;
    i64 begin, count;      // local positions
    i64 gcount;            // rows over all ranks
    i64 gq, hq;
  };
  struct Leaf { int tree, id, set; i64 begin, count; };

  void sync();
  template <class T>
  T* stage(const std::vector<T>& v);  // copies into the pinned arena
  template <class T>
  void upload(DevBuf<T>& dst, const std::vector<T>& v);
  template <class T>
  const T* download(const T* src, size_t n);  // into the arena; valid after sync()

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
  u64 slot_elems_ = 0;

  DevBuf<float> margin_;
  DevBuf<float2> gh_[2];
  DevBuf<u32> ridx_[2];
  DevBuf<TreeArrays> tarr_[2];
  DevBuf<u32> gmax_, hmax_;
  DevBuf<Scales> scales_;
  DevBuf<i64> hist_[2];
  DevBuf<HistTask> hist_tasks_;
  DevBuf<u32> hist_counter_;
  DevBuf<u32> triples_;
  DevBuf<EvalNode> eval_nodes_;
  DevBuf<SplitCand> cand_, best_;
  DevBuf<PartNode> part_nodes_;
  DevBuf<PartTask> part_tasks_;
  DevBuf<u32> cursors_;
  DevBuf<i64> counts_;
  DevBuf<LeafTask> leaf_tasks_;

  PinnedBuf<u8> arena_;
  size_t arena_off_ = 0;
  Profiler prof_;
};

}  // namespace dp
