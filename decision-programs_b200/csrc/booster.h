// Booster object behind the XGBoost-style handle: parameters, the tree
// ensemble, the training engine bound to one training matrix, and the
// borrowed output buffers the C ABI hands out (valid until the next call on
// the same handle, as the reference expects: native/class_study_train.hpp:63-64).
#pragma once
#include <memory>
#include <string>
#include <vector>

#include "comm.h"
#include "dmatrix.h"
#include "engine.h"
#include "model.h"
#include "predict.h"

namespace dp {

class Booster {
 public:
  TrainParams params;
  Model model;
  Comm* comm = nullptr;  // borrowed (dp_booster_set_comm)
  int profiling = 0;  // profiler mode (see Profiler::enable)

  void set_param(const std::string& key, const std::string& value);
  void update_one_iter(int iter, DMatrix* d);
  int boosted_rounds() const { return model.rounds(); }
  const std::string& save_model_json();
  const std::string& save_config_json();
  void load_model_json(const std::string& text);
  std::unique_ptr<Booster> slice(int begin, int end, int step) const;
  Engine* engine() const { return engine_.get(); }

  // Prediction over a dense fp32 device matrix (XGBoosterPredictFromCudaArray):
  // type 0 = the objective's output, 1 = raw margins; rounds
  // [it_begin, it_end), it_end == 0 meaning all.  Returns a device pointer
  // owned by the booster (valid until the next call on it) and the shape.
  struct PredictRequest {
    const float* x = nullptr;
    u64 rows = 0, cols = 0, stride = 0;
    int device = 0, type = 0, it_begin = 0, it_end = 0;
    bool strict_shape = false, has_mv = false;
    float mv = 0.f;
  };
  const float* predict(const PredictRequest& q, const u64** shape, u64* dims);

  std::string out_buf;      // borrowed text outputs
  std::string profile_buf;

 private:
  std::unique_ptr<Engine> engine_;
  bool params_changed_ = false;
  u64 model_version_ = 0;  // bumped whenever the ensemble changes
  // The ensemble laid out for prediction on one device, and the outputs.
  struct PredState {
    int device = -1;
    u64 version = ~u64(0);
    cudaStream_t stream = nullptr;
    DevBuf<PredNode> nodes;
    DevBuf<u32> tree_off, tree_class, bad;
    DevBuf<float> base, margin, out;
    u32 max_feature = 0;  // largest split feature + 1
    std::vector<u64> shape;
    ~PredState();
  };
  std::unique_ptr<PredState> pred_;
  std::string engine_objective_;
  int engine_classes_ = 0, engine_max_bin_ = 0;
};

}  // namespace dp
