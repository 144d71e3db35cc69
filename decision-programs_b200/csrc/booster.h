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

namespace dp {

class Booster {
 public:
  TrainParams params;
  Model model;
  Comm* comm = nullptr;  // borrowed (dp_booster_set_comm)
  bool profiling = false;

  void set_param(const std::string& key, const std::string& value);
  void update_one_iter(int iter, DMatrix* d);
  int boosted_rounds() const { return model.rounds(); }
  const std::string& save_model_json();
  const std::string& save_config_json();
  void load_model_json(const std::string& text);
  std::unique_ptr<Booster> slice(int begin, int end, int step) const;
  Engine* engine() const { return engine_.get(); }

  std::string out_buf;      // borrowed text outputs
  std::string profile_buf;

 private:
  std::unique_ptr<Engine> engine_;
  bool params_changed_ = false;
  std::string engine_objective_;
  int engine_classes_ = 0, engine_max_bin_ = 0;
};

}  // namespace dp
