// Booster parameters and the tree ensemble in the XGBoost 3.4.1 JSON layout
// the reference reads back (native/class_io.hpp:131-205,
// cmake/fixtures/xgboost-parser.json).
#pragma once
#include <map>
#include <string>
#include <vector>

#include "common.h"
#include "dp_math.cuh"
#include "kernels.h"

namespace dp {

struct TrainParams {
  std::string objective = "reg:squarederror";
  int num_class = 0;           // XGBoost convention: 0 for scalar objectives
  int max_depth = 6;
  int max_bin = 256;
  double eta = 0.3, lambda = 1.0, alpha = 0.0, gamma = 0.0, min_child_weight = 1.0;
  double subsample = 1.0, colsample_bytree = 1.0, colsample_bylevel = 1.0, colsample_bynode = 1.0;
  std::vector<float> base_score;  // empty: objective default (0.5 logistic, 0 otherwise)
  long long seed = 0;
  int device = -1;             // "cuda:N"; -1 = the caller's current device
  std::map<std::string, std::string> raw;  // every accepted key as given

  int K() const { return (objective.rfind("multi:", 0) == 0) ? num_class : 1; }
  int objective_id() const;
  SplitParams split_params() const {
    SplitParams p;
    p.lambda = lambda; p.alpha = alpha; p.gamma = gamma; p.min_child_weight = min_child_weight; p.eta = eta;
    return p;
  }
  // Initial margin of output k (base_score mapped through the link).
  float base_margin(int k) const;
  void set(const std::string& key, const std::string& value);
};

struct Tree {
  std::vector<i32> left, right, parent, feature;
  std::vector<float> cond, base_weight, loss_change, sum_hess;
  std::vector<u8> default_left;
  int klass = 0;
  int add_node(i32 par) {
    left.push_back(-1); right.push_back(-1); parent.push_back(par); feature.push_back(0);
    cond.push_back(0.f); base_weight.push_back(0.f); loss_change.push_back(0.f); sum_hess.push_back(0.f);
    default_left.push_back(0);
    return int(left.size()) - 1;
  }
  size_t size() const { return left.size(); }
};

struct Model {
  int num_feature = 0;
  std::vector<Tree> trees;
  std::vector<int> iteration_indptr{0};
  int rounds() const { return int(iteration_indptr.size()) - 1; }
};

std::string model_to_json(const Model& m, const TrainParams& p);
std::string config_to_json(const Model& m, const TrainParams& p);
// Parses a model written by model_to_json (or any XGBoost 3.x JSON model of
// numeric gbtree trees); fills `p` with the objective and shape.
void model_from_json(const std::string& text, Model& m, TrainParams& p);

}  // namespace dp
