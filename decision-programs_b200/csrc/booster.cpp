#include "booster.h"

namespace dp {

void Booster::set_param(const std::string& key, const std::string& value) {
  params.set(key, value);
  params_changed_ = true;
}

void Booster::update_one_iter(int iter, DMatrix* d) {
  need(d != nullptr, "training matrix handle is null");
  need(iter >= 0, "iteration must be non-negative");
  const int K = params.K();
  need(K >= 1, "num_class must be at least 1 for multi-class objectives");
  if (params.objective.rfind("multi:", 0) == 0) need(params.num_class >= 2, "num_class must be at least 2");
  need(params.subsample == 1.0 && params.colsample_bytree == 1.0 && params.colsample_bylevel == 1.0 &&
           params.colsample_bynode == 1.0,
       "row and column sampling (subsample / colsample_* below 1) are not implemented by this library");
  if (params.device >= 0) need(params.device == d->device(), "booster device differs from the matrix device");
  if (params.device < 0) params.device = d->device();
  const bool shape_changed = engine_ && (engine_->matrix() != d || engine_objective_ != params.objective ||
                                         engine_classes_ != K || engine_max_bin_ != params.max_bin);
  if (!engine_ || shape_changed) {
    need(model.trees.empty(),
         "continuing training on a different matrix, objective, num_class or max_bin is not supported");
    engine_.reset();
    engine_ = std::make_unique<Engine>(*d, params, comm);
    engine_objective_ = params.objective;
    engine_classes_ = K;
    engine_max_bin_ = params.max_bin;
    model.num_feature = int(d->cols());
  } else if (params_changed_) {
    engine_->update_params(params);
  }
  params_changed_ = false;
  engine_->profiler().enable(profiling);
  engine_->boost_round(model);
}

const std::string& Booster::save_model_json() {
  out_buf = model_to_json(model, params);
  return out_buf;
}

const std::string& Booster::save_config_json() {
  out_buf = config_to_json(model, params);
  return out_buf;
}

void Booster::load_model_json(const std::string& text) {
  Model m;
  TrainParams p = params;
  model_from_json(text, m, p);
  engine_.reset();
  model = std::move(m);
  params = p;
}

std::unique_ptr<Booster> Booster::slice(int begin, int end, int step) const {
  const int rounds = model.rounds();
  if (end == 0) end = rounds;
  need(begin >= 0 && begin <= end && end <= rounds && step >= 1, "invalid slice range");
  auto out = std::make_unique<Booster>();
  out->params = params;
  out->comm = comm;
  out->model.num_feature = model.num_feature;
  for (int r = begin; r < end; r += step) {
    for (int t = model.iteration_indptr[r]; t < model.iteration_indptr[r + 1]; ++t)
      out->model.trees.push_back(model.trees[t]);
    out->model.iteration_indptr.push_back(int(out->model.trees.size()));
  }
  return out;
}

}  // namespace dp
