#include "booster.h"

#include <algorithm>

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
  ++model_version_;
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
  ++model_version_;
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

Booster::PredState::~PredState() {
  if (stream) {
    DeviceGuard g(device);
    cudaStreamSynchronize(stream);
    cudaStreamDestroy(stream);
  }
}

const float* Booster::predict(const PredictRequest& q, const u64** shape, u64* dims) {
  need(q.type == 0 || q.type == 1, "only prediction types 0 (value) and 1 (margin) are supported");
  const int rounds = model.rounds();
  const int it_end = q.it_end == 0 ? rounds : q.it_end;
  need(q.it_begin >= 0 && q.it_begin <= it_end && it_end <= rounds, "iteration range outside the model's rounds");
  need(q.rows == 0 || q.x != nullptr, "prediction input pointer is null");
  const int K = params.K();
  // outputs are [rows][K]: with no class the transform would read an empty margin buffer
  need(K >= 1, "num_class must be at least 1 to predict with a multi-class objective");
  DeviceGuard g(q.device);
  if (!pred_ || pred_->device != q.device) {
    pred_ = std::make_unique<PredState>();
    pred_->device = q.device;
    DP_CUDA(cudaStreamCreateWithFlags(&pred_->stream, cudaStreamNonBlocking));
  }
  PredState& st = *pred_;
  cudaStream_t s = st.stream;
  if (st.version != model_version_) {
    // flatten the ensemble, checking every child id and feature
    std::vector<PredNode> nodes;
    std::vector<u32> off{0}, cls;
    u32 max_feature = 0;
    for (const Tree& t : model.trees) {
      const size_t n = t.size();
      need(n >= 1 && n < (size_t(1) << 31), "empty or oversized tree");
      for (size_t i = 0; i < n; ++i) {
        PredNode nd{t.cond[i], t.left[i], t.right[i], 0u};
        if (t.left[i] >= 0) {
          need(size_t(t.left[i]) < n && t.right[i] >= 0 && size_t(t.right[i]) < n, "tree child index out of range");
          need(t.feature[i] >= 0, "negative split feature");
          nd.feat_dl = u32(t.feature[i]) | (t.default_left[i] ? 0x80000000u : 0u);
          max_feature = std::max<u32>(max_feature, u32(t.feature[i]) + 1);
        } else {
          nd.left = nd.right = -1;
        }
        nodes.push_back(nd);
      }
      need(t.klass >= 0 && t.klass < K, "tree class outside num_class");
      off.push_back(u32(nodes.size()));
      cls.push_back(u32(t.klass));
    }
    if (nodes.empty()) nodes.push_back(PredNode{0.f, -1, -1, 0u});
    if (cls.empty()) cls.push_back(0u);
    st.nodes.resize(nodes.size());
    st.tree_off.resize(off.size());
    st.tree_class.resize(cls.size());
    DP_CUDA(cudaMemcpy(st.nodes.get(), nodes.data(), nodes.size() * sizeof(PredNode), cudaMemcpyHostToDevice));
    DP_CUDA(cudaMemcpy(st.tree_off.get(), off.data(), off.size() * sizeof(u32), cudaMemcpyHostToDevice));
    DP_CUDA(cudaMemcpy(st.tree_class.get(), cls.data(), cls.size() * sizeof(u32), cudaMemcpyHostToDevice));
    st.max_feature = max_feature;
    st.version = model_version_;
  }
  need(model.num_feature <= 0 || q.cols == u64(model.num_feature),
       "the input's column count differs from the model's num_feature");
  need(st.max_feature <= q.cols, "the input has fewer features than the model splits on");
  std::vector<float> base(K);
  for (int k = 0; k < K; ++k) base[k] = params.base_margin(k);
  st.base.reserve(K);
  st.bad.reserve(1);
  DP_CUDA(cudaMemcpyAsync(st.base.get(), base.data(), K * sizeof(float), cudaMemcpyHostToDevice, s));
  DP_CUDA(cudaMemsetAsync(st.bad.get(), 0, sizeof(u32), s));
  const int width = q.type == 1 || params.objective_id() == kSoftprob ? K : 1;
  const u64 R = q.rows;
  st.margin.reserve(std::max<u64>(R, 1) * u64(K));
  const u32 t_begin = u32(model.iteration_indptr[q.it_begin]), t_end = u32(model.iteration_indptr[it_end]);
  launch_predict_margins(q.x, R, q.stride, q.has_mv, q.mv, st.nodes.get(), st.tree_off.get(), st.tree_class.get(),
                         t_begin, t_end, K, st.base.get(), st.margin.get(), st.bad.get(), s);
  const float* result = st.margin.get();
  if (q.type == 0) {
    st.out.reserve(std::max<u64>(R, 1) * u64(width));
    launch_predict_transform(params.objective_id(), K, st.margin.get(), R, st.out.get(), s);
    result = st.out.get();
  }
  u32 bad = 0;
  DP_CUDA(cudaMemcpyAsync(&bad, st.bad.get(), sizeof(u32), cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaStreamSynchronize(s));
  need(bad == 0, "malformed tree: a prediction walk did not reach a leaf");
  if (q.strict_shape || width > 1) st.shape = {R, u64(width)};
  else st.shape = {R};
  *shape = st.shape.data();
  *dims = st.shape.size();
  return result;
}

}  // namespace dp
