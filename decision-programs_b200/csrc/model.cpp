// Parameter parsing (XGBoosterSetParam) and the JSON model / configuration
// documents (XGBoosterSaveModel, XGBoosterSaveModelToBuffer,
// XGBoosterSaveJsonConfig, XGBoosterLoadModelFromBuffer).
//
// The documents follow the XGBoost 3.4.1 JSON schema that the reference's
// callers check and read: version [3,4,1] (native/class_io.hpp:140-141),
// learner.objective.name and learner_model_param.{num_feature,num_class} as
// decimal strings (native/class_model_train.cu:50-51,
// native/class_study_train.cu:84-90), gbtree trees with consecutive numeric
// successors (native/class_native_source_contract.hpp:26-33), and the
// configuration keys learner.generic_param.device and
// learner.gradient_booster.updater[0].name (native/class_model_train.cu:48).
#include <algorithm>
#include <charconv>
#include <cmath>
#include <cstdio>
#include <exception>
#include <string>
#include <system_error>
#include <thread>
#include <vector>

#include "json.h"
#include "model.h"

namespace dp {

namespace {

std::string unquote(const std::string& v) {
  if (v.size() >= 2 && v.front() == '"' && v.back() == '"') return v.substr(1, v.size() - 2);
  return v;
}

double to_double(const std::string& key, const std::string& v) {
  const std::string s = unquote(v);
  char* end = nullptr;
  const double d = strtod_c(s.c_str(), &end);
  need(!s.empty() && end == s.c_str() + s.size(),
       "invalid numeric value for parameter " + printable(key) + ": " + printable(v));
  return d;
}

long long to_int(const std::string& key, const std::string& v) {
  const double d = to_double(key, v);
  need(std::isfinite(d) && d == std::floor(d) && std::fabs(d) < 9.0e15,
       "parameter " + printable(key) + " must be an integer: " + printable(v));
  return static_cast<long long>(d);
}

void range(const std::string& key, double v, double lo, double hi, bool strict_lo = false) {
  need(std::isfinite(v) && (strict_lo ? v > lo : v >= lo) && v <= hi,
       "parameter " + printable(key) + " is outside its supported range");
}

}  // namespace

int TrainParams::objective_id() const {
  if (objective == "reg:squarederror") return kSquaredError;
  if (objective == "binary:logistic") return kLogistic;
  if (objective == "multi:softprob") return kSoftprob;
  if (objective == "multi:softmax") return kSoftmax;
  fail("unsupported objective: " + printable(objective));
}

float TrainParams::base_margin(int k) const {
  const int oid = objective_id();
  double bs = oid == kLogistic ? 0.5 : 0.0;
  need(base_score.size() <= 1 || size_t(k) < base_score.size(), "base_score must have one value or one per class");
  if (!base_score.empty()) bs = base_score.size() == 1 ? base_score[0] : base_score[size_t(k)];
  if (oid == kLogistic) {
    need(bs > 0.0 && bs < 1.0, "base_score must be in (0,1) for logistic loss");
    return float(std::log(bs / (1.0 - bs)));
  }
  return float(bs);
}

void TrainParams::set(const std::string& key, const std::string& value) {
  const std::string v = unquote(value);
  if (key == "objective") {
    need(v == "reg:squarederror" || v == "binary:logistic" || v == "multi:softprob" || v == "multi:softmax",
         "unsupported objective: " + printable(v));
    objective = v;
  } else if (key == "num_class") {
    const long long n = to_int(key, v);
    need(n >= 0 && n <= (1 << 24), "num_class is outside its supported range");
    num_class = int(n);
  } else if (key == "max_depth") {
    const long long n = to_int(key, v);
    need(n >= 1 && n <= 30, "max_depth must be in [1, 30]");
    max_depth = int(n);
  } else if (key == "max_bin") {
    const long long n = to_int(key, v);
    need(n >= 2, "max_bin must be at least 2");
    max_bin = int(std::min<long long>(n, 256));
  } else if (key == "eta" || key == "learning_rate") {
    eta = to_double(key, v);
    range(key, eta, 0.0, 1e300);
  } else if (key == "lambda" || key == "reg_lambda") {
    lambda = to_double(key, v);
    range(key, lambda, 0.0, 1e300);
  } else if (key == "alpha" || key == "reg_alpha") {
    alpha = to_double(key, v);
    range(key, alpha, 0.0, 1e300);
  } else if (key == "gamma" || key == "min_split_loss") {
    gamma = to_double(key, v);
    range(key, gamma, 0.0, 1e300);
  } else if (key == "min_child_weight") {
    min_child_weight = to_double(key, v);
    range(key, min_child_weight, 0.0, 1e300);
  } else if (key == "subsample" || key == "colsample_bytree" || key == "colsample_bylevel" ||
             key == "colsample_bynode") {
    const double d = to_double(key, v);
    range(key, d, 0.0, 1.0, true);
    (key == "subsample" ? subsample
     : key == "colsample_bytree" ? colsample_bytree
     : key == "colsample_bylevel" ? colsample_bylevel
                                  : colsample_bynode) = d;
  } else if (key == "base_score") {
    base_score.clear();
    if (!v.empty() && v.front() == '[') {
      const json::Value a = json::parse(v);
      for (const auto& x : a.items()) base_score.push_back(float(x.as_double()));
    } else {
      base_score.push_back(float(to_double(key, v)));
    }
  } else if (key == "seed" || key == "random_state") {
    seed = to_int(key, v);
  } else if (key == "device") {
    if (v == "cuda" || v == "gpu") {
      device = -1;
    } else if (v.rfind("cuda:", 0) == 0 || v.rfind("gpu:", 0) == 0) {
      device = int(to_int(key, v.substr(v.find(':') + 1)));
      need(device >= 0, "invalid device ordinal");
    } else {
      fail("device must be a CUDA device (\"cuda\" or \"cuda:N\"); this library has no CPU training path");
    }
  } else if (key == "tree_method") {
    need(v == "hist" || v == "auto" || v == "gpu_hist", "tree_method must be hist");
  } else if (key == "booster") {
    need(v == "gbtree", "booster must be gbtree");
  } else if (key == "grow_policy") {
    need(v == "depthwise", "grow_policy must be depthwise");
  } else if (key == "max_delta_step") {
    need(to_double(key, v) == 0.0, "max_delta_step must be 0");
  } else if (key == "scale_pos_weight") {
    need(to_double(key, v) == 1.0, "scale_pos_weight must be 1");
  } else if (key == "num_parallel_tree") {
    need(to_int(key, v) == 1, "num_parallel_tree must be 1");
  } else if (key == "max_leaves") {
    need(to_int(key, v) == 0, "max_leaves must be 0");
  }
  // Every other key (nthread, verbosity, validate_parameters, seed_per_iteration,
  // boost_from_average, eval_metric, ...) is recorded and has no effect here.
  raw[key] = v;
}

// ------------------------------------------------------------------ writer
namespace {

// [v0,v1,...], each element appended by app(o, v[i]) without a temporary
// string: a model of depth-10 trees has millions of numbers.
template <class T, class App>
void put_array(std::string& o, const std::vector<T>& v, App app) {
  o.push_back('[');
  for (size_t i = 0; i < v.size(); ++i) {
    if (i) o.push_back(',');
    app(o, v[i]);
  }
  o.push_back(']');
}

std::string istr(long long v) { return std::to_string(v); }

std::string objective_json(const TrainParams& p) {
  std::string o = "{\"name\":" + json::quote(p.objective);
  if (p.objective.rfind("multi:", 0) == 0)
    o += ",\"softmax_multiclass_param\":{\"num_class\":\"" + istr(p.num_class) + "\"}";
  else
    o += ",\"reg_loss_param\":{\"scale_pos_weight\":\"1\"}";
  return o + "}";
}

std::string base_score_string(const TrainParams& p) {
  const int K = p.K();
  need(p.base_score.size() <= 1 || p.base_score.size() == size_t(std::max(1, K)),
       "base_score must have one value or one per class");
  std::string s = "[";
  for (int k = 0; k < K; ++k) {
    if (k) s += ",";
    double bs = p.objective_id() == kLogistic ? 0.5 : 0.0;
    if (!p.base_score.empty()) bs = p.base_score.size() == 1 ? p.base_score[0] : p.base_score[size_t(k)];
    s += json::format_float(float(bs));
  }
  return s + "]";
}

std::string learner_model_param(const Model& m, const TrainParams& p) {
  const bool multi = p.objective.rfind("multi:", 0) == 0;
  return "{\"base_score\":" + json::quote(base_score_string(p)) + ",\"boost_from_average\":\"0\"" +
         ",\"num_class\":\"" + istr(multi ? p.num_class : 0) + "\",\"num_feature\":\"" + istr(m.num_feature) +
         "\",\"num_target\":\"1\"}";
}

// One tree's JSON object, preceded by a comma unless it is tree 0.
void put_tree(std::string& o, const Tree& t, size_t i, int num_feature) {
  auto f = [](std::string& s, float v) { json::append_float(s, v); };
  auto n = [](std::string& s, i32 v) { json::append_int(s, v); };
  if (i) o += ",";
  o += "{\"base_weights\":";
  put_array(o, t.base_weight, f);
  o += ",\"categories\":[],\"categories_nodes\":[],\"categories_segments\":[],\"categories_sizes\":[]";
  o += ",\"default_left\":";
  put_array(o, t.default_left, [](std::string& s, u8 v) { s.push_back(v ? '1' : '0'); });
  o += ",\"id\":";
  json::append_int(o, long(i));
  o += ",\"left_children\":";
  put_array(o, t.left, n);
  o += ",\"loss_changes\":";
  put_array(o, t.loss_change, f);
  o += ",\"parents\":";
  put_array(o, t.parent, [](std::string& s, i32 v) { json::append_int(s, v < 0 ? 2147483647 : v); });
  o += ",\"right_children\":";
  put_array(o, t.right, n);
  o += ",\"split_conditions\":";
  put_array(o, t.cond, f);
  o += ",\"split_indices\":";
  put_array(o, t.feature, n);
  o += ",\"split_type\":";
  put_array(o, t.left, [](std::string& s, i32) { s.push_back('0'); });
  o += ",\"sum_hessian\":";
  put_array(o, t.sum_hess, f);
  o += ",\"tree_param\":{\"num_deleted\":\"0\",\"num_feature\":\"" + istr(num_feature) + "\",\"num_nodes\":\"" +
       istr(long(t.size())) + "\",\"size_leaf_vector\":\"1\"}}";
}

}  // namespace

std::string model_to_json(const Model& m, const TrainParams& p) {
  std::string o;
  size_t nodes = 0;
  for (const auto& t : m.trees) nodes += t.size();
  o.reserve(4096 + nodes * 96);
  o += "{\"learner\":{\"attributes\":{},\"feature_names\":[],\"feature_types\":[],";
  o += "\"gradient_booster\":{\"model\":{\"gbtree_model_param\":{\"num_parallel_tree\":\"1\",\"num_trees\":\"" +
       istr(long(m.trees.size())) + "\"},";
  o += "\"iteration_indptr\":";
  put_array(o, m.iteration_indptr, [](std::string& s, int v) { json::append_int(s, v); });
  o += ",\"tree_info\":[";
  for (size_t i = 0; i < m.trees.size(); ++i) {
    if (i) o += ",";
    o += istr(m.trees[i].klass);
  }
  o += "],\"trees\":[";
  // Trees are formatted in parallel chunks and joined in order (the text is
  // the same as one pass): a depth-10 model has ~2k nodes per tree and its
  // serialisation is part of every saved model's latency.
  const size_t T = m.trees.size();
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const size_t parts = nodes >= 20000 ? std::min<size_t>({T, size_t(8), size_t(hw)}) : 1;
  if (parts <= 1) {
    for (size_t i = 0; i < T; ++i) put_tree(o, m.trees[i], i, m.num_feature);
  } else {
    std::vector<std::string> chunk(parts);
    std::vector<std::exception_ptr> err(parts);
    auto format_chunk = [&](size_t q) {
      try {
        const size_t b = T * q / parts, e = T * (q + 1) / parts;
        size_t n = 0;
        for (size_t i = b; i < e; ++i) n += m.trees[i].size();
        chunk[q].reserve(1024 + n * 96);
        for (size_t i = b; i < e; ++i) put_tree(chunk[q], m.trees[i], i, m.num_feature);
      } catch (...) {
        err[q] = std::current_exception();
      }
    };
    std::vector<std::thread> pool;
    pool.reserve(parts);  // so that only the thread start itself can throw below
    size_t started = 0;
    try {
      for (; started < parts; ++started) pool.emplace_back(format_chunk, started);
    } catch (const std::system_error&) {
      // no more threads: the calling thread formats the chunks not started
    }
    for (size_t q = started; q < parts; ++q) format_chunk(q);
    for (auto& th : pool) th.join();
    for (auto& e : err)
      if (e) std::rethrow_exception(e);
    for (auto& c : chunk) o += c;
  }
  o += "]},\"name\":\"gbtree\"},";
  o += "\"learner_model_param\":" + learner_model_param(m, p) + ",";
  o += "\"objective\":" + objective_json(p) + "},";
  o += "\"version\":[3,4,1]}";
  return o;
}

std::string config_to_json(const Model& m, const TrainParams& p) {
  auto d = [](double v) { return json::quote(json::format_double(v)); };
  const std::string device = "cuda:" + std::to_string(p.device < 0 ? 0 : p.device);
  std::string train_param = "{\"alpha\":" + d(p.alpha) + ",\"colsample_bylevel\":" + d(p.colsample_bylevel) +
                            ",\"colsample_bynode\":" + d(p.colsample_bynode) + ",\"colsample_bytree\":" +
                            d(p.colsample_bytree) + ",\"eta\":" + d(p.eta) + ",\"gamma\":" + d(p.gamma) +
                            ",\"grow_policy\":\"depthwise\",\"lambda\":" + d(p.lambda) +
                            ",\"max_delta_step\":\"0\",\"max_depth\":\"" + istr(p.max_depth) +
                            "\",\"max_leaves\":\"0\",\"min_child_weight\":" + d(p.min_child_weight) +
                            ",\"subsample\":" + d(p.subsample) + "}";
  std::string o = "{\"learner\":{";
  o += "\"generic_param\":{\"device\":" + json::quote(device) +
       ",\"fail_on_invalid_gpu_id\":\"0\",\"nthread\":\"0\",\"random_state\":\"" + istr(p.seed) +
       "\",\"seed\":\"" + istr(p.seed) + "\",\"seed_per_iteration\":\"0\",\"validate_parameters\":\"1\"},";
  o += "\"gradient_booster\":{\"gbtree_model_param\":{\"num_parallel_tree\":\"1\",\"num_trees\":\"" +
       istr(long(m.trees.size())) + "\"},\"gbtree_train_param\":{\"process_type\":\"default\",\"tree_method\":\"hist\"," +
       "\"updater\":\"grow_gpu_hist\",\"updater_seq\":\"grow_gpu_hist\"},\"name\":\"gbtree\"," +
       "\"specified_updater\":false,\"updater\":[{\"hist_train_param\":{\"debug_synchronize\":\"0\",\"max_bin\":\"" +
       istr(p.max_bin) + "\"},\"name\":\"grow_gpu_hist\",\"train_param\":" + train_param + "}]},";
  o += "\"learner_model_param\":" + learner_model_param(m, p) + ",";
  o += "\"learner_train_param\":{\"booster\":\"gbtree\",\"disable_default_eval_metric\":\"0\"," +
       std::string("\"multi_strategy\":\"one_output_per_tree\",\"objective\":") + json::quote(p.objective) + "},";
  o += "\"metrics\":[],\"objective\":" + objective_json(p) + "},";
  o += "\"version\":[3,4,1],";
  // Identifies this implementation so receipts cannot be mistaken for XGBoost.
  o += "\"dp_b200_gbdt\":{\"engine\":\"libdp_gbdt sm_100a\",\"quantiser\":{\"grad_bits\":" + istr(kGradBits) +
       ",\"hess_bits\":" + istr(kHessBits) + ",\"window_rows\":" + istr(kWindowRows) + "}}}";
  return o;
}

// ------------------------------------------------------------------ reader
void model_from_json(const std::string& text, Model& m, TrainParams& p) {
  const json::Value doc = json::parse(text);
  const auto& version = doc.at("version");
  need(version.is_array() && version.size() == 3, "model version must be an array of three integers");
  const auto& learner = doc.at("learner");
  const auto& gb = learner.at("gradient_booster");
  need(gb.at("name").as_string() == "gbtree", "only gbtree models are supported");
  const auto& lmp = learner.at("learner_model_param");
  // counts are decimal strings in XGBoost's files (plain numbers are read
  // too); the whole string must be the integer
  auto dec = [](const json::Value& v) -> long long {
    if (!v.is_string()) return v.as_int();
    const std::string& t = v.as_string();
    long long x = 0;
    const auto r = std::from_chars(t.data(), t.data() + t.size(), x);
    if (t.empty() || r.ec != std::errc{} || r.ptr != t.data() + t.size())
      fail("invalid integer in learner_model_param: " + printable(t));
    return x;
  };
  Model out;
  const long long num_feature = dec(lmp.at("num_feature"));
  need(num_feature >= 0 && num_feature <= 0x7fffffffLL, "num_feature is outside its supported range");
  out.num_feature = int(num_feature);
  TrainParams q = p;
  q.objective = learner.at("objective").at("name").as_string();
  (void)q.objective_id();
  const long long num_class = dec(lmp.at("num_class"));
  need(num_class >= 0 && num_class <= (1 << 24), "num_class is outside its supported range");
  q.num_class = int(num_class);
  if (const auto* bs = lmp.find("base_score")) {
    json::Value b = bs->is_string() ? json::parse(bs->as_string()) : *bs;
    q.base_score.clear();
    if (b.is_array())
      for (const auto& x : b.items()) q.base_score.push_back(float(x.as_double()));
    else
      q.base_score.push_back(float(b.as_double()));
    need(q.base_score.size() <= 1 || q.base_score.size() == size_t(std::max(1, q.K())),
         "base_score must have one value or one per class");
  }
  const auto& model = gb.at("model");
  const auto& trees = model.at("trees");
  const auto& info = model.at("tree_info");
  need(trees.size() == info.size(), "tree_info size differs from the number of trees");
  for (size_t i = 0; i < trees.size(); ++i) {
    const auto& tj = trees[i];
    Tree t;
    const long long klass = info[i].as_int();
    need(klass >= 0 && klass < std::max(1, q.K()), "tree_info names a class outside num_class");
    t.klass = int(klass);
    auto ints = [&](const char* k) {
      std::vector<i32> v;
      for (const auto& x : tj.at(k).items()) v.push_back(i32(x.as_int()));
      return v;
    };
    auto floats = [&](const char* k) {
      std::vector<float> v;
      for (const auto& x : tj.at(k).items()) v.push_back(float(x.as_double()));
      return v;
    };
    t.left = ints("left_children");
    t.right = ints("right_children");
    t.feature = ints("split_indices");
    t.cond = floats("split_conditions");
    const size_t nn = t.left.size();
    need(t.right.size() == nn && t.feature.size() == nn && t.cond.size() == nn, "tree node arrays differ in size");
    for (const auto& x : tj.at("default_left").items()) t.default_left.push_back(u8(x.as_bool()));
    need(t.default_left.size() == nn, "tree node arrays differ in size");
    if (const auto* st = tj.find("split_type"))
      for (const auto& x : st->items()) need(x.as_int() == 0, "categorical splits are not supported");
    t.parent.assign(nn, -1);
    for (size_t j = 0; j < nn; ++j) {
      if (t.left[j] >= 0) {
        need(size_t(t.left[j]) < nn && size_t(t.right[j]) < nn, "tree child index out of range");
        t.parent[t.left[j]] = i32(j);
        t.parent[t.right[j]] = i32(j);
      }
    }
    t.base_weight = tj.contains("base_weights") ? floats("base_weights") : std::vector<float>(nn, 0.f);
    t.loss_change = tj.contains("loss_changes") ? floats("loss_changes") : std::vector<float>(nn, 0.f);
    t.sum_hess = tj.contains("sum_hessian") ? floats("sum_hessian") : std::vector<float>(nn, 0.f);
    if (t.base_weight.size() != nn) t.base_weight.assign(nn, 0.f);
    if (t.loss_change.size() != nn) t.loss_change.assign(nn, 0.f);
    if (t.sum_hess.size() != nn) t.sum_hess.assign(nn, 0.f);
    out.trees.push_back(std::move(t));
  }
  out.iteration_indptr.clear();
  if (const auto* ip = model.find("iteration_indptr")) {
    for (const auto& x : ip->items()) out.iteration_indptr.push_back(int(x.as_int()));
  } else {
    const int K = std::max(1, q.K());
    for (size_t i = 0; i <= trees.size(); i += size_t(K)) out.iteration_indptr.push_back(int(i));
  }
  need(!out.iteration_indptr.empty() && out.iteration_indptr.front() == 0 &&
           size_t(out.iteration_indptr.back()) == out.trees.size(),
       "iteration_indptr does not cover the stored trees");
  // every round's trees are [indptr[r], indptr[r + 1]) of the stored trees:
  // slicing and prediction index the trees and their device layout with them
  for (size_t r = 1; r < out.iteration_indptr.size(); ++r)
    need(out.iteration_indptr[r] >= out.iteration_indptr[r - 1] &&
             size_t(out.iteration_indptr[r]) <= out.trees.size(),
         "iteration_indptr must be non-decreasing and within the stored trees");
  m = std::move(out);
  p = q;
}

}  // namespace dp
