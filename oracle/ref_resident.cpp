// Test harness, not product code: drives the reference's resident trainer
// (class_study::ResidentTrainer, native/class_study_train.cu, compiled
// unmodified beside this file) against a libdp_gbdt.so through its dlopen'd
// C ABI.  It exercises the model-lifecycle calls the trainer makes for
// hyper-parameter search and out-of-fold scoring (class_study_train.cu:98-106,
// 118-162, 324-369, 472-495): XGBoosterCreate/SetParam/UpdateOneIter,
// SaveJsonConfig, BoostedRounds, SaveModelToBuffer, Slice, LoadModelFromBuffer
// and PredictFromCudaArray with device output.
//
//   ref_resident <library.so> <sha256 of library> <dir>
//
// <dir>/meta.json: {"rows", "features", "classes", "rounds", "max_depth",
// "slice_rounds"}; <dir>/values.f32 [rows][features]; <dir>/labels.u32 [rows].
// Writes model.json, slice.json (the first slice_rounds rounds), classes.f32
// [rows], margins.f32 / probs.f32 [rows][classes], slice_margins.f32 and
// restored_margins.f32 (after restoring model.json), model2.json (a second
// trial on the same matrix: depth second_max_depth, eta 0.5, lambda 2),
// session.json.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <iterator>
#include <memory>
#include <string>
#include <vector>

#include "class_study_data.hpp"
#include "class_study_train.hpp"

namespace {

std::string slurp(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot read " + path);
  return std::string(std::istreambuf_iterator<char>(f), {});
}

void spill(const std::string& path, const void* p, size_t n) {
  std::ofstream f(path, std::ios::binary);
  f.write(static_cast<const char*>(p), std::streamsize(n));
  if (!f) throw std::runtime_error("cannot write " + path);
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Copies a borrowed device output [n] to host (it expires at the next call).
std::vector<float> take(const float* d, size_t n) {
  std::vector<float> h(n);
  check(cudaMemcpy(h.data(), d, n * sizeof(float), cudaMemcpyDeviceToHost), "copy prediction");
  return h;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 4) {
    std::cerr << "usage: ref_resident <library.so> <sha256> <dir>\n";
    return 2;
  }
  try {
    const std::string lib = argv[1], sha = argv[2], dir = argv[3];
    const auto meta = nlohmann::json::parse(slurp(dir + "/meta.json"));
    const std::uint64_t R = meta.at("rows");
    const std::uint32_t F = meta.at("features"), K = meta.at("classes");
    const auto values_h = slurp(dir + "/values.f32");
    const auto labels_h = slurp(dir + "/labels.u32");
    if (values_h.size() != R * F * 4 || labels_h.size() != R * 4) throw std::runtime_error("input sizes differ");

    check(cudaSetDevice(0), "device");
    float* values = nullptr;
    std::uint32_t* labels = nullptr;
    check(cudaMalloc(&values, values_h.size()), "values");
    check(cudaMalloc(&labels, labels_h.size()), "labels");
    check(cudaMemcpy(values, values_h.data(), values_h.size(), cudaMemcpyHostToDevice), "upload values");
    check(cudaMemcpy(labels, labels_h.data(), labels_h.size(), cudaMemcpyHostToDevice), "upload labels");

    const nlohmann::json plan = {{"TEST_read", false}, {"VALID_read", false}, {"native_library_path", lib},
                                 {"native_library_sha256", sha}};
    class_study::ResidentDataView view;
    view.values = values;
    view.labels = labels;
    view.rows = view.fit_rows = R;
    view.row_stride = F;
    view.valid_rows = 0;
    view.features = F;
    view.classes = K;
    view.binding = {{"source", "ref_resident harness"}, {"rows", R}, {"features", F}};
    view.owner = std::make_shared<int>(0);

    class_study::ResidentTrainer trainer(plan, view);
    const nlohmann::json hp = {{"rounds", meta.at("rounds")}, {"max_depth", meta.at("max_depth")}, {"eta", 0.3},
                               {"lambda", 1.0}, {"max_bin", 256}, {"seed", 0}};
    const auto trained = trainer.train(hp);
    spill(dir + "/model.json", trained.model_json.data(), trained.model_json.size());

    auto classes = take(trainer.predict(values, R, false), R);
    auto margins = take(trainer.predict(values, R, true), R * K);
    auto probs = take(trainer.predict_probabilities(values, R), R * K);
    spill(dir + "/classes.f32", classes.data(), classes.size() * 4);
    spill(dir + "/margins.f32", margins.data(), margins.size() * 4);
    spill(dir + "/probs.f32", probs.data(), probs.size() * 4);

    const auto sliced = trainer.slice_prefix(meta.at("slice_rounds").get<std::uint32_t>());
    spill(dir + "/slice.json", sliced.model_json.data(), sliced.model_json.size());
    auto slice_margins = take(trainer.predict(values, R, true), R * K);
    spill(dir + "/slice_margins.f32", slice_margins.data(), slice_margins.size() * 4);

    trainer.restore_model(trained.model_json, trained.model_sha256);
    auto restored = take(trainer.predict(values, R, true), R * K);
    spill(dir + "/restored_margins.f32", restored.data(), restored.size() * 4);

    // a second trial on the same resident matrix, as hyper-parameter search
    // and out-of-fold teachers do (class_study_train.cu:324-332)
    nlohmann::json hp2 = hp;
    hp2["max_depth"] = meta.value("second_max_depth", 3);
    hp2["eta"] = 0.5;
    hp2["lambda"] = 2.0;
    const auto second = trainer.train(hp2);
    spill(dir + "/model2.json", second.model_json.data(), second.model_json.size());

    nlohmann::json out = {{"session", trainer.metadata()}, {"train_metrics", trained.metrics},
                          {"slice_metrics", sliced.metrics}, {"second_metrics", second.metrics}};
    const auto s = out.dump();
    spill(dir + "/session.json", s.data(), s.size());
    cudaFree(values);
    cudaFree(labels);
  } catch (const std::exception& e) {
    std::cerr << "ref_resident: " << e.what() << "\n";
    return 1;
  }
  return 0;
}
