// Test infrastructure: the reference converter's acceptance steps
// (native/class_model_convert.cpp, compiled unmodified from the reference
// sources and included here whole) run on a model written by libdp_gbdt.
//
//   usage: ref_convert_check shape <model.json>
//          ref_convert_check native <model.json> <library.so> <rows.f32> <rows>
//
// shape:  the converter's source_shape() (class_model_convert.cpp:49-60): the
//         gbtree / multi:softprob|softmax / decimal num_feature, num_class,
//         num_target / version 3.4.1 gate every source model must pass.
// native: source_shape(), then the converter's ResidentModel
//         (class_model_convert.cpp:93-164), which dlopens the native library,
//         checks its version and CUDA build, creates a booster, loads the model
//         from its buffer, sets device and threads, checks the feature count
//         and the JSON configuration against the source, and predicts the
//         given fp32 rows (copied to device 0) as margins and as the
//         objective's output.  Both predictions are printed as fp32 bits.
// Prints one JSON object; exit status 0 on success, 1 when the converter's
// code rejects the model or the library.  The converter's own main() is
// renamed and never run.  Built with DP_SHAPE_ONLY the harness has the shape
// mode alone and needs no CUDA driver (a CPU machine runs it).
#define main dp_reference_convert_main
#include "class_model_convert.cpp"
#undef main

#include <cstdint>
#include <cstring>
#include <fstream>
#include <vector>

namespace {

nlohmann::json bits(const std::vector<float>& v) {
  nlohmann::json a = nlohmann::json::array();
  for (float x : v) {
    std::uint32_t u = 0;
    std::memcpy(&u, &x, sizeof u);
    a.push_back(u);
  }
  return a;
}

#ifndef DP_SHAPE_ONLY
std::vector<float> predict_to_host(ResidentModel& m, const float* dev_rows, std::uint64_t rows, bool margin,
                                   std::uint64_t columns) {
  const float* out = m.predict(dev_rows, rows, margin);
  std::vector<float> host(rows * columns);
  cuda_check(cudaMemcpy(host.data(), out, host.size() * sizeof(float), cudaMemcpyDeviceToHost), "copy prediction");
  return host;
}
#endif

}  // namespace

int main(int argc, char** argv) {
  nlohmann::json out;
  try {
    require(argc >= 3, "usage: ref_convert_check shape|native <model.json> [library rows.f32 rows]");
    const std::string mode = argv[1];
    BoundFile model_file(argv[2]);
    const std::string model = model_file.bytes();
    SourceShape shape = source_shape(model);
    out["features"] = shape.features;
    out["classes"] = shape.classes;
    out["objective"] = shape.objective;
#ifndef DP_SHAPE_ONLY
    if (mode == "native") {
      require(argc == 6, "usage: ref_convert_check native <model.json> <library.so> <rows.f32> <rows>");
      const std::uint64_t rows = std::stoull(argv[5]);
      std::vector<float> x(rows * shape.features);
      std::ifstream in(argv[4], std::ios::binary);
      require(bool(in.read(reinterpret_cast<char*>(x.data()), std::streamsize(x.size() * sizeof(float)))),
              "short rows file");
      ResidentModel resident(argv[3], model, shape);
      float* d = nullptr;
      cuda_check(cudaMalloc(&d, x.size() * sizeof(float)), "cudaMalloc rows");
      cuda_check(cudaMemcpy(d, x.data(), x.size() * sizeof(float), cudaMemcpyHostToDevice), "copy rows");
      const std::uint64_t prob_cols = shape.objective == "multi:softprob" ? shape.classes : 1;
      out["margin_bits"] = bits(predict_to_host(resident, d, rows, true, shape.classes));
      out["output_bits"] = bits(predict_to_host(resident, d, rows, false, prob_cols));
      cudaFree(d);
    } else
#endif
    {
      require(mode == "shape", "mode must be shape or native");
    }
    out["ok"] = true;
    std::cout << out.dump() << "\n";
    return 0;
  } catch (const std::exception& e) {
    out["ok"] = false;
    out["error"] = e.what();
    std::cout << out.dump() << "\n";
    return 1;
  }
}
