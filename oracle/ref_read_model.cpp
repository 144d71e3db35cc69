// Test infrastructure: runs the reference converter's model reader
// (dpnative::read_source, native/class_io.hpp:99-242, compiled unmodified from
// the reference sources) on one XGBoost-JSON model file and prints what it
// parsed as one JSON object, so tests can check that models written by
// libdp_gbdt are accepted with their thresholds and leaf values intact.
//   usage: ref_read_model <model.json>
// Exit status 0 and {"ok":true,...} on success; status 1 and
// {"ok":false,"error":...} when the reader rejects the file.
#include <cstdint>
#include <cstring>
#include <iostream>

#include "class_io.hpp"

namespace {

template <class T>
nlohmann::json bits_of(const std::vector<T>& v) {
  nlohmann::json a = nlohmann::json::array();
  for (const T& x : v) {
    uint32_t u = 0;
    std::memcpy(&u, &x, sizeof(u));
    a.push_back(u);
  }
  return a;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 2) {
    std::cerr << "usage: ref_read_model <model.json>\n";
    return 2;
  }
  try {
    const dpnative::SourceData s = dpnative::read_source(argv[1]);
    nlohmann::json out;
    out["ok"] = true;
    out["features"] = s.features;
    out["outputs"] = s.outputs;
    out["depth"] = s.depth;
    out["roots"] = s.roots;
    out["channels"] = s.channels;
    out["feature"] = s.feature;
    out["left"] = s.left;
    out["right"] = s.right;
    out["missing_left"] = s.missing_left;
    out["cut_bits"] = bits_of(s.cut);
    out["value_bits"] = bits_of(s.value);
    out["bias"] = s.bias;
    std::cout << out.dump() << "\n";
    return 0;
  } catch (const std::exception& e) {
    std::cout << nlohmann::json{{"ok", false}, {"error", e.what()}}.dump() << "\n";
    return 1;
  }
}
