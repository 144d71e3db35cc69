// Test harness, not product code: runs the reference's CSV input transport
// (decision_programs_csv::decode, native/decision_programs_csv.hpp:36-67,
// compiled unmodified from its header) on a file, for the parity tests of the
// GPU CSV decoder and as the CPU baseline of its benchmark.
//
//   ref_csv <input.csv> <target or -> <header mode> <out dir> [repeats]
//   ref_csv --tokens <tokens file> <out file>
//
// The second form runs the reference's feature() on each line of the tokens
// file (lines end in '\n'; the token is the line's bytes) and writes one
// line per token: "1 <hex bits of the float>" when accepted, "0" otherwise.
//
// Writes <out>/values.f32, <out>/labels.u32 and <out>/meta.json (rows,
// features, classes, header, names, label_mapping, seconds per decode), or
// <out>/error.txt with the exception's message.  A target of "-" decodes
// without one.
#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <iterator>

#include "decision_programs_csv.hpp"

int main(int argc, char** argv) {
  if (argc == 4 && std::string(argv[1]) == "--tokens") {
    std::ifstream in(argv[2], std::ios::binary);
    std::ofstream out(argv[3]);
    std::string line;
    char buf[16];
    while (std::getline(in, line)) {
      float v = 0.0f;
      if (decision_programs_csv::feature(line, v)) {
        unsigned bits;
        std::memcpy(&bits, &v, 4);
        std::snprintf(buf, sizeof buf, "%08x", bits);
        out << "1 " << buf << "\n";
      } else {
        out << "0\n";
      }
    }
    return 0;
  }
  if (argc < 5) {
    std::cerr << "usage: ref_csv <input.csv> <target|-> <header> <out dir> [repeats]\n";
    return 2;
  }
  const std::string dir = argv[4];
  const int repeats = argc > 5 ? std::atoi(argv[5]) : 1;
  std::ifstream in(argv[1], std::ios::binary);
  const std::string bytes((std::istreambuf_iterator<char>(in)), {});
  const std::string target = std::string(argv[2]) == "-" ? std::string() : std::string(argv[2]);
  try {
    decision_programs_csv::Dense d;
    double best = 1e30;
    for (int r = 0; r < repeats; ++r) {
      const auto t0 = std::chrono::steady_clock::now();
      d = decision_programs_csv::decode(bytes, target, argv[3]);
      best = std::min(best, std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
    }
    std::ofstream(dir + "/values.f32", std::ios::binary).write(d.values.data(), std::streamsize(d.values.size()));
    std::ofstream(dir + "/labels.u32", std::ios::binary).write(d.labels.data(), std::streamsize(d.labels.size()));
    nlohmann::json meta = {{"rows", d.rows}, {"features", d.features}, {"classes", d.classes}, {"header", d.header},
                           {"names", d.names}, {"label_mapping", d.label_mapping}, {"seconds", best},
                           {"bytes", bytes.size()}};
    std::ofstream(dir + "/meta.json") << meta.dump();
  } catch (const std::exception& e) {
    std::ofstream(dir + "/error.txt") << e.what();
  }
  return 0;
}
