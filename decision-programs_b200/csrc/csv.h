// CSV input transport on the GPU: the reference's host-side CSV -> dense
// fp32 / u32-label conversion (decision_programs_csv::read and ::decode,
// native/decision_programs_csv.hpp:10-67, called by the CLI at
// native/decision_programs_cli.cpp:140) as device kernels, with the same
// accepted inputs, the same values bit for bit and the same error messages.
#pragma once
#include <memory>
#include <string>

#include "common.h"

namespace dp {

struct CsvDense {
  u64 rows = 0;
  u32 features = 0;
  u32 classes = 0;
  bool header = false;
  bool has_target = false;
  DevBuf<float> values;  // [rows][features] on the device
  DevBuf<u32> labels;    // [rows] (empty without a target)
  std::string meta;      // {"names": [...], "label_mapping": [...] | null}
  double ms_device = 0;  // device time of the decode (events), for measurement
};

// bytes: the whole file in host memory; target: "" for none, a header name,
// "last" or a zero-based column index; header_mode: "auto", "yes" or "no".
// Throws std::invalid_argument with the reference's message on bad input.
std::unique_ptr<CsvDense> csv_decode(const char* bytes, u64 n, const std::string& target,
                                     const std::string& header_mode, cudaStream_t s);

// The host build of the decoder's per-field rule (the reference's feature(),
// native/decision_programs_csv.hpp:28-34): true with *value set when the
// token is accepted.  The same code runs on the device for every cell.
bool csv_parse_feature_host(const unsigned char* p, u32 n, float* value);

}  // namespace dp
