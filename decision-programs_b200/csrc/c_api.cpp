// extern "C" entry points of libdp_gbdt (declared in include/dp_gbdt.h).
#include "../../include/dp_gbdt.h"

#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "booster.h"
#include "csv.h"
#include "comm.h"
#include "dmatrix.h"
#include "json.h"
#include "kernels.h"
#include "quantile.h"

namespace {

thread_local std::string g_last_error;

#define DP_API_BEGIN() try {
#define DP_API_END()                         \
  }                                          \
  catch (const std::exception& e) {          \
    g_last_error = e.what();                 \
    return -1;                               \
  }                                          \
  catch (...) {                              \
    g_last_error = "unknown error";          \
    return -1;                               \
  }                                          \
  return 0;

using dp::need;

struct ArrayInterface {
  std::uintptr_t ptr = 0;
  std::vector<dp::u64> shape;
  std::vector<dp::i64> strides;  // bytes; empty = C-contiguous
  std::string typestr;
};

ArrayInterface parse_array(const char* text) {
  need(text != nullptr, "array interface string is null");
  dp::json::Value v = dp::json::parse(text);
  if (v.is_array()) {
    need(v.size() == 1, "only one array interface (one column batch) is supported");
    v = dp::json::Value(v[0]);
  }
  need(v.is_object(), "array interface must be a JSON object");
  ArrayInterface a;
  const auto& data = v.at("data");
  need(data.is_array() && data.size() >= 1, "array interface data must be [pointer, read_only]");
  a.ptr = std::uintptr_t(data[0].as_uint());
  for (const auto& s : v.at("shape").items()) a.shape.push_back(s.as_uint());
  if (const auto* st = v.find("strides"))
    if (!st->is_null())
      for (const auto& s : st->items()) a.strides.push_back(s.as_int());
  a.typestr = v.at("typestr").as_string();
  if (const auto* m = v.find("mask")) need(m->is_null(), "masked arrays are not supported");
  return a;
}

int pointer_device(const void* p, bool allow_host) {
  cudaPointerAttributes attr{};
  dp::cuda_check(cudaPointerGetAttributes(&attr, p), "cudaPointerGetAttributes");
  if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) return attr.device;
  need(allow_host, "array memory must be CUDA device memory");
  int dev = 0;
  dp::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  return dev;
}

dp::DMatrix* as_dmatrix(void* h) {
  need(h != nullptr, "DMatrix handle is null");
  return static_cast<dp::DMatrix*>(h);
}
dp::Booster* as_booster(void* h) {
  need(h != nullptr, "Booster handle is null");
  return static_cast<dp::Booster*>(h);
}

std::string read_file(const char* path) {
  std::ifstream f(path, std::ios::binary);
  need(bool(f), "cannot read " + dp::printable(path));
  std::ostringstream s;
  s << f.rdbuf();
  return s.str();
}

bool ends_with(const std::string& s, const std::string& suf) {
  return s.size() >= suf.size() && s.compare(s.size() - suf.size(), suf.size(), suf) == 0;
}

}  // namespace

namespace dp {
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace dp

extern "C" {

void XGBoostVersion(int* major, int* minor, int* patch) {
  if (major) *major = 3;
  if (minor) *minor = 4;
  if (patch) *patch = 1;
}

int XGBuildInfo(const char** out) {
  static const char* info =
      "{\"USE_CUDA\":true,\"USE_NCCL\":true,\"USE_OPENMP\":false,\"CUDA_VERSION\":[12,9],"
      "\"GPU_ARCH\":\"sm_100a\",\"DP_B200_GBDT\":true}";
  if (out) *out = info;
  return 0;
}

const char* XGBGetLastError(void) { return g_last_error.c_str(); }

namespace {
// Shape, row stride (elements) and missing value of a dense fp32 matrix
// described by an array interface and an XGBoost DMatrix config.
struct DenseSpec {
  dp::u64 rows = 0, cols = 0, stride = 0;
  bool has_mv = false;
  float mv = 0.f;
  const float* ptr = nullptr;
};

DenseSpec dense_spec(const char* data, const char* config) {
  const ArrayInterface a = parse_array(data);
  need(a.typestr == "<f4", "only little-endian float32 (<f4) matrices are supported");
  need(a.shape.size() == 2, "matrix array interface must be two-dimensional");
  DenseSpec d;
  d.rows = a.shape[0];
  d.cols = a.shape[1];
  need(d.cols > 0 && d.cols <= 0x7fffffffULL, "matrix column count out of range");
  d.stride = d.cols;
  if (!a.strides.empty()) {
    need(a.strides.size() == 2 && a.strides[1] == 4 && a.strides[0] > 0 && a.strides[0] % 4 == 0,
         "matrix strides must be row-major with 4-byte elements");
    d.stride = dp::u64(a.strides[0]) / 4;
  }
  if (config && *config) {
    const dp::json::Value c = dp::json::parse(config);
    if (const auto* m = c.find("missing")) {
      const double v = m->as_double();
      if (!std::isnan(v)) { d.has_mv = true; d.mv = float(v); }
    }
  }
  need(d.rows == 0 || a.ptr != 0, "matrix data pointer is null");
  // every kernel addresses rows * stride elements with 64-bit byte offsets
  need(d.stride <= (dp::u64(1) << 40), "matrix row stride out of range");
  need(d.rows <= (dp::u64(1) << 62) / 4 / d.stride, "matrix size overflows 64-bit byte offsets");
  d.ptr = reinterpret_cast<const float*>(a.ptr);
  return d;
}
}  // namespace

int XGDMatrixCreateFromCudaArrayInterface(const char* data, const char* config, DMatrixHandle* out) {
  DP_API_BEGIN();
  need(out != nullptr, "output handle pointer is null");
  const DenseSpec m = dense_spec(data, config);
  const int dev = m.rows ? pointer_device(m.ptr, false) : 0;
  {
    dp::DeviceGuard g(dev);
    // the producer may still be writing on its own stream
    dp::cuda_check(cudaDeviceSynchronize(), "synchronise producer");
  }
  auto d = std::make_unique<dp::DMatrix>(m.ptr, m.rows, dp::u32(m.cols), m.stride, dev, m.has_mv, m.mv);
  *out = d.release();
  DP_API_END();
}

int XGDMatrixCreateFromDense(const char* data, const char* config, DMatrixHandle* out) {
  DP_API_BEGIN();
  need(out != nullptr, "output handle pointer is null");
  const DenseSpec m = dense_spec(data, config);
  int dev = 0;
  dp::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (m.rows) {
    cudaPointerAttributes attr{};
    dp::cuda_check(cudaPointerGetAttributes(&attr, m.ptr), "cudaPointerGetAttributes");
    need(attr.type == cudaMemoryTypeHost || attr.type == cudaMemoryTypeUnregistered,
         "XGDMatrixCreateFromDense takes host memory; use XGDMatrixCreateFromCudaArrayInterface for device memory");
  }
  auto d = dp::DMatrix::from_host(m.ptr, m.rows, dp::u32(m.cols), m.stride, dev, m.has_mv, m.mv);
  *out = d.release();
  DP_API_END();
}

int XGDMatrixSetInfoFromInterface(DMatrixHandle handle, const char* field, const char* data) {
  DP_API_BEGIN();
  need(field != nullptr && std::string(field) == "label", "only the \"label\" field is supported");
  const ArrayInterface a = parse_array(data);
  need(a.typestr == "<f4", "labels must be little-endian float32 (<f4)");
  need(a.shape.size() == 1 || (a.shape.size() == 2 && a.shape[1] == 1), "labels must be a vector");
  // consecutive labels 4 bytes apart: for an [n, 1] array that is the stride
  // between rows (a column of a wider matrix is refused, not read wrongly)
  need(a.strides.empty() || (a.strides.size() == a.shape.size() && (a.shape[0] <= 1 || a.strides[0] == 4)),
       "labels must be contiguous");
  need(a.shape[0] == 0 || a.ptr != 0, "label pointer is null");
  dp::DMatrix* d = as_dmatrix(handle);
  {
    dp::DeviceGuard g(d->device());
    dp::cuda_check(cudaDeviceSynchronize(), "synchronise producer");
  }
  d->set_labels_device(reinterpret_cast<const float*>(a.ptr), a.shape[0]);
  DP_API_END();
}

int XGDMatrixSetFloatInfo(DMatrixHandle handle, const char* field, const float* data, bst_ulong len) {
  DP_API_BEGIN();
  dp::DMatrix* d = as_dmatrix(handle);
  need(field != nullptr && std::string(field) == "label", "only the \"label\" field is supported");
  need(len == 0 || data != nullptr, "label pointer is null");
  d->set_labels_host(data, len);
  DP_API_END();
}

int XGDMatrixNumRow(DMatrixHandle handle, bst_ulong* out) {
  DP_API_BEGIN();
  need(out != nullptr, "output pointer is null");
  *out = as_dmatrix(handle)->rows();
  DP_API_END();
}

int XGDMatrixNumCol(DMatrixHandle handle, bst_ulong* out) {
  DP_API_BEGIN();
  need(out != nullptr, "output pointer is null");
  *out = as_dmatrix(handle)->cols();
  DP_API_END();
}

int XGDMatrixFree(DMatrixHandle handle) {
  DP_API_BEGIN();
  delete static_cast<dp::DMatrix*>(handle);
  DP_API_END();
}

int XGBoosterCreate(const DMatrixHandle dmats[], bst_ulong len, BoosterHandle* out) {
  DP_API_BEGIN();
  need(out != nullptr, "output handle pointer is null");
  need(len == 0 || dmats != nullptr, "matrix list is null");
  for (bst_ulong i = 0; i < len; ++i) need(dmats[i] != nullptr, "matrix handle is null");
  *out = new dp::Booster();
  DP_API_END();
}

int XGBoosterFree(BoosterHandle handle) {
  DP_API_BEGIN();
  delete static_cast<dp::Booster*>(handle);
  DP_API_END();
}

int XGBoosterSetParam(BoosterHandle handle, const char* name, const char* value) {
  DP_API_BEGIN();
  need(name != nullptr && value != nullptr, "parameter name / value is null");
  as_booster(handle)->set_param(name, value);
  DP_API_END();
}

int XGBoosterUpdateOneIter(BoosterHandle handle, int iter, DMatrixHandle dtrain) {
  DP_API_BEGIN();
  as_booster(handle)->update_one_iter(iter, as_dmatrix(dtrain));
  DP_API_END();
}

int XGBoosterBoostedRounds(BoosterHandle handle, int* out) {
  DP_API_BEGIN();
  need(out != nullptr, "output pointer is null");
  *out = as_booster(handle)->boosted_rounds();
  DP_API_END();
}

int XGBoosterSaveJsonConfig(BoosterHandle handle, bst_ulong* out_len, const char** out) {
  DP_API_BEGIN();
  need(out_len != nullptr && out != nullptr, "output pointers are null");
  const std::string& s = as_booster(handle)->save_config_json();
  *out_len = s.size();
  *out = s.c_str();
  DP_API_END();
}

int XGBoosterSaveModel(BoosterHandle handle, const char* fname) {
  DP_API_BEGIN();
  need(fname != nullptr, "file name is null");
  const std::string path(fname);
  need(ends_with(path, ".json"), "only JSON models (a .json file name) are supported");
  const std::string& s = as_booster(handle)->save_model_json();
  std::ofstream f(path, std::ios::binary | std::ios::trunc);
  need(bool(f), "cannot write " + dp::printable(path));
  f.write(s.data(), std::streamsize(s.size()));
  f.flush();
  need(bool(f), "cannot write " + dp::printable(path));
  DP_API_END();
}

int XGBoosterSaveModelToBuffer(BoosterHandle handle, const char* config, bst_ulong* out_len, const char** out) {
  DP_API_BEGIN();
  need(config != nullptr, "config is null");
  need(out_len != nullptr && out != nullptr, "output pointers are null");
  const dp::json::Value c = dp::json::parse(config);
  need(c.at("format").as_string() == "json", "only {\"format\":\"json\"} is supported");
  const std::string& s = as_booster(handle)->save_model_json();
  *out_len = s.size();
  *out = s.c_str();
  DP_API_END();
}

int XGBoosterLoadModelFromBuffer(BoosterHandle handle, const void* buf, bst_ulong len) {
  DP_API_BEGIN();
  need(buf != nullptr && len > 0, "model buffer is empty");
  as_booster(handle)->load_model_json(std::string(static_cast<const char*>(buf), len));
  DP_API_END();
}

int XGBoosterLoadModel(BoosterHandle handle, const char* fname) {
  DP_API_BEGIN();
  need(fname != nullptr, "file name is null");
  as_booster(handle)->load_model_json(read_file(fname));
  DP_API_END();
}

int XGBoosterSlice(BoosterHandle handle, int begin_layer, int end_layer, int step, BoosterHandle* out) {
  DP_API_BEGIN();
  need(out != nullptr, "output handle pointer is null");
  *out = as_booster(handle)->slice(begin_layer, end_layer, step).release();
  DP_API_END();
}

int XGBoosterPredictFromCudaArray(BoosterHandle handle, const char* values, const char* config, DMatrixHandle m,
                                  const bst_ulong** out_shape, bst_ulong* out_dim, const float** out_result) {
  DP_API_BEGIN();
  (void)m;  // the proxy DMatrix of XGBoost's inplace prediction carries nothing needed here
  dp::Booster* b = as_booster(handle);
  need(out_shape && out_dim && out_result, "output pointers are null");
  need(config != nullptr, "prediction config is null");
  const DenseSpec spec = dense_spec(values, config);
  const dp::json::Value c = dp::json::parse(config);
  dp::Booster::PredictRequest q;
  q.x = spec.ptr;
  q.rows = spec.rows;
  q.cols = spec.cols;
  q.stride = spec.stride;
  q.has_mv = spec.has_mv;
  q.mv = spec.mv;
  // checked before narrowing, so that no value wraps into a valid-looking one
  auto small_int = [&](const char* key, long long lo, long long hi, int dflt, const char* what) {
    const auto* v = c.find(key);
    if (!v) return dflt;
    const long long x = v->as_int();
    need(x >= lo && x <= hi, std::string("prediction config ") + key + " is out of range: " + what);
    return int(x);
  };
  q.type = small_int("type", 0, 1, q.type, "only types 0 (value) and 1 (margin) are supported");
  q.it_begin = small_int("iteration_begin", 0, b->model.rounds(), q.it_begin,
                         "iteration range outside the model's rounds");
  q.it_end = small_int("iteration_end", 0, b->model.rounds(), q.it_end, "iteration range outside the model's rounds");
  if (const auto* v = c.find("strict_shape")) q.strict_shape = v->as_bool();
  need(b->params.K() >= 1, "num_class must be at least 1 to predict with a multi-class objective");
  q.device = q.rows ? pointer_device(spec.ptr, false) : 0;
  {
    dp::DeviceGuard g(q.device);
    // the producer may still be writing on its own stream
    dp::cuda_check(cudaDeviceSynchronize(), "synchronise producer");
  }
  const dp::u64* shape = nullptr;
  dp::u64 dims = 0;
  *out_result = b->predict(q, &shape, &dims);
  *out_shape = reinterpret_cast<const bst_ulong*>(shape);
  *out_dim = bst_ulong(dims);
  DP_API_END();
}

int XGBoosterGetNumFeature(BoosterHandle handle, bst_ulong* out) {
  DP_API_BEGIN();
  need(out != nullptr, "output pointer is null");
  *out = bst_ulong(as_booster(handle)->model.num_feature);
  DP_API_END();
}

// ---- extensions --------------------------------------------------------------
int dp_comm_unique_id(void* out128) {
  DP_API_BEGIN();
  need(out128 != nullptr, "output pointer is null");
  dp::nccl_unique_id(out128);
  DP_API_END();
}

int dp_comm_create(const void* unique_id128, int nranks, int rank, int device, void** out) {
  DP_API_BEGIN();
  need(unique_id128 != nullptr && out != nullptr, "null argument");
  *out = dp::make_nccl_comm(unique_id128, nranks, rank, device);
  DP_API_END();
}

int dp_comm_free(void* comm) {
  DP_API_BEGIN();
  delete static_cast<dp::Comm*>(comm);
  DP_API_END();
}

int dp_comm_set_timeout(void* comm, int64_t timeout_ms) {
  DP_API_BEGIN();
  need(comm != nullptr, "communicator is null");
  static_cast<dp::Comm*>(comm)->set_timeout_ms(timeout_ms);
  DP_API_END();
}

int dp_release_cached_memory(void) {
  DP_API_BEGIN();
  dp::SlabCache::release_all();
  DP_API_END();
}

int dp_comm_reduce_scatter_hist(void* comm, const int64_t* send, int64_t* recv, uint64_t recv_n, void* stream) {
  DP_API_BEGIN();
  need(comm != nullptr, "communicator is null");
  need(recv_n == 0 || (send != nullptr && recv != nullptr), "null buffer");
  static_cast<dp::Comm*>(comm)->reduce_scatter_i64(send, recv, recv_n, static_cast<cudaStream_t>(stream));
  DP_API_END();
}

int dp_booster_set_comm(BoosterHandle handle, void* comm) {
  DP_API_BEGIN();
  dp::Booster* b = as_booster(handle);
  need(b->boosted_rounds() == 0, "the communicator must be attached before the first round");
  b->comm = static_cast<dp::Comm*>(comm);
  DP_API_END();
}

int dp_booster_set_profiling(BoosterHandle handle, int on) {
  DP_API_BEGIN();
  dp::Booster* b = as_booster(handle);
  need(on >= 0 && on <= 2, "profiling mode must be 0, 1 or 2");
  b->profiling = on;
  if (b->engine()) {
    b->engine()->profiler().enable(b->profiling);
    if (b->profiling) b->engine()->profiler().reset();
  }
  DP_API_END();
}

int dp_booster_profile(BoosterHandle handle, const char** out_json) {
  DP_API_BEGIN();
  need(out_json != nullptr, "output pointer is null");
  dp::Booster* b = as_booster(handle);
  b->profile_buf = b->engine() ? b->engine()->profiler().json() : std::string("{}");
  *out_json = b->profile_buf.c_str();
  DP_API_END();
}

int dp_booster_margins(BoosterHandle handle, float* out, bst_ulong len) {
  DP_API_BEGIN();
  dp::Booster* b = as_booster(handle);
  need(b->engine() != nullptr, "the booster has not been trained on a matrix");
  const std::vector<float> m = b->engine()->margins();
  need(len == m.size(), "margin buffer size differs from rows * outputs");
  need(len == 0 || out != nullptr, "margin buffer is null");
  std::memcpy(out, m.data(), m.size() * sizeof(float));
  DP_API_END();
}

uint64_t dp_launch_count(void) { return dp::launch_counter().load(); }

int dp_quantile_cuts(const float* x, uint64_t rows, uint32_t features, uint64_t row_stride, int max_bin,
                     float* cut, uint16_t* nbins, uint8_t* has_missing, void* stream) {
  DP_API_BEGIN();
  need(rows == 0 || x != nullptr, "matrix pointer is null");
  need(cut != nullptr && nbins != nullptr && has_missing != nullptr, "output pointer is null");
  need(row_stride >= features, "row_stride must cover the features");
  dp::CutsDevice cd{cut, nbins, has_missing};
  dp::compute_cuts(x, rows, features, row_stride, max_bin, false, 0.f, rows, nullptr, cd,
                   static_cast<cudaStream_t>(stream));
  DP_API_END();
}

int dp_bin_matrix(const float* x, uint64_t rows, uint32_t features, uint64_t row_stride, const float* cut,
                  const uint16_t* nbins, uint8_t* bins, uint64_t bin_stride, void* stream) {
  DP_API_BEGIN();
  need(bin_stride >= features && bin_stride % 16 == 0, "bin_stride must cover the features and be a multiple of 16");
  need(rows == 0 || (x != nullptr && bins != nullptr), "matrix or bins pointer is null");
  need(cut != nullptr && nbins != nullptr, "cuts pointer is null");
  need(row_stride >= features, "row_stride must cover the features");
  dp::CutsDevice cd{const_cast<float*>(cut), const_cast<uint16_t*>(nbins), nullptr};
  dp::launch_bin_matrix(x, rows, features, row_stride, false, 0.f, cd, bins, bin_stride,
                        static_cast<cudaStream_t>(stream));
  DP_API_END();
}

int dp_gradients(int objective, int num_class, const float* margin, const float* label, uint64_t rows, float* gh,
                 float* scales, void* stream) {
  DP_API_BEGIN();
  need(objective >= 0 && objective <= 3, "objective id must be 0..3");
  const int K = (objective >= 2) ? num_class : 1;
  need(K >= 1, "num_class must be at least 1");
  need(rows == 0 || (margin != nullptr && label != nullptr && gh != nullptr), "margin, label or gh pointer is null");
  need(scales != nullptr, "scales pointer is null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dp::DevBuf<dp::u32> mx(2 * size_t(K));
  dp::cuda_check(cudaMemsetAsync(mx.get(), 0, 2 * K * sizeof(dp::u32), s), "memset");
  dp::launch_gradients(objective, K, margin, label, rows, reinterpret_cast<float2*>(gh), mx.get(), mx.get() + K, s);
  dp::launch_scales(K, mx.get(), mx.get() + K, reinterpret_cast<dp::Scales*>(scales), s);
  dp::cuda_check(cudaStreamSynchronize(s), "gradients");
  DP_API_END();
}

}  // extern "C"

namespace {

// Task list and device descriptors of one histogram build.
struct HistPlan {
  const uint8_t* bins = nullptr;
  uint64_t bin_stride = 0;
  uint32_t features = 0;
  int kernel_bins = 256;         // bin budget of the 32-feature kernel launched
  bool quantized = false;
  int64_t* hist = nullptr;
  int32_t nseg = 0;
  dp::u32 ntasks = 0;
  dp::DevBuf<dp::HistTask> tasks;
  dp::DevBuf<dp::TreeArrays> trees;
  dp::DevBuf<dp::Scales> scales;
  dp::DevBuf<dp::u32> counter;
  bool wide = false;             // the 64-feature kernel
  int device = 0;
};

HistPlan* make_hist_plan(const uint8_t* bins, uint64_t bin_stride, uint32_t features, int32_t num_bins,
                         bool quantized, const void* gh, const uint32_t* ridx, const int64_t* seg_begin,
                         const int64_t* seg_end, int32_t nseg, float sg, float sh, int64_t* hist) {
  need(nseg >= 0 && (nseg == 0 || (seg_begin && seg_end)), "invalid segments");
  need(num_bins >= 1 && num_bins <= 256, "num_bins must be in [1, 256]");
  need(bin_stride % 16 == 0 && bin_stride >= features, "bin_stride must cover the features and be a multiple of 16");
  auto p = std::make_unique<HistPlan>();
  dp::cuda_check(cudaGetDevice(&p->device), "cudaGetDevice");
  p->bins = bins;
  p->bin_stride = bin_stride;
  p->features = features;
  p->quantized = quantized;
  p->hist = hist;
  p->nseg = nseg;
  need(nseg == 0 || hist != nullptr, "hist pointer is null");
  std::vector<dp::HistTask> tasks;
  // the training path's choice on one GPU: 256-bin matrices of more than 64
  // features use the 64-feature kernel (DP_HIST_WIDE=0 / 1 overrides above
  // 32 features)
  const char* wide_env = std::getenv("DP_HIST_WIDE");
  const bool wide_default = features > 2 * dp::kHistFeatureTile;
  p->wide = num_bins > 64 && features > dp::kHistFeatureTile &&
            (wide_env && *wide_env ? std::string(wide_env) != "0" : wide_default);
  const dp::u32 tile = p->wide ? dp::kHistWideTile : dp::kHistFeatureTile;
  const dp::u32 ftiles = (features + tile - 1) / tile;
  dp::u64 total = 0, filled = 0;
  for (int32_t i = 0; i < nseg; ++i) {
    need(seg_begin[i] >= 0 && seg_end[i] >= seg_begin[i] && seg_end[i] < (int64_t(1) << 31),
         "invalid segment bounds (positions must be below 2^31)");
    total += dp::u64(seg_end[i] - seg_begin[i]);
    filled += seg_end[i] > seg_begin[i] ? 1 : 0;
  }
  p->kernel_bins = dp::hist_kernel_bins(num_bins, filled);
  need(total == 0 || (bins != nullptr && gh != nullptr && ridx != nullptr), "bins, gh or ridx pointer is null");
  int64_t chunk = int64_t(dp::hist_chunk_rows(total * ftiles, dp::u64(nseg), bin_stride % 128 == 0));
  // testing knob: longer tasks, so that tests reach the multi-window folds
  if (const char* c = std::getenv("DP_HIST_MIN_CHUNK")) chunk = std::max<int64_t>(chunk, std::atoll(c));
  // Queue order: piece index first, then segment, then feature tile.  With
  // row lists grouped by node and ascending inside a node, the p-th pieces of
  // all nodes cover about the same range of rows, so the blocks running at
  // one time read neighbouring rows of the bin matrix instead of every
  // N-th row of one node.
  std::vector<int64_t> pieces(size_t(std::max(nseg, 0))), piece(size_t(std::max(nseg, 0)));
  int64_t max_pieces = 0;
  for (int32_t i = 0; i < nseg; ++i) {
    const int64_t n = seg_end[i] - seg_begin[i];
    pieces[i] = n ? (n + chunk - 1) / chunk : 0;
    piece[i] = n ? (n + pieces[i] - 1) / pieces[i] : 0;
    max_pieces = std::max(max_pieces, pieces[i]);
  }
  for (int64_t q = 0; q < max_pieces; ++q)
    for (int32_t i = 0; i < nseg; ++i) {
      const int64_t b = seg_begin[i] + q * piece[i];
      if (q >= pieces[i] || b >= seg_end[i]) continue;
      for (dp::u32 ft = 0; ft < ftiles; ++ft)
        tasks.push_back(dp::HistTask{dp::u32(i), ft * tile, 0, 0, b, std::min<int64_t>(seg_end[i], b + piece[i])});
    }
  p->ntasks = dp::u32(tasks.size());
  p->tasks.resize(std::max<size_t>(tasks.size(), 1));
  p->trees.resize(1);
  p->scales.resize(1);
  p->counter.resize(1);
  const dp::TreeArrays th{const_cast<uint32_t*>(ridx), reinterpret_cast<float2*>(const_cast<void*>(gh))};
  const dp::Scales sc{sg, sh};
  dp::cuda_check(cudaMemcpy(p->trees.get(), &th, sizeof th, cudaMemcpyHostToDevice), "upload");
  dp::cuda_check(cudaMemcpy(p->scales.get(), &sc, sizeof sc, cudaMemcpyHostToDevice), "upload");
  if (!tasks.empty())
    dp::cuda_check(cudaMemcpy(p->tasks.get(), tasks.data(), tasks.size() * sizeof(dp::HistTask),
                              cudaMemcpyHostToDevice),
                   "upload");
  return p.release();
}

void run_hist_plan(const HistPlan& p, cudaStream_t s) {
  const dp::u64 slot = dp::u64(p.features) * dp::kMaxBins * 2;
  if (p.nseg) dp::cuda_check(cudaMemsetAsync(p.hist, 0, dp::u64(p.nseg) * slot * sizeof(int64_t), s), "memset");
  if (p.wide)
    dp::launch_histograms_wide(p.bins, p.bin_stride, p.features, p.quantized, p.trees.get(), p.scales.get(),
                               p.tasks.get(), p.ntasks, p.counter.get(), p.hist, s, nullptr, nullptr);
  else
    dp::launch_histograms(p.bins, p.bin_stride, p.features, p.kernel_bins, p.quantized, p.trees.get(),
                          p.scales.get(), p.tasks.get(), p.ntasks, p.counter.get(), p.hist, s);
}

}  // namespace

extern "C" {

int dp_hist_build(const uint8_t* bins, uint64_t bin_stride, uint32_t features, int32_t num_bins, const float* gh,
                  const uint32_t* ridx, const int64_t* seg_begin, const int64_t* seg_end, int32_t nseg, float sg,
                  float sh, int64_t* hist, void* stream) {
  DP_API_BEGIN();
  std::unique_ptr<HistPlan> p(make_hist_plan(bins, bin_stride, features, num_bins, false, gh, ridx, seg_begin,
                                             seg_end, nseg, sg, sh, hist));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  run_hist_plan(*p, s);
  dp::cuda_check(cudaStreamSynchronize(s), "histograms");
  DP_API_END();
}

int dp_hist_prepare(const uint8_t* bins, uint64_t bin_stride, uint32_t features, int32_t num_bins, int32_t gh_kind,
                    const void* gh, const uint32_t* ridx, const int64_t* seg_begin, const int64_t* seg_end,
                    int32_t nseg, float sg, float sh, int64_t* hist, void** out_plan) {
  DP_API_BEGIN();
  need(out_plan != nullptr, "output pointer is null");
  need(gh_kind == 0 || gh_kind == 1, "gh_kind must be 0 (fp32 pairs) or 1 (quantised int32 pairs)");
  *out_plan = make_hist_plan(bins, bin_stride, features, num_bins, gh_kind == 1, gh, ridx, seg_begin, seg_end,
                             nseg, sg, sh, hist);
  DP_API_END();
}

int dp_hist_run(void* plan, void* stream) {
  DP_API_BEGIN();
  need(plan != nullptr, "plan is null");
  const HistPlan& p = *static_cast<HistPlan*>(plan);
  dp::DeviceGuard g(p.device);
  run_hist_plan(p, static_cast<cudaStream_t>(stream));
  DP_API_END();
}

int dp_hist_free(void* plan) {
  DP_API_BEGIN();
  delete static_cast<HistPlan*>(plan);
  DP_API_END();
}

int dp_quantize_gh(float* gh, uint64_t n, float sg, float sh, void* stream) {
  DP_API_BEGIN();
  need(n == 0 || gh != nullptr, "gh pointer is null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dp::DevBuf<dp::Scales> sc(1);
  const dp::Scales h{sg, sh};
  dp::cuda_check(cudaMemcpyAsync(sc.get(), &h, sizeof h, cudaMemcpyHostToDevice, s), "upload");
  dp::launch_quantize_gh(reinterpret_cast<float2*>(gh), n, 1, sc.get(), s);
  dp::cuda_check(cudaStreamSynchronize(s), "quantize");
  DP_API_END();
}

int dp_eval_splits(const int64_t* hist, int32_t nnodes, uint32_t features, const uint16_t* nbins,
                   const uint8_t* has_missing, const int64_t* totals, float sg, float sh, double lambda, double alpha,
                   double gamma, double min_child_weight, int32_t* out_i, double* out_gain, int64_t* out_left) {
  DP_API_BEGIN();
  need(nnodes >= 0, "invalid node count");
  if (nnodes == 0) return 0;
  need(hist != nullptr && nbins != nullptr && has_missing != nullptr && totals != nullptr, "input pointer is null");
  need(out_i != nullptr && out_gain != nullptr && out_left != nullptr, "output pointer is null");
  need(features > 0, "features must be positive");
  std::vector<dp::EvalNode> en(nnodes);
  for (int32_t n = 0; n < nnodes; ++n)
    en[n] = dp::EvalNode{dp::u32(n), 0, totals[2 * n], totals[2 * n + 1], dp::kNoSlot, 0};
  const dp::u32 nchunks = (features + dp::kEvalFeatureChunk - 1) / dp::kEvalFeatureChunk;
  dp::DevBuf<dp::EvalNode> de(nnodes);
  dp::DevBuf<dp::SplitCand> cand(size_t(nnodes) * nchunks), best(nnodes);
  dp::DevBuf<dp::Scales> sc(1);
  const dp::Scales s{sg, sh};
  dp::cuda_check(cudaMemcpy(de.get(), en.data(), en.size() * sizeof(dp::EvalNode), cudaMemcpyHostToDevice), "upload");
  dp::cuda_check(cudaMemcpy(sc.get(), &s, sizeof s, cudaMemcpyHostToDevice), "upload");
  dp::SplitParams p;
  p.lambda = lambda;
  p.alpha = alpha;
  p.gamma = gamma;
  p.min_child_weight = min_child_weight;
  dp::launch_eval_splits(hist, features, nbins, has_missing, de.get(), dp::u32(nnodes), sc.get(), p, cand.get(),
                         best.get(), nullptr);
  std::vector<dp::SplitCand> b(nnodes);
  dp::cuda_check(cudaMemcpy(b.data(), best.get(), b.size() * sizeof(dp::SplitCand), cudaMemcpyDeviceToHost),
                 "download");
  for (int32_t n = 0; n < nnodes; ++n) {
    out_i[4 * n] = b[n].feature;
    out_i[4 * n + 1] = b[n].bin;
    out_i[4 * n + 2] = b[n].default_left;
    out_i[4 * n + 3] = b[n].feature >= 0;
    out_gain[n] = b[n].gain;
    out_left[2 * n] = b[n].gl;
    out_left[2 * n + 1] = b[n].hl;
  }
  DP_API_END();
}

// ---- CSV input transport (native/decision_programs_csv.hpp:36-67)
namespace {
struct CsvHandle {
  std::unique_ptr<dp::CsvDense> d;
  int device = 0;
};
CsvHandle* csv_handle(void* h) {
  dp::need(h != nullptr, "invalid CSV handle");
  return static_cast<CsvHandle*>(h);
}
}  // namespace

int dp_csv_decode(const char* bytes, uint64_t size, const char* target, const char* header_mode, void* stream,
                  void** out) {
  DP_API_BEGIN();
  dp::need(out != nullptr && (bytes != nullptr || size == 0), "dp_csv_decode: invalid arguments");
  auto h = std::make_unique<CsvHandle>();
  dp::cuda_check(cudaGetDevice(&h->device), "cudaGetDevice");
  h->d = dp::csv_decode(bytes, size, target ? target : "", header_mode ? header_mode : "auto",
                        static_cast<cudaStream_t>(stream));
  *out = h.release();
  DP_API_END();
}

int dp_csv_shape(void* csv, uint64_t* rows, uint32_t* features, uint32_t* classes, int32_t* header) {
  DP_API_BEGIN();
  const auto& d = *csv_handle(csv)->d;
  if (rows) *rows = d.rows;
  if (features) *features = d.features;
  if (classes) *classes = d.classes;
  if (header) *header = d.header ? 1 : 0;
  DP_API_END();
}

int dp_csv_data(void* csv, const float** values, const uint32_t** labels) {
  DP_API_BEGIN();
  const auto& d = *csv_handle(csv)->d;
  if (values) *values = d.values.get();
  if (labels) *labels = d.has_target ? d.labels.get() : nullptr;
  DP_API_END();
}

int dp_csv_metadata(void* csv, const char** json, double* device_ms) {
  DP_API_BEGIN();
  const auto& d = *csv_handle(csv)->d;
  if (json) *json = d.meta.c_str();
  if (device_ms) *device_ms = d.ms_device;
  DP_API_END();
}

int dp_csv_copy(void* csv, float* values, uint32_t* labels) {
  DP_API_BEGIN();
  CsvHandle* h = csv_handle(csv);
  dp::DeviceGuard g(h->device);
  const auto& d = *h->d;
  if (values && d.rows)
    dp::cuda_check(cudaMemcpy(values, d.values.get(), d.rows * d.features * sizeof(float), cudaMemcpyDeviceToHost),
                   "copy CSV values");
  if (labels && d.has_target && d.rows)
    dp::cuda_check(cudaMemcpy(labels, d.labels.get(), d.rows * sizeof(uint32_t), cudaMemcpyDeviceToHost),
                   "copy CSV labels");
  DP_API_END();
}

int dp_csv_parse_feature(const char* token, uint64_t size, float* value) {
  DP_API_BEGIN();
  dp::need(token != nullptr || size == 0, "dp_csv_parse_feature: token missing");
  dp::need(size < (uint64_t(1) << 32), "dp_csv_parse_feature: token too long");
  float v = 0.0f;
  const bool ok =
      dp::csv_parse_feature_host(reinterpret_cast<const unsigned char*>(token), static_cast<dp::u32>(size), &v);
  if (value) *value = v;
  if (!ok) {
    g_last_error = "token refused";
    return 1;
  }
  DP_API_END();
}

int dp_csv_free(void* csv) {
  DP_API_BEGIN();
  if (csv) {
    CsvHandle* h = static_cast<CsvHandle*>(csv);
    dp::DeviceGuard g(h->device);
    delete h;
  }
  DP_API_END();
}

}  // extern "C"
