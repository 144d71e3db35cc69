/* libdp_gbdt -- B200 (sm_100a) gradient-boosted-tree training behind the
 * XGBoost 3.4.1 C-API subset that the decision-programs trainer binds with
 * dlopen/dlsym (native/class_model_native_adapter.cuh:20-31).
 *
 * Conventions (as the reference expects them):
 *  - every int-returning call returns 0 on success and -1 on failure; the
 *    message is then available from XGBGetLastError() (thread-local)
 *    (native/class_model_native_adapter.cuh:23);
 *  - handles are opaque; string / array outputs are borrowed and stay valid
 *    until the next call on the same handle (native/class_study_train.hpp:63-64);
 *  - matrices borrow the caller's CUDA fp32 memory, which must outlive the
 *    DMatrix (native/class_study_oof.cu:532-534);
 *  - training runs on the device that holds the matrix; there is no CPU path.
 */
#ifndef DP_GBDT_H_
#define DP_GBDT_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DP_API __attribute__((visibility("default")))

typedef void* DMatrixHandle;
typedef void* BoosterHandle;
typedef uint64_t bst_ulong;

/* ---- XGBoost C-API subset ------------------------------------------------ */

/* Reports 3,4,1 for ABI compatibility; the reference refuses any other
 * version (native/class_model_native_adapter.cuh:24). */
DP_API void XGBoostVersion(int* major, int* minor, int* patch);

/* JSON with "USE_CUDA":true (checked at native/class_model_native_adapter.cuh:24)
 * and "DP_B200_GBDT":true identifying this implementation. */
DP_API int XGBuildInfo(const char** out);

/* Thread-local message of the last failure (native/class_model_native_adapter.cuh:21,23). */
DP_API const char* XGBGetLastError(void);

/* Dense fp32 CUDA matrix from a __cuda_array_interface__ JSON object
 * {"data":[ptr,ro],"shape":[R,F],"strides":null|[bytes,4],"typestr":"<f4",...}
 * and config {"missing":NaN|value,"nthread":n}.  Rejects +-inf.
 * Replaces native/class_native_training.cuh:51 (array JSON built at
 * native/class_model_native_adapter.cuh:26). */
DP_API int XGDMatrixCreateFromCudaArrayInterface(const char* data, const char* config, DMatrixHandle* out);

/* Dense fp32 HOST matrix (same array-interface and config JSON, host data
 * pointer), copied to the calling thread's current CUDA device.  XGBoost C API
 * function; the reference binds only the CUDA variant above.  The copy runs in
 * chunks that overlap the first counting pass of the quantile cuts; pinned
 * host memory lets the chunks stream at the host link's rate.  The host
 * buffer may be released when the call returns. */
DP_API int XGDMatrixCreateFromDense(const char* data, const char* config, DMatrixHandle* out);

/* field "label": f32 [R] array interface (device or host memory); copied.
 * Replaces native/class_native_training.cuh:52. */
DP_API int XGDMatrixSetInfoFromInterface(DMatrixHandle handle, const char* field, const char* data);

/* field "label" from host memory (XGBoost C API; used by host-side callers). */
DP_API int XGDMatrixSetFloatInfo(DMatrixHandle handle, const char* field, const float* data, bst_ulong len);

DP_API int XGDMatrixNumRow(DMatrixHandle handle, bst_ulong* out);
DP_API int XGDMatrixNumCol(DMatrixHandle handle, bst_ulong* out);

/* Replaces the free calls at native/class_model_native_adapter.cuh:21,25. */
DP_API int XGDMatrixFree(DMatrixHandle handle);

/* native/class_native_training.cuh:56 (with the training matrix) and
 * native/class_study_train.cu:98 (with nullptr, 0). */
DP_API int XGBoosterCreate(const DMatrixHandle dmats[], bst_ulong len, BoosterHandle* out);
DP_API int XGBoosterFree(BoosterHandle handle);

/* Parameters as the reference sets them (native/class_native_training.cuh:57-65,
 * native/class_model_native_adapter.cuh:27): objective in {multi:softmax,
 * multi:softprob, binary:logistic, reg:squarederror}, num_class, max_depth,
 * max_bin, eta, lambda, alpha, gamma, min_child_weight, subsample,
 * colsample_*, base_score (scalar or JSON array), seed, device "cuda:N",
 * tree_method "hist"; bookkeeping keys (nthread, verbosity, ...) are accepted. */
DP_API int XGBoosterSetParam(BoosterHandle handle, const char* name, const char* value);

/* One boosting round (K trees for K-class objectives); synchronous.
 * The hot path: replaces native/class_native_training.cuh:67. */
DP_API int XGBoosterUpdateOneIter(BoosterHandle handle, int iter, DMatrixHandle dtrain);

/* native/class_model_train.cu:49, native/class_study_train.cu:104,127,328. */
DP_API int XGBoosterBoostedRounds(BoosterHandle handle, int* out);

/* Configuration JSON; learner.generic_param.device == "cuda:N" and
 * learner.gradient_booster.updater[0].name == "grow_gpu_hist" as checked at
 * native/class_model_train.cu:48 and native/class_study_train.cu:327.
 * Replaces native/class_native_training.cuh:68. */
DP_API int XGBoosterSaveJsonConfig(BoosterHandle handle, bst_ulong* out_len, const char** out);

/* XGBoost-3.4.1-schema JSON model (".json" paths only).
 * Replaces native/class_native_training.cuh:69. */
DP_API int XGBoosterSaveModel(BoosterHandle handle, const char* fname);

/* config {"format":"json"}; replaces native/class_study_train.cu:329,363. */
DP_API int XGBoosterSaveModelToBuffer(BoosterHandle handle, const char* config, bst_ulong* out_len,
                                      const char** out);

/* native/class_study_train.cu:101 and native/class_model_native_adapter.cuh:29. */
DP_API int XGBoosterLoadModelFromBuffer(BoosterHandle handle, const void* buf, bst_ulong len);
DP_API int XGBoosterLoadModel(BoosterHandle handle, const char* fname);

/* Rounds [begin, end) with step; end == 0 means all rounds.
 * native/class_study_train.cu:130,355. */
DP_API int XGBoosterSlice(BoosterHandle handle, int begin_layer, int end_layer, int step, BoosterHandle* out);

/* native/class_model_convert.cpp:112. */
DP_API int XGBoosterGetNumFeature(BoosterHandle handle, bst_ulong* out);

/* Prediction over a dense fp32 CUDA matrix (array interface as for
 * XGDMatrixCreateFromCudaArrayInterface).  config: {"type":0|1,
 * "training":false,"iteration_begin":b,"iteration_end":e (0 = all rounds),
 * "strict_shape":true|false,"cache_id":0,"missing":NaN|value}.  type 0 is the
 * objective's output (squared error: the margin; logistic: probability;
 * multi:softprob: K probabilities; multi:softmax: the class index as float),
 * type 1 the raw margins [R][K].  *out_result is a device pointer on the
 * input's device, owned by the booster until the next call on it; out_shape
 * is [R, width] with strict_shape (width K for margins and probabilities,
 * else 1), else [R] when width is 1.  The proxy handle m may be null.
 * Replaces native/class_study_train.cu:158 and
 * native/class_model_native_adapter.cuh:30. */
DP_API int XGBoosterPredictFromCudaArray(BoosterHandle handle, const char* values, const char* config,
                                         DMatrixHandle m, const bst_ulong** out_shape, bst_ulong* out_dim,
                                         const float** out_result);

/* ---- extensions (no counterpart in the reference, which is single-GPU) --- */

/* Multi-GPU: rank 0 creates a 128-byte NCCL unique id, every rank creates a
 * communicator with it and attaches it to its booster before the first
 * round.  Rows are sharded across ranks; trees are identical on every rank. */
DP_API int dp_comm_unique_id(void* out128);
DP_API int dp_comm_create(const void* unique_id128, int nranks, int rank, int device, void** out);
/* Free every booster attached to a communicator before the communicator:
 * a booster's rounds are CUDA graphs that hold the communicator's calls, and
 * NCCL's destroy waits until those graphs are released. */
DP_API int dp_comm_free(void* comm);
DP_API int dp_booster_set_comm(BoosterHandle handle, void* comm);
/* Failure detection: every host wait of a round that has collectives in
 * flight polls the communicator for an asynchronous error and gives up after
 * timeout_ms (<= 0: no deadline; default DP_COMM_TIMEOUT_MS, else 600000).
 * Either aborts the communicator, which ends its kernels in flight, and the
 * training call returns -1 with the reason in XGBGetLastError(); the
 * communicator and the booster are unusable afterwards. */
DP_API int dp_comm_set_timeout(void* comm, int64_t timeout_ms);
/* The sharded path's histogram exchange on its own, for kernel-level builds
 * over rows sharded across ranks: recv[0, recv_n) = the sum over ranks of
 * each rank's block send[rank * recv_n, (rank + 1) * recv_n) of int64
 * partial histograms (send holds nranks blocks), ordered on `stream`. */
DP_API int dp_comm_reduce_scatter_hist(void* comm, const int64_t* send, int64_t* recv, uint64_t recv_n, void* stream);

/* Frees the device memory kept for reuse: the library keeps the memory of
 * freed boosters and matrices (at most four allocations, at most half of a
 * device's memory) so that the next booster or matrix there (a search or
 * out-of-fold fits create one per fit) does not pay for cudaMalloc and
 * cudaFree, which wait for the device.  No counterpart in the reference. */
DP_API int dp_release_cached_memory(void);

/* Per-kernel CUDA-event timings of the training rounds ({"name":{"launches",
 * "ms","alg_bytes"}}), collected on the launching stream while enabled:
 * mode 1 times every instrumented launch, mode 2 only the histogram launches
 * (the least instrumentation), 0 turns timing off.  Enabling resets the
 * counters. */
DP_API int dp_booster_set_profiling(BoosterHandle handle, int on);
DP_API int dp_booster_profile(BoosterHandle handle, const char** out_json);

/* Training margins [R][K] of the booster's training matrix (host copy). */
DP_API int dp_booster_margins(BoosterHandle handle, float* out, bst_ulong len);

/* Number of CUDA kernels this library has launched in the process. */
DP_API uint64_t dp_launch_count(void);

/* ---- kernel-level entry points (device pointers; stream may be NULL) ----- */

/* Exact quantile cuts: cut[F][256], nbins[F], has_missing[F]. */
DP_API int dp_quantile_cuts(const float* x, uint64_t rows, uint32_t features, uint64_t row_stride, int max_bin,
                            float* cut, uint16_t* nbins, uint8_t* has_missing, void* stream);
/* bins[R][bin_stride] (bin_stride >= features, multiple of 16). */
DP_API int dp_bin_matrix(const float* x, uint64_t rows, uint32_t features, uint64_t row_stride, const float* cut,
                         const uint16_t* nbins, uint8_t* bins, uint64_t bin_stride, void* stream);
/* gh[K][R][2] and per-class quantiser scales scales[K][2] (sg, sh; device). */
DP_API int dp_gradients(int objective, int num_class, const float* margin, const float* label, uint64_t rows,
                        float* gh, float* scales, void* stream);
/* hist[nseg][F][256][2] (int64, overwritten) of position segments
 * [seg_begin[i], seg_end[i]) (host arrays) of (ridx, gh) in position order.
 * Every bin code must be < num_bins (1..256).  num_bins and the segment count
 * select the kernel, so a code at or above num_bins is outside the contract:
 * it may be counted in its own bin or dropped. */
DP_API int dp_hist_build(const uint8_t* bins, uint64_t bin_stride, uint32_t features, int32_t num_bins,
                         const float* gh, const uint32_t* ridx, const int64_t* seg_begin, const int64_t* seg_end,
                         int32_t nseg, float sg, float sh, int64_t* hist, void* stream);
/* In place: gh[n][2] fp32 pairs -> int32 pairs rint(g*sg), rint(h*sh), the
 * layout the training engine's histogram pass reads. */
DP_API int dp_quantize_gh(float* gh, uint64_t n, float sg, float sh, void* stream);
/* The same histogram build with its task list prepared once: dp_hist_prepare
 * uploads the tasks of the segments; dp_hist_run zeroes `hist` and enqueues
 * the kernel on `stream` without synchronising (for timing loops).  gh_kind 0:
 * fp32 pairs quantised with sg/sh in the kernel; 1: int32 pairs from
 * dp_quantize_gh. */
DP_API int dp_hist_prepare(const uint8_t* bins, uint64_t bin_stride, uint32_t features, int32_t num_bins,
                           int32_t gh_kind, const void* gh, const uint32_t* ridx, const int64_t* seg_begin,
                           const int64_t* seg_end, int32_t nseg, float sg, float sh, int64_t* hist, void** out_plan);
DP_API int dp_hist_run(void* plan, void* stream);
DP_API int dp_hist_free(void* plan);

/* CSV input transport on the GPU.  Replaces the reference's host-side
 * decision_programs_csv::decode(bytes, target, header) at
 * native/decision_programs_csv.hpp:36-67 (called at
 * native/decision_programs_cli.cpp:140): the same accepted inputs (RFC 4180
 * quoting, "\r\n" / "\r" / "\n" record ends, dropped empty lines, equal
 * column counts), the same header detection and target resolution (a header
 * name, "last" or a zero-based index; NULL or "" for none), the same feature
 * parsing (trimmed; empty, nan, na, null -> NaN; correctly rounded finite
 * binary32, bit for bit) and class labels (unsigned integers, or any text
 * numbered in order of first appearance), and the same error messages
 * (XGBGetLastError).  `bytes` is host memory; the decoded matrix stays on the
 * current device as row-major fp32 [rows][features] (a borrowed input for
 * XGDMatrixCreateFromCudaArrayInterface while the handle lives) with u32
 * labels.  dp_csv_metadata gives {"header": bool, "names": [...],
 * "label_mapping": null | [{"class": id, "label": text}, ...]} (what the
 * reference's Dense holds) and the device time of the decode. */
DP_API int dp_csv_decode(const char* bytes, uint64_t size, const char* target, const char* header_mode,
                         void* stream, void** out);
DP_API int dp_csv_shape(void* csv, uint64_t* rows, uint32_t* features, uint32_t* classes, int32_t* header);
DP_API int dp_csv_data(void* csv, const float** values, const uint32_t** labels);
DP_API int dp_csv_metadata(void* csv, const char** json, double* device_ms);
DP_API int dp_csv_copy(void* csv, float* values, uint32_t* labels);
DP_API int dp_csv_free(void* csv);
/* The decoder's rule for one feature token, on the host (the reference's
 * feature(), native/decision_programs_csv.hpp:28-34): returns 0 with *value
 * set when the token is accepted, 1 when it is refused, -1 on bad arguments. */
DP_API int dp_csv_parse_feature(const char* token, uint64_t size, float* value);

/* Shared-memory update ceiling of the histogram kernel on the current device:
 * the kernel's inner loop (two 32-bit shared atomics per (row, feature) pair,
 * 32 distinct banks per warp step, one 1024-thread block per SM) run alone for
 * `steps` warp steps over register-generated bin codes, with no global-memory
 * traffic.  Writes the measured (row, feature) pairs per second.  No
 * counterpart in the reference; a measurement aid for the histogram roofline. */
DP_API int dp_probe_hist_atomics(uint32_t steps, double* pairs_per_second, void* stream);

/* dp_hist_build for callers that cannot allocate device memory (a process
 * whose device memory is reserved up front by its own pool, or a latency path
 * that must not call cudaMalloc/cudaFree).  No counterpart in the reference.
 * Same arguments and result as dp_hist_build, but the scratch (task list, task
 * counter, descriptors) lives in one fixed file-scope device array of about
 * 1 MiB that every GPU loading the library keeps until exit; nothing is
 * allocated per call.  Limit: at most 32768 histogram tasks, i.e. roughly
 * (non-empty segments) x ceil(features / 32) <= 32768; larger calls fail with
 * a message (XGBGetLastError) naming the need and the capacity.  Every call
 * looks up the array's device address on its device (cudaGetSymbolAddress);
 * the first call on a device also loads the library's device code there, so
 * make it before any stream capture.  The call waits for `stream`
 * (cudaStreamSynchronize) before it returns.  Calls share the array: calls
 * that overlap on the GPU (other streams or threads) race, so serialise them.
 * The task counter is zeroed on every call and only tasks written by the call
 * are read. */
DP_API int dp_hist_build_noalloc(const uint8_t* bins, uint64_t bin_stride, uint32_t features, int32_t num_bins,
                                 const float* gh, const uint32_t* ridx, const int64_t* seg_begin,
                                 const int64_t* seg_end, int32_t nseg, float sg, float sh, int64_t* hist,
                                 void* stream);

/* Best split per node from hist[N][F][256][2] (device) and quantised totals
 * totals[N][2] (host); outputs on the host: out_i[N][4] = feature, bin,
 * default_left, valid; out_gain[N]; out_left[N][2]. */
DP_API int dp_eval_splits(const int64_t* hist, int32_t nnodes, uint32_t features, const uint16_t* nbins,
                          const uint8_t* has_missing, const int64_t* totals, float sg, float sh, double lambda,
                          double alpha, double gamma, double min_child_weight, int32_t* out_i, double* out_gain,
                          int64_t* out_left);

#ifdef __cplusplus
}
#endif

#endif /* DP_GBDT_H_ */
