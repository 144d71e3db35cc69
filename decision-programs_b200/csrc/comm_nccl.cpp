// NCCL communicator for row-sharded training: one process per GPU, sums of
// integer histograms / counts and maxima of gradient magnitudes over NVLink.
// libnccl.so.2 is opened with dlopen on first use, so the library has no
// link-time NCCL dependency and a process that already loaded NCCL (for
// example through torch.distributed) shares that copy.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "comm.h"
#include "common.h"
#include "watchdog.h"

namespace dp {

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                 cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  static std::string error;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) { error = std::string("cannot load NCCL: ") + dlerror(); return; }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.reduce_scatter = reinterpret_cast<decltype(api.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(h, "ncclCommAbort"));
    api.get_async_error = reinterpret_cast<decltype(api.get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!api.get_unique_id || !api.comm_init_rank || !api.all_reduce || !api.reduce_scatter || !api.all_gather ||
        !api.comm_destroy || !api.comm_abort || !api.get_async_error || !api.error_string) {
      error = "NCCL library lacks a required symbol";
      api = NcclApi{};
    }
  });
  need(api.all_reduce != nullptr, error.empty() ? "NCCL unavailable" : error);
  return api;
}

void check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) fail(std::string(what) + ": " + nccl().error_string(r));
}

class NcclComm final : public Comm {
 public:
  NcclComm(const void* id, int nranks, int rank, int device) : rank_(rank), size_(nranks), device_(device) {
    need(nranks >= 1 && rank >= 0 && rank < nranks, "invalid NCCL rank / size");
    ncclUniqueId uid;
    static_assert(sizeof(uid) == 128, "ncclUniqueId is 128 bytes");
    std::memcpy(&uid, id, sizeof uid);
    DeviceGuard g(device_);
    check(nccl().comm_init_rank(&comm_, nranks, uid, rank), "ncclCommInitRank");
    DP_CUDA(cudaMalloc(&scratch_, sizeof(u64)));
    if (const char* t = std::getenv("DP_COMM_TIMEOUT_MS")) timeout_ms_ = std::strtoll(t, nullptr, 10);
  }
  ~NcclComm() override {
    DeviceGuard g(device_);
    if (scratch_) cudaFree(scratch_);
    if (comm_) nccl().comm_destroy(comm_);
  }
  void wait(cudaStream_t s, const std::function<void()>& before_abort) override {
    live();
    const std::string why = wait_or_abort(
        [&] {
          const cudaError_t e = cudaStreamQuery(s);
          if (e == cudaErrorNotReady) return false;
          DP_CUDA(e);
          return true;
        },
        [&] {
          ncclResult_t r = ncclSuccess;
          const ncclResult_t q = nccl().get_async_error(comm_, &r);
          if (q != ncclSuccess) return std::string("ncclCommGetAsyncError: ") + nccl().error_string(q);
          return (r == ncclSuccess || r == ncclInProgress) ? std::string() : std::string(nccl().error_string(r));
        },
        [&] {
          if (before_abort) before_abort();
          // ends this communicator's kernels in flight; the comm is unusable after
          nccl().comm_abort(comm_);
          comm_ = nullptr;
        },
        timeout_ms_);
    if (!why.empty()) fail("NCCL communicator of rank " + std::to_string(rank_) + " aborted: " + why);
  }
  void set_timeout_ms(i64 ms) override { timeout_ms_ = ms; }
  int rank() const override { return rank_; }
  int size() const override { return size_; }
  void sum_u32(u32* d, size_t n, cudaStream_t s) override {
    live();
    if (n) check(nccl().all_reduce(d, d, n, ncclUint32, ncclSum, comm_, s), "ncclAllReduce(u32 sum)");
  }
  void reduce_scatter_i64(const i64* send, i64* recv, size_t recv_n, cudaStream_t s) override {
    live();
    if (recv_n)
      check(nccl().reduce_scatter(send, recv, recv_n, ncclInt64, ncclSum, comm_, s), "ncclReduceScatter(i64 sum)");
  }
  void all_gather_bytes(const void* send, void* recv, size_t bytes, cudaStream_t s) override {
    live();
    if (bytes) check(nccl().all_gather(send, recv, bytes, ncclUint8, comm_, s), "ncclAllGather(bytes)");
  }
  void sum_i64(i64* d, size_t n, cudaStream_t s) override {
    live();
    if (n) check(nccl().all_reduce(d, d, n, ncclInt64, ncclSum, comm_, s), "ncclAllReduce(i64 sum)");
  }
  void max_u32(u32* d, size_t n, cudaStream_t s) override {
    live();
    if (n) check(nccl().all_reduce(d, d, n, ncclUint32, ncclMax, comm_, s), "ncclAllReduce(u32 max)");
  }
  u64 sum_host_u64(u64 v, cudaStream_t s) override {
    live();
    DP_CUDA(cudaMemcpyAsync(scratch_, &v, sizeof v, cudaMemcpyHostToDevice, s));
    check(nccl().all_reduce(scratch_, scratch_, 1, ncclUint64, ncclSum, comm_, s), "ncclAllReduce(u64 sum)");
    u64 out = 0;
    DP_CUDA(cudaMemcpyAsync(&out, scratch_, sizeof out, cudaMemcpyDeviceToHost, s));
    wait(s, {});  // no graph holds this call
    return out;
  }

 private:
  void live() const { need(comm_ != nullptr, "the NCCL communicator was aborted after an earlier failure"); }
  ncclComm_t comm_ = nullptr;
  i64 timeout_ms_ = 600000;
  int rank_, size_, device_;
  u64* scratch_ = nullptr;
};

}  // namespace

Comm* make_nccl_comm(const void* unique_id, int nranks, int rank, int device) {
  return new NcclComm(unique_id, nranks, rank, device);
}

void nccl_unique_id(void* out128) {
  ncclUniqueId uid;
  check(nccl().get_unique_id(&uid), "ncclGetUniqueId");
  std::memcpy(out128, &uid, sizeof uid);
}

}  // namespace dp
