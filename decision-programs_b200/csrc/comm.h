// Collective interface used by the training path when rows are sharded over
// several GPUs (one process per GPU).  The reference is single-GPU
// (native/class_model_train.cu:42); the exchange steps the sharded path needs
// are sums of integer counts, maxima of floats, a reduce-scatter of integer
// histograms over feature groups and an all-gather of split candidates.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>

namespace dp {

class Comm {
 public:
  virtual ~Comm() = default;
  virtual int rank() const = 0;
  virtual int size() const = 0;
  // In-place element-wise sums / maxima over all ranks, stream ordered.
  virtual void sum_u32(std::uint32_t* d, size_t n, cudaStream_t s) = 0;
  virtual void sum_i64(std::int64_t* d, size_t n, cudaStream_t s) = 0;
  virtual void max_u32(std::uint32_t* d, size_t n, cudaStream_t s) = 0;
  // recv[0, recv_n) = the element-wise sum over ranks of this rank's block
  // send[rank * recv_n, (rank + 1) * recv_n); send holds size() blocks.
  virtual void reduce_scatter_i64(const std::int64_t* send, std::int64_t* recv, size_t recv_n, cudaStream_t s) = 0;
  // recv[r * bytes, (r + 1) * bytes) = rank r's send[0, bytes).
  virtual void all_gather_bytes(const void* send, void* recv, size_t bytes, cudaStream_t s) = 0;
  // Host scalar helpers (synchronous).
  virtual std::uint64_t sum_host_u64(std::uint64_t v, cudaStream_t s) = 0;
  // Waits until stream s has drained.  A communicator error, or no completion
  // within the timeout, aborts the communicator (its kernels in flight end on
  // every stream; later calls fail) and throws std::runtime_error.
  // before_abort runs just before the abort: it must release every CUDA graph
  // that holds this communicator's calls, because NCCL's abort waits until
  // those graphs are gone (a graph still in flight is freed when it ends).
  virtual void wait(cudaStream_t s, const std::function<void()>& before_abort) = 0;
  // Deadline of wait() in milliseconds; <= 0 waits without one.  The default
  // is DP_COMM_TIMEOUT_MS from the environment, else 600000 (ten minutes).
  virtual void set_timeout_ms(std::int64_t ms) = 0;
};

// NCCL communicator over NVLink (libnccl.so.2 loaded with dlopen so that a
// single-GPU caller never needs it).  `unique_id` is the 128-byte
// ncclUniqueId produced by dp_comm_unique_id on rank 0.
Comm* make_nccl_comm(const void* unique_id, int nranks, int rank, int device);
// Fills 128 bytes of a fresh ncclUniqueId.
void nccl_unique_id(void* out128);

}  // namespace dp
