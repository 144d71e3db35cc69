// Collective interface used by the training path when rows are sharded over
// several GPUs (one process per GPU).  The reference is single-GPU
// (native/class_model_train.cu:42); the only exchange steps the sharded path
// needs are sums of integer count / histogram arrays and maxima of floats.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
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
  // Host scalar helpers (synchronous).
  virtual std::uint64_t sum_host_u64(std::uint64_t v, cudaStream_t s) = 0;
};

// NCCL communicator over NVLink (libnccl.so.2 loaded with dlopen so that a
// single-GPU caller never needs it).  `unique_id` is the 128-byte
// ncclUniqueId produced by dp_comm_unique_id on rank 0.
Comm* make_nccl_comm(const void* unique_id, int nranks, int rank, int device);
// Fills 128 bytes of a fresh ncclUniqueId.
void nccl_unique_id(void* out128);

}  // namespace dp
