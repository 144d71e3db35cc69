// Shared host-side helpers of libdp_gbdt: errors, CUDA checks, device guard,
// launch accounting.
#pragma once
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <atomic>
#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

namespace dp {

using u8 = std::uint8_t;
using u16 = std::uint16_t;
using u32 = std::uint32_t;
using u64 = std::uint64_t;
using i32 = std::int32_t;
using i64 = std::int64_t;

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

[[noreturn]] inline void fail(const std::string& msg) { throw Error(msg); }
// Sets the thread-local message returned by XGBGetLastError (defined beside it).
void set_last_error(const std::string& msg);
inline void need(bool ok, const std::string& msg) {
  if (!ok) fail(msg);
}

inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(std::string(what) + ": " + cudaGetErrorString(e));
}
#define DP_CUDA(expr) ::dp::cuda_check((expr), #expr)

// Count of kernels launched by this library in this process (a statistic the
// benchmark reports; kernel launches never read it).
std::atomic<u64>& launch_counter();
inline void count_launch(u64 n = 1) { launch_counter().fetch_add(n, std::memory_order_relaxed); }

// NVTX range for the duration of a scope (what a system profiler shows for
// the host side of rounds, levels and decodes; no cost without a profiler).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
// Checks the launch that was just issued and counts it.
inline void after_launch(const char* what) {
  cuda_check(cudaGetLastError(), what);
  count_launch();
}

// Makes `device` current for the scope and restores the caller's device.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    DP_CUDA(cudaGetDevice(&prev_));
    if (prev_ != device) DP_CUDA(cudaSetDevice(device));
    dev_ = device;
  }
  ~DeviceGuard() {
    if (prev_ != dev_) cudaSetDevice(prev_);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;

 private:
  int prev_ = 0, dev_ = 0;
};

// Device buffer: an owned allocation, or a view into a slab (see SlabPlan)
// that it never frees.  Stream-ordered frees are not needed: every owner
// synchronises its stream before it is destroyed.
template <class T>
class DevBuf {
 public:
  DevBuf() = default;
  explicit DevBuf(size_t n) { resize(n); }
  ~DevBuf() { release(); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p_(o.p_), n_(o.n_), owned_(o.owned_) { o.p_ = nullptr; o.n_ = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) {
      release();
      p_ = o.p_;
      n_ = o.n_;
      owned_ = o.owned_;
      o.p_ = nullptr;
      o.n_ = 0;
    }
    return *this;
  }
  void resize(size_t n) {
    if (n == n_) return;
    release();
    if (n) DP_CUDA(cudaMalloc(&p_, n * sizeof(T)));
    n_ = n;
    owned_ = true;
  }
  // Grows (never shrinks) the capacity; contents are not preserved.
  void reserve(size_t n) {
    if (n > n_) resize(n);
  }
  // Becomes a view of n elements at p (memory owned elsewhere).
  void adopt(T* p, size_t n) {
    release();
    p_ = p;
    n_ = n;
    owned_ = false;
  }
  void release() {
    if (p_ && owned_) cudaFree(p_);
    p_ = nullptr;
    n_ = 0;
    owned_ = true;
  }
  T* get() const { return p_; }
  size_t size() const { return n_; }

 private:
  T* p_ = nullptr;
  size_t n_ = 0;
  bool owned_ = true;
};

// Places several buffers in one device allocation: on this class of GPU a
// cudaMalloc or cudaFree costs about half a millisecond whatever its size.
// want() records a buffer that must hold n elements (ignored when it already
// does); commit() allocates the slab, appends it to `slabs` (which must
// outlive the views) and turns every recorded buffer into a view of it,
// 256-byte aligned.
class SlabPlan {
 public:
  template <class T>
  void want(DevBuf<T>& b, size_t n) {
    if (n <= b.size()) return;
    const size_t off = (bytes_ + 255) & ~size_t(255);
    bytes_ = off + n * sizeof(T);
    DevBuf<T>* bp = &b;
    binds_.push_back([bp, off, n](unsigned char* base) { bp->adopt(reinterpret_cast<T*>(base + off), n); });
  }
  void commit(std::vector<DevBuf<unsigned char>>& slabs) {
    if (binds_.empty()) return;
    slabs.emplace_back(bytes_);
    unsigned char* base = slabs.back().get();
    for (auto& f : binds_) f(base);
    binds_.clear();
    bytes_ = 0;
  }
  size_t bytes() const { return bytes_; }

 private:
  size_t bytes_ = 0;
  std::vector<std::function<void(unsigned char*)>> binds_;
};

// Owned pinned host staging buffer.
template <class T>
class PinnedBuf {
 public:
  PinnedBuf() = default;
  ~PinnedBuf() { if (p_) cudaFreeHost(p_); }
  PinnedBuf(const PinnedBuf&) = delete;
  PinnedBuf& operator=(const PinnedBuf&) = delete;
  void reserve(size_t n) {
    if (n <= n_) return;
    if (p_) cudaFreeHost(p_);
    p_ = nullptr;
    DP_CUDA(cudaMallocHost(&p_, n * sizeof(T)));
    n_ = n;
  }
  void swap(PinnedBuf& o) noexcept {
    T* p = p_; p_ = o.p_; o.p_ = p;
    size_t n = n_; n_ = o.n_; o.n_ = n;
  }
  T* get() const { return p_; }
  T& operator[](size_t i) const { return p_[i]; }
  size_t size() const { return n_; }

 private:
  T* p_ = nullptr;
  size_t n_ = 0;
};

}  // namespace dp
