// Shared host-side helpers of libdp_gbdt: errors, CUDA checks, device guard,
// launch accounting.
#pragma once
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <locale.h>
#include <stdlib.h>

#include <atomic>
#include <cstdlib>
#include <cstdint>
#include <functional>
#include <mutex>
#include <utility>
#include <stdexcept>
#include <string>
#include <string_view>
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
// strtod in the "C" locale whatever the process's LC_NUMERIC: JSON and the
// parameter strings always write the decimal point as '.', and a caller that
// set a locale with a decimal comma must not change how they read.
inline double strtod_c(const char* s, char** end) {
  static const locale_t c_numeric = newlocale(LC_NUMERIC_MASK, "C", locale_t(0));
  return c_numeric ? strtod_l(s, end, c_numeric) : std::strtod(s, end);
}
// Caller-supplied text quoted in an error message, as printable ASCII (other
// bytes as \xHH), so that the message stays plain text whatever was passed.
inline std::string printable(std::string_view s) {
  static const char kHex[] = "0123456789abcdef";
  std::string o;
  for (const char ch : s) {
    const unsigned char c = static_cast<unsigned char>(ch);
    if (c >= 0x20 && c < 0x7f) {
      o.push_back(ch);
    } else {
      o += "\\x";
      o.push_back(kHex[c >> 4]);
      o.push_back(kHex[c & 15]);
    }
  }
  return o;
}
// Sets the thread-local message returned by XGBGetLastError (defined beside it).
void set_last_error(const std::string& msg);
inline void need(bool ok, const std::string& msg) {
  if (!ok) fail(msg);
}
// A literal message is turned into a string only when the check fails (the
// parser and the model reader call this per array element).
inline void need(bool ok, const char* msg) {
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
  // Owns p (n elements, from cudaMalloc) from now on.
  void take_ownership(T* p, size_t n) {
    release();
    p_ = p;
    n_ = n;
    owned_ = true;
  }
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
  // With device >= 0 (the current device) the slab may come from SlabCache.
  void commit(std::vector<DevBuf<unsigned char>>& slabs, int device = -1);
  size_t bytes() const { return bytes_; }

 private:
  size_t bytes_ = 0;
  std::vector<std::function<void(unsigned char*)>> binds_;
};

// Process-wide cache of freed device slabs, for the matrices and engines of
// jobs that come and go in one process (a hyper-parameter search or
// out-of-fold fits create a booster per fit, and repeated jobs a matrix per
// job): cudaMalloc of a slab costs milliseconds and cudaFree waits for the
// whole device.  A freed slab stays allocated until a later request reuses it
// (the smallest cached slab of the device that holds at least what is asked
// for and at most twice that), the cache drops it (it keeps at most kMaxSlabs
// slabs, and at most half of a device's memory, dropping the oldest first),
// an allocation fails (the device's cached slabs are freed and the allocation
// retried), or release_all() (dp_release_cached_memory) frees everything.
// A slab is handed back only when no work on it is in flight.
class SlabCache {
 public:
  static constexpr size_t kMaxSlabs = 4;

  static DevBuf<unsigned char> take(int device, size_t bytes) {
    DevBuf<unsigned char> out;
    {
      std::lock_guard<std::mutex> lock(mu());
      auto& c = slots();
      size_t best = c.size();
      for (size_t i = 0; i < c.size(); ++i) {
        const size_t sz = c[i].second.size();
        if (c[i].first == device && sz >= bytes && sz <= 2 * bytes && (best == c.size() || sz < c[best].second.size()))
          best = i;
      }
      if (best < c.size()) {
        out = std::move(c[best].second);
        c.erase(c.begin() + std::ptrdiff_t(best));
      }
    }
    if (!out.get()) {
      if (cudaMalloc_fits(out, bytes)) return out;
      release_device(device);
      out.resize(bytes);
    }
    return out;
  }

  static void give(int device, DevBuf<unsigned char>&& slab) {
    if (!slab.get()) return;
    const size_t total = device_memory(device);
    std::lock_guard<std::mutex> lock(mu());
    auto& c = slots();
    c.emplace_back(device, std::move(slab));
    auto device_bytes = [&] {
      size_t n = 0;
      for (auto& e : c)
        if (e.first == device) n += e.second.size();
      return n;
    };
    while (c.size() > kMaxSlabs || (total && device_bytes() > total / 2)) {
      size_t drop = 0;  // the oldest (of this device when over its share)
      if (c.size() <= kMaxSlabs)
        while (c[drop].first != device) ++drop;
      c.erase(c.begin() + std::ptrdiff_t(drop));
    }
  }

  static void release_all() {
    std::lock_guard<std::mutex> lock(mu());
    slots().clear();
  }

 private:
  // One allocation attempt; false (error state cleared) when the device is out of memory.
  static bool cudaMalloc_fits(DevBuf<unsigned char>& out, size_t bytes) {
    unsigned char* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) {
      out.take_ownership(p, bytes);
      return true;
    }
    cudaGetLastError();
    if (e != cudaErrorMemoryAllocation) DP_CUDA(e);
    return false;
  }
  // Total memory of a device (0 if unknown), looked up once per device.
  static size_t device_memory(int device) {
    static std::mutex m;
    static std::vector<size_t> known;
    std::lock_guard<std::mutex> lock(m);
    if (device < 0) return 0;
    if (size_t(device) >= known.size()) known.resize(size_t(device) + 1, ~size_t(0));
    if (known[device] == ~size_t(0)) {
      cudaDeviceProp prop{};
      known[device] = cudaGetDeviceProperties(&prop, device) == cudaSuccess ? prop.totalGlobalMem : 0;
    }
    return known[device];
  }
  static void release_device(int device) {
    std::lock_guard<std::mutex> lock(mu());
    auto& c = slots();
    for (size_t i = c.size(); i-- > 0;)
      if (c[i].first == device) c.erase(c.begin() + std::ptrdiff_t(i));
  }
  static std::mutex& mu() {
    static std::mutex m;
    return m;
  }
  static std::vector<std::pair<int, DevBuf<unsigned char>>>& slots() {
    static auto* c = new std::vector<std::pair<int, DevBuf<unsigned char>>>();  // outlives static destruction
    return *c;
  }
};

inline void SlabPlan::commit(std::vector<DevBuf<unsigned char>>& slabs, int device) {
  if (binds_.empty()) return;
  if (device >= 0) slabs.push_back(SlabCache::take(device, bytes_));
  else slabs.emplace_back(bytes_);
  unsigned char* base = slabs.back().get();
  for (auto& f : binds_) f(base);
  binds_.clear();
  bytes_ = 0;
}

// Process-wide cache of pinned host blocks.  cudaMallocHost costs about a
// millisecond and cudaFreeHost waits for the whole device, so the staging
// buffers of engines that come and go (a booster per fit in a
// hyper-parameter search) reuse the blocks of engines already freed.  A
// bounded number of blocks up to kMaxBytes each is kept; anything else is
// freed.  Cached blocks are never handed to two owners at once.
class PinnedCache {
 public:
  static constexpr size_t kMaxBlocks = 8, kMaxBytes = size_t(64) << 20;
  // A block of at least `bytes`, and its actual size.
  static void* take(size_t bytes, size_t* got) {
    {
      std::lock_guard<std::mutex> lock(mu());
      auto& f = free_list();
      size_t best = f.size();
      for (size_t i = 0; i < f.size(); ++i)
        if (f[i].second >= bytes && (best == f.size() || f[i].second < f[best].second)) best = i;
      if (best < f.size()) {
        void* p = f[best].first;
        *got = f[best].second;
        f.erase(f.begin() + long(best));
        return p;
      }
    }
    void* p = nullptr;
    DP_CUDA(cudaMallocHost(&p, bytes));
    *got = bytes;
    return p;
  }
  static void give(void* p, size_t bytes) {
    if (!p) return;
    if (bytes <= kMaxBytes) {
      std::lock_guard<std::mutex> lock(mu());
      auto& f = free_list();
      if (f.size() < kMaxBlocks) {
        f.emplace_back(p, bytes);
        return;
      }
    }
    cudaFreeHost(p);
  }

 private:
  static std::mutex& mu() {
    static std::mutex m;
    return m;
  }
  static std::vector<std::pair<void*, size_t>>& free_list() {
    static auto* f = new std::vector<std::pair<void*, size_t>>();  // outlives static destruction
    return *f;
  }
};

// Owned pinned host staging buffer (blocks from PinnedCache).
template <class T>
class PinnedBuf {
 public:
  PinnedBuf() = default;
  ~PinnedBuf() { PinnedCache::give(p_, n_ * sizeof(T)); }
  PinnedBuf(const PinnedBuf&) = delete;
  PinnedBuf& operator=(const PinnedBuf&) = delete;
  void reserve(size_t n) {
    if (n <= n_) return;
    PinnedCache::give(p_, n_ * sizeof(T));
    p_ = nullptr;
    n_ = 0;
    size_t got = 0;
    p_ = static_cast<T*>(PinnedCache::take(n * sizeof(T), &got));
    n_ = got / sizeof(T);
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
