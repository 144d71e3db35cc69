// Host-side failure detection for collectives in flight: instead of blocking
// in a stream synchronisation that never returns when a peer rank has stopped
// (its NCCL kernels wait for it forever), the host polls for completion, for
// an asynchronous error of the communicator, and for a deadline.  An error or
// the deadline aborts the communicator, which ends its kernels on every
// stream, and the caller turns the returned reason into an exception.
//
// Plain C++ (no CUDA types), so that the polling logic is tested on a host
// without a GPU against fake completion, error and abort functions.
#pragma once
#include <chrono>
#include <cstdint>
#include <string>
#include <thread>

namespace dp {

// done() -> bool: the awaited work has completed.
// error() -> std::string: an asynchronous failure ("" while there is none).
// abort(): called at most once, before a non-empty return.
// timeout_ms <= 0 waits without a deadline.  The first spin_us of the wait
// poll back to back, as a spinning stream synchronisation would, so that a
// healthy round (a few milliseconds) returns as soon as it ends; later polls
// sleep poll_us.
// Returns "" on completion, otherwise the reason the wait was given up.
template <class Done, class Error, class Abort>
std::string wait_or_abort(Done&& done, Error&& error, Abort&& abort, std::int64_t timeout_ms,
                          std::int64_t spin_us = 50000, std::int64_t poll_us = 100) {
  using clock = std::chrono::steady_clock;
  const auto t0 = clock::now();
  for (;;) {
    if (done()) return std::string();
    std::string e = error();
    if (!e.empty()) {
      abort();
      return "asynchronous communicator error: " + e;
    }
    const auto waited = std::chrono::duration_cast<std::chrono::microseconds>(clock::now() - t0).count();
    if (timeout_ms > 0 && waited >= timeout_ms * 1000) {
      abort();
      return "no completion within " + std::to_string(timeout_ms) + " ms (a peer rank stopped or is stalled)";
    }
    if (waited >= spin_us) std::this_thread::sleep_for(std::chrono::microseconds(poll_us));
  }
}

}  // namespace dp
