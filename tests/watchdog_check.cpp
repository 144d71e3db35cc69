// Test driver (host only, no GPU) of dp::wait_or_abort, the polling wait that
// replaces a blocking stream synchronisation while collectives are in flight.
// Each case prints one JSON object: the returned reason, how often abort()
// ran, how many polls happened and the milliseconds waited.
#include <chrono>
#include <cstdio>
#include <string>

#include "watchdog.h"

namespace {

struct Result {
  std::string reason;
  int aborts = 0;
  int polls = 0;
  double ms = 0;
};

void print(const char* name, const Result& r) {
  std::printf("{\"case\": \"%s\", \"reason\": \"%s\", \"aborts\": %d, \"polls\": %d, \"ms\": %.3f}\n", name,
              r.reason.c_str(), r.aborts, r.polls, r.ms);
}

// done_after: completion on that poll (< 0: never); error_at: the error
// appears on that poll (< 0: never); done_after_ms: completion after that
// much time (< 0: unused).
Result run(int done_after, int error_at, long long timeout_ms, double done_after_ms = -1) {
  Result r;
  const auto t0 = std::chrono::steady_clock::now();
  auto ms = [&] { return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count(); };
  r.reason = dp::wait_or_abort(
      [&] {
        ++r.polls;
        if (r.aborts) return true;  // must not be asked again after an abort
        if (done_after >= 0 && r.polls >= done_after) return true;
        return done_after_ms >= 0 && ms() >= done_after_ms;
      },
      [&]() -> std::string { return (error_at >= 0 && r.polls >= error_at) ? "remote process exited" : ""; },
      [&] { ++r.aborts; }, timeout_ms, 500, 50);
  r.ms = ms();
  return r;
}

}  // namespace

int main() {
  print("completes", run(5, -1, 1000));
  print("error", run(-1, 3, 1000));
  print("timeout", run(-1, -1, 20));
  print("no_deadline", run(-1, -1, 0, 50.0));
  print("done_before_error", run(3, 3, 1000));
  return 0;
}
