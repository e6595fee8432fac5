// Env-gated slow-path diagnostics (reference csrc/common/slow_path_diagnostics.h:
// 12-72, gated there by PD_SERVING_PERF).  When LMC_PERF is set, a scope that
// takes at least LMC_PERF_MIN_MS milliseconds (default 100) prints one JSON
// line `[LMCACHE_SLOW_PATH] {...}` with wall and CPU time to stderr.
#pragma once

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <ctime>

namespace lmc {

inline bool slow_path_enabled() {
  static const bool on = std::getenv("LMC_PERF") != nullptr;
  return on;
}

inline double slow_path_min_ms() {
  static const double v = [] {
    const char *s = std::getenv("LMC_PERF_MIN_MS");
    return s ? std::atof(s) : 100.0;
  }();
  return v;
}

class SlowPathScope {
 public:
  SlowPathScope(const char *what, long long bytes)
      : what_(what), bytes_(bytes), on_(slow_path_enabled()) {
    if (on_) {
      t0_ = std::chrono::steady_clock::now();
      c0_ = std::clock();
    }
  }
  ~SlowPathScope() {
    if (!on_) return;
    const double wall_ms = std::chrono::duration<double, std::milli>(
                               std::chrono::steady_clock::now() - t0_)
                               .count();
    const double cpu_ms = 1000.0 * double(std::clock() - c0_) / CLOCKS_PER_SEC;
    if (wall_ms >= slow_path_min_ms())
      std::fprintf(stderr,
                   "[LMCACHE_SLOW_PATH] {\"what\": \"%s\", \"bytes\": %lld, "
                   "\"wall_ms\": %.3f, \"cpu_ms\": %.3f}\n",
                   what_, bytes_, wall_ms, cpu_ms);
  }

 private:
  const char *what_;
  long long bytes_;
  bool on_;
  std::chrono::steady_clock::time_point t0_;
  std::clock_t c0_ = 0;
};

}  // namespace lmc
