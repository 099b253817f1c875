// Optional NVTX ranges around b200ar host entry points (enable with
// B200AR_NVTX=1; off by default so the hot path pays one branch).
#pragma once

#include <nvtx3/nvToolsExt.h>

#include <cstdlib>

namespace b200ar {

inline bool nvtx_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("B200AR_NVTX");
    return v != nullptr && v[0] == '1';
  }();
  return on;
}

class TraceRange {
 public:
  explicit TraceRange(const char* name) : on_(nvtx_enabled()) {
    if (on_) nvtxRangePushA(name);
  }
  ~TraceRange() {
    if (on_) nvtxRangePop();
  }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;

 private:
  bool on_;
};

}  // namespace b200ar
