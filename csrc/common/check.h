// Host-side error checking shared by every native source of b200ar.
//
// Equivalent of the reference's CHECK_CUDA_SUCCESS macro
// (pcie_allreduce/pcie_allreduce.cu:31-40): a failing CUDA runtime call throws
// std::runtime_error carrying the call text, the CUDA error string and file:line.
// b200ar adds a distinct exception type for communicator timeouts so that the
// Python layer can map it to its own CommTimeoutError.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <sstream>
#include <stdexcept>
#include <string>

namespace b200ar {

struct CommTimeout : public std::runtime_error {
  using std::runtime_error::runtime_error;
};

[[noreturn]] inline void throw_cuda(cudaError_t e, const char* what, const char* file, int line) {
  std::ostringstream os;
  os << what << " failed: " << cudaGetErrorString(e) << " (" << static_cast<int>(e) << ") at " << file << ':'
     << line;
  throw std::runtime_error(os.str());
}

}  // namespace b200ar

#define B200AR_CUDA(cmd)                                              \
  do {                                                                \
    cudaError_t b200ar_err__ = (cmd);                                 \
    if (b200ar_err__ != cudaSuccess) {                                \
      ::b200ar::throw_cuda(b200ar_err__, #cmd, __FILE__, __LINE__);   \
    }                                                                 \
  } while (0)

#define B200AR_CHECK(cond, msg)                                       \
  do {                                                                \
    if (!(cond)) {                                                    \
      std::ostringstream b200ar_os__;                                 \
      b200ar_os__ << msg << " [" << __FILE__ << ':' << __LINE__ << ']'; \
      throw std::invalid_argument(b200ar_os__.str());                 \
    }                                                                 \
  } while (0)

namespace b200ar {

// Runs a set-up step once per CUDA device (devices 0-63), e.g. raising a
// kernel's dynamic shared-memory limit with cudaFuncSetAttribute, which is a
// per-device attribute: a process that drives several GPUs needs it on each.
// Two threads may both run the step for one device; the steps used here are
// idempotent.
class PerDeviceOnce {
 public:
  template <typename Fn>
  void operator()(Fn&& fn) {
    int dev = 0;
    B200AR_CUDA(cudaGetDevice(&dev));
    const uint64_t bit = 1ull << (static_cast<unsigned>(dev) & 63u);
    if (done_.load(std::memory_order_acquire) & bit) return;
    fn();
    done_.fetch_or(bit, std::memory_order_acq_rel);
  }

 private:
  std::atomic<uint64_t> done_{0};
};

}  // namespace b200ar
