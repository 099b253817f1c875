// CPU emulation of the b200ar data plane over POSIX shared memory.
//
// Each rank maps one shared-memory segment per rank with exactly the GPU
// workspace layout (layout.h: Signal block, then two slots). The one-shot push,
// one-shot pull and two-shot algorithms run with the same per-CTA partitioning,
// the same generation/epoch arithmetic and the same release/acquire flag
// protocol as the sm_100a kernels; "CTAs" are executed one after the other by
// the calling thread. Bootstrap (segment names) goes through torch.distributed
// (gloo) in the Python layer.
//
// The reference has no CPU path at all (its tests need GPUs with P2P,
// test_pcie_ar.py, stress_test.py); this backend lets the protocol, the
// double-buffer slot logic and the timeout path be tested without a GPU.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "../common/layout.h"

namespace b200ar {

class ShmComm {
 public:
  // Creates (and zeroes) this rank's segment `<prefix>-r<rank>`. With
  // lamport_capacity > 0 the segment also holds the Lamport buffers
  // (layout.h), filled with the marker.
  ShmComm(const std::string& prefix, int rank, int world, int64_t slot_capacity, int64_t lamport_capacity = 0);
  ~ShmComm();
  ShmComm(const ShmComm&) = delete;
  ShmComm& operator=(const ShmComm&) = delete;

  const std::string& segment_name() const { return names_[rank_]; }
  // Maps every rank's segment; names[i] is rank i's segment name.
  void connect(const std::vector<std::string>& names);

  // Sum all-reduce of `bytes` bytes (multiple of 16) with `ctas` emulated CTAs.
  // Throws CommTimeout when a peer does not arrive within the timeout.
  void allreduce(const void* in, void* out, int64_t bytes, DType dt, int variant, int ctas);

  void set_timeout_ms(int64_t ms) { timeout_ms_ = ms; }
  int64_t slot_capacity() const { return cap_; }
  int64_t lamport_capacity() const { return lam_cap_; }
  const Status& status() const { return status_; }
  uint32_t generation() const;
  // Zeroes this rank's signal block and clears the status (call collectively).
  void reset();
  // Skips the next `n` calls' barriers on this rank (host-side fault injection
  // for tests: the peers must time out).
  void inject_skip(int n) { skip_ = n; }
  // Overwrites flags[cta][src] of this rank's own signal block with `value`
  // (host-side fault injection for tests: a stale or foreign epoch).
  void inject_flag(int cta, int src, uint32_t value);

 private:
  bool barrier(int cta, uint32_t epoch);
  template <typename T>
  void run_lamport(const char* in, char* out, int64_t packets, int ctas);
  template <typename T>
  void run(const char* in, char* out, int64_t packets, int variant, int ctas);

  int rank_;
  int world_;
  int64_t cap_;
  int64_t lam_cap_ = 0;
  int64_t seg_bytes_;
  std::vector<std::string> names_;
  std::vector<char*> base_;  // mapped segment of every rank
  int64_t timeout_ms_ = 2000;
  Status status_{};
  int skip_ = 0;
  bool owner_unlinked_ = false;
};

}  // namespace b200ar
