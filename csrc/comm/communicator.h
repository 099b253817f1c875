// Host-side communicator of b200ar: CUDA-IPC buffer registry, rank-data arena,
// double-buffered workspace, graph-capture buffer registration, status/timeout
// handling and kernel dispatch.
//
// Counterpart of the reference's `class PCIeAllreduce`
// (pcie_allreduce/pcie_allreduce.cu:278-482). The registry keeps the
// reference's two-phase graph protocol (get_graph_buffer_ipc_meta /
// register_graph_buffers, cu:327-341 and cu:376-398) and its arena bump
// allocator (cu:293, 343-346), but:
//  * the double-buffer slot is chosen on the device (generation counter), so the
//    staged fast paths also work inside CUDA graphs;
//  * every variant checks the slot capacity it needs (cu:420-446 did not for pull);
//  * barriers are bounded; a timeout is reported through a host-mapped status
//    record and turns into a CommTimeout exception on the next host call.
#pragma once

#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

#include "../common/check.h"
#include "../common/layout.h"
#include "arena.h"

namespace b200ar {

// Process-wide cache of opened CUDA IPC handles with reference counts.
// Opening the same handle twice returns the same mapping; the mapping is closed
// when the last holder releases it (the reference never closed script-opened
// handles, cuda_ipc.py has no close; its class closed only graph handles,
// pcie_allreduce.cu:479-481).
class IpcRegistry {
 public:
  static IpcRegistry& get();
  char* open(const std::string& handle);
  void release(char* ptr);
  int64_t open_count() const;

 private:
  struct Entry {
    char* ptr;
    int64_t refs;
  };
  std::map<std::string, Entry> by_handle_;
  std::map<char*, std::string> by_ptr_;
};

// Device allocation helpers (cudaMalloc-backed so that cudaIpcGetMemHandle works).
void* ipc_malloc(int64_t bytes);
void ipc_free(void* p);
std::string ipc_get_handle(const void* p);
// Start and size of the allocation that contains `p`.
std::pair<void*, int64_t> allocation_range(const void* p);

struct RankData;
struct CommCtx;
class NvlsBuffer;

// One entry of the size-based selector: messages of at most `max_bytes` use
// `variant` with `ctas` CTAs (0 = derive from size).
struct SelectorEntry {
  int64_t max_bytes;
  int variant;
  int ctas;
};

// CTA count of a collective launch: `requested` (> 0) or one derived from the
// size, never above `resident` (the CTAs of that kernel that fit on the device
// at once; ranks wait on each other's CTAs, so all of them must run together)
// nor kMaxCTAs. 0 for variants that are not barrier kernels (copy, NCCL).
int plan_ctas(int variant, int64_t bytes, int world, int requested, int resident);

constexpr int kNumVariants = 10;

struct LaunchInfo {
  int variant = kAuto;
  int ctas = 0;
  int threads = 0;
};

class Communicator {
 public:
  // `signals[i]` is rank i's Signal block as mapped in this process
  // (signals[rank] is local). `rank_data`/`rank_data_bytes` is device memory
  // used as the RankData arena.
  Communicator(const std::vector<int64_t>& signals, void* rank_data, int64_t rank_data_bytes, int rank);
  ~Communicator();

  Communicator(const Communicator&) = delete;
  Communicator& operator=(const Communicator&) = delete;

  int rank() const { return rank_; }
  int world() const { return world_; }

  // --- IPC registry -------------------------------------------------------
  // Opens (through the process-wide IpcRegistry, so at most once per process)
  // a peer's cudaIpcMemHandle_t given as raw bytes; released in the destructor.
  char* open_ipc_handle(const std::string& handle);

  // Registers the two double-buffer slot sets (ptrs0[i]/ptrs1[i] = rank i's
  // slot buffer) with `capacity` bytes per slot. capacity == 0 means "query the
  // allocation size of this rank's buffers".
  void register_slots(const std::vector<int64_t>& ptrs0, const std::vector<int64_t>& ptrs1, int64_t capacity);

  // Registers the Lamport regions (ptrs[i] = rank i's region of
  // lamport_bytes(cap, world) bytes) and fills this rank's region with the
  // marker. Every rank must finish this before any rank uses kLamport.
  void register_lamport(const std::vector<int64_t>& ptrs, int64_t cap);
  int64_t lamport_capacity() const { return lam_cap_; }
  char* lamport_ptr(int r) const { return lam_[r]; }

  // Registers a static user buffer: ptrs[i] = rank i's copy (already mapped).
  void register_buffer(const std::vector<int64_t>& ptrs);

  // Graph-capture protocol: export IPC handles of the inputs recorded during
  // capture, then import every rank's handles and fill the reserved arena slots.
  std::pair<std::string, std::vector<int64_t>> graph_buffer_meta() const;
  void register_graph_buffers(const std::vector<std::string>& handles,
                              const std::vector<std::vector<int64_t>>& offsets);
  int64_t pending_graph_buffers() const { return static_cast<int64_t>(graph_pending_.size()); }

  // --- NVLS ---------------------------------------------------------------------
  // Attaches a mapped multicast buffer (not owned); variant kNvls then runs the
  // switch-reduction kernel for messages that fit it.
  void set_nvls(NvlsBuffer* b) { nvls_ = b; }
  bool has_nvls() const { return nvls_ != nullptr; }

  // --- configuration -------------------------------------------------------
  void set_timeout_ns(uint64_t ns) { timeout_ns_ = ns; }
  uint64_t timeout_ns() const { return timeout_ns_; }
  void set_selector(const std::vector<SelectorEntry>& table) { selector_ = table; }
  const std::vector<SelectorEntry>& selector() const { return selector_; }
  int64_t slot_capacity() const { return slot_cap_; }
  bool slots_registered() const { return slots_ok_; }

  // --- collectives ----------------------------------------------------------
  // Sum all-reduce of `bytes` bytes (multiple of 16) from `in` to `out` on
  // `stream`. `variant` kAuto consults the selector. Returns the variant that
  // was launched, or kNccl when the caller must fall back to NCCL.
  LaunchInfo allreduce(cudaStream_t stream, const void* in, void* out, int64_t bytes, DType dt, int variant,
                       int ctas);

  // Picks variant and CTA count for a message (pure function of inputs, so
  // identical on every rank).
  LaunchInfo plan(int64_t bytes, int variant, int ctas, bool capturing, bool registered_input) const;

  // CTAs of `variant`'s kernel that can be resident on this device at once
  // (occupancy x SM count, smallest over dtypes; cached).
  int resident_ctas(int variant) const;

  // --- status ----------------------------------------------------------------
  // Throws CommTimeout if a kernel recorded an error.
  void check_status() const;
  Status status() const;
  // Clears the status record and zeroes this rank's signal block (the caller
  // must make every rank do this between two host barriers).
  void reset(cudaStream_t stream);
  uint64_t launches() const { return launches_; }

  // Device-side context for kernels of other translation units (nvcc only).
  void fill_ctx(CommCtx* c) const;
  Signal* self_signal() const { return signals_[rank_]; }
  Signal* signal(int i) const { return signals_[i]; }
  Status* device_status() const { return status_dev_; }
  char* slot_ptr(int slot, int r) const { return slots_[slot][r]; }

 private:
  int rank_ = 0;
  int world_ = 0;
  Signal* signals_[kMaxRanks] = {};
  RankDataArena arena_;

  std::unordered_map<const void*, RankData*> buffers_;
  std::vector<const void*> graph_pending_;
  std::vector<char*> opened_;  // IPC mappings this communicator holds

  char* slots_[2][kMaxRanks] = {};
  int64_t slot_cap_ = 0;
  bool slots_ok_ = false;

  Status* status_host_ = nullptr;
  Status* status_dev_ = nullptr;
  uint64_t timeout_ns_ = 2000000000ull;
  std::vector<SelectorEntry> selector_;
  uint64_t launches_ = 0;
  NvlsBuffer* nvls_ = nullptr;
  mutable int resident_[kNumVariants] = {};
  char* lam_[kMaxRanks] = {};
  int64_t lam_cap_ = 0;

 public:
  // Counts a kernel launched on behalf of this communicator (fused ops too).
  void count_launch() { ++launches_; }
};

}  // namespace b200ar
