// Host communicator implementation (see communicator.h).
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "ar_kernels.cuh"
#include "communicator.h"
#include "../common/trace.h"
#include "../nvls/nvls.h"

namespace b200ar {

namespace {

std::mutex g_ipc_mu;

using MemRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

MemRangeFn get_mem_range_fn() {
  static MemRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    B200AR_CUDA(cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuMemGetAddressRange is not available from the driver");
    return reinterpret_cast<MemRangeFn>(p);
  }();
  return fn;
}

constexpr size_t kIpcHandleBytes = sizeof(cudaIpcMemHandle_t);

}  // namespace

// ---------------------------------------------------------------------------
// IPC helpers
// ---------------------------------------------------------------------------

IpcRegistry& IpcRegistry::get() {
  static IpcRegistry* r = new IpcRegistry();  // never destroyed: the CUDA context may be gone at exit
  return *r;
}

char* IpcRegistry::open(const std::string& handle) {
  B200AR_CHECK(handle.size() == kIpcHandleBytes, "IPC handle must be " << kIpcHandleBytes << " bytes, got "
                                                                       << handle.size());
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  auto it = by_handle_.find(handle);
  if (it != by_handle_.end()) {
    ++it->second.refs;
    return it->second.ptr;
  }
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), kIpcHandleBytes);
  void* p = nullptr;
  B200AR_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  by_handle_[handle] = Entry{static_cast<char*>(p), 1};
  by_ptr_[static_cast<char*>(p)] = handle;
  return static_cast<char*>(p);
}

void IpcRegistry::release(char* ptr) {
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  auto it = by_ptr_.find(ptr);
  if (it == by_ptr_.end()) return;
  auto& e = by_handle_[it->second];
  if (--e.refs == 0) {
    cudaIpcCloseMemHandle(ptr);  // best effort during teardown
    by_handle_.erase(it->second);
    by_ptr_.erase(it);
  }
}

int64_t IpcRegistry::open_count() const {
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  return static_cast<int64_t>(by_handle_.size());
}

void* ipc_malloc(int64_t bytes) {
  void* p = nullptr;
  B200AR_CUDA(cudaMalloc(&p, static_cast<size_t>(bytes)));
  B200AR_CUDA(cudaMemset(p, 0, static_cast<size_t>(bytes)));
  return p;
}

void ipc_free(void* p) {
  if (p) B200AR_CUDA(cudaFree(p));
}

std::string ipc_get_handle(const void* p) {
  cudaIpcMemHandle_t h;
  B200AR_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(p)));
  return std::string(reinterpret_cast<const char*>(&h), kIpcHandleBytes);
}

std::pair<void*, int64_t> allocation_range(const void* p) {
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = get_mem_range_fn()(&base, &size, reinterpret_cast<CUdeviceptr>(p));
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuMemGetAddressRange failed with CUresult " + std::to_string(r));
  return {reinterpret_cast<void*>(base), static_cast<int64_t>(size)};
}

// ---------------------------------------------------------------------------
// Communicator
// ---------------------------------------------------------------------------

Communicator::Communicator(const std::vector<int64_t>& signals, void* rank_data, int64_t rank_data_bytes,
                           int rank)
    : rank_(rank), world_(static_cast<int>(signals.size())) {
  B200AR_CHECK(world_ >= 1 && world_ <= kMaxRanks, "world size must be in [1, " << kMaxRanks << "], got " << world_);
  B200AR_CHECK(rank_ >= 0 && rank_ < world_, "invalid rank " << rank_ << " for world size " << world_);
  for (int i = 0; i < world_; ++i) {
    B200AR_CHECK(signals[i] != 0, "null signal pointer for rank " << i);
    B200AR_CHECK(signals[i] % 256 == 0, "signal block of rank " << i << " must be 256-byte aligned");
    signals_[i] = reinterpret_cast<Signal*>(signals[i]);
  }
  arena_ = RankDataArena(rank_data, rank_data_bytes);
  B200AR_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&status_host_), sizeof(Status), cudaHostAllocMapped));
  std::memset(status_host_, 0, sizeof(Status));
  B200AR_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&status_dev_), status_host_, 0));
  // Default selector, replaced by a measured table from the Python layer.
  selector_ = {
      {512 * 1024, kOneshotPush, 0},
      {INT64_MAX, kTwoshot, 0},
  };
}

Communicator::~Communicator() {
  for (char* p : opened_) IpcRegistry::get().release(p);
  if (status_host_) cudaFreeHost(status_host_);
}

char* Communicator::open_ipc_handle(const std::string& handle) {
  char* p = IpcRegistry::get().open(handle);
  opened_.push_back(p);
  return p;
}

void Communicator::register_slots(const std::vector<int64_t>& ptrs0, const std::vector<int64_t>& ptrs1,
                                  int64_t capacity) {
  B200AR_CHECK(static_cast<int>(ptrs0.size()) == world_ && static_cast<int>(ptrs1.size()) == world_,
               "need one slot pointer per rank");
  for (int i = 0; i < world_; ++i) {
    B200AR_CHECK(ptrs0[i] % 16 == 0 && ptrs1[i] % 16 == 0, "slot buffers must be 16-byte aligned");
    slots_[0][i] = reinterpret_cast<char*>(ptrs0[i]);
    slots_[1][i] = reinterpret_cast<char*>(ptrs1[i]);
  }
  if (capacity <= 0) {
    // Unknown capacity: the usable size is what is left of this rank's allocations.
    int64_t cap = INT64_MAX;
    for (int s = 0; s < 2; ++s) {
      auto [base, size] = allocation_range(slots_[s][rank_]);
      cap = std::min<int64_t>(cap, size - (slots_[s][rank_] - static_cast<char*>(base)));
    }
    capacity = cap;
  }
  slot_cap_ = capacity;
  slots_ok_ = true;
  // Static registration of the slot buffers, like the reference (cu:362-363),
  // so that a caller staging into them can use the registered path.
  for (int s = 0; s < 2; ++s) {
    std::vector<int64_t> ptrs(s == 0 ? ptrs0 : ptrs1);
    if (arena_.fits(1)) register_buffer(ptrs);
  }
}

void Communicator::register_lamport(const std::vector<int64_t>& ptrs, int64_t cap) {
  B200AR_CHECK(static_cast<int>(ptrs.size()) == world_, "need one Lamport region per rank");
  B200AR_CHECK(cap > 0 && cap % 16 == 0, "Lamport capacity must be a positive multiple of 16");
  for (int i = 0; i < world_; ++i) {
    B200AR_CHECK(ptrs[i] % 16 == 0, "Lamport regions must be 16-byte aligned");
    lam_[i] = reinterpret_cast<char*>(ptrs[i]);
  }
  lam_cap_ = cap;
  launch_lamport_init(lam_[rank_], lamport_bytes(cap, world_), nullptr);
  B200AR_CUDA(cudaDeviceSynchronize());
}

void Communicator::register_buffer(const std::vector<int64_t>& ptrs) {
  B200AR_CHECK(static_cast<int>(ptrs.size()) == world_, "need one buffer pointer per rank");
  // Kernels captured since the last register_graph_buffers() reference the
  // next arena records by position: taking one now would shift them.
  B200AR_CHECK(graph_pending_.empty(), "register_graph_buffers() must follow the capture of "
                                           << graph_pending_.size()
                                           << " registered all-reduce(s) before another buffer is registered");
  RankData rd{};
  for (int i = 0; i < world_; ++i) rd.ptrs[i] = reinterpret_cast<const void*>(ptrs[i]);
  RankData* d = arena_.take(1);
  B200AR_CUDA(cudaMemcpy(d, &rd, sizeof(RankData), cudaMemcpyHostToDevice));
  buffers_[reinterpret_cast<const void*>(ptrs[rank_])] = d;
}

std::pair<std::string, std::vector<int64_t>> Communicator::graph_buffer_meta() const {
  const size_t n = graph_pending_.size();
  std::string handles(kIpcHandleBytes * n, '\0');
  std::vector<int64_t> offsets(n);
  for (size_t i = 0; i < n; ++i) {
    auto [base, size] = allocation_range(graph_pending_[i]);
    (void)size;
    const std::string h = ipc_get_handle(base);
    std::memcpy(&handles[i * kIpcHandleBytes], h.data(), kIpcHandleBytes);
    offsets[i] = static_cast<const char*>(graph_pending_[i]) - static_cast<const char*>(base);
  }
  return {handles, offsets};
}

void Communicator::register_graph_buffers(const std::vector<std::string>& handles,
                                          const std::vector<std::vector<int64_t>>& offsets) {
  const size_t n = graph_pending_.size();
  B200AR_CHECK(static_cast<int>(handles.size()) == world_ && static_cast<int>(offsets.size()) == world_,
               "need graph metadata from every rank");
  for (int j = 0; j < world_; ++j) {
    B200AR_CHECK(handles[j].size() == n * kIpcHandleBytes && offsets[j].size() == n,
                 "rank " << j << " captured a different number of all-reduces (" << offsets[j].size() << " vs "
                         << n << ")");
  }
  if (n == 0) return;
  std::vector<RankData> rds(n);
  for (size_t i = 0; i < n; ++i) {
    for (int j = 0; j < world_; ++j) {
      if (j == rank_) {
        rds[i].ptrs[j] = graph_pending_[i];
      } else {
        char* base = open_ipc_handle(handles[j].substr(i * kIpcHandleBytes, kIpcHandleBytes));
        rds[i].ptrs[j] = base + offsets[j][i];
      }
    }
  }
  RankData* d = arena_.take(static_cast<int64_t>(n));
  B200AR_CUDA(cudaMemcpy(d, rds.data(), n * sizeof(RankData), cudaMemcpyHostToDevice));
  graph_pending_.clear();
}

LaunchInfo Communicator::plan(int64_t bytes, int variant, int ctas, bool capturing, bool registered_input) const {
  LaunchInfo li;
  li.threads = kArThreads;
  if (world_ == 1) {
    li.variant = kCopy;
    return li;
  }
  int v = variant;
  int c = ctas;
  if (v == kAuto) {
    if (registered_input && !slots_ok_) {
      v = kRegistered;
    } else if (!slots_ok_) {
      v = capturing ? kRegistered : kNccl;
    } else {
      v = kTwoshot;
      for (const auto& e : selector_) {
        if (bytes <= e.max_bytes) {
          v = e.variant;
          c = ctas > 0 ? ctas : e.ctas;
          break;
        }
      }
      if (v == kNvls && (nvls_ == nullptr || bytes > nvls_->bytes())) v = kTwoshot;
      if (v == kLamport && (lam_cap_ == 0 || bytes > lam_cap_)) v = kOneshotPush;
      // Fall back to the least demanding variant whose slot requirement fits.
      if (v == kOneshotPush || v == kOneshotPull || v == kTwoshot || v == kTwoshotPush) {
        if (variant_slot_bytes(v, bytes, world_) > slot_cap_) {
          if (variant_slot_bytes(kTwoshot, bytes, world_) <= slot_cap_) v = kTwoshot;
          else if (variant_slot_bytes(kOneshotPull, bytes, world_) <= slot_cap_) v = kOneshotPull;
          else v = registered_input ? kRegistered : kNccl;
          c = ctas;
        }
      }
    }
  }
  li.variant = v;
  li.ctas = plan_ctas(v, bytes, world_, c, resident_ctas(v));
  return li;
}

int plan_ctas(int variant, int64_t bytes, int world, int requested, int resident) {
  int64_t want = 0;
  if (variant == kOneshotPush || variant == kOneshotPull || variant == kRegistered || variant == kLamport) {
    const int64_t packets = bytes / 16;
    want = (packets + 2 * kArThreads - 1) / (2 * kArThreads);
  } else if (variant == kTwoshot || variant == kTwoshotPush || variant == kNvls) {
    const int64_t part = bytes / 16 / std::max(world, 1);
    want = (part + kArThreads - 1) / kArThreads;
  } else {
    return 0;  // copy / NCCL: not a barrier kernel of this module
  }
  int64_t c = requested > 0 ? requested : want;
  // CTA j of every rank waits for CTA j of its peers, so all CTAs of a launch
  // must be able to run at once: never more than fit on the device together.
  c = std::min<int64_t>(c, std::max(resident, 1));
  return static_cast<int>(std::clamp<int64_t>(c, 1, kMaxCTAs));
}

int Communicator::resident_ctas(int variant) const {
  if (variant < 0 || variant >= kNumVariants) return kMaxCTAs;
  int& cached = resident_[variant];
  if (cached == 0) {
    int dev = 0, sms = 0;
    B200AR_CUDA(cudaGetDevice(&dev));
    B200AR_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // The smallest per-SM occupancy over the three dtypes (they differ in registers).
    int per_sm = INT32_MAX;
    for (DType dt : {DType::kFloat32, DType::kFloat16, DType::kBFloat16}) {
      const int b = variant == kNvls ? nvls_blocks_per_sm(dt, world_) : ar_blocks_per_sm(variant, dt, world_);
      per_sm = std::min(per_sm, b);
    }
    cached = std::max(1, per_sm) * sms;
  }
  return cached;
}

LaunchInfo Communicator::allreduce(cudaStream_t stream, const void* in, void* out, int64_t bytes, DType dt,
                                   int variant, int ctas) {
  TraceRange trace("b200ar.all_reduce");
  check_status();
  B200AR_CHECK(bytes % 16 == 0, "all-reduce size must be a multiple of 16 bytes, got " << bytes);
  B200AR_CHECK(reinterpret_cast<uintptr_t>(in) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0,
               "all-reduce input and output must be 16-byte aligned");
  B200AR_CHECK(ctas >= 0 && ctas <= kMaxCTAs, "ctas must be in [0, " << kMaxCTAs << "]");
  LaunchInfo li;
  if (bytes == 0) {
    li.variant = kCopy;
    return li;
  }
  const auto reg = buffers_.find(in);
  const bool registered_input = reg != buffers_.end();
  bool capturing = false;
  if (!slots_ok_ || variant == kRegistered) {
    cudaStreamCaptureStatus cs;
    B200AR_CUDA(cudaStreamIsCapturing(stream, &cs));
    capturing = cs == cudaStreamCaptureStatusActive;
  }
  li = plan(bytes, variant, ctas, capturing, registered_input);
  if (li.variant == kNccl) return li;
  if (li.variant == kCopy) {
    if (in != out) {
      launch_copy(in, out, bytes / 16, stream);
      ++launches_;
    }
    return li;
  }
  if (li.variant == kNvls) {
    B200AR_CHECK(nvls_ != nullptr, "variant nvls requested but no NVLS buffer is attached");
    nvls_allreduce(*this, *nvls_, stream, in, out, bytes, static_cast<int>(dt), li.ctas);
    return li;
  }
  if (li.variant == kLamport) {
    B200AR_CHECK(lam_cap_ > 0 && bytes <= lam_cap_, "message of " << bytes << " bytes exceeds the Lamport capacity "
                                                                   << lam_cap_);
  } else if (li.variant != kRegistered) {
    B200AR_CHECK(slots_ok_, "variant " << li.variant << " needs registered slot buffers");
    B200AR_CHECK(variant_slot_bytes(li.variant, bytes, world_) <= slot_cap_,
                 "message of " << bytes << " bytes needs " << variant_slot_bytes(li.variant, bytes, world_)
                               << " bytes per slot for variant " << li.variant << ", slot capacity is "
                               << slot_cap_);
  }

  ArArgs a{};
  fill_ctx(&a.ctx);
  for (int s = 0; s < 2; ++s)
    for (int i = 0; i < world_; ++i) a.slot[s][i] = slots_[s][i];
  a.in = static_cast<const char*>(in);
  a.out = static_cast<char*>(out);
  a.packets = bytes / 16;
  for (int i = 0; i < world_; ++i) a.lam[i] = lam_[i];
  a.lam_cap = lam_cap_;
#if defined(B200AR_CHECKS)
  a.slot_cap = slot_cap_;
#endif
  if (li.variant == kRegistered) {
    if (capturing) {
      a.rd = arena_.peek(static_cast<int64_t>(graph_pending_.size()));  // throws when the arena is full
      graph_pending_.push_back(in);
    } else {
      if (!registered_input)
        throw std::runtime_error("buffer address " + std::to_string(reinterpret_cast<uint64_t>(in)) +
                                 " is not registered!");
      a.rd = reg->second;
    }
  }
  launch_ar_kernel(li.variant, dt, world_, li.ctas, li.threads, a, stream);
  ++launches_;
  return li;
}

void Communicator::fill_ctx(CommCtx* c) const {
  c->self = signals_[rank_];
  for (int i = 0; i < kMaxRanks; ++i) c->peers[i] = i < world_ ? signals_[i] : nullptr;
  c->status = status_dev_;
  c->timeout_ns = timeout_ns_;
  c->rank = rank_;
  c->world = world_;
}

Status Communicator::status() const {
  Status s;
  std::memcpy(&s, const_cast<const Status*>(status_host_), sizeof(Status));
  return s;
}

void Communicator::check_status() const {
  const volatile Status* v = status_host_;
  if (v->code == kStatusOk) return;
  Status s = status();
  std::ostringstream os;
  if (s.code == kStatusTimeout) {
    os << "b200ar: rank " << s.rank << " timed out waiting for rank " << s.peer << " (cta " << s.cta << ", epoch "
       << s.epoch << ", last seen " << s.seen << ", " << s.count << " CTA(s) affected); the communicator must be "
       << "reset() collectively";
    throw CommTimeout(os.str());
  }
  if (s.code == kStatusBadEpoch) {
    os << "b200ar: rank " << s.rank << " found flag " << s.seen << " from rank " << s.peer << " while waiting for "
       << "epoch " << s.epoch << " (cta " << s.cta << "): the signal block holds data the protocol never writes "
       << "(stale or corrupted); the communicator must be reset() collectively";
    throw CommTimeout(os.str());
  }
  if (s.code == kStatusOutOfBounds) {
    os << "b200ar: rank " << s.rank << " skipped a call whose " << (s.peer == 2u ? "Lamport" : "slot")
       << " footprint (" << s.epoch << " bytes, low word) exceeds its buffer (" << s.seen
       << " bytes, low word); the communicator must be reset() collectively";
    throw CommTimeout(os.str());
  }
  os << "b200ar: device reported error code " << s.code;
  throw std::runtime_error(os.str());
}

void Communicator::reset(cudaStream_t stream) {
  B200AR_CUDA(cudaStreamSynchronize(stream));
  B200AR_CUDA(cudaMemset(signals_[rank_], 0, sizeof(Signal)));
  // Restore the Lamport markers (an aborted call may have left peer packets).
  if (lam_cap_ > 0) launch_lamport_init(lam_[rank_], lamport_bytes(lam_cap_, world_), nullptr);
  B200AR_CUDA(cudaDeviceSynchronize());
  std::memset(status_host_, 0, sizeof(Status));
}

}  // namespace b200ar
