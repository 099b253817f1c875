// CPU shared-memory backend (see shm_comm.h).
#include "shm_comm.h"

#include <c10/util/BFloat16.h>
#include <c10/util/Half.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <sstream>
#include <stdexcept>
#include <thread>

#include "../common/check.h"

namespace b200ar {

namespace {

inline void st_release(uint32_t* p, uint32_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }
inline uint32_t ld_acquire(const uint32_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }

template <typename T>
inline float to_f(T v) {
  return static_cast<float>(v);
}
template <typename T>
inline T from_f(float v) {
  return static_cast<T>(v);  // c10::BFloat16 / c10::Half round to nearest even
}

template <typename T>
constexpr int elems() {
  return 16 / static_cast<int>(sizeof(T));
}

template <typename T>
inline void packet_set(const char* p, float* acc) {
  const T* e = reinterpret_cast<const T*>(p);
  for (int i = 0; i < elems<T>(); ++i) acc[i] = to_f(e[i]);
}
template <typename T>
inline void packet_add(const char* p, float* acc) {
  const T* e = reinterpret_cast<const T*>(p);
  for (int i = 0; i < elems<T>(); ++i) acc[i] += to_f(e[i]);
}
template <typename T>
inline void packet_store(char* p, const float* acc) {
  T* e = reinterpret_cast<T*>(p);
  for (int i = 0; i < elems<T>(); ++i) e[i] = from_f<T>(acc[i]);
}

void write_header(Signal* sig, int rank, int world, int64_t slot_cap, int64_t lam_cap) {
  sig->owner_rank = static_cast<uint32_t>(rank);
  sig->world = static_cast<uint32_t>(world);
  sig->slot_cap_lo = static_cast<uint32_t>(slot_cap & 0xffffffffu);
  sig->slot_cap_hi = static_cast<uint32_t>(slot_cap >> 32);
  sig->lamport_cap = static_cast<uint32_t>(lam_cap);
  __atomic_store_n(&sig->magic, kSegmentMagic, __ATOMIC_RELEASE);
}

}  // namespace

ShmComm::ShmComm(const std::string& prefix, int rank, int world, int64_t slot_capacity, int64_t lamport_capacity)
    : rank_(rank), world_(world), cap_(slot_capacity), lam_cap_(lamport_capacity), names_(world), base_(world, nullptr) {
  B200AR_CHECK(world >= 1 && world <= kMaxRanks, "world size must be in [1, " << kMaxRanks << "]");
  B200AR_CHECK(rank >= 0 && rank < world, "invalid rank " << rank);
  B200AR_CHECK(slot_capacity > 0 && slot_capacity % 16 == 0, "slot capacity must be a positive multiple of 16");
  B200AR_CHECK(lamport_capacity >= 0 && lamport_capacity % 16 == 0, "Lamport capacity must be a multiple of 16");
  seg_bytes_ = workspace_bytes(cap_) + lamport_bytes(lam_cap_, world);
  names_[rank] = prefix + "-r" + std::to_string(rank);
  const int fd = shm_open(names_[rank].c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
  if (fd < 0) throw std::runtime_error("shm_open(" + names_[rank] + ") failed: " + std::strerror(errno));
  if (ftruncate(fd, seg_bytes_) != 0) {
    close(fd);
    shm_unlink(names_[rank].c_str());
    throw std::runtime_error("ftruncate of shared segment failed");
  }
  void* p = mmap(nullptr, seg_bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) {
    shm_unlink(names_[rank].c_str());
    throw std::runtime_error("mmap of shared segment failed");
  }
  std::memset(p, 0, sizeof(Signal));
  write_header(static_cast<Signal*>(p), rank, world, slot_capacity, lamport_capacity);
  uint32_t* lam = reinterpret_cast<uint32_t*>(static_cast<char*>(p) + workspace_bytes(cap_));
  for (int64_t i = 0; i < lamport_bytes(lam_cap_, world) / 4; ++i) lam[i] = kLamportMarker;
  base_[rank] = static_cast<char*>(p);
}

ShmComm::~ShmComm() {
  for (int i = 0; i < world_; ++i)
    if (base_[i]) munmap(base_[i], seg_bytes_);
  if (!owner_unlinked_) shm_unlink(names_[rank_].c_str());
}

void ShmComm::connect(const std::vector<std::string>& names) {
  B200AR_CHECK(static_cast<int>(names.size()) == world_, "need one segment name per rank");
  B200AR_CHECK(names[rank_] == names_[rank_], "names[rank] must be this rank's own segment");
  for (int i = 0; i < world_; ++i) {
    if (i == rank_) continue;
    const int fd = shm_open(names[i].c_str(), O_RDWR, 0600);
    if (fd < 0) throw std::runtime_error("shm_open(" + names[i] + ") failed: " + std::strerror(errno));
    // A segment of the wrong size would fault on access: check before mapping.
    struct stat sb {};
    if (fstat(fd, &sb) != 0 || static_cast<int64_t>(sb.st_size) != seg_bytes_) {
      close(fd);
      std::ostringstream os;
      os << "b200ar(cpu): segment '" << names[i] << "' given for rank " << i << " has " << sb.st_size
         << " bytes, expected " << seg_bytes_ << " (corrupted or mismatched handle exchange)";
      throw std::runtime_error(os.str());
    }
    void* p = mmap(nullptr, seg_bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (p == MAP_FAILED) throw std::runtime_error("mmap of peer segment failed");
    const Signal* sig = static_cast<const Signal*>(p);
    const int64_t cap = static_cast<int64_t>(sig->slot_cap_lo) | (static_cast<int64_t>(sig->slot_cap_hi) << 32);
    if (__atomic_load_n(&sig->magic, __ATOMIC_ACQUIRE) != kSegmentMagic || sig->owner_rank != static_cast<uint32_t>(i) ||
        sig->world != static_cast<uint32_t>(world_) || cap != cap_ || sig->lamport_cap != static_cast<uint32_t>(lam_cap_)) {
      std::ostringstream os;
      os << "b200ar(cpu): segment '" << names[i] << "' given for rank " << i << " does not match (magic 0x" << std::hex
         << sig->magic << std::dec << ", owner " << sig->owner_rank << ", world " << sig->world << ", slot capacity "
         << cap << "; expected rank " << i << ", world " << world_ << ", slot capacity " << cap_
         << "): corrupted or mismatched handle exchange";
      munmap(p, seg_bytes_);
      throw std::runtime_error(os.str());
    }
    if (base_[i]) munmap(base_[i], seg_bytes_);  // re-connect: drop the old mapping
    base_[i] = static_cast<char*>(p);
    names_[i] = names[i];
  }
}

uint32_t ShmComm::generation() const { return ld_acquire(&reinterpret_cast<Signal*>(base_[rank_])->gen); }

void ShmComm::reset() {
  std::memset(base_[rank_], 0, sizeof(Signal));
  write_header(reinterpret_cast<Signal*>(base_[rank_]), rank_, world_, cap_, lam_cap_);
  // Peers' packets of an aborted call may sit in the Lamport buffers: restore
  // the markers so the next Lamport call does not read stale data.
  uint32_t* lam = reinterpret_cast<uint32_t*>(base_[rank_] + workspace_bytes(cap_));
  for (int64_t i = 0; i < lamport_bytes(lam_cap_, world_) / 4; ++i) lam[i] = kLamportMarker;
  std::atomic_thread_fence(std::memory_order_seq_cst);
  status_ = Status{};
  skip_ = 0;
}

void ShmComm::inject_flag(int cta, int src, uint32_t value) {
  B200AR_CHECK(cta >= 0 && cta < kMaxCTAs && src >= 0 && src < world_, "flag index out of range");
  st_release(&reinterpret_cast<Signal*>(base_[rank_])->flags[cta][src], value);
}

bool ShmComm::barrier(int cta, uint32_t epoch) {
  Signal* self = reinterpret_cast<Signal*>(base_[rank_]);
  for (int p = 0; p < world_; ++p)
    st_release(&reinterpret_cast<Signal*>(base_[p])->flags[cta][rank_], epoch);
  const auto start = std::chrono::steady_clock::now();
  auto fail = [&](uint32_t code, int p, uint32_t seen) {
    if (status_.code == kStatusOk) {
      status_.code = code;
      status_.rank = rank_;
      status_.peer = p;
      status_.cta = cta;
      status_.epoch = epoch;
      status_.seen = seen;
    }
    ++status_.count;
    return false;
  };
  for (int p = 0; p < world_; ++p) {
    uint32_t seen;
    uint32_t spins = 0;
    while (!epoch_reached(seen = ld_acquire(&self->flags[cta][p]), epoch)) {
      if ((++spins & 255u) == 0u) {
        std::this_thread::yield();
        const auto ms =
            std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - start).count();
        if (ms > timeout_ms_) return fail(kStatusTimeout, p, seen);
      }
    }
    if (epoch_too_far(seen, epoch)) return fail(kStatusBadEpoch, p, seen);
  }
  return true;
}

template <typename T>
void ShmComm::run(const char* in, char* out, int64_t P, int variant, int G) {
  Signal* self = reinterpret_cast<Signal*>(base_[rank_]);
  const uint32_t gen = self->gen;
  const int slot = gen & 1u;
  const int N = world_;
  const int r = rank_;
  auto slotp = [&](int p) { return base_[p] + slot_offset(slot, cap_); };
  constexpr int E = elems<T>();
  float acc[E];
  bool ok = true;
  const bool skip = skip_ > 0;

  for (int j = 0; j < G && ok; ++j) {
    if (variant == kOneshotPush || variant == kOneshotPull) {
      const int64_t b = part_begin(P, G, j), e = part_begin(P, G, j + 1);
      if (variant == kOneshotPush) {
        for (int64_t i = b; i < e; ++i)
          for (int k = 0; k < N; ++k) {
            const int p = (r + k) % N;
            std::memcpy(slotp(p) + (static_cast<int64_t>(r) * P + i) * 16, in + i * 16, 16);
          }
      } else {
        std::memcpy(slotp(r) + b * 16, in + b * 16, (e - b) * 16);
      }
      if (skip) continue;
      if (!(ok = barrier(j, epoch_of(gen, 0)))) break;
      for (int64_t i = b; i < e; ++i) {
        if (variant == kOneshotPush) {
          const char* mine = slotp(r);
          packet_set<T>(mine + i * 16, acc);
          for (int q = 1; q < N; ++q) packet_add<T>(mine + (static_cast<int64_t>(q) * P + i) * 16, acc);
        } else {
          packet_set<T>(slotp(0) + i * 16, acc);
          for (int q = 1; q < N; ++q) packet_add<T>(slotp(q) + i * 16, acc);
        }
        packet_store<T>(out + i * 16, acc);
      }
    } else if (variant == kTwoshot || variant == kTwoshotPush) {
      const int64_t part = (P + N - 1) / N;
      auto sub = [&](int p, int64_t* pb, int64_t* sb, int64_t* sl) {
        *pb = part_begin(P, N, p);
        const int64_t plen = part_begin(P, N, p + 1) - *pb;
        *sb = part_begin(plen, G, j);
        *sl = part_begin(plen, G, j + 1) - *sb;
      };
      int64_t pb, sb, sl;
      for (int k = 0; k < N; ++k) {
        const int p = (r + k) % N;
        sub(p, &pb, &sb, &sl);
        std::memcpy(slotp(p) + (static_cast<int64_t>(r) * part + sb) * 16, in + (pb + sb) * 16, sl * 16);
      }
      if (skip) continue;
      if (!(ok = barrier(j, epoch_of(gen, 0)))) break;
      sub(r, &pb, &sb, &sl);
      char* mine = slotp(r);
      const bool push = variant == kTwoshotPush;
      const int64_t gathered = static_cast<int64_t>(N) * part;
      for (int64_t o = sb; o < sb + sl; ++o) {
        packet_set<T>(mine + o * 16, acc);
        for (int q = 1; q < N; ++q) packet_add<T>(mine + (static_cast<int64_t>(q) * part + o) * 16, acc);
        packet_store<T>(out + (pb + o) * 16, acc);
        if (push) {
          // Reduced packet into row r of every peer's gathered area.
          for (int k = 1; k < N; ++k)
            std::memcpy(slotp((r + k) % N) + (gathered + static_cast<int64_t>(r) * part + o) * 16,
                        out + (pb + o) * 16, 16);
        } else {
          std::memcpy(mine + (gathered + o) * 16, out + (pb + o) * 16, 16);
        }
      }
      if (!(ok = barrier(j, epoch_of(gen, 1)))) break;
      for (int k = 1; k < N; ++k) {
        const int p = (r + k) % N;
        sub(p, &pb, &sb, &sl);
        if (push)
          std::memcpy(out + (pb + sb) * 16, mine + (gathered + static_cast<int64_t>(p) * part + sb) * 16, sl * 16);
        else
          std::memcpy(out + (pb + sb) * 16, slotp(p) + (gathered + sb) * 16, sl * 16);
      }
    } else {
      throw std::invalid_argument(
          "CPU backend supports variants push (1), pull (2), two-shot (3), Lamport (8), two-shot push (9)");
    }
  }
  if (skip) --skip_;
  __atomic_store_n(&self->gen, gen + 1u, __ATOMIC_RELEASE);
  if (!ok) {
    std::ostringstream os;
    if (status_.code == kStatusBadEpoch)
      os << "b200ar(cpu): rank " << status_.rank << " found flag " << status_.seen << " from rank " << status_.peer
         << " while waiting for epoch " << status_.epoch << " (cta " << status_.cta
         << "): the signal block holds data the protocol never writes (stale or corrupted)";
    else
      os << "b200ar(cpu): rank " << status_.rank << " timed out waiting for rank " << status_.peer << " (cta "
         << status_.cta << ", epoch " << status_.epoch << ", last seen " << status_.seen << ")";
    throw CommTimeout(os.str());
  }
}

// Lamport one-shot, as oneshot_lamport_kernel: write own packets (-0.0 turned
// into +0.0) into every rank's buffer gen % 3, poll own buffer until no word
// is the marker, sum in rank order, restore the markers. Emulated CTAs run
// one after the other; CTA j only waits for the peers' CTA j packets.
template <typename T>
void ShmComm::run_lamport(const char* in, char* out, int64_t P, int G) {
  Signal* self = reinterpret_cast<Signal*>(base_[rank_]);
  const uint32_t gen = self->gen;
  const int N = world_;
  const int r = rank_;
  const int64_t buf = workspace_bytes(cap_) + static_cast<int64_t>(gen % kLamportBuffers) * N * lam_cap_;
  constexpr int E = elems<T>();
  float acc[E];
  const bool skip = skip_ > 0;
  bool ok = true;
  for (int j = 0; j < G && ok; ++j) {
    const int64_t b = part_begin(P, G, j), e = part_begin(P, G, j + 1);
    for (int64_t i = b; i < e; ++i) {
      uint32_t w[4];
      std::memcpy(w, in + i * 16, 16);
      for (int k = 0; k < 4; ++k) {
        if (sizeof(T) == 4) {
          if (w[k] == kLamportMarker) w[k] = 0;
        } else {
          if ((w[k] & 0xffffu) == 0x8000u) w[k] &= 0xffff0000u;
          if ((w[k] >> 16) == 0x8000u) w[k] &= 0x0000ffffu;
        }
      }
      for (int p = 0; p < N; ++p) {
        uint32_t* dst = reinterpret_cast<uint32_t*>(base_[p] + buf + static_cast<int64_t>(r) * lam_cap_ + i * 16);
        for (int k = 0; k < 4; ++k) __atomic_store_n(dst + k, w[k], __ATOMIC_RELAXED);
      }
    }
    if (skip) continue;
    for (int64_t i = b; i < e && ok; ++i) {
      for (int q = 0; q < N && ok; ++q) {
        uint32_t* src = reinterpret_cast<uint32_t*>(base_[r] + buf + static_cast<int64_t>(q) * lam_cap_ + i * 16);
        const auto start = std::chrono::steady_clock::now();
        uint32_t spins = 0;
        for (;;) {
          bool ready = true;
          for (int k = 0; k < 4; ++k) ready &= __atomic_load_n(src + k, __ATOMIC_ACQUIRE) != kLamportMarker;
          if (ready) break;
          if ((++spins & 255u) == 0u) {
            std::this_thread::yield();
            const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                                std::chrono::steady_clock::now() - start).count();
            if (ms > timeout_ms_) {
              if (status_.code == kStatusOk) {
                status_.code = kStatusTimeout;
                status_.rank = r;
                status_.peer = q;
                status_.cta = j;
                status_.epoch = gen;
              }
              ++status_.count;
              ok = false;
              break;
            }
          }
        }
      }
      if (!ok) break;
      for (int q = 0; q < N; ++q) {
        const char* src = base_[r] + buf + static_cast<int64_t>(q) * lam_cap_ + i * 16;
        if (q == 0)
          packet_set<T>(src, acc);
        else
          packet_add<T>(src, acc);
      }
      packet_store<T>(out + i * 16, acc);
      for (int q = 0; q < N; ++q) {
        uint32_t* src = reinterpret_cast<uint32_t*>(base_[r] + buf + static_cast<int64_t>(q) * lam_cap_ + i * 16);
        for (int k = 0; k < 4; ++k) __atomic_store_n(src + k, kLamportMarker, __ATOMIC_RELAXED);
      }
    }
  }
  if (skip) --skip_;
  __atomic_store_n(&self->gen, gen + 1u, __ATOMIC_RELEASE);
  if (!ok) {
    std::ostringstream os;
    os << "b200ar(cpu): rank " << status_.rank << " timed out waiting for rank " << status_.peer
       << " (Lamport packets, cta " << status_.cta << ", generation " << status_.epoch << ")";
    throw CommTimeout(os.str());
  }
}

void ShmComm::allreduce(const void* in, void* out, int64_t bytes, DType dt, int variant, int ctas) {
  B200AR_CHECK(bytes % 16 == 0, "all-reduce size must be a multiple of 16 bytes");
  B200AR_CHECK(base_.size() == static_cast<size_t>(world_), "not connected");
  for (int i = 0; i < world_; ++i) B200AR_CHECK(base_[i] != nullptr, "not connected to rank " << i);
  if (status_.code != kStatusOk)
    throw CommTimeout("b200ar(cpu): communicator is in error state; reset() it collectively");
  if (bytes == 0) return;
  if (world_ == 1) {
    if (in != out) std::memmove(out, in, bytes);
    return;
  }
  if (variant == kAuto) variant = bytes <= 256 * 1024 ? kOneshotPush : kTwoshot;
  if (variant == kLamport) {
    B200AR_CHECK(bytes <= lam_cap_, "message of " << bytes << " bytes exceeds the Lamport capacity " << lam_cap_);
    const int G = ctas > 0 ? std::min(ctas, kMaxCTAs) : 4;
    const char* i = static_cast<const char*>(in);
    char* o = static_cast<char*>(out);
    switch (dt) {
      case DType::kFloat32: run_lamport<float>(i, o, bytes / 16, G); break;
      case DType::kFloat16: run_lamport<c10::Half>(i, o, bytes / 16, G); break;
      case DType::kBFloat16: run_lamport<c10::BFloat16>(i, o, bytes / 16, G); break;
    }
    return;
  }
  const int64_t need = variant_slot_bytes(variant, bytes, world_);
  if (need > cap_) {
    variant = variant_slot_bytes(kTwoshot, bytes, world_) <= cap_ ? kTwoshot : kOneshotPull;
    B200AR_CHECK(variant_slot_bytes(variant, bytes, world_) <= cap_,
                 "message of " << bytes << " bytes does not fit the slot capacity " << cap_);
  }
  const int64_t P = bytes / 16;
  const int G = ctas > 0 ? std::min(ctas, kMaxCTAs) : 4;
  const char* i = static_cast<const char*>(in);
  char* o = static_cast<char*>(out);
  switch (dt) {
    case DType::kFloat32: run<float>(i, o, P, variant, G); break;
    case DType::kFloat16: run<c10::Half>(i, o, P, variant, G); break;
    case DType::kBFloat16: run<c10::BFloat16>(i, o, P, variant, G); break;
  }
}

}  // namespace b200ar
