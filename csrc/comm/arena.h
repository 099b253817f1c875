// Rank-data arena: bump allocation of RankData records in a caller-supplied
// device buffer (the reference's d_rank_data_base_/end_ and
// check_rank_data_capacity, pcie_allreduce.cu:293, 343-346). Records live as
// long as the communicator. This class is host-only bookkeeping over the
// buffer's addresses; the owner writes records with cudaMemcpy.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>

#include "../common/layout.h"

namespace b200ar {

class RankDataArena {
 public:
  RankDataArena() = default;
  RankDataArena(void* base, int64_t bytes)
      : base_(static_cast<RankData*>(base)),
        cap_(base != nullptr && bytes > 0 ? bytes / static_cast<int64_t>(sizeof(RankData)) : 0) {}

  int64_t capacity() const { return cap_; }
  int64_t used() const { return used_; }
  int64_t remaining() const { return cap_ - used_; }
  bool fits(int64_t n) const { return n >= 0 && n <= remaining(); }

  // Address of the k-th record after those taken so far (k = 0: the next
  // take). CUDA-graph capture hands these addresses to captured kernels and
  // takes the records when the captured inputs are registered.
  RankData* peek(int64_t k) const {
    if (!fits(k + 1)) throw std::runtime_error("Rank data buffer overflow");
    return base_ + used_ + k;
  }

  RankData* take(int64_t n) {
    if (!fits(n))
      throw std::runtime_error("Rank data buffer overflow: " + std::to_string(n) + " record(s) requested, " +
                               std::to_string(remaining()) + " left of " + std::to_string(cap_));
    RankData* r = base_ + used_;
    used_ += n;
    return r;
  }

 private:
  RankData* base_ = nullptr;
  int64_t cap_ = 0;
  int64_t used_ = 0;
};

}  // namespace b200ar
