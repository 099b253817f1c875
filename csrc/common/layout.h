// Shared-memory protocol of b200ar: signal block, workspace layout, epochs and
// message partitioning. Compiled both by nvcc (device kernels) and by the host
// compiler (the CPU shared-memory backend), so that the GPU data plane and its
// CPU emulation use the same layout and the same epoch arithmetic.
//
// Relation to the reference (pcie_allreduce/pcie_allreduce.cu):
//  * Signal (cu:52-56) held per-CTA self counters plus a parity-banked mailbox
//    and the host picked the double-buffer slot (cu:413-414). Here the device
//    owns a per-call generation counter `gen`: every kernel reads it on entry,
//    the last CTA to finish bumps it. The slot is gen & 1 and the barrier epochs
//    are derived from gen, so CUDA-graph replays alternate slots correctly and
//    no host state is captured.
//  * Flags are compared with a signed difference against monotonically
//    increasing epochs, so one bank suffices and a peer that is ahead can never
//    be mistaken for one that is behind.
//  * The 128-byte flag stride that the reference used against PCIe false sharing
//    (cu:49-50) is not needed on NVSwitch; flags are packed [cta][peer].
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define B200AR_HD __host__ __device__ __forceinline__
#else
#define B200AR_HD inline
#endif

namespace b200ar {

constexpr int kMaxRanks = 8;
// Upper bound on CTAs of one collective launch (flags are kept per CTA).
constexpr int kMaxCTAs = 512;
// Every collective call reserves this many barrier epochs.
constexpr uint32_t kEpochsPerCall = 2;
// Upper bound on output tiles of one fused GEMM + all-reduce call.
constexpr int kMaxTiles = 4096;

// Identifies a b200ar CPU segment ("b2ar").
constexpr uint32_t kSegmentMagic = 0x72613262u;

enum class DType : int { kFloat32 = 0, kFloat16 = 1, kBFloat16 = 2 };

B200AR_HD int dtype_size(DType d) { return d == DType::kFloat32 ? 4 : 2; }

// Error codes written into the status word.
enum StatusCode : uint32_t {
  kStatusOk = 0,
  kStatusTimeout = 1,      // a peer did not arrive at a barrier before the deadline
  kStatusBadArgs = 2,      // a kernel found arguments it cannot serve
  kStatusBadEpoch = 3,     // a peer's flag is further ahead than the protocol allows:
                           // the signal block was overwritten (stale or foreign data)
  kStatusOutOfBounds = 4,  // checked builds: an access range exceeded its buffer
};

// Error record. Lives in host-mapped pinned memory (GPU) or process memory
// (CPU backend) so the host can read it without synchronising the device.
struct alignas(64) Status {
  uint32_t code;   // StatusCode; first error wins
  uint32_t rank;   // rank that detected the error
  uint32_t peer;   // peer that failed to arrive
  uint32_t cta;    // CTA index (GPU) or 0
  uint32_t epoch;  // epoch that was awaited
  uint32_t seen;   // last flag value observed from the peer
  uint32_t count;  // number of CTAs that reported an error
  uint32_t pad[9];
};

// Peer pointers of one registered buffer (entry i = rank i's copy as mapped
// in this process). Kept in a device-memory arena so that a CUDA-graph capture
// can reference a record that is filled after capture (the reference's
// RankData, pcie_allreduce.cu:58-61).
struct alignas(16) RankData {
  const void* ptrs[kMaxRanks];
};

// Per-rank signal block, placed at offset 0 of each rank's shared workspace.
// It must be zero-initialised before first use (like the reference's
// memset of its Signal buffer, test_pcie_ar.py:36).
struct alignas(256) Signal {
  // Generation = number of completed collective calls on this rank (local only).
  uint32_t gen;
  // CTAs of the current call that have finished (local only, reset by the last).
  uint32_t done;
  // Segment header (CPU backend): written by the owner, checked by every peer
  // when it maps the segment, so a wrong or corrupted exchanged name fails on
  // the host instead of mapping foreign memory. The GPU path leaves it zero.
  uint32_t magic;          // kSegmentMagic
  uint32_t owner_rank;     // rank that created the segment
  uint32_t world;          // world size it was created for
  uint32_t slot_cap_lo;    // slot capacity in bytes (low / high word)
  uint32_t slot_cap_hi;
  uint32_t lamport_cap;    // Lamport capacity in bytes
  uint32_t reserved[56];
  // flags[cta][src]: highest epoch that rank `src` reached in CTA `cta`.
  // Written remotely by rank `src`, read locally.
  uint32_t flags[kMaxCTAs][kMaxRanks];
  // Fused GEMM + all-reduce: tile_flags[t][src] = call epoch once rank `src`
  // pushed its partial of tile t here; tile_ready[t] = call epoch once this
  // rank (the tile's owner) published the reduced tile.
  uint32_t tile_flags[kMaxTiles][kMaxRanks];
  uint32_t tile_ready[kMaxTiles];
};

static_assert(sizeof(Signal) % 256 == 0, "Signal must keep 256-byte alignment of what follows");

// Epoch of barrier `b` (0-based, < kEpochsPerCall) of the call with generation `gen`.
B200AR_HD uint32_t epoch_of(uint32_t gen, uint32_t b) { return gen * kEpochsPerCall + b + 1u; }

// True once `seen` has reached `want` under wrap-around arithmetic.
B200AR_HD bool epoch_reached(uint32_t seen, uint32_t want) { return static_cast<int32_t>(seen - want) >= 0; }

// True if `seen` is further ahead of `want` than any peer can legitimately be.
// A peer passes a barrier only after this rank arrived at it, so while this
// rank waits for epoch e of a flag row the peer can have finished the current
// call and arrived at the next barrier of that row: at most e + kEpochsPerCall
// (one-barrier calls use epoch 2g + 1 of each call). Anything beyond is data
// that the protocol never writes.
B200AR_HD bool epoch_too_far(uint32_t seen, uint32_t want) {
  return static_cast<int32_t>(seen - want) > static_cast<int32_t>(kEpochsPerCall);
}

// Start of part `i` when `total` items are split into `parts` nearly equal parts.
B200AR_HD int64_t part_begin(int64_t total, int parts, int i) { return (total * i) / parts; }

// Workspace of one rank: [Signal][slot 0][slot 1]; `cap` bytes per slot.
B200AR_HD int64_t signal_bytes() { return static_cast<int64_t>(sizeof(Signal)); }
B200AR_HD int64_t workspace_bytes(int64_t cap) { return signal_bytes() + 2 * cap; }

B200AR_HD int64_t slot_offset(int slot, int64_t cap) { return signal_bytes() + slot * cap; }

// Algorithm variants. The integer values are part of the Python API.
enum Variant : int {
  kAuto = 0,
  kOneshotPush = 1,   // push input to every peer's slot[rank], barrier, local reduce
  kOneshotPull = 2,   // copy input to own slot, barrier, pull-reduce from all peers
  kTwoshot = 3,       // push-reduce-scatter, barrier, reduce own part, barrier, pull-all-gather
  kNvls = 4,          // multimem.ld_reduce / multimem.st through NVSwitch
  kRegistered = 5,    // pull directly from registered peer buffers, start + end barrier
  kNccl = 6,          // fall back to NCCL (handled by the Python layer)
  kCopy = 7,          // world size 1: plain copy
  kLamport = 8,       // push with in-band "not yet written" markers: no barrier, no fence
  kTwoshotPush = 9,   // push-reduce-scatter, barrier, reduce own part and push it to every peer,
                      // barrier, local copy of the gathered parts
};

// The one-shot Lamport variant keeps kLamportBuffers rotating buffers of
// world x lamport_cap bytes per rank, pre-filled with this 32-bit marker
// (the bit pattern of -0.0f; for 16-bit types the word (+0, -0)). Writers turn
// every -0.0 element into +0.0, so real data never contains the marker word.
constexpr int kLamportBuffers = 3;
constexpr uint32_t kLamportMarker = 0x80000000u;

B200AR_HD int64_t lamport_bytes(int64_t lamport_cap, int world) { return kLamportBuffers * world * lamport_cap; }

// Slot bytes a variant needs for a message of `bytes` bytes on `world` ranks.
// Two-shot: world parts of ceil(packets / world) 16-byte packets for the
// reduce-scatter inbox plus one such part for the all-gather outbox.
B200AR_HD int64_t variant_slot_bytes(int variant, int64_t bytes, int world) {
  const int64_t packets = bytes / 16;
  switch (variant) {
    case kOneshotPush: return bytes * world;
    case kOneshotPull: return bytes;
    case kTwoshot: {
      const int64_t part = (packets + world - 1) / world;
      return (world + 1) * part * 16;
    }
    case kTwoshotPush: {
      const int64_t part = (packets + world - 1) / world;
      return 2 * world * part * 16;  // inbox rows + gathered rows, one of each per source
    }
    default: return 0;
  }
}

}  // namespace b200ar
