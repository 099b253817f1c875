// Device primitives for the b200ar data plane (sm_100a):
//  * 16-byte packets of bf16/fp16/fp32 with fp32 accumulation,
//  * system-scope release/acquire flag operations (inline PTX),
//  * cache-controlled 16-byte loads/stores for peer and local buffers,
//  * a bounded per-CTA cross-GPU barrier that reports a timeout instead of
//    spinning forever.
//
// Counterparts in the reference (pcie_allreduce/pcie_allreduce.cu):
// array_t/packed_t (cu:66-77), upcast/downcast (cu:79-129),
// st/ld_flag_relaxed (cu:133-141), multi_gpu_barrier (cu:147-159) and
// packed_reduce (cu:163-169). Differences: flags are released and acquired at
// system scope instead of relaxed + fence, the spin is bounded by %globaltimer,
// and the epoch comes from the device-side generation counter (layout.h).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "layout.h"

namespace b200ar {

#define B200AR_DEV __device__ __forceinline__

// ---------------------------------------------------------------------------
// 16-byte packets
// ---------------------------------------------------------------------------

template <typename T>
struct PackTraits {
  static constexpr int kElems = 16 / sizeof(T);
};

// Converts a 16-byte packet to kElems floats.
template <typename T>
B200AR_DEV void unpack_add(const uint4& v, float* acc);
template <typename T>
B200AR_DEV void unpack_set(const uint4& v, float* acc);
template <typename T>
B200AR_DEV uint4 pack(const float* acc);

template <>
B200AR_DEV void unpack_set<float>(const uint4& v, float* a) {
  a[0] = __uint_as_float(v.x);
  a[1] = __uint_as_float(v.y);
  a[2] = __uint_as_float(v.z);
  a[3] = __uint_as_float(v.w);
}
template <>
B200AR_DEV void unpack_add<float>(const uint4& v, float* a) {
  a[0] += __uint_as_float(v.x);
  a[1] += __uint_as_float(v.y);
  a[2] += __uint_as_float(v.z);
  a[3] += __uint_as_float(v.w);
}
template <>
B200AR_DEV uint4 pack<float>(const float* a) {
  return make_uint4(__float_as_uint(a[0]), __float_as_uint(a[1]), __float_as_uint(a[2]), __float_as_uint(a[3]));
}

template <>
B200AR_DEV void unpack_set<__nv_bfloat16>(const uint4& v, float* a) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bf16 -> fp32 is an exact 16-bit shift.
    a[2 * i] = __uint_as_float(w[i] << 16);
    a[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
B200AR_DEV void unpack_add<__nv_bfloat16>(const uint4& v, float* a) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    a[2 * i] += __uint_as_float(w[i] << 16);
    a[2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
B200AR_DEV uint4 pack<__nv_bfloat16>(const float* a) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <>
B200AR_DEV void unpack_set<__half>(const uint4& v, float* a) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 f = __half22float2(h);
    a[2 * i] = f.x;
    a[2 * i + 1] = f.y;
  }
}
template <>
B200AR_DEV void unpack_add<__half>(const uint4& v, float* a) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 f = __half22float2(h);
    a[2 * i] += f.x;
    a[2 * i + 1] += f.y;
  }
}
template <>
B200AR_DEV uint4 pack<__half>(const float* a) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ---------------------------------------------------------------------------
// Memory operations
// ---------------------------------------------------------------------------

// Plain 16-byte load of data that is not written during this kernel.
B200AR_DEV uint4 ld_in(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// 16-byte load that bypasses L1: used for buffers written by peers (local
// buffer filled by remote stores) and for loads from peer memory.
B200AR_DEV uint4 ld_cg(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

// 16-byte store that bypasses L1 (local or peer memory).
B200AR_DEV void st_cg(void* p, const uint4& v) { __stcg(reinterpret_cast<uint4*>(p), v); }

// Plain 16-byte store to local output.
B200AR_DEV void st_out(void* p, const uint4& v) { *reinterpret_cast<uint4*>(p) = v; }

B200AR_DEV void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

B200AR_DEV uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

B200AR_DEV uint32_t ld_relaxed_gpu(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

B200AR_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// Kernel context: generation, barrier, status
// ---------------------------------------------------------------------------

// Per-rank collective context handed to every kernel by value.
struct CommCtx {
  Signal* self;                 // this rank's signal block (local)
  Signal* peers[kMaxRanks];     // every rank's signal block (peer mappings; [rank] == self)
  Status* status;               // host-mapped error record
  uint64_t timeout_ns;          // barrier deadline per wait
  int rank;
  int world;
};

// Reads the call generation (one thread), shares it through shared memory.
B200AR_DEV uint32_t read_generation(const CommCtx& c, uint32_t* s_gen) {
  if (threadIdx.x == 0) *s_gen = ld_relaxed_gpu(&c.self->gen);
  __syncthreads();
  return *s_gen;
}

// Called by every CTA at the very end of a collective kernel: the last CTA to
// finish advances the generation for the next call on this stream.
B200AR_DEV void finish_generation(const CommCtx& c, uint32_t gen) {
  __syncthreads();
  if (gridDim.x == 1) {
    // One CTA: no arrival count needed (saves an atomic round trip to L2).
    if (threadIdx.x == 0) c.self->gen = gen + 1u;
    return;
  }
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&c.self->done, 1u);
    if (prev == gridDim.x - 1) {
      c.self->done = 0;
      __threadfence();
      atomicExch(&c.self->gen, gen + 1u);
    }
  }
}

B200AR_DEV void report_status(Status* st, uint32_t code, uint32_t rank, uint32_t peer, uint32_t cta,
                              uint32_t epoch, uint32_t seen) {
  if (atomicCAS(&st->code, 0u, code) == 0u) {
    st->rank = rank;
    st->peer = peer;
    st->cta = cta;
    st->epoch = epoch;
    st->seen = seen;
  }
  atomicAdd(&st->count, 1u);
  __threadfence_system();
}

// Per-CTA barrier among `world` ranks for flag row `cta`.
// Every thread's prior global writes (ordered by __syncthreads) are released at
// system scope with the flag store; the wait acquires the peer's writes.
// Returns false (uniformly across the CTA) if any wait timed out; the timeout is
// recorded in the status word and the caller must skip dependent work.
template <int N>
B200AR_DEV bool cta_barrier(const CommCtx& c, int cta, uint32_t epoch) {
  __syncthreads();
  int fail = 0;
  if (threadIdx.x < N) {
    const int peer = threadIdx.x;
    st_release_sys(&c.peers[peer]->flags[cta][c.rank], epoch);
    const uint32_t* mine = &c.self->flags[cta][peer];
    uint32_t seen = ld_acquire_sys(mine);
    if (!epoch_reached(seen, epoch)) {
      const uint64_t start = global_ns();
      uint32_t spins = 0;
      while (!epoch_reached(seen = ld_acquire_sys(mine), epoch)) {
        if ((++spins & 63u) == 0u && global_ns() - start > c.timeout_ns) {
          report_status(c.status, kStatusTimeout, c.rank, peer, cta, epoch, seen);
          fail = 1;
          break;
        }
      }
    }
#if defined(B200AR_CHECKS)
    // Checked builds: a flag further ahead than any peer can be means the
    // signal block was overwritten; fail instead of trusting the data.
    if (!fail && epoch_too_far(seen, epoch)) {
      report_status(c.status, kStatusBadEpoch, c.rank, peer, cta, epoch, seen);
      fail = 1;
    }
#endif
  }
  return __syncthreads_or(fail) == 0;
}

// Checked builds (-DB200AR_CHECKS): a kernel verifies on entry that the byte
// range it is about to touch, [0, need), lies inside its buffer of `cap`
// bytes. On failure it records kStatusOutOfBounds (peer = `what`, epoch and
// seen = low words of need and cap) and the caller skips every access; peers
// then time out at their next barrier. Without the flag this is `true`.
B200AR_DEV bool range_ok(const CommCtx& c, int64_t need, int64_t cap, uint32_t what) {
#if defined(B200AR_CHECKS)
  if (need > cap) {
    if (threadIdx.x == 0)
      report_status(c.status, kStatusOutOfBounds, c.rank, what, blockIdx.x, static_cast<uint32_t>(need),
                    static_cast<uint32_t>(cap));
    return false;
  }
#else
  (void)c;
  (void)need;
  (void)cap;
  (void)what;
#endif
  return true;
}

}  // namespace b200ar
