// All-reduce kernels of b200ar for sm_100a (sum, fp32 accumulation).
//
// All kernels are multi-CTA; CTA j of every rank works on the same packet range
// and synchronises only with CTA j of the peers (per-CTA flags), so the ranks
// must launch identical grids for the same call. Data moves as 16-byte packets
// with P2P loads/stores over NVLink to peer HBM mapped with CUDA IPC.
//
// Variants (kernel <-> reference kernel):
//  * oneshot_push  <-> fused_push_reduce_kernel (pcie_allreduce.cu:182-220):
//    push own input into every rank's slot[rank], barrier, reduce locally.
//    The reference runs it on a single CTA; here every CTA pushes its chunk.
//  * oneshot_pull  <-> fused_pull_reduce_kernel (cu:227-257): copy-in fused,
//    barrier, rotated pull-reduce from every peer.
//  * twoshot (new): push-reduce-scatter, barrier, reduce own part, barrier,
//    pull-all-gather. Moves 2(N-1)/N of the message per direction per rank.
//  * twoshot_push (new): the same traffic with the reduced parts pushed to
//    the peers while they are reduced, then a local copy.
//  * registered    <-> pcie_allreduce_kernel (cu:261-276): pull directly from
//    registered peer buffers. Adds the end barrier the reference lacks, so a
//    rank cannot overwrite its input while a peer still reads it.
#pragma once

#include "../common/device.cuh"

namespace b200ar {

constexpr int kArThreads = 512;

struct ArArgs {
  CommCtx ctx;
  char* slot[2][kMaxRanks];  // base of slot s on every rank (peer mappings)
  const char* in;            // local input
  char* out;                 // local output
  const RankData* rd;        // registered variant only
  int64_t packets;           // message size in 16-byte packets
  char* lam[kMaxRanks];      // Lamport region of every rank (peer mappings)
  int64_t lam_cap;           // bytes per (buffer, source) block of the Lamport region
#if defined(B200AR_CHECKS)
  int64_t slot_cap;          // bytes per slot (checked builds verify footprints against it)
#endif
};

// Checked builds: skip the whole call (but keep the generation in step) when
// the footprint of this call does not fit its buffer. `what` names the buffer
// in the status record: 1 slot, 2 Lamport block.
#if defined(B200AR_CHECKS)
#define B200AR_ENTRY_RANGE(need, cap, what)            \
  if (!range_ok(a.ctx, (need), (cap), (what))) {       \
    finish_generation(a.ctx, gen);                     \
    return;                                            \
  }
#else
#define B200AR_ENTRY_RANGE(need, cap, what)
#endif

// Fills d[k] = base[(rank + k) % N] without dynamic indexing of a local array.
template <int N>
B200AR_DEV void rotate_ptrs(char* const* base, int rank, char** d) {
#pragma unroll
  for (int k = 0; k < N; ++k) {
    char* v = nullptr;
    const int want = (rank + k) % N;
#pragma unroll
    for (int p = 0; p < N; ++p)
      if (p == want) v = base[p];
    d[k] = v;
  }
}

template <typename T, int N>
__global__ void __launch_bounds__(kArThreads) oneshot_push_kernel(ArArgs a) {
  __shared__ uint32_t s_gen;
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int slot = gen & 1u;
  const int r = a.ctx.rank;
  const int64_t P = a.packets;
  const int64_t b = part_begin(P, gridDim.x, blockIdx.x);
  const int64_t e = part_begin(P, gridDim.x, blockIdx.x + 1);

  B200AR_ENTRY_RANGE(static_cast<int64_t>(N) * P * 16, a.slot_cap, 1u)

  char* dst[N];
  rotate_ptrs<N>(a.slot[slot], r, dst);
  const int64_t my_off = static_cast<int64_t>(r) * P * 16;

  for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) {
    const uint4 v = ld_in(a.in + i * 16);
#pragma unroll
    for (int k = 0; k < N; ++k) st_cg(dst[k] + my_off + i * 16, v);
  }

  if (cta_barrier<N>(a.ctx, blockIdx.x, epoch_of(gen, 0))) {
    const char* mine = a.slot[slot][r];
    for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) {
      uint4 v[N];
#pragma unroll
      for (int q = 0; q < N; ++q) v[q] = ld_cg(mine + (static_cast<int64_t>(q) * P + i) * 16);
      float acc[PackTraits<T>::kElems];
      unpack_set<T>(v[0], acc);
#pragma unroll
      for (int q = 1; q < N; ++q) unpack_add<T>(v[q], acc);
      st_out(a.out + i * 16, pack<T>(acc));
    }
  }
  finish_generation(a.ctx, gen);
}

template <typename T, int N>
__global__ void __launch_bounds__(kArThreads) oneshot_pull_kernel(ArArgs a) {
  __shared__ uint32_t s_gen;
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int slot = gen & 1u;
  const int r = a.ctx.rank;
  const int64_t P = a.packets;
  const int64_t b = part_begin(P, gridDim.x, blockIdx.x);
  const int64_t e = part_begin(P, gridDim.x, blockIdx.x + 1);

  // Peers are summed in rank order 0..N-1 on every rank, so all ranks get
  // bitwise identical results (the reference rotated the order per rank,
  // pcie_allreduce.cu:248-253, which makes results rank dependent).
  B200AR_ENTRY_RANGE(P * 16, a.slot_cap, 1u)
  char* const* src = a.slot[slot];
  char* mine = src[r];
  for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) st_cg(mine + i * 16, ld_in(a.in + i * 16));

  if (cta_barrier<N>(a.ctx, blockIdx.x, epoch_of(gen, 0))) {
    for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) {
      uint4 v[N];
#pragma unroll
      for (int k = 0; k < N; ++k) v[k] = ld_cg(src[k] + i * 16);
      float acc[PackTraits<T>::kElems];
      unpack_set<T>(v[0], acc);
#pragma unroll
      for (int k = 1; k < N; ++k) unpack_add<T>(v[k], acc);
      st_out(a.out + i * 16, pack<T>(acc));
    }
  }
  finish_generation(a.ctx, gen);
}

// Two-shot. Slot layout on every rank (in packets, part = ceil(P / N)):
//   [0, N*part)        reduce-scatter inbox, row q holds rank q's copy of this rank's part
//   [N*part, (N+1)*part) all-gather outbox: this rank's reduced part
template <typename T, int N>
__global__ void __launch_bounds__(kArThreads) twoshot_kernel(ArArgs a) {
  __shared__ uint32_t s_gen;
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int slot = gen & 1u;
  const int r = a.ctx.rank;
  const int64_t P = a.packets;
  const int64_t part = (P + N - 1) / N;
  const int G = gridDim.x;
  const int j = blockIdx.x;
  B200AR_ENTRY_RANGE(static_cast<int64_t>(N + 1) * part * 16, a.slot_cap, 1u)

  char* peer[N];  // peer[k] = slot base of rank (r + k) % N
  rotate_ptrs<N>(a.slot[slot], r, peer);

  // Sub-range of part p = (r + k) % N handled by this CTA: absolute packet
  // start ab[k], start relative to the part rb[k], length ln[k].
  int64_t ab[N];
  int rb[N], ln[N];
  int smax = 0;
#pragma unroll
  for (int k = 0; k < N; ++k) {
    const int p = (r + k) % N;
    const int64_t pb = part_begin(P, N, p);
    const int64_t plen = part_begin(P, N, p + 1) - pb;
    const int64_t sb = part_begin(plen, G, j);
    rb[k] = static_cast<int>(sb);
    ln[k] = static_cast<int>(part_begin(plen, G, j + 1) - sb);
    ab[k] = pb + sb;
    smax = ln[k] > smax ? ln[k] : smax;
  }

  // Phase 1: scatter. Rank r's copy of part p goes to row r of p's inbox.
  // With few ranks, U offsets per thread keep about 8 packets in flight.
  constexpr int U = N >= 8 ? 1 : (8 + N - 1) / N;
  const int64_t row = static_cast<int64_t>(r) * part;
  for (int o0 = threadIdx.x; o0 < smax; o0 += U * blockDim.x) {
    uint4 v[U][N];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int o = o0 + u * blockDim.x;
#pragma unroll
      for (int k = 0; k < N; ++k)
        if (o < ln[k]) v[u][k] = ld_in(a.in + (ab[k] + o) * 16);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int o = o0 + u * blockDim.x;
#pragma unroll
      for (int k = 0; k < N; ++k)
        if (o < ln[k]) st_cg(peer[k] + (row + rb[k] + o) * 16, v[u][k]);
    }
  }

  bool ok = cta_barrier<N>(a.ctx, j, epoch_of(gen, 0));

  // Phase 2: reduce own part (k == 0), write result to output and outbox.
  if (ok) {
    char* mine = peer[0];
    for (int o = threadIdx.x; o < ln[0]; o += blockDim.x) {
      const int64_t rel = rb[0] + o;
      uint4 v[N];
#pragma unroll
      for (int q = 0; q < N; ++q) v[q] = ld_cg(mine + (static_cast<int64_t>(q) * part + rel) * 16);
      float acc[PackTraits<T>::kElems];
      unpack_set<T>(v[0], acc);
#pragma unroll
      for (int q = 1; q < N; ++q) unpack_add<T>(v[q], acc);
      const uint4 res = pack<T>(acc);
      st_out(a.out + (ab[0] + o) * 16, res);
      st_cg(mine + (static_cast<int64_t>(N) * part + rel) * 16, res);
    }
  }

  ok = cta_barrier<N>(a.ctx, j, epoch_of(gen, 1)) && ok;

  // Phase 3: gather reduced parts of the peers.
  if (ok) {
    const int64_t outbox = static_cast<int64_t>(N) * part;
    for (int o0 = threadIdx.x; o0 < smax; o0 += U * blockDim.x) {
      uint4 v[U][N];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int o = o0 + u * blockDim.x;
#pragma unroll
        for (int k = 1; k < N; ++k)
          if (o < ln[k]) v[u][k] = ld_cg(peer[k] + (outbox + rb[k] + o) * 16);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int o = o0 + u * blockDim.x;
#pragma unroll
        for (int k = 1; k < N; ++k)
          if (o < ln[k]) st_out(a.out + (ab[k] + o) * 16, v[u][k]);
      }
    }
  }
  finish_generation(a.ctx, gen);
}

// Two-shot with a pushed all-gather. Slot layout on every rank (in packets,
// part = ceil(P / N)):
//   [0, N*part)          reduce-scatter inbox, row q = rank q's copy of this rank's part
//   [N*part, 2*N*part)   gathered parts, row p = rank p's reduced part
// Phase 1 is the two-shot scatter. In phase 2 each rank reduces its part and
// stores the result straight into row r of every peer's gathered area
// (stores, not the pulls of twoshot_kernel's phase 3), so that the NVLink
// transfer of the reduced part overlaps the reduction; phase 3 is a local copy
// of the gathered rows to the output.
template <typename T, int N>
__global__ void __launch_bounds__(kArThreads) twoshot_push_kernel(ArArgs a) {
  __shared__ uint32_t s_gen;
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int slot = gen & 1u;
  const int r = a.ctx.rank;
  const int64_t P = a.packets;
  const int64_t part = (P + N - 1) / N;
  const int G = gridDim.x;
  const int j = blockIdx.x;
  B200AR_ENTRY_RANGE(static_cast<int64_t>(2 * N) * part * 16, a.slot_cap, 1u)

  char* peer[N];  // peer[k] = slot base of rank (r + k) % N
  rotate_ptrs<N>(a.slot[slot], r, peer);
  int64_t ab[N];
  int rb[N], ln[N];
  int smax = 0;
#pragma unroll
  for (int k = 0; k < N; ++k) {
    const int p = (r + k) % N;
    const int64_t pb = part_begin(P, N, p);
    const int64_t plen = part_begin(P, N, p + 1) - pb;
    const int64_t sb = part_begin(plen, G, j);
    rb[k] = static_cast<int>(sb);
    ln[k] = static_cast<int>(part_begin(plen, G, j + 1) - sb);
    ab[k] = pb + sb;
    smax = ln[k] > smax ? ln[k] : smax;
  }

  // Phase 1: scatter (as twoshot_kernel).
  constexpr int U = N >= 8 ? 1 : (8 + N - 1) / N;
  const int64_t row = static_cast<int64_t>(r) * part;
  for (int o0 = threadIdx.x; o0 < smax; o0 += U * blockDim.x) {
    uint4 v[U][N];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int o = o0 + u * blockDim.x;
#pragma unroll
      for (int k = 0; k < N; ++k)
        if (o < ln[k]) v[u][k] = ld_in(a.in + (ab[k] + o) * 16);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int o = o0 + u * blockDim.x;
#pragma unroll
      for (int k = 0; k < N; ++k)
        if (o < ln[k]) st_cg(peer[k] + (row + rb[k] + o) * 16, v[u][k]);
    }
  }

  bool ok = cta_barrier<N>(a.ctx, j, epoch_of(gen, 0));

  // Phase 2: reduce own part, write it to the output and push it to every peer.
  const int64_t gathered = static_cast<int64_t>(N) * part;
  if (ok) {
    char* mine = peer[0];
    for (int o = threadIdx.x; o < ln[0]; o += blockDim.x) {
      const int64_t rel = rb[0] + o;
      uint4 v[N];
#pragma unroll
      for (int q = 0; q < N; ++q) v[q] = ld_cg(mine + (static_cast<int64_t>(q) * part + rel) * 16);
      float acc[PackTraits<T>::kElems];
      unpack_set<T>(v[0], acc);
#pragma unroll
      for (int q = 1; q < N; ++q) unpack_add<T>(v[q], acc);
      const uint4 res = pack<T>(acc);
      st_out(a.out + (ab[0] + o) * 16, res);
#pragma unroll
      for (int k = 1; k < N; ++k) st_cg(peer[k] + (gathered + row + rel) * 16, res);
    }
  }

  ok = cta_barrier<N>(a.ctx, j, epoch_of(gen, 1)) && ok;

  // Phase 3: copy the peers' reduced parts from the gathered rows.
  if (ok) {
    const char* mine = peer[0];
    for (int o0 = threadIdx.x; o0 < smax; o0 += U * blockDim.x) {
      uint4 v[U][N];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int o = o0 + u * blockDim.x;
#pragma unroll
        for (int k = 1; k < N; ++k) {
          const int64_t prow = static_cast<int64_t>((r + k) % N) * part;
          if (o < ln[k]) v[u][k] = ld_cg(mine + (gathered + prow + rb[k] + o) * 16);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int o = o0 + u * blockDim.x;
#pragma unroll
        for (int k = 1; k < N; ++k)
          if (o < ln[k]) st_out(a.out + (ab[k] + o) * 16, v[u][k]);
      }
    }
  }
  finish_generation(a.ctx, gen);
}

// Pull-reduce straight from registered peer buffers (no staging copy).
template <typename T, int N>
__global__ void __launch_bounds__(kArThreads) registered_kernel(ArArgs a) {
  __shared__ uint32_t s_gen;
  __shared__ const char* s_ptr[kMaxRanks];
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  if (threadIdx.x < N) s_ptr[threadIdx.x] = static_cast<const char*>(a.rd->ptrs[threadIdx.x]);  // rank order
  const int64_t P = a.packets;
  const int64_t b = part_begin(P, gridDim.x, blockIdx.x);
  const int64_t e = part_begin(P, gridDim.x, blockIdx.x + 1);

  if (cta_barrier<N>(a.ctx, blockIdx.x, epoch_of(gen, 0))) {
    const char* src[N];
#pragma unroll
    for (int k = 0; k < N; ++k) src[k] = s_ptr[k];
    for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) {
      uint4 v[N];
#pragma unroll
      for (int k = 0; k < N; ++k) v[k] = ld_cg(src[k] + i * 16);
      float acc[PackTraits<T>::kElems];
      unpack_set<T>(v[0], acc);
#pragma unroll
      for (int k = 1; k < N; ++k) unpack_add<T>(v[k], acc);
      st_out(a.out + i * 16, pack<T>(acc));
    }
  }
  // End barrier: no rank leaves (and overwrites its input) while peers read it.
  cta_barrier<N>(a.ctx, blockIdx.x, epoch_of(gen, 1));
  finish_generation(a.ctx, gen);
}

// ---------------------------------------------------------------------------
// One-shot Lamport: no barrier and no fence. Every rank writes its packets
// straight into the peers' current buffer; a receiver polls its own buffer
// until no 32-bit word of a packet is the marker, sums in rank order, then
// restores the marker so the buffer is ready for its next use.
//
// Buffer b = gen % 3 on rank r is [N sources][lam_cap bytes]. Reuse is safe:
// a writer reaches the same buffer again only at gen + 3, after it consumed
// this rank's data of gen + 1 and gen + 2, which this rank pushed after it had
// restored the markers of gen (stream order).
// ---------------------------------------------------------------------------

B200AR_DEV uint4 ld_volatile16(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

B200AR_DEV bool lamport_ready(const uint4& v) {
  return v.x != kLamportMarker && v.y != kLamportMarker && v.z != kLamportMarker && v.w != kLamportMarker;
}

// Replaces -0.0 elements by +0.0 so that no word equals the marker.
template <typename T>
B200AR_DEV uint32_t lamport_clean(uint32_t w) {
  if constexpr (sizeof(T) == 4) {
    return w == kLamportMarker ? 0u : w;
  } else {
    if ((w & 0xffffu) == 0x8000u) w &= 0xffff0000u;
    if ((w >> 16) == 0x8000u) w &= 0x0000ffffu;
    return w;
  }
}

template <typename T, int N>
__global__ void __launch_bounds__(kArThreads) oneshot_lamport_kernel(ArArgs a) {
  __shared__ uint32_t s_gen;
  const int r = a.ctx.rank;
  const int64_t P = a.packets;
  const int64_t b = part_begin(P, gridDim.x, blockIdx.x);
  const int64_t e = part_begin(P, gridDim.x, blockIdx.x + 1);
  // The first input packet is loaded before the generation so that the two
  // cold loads overlap (decode-size messages have one packet per thread).
  const int64_t i0 = b + threadIdx.x;
  uint4 first = make_uint4(0u, 0u, 0u, 0u);
  if (i0 < e) first = ld_in(a.in + i0 * 16);
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int64_t buf_off = static_cast<int64_t>(gen % kLamportBuffers) * N * a.lam_cap;
  B200AR_ENTRY_RANGE(P * 16, a.lam_cap, 2u)

  char* dst[N];
  rotate_ptrs<N>(a.lam, r, dst);
  const int64_t my_off = buf_off + static_cast<int64_t>(r) * a.lam_cap;
  for (int64_t i = i0; i < e; i += blockDim.x) {
    uint4 v = i == i0 ? first : ld_in(a.in + i * 16);
    v.x = lamport_clean<T>(v.x);
    v.y = lamport_clean<T>(v.y);
    v.z = lamport_clean<T>(v.z);
    v.w = lamport_clean<T>(v.w);
#pragma unroll
    for (int k = 0; k < N; ++k) st_cg(dst[k] + my_off + i * 16, v);
  }

  char* mine = a.lam[r] + buf_off;
  const uint4 marker = make_uint4(kLamportMarker, kLamportMarker, kLamportMarker, kLamportMarker);
  bool fail = false;
  for (int64_t i = b + threadIdx.x; i < e && !fail; i += blockDim.x) {
    uint4 v[N];
#pragma unroll
    for (int q = 0; q < N; ++q) v[q] = ld_volatile16(mine + q * a.lam_cap + i * 16);
#pragma unroll
    for (int q = 0; q < N; ++q) {
      if (!lamport_ready(v[q]) && !fail) {
        const uint64_t start = global_ns();
        uint32_t spins = 0;
        while (!lamport_ready(v[q] = ld_volatile16(mine + q * a.lam_cap + i * 16))) {
          if ((++spins & 63u) == 0u && global_ns() - start > a.ctx.timeout_ns) {
            report_status(a.ctx.status, kStatusTimeout, r, q, blockIdx.x, gen, 0);
            fail = true;
            break;
          }
        }
      }
    }
    if (fail) break;
    float acc[PackTraits<T>::kElems];
    unpack_set<T>(v[0], acc);
#pragma unroll
    for (int q = 1; q < N; ++q) unpack_add<T>(v[q], acc);
    st_out(a.out + i * 16, pack<T>(acc));
#pragma unroll
    for (int q = 0; q < N; ++q) st_cg(mine + q * a.lam_cap + i * 16, marker);
  }
  finish_generation(a.ctx, gen);
}

// Fills `words` 32-bit words at p with `value` (Lamport region initialisation).
__global__ void fill_u32_kernel(uint32_t* p, int64_t words, uint32_t value);

}  // namespace b200ar

namespace b200ar {
// Host launcher for the kernels above (ar_kernels.cu).
void launch_ar_kernel(int variant, DType dt, int world, int ctas, int threads, const ArArgs& args,
                      cudaStream_t stream);
// Fills a device range with the Lamport marker.
void launch_lamport_init(void* p, int64_t bytes, cudaStream_t stream);
// Occupancy (resident CTAs per SM at kArThreads threads) of a variant's kernel.
int ar_blocks_per_sm(int variant, DType dt, int world);
int nvls_blocks_per_sm(DType dt, int world);
// World size 1: out = in (16-byte packets) with a b200ar kernel.
void launch_copy(const void* in, void* out, int64_t packets, cudaStream_t stream);
}  // namespace b200ar
