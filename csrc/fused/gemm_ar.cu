// Row-parallel linear fused with its all-reduce (reduce-scatter + all-gather)
// over NVLink, in one persistent sm_100a kernel:
//
//   out[M, N] = sum over ranks of  A_r[M, K] * W_r[N, K]^T
//
// The tcgen05 GEMM main loop (gemm.cuh) computes this rank's partial tiles.
// Output tile t (128 x 256) is owned by rank t % world.
//   A (epilogue, overlapped with the MMAs of the next tile): the partial tile is
//     converted to bf16 straight from TMEM and stored into the owner's inbox
//     row [this rank] with P2P stores; one thread then releases
//     owner.tile_flags[t][rank] = epoch.
//   B (after the CTA's last tile): for the owned tiles assigned to this CTA,
//     wait for every rank's flag, sum the `world` partials in rank order (fp32),
//     write the bf16 result to `out` and to this rank's outbox, release
//     tile_ready[t] = epoch.
//   C: for the other tiles assigned to this CTA, wait for the owner's ready flag
//     and copy the reduced tile from the owner's outbox (P2P loads) into `out`.
// Per rank this moves (N-1)/N of the output each way, like a two-shot
// all-reduce, but the reduce-scatter half rides on the GEMM epilogue.
//
// The reference has no GEMM; this is the "GEMM + reduce-scatter epilogue" path.
// Slots alternate with the call generation exactly as for the plain
// all-reduce; every wait is bounded and reports through the status record.
#include <algorithm>
#include <stdexcept>

#include "../comm/ar_kernels.cuh"
#include "../comm/communicator.h"
#include "../common/trace.h"
#include "../gemm/gemm.cuh"
#include "../gemm/gemm_api.h"
#include "fused.h"

namespace b200ar {

namespace {

constexpr int64_t kTileElems = static_cast<int64_t>(gemm::BM) * gemm::BN;
constexpr int64_t kTileBytes = kTileElems * 2;

struct ArEpi {
  CommCtx ctx;
  char* slot[2][kMaxRanks];
  __nv_bfloat16* out;
  int world;
  int tiles_per_owner;  // ceil(T / world)

  static constexpr bool kTileDone = true;
  static constexpr bool kPost = true;

  __device__ __forceinline__ char* inbox(uint32_t gen, int owner, int src, int ti) const {
    return slot[gen & 1u][owner] + (static_cast<int64_t>(src) * tiles_per_owner + ti) * kTileBytes;
  }
  __device__ __forceinline__ char* outbox(uint32_t gen, int owner, int ti) const {
    return slot[gen & 1u][owner] + (static_cast<int64_t>(world) * tiles_per_owner + ti) * kTileBytes;
  }

  __device__ __forceinline__ uint32_t begin() const {
    __shared__ uint32_t s_gen;
    return read_generation(ctx, &s_gen);
  }

  // Each epilogue warp stages its 32 rows x 128 columns (bf16) in shared
  // memory, then copies them to the owner's inbox two rows (2 x 256 bytes
  // contiguous) per store instruction, so the P2P writes go out as long runs.
  // Row stride 256 bytes; 16-byte chunk j of row r is stored at chunk j ^ (r & 15)
  // so that the row-wise writes and the chunk-wise reads avoid bank conflicts.
  static constexpr int kStageRow = 128 * 2;
  static constexpr size_t kStageBytes = 4 * 32 * kStageRow;

  __device__ __forceinline__ void store(const gemm::Shape& s, int row, int col, const float* v, int tm, int tn,
                                        uint32_t gen, uint8_t* smem) const {
    const int warp = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;
    const int lc = col - tn * gemm::BN;  // 0, 32, ..., 224
    uint8_t* stage = smem + warp * 32 * kStageRow;
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = sm100::pack_bf16x2(v[2 * i], v[2 * i + 1]);
    uint8_t* mine = stage + lane * kStageRow;
    const int chunk0 = (lc % 128) / 8;  // first logical 16-byte chunk of these 32 columns
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<uint4*>(mine + (((chunk0 + i) ^ (lane & 15)) * 16)) =
          make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    if (lc % 128 != 96) return;
    __syncwarp();
    const int t = tn * s.tiles_m + tm;
    const int lr0 = row - lane - tm * gemm::BM;  // first row of this warp within the tile
    char* dst = inbox(gen, t % world, ctx.rank, t / world) +
                (static_cast<int64_t>(lr0) * gemm::BN + (lc / 128) * 128) * 2;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int r = 2 * i + (lane >> 4), c16 = lane & 15;
      const uint4 val = *reinterpret_cast<const uint4*>(stage + r * kStageRow + ((c16 ^ (r & 15)) * 16));
      st_cg(dst + static_cast<int64_t>(r) * gemm::BN * 2 + c16 * 16, val);
    }
    __syncwarp();
  }

  // After the 4 epilogue warps stored the tile (named barrier in the caller).
  __device__ __forceinline__ void tile_done(const gemm::Shape& s, int tm, int tn, uint32_t gen) const {
    const int t = tn * s.tiles_m + tm;
    st_release_sys(&ctx.peers[t % world]->tile_flags[t][ctx.rank], gen + 1u);
  }

  // Bounded wait on a flag (one thread); false on timeout (status recorded).
  __device__ bool wait_flag(const uint32_t* f, uint32_t want, int peer, int tile) const {
    uint32_t seen = ld_acquire_sys(f);
    if (epoch_reached(seen, want)) return true;
    const uint64_t start = global_ns();
    for (uint32_t i = 1;; ++i) {
      seen = ld_acquire_sys(f);
      if (epoch_reached(seen, want)) return true;
      if ((i & 63u) == 0u && global_ns() - start > ctx.timeout_ns) {
        report_status(ctx.status, kStatusTimeout, ctx.rank, peer, tile, want, seen);
        return false;
      }
    }
  }

  __device__ void post(const gemm::Shape& s, uint32_t gen, volatile int* s_err) const {
    const uint32_t epoch = gen + 1u;
    const int T = s.tiles_m * s.tiles_n;
    const int r = ctx.rank;
    __shared__ int s_fail;
    if (threadIdx.x == 0) s_fail = 0;
    __syncthreads();
    // B: reduce owned tiles.
    for (int t = r + world * blockIdx.x; t < T; t += world * gridDim.x) {
      const int ti = t / world;
      if (threadIdx.x < world && !wait_flag(&ctx.self->tile_flags[t][threadIdx.x], epoch, threadIdx.x, t))
        atomicExch(&s_fail, 1);
      __syncthreads();
      if (s_fail) break;
      const int tm = t % s.tiles_m, tn = t / s.tiles_m;
      char* ob = outbox(gen, r, ti);
      constexpr int kPk = static_cast<int>(kTileBytes / 16);
      constexpr int U = 4;  // packets in flight per thread
      for (int p0 = threadIdx.x; p0 < kPk; p0 += U * blockDim.x) {
        float acc[U][8];
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int p = p0 + u * blockDim.x;
          v[u] = p < kPk ? ld_cg(inbox(gen, r, 0, ti) + static_cast<int64_t>(p) * 16) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) unpack_set<__nv_bfloat16>(v[u], acc[u]);
        for (int q = 1; q < world; ++q) {
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int p = p0 + u * blockDim.x;
            v[u] = p < kPk ? ld_cg(inbox(gen, r, q, ti) + static_cast<int64_t>(p) * 16) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int u = 0; u < U; ++u) unpack_add<__nv_bfloat16>(v[u], acc[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int p = p0 + u * blockDim.x;
          if (p >= kPk) continue;
          const uint4 o = pack<__nv_bfloat16>(acc[u]);
          st_cg(ob + static_cast<int64_t>(p) * 16, o);
          const int lr = p / (gemm::BN / 8), lc = (p % (gemm::BN / 8)) * 8;
          const int row = tm * gemm::BM + lr, col = tn * gemm::BN + lc;
          if (row < s.M && col < s.N) st_out(out + static_cast<int64_t>(row) * s.N + col, o);
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) st_release_sys(&ctx.self->tile_ready[t], epoch);
    }
    // C: gather the tiles reduced by the other ranks.
    if (!s_fail) {
      for (int t = blockIdx.x; t < T; t += gridDim.x) {
        const int owner = t % world;
        if (owner == r) continue;
        if (threadIdx.x == 0 && !wait_flag(&ctx.peers[owner]->tile_ready[t], epoch, owner, t)) s_fail = 1;
        __syncthreads();
        if (s_fail) break;
        const int tm = t % s.tiles_m, tn = t / s.tiles_m;
        const char* ob = outbox(gen, owner, t / world);
        constexpr int kPk = static_cast<int>(kTileBytes / 16);
        constexpr int U = 8;  // remote loads in flight per thread
        for (int p0 = threadIdx.x; p0 < kPk; p0 += U * blockDim.x) {
          uint4 v[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int p = p0 + u * blockDim.x;
            v[u] = p < kPk ? ld_cg(ob + static_cast<int64_t>(p) * 16) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int p = p0 + u * blockDim.x;
            const int lr = p / (gemm::BN / 8), lc = (p % (gemm::BN / 8)) * 8;
            const int row = tm * gemm::BM + lr, col = tn * gemm::BN + lc;
            if (p < kPk && row < s.M && col < s.N) st_out(out + static_cast<int64_t>(row) * s.N + col, v[u]);
          }
        }
        __syncthreads();
      }
    }
    if (s_fail && threadIdx.x == 0) *s_err = 1;
    finish_generation(ctx, gen);
  }
};

}  // namespace

int64_t gemm_ar_slot_bytes(int64_t M, int64_t N, int world) {
  const int64_t T = ((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
  const int64_t tpo = (T + world - 1) / world;
  return (world + 1) * tpo * kTileBytes;
}

bool gemm_ar_supported(Communicator& comm, int64_t M, int64_t N) {
  const int64_t T = ((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
  return comm.slots_registered() && T >= comm.world() && T <= kMaxTiles && N % 8 == 0 &&
         gemm_ar_slot_bytes(M, N, comm.world()) <= comm.slot_capacity();
}

void gemm_allreduce(Communicator& comm, cudaStream_t stream, const void* A, const void* W, void* out, int64_t M,
                    int64_t N, int64_t K, int* err) {
  TraceRange trace("b200ar.gemm_allreduce");
  comm.check_status();
  B200AR_CHECK(gemm_ar_supported(comm, M, N),
               "fused GEMM + all-reduce of " << M << "x" << N << " needs at least world tiles, at most " << kMaxTiles
                                             << " tiles and " << gemm_ar_slot_bytes(M, N, comm.world())
                                             << " slot bytes (capacity " << comm.slot_capacity() << ")");
  const gemm::Shape s = gemm_shape(M, N, K);
  const gemm::TmapA ta{make_tmap_bf16_2d(A, M, K, K, gemm::BM, gemm::BK)};
  const CUtensorMap tb = make_tmap_bf16_2d(W, N, K, K, gemm::BN, gemm::BK);
  ArEpi epi{};
  comm.fill_ctx(&epi.ctx);
  for (int sl = 0; sl < 2; ++sl)
    for (int i = 0; i < comm.world(); ++i) epi.slot[sl][i] = comm.slot_ptr(sl, i);
  epi.out = static_cast<__nv_bfloat16*>(out);
  epi.world = comm.world();
  epi.tiles_per_owner = (s.tiles_m * s.tiles_n + comm.world() - 1) / comm.world();
  auto kern = gemm::gemm_kernel<ArEpi>;
  static PerDeviceOnce smem_attr;
  smem_attr([&] {
    B200AR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(gemm::smem_bytes<ArEpi>())));
  });
  // Every CTA must be resident (ranks wait on each other's CTAs): one per SM.
  int dev = 0, sms = 0;
  B200AR_CUDA(cudaGetDevice(&dev));
  B200AR_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = std::max(1, std::min(sms, kMaxCTAs));
  kern<<<grid, gemm::THREADS, gemm::smem_bytes<ArEpi>(), stream>>>(ta, tb, s, epi, err);
  B200AR_CUDA(cudaGetLastError());
  comm.count_launch();
}

}  // namespace b200ar
