// All-gather fused into the prologue of a column-parallel GEMM (sm_100a):
//
//   Y[M, N] = X[M, K] * W[N, K]^T,   X = concat over ranks of X_r[M / world, K]
//
// Step 1 (publish kernel): every rank copies its shard X_r into its current
// slot (the slot alternates with the call generation) and passes a per-CTA
// cross-rank barrier, so afterwards every shard is readable by every rank.
// Step 2 (GEMM): the TMA producer fetches each 16-row slice of an A tile
// straight from the shard owner's slot over NVLink (plain TMA loads from peer
// memory, never multicast); no gathered copy of X is materialised.
//
// Rows per rank must be a multiple of 16 (one TMA box per 16-row slice).
// The reference has no GEMM; this is the "all-gather + GEMM prologue" path.
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

constexpr int kSliceRows = 16;

// A-operand source gathering 16-row slices from the rank that owns them.
// The publish kernel ran with generation g and left g + 1 in the signal block,
// so the shards sit in slot g & 1 = (current - 1) & 1 on every rank.
struct GatherA {
  CUtensorMap maps[2][kMaxRanks];  // rank p's shard [rows_per_rank, K] in its slot s
  const uint32_t* gen;             // this rank's generation counter
  int rows_per_rank;
  int world;
  __device__ __forceinline__ void prefetch() const {
    for (int p = 0; p < world; ++p) {
      sm100::prefetch_tmap(&maps[0][p]);
      sm100::prefetch_tmap(&maps[1][p]);
    }
  }
  __device__ __forceinline__ void load(void* dst, uint64_t* bar, int kx, int tm) const {
    const int sl = static_cast<int>((*reinterpret_cast<const volatile uint32_t*>(gen) - 1u) & 1u);
#pragma unroll
    for (int i = 0; i < gemm::BM / kSliceRows; ++i) {
      const int row = tm * gemm::BM + i * kSliceRows;
      int p = row / rows_per_rank;
      int local = row - p * rows_per_rank;
      if (p >= world) {  // beyond M: read past the last shard (zero fill keeps the byte count)
        p = world - 1;
        local = rows_per_rank;
      }
      sm100::tma_load_2d(static_cast<char*>(dst) + i * kSliceRows * 128, &maps[sl][p], bar, kx, local);
    }
  }
};

struct PublishArgs {
  CommCtx ctx;
  char* slot[2];  // this rank's two slots
  const char* x;
  int64_t packets;
};

template <int N>
__global__ void __launch_bounds__(kArThreads) publish_kernel(PublishArgs a) {
  __shared__ uint32_t s_gen;
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  char* dst = a.slot[gen & 1u];
  const int64_t b = part_begin(a.packets, gridDim.x, blockIdx.x);
  const int64_t e = part_begin(a.packets, gridDim.x, blockIdx.x + 1);
  for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) st_cg(dst + i * 16, ld_in(a.x + i * 16));
  cta_barrier<N>(a.ctx, blockIdx.x, epoch_of(gen, 0));
  finish_generation(a.ctx, gen);
}

void launch_publish(int world, int ctas, const PublishArgs& a, cudaStream_t s) {
  switch (world) {
    case 2: publish_kernel<2><<<ctas, kArThreads, 0, s>>>(a); break;
    case 3: publish_kernel<3><<<ctas, kArThreads, 0, s>>>(a); break;
    case 4: publish_kernel<4><<<ctas, kArThreads, 0, s>>>(a); break;
    case 5: publish_kernel<5><<<ctas, kArThreads, 0, s>>>(a); break;
    case 6: publish_kernel<6><<<ctas, kArThreads, 0, s>>>(a); break;
    case 7: publish_kernel<7><<<ctas, kArThreads, 0, s>>>(a); break;
    case 8: publish_kernel<8><<<ctas, kArThreads, 0, s>>>(a); break;
    default: throw std::invalid_argument("all-gather GEMM needs 2..8 ranks");
  }
}

}  // namespace

bool ag_gemm_supported(Communicator& comm, int64_t rows_per_rank, int64_t K) {
  return comm.slots_registered() && comm.world() >= 2 && rows_per_rank % kSliceRows == 0 && rows_per_rank > 0 &&
         K % 8 == 0 && rows_per_rank * K * 2 <= comm.slot_capacity();
}

void ag_gemm(Communicator& comm, cudaStream_t stream, const void* x_shard, const void* W, void* Y,
             int64_t rows_per_rank, int64_t N, int64_t K, int* err) {
  TraceRange trace("b200ar.ag_gemm");
  comm.check_status();
  B200AR_CHECK(ag_gemm_supported(comm, rows_per_rank, K),
               "all-gather GEMM needs rows per rank a multiple of " << kSliceRows << " and a shard of at most "
                                                                    << comm.slot_capacity() << " bytes");
  B200AR_CHECK(N % 8 == 0 && reinterpret_cast<uintptr_t>(Y) % 16 == 0, "Y must have 16-byte aligned rows");
  const int world = comm.world();
  const int rank = comm.rank();
  // 1. publish this rank's shard.
  PublishArgs pa{};
  comm.fill_ctx(&pa.ctx);
  pa.slot[0] = comm.slot_ptr(0, rank);
  pa.slot[1] = comm.slot_ptr(1, rank);
  pa.x = static_cast<const char*>(x_shard);
  pa.packets = rows_per_rank * K * 2 / 16;
  const int pctas = static_cast<int>(std::clamp<int64_t>((pa.packets + 2 * kArThreads - 1) / (2 * kArThreads), 1, 148));
  launch_publish(world, pctas, pa, stream);
  comm.count_launch();
  // 2. GEMM whose producer gathers A from the shards (maps for both slots; the
  // device picks the one the publish kernel filled).
  const int64_t M = rows_per_rank * world;
  const gemm::Shape s = gemm_shape(M, N, K);
  const CUtensorMap tb = make_tmap_bf16_2d(W, N, K, K, gemm::BN, gemm::BK);
  gemm::StoreC epi{static_cast<__nv_bfloat16*>(Y), N};
  GatherA ga{};
  ga.gen = &comm.self_signal()->gen;
  ga.rows_per_rank = static_cast<int>(rows_per_rank);
  ga.world = world;
  for (int sl = 0; sl < 2; ++sl)
    for (int p = 0; p < world; ++p)
      ga.maps[sl][p] = make_tmap_bf16_2d(comm.slot_ptr(sl, p), rows_per_rank, K, K, kSliceRows, gemm::BK);
  auto kern = gemm::gemm_kernel<gemm::StoreC, GatherA>;
  static PerDeviceOnce smem_attr;
  smem_attr([&] {
    B200AR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(gemm::smem_bytes<gemm::StoreC>())));
  });
  kern<<<gemm_grid(s, 0), gemm::THREADS, gemm::smem_bytes<gemm::StoreC>(), stream>>>(ga, tb, s, epi, err);
  B200AR_CUDA(cudaGetLastError());
  comm.count_launch();
}

}  // namespace b200ar
