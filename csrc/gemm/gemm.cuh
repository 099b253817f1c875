// Persistent warp-specialised bf16 GEMM for sm_100a: C[M, N] = A[M, K] * B[N, K]^T
// (A and B K-major, fp32 accumulation in TMEM, bf16 output).
//
//   warp 0      : TMA producer (one elected thread), 4-stage smem ring
//   warp 1      : TMEM allocator + tcgen05.mma issuer (one elected thread)
//   warps 2..5  : epilogue; warp w reads TMEM lanes 32*(w % 4) .. +31
//
// Tile 128 x 256 x 64 (one UMMA 128x256x16 per 16-wide K step), two TMEM
// accumulators of 256 columns so the epilogue of tile t overlaps the MMAs of
// tile t+1. TMA loads use no multicast. Every wait is bounded: on expiry the
// kernel records an error, drains its own TMA copies, frees TMEM and returns.
//
// The epilogue is a policy (`Epi::store`) so fused kernels (e.g. GEMM +
// reduce-scatter) reuse the main loop.
#pragma once

#include "tcgen05.cuh"

namespace b200ar {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int THREADS = 192;
constexpr uint32_t A_BYTES = BM * BK * 2;  // 16 KB
constexpr uint32_t B_BYTES = BN * BK * 2;  // 32 KB
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr size_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
// Dynamic shared memory of a kernel instance: ring + barriers + the
// epilogue's staging area (Epi::kStageBytes, 0 for direct stores).
template <class Epi>
constexpr size_t smem_bytes() {
  return SMEM_BYTES + Epi::kStageBytes;
}
constexpr uint32_t TMEM_COLS = 2 * BN;

enum GemmError : int { kGemmOk = 0, kGemmTimeout = 1 };

struct Shape {
  int M, N, K;
  int tiles_m, tiles_n, kblocks;
};

// Plain epilogue: bf16 C, row-major with leading dimension ldc elements.
struct StoreC {
  __nv_bfloat16* c;
  int64_t ldc;
  // Writes 32 consecutive columns [col, col + 32) of `row` (fp32 values v).
  static constexpr size_t kStageBytes = 0;
  __device__ __forceinline__ void store(const Shape& s, int row, int col, const float* v, int, int, uint32_t,
                                        uint8_t*) const {
    if (row >= s.M) return;
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = sm100::pack_bf16x2(v[2 * i], v[2 * i + 1]);
    char* dst = reinterpret_cast<char*>(c + row * ldc + col);
    if (col + 32 <= s.N) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(dst + 16 * i) = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    } else {
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(w);
      for (int i = 0; col + i < s.N && i < 32; ++i) c[row * ldc + col + i] = h[i];
    }
  }
  // tile_done(s, tm, tn) is called by one epilogue thread once the whole tile
  // was stored, for epilogues that set kTileDone.
  static constexpr bool kTileDone = false;
  __device__ __forceinline__ void tile_done(const Shape&, int, int, uint32_t) const {}
  // begin() runs on every thread before the roles split and returns a value
  // handed to every other hook (fused epilogues read their call generation).
  // post() runs on every thread after all tiles, TMEM already released.
  static constexpr bool kPost = false;
  __device__ __forceinline__ uint32_t begin() const { return 0; }
  __device__ __forceinline__ void post(const Shape&, uint32_t, volatile int*) const {}
};

// A-operand source: one tensor map, 128-row boxes.
struct TmapA {
  CUtensorMap map;
  __device__ __forceinline__ void prefetch() const { sm100::prefetch_tmap(&map); }
  __device__ __forceinline__ void load(void* dst, uint64_t* bar, int kx, int tm) const {
    sm100::tma_load_2d(dst, &map, bar, kx, tm * BM);
  }
};

template <class Epi, class ASrc = TmapA>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ ASrc asrc, const __grid_constant__ CUtensorMap tmap_b, Shape s, Epi epi,
                int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* s_err = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* epi_smem = smem + STAGES * STAGE_BYTES + 256;  // Epi::kStageBytes, 16-byte aligned

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntiles = s.tiles_m * s.tiles_n;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&tfull[i], 1);
      sm100::mbar_init(&tempty[i], 4);  // one arrival per epilogue warp
    }
    *s_err = 0;
    sm100::fence_barrier_init();
    asrc.prefetch();
    sm100::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t hook = epi.begin();

  if (warp == 0) {
    // ---------------- TMA producer
    if (sm100::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int i = 0; i < STAGES; ++i) issued[i] = false, issued_phase[i] = 0;
      for (int t = blockIdx.x; t < ntiles && !*s_err; t += gridDim.x) {
        const int tm = t % s.tiles_m, tn = t / s.tiles_m;
        for (int kb = 0; kb < s.kblocks; ++kb) {
          if (!sm100::mbar_wait(&empty[stage], phase ^ 1u)) {
            *s_err = 1;
            break;
          }
          sm100::mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          asrc.load(sA + stage * A_BYTES, &full[stage], kb * BK, tm);
          sm100::tma_load_2d(sB + stage * B_BYTES, &tmap_b, &full[stage], kb * BK, tn * BN);
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
      }
      // Never leave while a TMA copy into this CTA's shared memory is in flight.
      for (int i = 0; i < STAGES; ++i)
        if (issued[i]) sm100::mbar_wait(&full[i], issued_phase[i]);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (sm100::elect_one()) {
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = blockIdx.x; t < ntiles && !*s_err; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1u;
        if (!sm100::mbar_wait(&tempty[acc], acc_phase ^ 1u)) {
          *s_err = 1;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < s.kblocks; ++kb) {
          if (!sm100::mbar_wait(&full[stage], phase)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint64_t da = sm100::smem_desc_sw128(sA + stage * A_BYTES);
          const uint64_t db = sm100::smem_desc_sw128(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // +32 bytes along K = +2 in the encoded start address
            sm100::mma_bf16(d, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          sm100::mma_commit(&empty[stage]);
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
        if (!ok) {
          *s_err = 1;
          break;
        }
        sm100::mma_commit(&tfull[acc]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5)
    const int quarter = warp & 3;
    int local = 0;
    // No early exit on *s_err here: the four epilogue warps leave only through
    // the same expired wait, so they stay in step at the named barrier.
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++local) {
      const int tm = t % s.tiles_m, tn = t / s.tiles_m;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1u;
      if (!sm100::mbar_wait(&tfull[acc], acc_phase)) {
        *s_err = 1;
        break;
      }
      sm100::tc_fence_after();
      const int row = tm * BM + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        sm100::tmem_ld_32x32b_x32(taddr + c, r);
        sm100::tmem_ld_wait();
        const int col = tn * BN + c;
        if (col < s.N || Epi::kStageBytes) epi.store(s, row, col, reinterpret_cast<const float*>(r), tm, tn, hook, epi_smem);
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&tempty[acc]);
      if constexpr (Epi::kTileDone) {
        // All four epilogue warps finished this tile's stores.
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (warp == 2 && lane == 0) epi.tile_done(s, tm, tn, hook);
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if constexpr (Epi::kPost) epi.post(s, hook, s_err);
  if (threadIdx.x == 0 && *s_err) atomicExch(err, kGemmTimeout);
}

}  // namespace gemm
}  // namespace b200ar
