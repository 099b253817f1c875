// Persistent bf16 GEMM on CTA pairs (tcgen05 cta_group::2) for sm_100a:
// C[M, N] = A[M, K] * B[N, K]^T, A and B K-major, fp32 accumulation in TMEM.
//
// A cluster of two CTAs (one per SM of a TPC pair) computes 256 x 256 output
// tiles: CTA r loads rows [128 r, 128 r + 128) of the tile's A block and of its
// B block into its own shared memory, and the leader (rank 0) issues
// tcgen05.mma.cta_group::2 with M = 256, N = 256, which reads both CTAs'
// shared memory and accumulates rows [128 r, ...) of the tile in CTA r's TMEM.
// Per SM and K block of 64 that is 32 KB of operand traffic instead of the
// 48 KB of a 128 x 256 single-CTA tile for the same MMA work.
//
//   warp 0      TMA producer in both CTAs (no multicast; completion counted on
//               the leader's `full` barrier)
//   warp 1      TMEM allocation in both CTAs; MMA issuer in the leader
//   warps 2..5  epilogue in both CTAs (own TMEM lanes, own 128 rows)
//
// Ring of 6 stages of 32 KB per CTA; two TMEM accumulators of 256 columns
// (all 512) so a tile's epilogue overlaps the next tile's MMAs. Every wait is
// bounded: on expiry the kernel records an error and unwinds.
#pragma once

#include "gemm.cuh"

namespace b200ar {
namespace gemm2 {

constexpr int BM = 256;  // rows of a pair tile (128 per CTA)
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int THREADS = 192;
constexpr uint32_t A_BYTES = 128 * BK * 2;  // 16 KB per CTA
constexpr uint32_t B_BYTES = 128 * BK * 2;  // 16 KB per CTA (half of the tile's 256 B rows)
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr size_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint32_t TMEM_COLS = 2 * BN;

struct Shape {
  int M, N, K;
  int tiles_m, tiles_n, kblocks;
};

__global__ void __launch_bounds__(THREADS, 1)
    gemm2sm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, Shape s,
                   __nv_bfloat16* c, int64_t ldc, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2]
  uint64_t* tempty = tfull + 2;       // [2] (leader's: 8 arrivals, 4 warps of each CTA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* s_err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = sm100::cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int ntiles = s.tiles_m * s.tiles_n;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&tfull[i], 1);
      sm100::mbar_init(&tempty[i], 8);
    }
    *s_err = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmap_a);
    sm100::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    sm100::tmem_alloc_pair(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish_pair();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (sm100::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool issued[STAGES] = {};
      uint32_t issued_phase[STAGES] = {};
      for (int t = pair; t < ntiles && !*s_err; t += npairs) {
        const int tm = t % s.tiles_m, tn = t / s.tiles_m;
        for (int kb = 0; kb < s.kblocks; ++kb) {
          if (!sm100::mbar_wait_cluster(&empty[stage], phase ^ 1u)) {
            *s_err = 1;
            break;
          }
          const uint32_t fbar = sm100::mapa_shared(sm100::smem_u32(&full[stage]), 0);
          // The leader's barrier expects both CTAs' bytes.
          if (leader) sm100::mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
          sm100::tma_load_2d_pair(sA + stage * A_BYTES, &tmap_a, fbar, kb * BK, tm * BM + static_cast<int>(rank) * 128);
          sm100::tma_load_2d_pair(sB + stage * B_BYTES, &tmap_b, fbar, kb * BK, tn * BN + static_cast<int>(rank) * 128);
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
      }
      // Never leave while a copy into this CTA's shared memory is in flight
      // (the leader sees every stage complete on its own barriers).
      if (leader)
        for (int i = 0; i < STAGES; ++i)
          if (issued[i]) sm100::mbar_wait_cluster(&full[i], issued_phase[i]);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only)
    if (leader && sm100::elect_one()) {
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = pair; t < ntiles && ok && !*s_err; t += npairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1u;
        if (!sm100::mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < s.kblocks; ++kb) {
          if (!sm100::mbar_wait_cluster(&full[stage], phase)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint64_t da = sm100::smem_desc_sw128(sA + stage * A_BYTES);
          const uint64_t db = sm100::smem_desc_sw128(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            sm100::mma_bf16_pair(d, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          // Stage free in both CTAs once these MMAs have read it.
          sm100::mma_commit_pair(sm100::mapa_shared(sm100::smem_u32(&empty[stage]), 0));
          sm100::mma_commit_pair(sm100::mapa_shared(sm100::smem_u32(&empty[stage]), 1));
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        sm100::mma_commit_pair(sm100::mapa_shared(sm100::smem_u32(&tfull[acc]), 0));
        sm100::mma_commit_pair(sm100::mapa_shared(sm100::smem_u32(&tfull[acc]), 1));
      }
      if (!ok) *s_err = 1;
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs)
    const int quarter = warp & 3;
    int local = 0;
    const uint32_t tempty_leader[2] = {sm100::mapa_shared(sm100::smem_u32(&tempty[0]), 0),
                                       sm100::mapa_shared(sm100::smem_u32(&tempty[1]), 0)};
    for (int t = pair; t < ntiles; t += npairs, ++local) {
      const int tm = t % s.tiles_m, tn = t / s.tiles_m;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1u;
      if (!sm100::mbar_wait_cluster(&tfull[acc], acc_phase)) {
        *s_err = 1;
        break;
      }
      sm100::tc_fence_after();
      const int row = tm * BM + static_cast<int>(rank) * 128 + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int cc = 0; cc < BN; cc += 32) {
        uint32_t r[32];
        sm100::tmem_ld_32x32b_x32(taddr + cc, r);
        sm100::tmem_ld_wait();
        const int col = tn * BN + cc;
        if (row < s.M && col < s.N) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = sm100::pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
          __nv_bfloat16* dst = c + static_cast<int64_t>(row) * ldc + col;
          if (col + 32 <= s.N) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<uint4*>(dst)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          } else {
            const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(w);
            for (int i = 0; col + i < s.N && i < 32; ++i) dst[i] = h[i];
          }
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive_cluster(tempty_leader[acc]);
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // neither CTA leaves while the pair's MMAs or signals may touch it
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  if (threadIdx.x == 0 && *s_err) atomicExch(err, gemm::kGemmTimeout);
}

}  // namespace gemm2
}  // namespace b200ar
