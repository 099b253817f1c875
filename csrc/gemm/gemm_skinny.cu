// Skinny (decode) GEMM for sm_100a: out[M, N] = x[M, K] * W[N, K]^T with M <= 128.
//
// Decode GEMMs stream the weights once and do little math per byte, so the
// work must be spread over every SM. The kernel swaps the operands (the
// weight rows become the 128-wide UMMA M dimension, the padded batch the UMMA
// N dimension, 16..128) and splits K over `splits` CTAs:
//   CTA (b, s): weight rows [128 b, 128 b + 128), K blocks of split s.
//   warp 0: TMA producer (W tile 128 x 64, x tile MP x 64, 6-stage ring)
//   warp 1: tcgen05.mma issuer, accumulator 128 lanes x MP columns in TMEM
//   warps 0-3: epilogue, thread = one weight row n, MP batch columns.
// With one split the bf16 result is written directly. Otherwise each CTA
// writes its fp32 partial to `partials[s][m][n]`, and the last CTA of a row
// block (per-block arrival counter) sums the partials in split order and
// writes bf16, so results do not depend on arrival order. The counter is
// reset by that last CTA for the next call.
// Epilogue mode 1 (SiLU-gate): the weight rows hold gate and up projections
// interleaved in groups of 64 (rows [128 b, 128 b + 64) = gate rows
// [64 b, 64 b + 64), the next 64 rows = the matching up rows). The partials
// always go through the reduction, which rounds g and u to bf16 (as a stored
// gate-up product would be) and writes silu(g) * u to out[M, N / 2]: the
// activation kernel and the gate-up round trip disappear.
// Epilogue mode 2 (RoPE + KV write): W is the QKV projection, one 128-row
// block per head ([q heads | k heads | v heads], head_dim 128). The reduction
// rounds each pair (c, c + 64) of a head to bf16, rotates q and k heads by
// the position of the row's sequence (rotate-half), and writes q heads to
// q_out[M, hq, 128] and k, v heads into the caches at that position: the
// separate RoPE kernel and the qkv round trip disappear.
#include <cuda.h>

#include <algorithm>
#include <stdexcept>

#include "../common/check.h"
#include "../common/trace.h"
#include "gemm_api.h"
#include "tcgen05.cuh"
#include "../common/pdl.h"

namespace b200ar {

namespace {

constexpr int SBM = 128;
constexpr int SBK = 64;
// Ring depth per batch width: as many stages as fit in ~200 KB of shared
// memory (11 at MP = 16, 6 at MP = 128), so that a CTA's whole K range of a
// decode GEMM is usually in flight after one round trip.
template <int MP>
constexpr int skinny_stages() {
  return (200 * 1024) / (SBM * SBK * 2 + MP * SBK * 2) > 12 ? 12 : (200 * 1024) / (SBM * SBK * 2 + MP * SBK * 2);
}
constexpr int STHREADS = 128;

template <int MP>
struct SkinnyCfg {
  static constexpr uint32_t W_BYTES = SBM * SBK * 2;
  static constexpr uint32_t X_BYTES = MP * SBK * 2;
  static constexpr uint32_t STAGE = W_BYTES + X_BYTES;
  static constexpr int STAGES = skinny_stages<MP>();
  static constexpr size_t SMEM = STAGES * STAGE + 1024 + 256;
  static constexpr uint32_t TMEM_COLS = MP < 32 ? 32 : MP;
};

struct SkinnyArgs {
  __nv_bfloat16* out;
  float* partials;      // [splits, M, N] when splits > 1
  unsigned* counters;   // [N / 128] arrival counters, zero between calls
  int M, N, K;
  int nblocks, splits, kblocks;
  int epi;              // 0: out[M, N] = x W^T; 1: SiLU-gate over 64-row groups, out[M, N / 2]; 2: RoPE + KV
  RopeKvArgs rope;      // epi 2 only
};

template <int MP>
__global__ void __launch_bounds__(STHREADS, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                  SkinnyArgs a, int* err) {
  using C = SkinnyCfg<MP>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + C::STAGES * C::W_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE);
  uint64_t* empty = full + C::STAGES;
  uint64_t* done = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* s_err = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_last = const_cast<int*>(s_err) + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x % a.nblocks;
  const int sp = blockIdx.x / a.nblocks;
  const int kb0 = static_cast<int>((static_cast<int64_t>(a.kblocks) * sp) / a.splits);
  const int kb1 = static_cast<int>((static_cast<int64_t>(a.kblocks) * (sp + 1)) / a.splits);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
    }
    sm100::mbar_init(done, 1);
    *s_err = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmap_w);
    sm100::prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, C::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();  // the next kernel of a decode step may start its own set-up

  if (warp == 0) {
    if (sm100::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool issued[C::STAGES] = {};
      uint32_t iphase[C::STAGES] = {};
      // Weights are never written by another kernel: the first ring's worth
      // of weight tiles is requested before waiting for the previous kernel
      // (which produces x), the matching activation tiles after it.
      const int pre = min(kb1 - kb0, C::STAGES);
      for (int i = 0; i < pre; ++i) {
        sm100::mbar_arrive_expect_tx(&full[i], C::STAGE);
        sm100::tma_load_2d(sW + i * C::W_BYTES, &tmap_w, &full[i], (kb0 + i) * SBK, b * SBM);
        issued[i] = true;
        iphase[i] = 0;
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) sm100::tma_load_2d(sX + i * C::X_BYTES, &tmap_x, &full[i], (kb0 + i) * SBK, 0);
      stage = pre % C::STAGES;
      phase = pre == C::STAGES ? 1u : 0u;
      for (int kb = kb0 + pre; kb < kb1; ++kb) {
        if (!sm100::mbar_wait(&empty[stage], phase ^ 1u)) {
          *s_err = 1;
          break;
        }
        sm100::mbar_arrive_expect_tx(&full[stage], C::STAGE);
        sm100::tma_load_2d(sW + stage * C::W_BYTES, &tmap_w, &full[stage], kb * SBK, b * SBM);
        sm100::tma_load_2d(sX + stage * C::X_BYTES, &tmap_x, &full[stage], kb * SBK, 0);
        issued[stage] = true;
        iphase[stage] = phase;
        if (++stage == C::STAGES) stage = 0, phase ^= 1u;
      }
      for (int i = 0; i < C::STAGES; ++i)
        if (issued[i]) sm100::mbar_wait(&full[i], iphase[i]);
    }
  } else if (warp == 1) {
    if (sm100::elect_one()) {
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(SBM, MP);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!sm100::mbar_wait(&full[stage], phase)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint64_t dw = sm100::smem_desc_sw128(sW + stage * C::W_BYTES);
        const uint64_t dx = sm100::smem_desc_sw128(sX + stage * C::X_BYTES);
#pragma unroll
        for (int k = 0; k < SBK / 16; ++k) sm100::mma_bf16(tmem, dw + 2 * k, dx + 2 * k, idesc, (kb > kb0 || k > 0));
        sm100::mma_commit(&empty[stage]);
        if (++stage == C::STAGES) stage = 0, phase ^= 1u;
      }
      if (!ok) *s_err = 1;
      sm100::mma_commit(done);  // also fires when no MMA was issued
    }
  }
  __syncwarp();
  pdl_wait();  // outputs, partials and counters are written only after the previous kernel completed

  // ---------------- epilogue: all 4 warps; thread = weight row n
  const bool have = kb1 > kb0;
  const bool ok = sm100::mbar_wait(done, 0);
  if (!ok) *s_err = 1;
  sm100::tc_fence_after();
  const int n = b * SBM + warp * 32 + lane;
  // Partial (or final) values leave TMEM 32 batch columns at a time.
  constexpr int CH = MP < 32 ? MP : 32;
  if (ok) {
#pragma unroll 1
    for (int c = 0; c < MP; c += CH) {
      uint32_t r[32];
      sm100::tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c, r);
      sm100::tmem_ld_wait();
      if (n < a.N) {
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int m = c + i;
          if (m < a.M) {
            const float v = have ? __uint_as_float(r[i]) : 0.f;
            if (a.splits == 1 && a.epi == 0)
              a.out[static_cast<int64_t>(m) * a.N + n] = __float2bfloat16_rn(v);
            else
              a.partials[(static_cast<int64_t>(sp) * a.M + m) * a.N + n] = v;
          }
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(err, 1);
    return;
  }
  if (a.splits == 1 && a.epi == 0) return;
  // Split-K: the last CTA of this row block sums the partials in split order.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) *s_last = atomicAdd(&a.counters[b], 1u) == static_cast<unsigned>(a.splits - 1);
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  if (a.epi != 0) {
    // Paired epilogues: thread item = (row m, columns c .. c + 3 of this block
    // and the partner columns c + 64 .. c + 67); sums in split order, rounded
    // to bf16 as a stored product would be, then the epilogue.
    constexpr int HALF = SBM / 2;
    const int64_t sstride = static_cast<int64_t>(a.M) * a.N;
    const int items = a.M * (HALF / 4);
    for (int i0 = threadIdx.x; i0 < items; i0 += 2 * STHREADS) {
      float4 lo[2], hi[2];
      int64_t off[2];
      int mm[2], cc[2];
      bool act[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int it = i0 + j * STHREADS;
        mm[j] = it / (HALF / 4);
        cc[j] = (it % (HALF / 4)) * 4;
        act[j] = it < items && b * SBM + HALF + cc[j] < a.N;
        off[j] = static_cast<int64_t>(mm[j]) * a.N + b * SBM + cc[j];
        lo[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        hi[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      for (int q = 0; q < a.splits; ++q) {
        float4 vl[2], vh[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float* base = a.partials + q * sstride + off[j];
          vl[j] = act[j] ? __ldcg(reinterpret_cast<const float4*>(base)) : make_float4(0.f, 0.f, 0.f, 0.f);
          vh[j] = act[j] ? __ldcg(reinterpret_cast<const float4*>(base + HALF)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          lo[j].x += vl[j].x; lo[j].y += vl[j].y; lo[j].z += vl[j].z; lo[j].w += vl[j].w;
          hi[j].x += vh[j].x; hi[j].y += vh[j].y; hi[j].z += vh[j].z; hi[j].w += vh[j].w;
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (!act[j]) continue;
        const float ls[4] = {lo[j].x, lo[j].y, lo[j].z, lo[j].w};
        const float hs[4] = {hi[j].x, hi[j].y, hi[j].z, hi[j].w};
        float x0[4], x1[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          x0[e] = __bfloat162float(__float2bfloat16_rn(ls[e]));
          x1[e] = __bfloat162float(__float2bfloat16_rn(hs[e]));
        }
        const int m = mm[j], c = cc[j];
        if (a.epi == 1) {
          // SiLU-gate: x0 = gate, x1 = up; out[m, 64 b + c ..].
          float y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) y[e] = x0[e] / (1.f + __expf(-x0[e])) * x1[e];
          uint2 w;
          w.x = sm100::pack_bf16x2(y[0], y[1]);
          w.y = sm100::pack_bf16x2(y[2], y[3]);
          *reinterpret_cast<uint2*>(a.out + static_cast<int64_t>(m) * (a.N / 2) + b * HALF + c) = w;
        } else {
          // RoPE + KV write: block b is head b of [q heads | k heads | v heads].
          const RopeKvArgs& r = a.rope;
          const int p = r.pos[m];
          // A position past the cache (or the rotary table) is skipped, never written.
          if (p < 0 || p >= r.max_len) continue;
          uint2 w0, w1;
          if (b < r.hq + r.hkv) {
            float y0[4], y1[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float cs = r.cos_t[static_cast<int64_t>(p) * HALF + c + e];
              const float sn = r.sin_t[static_cast<int64_t>(p) * HALF + c + e];
              y0[e] = x0[e] * cs - x1[e] * sn;
              y1[e] = x1[e] * cs + x0[e] * sn;
            }
            w0.x = sm100::pack_bf16x2(y0[0], y0[1]);
            w0.y = sm100::pack_bf16x2(y0[2], y0[3]);
            w1.x = sm100::pack_bf16x2(y1[0], y1[1]);
            w1.y = sm100::pack_bf16x2(y1[2], y1[3]);
          } else {
            w0.x = sm100::pack_bf16x2(x0[0], x0[1]);
            w0.y = sm100::pack_bf16x2(x0[2], x0[3]);
            w1.x = sm100::pack_bf16x2(x1[0], x1[1]);
            w1.y = sm100::pack_bf16x2(x1[2], x1[3]);
          }
          __nv_bfloat16* dst;
          if (b < r.hq) {
            dst = r.q_out + (static_cast<int64_t>(m) * r.hq + b) * SBM;
          } else {
            const bool is_k = b < r.hq + r.hkv;
            const int kh = is_k ? b - r.hq : b - r.hq - r.hkv;
            dst = (is_k ? r.k_cache : r.v_cache) +
                  ((static_cast<int64_t>(m) * r.max_len + p) * r.hkv + kh) * SBM;
          }
          *reinterpret_cast<uint2*>(dst + c) = w0;
          *reinterpret_cast<uint2*>(dst + HALF + c) = w1;
        }
      }
    }
  } else {
    // 16-byte loads: thread item = (row m, 4 consecutive columns of this
    // block); four items and four splits of loads in flight, sums in split order.
    const int64_t sstride = static_cast<int64_t>(a.M) * a.N;
    const int items = a.M * (SBM / 4);
    for (int i0 = threadIdx.x; i0 < items; i0 += 4 * STHREADS) {
      float4 acc[4];
      int64_t off[4];
      bool on[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int it = i0 + j * STHREADS;
        const int m = it / (SBM / 4), c = (it % (SBM / 4)) * 4;
        const int col = b * SBM + c;
        on[j] = it < items && col < a.N;
        off[j] = static_cast<int64_t>(m) * a.N + col;
        acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      for (int q0 = 0; q0 < a.splits; q0 += 4) {
        float4 v[4][4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            v[q][j] = (on[j] && q0 + q < a.splits)
                          ? __ldcg(reinterpret_cast<const float4*>(a.partials + (q0 + q) * sstride + off[j]))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[j].x += v[q][j].x;
            acc[j].y += v[q][j].y;
            acc[j].z += v[q][j].z;
            acc[j].w += v[q][j].w;
          }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (on[j]) {
          uint2 w;
          w.x = sm100::pack_bf16x2(acc[j].x, acc[j].y);
          w.y = sm100::pack_bf16x2(acc[j].z, acc[j].w);
          *reinterpret_cast<uint2*>(a.out + off[j]) = w;
        }
    }
  }
  if (threadIdx.x == 0) a.counters[b] = 0;
}

template <int MP>
void launch_skinny(const void* x, const void* w, void* out, float* partials, unsigned* counters, int64_t M, int64_t N,
                   int64_t K, int splits, int epi, const RopeKvArgs* rope, int* err, cudaStream_t stream) {
  using C = SkinnyCfg<MP>;
  const CUtensorMap tw = make_tmap_bf16_2d(w, N, K, K, SBM, SBK);
  const CUtensorMap tx = make_tmap_bf16_2d(x, M, K, K, MP, SBK);
  SkinnyArgs a{};
  a.out = static_cast<__nv_bfloat16*>(out);
  a.partials = partials;
  a.counters = counters;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.nblocks = static_cast<int>((N + SBM - 1) / SBM);
  a.kblocks = static_cast<int>((K + SBK - 1) / SBK);
  a.splits = splits;
  a.epi = epi;
  if (rope) a.rope = *rope;
  auto kern = skinny_kernel<MP>;
  static PerDeviceOnce smem_attr;
  smem_attr([&] {
    B200AR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::SMEM)));
  });
  launch_pdl(kern, dim3(static_cast<unsigned>(a.nblocks * splits)), dim3(STHREADS), C::SMEM, stream, 1, tw, tx, a, err);
  B200AR_CUDA(cudaGetLastError());
}

}  // namespace

int skinny_splits(int64_t N, int64_t K, int sms) {
  const int64_t nblocks = (N + SBM - 1) / SBM;
  const int64_t kblocks = (K + SBK - 1) / SBK;
  int64_t s = std::max<int64_t>(1, sms / nblocks);
  s = std::min<int64_t>(s, std::max<int64_t>(1, kblocks / 2));  // at least two K blocks per split
  return static_cast<int>(std::min<int64_t>(s, 16));
}

void gemm_skinny(const void* x, const void* w, void* out, float* partials, unsigned* counters, int64_t M, int64_t N,
                 int64_t K, int splits, int* err, cudaStream_t stream, int epilogue, const RopeKvArgs* rope) {
  const TraceRange trace("b200ar::gemm_skinny");
  B200AR_CHECK(M >= 1 && M <= SBM, "skinny GEMM serves 1 <= M <= 128, got " << M);
  B200AR_CHECK(K % 8 == 0 && N % 8 == 0, "K and N must be multiples of 8");
  B200AR_CHECK(epilogue >= 0 && epilogue <= 2, "unknown skinny GEMM epilogue " << epilogue);
  B200AR_CHECK(epilogue != 1 || N % SBM == 0, "the SiLU-gate epilogue needs N (gate + up rows) a multiple of 128");
  B200AR_CHECK(epilogue != 2 || (rope && N == static_cast<int64_t>(rope->hq + 2 * rope->hkv) * SBM),
               "the RoPE + KV epilogue needs its arguments and N = (hq + 2 hkv) * 128");
  B200AR_CHECK((splits == 1 && epilogue == 0) || (partials && counters), "split-K needs partials and counters");
  B200AR_CHECK(splits >= 1, "splits must be positive");
  if (M <= 16)
    launch_skinny<16>(x, w, out, partials, counters, M, N, K, splits, epilogue, rope, err, stream);
  else if (M <= 32)
    launch_skinny<32>(x, w, out, partials, counters, M, N, K, splits, epilogue, rope, err, stream);
  else if (M <= 64)
    launch_skinny<64>(x, w, out, partials, counters, M, N, K, splits, epilogue, rope, err, stream);
  else
    launch_skinny<128>(x, w, out, partials, counters, M, N, K, splits, epilogue, rope, err, stream);
}

}  // namespace b200ar
