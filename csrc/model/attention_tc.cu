// GQA decode attention on the 5th-generation tensor cores (sm_100a).
//
// Swap-AB flash-decoding: per chunk of 128 cached tokens,
//   S^T [128 tokens x 16 heads] = K_chunk [128 x 128 dims] . Q^T    (tcgen05.mma, M = 128 tokens)
//   O^T [128 dims x 16 heads]   = V_chunk^T [128 x 128 tokens] . P^T (tcgen05.mma, M = 128 dims)
// so the large dimension (tokens, then head dims) is the MMA's M = 128 and the
// G query heads of one KV head (padded to 16) are its N. K and V tiles come in
// by TMA (4-D tensor map over the [batch, max_len, kv_heads, 128] cache, no
// multicast) into a 3-stage ring; V is consumed in place as an MN-major
// operand, P is written by the softmax warps into a K-major shared tile.
//
//   warp 0      TMA producer (one elected thread)
//   warp 1      TMEM allocator and MMA issuer (one elected thread)
//   warps 2..5  softmax and output accumulation: during the scores step thread
//               t owns token t of the chunk (TMEM lane t), during the output
//               step it owns head dimension t.
//
// Online softmax in the log2 domain: every softmax thread keeps the running
// max per head (identical in all threads: the chunk max is combined across
// the four warps through shared memory), its own partial sum of
// probabilities, and its dimension's output accumulator, rescaled by
// exp2(m_old - m_new) when a chunk raises the max.
//
// Pipelining: scores and output live in two TMEM buffers each and P in two
// shared tiles, so the scores MMA of chunk c + 1 and the output MMA of chunk c
// run while the softmax warps work on chunk c + 1, and the output of chunk c
// is added once the softmax of chunk c + 1 is done.
//
// Splits: CTA (b, kv head, split) handles a run of whole 128-token chunks of
// sequence b and writes its partial (o, max, sum); the CTA that finishes last
// merges the splits and re-arms the arrival counter. Every wait is bounded (2 s): on expiry the
// kernel records kAttnTimeout in `err`, drains its TMA copies, frees TMEM and
// returns.
//
// The reference library has no model code (it is an all-reduce library); this
// kernel serves the tensor-parallel decoder slice.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "../common/check.h"
#include "../common/trace.h"
#include "../gemm/tcgen05.cuh"
#include "model.h"
#include "../common/pdl.h"

namespace b200ar {

namespace {

constexpr int kTD = 128;                 // head dim
constexpr int kTChunk = 128;             // tokens per chunk (MMA M of the scores)
constexpr int kTN = 16;                  // padded query heads per KV head (MMA N)
constexpr int kTStages = 3;
constexpr int kTThreads = 192;
constexpr uint32_t kHalfTile = kTChunk * 128;        // 128 rows x 128 B (64 dims): 16 KB
constexpr uint32_t kStageBytes = 4 * kHalfTile;      // K lo, K hi, V lo, V hi
constexpr uint32_t kQHalf = kTN * 128;               // 16 rows x 128 B: 2 KB
constexpr uint32_t kPHalf = kTN * 128;               // 16 heads x 64 tokens: 2 KB
constexpr size_t kTSmem = 1024 /*align*/ + kTStages * kStageBytes + 2 * kQHalf + 4 * kPHalf +
                          2 * 4 * kTN * sizeof(float) /*chunk max*/ + 4 * kTN * sizeof(float) /*sums*/ +
                          256 /*barriers*/;
constexpr uint32_t kTmemCols = 64;       // two scores buffers, two output buffers
constexpr int kAttnTimeout = 2;

struct AttnTcParams {
  const int* seq_len;
  float* part_acc;
  float* part_ml;
  unsigned* done_count;
  __nv_bfloat16* out;
  int* err;
  int hkv, group, splits;
  float scale_log2;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// G: query heads handled per KV head (8 or 16); the MMA N stays 16 (its
// minimum at M = 128), columns G..15 of S and O are never read.
template <int G>
__global__ void __launch_bounds__(kTThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, AttnTcParams p) {
  extern __shared__ __align__(1024) uint8_t attn_tc_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(attn_tc_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sKV = smem;                                   // [stage][K lo, K hi, V lo, V hi]
  uint8_t* sQ = sKV + kTStages * kStageBytes;            // [2 halves][16 rows x 128 B]
  uint8_t* sP = sQ + 2 * kQHalf;                         // [2 buffers][2 halves][16 rows x 128 B]
  float* red = reinterpret_cast<float*>(sP + 4 * kPHalf);  // [2][4][16] chunk max per warp
  float* sums = red + 2 * 4 * kTN;                       // [4][16] final sums per warp
  uint64_t* full = reinterpret_cast<uint64_t*>(sums + 4 * kTN);
  uint64_t* empty = full + kTStages;
  uint64_t* qbar = empty + kTStages;
  uint64_t* sfull = qbar + 1;    // [2]: scores of chunk c in TMEM buffer c & 1
  uint64_t* ofull = sfull + 2;   // [2]: output of chunk c in TMEM buffer c & 1
  uint64_t* pready = ofull + 2;  // [2]: P of chunk c written (S buffer c & 1 consumed)
  uint64_t* oempty = pready + 2; // [2]: output buffer c & 1 consumed
  uint64_t* redbar = oempty + 2;
  uint64_t* sumbar = redbar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sumbar + 1);
  volatile int* s_err = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x, kh = blockIdx.y, sp = blockIdx.z;
  const int splits = p.splits, group = p.group;
  // Everything this kernel reads may come from the previous kernel of the
  // step (q and the new K/V row from the QKV projection): wait for it first;
  // only the launch itself overlaps the previous kernel's tail.
  pdl_wait();
  pdl_trigger();
  const int len = p.seq_len[b];
  // Splits cover whole chunks: the partial chunk is the sequence's last.
  const int chunks = (len + kTChunk - 1) / kTChunk;
  const int per = (chunks + splits - 1) / splits;
  const int t0 = min(len, sp * per * kTChunk);
  const int t1 = min(len, (sp + 1) * per * kTChunk);
  const int nch = (t1 - t0 + kTChunk - 1) / kTChunk;
  const int hq = p.hkv * group;
  const int head0 = b * hq + kh * group;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTStages; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
    }
    sm100::mbar_init(qbar, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&sfull[i], 1);
      sm100::mbar_init(&ofull[i], 1);
      sm100::mbar_init(&pready[i], 4);
      sm100::mbar_init(&oempty[i], 4);
    }
    sm100::mbar_init(redbar, 4);
    sm100::mbar_init(sumbar, 4);
    *s_err = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tq);
    sm100::prefetch_tmap(&tk);
    sm100::prefetch_tmap(&tv);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, kTmemCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: scores buffers at 0 and 16, output buffers at 32 and 48.
  auto tS = [&](int c) { return tmem + static_cast<uint32_t>((c & 1) * kTN); };
  auto tO = [&](int c) { return tmem + static_cast<uint32_t>(2 * kTN + (c & 1) * kTN); };
  auto sPb = [&](int c) { return sP + (c & 1) * 2 * kPHalf; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (sm100::elect_one()) {
      sm100::mbar_arrive_expect_tx(qbar, 2 * kQHalf);
      sm100::tma_load_2d(sQ, &tq, qbar, 0, head0);
      sm100::tma_load_2d(sQ + kQHalf, &tq, qbar, 64, head0);
      bool issued[kTStages] = {};
      uint32_t issued_phase[kTStages] = {};
      for (int c = 0; c < nch && !*s_err; ++c) {
        const int st = c % kTStages;
        const uint32_t ph = (c / kTStages) & 1u;
        if (!sm100::mbar_wait(&empty[st], ph ^ 1u)) {
          *s_err = 1;
          break;
        }
        uint8_t* dst = sKV + st * kStageBytes;
        const int tok = t0 + c * kTChunk;
        sm100::mbar_arrive_expect_tx(&full[st], kStageBytes);
        sm100::tma_load_4d(dst, &tk, &full[st], 0, kh, tok, b);
        sm100::tma_load_4d(dst + kHalfTile, &tk, &full[st], 64, kh, tok, b);
        sm100::tma_load_4d(dst + 2 * kHalfTile, &tv, &full[st], 0, kh, tok, b);
        sm100::tma_load_4d(dst + 3 * kHalfTile, &tv, &full[st], 64, kh, tok, b);
        issued[st] = true;
        issued_phase[st] = ph;
      }
      // Never leave while a copy into this CTA's shared memory is in flight.
      sm100::mbar_wait(qbar, 0);
      for (int i = 0; i < kTStages; ++i)
        if (issued[i]) sm100::mbar_wait(&full[i], issued_phase[i]);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Order: scores of chunk c, then the output of chunk c - 1, so that the
    // softmax of chunk c overlaps the output MMA of chunk c - 1.
    if (sm100::elect_one()) {
      constexpr uint32_t idesc_s = sm100::idesc_bf16_f32(kTChunk, kTN);           // A, B K-major
      constexpr uint32_t idesc_o = sm100::idesc_bf16_f32(kTD, kTN) | (1u << 15);  // A MN-major
      auto issue_output = [&](int c) -> bool {
        // P of chunk c written; output buffer c & 1 free (consumed for chunk c - 2).
        if (!sm100::mbar_wait(&pready[c & 1], (c >> 1) & 1u)) return false;
        if (c >= 2 && !sm100::mbar_wait(&oempty[c & 1], ((c - 2) >> 1) & 1u)) return false;
        sm100::tc_fence_after();
        const uint8_t* vt = sKV + (c % kTStages) * kStageBytes + 2 * kHalfTile;
        const uint8_t* pb = sPb(c);
        // 8 K-steps of 16 tokens. V^T is MN-major: 16 tokens = 2048 bytes
        // further in the V tile; its second 64 dims are one half tile away.
#pragma unroll
        for (int k = 0; k < kTChunk / 16; ++k) {
          const uint64_t da = sm100::smem_desc_mn_sw128(vt + k * 2048, kHalfTile, 1024);
          const uint64_t db = sm100::smem_desc_sw128(pb + (k >> 2) * kPHalf) + 2 * (k & 3);
          sm100::mma_bf16(tO(c), da, db, idesc_o, k > 0 ? 1u : 0u);
        }
        sm100::mma_commit(&ofull[c & 1]);
        sm100::mma_commit(&empty[c % kTStages]);
        return true;
      };
      bool ok = nch == 0 || sm100::mbar_wait(qbar, 0);
      for (int c = 0; c < nch && ok && !*s_err; ++c) {
        const int st = c % kTStages;
        if (!sm100::mbar_wait(&full[st], (c / kTStages) & 1u)) {
          ok = false;
          break;
        }
        // Scores buffer c & 1 was last read for chunk c - 2 (its P is written).
        if (c >= 2 && !sm100::mbar_wait(&pready[c & 1], ((c - 2) >> 1) & 1u)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint8_t* kt = sKV + st * kStageBytes;
        // 8 K-steps of 16 dims; dims 0-63 in the low half tiles, 64-127 in the high ones.
#pragma unroll
        for (int k = 0; k < kTD / 16; ++k) {
          const uint64_t da = sm100::smem_desc_sw128(kt + (k >> 2) * kHalfTile) + 2 * (k & 3);
          const uint64_t db = sm100::smem_desc_sw128(sQ + (k >> 2) * kQHalf) + 2 * (k & 3);
          sm100::mma_bf16(tS(c), da, db, idesc_s, k > 0 ? 1u : 0u);
        }
        sm100::mma_commit(&sfull[c & 1]);
        if (c >= 1 && !issue_output(c - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && nch > 0 && !*s_err) ok = issue_output(nch - 1);
      if (!ok) *s_err = 1;
    }
  } else {
    // ------------------------------------------------------------ softmax + output
    const int q4 = warp & 3;         // TMEM lane quarter of this warp
    const int row = q4 * 32 + lane;  // token of the chunk (scores), head dim (output)
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    float m[G], l[G], o[G], alpha_prev[G];
#pragma unroll
    for (int h = 0; h < G; ++h) m[h] = -INFINITY, l[h] = 0.f, o[h] = 0.f, alpha_prev[h] = 0.f;
    bool ok = true;
    // Adds the output MMA of chunk c (relative to that chunk's running max) to o.
    auto accumulate = [&](int c, const float* alpha) -> bool {
      if (!sm100::mbar_wait(&ofull[c & 1], (c >> 1) & 1u)) return false;
      sm100::tc_fence_after();
      uint32_t orr[G];
      if constexpr (G == 16) sm100::tmem_ld_32x32b_x16(tO(c) + lane_off, orr);
      else sm100::tmem_ld_32x32b_x8(tO(c) + lane_off, orr);
      sm100::tmem_ld_wait();
#pragma unroll
      for (int h = 0; h < G; ++h) o[h] = o[h] * alpha[h] + __uint_as_float(orr[h]);
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&oempty[c & 1]);
      return true;
    };
    for (int c = 0; c < nch; ++c) {
      if (!sm100::mbar_wait(&sfull[c & 1], (c >> 1) & 1u)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      uint32_t sr[G];
      if constexpr (G == 16) sm100::tmem_ld_32x32b_x16(tS(c) + lane_off, sr);
      else sm100::tmem_ld_32x32b_x8(tS(c) + lane_off, sr);
      sm100::tmem_ld_wait();
      const int tok = t0 + c * kTChunk + row;
      const bool valid = tok < t1;
      float x[G];
#pragma unroll
      for (int h = 0; h < G; ++h) x[h] = (valid && h < group) ? __uint_as_float(sr[h]) * p.scale_log2 : -INFINITY;
      // Chunk max per head over this warp's 32 tokens, then over the 4 warps.
      float* rb = red + (c & 1) * 4 * kTN;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float mx = warp_max(x[h]);
        if (lane == h) rb[q4 * kTN + h] = mx;
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(redbar);
      if (!sm100::mbar_wait(redbar, c & 1u)) {
        ok = false;
        break;
      }
      float alpha[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float cm = fmaxf(fmaxf(rb[h], rb[kTN + h]), fmaxf(rb[2 * kTN + h], rb[3 * kTN + h]));
        const float mn = fmaxf(m[h], cm);
        alpha[h] = m[h] == -INFINITY ? 0.f : exp2f(m[h] - mn);
        m[h] = mn;
        const float pv = x[h] == -INFINITY ? 0.f : exp2f(x[h] - mn);
        l[h] = l[h] * alpha[h] + pv;
        x[h] = pv;
      }
      // Rows past the sequence may hold anything (the cache is not cleared):
      // zero them in V so that P = 0 there cannot meet a NaN.
      const int st = c % kTStages;
      if (tok >= len) {
        if (!sm100::mbar_wait(&full[st], (c / kTStages) & 1u)) {
          ok = false;
          break;
        }
        uint8_t* vt = sKV + st * kStageBytes + 2 * kHalfTile;
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          *reinterpret_cast<uint4*>(vt + row * 128 + i * 16) = z;
          *reinterpret_cast<uint4*>(vt + kHalfTile + row * 128 + i * 16) = z;
        }
      }
      // P^T as the K-major B operand: row h (head), K index = token `row`,
      // 128-byte swizzle (16-byte chunk index XOR row % 8). Buffer c & 1 was
      // last read by the output MMA of chunk c - 2, complete once that
      // chunk's output was accumulated (previous iteration).
      {
        uint8_t* pt = sPb(c) + (row >> 6) * kPHalf;
        const int col = row & 63;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const uint32_t off = h * 128 + ((((col >> 3) ^ (h & 7)) << 4) | ((col & 7) * 2));
          *reinterpret_cast<__nv_bfloat16*>(pt + off) = __float2bfloat16_rn(x[h]);
        }
      }
      sm100::fence_proxy_async_smem();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&pready[c & 1]);
      // The output of chunk c - 1 (its MMA overlapped this chunk's softmax).
      if (c >= 1 && !accumulate(c - 1, alpha_prev)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int h = 0; h < G; ++h) alpha_prev[h] = alpha[h];
    }
    if (ok && nch > 0) {
      // o is relative to the max before the last chunk: the last chunk's factor
      // rescales it, then its own output adds in.
      ok = accumulate(nch - 1, alpha_prev);
    }
    if (!ok) *s_err = 1;
    // Sum of probabilities per head over the 128 token threads.
    if (ok) {
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float sv = warp_sum32(l[h]);
        if (lane == h) sums[q4 * kTN + h] = sv;
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sumbar);
      if (!sm100::mbar_wait(sumbar, 0)) ok = false;
    }
    if (ok) {
#pragma unroll
      for (int h = 0; h < G; ++h) {
        if (h >= group) break;
        const int64_t base = static_cast<int64_t>(head0 + h) * splits + sp;
        p.part_acc[base * kTD + row] = o[h];
        if (row == 0) {
          p.part_ml[base * 2 + 0] = m[h];
          p.part_ml[base * 2 + 1] = sums[h] + sums[kTN + h] + sums[2 * kTN + h] + sums[3 * kTN + h];
        }
      }
    } else {
      *s_err = 1;
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kTmemCols);
  }
  // On an expired wait the partials of this CTA are incomplete: the error word
  // tells the host; the split count below still runs so the counter re-arms.
  if (*s_err && threadIdx.x == 0) atomicExch(p.err, kAttnTimeout);

  // Merge the splits: the CTA that finishes last combines every partial of its
  // (batch, KV head) and re-arms the counter for the next launch.
  __shared__ unsigned is_last;
  __threadfence();
  __syncthreads();
  unsigned* cnt = p.done_count + static_cast<int64_t>(b) * p.hkv + kh;
  if (threadIdx.x == 0) is_last = atomicAdd(cnt, 1u) == static_cast<unsigned>(splits - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (threadIdx.x == 0) *cnt = 0u;
  constexpr int kWarps = kTThreads / 32;
  for (int h = warp; h < group; h += kWarps) {
    const int64_t head = head0 + h;
    const float* ml = p.part_ml + head * splits * 2;
    const float* pp = p.part_acc + head * splits * kTD + lane * 4;
    float mm = -INFINITY;
    for (int s2 = 0; s2 < splits; ++s2) mm = fmaxf(mm, __ldcg(ml + 2 * s2));
    float ll = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int s2 = 0; s2 < splits; ++s2) {
      const float ms = __ldcg(ml + 2 * s2);
      const float f = ms == -INFINITY ? 0.f : exp2f(ms - mm);
      ll += __ldcg(ml + 2 * s2 + 1) * f;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(pp + static_cast<int64_t>(s2) * kTD));
      acc[0] += a.x * f;
      acc[1] += a.y * f;
      acc[2] += a.z * f;
      acc[3] += a.w * f;
    }
    const float inv = ll > 0.f ? 1.f / ll : 0.f;
    __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(p.out + head * kTD + lane * 4);
    dst[0] = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
    dst[1] = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
  }
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode() {
  static EncodeFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    B200AR_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !ptr) throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<EncodeFn>(ptr);
  }();
  return fn;
}

// 4-D map over a KV cache [batch, max_len, hkv, 128] (bf16), box of 64 dims x
// 1 head x 128 tokens x 1 sequence, 128-byte swizzle. Tokens past max_len read
// as zero.
CUtensorMap kv_map(const void* cache, int64_t batch, int max_len, int hkv) {
  B200AR_CHECK(reinterpret_cast<uintptr_t>(cache) % 16 == 0, "KV cache must be 16-byte aligned");
  CUtensorMap m;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kTD), static_cast<cuuint64_t>(hkv),
                              static_cast<cuuint64_t>(max_len), static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(kTD) * 2, static_cast<cuuint64_t>(hkv) * kTD * 2,
                                 static_cast<cuuint64_t>(max_len) * hkv * kTD * 2};
  const cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(kTChunk), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(cache), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (KV cache) failed: " + std::to_string(r));
  return m;
}

// 2-D map over q [rows, 128] (bf16), box of 16 rows x 64 dims.
CUtensorMap q_map(const void* q, int64_t rows) {
  B200AR_CHECK(reinterpret_cast<uintptr_t>(q) % 16 == 0, "q must be 16-byte aligned");
  CUtensorMap m;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kTD), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kTD) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kTN)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(q), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (q) failed: " + std::to_string(r));
  return m;
}

}  // namespace

int attention_tc_splits(int64_t batch, int hkv, int max_len) {
  // One wave of one CTA per SM; at least one chunk of cache per split.
  const int64_t ctas = std::max<int64_t>(batch * hkv, 1);
  int s = static_cast<int>(std::max<int64_t>(1, 148 / ctas));
  s = std::min(s, std::max(1, (max_len + kTChunk - 1) / kTChunk));
  return std::min(s, 64);
}

void decode_attention_tc(const void* q, const void* k_cache, const void* v_cache, const int* seq_len, void* out,
                         float* part_acc, float* part_ml, unsigned* done_count, int* err, int64_t batch, int hq,
                         int hkv, int head_dim, int max_len, int splits, float scale, cudaStream_t s) {
  const TraceRange trace("b200ar::decode_attention_tc");
  B200AR_CHECK(head_dim == kTD, "decode attention is built for head_dim 128");
  B200AR_CHECK(hkv > 0 && hq % hkv == 0, "query heads must be a multiple of KV heads");
  const int group = hq / hkv;
  B200AR_CHECK(group <= kTN, "GQA group size must be at most 16");
  B200AR_CHECK(splits >= 1 && splits <= 65535 && batch >= 1 && batch <= 2147483647 && hkv <= 65535,
               "bad attention grid");
  B200AR_CHECK(max_len >= 1, "bad cache length");
  const CUtensorMap tq = q_map(q, batch * hq);
  const CUtensorMap tk = kv_map(k_cache, batch, max_len, hkv);
  const CUtensorMap tv = kv_map(v_cache, batch, max_len, hkv);
  AttnTcParams prm{seq_len, part_acc, part_ml, done_count, static_cast<__nv_bfloat16*>(out), err, hkv, group, splits,
                   scale * 1.4426950408889634f};
  auto kern = group <= 8 ? attn_tc_kernel<8> : attn_tc_kernel<16>;
  static PerDeviceOnce smem_attr;
  smem_attr([&] {
    for (auto k : {attn_tc_kernel<8>, attn_tc_kernel<16>})
      B200AR_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTSmem)));
  });
  const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(hkv), static_cast<unsigned>(splits));
  launch_pdl(kern, grid, dim3(kTThreads), kTSmem, s, 1, tq, tk, tv, prm);
  B200AR_CUDA(cudaGetLastError());
}

}  // namespace b200ar
