// Model kernels for the tensor-parallel Llama decoder slice (sm_100a):
//   rmsnorm        y = x * rsqrt(mean(x^2) + eps) * gamma               (bf16 rows)
//   rope_kv        rotary embedding of q and k (rotate-half convention), q to a
//                  contiguous buffer, k and v written into the KV cache at `pos`
//   attention      GQA decode attention, split over the KV length
//                  (flash-decoding) with both products on the tensor cores
//                  (mma.sync m16n8k16): partial softmax state per split; the
//                  last split CTA of each (batch, KV head) to finish merges the
//                  partials (L2-resident) in the same launch; K/V of one KV
//                  head are read once for all the query heads of its group
//   silu_mul       y = silu(gate) * up for gate_up = [gate | up]
// All kernels move 16-byte packets and accumulate in fp32. The reference
// library has no model code; these serve the TP decoder slice.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>

#include "../common/check.h"
#include "../common/trace.h"
#include "../common/device.cuh"
#include "model.h"

namespace b200ar {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------ RMSNorm
// One CTA per row, threads hold 8 elements (16 bytes) per step.
__global__ void __launch_bounds__(512) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ gamma,
                                                      __nv_bfloat16* __restrict__ y, int hidden, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const char* xr = reinterpret_cast<const char*>(x + row * hidden);
  char* yr = reinterpret_cast<char*>(y + row * hidden);
  const int hp = hidden / 8;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hp; i += blockDim.x) {
    float v[8];
    unpack_set<__nv_bfloat16>(ld_in(xr + i * 16), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = (threadIdx.x & 31) < (blockDim.x >> 5) ? red[threadIdx.x & 31] : 0.f;
  t = warp_sum(t);
  const float inv = rsqrtf(t / hidden + eps);
  for (int i = threadIdx.x; i < hp; i += blockDim.x) {
    float v[8], g[8];
    unpack_set<__nv_bfloat16>(ld_in(xr + i * 16), v);
    unpack_set<__nv_bfloat16>(ld_in(reinterpret_cast<const char*>(gamma) + i * 16), g);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = v[e] * inv * g[e];
    st_out(yr + i * 16, pack<__nv_bfloat16>(v));
  }
}

// ------------------------------------------------------------------ RoPE + KV write
// Grid (B, Hq + Hkv); block = D / 2 threads; thread i rotates the pair (i, i + D/2).
__global__ void rope_kv_kernel(const __nv_bfloat16* __restrict__ qkv, const int* __restrict__ pos,
                               const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                               __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                               __nv_bfloat16* __restrict__ v_cache, int hq, int hkv, int d, int max_len) {
  const int b = blockIdx.x, h = blockIdx.y, i = threadIdx.x, half = d / 2;
  const int p = pos[b];
  if (p < 0 || p >= max_len) return;  // past the cache and the rotary table: nothing to write
  const int64_t row = static_cast<int64_t>(b) * (hq + 2 * hkv) * d;
  const float c = cos_t[static_cast<int64_t>(p) * half + i];
  const float s = sin_t[static_cast<int64_t>(p) * half + i];
  const __nv_bfloat16* src = qkv + row + static_cast<int64_t>(h) * d;
  const float x0 = __bfloat162float(src[i]), x1 = __bfloat162float(src[i + half]);
  const __nv_bfloat16 r0 = __float2bfloat16_rn(x0 * c - x1 * s);
  const __nv_bfloat16 r1 = __float2bfloat16_rn(x1 * c + x0 * s);
  if (h < hq) {
    __nv_bfloat16* dst = q_out + (static_cast<int64_t>(b) * hq + h) * d;
    dst[i] = r0;
    dst[i + half] = r1;
  } else {
    const int kh = h - hq;
    const int64_t off = ((static_cast<int64_t>(b) * max_len + p) * hkv + kh) * d;
    k_cache[off + i] = r0;
    k_cache[off + i + half] = r1;
    const __nv_bfloat16* vs = qkv + row + static_cast<int64_t>(hq + hkv + kh) * d;
    v_cache[off + i] = vs[i];
    v_cache[off + i + half] = vs[i + half];
  }
}

// ------------------------------------------------------------------ decode attention
// Grid (B, Hkv, splits), 4 warps. Both products run on the tensor cores with
// mma.sync m16n8k16 (bf16 in, fp32 accumulate):
//   S = Q K^T   rows = the G query heads of the KV head (padded to 16),
//               columns = tokens; K fragments come from shared memory with
//               ldmatrix, so every K element is read from shared memory once
//               per CTA whatever G is;
//   O += P V    P is the softmax numerator, re-used from the S accumulators as
//               the A operand (the accumulator layout of m16n8k16 is the A
//               layout of the next m16n8k16); V fragments via ldmatrix.trans.
// The CTA walks its token range in chunks of kChunk tokens, double-buffered
// with cp.async; warp w owns tokens [16 w, 16 w + 16) of every chunk and keeps
// its own online-softmax state (max and sum in the log2 domain). The four
// warp states are merged through shared memory at the end, and the last split
// CTA of the (batch, KV head) merges the split states.
// Launch bounds: 128 threads; shared memory 68 KB -> 3 CTAs per SM.
constexpr int kHeadDim = 128;
constexpr int kChunk = 64;
constexpr int kAttnWarps = kChunk / 16;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kAttnMaxGroup = 16;
constexpr int kRowPad = kHeadDim + 8;  // bf16 per shared K/V row: 272 B, so 8 ldmatrix rows hit 8 bank groups
constexpr size_t kAttnSmem = 4 * kChunk * kRowPad * sizeof(__nv_bfloat16);
static_assert(kAttnThreads == kHeadDim, "the CTA merge gives one head dimension to each thread");
static_assert(kAttnWarps * kAttnMaxGroup * (kHeadDim + 2) * sizeof(float) <= kAttnSmem,
              "the merge area aliases the K/V buffers");

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int n = pred ? 16 : 0;  // zero-fill beyond the sequence
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
// D += A B for one m16n8k16 tile (A row-major 16x16, B column-major 16x8).
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__global__ void __launch_bounds__(kAttnThreads)
    attn_partial_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
                        const __nv_bfloat16* __restrict__ v_cache, const int* __restrict__ seq_len,
                        float* __restrict__ part_acc, float* __restrict__ part_ml,
                        unsigned* __restrict__ done_count, __nv_bfloat16* __restrict__ out, int hkv, int group,
                        int max_len, int splits, float scale_log2) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(attn_smem);  // [2][kChunk][kRowPad]
  __nv_bfloat16* sV = sK + 2 * kChunk * kRowPad;                     // [2][kChunk][kRowPad]

  const int b = blockIdx.x, kh = blockIdx.y, sp = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;  // fragment row group and thread-in-group
  const int len = seq_len[b];
  const int t0 = static_cast<int>((static_cast<int64_t>(len) * sp) / splits);
  const int t1 = static_cast<int>((static_cast<int64_t>(len) * (sp + 1)) / splits);
  const int hq = hkv * group;
  const int64_t tok_stride = static_cast<int64_t>(hkv) * kHeadDim;
  const __nv_bfloat16* kbase = k_cache + (static_cast<int64_t>(b) * max_len * hkv + kh) * kHeadDim;
  const __nv_bfloat16* vbase = v_cache + (static_cast<int64_t>(b) * max_len * hkv + kh) * kHeadDim;

  auto load_chunk = [&](int c, int buf) {
    const int tb = t0 + c * kChunk;
    // kChunk tokens x 16 packets each, for K and for V.
    for (int i = threadIdx.x; i < kChunk * 16; i += kAttnThreads) {
      const int tt = i >> 4, pk = i & 15;
      const bool ok = tb + tt < t1;
      const int64_t off = static_cast<int64_t>(ok ? tb + tt : t0) * tok_stride + pk * 8;
      cp_async16(sK + (buf * kChunk + tt) * kRowPad + pk * 8, kbase + off, ok);
      cp_async16(sV + (buf * kChunk + tt) * kRowPad + pk * 8, vbase + off, ok);
    }
    cp_async_commit();
  };
  const int nchunks = (t1 - t0 + kChunk - 1) / kChunk;
  if (nchunks > 0) load_chunk(0, 0);

  // Q as A fragments, one per 16-dim k step: rows g and g + 8 of the group
  // (zero rows beyond the group size).
  const __nv_bfloat16* qg = q + (static_cast<int64_t>(b) * hq + static_cast<int64_t>(kh) * group) * kHeadDim;
  uint32_t qf[kHeadDim / 16][4];
#pragma unroll
  for (int ks = 0; ks < kHeadDim / 16; ++ks) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int row = g + 8 * (j & 1);
      const int col = ks * 16 + 8 * (j >> 1) + 2 * tig;
      qf[ks][j] = row < group ? __ldg(reinterpret_cast<const unsigned*>(qg + row * kHeadDim + col)) : 0u;
    }
  }

  float o[kHeadDim / 8][4];
#pragma unroll
  for (int nd = 0; nd < kHeadDim / 8; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};  // rows g and g + 8
  const int mi = lane >> 3, r8 = lane & 7;                   // ldmatrix: matrix index, row in matrix

  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunks) {
      load_chunk(c + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int wt = t0 + c * kChunk + warp * 16;  // first token of this warp's slice
    if (wt < t1) {
      const __nv_bfloat16* K = sK + (buf * kChunk + warp * 16) * kRowPad;
      const __nv_bfloat16* V = sV + (buf * kChunk + warp * 16) * kRowPad;
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int kp = 0; kp < kHeadDim / 32; ++kp) {
          uint32_t kb[4];  // B fragments of k steps 2 kp and 2 kp + 1 for 8 tokens
          ldsm_x4(kb, K + (nt * 8 + r8) * kRowPad + kp * 32 + mi * 8);
          mma_bf16(s[nt], qf[2 * kp], kb[0], kb[1]);
          mma_bf16(s[nt], qf[2 * kp + 1], kb[2], kb[3]);
        }
      }
      // Scale into the log2 domain and mask tokens past the range.
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          s[nt][e] = wt + nt * 8 + 2 * tig + (e & 1) < t1 ? s[nt][e] * scale_log2 : -INFINITY;
      uint32_t pa[4];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float mx = fmaxf(fmaxf(s[0][2 * r], s[0][2 * r + 1]), fmaxf(s[1][2 * r], s[1][2 * r + 1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m[r], mx);
        const float corr = m[r] == -INFINITY ? 0.f : exp2f(m[r] - mn);
        m[r] = mn;
        float p[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) p[nt][e] = s[nt][2 * r + e] == -INFINITY ? 0.f : exp2f(s[nt][2 * r + e] - mn);
        l[r] = l[r] * corr + p[0][0] + p[0][1] + p[1][0] + p[1][1];
#pragma unroll
        for (int nd = 0; nd < kHeadDim / 8; ++nd) {
          o[nd][2 * r] *= corr;
          o[nd][2 * r + 1] *= corr;
        }
        pa[r] = pack_bf16(p[0][0], p[0][1]);      // a0 (row g) / a1 (row g + 8): tokens 2 tig, 2 tig + 1
        pa[2 + r] = pack_bf16(p[1][0], p[1][1]);  // a2 / a3: tokens 8 + 2 tig, 9 + 2 tig
      }
#pragma unroll
      for (int ndp = 0; ndp < kHeadDim / 16; ++ndp) {
        uint32_t vb[4];  // B fragments (tokens 0-7, 8-15) of dim tiles 2 ndp and 2 ndp + 1
        ldsm_x4_trans(vb, V + ((mi & 1) * 8 + r8) * kRowPad + (2 * ndp + (mi >> 1)) * 8);
        mma_bf16(o[2 * ndp], pa, vb[0], vb[1]);
        mma_bf16(o[2 * ndp + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();  // the buffer is refilled by the next iteration's prefetch
  }

  // Merge the four warp states of this CTA (the merge area aliases K/V).
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
  float* sO = reinterpret_cast<float*>(attn_smem);             // [warps][16][kHeadDim]
  float* sML = sO + kAttnWarps * kAttnMaxGroup * kHeadDim;      // [warps][16][2]
#pragma unroll
  for (int nd = 0; nd < kHeadDim / 8; ++nd)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      sO[(warp * kAttnMaxGroup + g + 8 * (e >> 1)) * kHeadDim + nd * 8 + 2 * tig + (e & 1)] = o[nd][e];
  if (tig == 0) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      sML[(warp * kAttnMaxGroup + g + 8 * r) * 2 + 0] = m[r];
      sML[(warp * kAttnMaxGroup + g + 8 * r) * 2 + 1] = l[r];
    }
  }
  __syncthreads();
  const int64_t head0 = static_cast<int64_t>(b) * hq + static_cast<int64_t>(kh) * group;
  for (int h = 0; h < group; ++h) {
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, sML[(w * kAttnMaxGroup + h) * 2]);
    float acc = 0.f, ll = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float mw = sML[(w * kAttnMaxGroup + h) * 2];
      const float f = mw == -INFINITY ? 0.f : exp2f(mw - mm);
      acc += sO[(w * kAttnMaxGroup + h) * kHeadDim + threadIdx.x] * f;
      ll += sML[(w * kAttnMaxGroup + h) * 2 + 1] * f;
    }
    const int64_t base = (head0 + h) * splits + sp;
    part_acc[base * kHeadDim + threadIdx.x] = acc;
    if (threadIdx.x == 0) {
      part_ml[base * 2 + 0] = mm;
      part_ml[base * 2 + 1] = ll;
    }
  }

  // Merge the splits: the split CTA that finishes last combines all partials
  // of its (batch, KV head) and re-arms the counter for the next launch
  // (counters start at zero). Fence, then count: the classic last-block
  // reduction.
  __shared__ unsigned is_last;
  __threadfence();
  __syncthreads();
  unsigned* cnt = done_count + static_cast<int64_t>(b) * hkv + kh;
  if (threadIdx.x == 0) is_last = atomicAdd(cnt, 1u) == static_cast<unsigned>(splits - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (threadIdx.x == 0) *cnt = 0u;
  for (int h = warp; h < group; h += kAttnWarps) {
    const int64_t head = head0 + h;
    const float* ml = part_ml + head * splits * 2;
    const float* pp = part_acc + head * splits * kHeadDim + lane * 4;
    float mm = -INFINITY;
    for (int s2 = 0; s2 < splits; ++s2) mm = fmaxf(mm, __ldcg(ml + 2 * s2));
    float ll = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int s2 = 0; s2 < splits; ++s2) {
      const float ms = __ldcg(ml + 2 * s2);
      const float f = ms == -INFINITY ? 0.f : exp2f(ms - mm);
      ll += __ldcg(ml + 2 * s2 + 1) * f;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(pp + static_cast<int64_t>(s2) * kHeadDim));
      acc[0] += a.x * f;
      acc[1] += a.y * f;
      acc[2] += a.z * f;
      acc[3] += a.w * f;
    }
    const float inv = ll > 0.f ? 1.f / ll : 0.f;
    __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(out + head * kHeadDim + lane * 4);
    dst[0] = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
    dst[1] = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
  }
}

// ------------------------------------------------------------------ SiLU gate
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ y, int inter,
                                int64_t rows, int group) {
  const int ip = inter / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < rows * ip;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / ip, c = i % ip;
    const char* row = reinterpret_cast<const char*>(gu + r * 2 * inter);
    // Element offsets of this packet's gate and up values.
    int64_t go = c * 8, uo = static_cast<int64_t>(inter) + c * 8;
    if (group > 0) {
      const int64_t j = c * 8;
      go = (j / group) * 2 * group + j % group;
      uo = go + group;
    }
    float g[8], u[8];
    unpack_set<__nv_bfloat16>(ld_in(row + go * 2), g);
    unpack_set<__nv_bfloat16>(ld_in(row + uo * 2), u);
#pragma unroll
    for (int e = 0; e < 8; ++e) g[e] = g[e] / (1.f + __expf(-g[e])) * u[e];
    st_out(reinterpret_cast<char*>(y + r * inter) + c * 16, pack<__nv_bfloat16>(g));
  }
}

}  // namespace

void rmsnorm(const void* x, const void* gamma, void* y, int64_t rows, int64_t hidden, float eps, cudaStream_t s) {
  const TraceRange trace("b200ar::rmsnorm");
  B200AR_CHECK(hidden % 8 == 0, "hidden must be a multiple of 8");
  const int threads = static_cast<int>(std::min<int64_t>(512, std::max<int64_t>(32, (hidden / 8 + 31) / 32 * 32)));
  rmsnorm_kernel<<<static_cast<unsigned>(rows), threads, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                                 static_cast<const __nv_bfloat16*>(gamma),
                                                                 static_cast<__nv_bfloat16*>(y),
                                                                 static_cast<int>(hidden), eps);
  B200AR_CUDA(cudaGetLastError());
}

void rope_kv(const void* qkv, const int* pos, const float* cos_t, const float* sin_t, void* q_out, void* k_cache,
             void* v_cache, int64_t batch, int hq, int hkv, int head_dim, int max_len, cudaStream_t s) {
  const TraceRange trace("b200ar::rope_kv");
  B200AR_CHECK(head_dim % 2 == 0 && head_dim <= 1024, "bad head dim");
  rope_kv_kernel<<<dim3(static_cast<unsigned>(batch), hq + hkv), head_dim / 2, 0, s>>>(
      static_cast<const __nv_bfloat16*>(qkv), pos, cos_t, sin_t, static_cast<__nv_bfloat16*>(q_out),
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), hq, hkv, head_dim, max_len);
  B200AR_CUDA(cudaGetLastError());
}

int attention_splits(int64_t batch, int hkv, int max_len) {
  // One wave of 3 CTAs per SM (the kernel's shared memory allows 3), rounded
  // down so no second partial wave forms; at least two chunks of cache per
  // split, which keeps the final merge (serial over splits) short.
  const int64_t ctas = std::max<int64_t>(batch * hkv, 1);
  int s = static_cast<int>(std::max<int64_t>(1, (3 * 148) / ctas));
  s = std::min(s, std::max(1, max_len / (2 * kChunk)));
  return std::min(s, 64);
}

void decode_attention(const void* q, const void* k_cache, const void* v_cache, const int* seq_len, void* out,
                      float* part_acc, float* part_ml, unsigned* done_count, int64_t batch, int hq, int hkv,
                      int head_dim, int max_len, int splits, float scale, cudaStream_t s) {
  const TraceRange trace("b200ar::decode_attention");
  B200AR_CHECK(head_dim == kHeadDim, "decode attention is built for head_dim 128");
  B200AR_CHECK(hkv > 0 && hq % hkv == 0, "query heads must be a multiple of KV heads");
  const int group = hq / hkv;
  B200AR_CHECK(group <= kAttnMaxGroup, "GQA group size must be at most 16");
  B200AR_CHECK(splits >= 1, "splits must be positive");
  static PerDeviceOnce smem_attr;
  smem_attr([&] {
    B200AR_CUDA(cudaFuncSetAttribute(attn_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kAttnSmem)));
  });
  const dim3 grid(static_cast<unsigned>(batch), hkv, splits);
  attn_partial_kernel<<<grid, kAttnThreads, kAttnSmem, s>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k_cache),
      static_cast<const __nv_bfloat16*>(v_cache), seq_len, part_acc, part_ml, done_count,
      static_cast<__nv_bfloat16*>(out), hkv, group, max_len, splits, scale * 1.4426950408889634f);
  B200AR_CUDA(cudaGetLastError());
}

void silu_mul(const void* gate_up, void* y, int64_t rows, int64_t inter, cudaStream_t s, int group) {
  const TraceRange trace("b200ar::silu_mul");
  B200AR_CHECK(inter % 8 == 0, "intermediate size must be a multiple of 8");
  B200AR_CHECK(group == 0 || (group % 8 == 0 && inter % group == 0),
               "interleave group must be a multiple of 8 that divides the intermediate size");
  const int64_t items = rows * inter / 8;
  const int blocks = static_cast<int>(std::min<int64_t>((items + 255) / 256, 4 * 148));
  silu_mul_kernel<<<std::max(blocks, 1), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gate_up),
                                                     static_cast<__nv_bfloat16*>(y), static_cast<int>(inter), rows,
                                                     group);
  B200AR_CUDA(cudaGetLastError());
}

}  // namespace b200ar
