// Model kernels for the tensor-parallel Llama decoder slice (sm_100a):
//   rmsnorm        y = x * rsqrt(mean(x^2) + eps) * gamma               (bf16 rows)
//   rope_kv        rotary embedding of q and k (rotate-half convention), q to a
//                  contiguous buffer, k and v written into the KV cache at `pos`
//   attention      GQA decode attention, split over the KV length
//                  (flash-decoding): partial softmax state per split; the
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
// Grid (B, Hkv, splits); one warp per query head of the group (G warps).
// The CTA walks its token range in chunks of kChunk tokens: K and V of the
// next chunk are copied to shared memory with cp.async while the current
// chunk is processed, so global latency is paid once per chunk, not per token.
//   scores: lane j of warp h scores tokens j and j + 32 of the chunk
//           (128-wide dot product from shared memory, no shuffles);
//   softmax: one max and one sum reduction per warp and chunk (online);
//   P.V:    lane j accumulates head dims [4 j, 4 j + 4) over the chunk.
constexpr int kHeadDim = 128;
constexpr int kChunk = 64;
constexpr int kRowPad = kHeadDim + 8;  // bf16 per shared K/V row (16-byte pad: no bank conflicts)

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

template <int G>
__global__ void __launch_bounds__(G * 32)
    attn_partial_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
                        const __nv_bfloat16* __restrict__ v_cache, const int* __restrict__ seq_len,
                        float* __restrict__ part_acc, float* __restrict__ part_ml,
                        unsigned* __restrict__ done_count, __nv_bfloat16* __restrict__ out, int hkv, int max_len,
                        int splits, float scale) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(attn_smem);          // [2][kChunk][kRowPad]
  __nv_bfloat16* sV = sK + 2 * kChunk * kRowPad;                             // [2][kChunk][kRowPad]
  float* sQ = reinterpret_cast<float*>(sV + 2 * kChunk * kRowPad);           // [G][kHeadDim]
  float* sP = sQ + G * kHeadDim;                                             // [G][kChunk]

  const int b = blockIdx.x, kh = blockIdx.y, sp = blockIdx.z;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = seq_len[b];
  const int t0 = static_cast<int>((static_cast<int64_t>(len) * sp) / splits);
  const int t1 = static_cast<int>((static_cast<int64_t>(len) * (sp + 1)) / splits);
  const int hq = hkv * G;
  const int64_t tok_stride = static_cast<int64_t>(hkv) * kHeadDim;
  const __nv_bfloat16* kbase = k_cache + (static_cast<int64_t>(b) * max_len * hkv + kh) * kHeadDim;
  const __nv_bfloat16* vbase = v_cache + (static_cast<int64_t>(b) * max_len * hkv + kh) * kHeadDim;

  // Queries (scaled) to shared memory as fp32.
  for (int i = threadIdx.x; i < G * kHeadDim; i += blockDim.x)
    sQ[i] = __bfloat162float(q[(static_cast<int64_t>(b) * hq + kh * G) * kHeadDim + i]) * scale;

  auto load_chunk = [&](int c, int buf) {
    const int tb = t0 + c * kChunk;
    // 64 tokens x 16 packets each for K and for V.
    for (int i = threadIdx.x; i < kChunk * 16; i += blockDim.x) {
      const int tt = i >> 4, pk = i & 15;
      const bool ok = tb + tt < t1;
      const int64_t off = static_cast<int64_t>(ok ? tb + tt : t0) * tok_stride + pk * 8;
      cp_async16(sK + (buf * kChunk + tt) * kRowPad + pk * 8, kbase + off, ok);
      cp_async16(sV + (buf * kChunk + tt) * kRowPad + pk * 8, vbase + off, ok);
    }
    cp_async_commit();
  };

  const int nchunks = (t1 - t0 + kChunk - 1) / kChunk;
  float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (nchunks > 0) load_chunk(0, 0);
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunks) {
      load_chunk(c + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int tb = t0 + c * kChunk;
    const __nv_bfloat16* K = sK + buf * kChunk * kRowPad;
    const __nv_bfloat16* V = sV + buf * kChunk * kRowPad;
    const float* qh = sQ + h * kHeadDim;
    // Scores of tokens lane and lane + 32.
    float sc[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int tt = lane + 32 * u;
      const uint4* kr = reinterpret_cast<const uint4*>(K + tt * kRowPad);
      float s = 0.f;
#pragma unroll
      for (int d8 = 0; d8 < kHeadDim / 8; ++d8) {
        float kx[8];
        unpack_set<__nv_bfloat16>(kr[d8], kx);
        const float4 qa = *reinterpret_cast<const float4*>(qh + d8 * 8);
        const float4 qb = *reinterpret_cast<const float4*>(qh + d8 * 8 + 4);
        s += qa.x * kx[0] + qa.y * kx[1] + qa.z * kx[2] + qa.w * kx[3] + qb.x * kx[4] + qb.y * kx[5] +
             qb.z * kx[6] + qb.w * kx[7];
      }
      sc[u] = tb + tt < t1 ? s : -INFINITY;
    }
    float cmax = fmaxf(sc[0], sc[1]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
    const float mn = fmaxf(m, cmax);
    const float corr = m == -INFINITY ? 0.f : __expf(m - mn);
    const float p0 = sc[0] == -INFINITY ? 0.f : __expf(sc[0] - mn);
    const float p1 = sc[1] == -INFINITY ? 0.f : __expf(sc[1] - mn);
    float psum = p0 + p1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l = l * corr + psum;
    m = mn;
    sP[h * kChunk + lane] = p0;
    sP[h * kChunk + lane + 32] = p1;
    __syncwarp();
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] *= corr;
    const int lim = min(kChunk, t1 - tb);
    for (int tt = 0; tt < lim; ++tt) {
      const float p = sP[h * kChunk + tt];
      const uint2 vr = *reinterpret_cast<const uint2*>(V + tt * kRowPad + lane * 4);
      acc[0] += p * __uint_as_float(vr.x << 16);
      acc[1] += p * __uint_as_float(vr.x & 0xffff0000u);
      acc[2] += p * __uint_as_float(vr.y << 16);
      acc[3] += p * __uint_as_float(vr.y & 0xffff0000u);
    }
    __syncthreads();  // the buffer is refilled by the next iteration's prefetch
  }
  const int64_t head = static_cast<int64_t>(b) * hq + kh * G + h;
  const int64_t base = head * splits + sp;
  *reinterpret_cast<float4*>(part_acc + base * kHeadDim + lane * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  if (lane == 0) {
    part_ml[base * 2 + 0] = m;
    part_ml[base * 2 + 1] = l;
  }

  // Merge: the split CTA that finishes last combines all partials of its
  // (batch, KV head) and re-arms the counter for the next launch (counters
  // start at zero). Fence, then count: the classic last-block reduction.
  __shared__ unsigned is_last;
  __threadfence();
  __syncthreads();
  unsigned* cnt = done_count + static_cast<int64_t>(b) * hkv + kh;
  if (threadIdx.x == 0) is_last = atomicAdd(cnt, 1u) == static_cast<unsigned>(splits - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (threadIdx.x == 0) *cnt = 0u;
  const float* ml = part_ml + head * splits * 2;
  const float* pa = part_acc + head * splits * kHeadDim + lane * 4;
  float mm = -INFINITY;
  for (int s2 = 0; s2 < splits; ++s2) mm = fmaxf(mm, __ldcg(ml + 2 * s2));
  float ll = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int s2 = 0; s2 < splits; ++s2) {
    const float ms = __ldcg(ml + 2 * s2);
    const float f = ms == -INFINITY ? 0.f : __expf(ms - mm);
    ll += __ldcg(ml + 2 * s2 + 1) * f;
    const float4 a = __ldcg(reinterpret_cast<const float4*>(pa + static_cast<int64_t>(s2) * kHeadDim));
    o[0] += a.x * f;
    o[1] += a.y * f;
    o[2] += a.z * f;
    o[3] += a.w * f;
  }
  const float inv = ll > 0.f ? 1.f / ll : 0.f;
  __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(out + head * kHeadDim + lane * 4);
  dst[0] = __floats2bfloat162_rn(o[0] * inv, o[1] * inv);
  dst[1] = __floats2bfloat162_rn(o[2] * inv, o[3] * inv);
}

template <int G>
constexpr size_t attn_smem_bytes() {
  return (4 * kChunk * kRowPad) * sizeof(__nv_bfloat16) + (G * kHeadDim + G * kChunk) * sizeof(float);
}

// ------------------------------------------------------------------ SiLU gate
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ y, int inter,
                                int64_t rows) {
  const int ip = inter / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < rows * ip;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / ip, c = i % ip;
    const char* row = reinterpret_cast<const char*>(gu + r * 2 * inter);
    float g[8], u[8];
    unpack_set<__nv_bfloat16>(ld_in(row + c * 16), g);
    unpack_set<__nv_bfloat16>(ld_in(row + static_cast<int64_t>(inter) * 2 + c * 16), u);
#pragma unroll
    for (int e = 0; e < 8; ++e) g[e] = g[e] / (1.f + __expf(-g[e])) * u[e];
    st_out(reinterpret_cast<char*>(y + r * inter) + c * 16, pack<__nv_bfloat16>(g));
  }
}

}  // namespace

void rmsnorm(const void* x, const void* gamma, void* y, int64_t rows, int64_t hidden, float eps, cudaStream_t s) {
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
  B200AR_CHECK(head_dim % 2 == 0 && head_dim <= 1024, "bad head dim");
  rope_kv_kernel<<<dim3(static_cast<unsigned>(batch), hq + hkv), head_dim / 2, 0, s>>>(
      static_cast<const __nv_bfloat16*>(qkv), pos, cos_t, sin_t, static_cast<__nv_bfloat16*>(q_out),
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), hq, hkv, head_dim, max_len);
  B200AR_CUDA(cudaGetLastError());
}

int attention_splits(int64_t batch, int hkv, int max_len) {
  const int64_t ctas = batch * hkv;
  // About four CTAs per SM, and at least two chunks of tokens per split.
  int s = static_cast<int>(std::max<int64_t>(1, (4 * 148 + ctas - 1) / std::max<int64_t>(ctas, 1)));
  s = std::min(s, std::max(1, max_len / (2 * kChunk)));
  return std::min(s, 64);
}

void decode_attention(const void* q, const void* k_cache, const void* v_cache, const int* seq_len, void* out,
                      float* part_acc, float* part_ml, unsigned* done_count, int64_t batch, int hq, int hkv,
                      int head_dim, int max_len, int splits, float scale, cudaStream_t s) {
  B200AR_CHECK(head_dim == kHeadDim, "decode attention is built for head_dim 128");
  B200AR_CHECK(hq % hkv == 0, "query heads must be a multiple of KV heads");
  const int G = hq / hkv;
  const dim3 grid(static_cast<unsigned>(batch), hkv, splits);
  const auto* qp = static_cast<const __nv_bfloat16*>(q);
  const auto* kp = static_cast<const __nv_bfloat16*>(k_cache);
  const auto* vp = static_cast<const __nv_bfloat16*>(v_cache);
  switch (G) {
#define B200AR_ATTN(g)                                                                                      \
  case g: {                                                                                                 \
    auto kern = attn_partial_kernel<g>;                                                                     \
    static bool attr = false;                                                                               \
    if (!attr) {                                                                                            \
      B200AR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,                  \
                                       static_cast<int>(attn_smem_bytes<g>())));                            \
      attr = true;                                                                                          \
    }                                                                                                       \
    kern<<<grid, g * 32, attn_smem_bytes<g>(), s>>>(qp, kp, vp, seq_len, part_acc, part_ml, done_count,     \
                                                    static_cast<__nv_bfloat16*>(out), hkv, max_len, splits, \
                                                    scale);                                                 \
    break;                                                                                                  \
  }
    B200AR_ATTN(1)
    B200AR_ATTN(2)
    B200AR_ATTN(4)
    B200AR_ATTN(8)
#undef B200AR_ATTN
    default: throw std::invalid_argument("GQA group size must be 1, 2, 4 or 8");
  }
  B200AR_CUDA(cudaGetLastError());
}

void silu_mul(const void* gate_up, void* y, int64_t rows, int64_t inter, cudaStream_t s) {
  B200AR_CHECK(inter % 8 == 0, "intermediate size must be a multiple of 8");
  const int64_t items = rows * inter / 8;
  const int blocks = static_cast<int>(std::min<int64_t>((items + 255) / 256, 4 * 148));
  silu_mul_kernel<<<std::max(blocks, 1), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gate_up),
                                                     static_cast<__nv_bfloat16*>(y), static_cast<int>(inter), rows);
  B200AR_CUDA(cudaGetLastError());
}

}  // namespace b200ar
