// Model kernels for the tensor-parallel Llama decoder slice (sm_100a):
//   rmsnorm        y = x * rsqrt(mean(x^2) + eps) * gamma               (bf16 rows)
//   rope_kv        rotary embedding of q and k (rotate-half convention), q to a
//                  contiguous buffer, k and v written into the KV cache at `pos`
//   attention      GQA decode attention, split over the KV length
//                  (flash-decoding): partial softmax state per split, then a
//                  combine kernel; K/V of one KV head are read once for all the
//                  query heads of its group
//   silu_mul       y = silu(gate) * up for gate_up = [gate | up]
// All kernels move 16-byte packets and accumulate in fp32. The reference
// library has no model code; these serve BASELINE configuration 5.
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
// Grid (B, Hkv, splits); 4 warps. Head dim 128: lane holds dims [4 lane, 4 lane + 4).
// Every warp walks tokens t = split_begin + warp, +4, ...; for each token it
// scores all G query heads of the group, keeps an online softmax per head.
constexpr int kAttnWarps = 4;
constexpr int kHeadDim = 128;

template <int G>
__global__ void __launch_bounds__(kAttnWarps * 32)
    attn_partial_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
                        const __nv_bfloat16* __restrict__ v_cache, const int* __restrict__ seq_len,
                        float* __restrict__ part_acc, float* __restrict__ part_ml, int hkv, int max_len,
                        int splits, float scale) {
  const int b = blockIdx.x, kh = blockIdx.y, sp = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = seq_len[b];
  const int t0 = static_cast<int>((static_cast<int64_t>(len) * sp) / splits);
  const int t1 = static_cast<int>((static_cast<int64_t>(len) * (sp + 1)) / splits);
  const int hq = hkv * G;

  float qv[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const __nv_bfloat16* qp = q + (static_cast<int64_t>(b) * hq + kh * G + g) * kHeadDim + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(qp);
    qv[g][0] = __uint_as_float(raw.x << 16) * scale;
    qv[g][1] = __uint_as_float(raw.x & 0xffff0000u) * scale;
    qv[g][2] = __uint_as_float(raw.y << 16) * scale;
    qv[g][3] = __uint_as_float(raw.y & 0xffff0000u) * scale;
  }
  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
    acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
  }
  // Each warp takes kUnroll consecutive tokens per step: their K/V loads are
  // issued together, then scored one after the other (hides load latency).
  constexpr int kUnroll = 4;
  for (int tb = t0 + warp * kUnroll; tb < t1; tb += kAttnWarps * kUnroll) {
    uint2 kr[kUnroll], vr[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int t = tb + u < t1 ? tb + u : t1 - 1;
      const int64_t off = ((static_cast<int64_t>(b) * max_len + t) * hkv + kh) * kHeadDim + lane * 4;
      kr[u] = __ldg(reinterpret_cast<const uint2*>(k_cache + off));
      vr[u] = __ldg(reinterpret_cast<const uint2*>(v_cache + off));
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (tb + u >= t1) break;
      const float kx[4] = {__uint_as_float(kr[u].x << 16), __uint_as_float(kr[u].x & 0xffff0000u),
                           __uint_as_float(kr[u].y << 16), __uint_as_float(kr[u].y & 0xffff0000u)};
      const float vx[4] = {__uint_as_float(vr[u].x << 16), __uint_as_float(vr[u].x & 0xffff0000u),
                           __uint_as_float(vr[u].y << 16), __uint_as_float(vr[u].y & 0xffff0000u)};
      float sc[G];
#pragma unroll
      for (int g = 0; g < G; ++g) sc[g] = qv[g][0] * kx[0] + qv[g][1] * kx[1] + qv[g][2] * kx[2] + qv[g][3] * kx[3];
      // All G reductions interleaved (independent shuffle chains).
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], o);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float mn = fmaxf(m[g], sc[g]);
        const float corr = __expf(m[g] - mn);
        const float pexp = __expf(sc[g] - mn);
        l[g] = l[g] * corr + pexp;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[g][e] = acc[g][e] * corr + pexp * vx[e];
        m[g] = mn;
      }
    }
  }
  // Merge the 4 warps through shared memory.
  __shared__ float s_m[kAttnWarps][G], s_l[kAttnWarps][G];
  __shared__ float s_acc[kAttnWarps][G][kHeadDim];
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 4; ++e) s_acc[warp][g][lane * 4 + e] = acc[g][e];
  __syncthreads();
  // Thread layout for the merge: (g, dim) pairs over the 128 threads.
  for (int idx = threadIdx.x; idx < G * kHeadDim; idx += blockDim.x) {
    const int g = idx / kHeadDim, dmn = idx % kHeadDim;
    float mm = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, s_m[w][g]);
    float ll = 0.f, aa = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = s_m[w][g] == -INFINITY ? 0.f : __expf(s_m[w][g] - mm);
      ll += s_l[w][g] * f;
      aa += s_acc[w][g][dmn] * f;
    }
    const int64_t base = ((static_cast<int64_t>(b) * hq + kh * G + g) * splits + sp);
    part_acc[base * kHeadDim + dmn] = aa;
    if (dmn == 0) {
      part_ml[base * 2 + 0] = mm;
      part_ml[base * 2 + 1] = ll;
    }
  }
}

// Grid (B * Hq); 128 threads = head dims.
__global__ void attn_combine_kernel(const float* __restrict__ part_acc, const float* __restrict__ part_ml,
                                    __nv_bfloat16* __restrict__ out, int splits) {
  const int64_t bh = blockIdx.x;
  const int dmn = threadIdx.x;
  const float* ml = part_ml + bh * splits * 2;
  const float* pa = part_acc + bh * splits * kHeadDim + dmn;
  float mm = -INFINITY;
#pragma unroll 8
  for (int s = 0; s < splits; ++s) mm = fmaxf(mm, ml[2 * s]);
  float ll = 0.f, aa = 0.f;
#pragma unroll 8
  for (int s = 0; s < splits; ++s) {
    const float ms = ml[2 * s];
    const float f = ms == -INFINITY ? 0.f : __expf(ms - mm);
    ll += ml[2 * s + 1] * f;
    aa += pa[static_cast<int64_t>(s) * kHeadDim] * f;
  }
  out[bh * kHeadDim + dmn] = __float2bfloat16_rn(ll > 0.f ? aa / ll : 0.f);
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
  int s = static_cast<int>(std::max<int64_t>(1, 2 * 148 / std::max<int64_t>(ctas, 1)));
  s = std::min(s, std::max(1, max_len / 128));  // at least ~128 tokens per split
  return std::min(s, 64);
}

void decode_attention(const void* q, const void* k_cache, const void* v_cache, const int* seq_len, void* out,
                      float* part_acc, float* part_ml, int64_t batch, int hq, int hkv, int head_dim, int max_len,
                      int splits, float scale, cudaStream_t s) {
  B200AR_CHECK(head_dim == kHeadDim, "decode attention is built for head_dim 128");
  B200AR_CHECK(hq % hkv == 0, "query heads must be a multiple of KV heads");
  const int G = hq / hkv;
  const dim3 grid(static_cast<unsigned>(batch), hkv, splits);
  const auto* qp = static_cast<const __nv_bfloat16*>(q);
  const auto* kp = static_cast<const __nv_bfloat16*>(k_cache);
  const auto* vp = static_cast<const __nv_bfloat16*>(v_cache);
  switch (G) {
    case 1: attn_partial_kernel<1><<<grid, kAttnWarps * 32, 0, s>>>(qp, kp, vp, seq_len, part_acc, part_ml, hkv, max_len, splits, scale); break;
    case 2: attn_partial_kernel<2><<<grid, kAttnWarps * 32, 0, s>>>(qp, kp, vp, seq_len, part_acc, part_ml, hkv, max_len, splits, scale); break;
    case 4: attn_partial_kernel<4><<<grid, kAttnWarps * 32, 0, s>>>(qp, kp, vp, seq_len, part_acc, part_ml, hkv, max_len, splits, scale); break;
    case 8: attn_partial_kernel<8><<<grid, kAttnWarps * 32, 0, s>>>(qp, kp, vp, seq_len, part_acc, part_ml, hkv, max_len, splits, scale); break;
    default: throw std::invalid_argument("GQA group size must be 1, 2, 4 or 8");
  }
  B200AR_CUDA(cudaGetLastError());
  attn_combine_kernel<<<static_cast<unsigned>(batch * hq), kHeadDim, 0, s>>>(part_acc, part_ml,
                                                                             static_cast<__nv_bfloat16*>(out), splits);
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
