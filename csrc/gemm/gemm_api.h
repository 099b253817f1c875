// Host API of the tcgen05 GEMM (gemm.cu).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace b200ar {

namespace gemm {
struct Shape;
}

// 2-D bf16 tensor map (row-major [rows, cols], leading dimension ld elements)
// with a box of box_rows x box_cols and 128-byte swizzle; no multicast.
CUtensorMap make_tmap_bf16_2d(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols);

// Tile counts for an M x N x K problem (validates the shape).
gemm::Shape gemm_shape(int64_t M, int64_t N, int64_t K);

// Persistent grid size for a shape (at most one CTA per SM, `max_ctas` if > 0).
int gemm_grid(const gemm::Shape& s, int max_ctas);

// C[M, N] (bf16, row-major) = A[M, K] * B[N, K]^T. `err` is a device int that
// receives a non-zero code if a bounded wait expired.
void gemm_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int* err,
               cudaStream_t stream, int max_ctas = 0);

// The same product on CTA pairs (tcgen05 cta_group::2, 256 x 256 tiles,
// clusters of 2): half the operand traffic per SM of the single-CTA kernel.
void gemm_bf16_2sm(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int* err,
                   cudaStream_t stream, int max_pairs = 0);

// Decode GEMM for M <= 128 (swap-AB, split-K over `splits` CTAs per 128-row
// weight block). `partials` (fp32 [splits, M, N]) and `counters` (zeroed
// uint32 [ceil(N / 128)]) are needed when splits > 1; calls that share them
// must be ordered on one stream. `epilogue` 1 treats W as gate and up rows
// interleaved in groups of 64 and writes silu(gate) * up to out[M, N / 2]
// (N a multiple of 128; partials and counters are needed for every split
// count).
// `epilogue` 2 treats W as the QKV projection (one 128-row block per head,
// [q | k | v]) and, instead of writing `out`, rotates q and k (rotate-half
// RoPE at pos[m]) and writes q to q_out[M, hq, 128] and k, v into the caches
// [M, max_len, hkv, 128] at pos[m].
struct RopeKvArgs {
  const int* pos;
  const float* cos_t;  // [positions, 64]
  const float* sin_t;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int hq, hkv, max_len;
};
int skinny_splits(int64_t N, int64_t K, int sms);
void gemm_skinny(const void* x, const void* w, void* out, float* partials, unsigned* counters, int64_t M, int64_t N,
                 int64_t K, int splits, int* err, cudaStream_t stream, int epilogue = 0,
                 const RopeKvArgs* rope = nullptr);

}  // namespace b200ar
