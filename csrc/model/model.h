// Host API of the decoder model kernels (model_kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace b200ar {

void rmsnorm(const void* x, const void* gamma, void* y, int64_t rows, int64_t hidden, float eps, cudaStream_t s);
void rope_kv(const void* qkv, const int* pos, const float* cos_t, const float* sin_t, void* q_out, void* k_cache,
             void* v_cache, int64_t batch, int hq, int hkv, int head_dim, int max_len, cudaStream_t s);
int attention_splits(int64_t batch, int hkv, int max_len);
void decode_attention(const void* q, const void* k_cache, const void* v_cache, const int* seq_len, void* out,
                      float* part_acc, float* part_ml, unsigned* done_count, int64_t batch, int hq, int hkv,
                      int head_dim, int max_len, int splits, float scale, cudaStream_t s);
// Tensor-core (tcgen05) decode attention with TMA-fed K/V (attention_tc.cu);
// same workspace and split semantics as decode_attention, plus an error word
// that receives a non-zero code if a bounded wait expired.
int attention_tc_splits(int64_t batch, int hkv, int max_len);
void decode_attention_tc(const void* q, const void* k_cache, const void* v_cache, const int* seq_len, void* out,
                         float* part_acc, float* part_ml, unsigned* done_count, int* err, int64_t batch, int hq,
                         int hkv, int head_dim, int max_len, int splits, float scale, cudaStream_t s);
// y = silu(gate) * up. group 0: gate_up = [gate | up] (halves); group g > 0
// (a multiple of 8): gate and up columns interleaved in groups of g.
void silu_mul(const void* gate_up, void* y, int64_t rows, int64_t inter, cudaStream_t s, int group = 0);

}  // namespace b200ar
