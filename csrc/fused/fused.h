// Fused tensor-parallel collectives built on the Communicator's slots/signals.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace b200ar {

class Communicator;

// Slot bytes the fused all-reduce + RMSNorm needs for `rows` x `hidden` bf16.
int64_t ar_rmsnorm_slot_bytes(int variant, int64_t rows, int64_t hidden, int world);

// y = RMSNorm(sum_ranks(x) + residual) * gamma, residual_out = sum_ranks(x) + residual
// (bf16 [rows, hidden]; residual_out may alias residual, y may alias x).
// Returns the variant launched (kOneshotPush or kTwoshot).
int ar_rmsnorm(Communicator& comm, cudaStream_t stream, const void* x, const void* residual, const void* gamma,
               void* y, void* residual_out, int64_t rows, int64_t hidden, float eps, int variant, int ctas);

// Fused row-parallel linear + all-reduce: out = sum_ranks(A_r @ W_r^T)
// (bf16 A [M, K], W [N, K], out [M, N]). `err` receives GEMM wait errors.
int64_t gemm_ar_slot_bytes(int64_t M, int64_t N, int world);
bool gemm_ar_supported(Communicator& comm, int64_t M, int64_t N);
void gemm_allreduce(Communicator& comm, cudaStream_t stream, const void* A, const void* W, void* out, int64_t M,
                    int64_t N, int64_t K, int* err);

// Column-parallel linear with the all-gather fused into the GEMM prologue:
// Y[rows_per_rank * world, N] = concat_ranks(x_shard) @ W^T.
bool ag_gemm_supported(Communicator& comm, int64_t rows_per_rank, int64_t K);
void ag_gemm(Communicator& comm, cudaStream_t stream, const void* x_shard, const void* W, void* Y,
             int64_t rows_per_rank, int64_t N, int64_t K, int* err);

}  // namespace b200ar
