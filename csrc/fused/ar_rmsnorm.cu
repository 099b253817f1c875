// Fused all-reduce + residual add + RMSNorm for tensor-parallel decode (sm_100a).
//
//   z = sum_ranks(x) + residual        (fp32 accumulation, rank order, rounded once)
//   y = z * rsqrt(mean(z^2) + eps) * gamma
//
// Outputs: y and the new residual z (may alias the residual input). The
// reference has no fused op (its kernels only sum, pcie_allreduce.cu:171-276);
// this is the all-reduce fused with residual-add + RMSNorm of tensor-parallel
// decode, built on the same signal/slot protocol as the plain
// all-reduce (generation counter, per-CTA bounded barriers, double-buffered slots).
//
// One CTA owns whole rows: a row of H bf16 values is H/8 16-byte packets and
// every thread holds PPT packets of it in registers across the row reduction.
//  * oneshot: every rank pushes its partial rows into slot[rank] of every peer,
//    one barrier, then each rank reduces all rows locally (latency optimal).
//  * twoshot: rows are split into N parts; rank p reduces and normalises part p,
//    then every rank pulls the finished y and z rows of the other parts
//    (2(N-1)/N of the bytes of one-shot's (N-1)).
//  * lamport: barrier-free one-shot (marker protocol); for decode batches the
//    cluster form splits every row over the C CTAs of a thread-block cluster
//    and combines the sum of squares through distributed shared memory.
#include <cooperative_groups.h>

#include <algorithm>
#include <stdexcept>

#include "../comm/ar_kernels.cuh"
#include "../comm/communicator.h"
#include "../common/trace.h"
#include "fused.h"
#include "../common/pdl.h"

namespace b200ar {

namespace {

constexpr int kMaxRowThreads = 512;

struct NormArgs {
  CommCtx ctx;
  char* slot[2][kMaxRanks];
  const char* x;      // [T, H] partial sums of this rank
  const char* res;    // [T, H] residual in
  const char* gamma;  // [H]
  char* y;            // [T, H] normalised output
  char* z;            // [T, H] new residual (may alias res)
  int rows;           // T
  int hp;             // H / 8 packets per row
  float eps;
  float inv_h;
  char* lam[kMaxRanks];  // Lamport regions (barrier-free variant)
  int64_t lam_cap;
};

// Sum over the CTA; every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] may still be read from the previous row
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// Reduces row `row` from `n` copies (copy q at src + q * stride), adds the
// residual, rounds z to bf16, normalises and stores y and z to the given
// destinations (y2/z2 optional second destinations, e.g. an outbox).
template <int N, int PPT>
__device__ __forceinline__ void reduce_norm_row(const NormArgs& a, const char* src, int64_t stride_bytes,
                                                int64_t row, char* ydst, char* zdst, char* y2, char* z2,
                                                float* red) {
  float zf[PPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int idx = threadIdx.x + k * blockDim.x;
    if (idx < a.hp) {
      uint4 v[N];
#pragma unroll
      for (int q = 0; q < N; ++q) v[q] = ld_cg(src + q * stride_bytes + static_cast<int64_t>(idx) * 16);
      float acc[8];
      unpack_set<__nv_bfloat16>(v[0], acc);
#pragma unroll
      for (int q = 1; q < N; ++q) unpack_add<__nv_bfloat16>(v[q], acc);
      unpack_add<__nv_bfloat16>(ld_in(a.res + (row * a.hp + idx) * 16), acc);
      const uint4 zp = pack<__nv_bfloat16>(acc);
      st_out(zdst + (row * a.hp + idx) * 16, zp);
      if (z2) st_cg(z2 + static_cast<int64_t>(idx) * 16, zp);
      unpack_set<__nv_bfloat16>(zp, zf[k]);  // statistics of the stored (rounded) residual
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += zf[k][e] * zf[k][e];
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) * a.inv_h + a.eps);
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int idx = threadIdx.x + k * blockDim.x;
    if (idx < a.hp) {
      float g[8];
      unpack_set<__nv_bfloat16>(ld_in(a.gamma + static_cast<int64_t>(idx) * 16), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) zf[k][e] = zf[k][e] * inv * g[e];
      const uint4 yp = pack<__nv_bfloat16>(zf[k]);
      st_out(ydst + (row * a.hp + idx) * 16, yp);
      if (y2) st_cg(y2 + static_cast<int64_t>(idx) * 16, yp);
    }
  }
}

template <int N, int PPT>
__global__ void __launch_bounds__(kMaxRowThreads) ar_rmsnorm_oneshot_kernel(NormArgs a) {
  pdl_wait();  // x comes from the previous kernel of the step
  pdl_trigger();
  __shared__ uint32_t s_gen;
  __shared__ float red[32];
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int slot = gen & 1u;
  const int r = a.ctx.rank;
  const int64_t row_bytes = static_cast<int64_t>(a.hp) * 16;
  char* dst[N];
  rotate_ptrs<N>(a.slot[slot], r, dst);
  // Phase 1: push this CTA's rows into slot row block [r] of every rank.
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int idx = threadIdx.x + k * blockDim.x;
      if (idx < a.hp) {
        const uint4 v = ld_in(a.x + (row * a.hp + idx) * 16);
        const int64_t off = (static_cast<int64_t>(r) * a.rows + row) * row_bytes + static_cast<int64_t>(idx) * 16;
#pragma unroll
        for (int p = 0; p < N; ++p) st_cg(dst[p] + off, v);
      }
    }
  }
  if (cta_barrier<N>(a.ctx, blockIdx.x, epoch_of(gen, 0))) {
    const char* mine = a.slot[slot][r];
    const int64_t stride = static_cast<int64_t>(a.rows) * row_bytes;
    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x)
      reduce_norm_row<N, PPT>(a, mine + row * row_bytes, stride, row, a.y, a.z, nullptr, nullptr, red);
  }
  finish_generation(a.ctx, gen);
}

// Barrier-free one-shot: partial rows go straight into every rank's current
// Lamport buffer (markers replaced by data); each rank polls its own buffer,
// reduces, normalises and restores the markers (see oneshot_lamport_kernel).
template <int N, int PPT>
__global__ void __launch_bounds__(kMaxRowThreads) ar_rmsnorm_lamport_kernel(NormArgs a) {
  pdl_wait();  // x comes from the previous kernel of the step
  pdl_trigger();
  __shared__ uint32_t s_gen;
  __shared__ float red[32];
  __shared__ int s_fail;
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int r = a.ctx.rank;
  const int64_t row_bytes = static_cast<int64_t>(a.hp) * 16;
  const int64_t buf = static_cast<int64_t>(gen % kLamportBuffers) * N * a.lam_cap;
  char* dst[N];
  rotate_ptrs<N>(a.lam, r, dst);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int idx = threadIdx.x + k * blockDim.x;
      if (idx < a.hp) {
        uint4 v = ld_in(a.x + (row * a.hp + idx) * 16);
        v.x = lamport_clean<__nv_bfloat16>(v.x);
        v.y = lamport_clean<__nv_bfloat16>(v.y);
        v.z = lamport_clean<__nv_bfloat16>(v.z);
        v.w = lamport_clean<__nv_bfloat16>(v.w);
        const int64_t off = buf + static_cast<int64_t>(r) * a.lam_cap + row * row_bytes + static_cast<int64_t>(idx) * 16;
#pragma unroll
        for (int p = 0; p < N; ++p) st_cg(dst[p] + off, v);
      }
    }
  }
  char* mine = a.lam[r] + buf;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  const uint4 marker = make_uint4(kLamportMarker, kLamportMarker, kLamportMarker, kLamportMarker);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    // Wait until every source's packets of this row arrived (bounded). All
    // packets are loaded first, so the common case costs one round trip.
    bool ready[PPT][N];
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int idx = threadIdx.x + k * blockDim.x;
#pragma unroll
      for (int q = 0; q < N; ++q)
        ready[k][q] = idx >= a.hp ||
                      lamport_ready(ld_volatile16(mine + static_cast<int64_t>(q) * a.lam_cap + row * row_bytes +
                                                  static_cast<int64_t>(idx) * 16));
    }
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int idx = threadIdx.x + k * blockDim.x;
#pragma unroll
      for (int q = 0; q < N; ++q) {
        if (ready[k][q]) continue;
        const char* pk = mine + static_cast<int64_t>(q) * a.lam_cap + row * row_bytes + static_cast<int64_t>(idx) * 16;
        const uint64_t start = global_ns();
        uint32_t spins = 0;
        while (!lamport_ready(ld_volatile16(pk))) {
          if ((++spins & 63u) == 0u && global_ns() - start > a.ctx.timeout_ns) {
            report_status(a.ctx.status, kStatusTimeout, r, q, blockIdx.x, gen, 0);
            s_fail = 1;
            break;
          }
        }
      }
    }
    if (__syncthreads_or(s_fail)) break;
    reduce_norm_row<N, PPT>(a, mine + row * row_bytes, a.lam_cap, row, a.y, a.z, nullptr, nullptr, red);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int idx = threadIdx.x + k * blockDim.x;
      if (idx < a.hp)
        for (int q = 0; q < N; ++q)
          st_cg(mine + static_cast<int64_t>(q) * a.lam_cap + row * row_bytes + static_cast<int64_t>(idx) * 16, marker);
    }
  }
  finish_generation(a.ctx, gen);
}

// Cluster form of the Lamport kernel for decode batches. The C CTAs of a
// thread-block cluster share each row: CTA c pushes, polls, reduces and
// normalises packets [c * S, c * S + S) of the row (S = ceil(hp / C)), so
// C SMs move the row instead of one. The row's sum of squares is the sum of
// the C per-CTA partials, read from the other CTAs' shared memory (DSMEM)
// after a cluster barrier. A bounded poll that expires marks the CTA failed;
// the flags are combined through DSMEM too, so every CTA of the cluster leaves
// the row loop at the same point and the cluster barriers stay matched.
template <int N, int PPT>
__global__ void __launch_bounds__(kMaxRowThreads) ar_rmsnorm_lamport_cluster_kernel(NormArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  pdl_wait();  // x comes from the previous kernel of the step
  pdl_trigger();
  __shared__ uint32_t s_gen;
  __shared__ float red[32];
  __shared__ float s_part;  // this CTA's sum of squares of the current row slice
  __shared__ int s_fail;
  const int C = static_cast<int>(cluster.num_blocks());
  const int crank = static_cast<int>(cluster.block_rank());
  const int group = static_cast<int>(blockIdx.x) / C, groups = static_cast<int>(gridDim.x) / C;
  const int slice = (a.hp + C - 1) / C;
  const int p0 = crank * slice;
  const int plen = max(0, min(slice, a.hp - p0));
  const int r = a.ctx.rank;
  const int64_t row_bytes = static_cast<int64_t>(a.hp) * 16;
  // The first row's input, residual and gamma packets are loaded before the
  // generation is read, so their cold loads overlap (a decode step has one row
  // per cluster).
  uint4 x0[PPT], res0[PPT], gam[PPT];
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < plen && group < a.rows) {
      const int64_t idx = p0 + i;
      x0[k] = ld_in(a.x + (static_cast<int64_t>(group) * a.hp + idx) * 16);
      res0[k] = ld_in(a.res + (static_cast<int64_t>(group) * a.hp + idx) * 16);
      gam[k] = ld_in(a.gamma + idx * 16);
    }
  }
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int64_t buf = static_cast<int64_t>(gen % kLamportBuffers) * N * a.lam_cap;
  char* dst[N];
  rotate_ptrs<N>(a.lam, r, dst);
  for (int64_t row = group; row < a.rows; row += groups) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (i < plen) {
        const int64_t idx = p0 + i;
        uint4 v = row == group ? x0[k] : ld_in(a.x + (row * a.hp + idx) * 16);
        v.x = lamport_clean<__nv_bfloat16>(v.x);
        v.y = lamport_clean<__nv_bfloat16>(v.y);
        v.z = lamport_clean<__nv_bfloat16>(v.z);
        v.w = lamport_clean<__nv_bfloat16>(v.w);
        const int64_t off = buf + static_cast<int64_t>(r) * a.lam_cap + row * row_bytes + idx * 16;
#pragma unroll
        for (int p = 0; p < N; ++p) st_cg(dst[p] + off, v);
      }
    }
  }
  char* mine = a.lam[r] + buf;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  const uint4 marker = make_uint4(kLamportMarker, kLamportMarker, kLamportMarker, kLamportMarker);
  for (int64_t row = group; row < a.rows; row += groups) {
    const char* src = mine + row * row_bytes;
    // Bounded wait for every source's packets of this slice. All packets are
    // loaded first, so the common case costs one round trip, and the polled
    // values are the ones summed (no second load).
    // Wide rows (PPT > 1) keep only the first packet's sources in registers
    // and load the others again for the sum.
    uint4 pv[1][N];
    bool ready[PPT][N];
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
#pragma unroll
      for (int q = 0; q < N; ++q) {
        uint4 t = make_uint4(0u, 0u, 0u, 0u);
        if (i < plen) t = ld_volatile16(src + static_cast<int64_t>(q) * a.lam_cap + static_cast<int64_t>(p0 + i) * 16);
        ready[k][q] = i >= plen || lamport_ready(t);
        if (k == 0) pv[0][q] = t;
      }
    }
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (i >= plen) continue;
#pragma unroll
      for (int q = 0; q < N; ++q) {
        if (ready[k][q]) continue;
        const char* pk = src + static_cast<int64_t>(q) * a.lam_cap + static_cast<int64_t>(p0 + i) * 16;
        const uint64_t start = global_ns();
        uint32_t spins = 0;
        uint4 t;
        while (!lamport_ready(t = ld_volatile16(pk))) {
          if ((++spins & 63u) == 0u && global_ns() - start > a.ctx.timeout_ns) {
            report_status(a.ctx.status, kStatusTimeout, r, q, blockIdx.x, gen, 0);
            s_fail = 1;
            break;
          }
        }
        if (k == 0) pv[0][q] = t;
      }
    }
    const int failed = __syncthreads_or(s_fail);
    // Sum the sources, add the residual, keep z (rounded) in registers.
    float zf[PPT][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (failed || i >= plen) continue;
      const int64_t idx = p0 + i;
      uint4 v[N];
#pragma unroll
      for (int q = 0; q < N; ++q)
        v[q] = k == 0 ? pv[0][q] : ld_cg(src + static_cast<int64_t>(q) * a.lam_cap + idx * 16);
      float acc[8];
      unpack_set<__nv_bfloat16>(v[0], acc);
#pragma unroll
      for (int q = 1; q < N; ++q) unpack_add<__nv_bfloat16>(v[q], acc);
      unpack_add<__nv_bfloat16>(row == group ? res0[k] : ld_in(a.res + (row * a.hp + idx) * 16), acc);
      const uint4 zp = pack<__nv_bfloat16>(acc);
      st_out(a.z + (row * a.hp + idx) * 16, zp);
      unpack_set<__nv_bfloat16>(zp, zf[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += zf[k][e] * zf[k][e];
    }
    const float part = block_sum(ss, red);
    if (threadIdx.x == 0) {
      s_part = part;
      s_fail = failed;
    }
    cluster.sync();
    float tot = 0.f;
    int any_fail = 0;
    for (int c = 0; c < C; ++c) {
      tot += *cluster.map_shared_rank(&s_part, c);
      any_fail |= *cluster.map_shared_rank(&s_fail, c);
    }
    if (any_fail) {
      cluster.sync();  // peers may still read this CTA's flags
      break;
    }
    const float inv = rsqrtf(tot * a.inv_h + a.eps);
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (i >= plen) continue;
      const int64_t idx = p0 + i;
      float g[8];
      unpack_set<__nv_bfloat16>(gam[k], g);
#pragma unroll
      for (int e = 0; e < 8; ++e) zf[k][e] = zf[k][e] * inv * g[e];
      st_out(a.y + (row * a.hp + idx) * 16, pack<__nv_bfloat16>(zf[k]));
      for (int q = 0; q < N; ++q)
        st_cg(mine + static_cast<int64_t>(q) * a.lam_cap + row * row_bytes + idx * 16, marker);
    }
    cluster.sync();  // s_part and s_fail are rewritten for the next row
  }
  finish_generation(a.ctx, gen);
}

// Two-shot. Part p = rows [part_begin(T, N, p), part_begin(T, N, p + 1)); with
// prow = ceil(T / N) rows per part, every slot holds
//   inbox  [N][prow] rows : rank q's partial rows of this rank's part
//   outbox [2][prow] rows : finished y rows, then z rows of this rank's part
template <int N, int PPT>
__global__ void __launch_bounds__(kMaxRowThreads) ar_rmsnorm_twoshot_kernel(NormArgs a) {
  pdl_wait();  // x comes from the previous kernel of the step
  pdl_trigger();
  __shared__ uint32_t s_gen;
  __shared__ float red[32];
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int slot = gen & 1u;
  const int r = a.ctx.rank;
  const int64_t row_bytes = static_cast<int64_t>(a.hp) * 16;
  const int prow = (a.rows + N - 1) / N;
  char* peer[N];
  rotate_ptrs<N>(a.slot[slot], r, peer);

  // Phase 1: scatter partial rows of part p (k-th peer) to p's inbox row block r.
#pragma unroll 1
  for (int k = 0; k < N; ++k) {
    const int p = (r + k) % N;
    const int b = static_cast<int>(part_begin(a.rows, N, p));
    const int e = static_cast<int>(part_begin(a.rows, N, p + 1));
    for (int row = b + blockIdx.x; row < e; row += gridDim.x) {
      char* dst = peer[k] + (static_cast<int64_t>(r) * prow + (row - b)) * row_bytes;
#pragma unroll
      for (int kk = 0; kk < PPT; ++kk) {
        const int idx = threadIdx.x + kk * blockDim.x;
        if (idx < a.hp) st_cg(dst + static_cast<int64_t>(idx) * 16, ld_in(a.x + (row * static_cast<int64_t>(a.hp) + idx) * 16));
      }
    }
  }
  bool ok = cta_barrier<N>(a.ctx, blockIdx.x, epoch_of(gen, 0));

  // Phase 2: reduce + residual + norm of own part; results to outputs and outbox.
  const int64_t outbox = static_cast<int64_t>(N) * prow * row_bytes;
  if (ok) {
    char* mine = peer[0];
    const int b = static_cast<int>(part_begin(a.rows, N, r));
    const int e = static_cast<int>(part_begin(a.rows, N, r + 1));
    for (int row = b + blockIdx.x; row < e; row += gridDim.x) {
      const int64_t lr = row - b;
      reduce_norm_row<N, PPT>(a, mine + lr * row_bytes, static_cast<int64_t>(prow) * row_bytes, row, a.y, a.z,
                              mine + outbox + lr * row_bytes, mine + outbox + (prow + lr) * row_bytes, red);
    }
  }
  ok = cta_barrier<N>(a.ctx, blockIdx.x, epoch_of(gen, 1)) && ok;

  // Phase 3: pull finished rows of the other parts.
  if (ok) {
#pragma unroll 1
    for (int k = 1; k < N; ++k) {
      const int p = (r + k) % N;
      const int b = static_cast<int>(part_begin(a.rows, N, p));
      const int e = static_cast<int>(part_begin(a.rows, N, p + 1));
      for (int row = b + blockIdx.x; row < e; row += gridDim.x) {
        const char* ysrc = peer[k] + outbox + static_cast<int64_t>(row - b) * row_bytes;
        const char* zsrc = peer[k] + outbox + static_cast<int64_t>(prow + row - b) * row_bytes;
#pragma unroll
        for (int kk = 0; kk < PPT; ++kk) {
          const int idx = threadIdx.x + kk * blockDim.x;
          if (idx < a.hp) {
            const uint4 yv = ld_cg(ysrc + static_cast<int64_t>(idx) * 16);
            const uint4 zv = ld_cg(zsrc + static_cast<int64_t>(idx) * 16);
            st_out(a.y + (row * static_cast<int64_t>(a.hp) + idx) * 16, yv);
            st_out(a.z + (row * static_cast<int64_t>(a.hp) + idx) * 16, zv);
          }
        }
      }
    }
  }
  finish_generation(a.ctx, gen);
}

// kind: 0 one-shot push, 1 two-shot, 2 Lamport.
template <int N, int PPT>
void launch_n(int kind, int ctas, int threads, const NormArgs& a, cudaStream_t s) {
  if (kind == 1)
    launch_pdl(ar_rmsnorm_twoshot_kernel<N, PPT>, dim3(ctas), dim3(threads), 0, s, 1, a);
  else if (kind == 2)
    launch_pdl(ar_rmsnorm_lamport_kernel<N, PPT>, dim3(ctas), dim3(threads), 0, s, 1, a);
  else
    launch_pdl(ar_rmsnorm_oneshot_kernel<N, PPT>, dim3(ctas), dim3(threads), 0, s, 1, a);
}

template <int PPT>
void launch_ppt(int world, int kind, int ctas, int threads, const NormArgs& a, cudaStream_t s) {
  switch (world) {
    case 1: launch_n<1, PPT>(kind, ctas, threads, a, s); break;
    case 2: launch_n<2, PPT>(kind, ctas, threads, a, s); break;
    case 3: launch_n<3, PPT>(kind, ctas, threads, a, s); break;
    case 4: launch_n<4, PPT>(kind, ctas, threads, a, s); break;
    case 5: launch_n<5, PPT>(kind, ctas, threads, a, s); break;
    case 6: launch_n<6, PPT>(kind, ctas, threads, a, s); break;
    case 7: launch_n<7, PPT>(kind, ctas, threads, a, s); break;
    case 8: launch_n<8, PPT>(kind, ctas, threads, a, s); break;
    default: throw std::invalid_argument("unsupported world size");
  }
}

// Cluster launch of the Lamport kernel: `groups` clusters of C CTAs, a row
// per cluster at a time.
template <int N, int PPT>
void launch_cluster_n(int C, int groups, int threads, const NormArgs& a, cudaStream_t s) {
  launch_pdl(ar_rmsnorm_lamport_cluster_kernel<N, PPT>, dim3(static_cast<unsigned>(C * groups)),
             dim3(static_cast<unsigned>(threads)), 0, s, C, a);
}

template <int PPT>
void launch_cluster_ppt(int world, int C, int groups, int threads, const NormArgs& a, cudaStream_t s) {
  switch (world) {
    case 2: launch_cluster_n<2, PPT>(C, groups, threads, a, s); break;
    case 3: launch_cluster_n<3, PPT>(C, groups, threads, a, s); break;
    case 4: launch_cluster_n<4, PPT>(C, groups, threads, a, s); break;
    case 5: launch_cluster_n<5, PPT>(C, groups, threads, a, s); break;
    case 6: launch_cluster_n<6, PPT>(C, groups, threads, a, s); break;
    case 7: launch_cluster_n<7, PPT>(C, groups, threads, a, s); break;
    case 8: launch_cluster_n<8, PPT>(C, groups, threads, a, s); break;
    default: throw std::invalid_argument("the Lamport variant needs 2 to 8 ranks");
  }
}

// Rows up to which the Lamport variant runs in cluster form, and the cluster
// size (portable maximum 8; at least 32 packets per CTA).
constexpr int64_t kClusterMaxRows = 64;
int cluster_size(int hp) {
  int c = 8;
  while (c > 1 && hp / c < 32) c >>= 1;
  return c;
}

}  // namespace

int64_t ar_rmsnorm_slot_bytes(int variant, int64_t rows, int64_t hidden, int world) {
  const int64_t row_bytes = hidden * 2;
  if (variant == kOneshotPush) return world * rows * row_bytes;
  const int64_t prow = (rows + world - 1) / world;
  return (world + 2) * prow * row_bytes;
}

int ar_rmsnorm(Communicator& comm, cudaStream_t stream, const void* x, const void* residual, const void* gamma,
               void* y, void* residual_out, int64_t rows, int64_t hidden, float eps, int variant, int ctas) {
  TraceRange trace("b200ar.ar_rmsnorm");
  comm.check_status();
  B200AR_CHECK(hidden % 8 == 0 && hidden / 8 <= 4 * kMaxRowThreads,
               "hidden size must be a multiple of 8 and at most " << 32 * kMaxRowThreads);
  B200AR_CHECK(rows >= 1 && rows < (1 << 30), "bad row count " << rows);
  for (const void* p : {x, residual, gamma, static_cast<const void*>(y), static_cast<const void*>(residual_out)})
    B200AR_CHECK(reinterpret_cast<uintptr_t>(p) % 16 == 0, "fused all-reduce + RMSNorm needs 16-byte aligned tensors");
  const int world = comm.world();
  const int64_t bytes = rows * hidden * 2;
  if (variant == kAuto) {
    // Lamport (no barrier) while the rows fit its buffers; then one-shot push
    // for small messages; two-shot once the message is bandwidth bound.
    if (world > 1 && comm.lamport_capacity() >= bytes)
      variant = kLamport;
    else
      variant = (world <= 2 || bytes <= (512 << 10) || rows < 2 * world) ? kOneshotPush : kTwoshot;
  }
  B200AR_CHECK(variant == kOneshotPush || variant == kTwoshot || variant == kLamport,
               "fused RMSNorm supports oneshot_push, twoshot and lamport");
  if (world == 1) variant = kOneshotPush;
  if (variant == kLamport && comm.lamport_capacity() < bytes) variant = kOneshotPush;
  B200AR_CHECK(comm.slots_registered(), "communicator has no slot buffers");
  if (variant != kLamport) {
    const int64_t need = ar_rmsnorm_slot_bytes(variant, rows, hidden, world);
    if (need > comm.slot_capacity()) {
      const int other = variant == kTwoshot ? kOneshotPush : kTwoshot;
      B200AR_CHECK(ar_rmsnorm_slot_bytes(other, rows, hidden, world) <= comm.slot_capacity(),
                   "fused all-reduce + RMSNorm of " << rows << "x" << hidden << " needs " << need
                                                    << " slot bytes, capacity is " << comm.slot_capacity());
      variant = other;
    }
  }

  NormArgs a{};
  comm.fill_ctx(&a.ctx);
  for (int s = 0; s < 2; ++s)
    for (int i = 0; i < world; ++i) a.slot[s][i] = comm.slot_ptr(s, i);
  a.x = static_cast<const char*>(x);
  a.res = static_cast<const char*>(residual);
  a.gamma = static_cast<const char*>(gamma);
  a.y = static_cast<char*>(y);
  a.z = static_cast<char*>(residual_out);
  a.rows = static_cast<int>(rows);
  a.hp = static_cast<int>(hidden / 8);
  a.eps = eps;
  a.inv_h = 1.0f / static_cast<float>(hidden);
  for (int i = 0; i < world; ++i) a.lam[i] = comm.lamport_ptr(i);
  a.lam_cap = comm.lamport_capacity();
  if (variant == kLamport && ctas == 0 && rows <= kClusterMaxRows && cluster_size(a.hp) > 1) {
    const int C = cluster_size(a.hp);
    const int slice = (a.hp + C - 1) / C;
    const int cppt = slice <= kMaxRowThreads ? 1 : (slice <= 2 * kMaxRowThreads ? 2 : 4);
    const int cthreads = std::max(32, ((slice + cppt - 1) / cppt + 31) / 32 * 32);
    const int groups = static_cast<int>(std::min<int64_t>(rows, kMaxCTAs / C));
    switch (cppt) {
      case 1: launch_cluster_ppt<1>(world, C, groups, cthreads, a, stream); break;
      case 2: launch_cluster_ppt<2>(world, C, groups, cthreads, a, stream); break;
      default: launch_cluster_ppt<4>(world, C, groups, cthreads, a, stream); break;
    }
    comm.count_launch();
    return variant;
  }
  const int ppt = a.hp <= kMaxRowThreads ? 1 : (a.hp <= 2 * kMaxRowThreads ? 2 : 4);
  const int threads = std::max(32, ((a.hp + ppt - 1) / ppt + 31) / 32 * 32);
  const bool two = variant == kTwoshot;
  const int kind = two ? 1 : (variant == kLamport ? 2 : 0);
  const int64_t work_rows = two ? (rows + world - 1) / world : rows;
  int grid = ctas > 0 ? ctas : static_cast<int>(std::min<int64_t>(work_rows, 148));
  grid = std::max(1, std::min(grid, kMaxCTAs));
  switch (ppt) {
    case 1: launch_ppt<1>(world, kind, grid, threads, a, stream); break;
    case 2: launch_ppt<2>(world, kind, grid, threads, a, stream); break;
    default: launch_ppt<4>(world, kind, grid, threads, a, stream); break;
  }
  B200AR_CUDA(cudaGetLastError());
  comm.count_launch();
  return variant;
}

}  // namespace b200ar

// ---------------------------------------------------------------------------
// Allocation-free entry point (declared in noalloc.h). It runs the one-shot
// kernel above with world size 1; the signal block and both staging slots
// live in a file-scope device array instead of memory the caller allocates.
// ---------------------------------------------------------------------------

#include <mutex>
#include <string>

#include "noalloc.h"

namespace {

constexpr int64_t kNoallocSlot = B200AR_NOALLOC_MAX_BYTES;
constexpr int64_t kNoallocScratch = sizeof(b200ar::Signal) + 2 * kNoallocSlot;
constexpr int kNoallocMaxDevices = 64;

// Scratch for every GPU that loads this library: [Signal][slot 0][slot 1].
// In host code this name is only a stand-in for the symbol; the device address
// comes from cudaGetSymbolAddress.
static __device__ __align__(256) char g_noalloc_scratch[kNoallocScratch];

std::mutex g_noalloc_mu;
char* g_noalloc_ptr[kNoallocMaxDevices] = {};
thread_local std::string g_noalloc_err;

int noalloc_fail(int code, const std::string& msg) {
  g_noalloc_err = msg;
  return code;
}

// Once per device, with that device current: device address of the scratch
// array and a cleared signal block.
int noalloc_setup(int dev, char** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return noalloc_fail(3, std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    e = cudaMemset(p, 0, sizeof(b200ar::Signal));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return noalloc_fail(3, std::string("clearing the scratch signal block failed: ") +
                                                     cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<char*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int b200ar_residual_rmsnorm_noalloc(const void* x, const void* residual, const void* gamma, void* y,
                                               void* residual_out, int64_t rows, int64_t hidden, float eps,
                                               cudaStream_t stream) {
  using namespace b200ar;
  if (rows < 1 || hidden < 8 || hidden % 8 != 0 || hidden > 16384)
    return noalloc_fail(1, "hidden must be a multiple of 8 in [8, 16384] and rows >= 1");
  // Divide before multiplying: a huge `rows` must not wrap around and pass.
  if (rows > kNoallocSlot / (hidden * 2))
    return noalloc_fail(1, "rows * hidden * 2 (rows = " + std::to_string(rows) + ", hidden = " +
                               std::to_string(hidden) + ") exceeds the allocation-free limit of " +
                               std::to_string(kNoallocSlot) + " bytes");
  for (const void* p : {x, residual, gamma, static_cast<const void*>(y), static_cast<const void*>(residual_out)})
    if (p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 != 0)
      return noalloc_fail(1, "all tensors must be non-null and 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kNoallocMaxDevices) return noalloc_fail(3, "no usable current device");
  char* base = nullptr;
  if (int rc = noalloc_setup(dev, &base)) return rc;

  NormArgs a{};
  a.ctx.self = reinterpret_cast<Signal*>(base);
  a.ctx.peers[0] = a.ctx.self;
  a.ctx.status = nullptr;  // one rank: the barrier never waits on another GPU
  a.ctx.timeout_ns = 1000000000ull;
  a.ctx.rank = 0;
  a.ctx.world = 1;
  a.slot[0][0] = base + sizeof(Signal);
  a.slot[1][0] = base + sizeof(Signal) + kNoallocSlot;
  a.x = static_cast<const char*>(x);
  a.res = static_cast<const char*>(residual);
  a.gamma = static_cast<const char*>(gamma);
  a.y = static_cast<char*>(y);
  a.z = static_cast<char*>(residual_out);
  a.rows = static_cast<int>(rows);
  a.hp = static_cast<int>(hidden / 8);
  a.eps = eps;
  a.inv_h = 1.0f / static_cast<float>(hidden);
  const int ppt = a.hp <= kMaxRowThreads ? 1 : (a.hp <= 2 * kMaxRowThreads ? 2 : 4);
  const int threads = std::max(32, ((a.hp + ppt - 1) / ppt + 31) / 32 * 32);
  const int grid = static_cast<int>(std::min<int64_t>(rows, 148));
  try {
    switch (ppt) {
      case 1: launch_ppt<1>(1, 0, grid, threads, a, stream); break;
      case 2: launch_ppt<2>(1, 0, grid, threads, a, stream); break;
      default: launch_ppt<4>(1, 0, grid, threads, a, stream); break;
    }
  } catch (const std::exception& ex) {
    return noalloc_fail(2, ex.what());
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return noalloc_fail(2, std::string("launch failed: ") + cudaGetErrorString(e));
  return 0;
}

extern "C" const char* b200ar_noalloc_last_error(void) { return g_noalloc_err.c_str(); }

extern "C" int64_t b200ar_noalloc_scratch_bytes(void) { return kNoallocScratch; }
