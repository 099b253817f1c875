// Host side of the tcgen05 GEMM: tensor maps, launch, error reporting.
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "../common/check.h"
#include "../common/trace.h"
#include "gemm.cuh"
#include "gemm2sm.cuh"
#include "gemm_api.h"

namespace b200ar {

namespace {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    B200AR_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p) throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<EncodeFn>(p);
  }();
  return fn;
}

int sm_count(int dev) {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  B200AR_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  cache[dev] = n;
  return n;
}

}  // namespace

CUtensorMap make_tmap_bf16_2d(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols) {
  B200AR_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  B200AR_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return m;
}

gemm::Shape gemm_shape(int64_t M, int64_t N, int64_t K) {
  B200AR_CHECK(M > 0 && N > 0 && K > 0 && M < (1 << 30) && N < (1 << 30) && K < (1 << 30), "bad GEMM shape");
  B200AR_CHECK(K % 8 == 0, "K must be a multiple of 8 (16-byte rows for TMA)");
  gemm::Shape s;
  s.M = static_cast<int>(M);
  s.N = static_cast<int>(N);
  s.K = static_cast<int>(K);
  s.tiles_m = static_cast<int>((M + gemm::BM - 1) / gemm::BM);
  s.tiles_n = static_cast<int>((N + gemm::BN - 1) / gemm::BN);
  s.kblocks = static_cast<int>((K + gemm::BK - 1) / gemm::BK);
  return s;
}

int gemm_grid(const gemm::Shape& s, int max_ctas) {
  int dev = 0;
  B200AR_CUDA(cudaGetDevice(&dev));
  int g = std::min(s.tiles_m * s.tiles_n, sm_count(dev));
  if (max_ctas > 0) g = std::min(g, max_ctas);
  return std::max(g, 1);
}

void gemm_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int* err, cudaStream_t stream,
               int max_ctas) {
  const TraceRange trace("b200ar::gemm_bf16");
  const gemm::Shape s = gemm_shape(M, N, K);
  B200AR_CHECK(N % 8 == 0 && reinterpret_cast<uintptr_t>(C) % 16 == 0, "C must have 16-byte aligned rows");
  const gemm::TmapA ta{make_tmap_bf16_2d(A, M, K, K, gemm::BM, gemm::BK)};
  const CUtensorMap tb = make_tmap_bf16_2d(B, N, K, K, gemm::BN, gemm::BK);
  gemm::StoreC epi{static_cast<__nv_bfloat16*>(C), N};
  auto kern = gemm::gemm_kernel<gemm::StoreC>;
  static PerDeviceOnce smem_attr;
  smem_attr([&] {
    B200AR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(gemm::smem_bytes<gemm::StoreC>())));
  });
  kern<<<gemm_grid(s, max_ctas), gemm::THREADS, gemm::smem_bytes<gemm::StoreC>(), stream>>>(ta, tb, s, epi, err);
  B200AR_CUDA(cudaGetLastError());
}

void gemm_bf16_2sm(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int* err,
                   cudaStream_t stream, int max_pairs) {
  const TraceRange trace("b200ar::gemm_bf16_2sm");
  B200AR_CHECK(M > 0 && N > 0 && K > 0 && M < (1 << 30) && N < (1 << 30) && K < (1 << 30), "bad GEMM shape");
  B200AR_CHECK(K % 8 == 0, "K must be a multiple of 8 (16-byte rows for TMA)");
  B200AR_CHECK(N % 8 == 0 && reinterpret_cast<uintptr_t>(C) % 16 == 0, "C must have 16-byte aligned rows");
  gemm2::Shape s{};
  s.M = static_cast<int>(M);
  s.N = static_cast<int>(N);
  s.K = static_cast<int>(K);
  s.tiles_m = static_cast<int>((M + gemm2::BM - 1) / gemm2::BM);
  s.tiles_n = static_cast<int>((N + gemm2::BN - 1) / gemm2::BN);
  s.kblocks = static_cast<int>((K + gemm2::BK - 1) / gemm2::BK);
  const CUtensorMap ta = make_tmap_bf16_2d(A, M, K, K, 128, gemm2::BK);
  const CUtensorMap tb = make_tmap_bf16_2d(B, N, K, K, 128, gemm2::BK);
  static PerDeviceOnce smem_attr;
  smem_attr([&] {
    B200AR_CUDA(cudaFuncSetAttribute(gemm2::gemm2sm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(gemm2::SMEM_BYTES)));
  });
  int dev = 0;
  B200AR_CUDA(cudaGetDevice(&dev));
  int pairs = std::min(s.tiles_m * s.tiles_n, sm_count(dev) / 2);
  if (max_pairs > 0) pairs = std::min(pairs, max_pairs);
  pairs = std::max(pairs, 1);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.blockDim = dim3(gemm2::THREADS, 1, 1);
  cfg.dynamicSmemBytes = gemm2::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  __nv_bfloat16* c = static_cast<__nv_bfloat16*>(C);
  B200AR_CUDA(cudaLaunchKernelEx(&cfg, gemm2::gemm2sm_kernel, ta, tb, s, c, static_cast<int64_t>(N), err));
}

}  // namespace b200ar
