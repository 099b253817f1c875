// Instantiation and dispatch of the all-reduce kernels (ar_kernels.cuh) over
// dtype {fp32, fp16, bf16} x world size {2..8} x variant. The reference
// instantiated world sizes {2, 4, 6, 8} only (pcie_allreduce.cu:427-433);
// NVSwitch gives every rank count the same topology, so odd sizes are served too.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "../common/check.h"
#include "ar_kernels.cuh"

namespace b200ar {

namespace {

template <typename T, int N>
void launch_typed(int variant, int ctas, int threads, const ArArgs& a, cudaStream_t s) {
  switch (variant) {
    case kOneshotPush: oneshot_push_kernel<T, N><<<ctas, threads, 0, s>>>(a); break;
    case kOneshotPull: oneshot_pull_kernel<T, N><<<ctas, threads, 0, s>>>(a); break;
    case kTwoshot: twoshot_kernel<T, N><<<ctas, threads, 0, s>>>(a); break;
    case kTwoshotPush: twoshot_push_kernel<T, N><<<ctas, threads, 0, s>>>(a); break;
    case kRegistered: registered_kernel<T, N><<<ctas, threads, 0, s>>>(a); break;
    case kLamport: oneshot_lamport_kernel<T, N><<<ctas, threads, 0, s>>>(a); break;
    default: throw std::invalid_argument("unknown all-reduce variant " + std::to_string(variant));
  }
}

template <typename T>
void launch_world(int variant, int world, int ctas, int threads, const ArArgs& a, cudaStream_t s) {
  switch (world) {
    case 2: launch_typed<T, 2>(variant, ctas, threads, a, s); break;
    case 3: launch_typed<T, 3>(variant, ctas, threads, a, s); break;
    case 4: launch_typed<T, 4>(variant, ctas, threads, a, s); break;
    case 5: launch_typed<T, 5>(variant, ctas, threads, a, s); break;
    case 6: launch_typed<T, 6>(variant, ctas, threads, a, s); break;
    case 7: launch_typed<T, 7>(variant, ctas, threads, a, s); break;
    case 8: launch_typed<T, 8>(variant, ctas, threads, a, s); break;
    default: throw std::invalid_argument("unsupported world size " + std::to_string(world));
  }
}

// World size 1: the sum over one rank is the input itself (16-byte copy).
__global__ void __launch_bounds__(kArThreads) copy_kernel(const char* __restrict__ in, char* __restrict__ out,
                                                          int64_t packets) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < packets;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    st_out(out + i * 16, ld_in(in + i * 16));
}

}  // namespace

__global__ void fill_u32_kernel(uint32_t* p, int64_t words, uint32_t value) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < words;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = value;
}

void launch_lamport_init(void* p, int64_t bytes, cudaStream_t stream) {
  if (bytes <= 0) return;
  fill_u32_kernel<<<256, 256, 0, stream>>>(static_cast<uint32_t*>(p), bytes / 4, kLamportMarker);
  B200AR_CUDA(cudaGetLastError());
}

void launch_copy(const void* in, void* out, int64_t packets, cudaStream_t stream) {
  const int64_t want = std::max<int64_t>((packets + kArThreads - 1) / kArThreads, 1);
  const int ctas = static_cast<int>(std::min<int64_t>(want, 4 * 148));
  copy_kernel<<<ctas, kArThreads, 0, stream>>>(static_cast<const char*>(in), static_cast<char*>(out), packets);
  B200AR_CUDA(cudaGetLastError());
}

namespace {
template <typename T, int N>
const void* kernel_of(int variant) {
  switch (variant) {
    case kOneshotPush: return reinterpret_cast<const void*>(&oneshot_push_kernel<T, N>);
    case kOneshotPull: return reinterpret_cast<const void*>(&oneshot_pull_kernel<T, N>);
    case kTwoshot: return reinterpret_cast<const void*>(&twoshot_kernel<T, N>);
    case kTwoshotPush: return reinterpret_cast<const void*>(&twoshot_push_kernel<T, N>);
    case kRegistered: return reinterpret_cast<const void*>(&registered_kernel<T, N>);
    case kLamport: return reinterpret_cast<const void*>(&oneshot_lamport_kernel<T, N>);
    default: return nullptr;
  }
}

template <typename T>
const void* kernel_of_world(int variant, int world) {
  switch (world) {
    case 2: return kernel_of<T, 2>(variant);
    case 3: return kernel_of<T, 3>(variant);
    case 4: return kernel_of<T, 4>(variant);
    case 5: return kernel_of<T, 5>(variant);
    case 6: return kernel_of<T, 6>(variant);
    case 7: return kernel_of<T, 7>(variant);
    case 8: return kernel_of<T, 8>(variant);
    default: return nullptr;
  }
}
}  // namespace

int ar_blocks_per_sm(int variant, DType dt, int world) {
  const void* k = nullptr;
  switch (dt) {
    case DType::kFloat32: k = kernel_of_world<float>(variant, world); break;
    case DType::kFloat16: k = kernel_of_world<__half>(variant, world); break;
    case DType::kBFloat16: k = kernel_of_world<__nv_bfloat16>(variant, world); break;
  }
  if (k == nullptr) return kMaxCTAs;  // no barrier kernel: no limit from this module
  int n = 0;
  B200AR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kArThreads, 0));
  return n;
}

void launch_ar_kernel(int variant, DType dt, int world, int ctas, int threads, const ArArgs& a,
                      cudaStream_t stream) {
  if (ctas < 1 || ctas > kMaxCTAs) throw std::invalid_argument("bad CTA count " + std::to_string(ctas));
  if (threads < 32 || threads > kArThreads || threads % 32 != 0)
    throw std::invalid_argument("bad thread count " + std::to_string(threads));
  switch (dt) {
    case DType::kFloat32: launch_world<float>(variant, world, ctas, threads, a, stream); break;
    case DType::kFloat16: launch_world<__half>(variant, world, ctas, threads, a, stream); break;
    case DType::kBFloat16: launch_world<__nv_bfloat16>(variant, world, ctas, threads, a, stream); break;
    default: throw std::invalid_argument("only float32, float16 and bfloat16 are supported");
  }
  B200AR_CUDA(cudaGetLastError());
}

}  // namespace b200ar
