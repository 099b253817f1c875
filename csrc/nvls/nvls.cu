// NVLS multicast buffer management and the NVLS all-reduce kernel (see nvls.h).
#include <cuda.h>
#include <unistd.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "../comm/ar_kernels.cuh"
#include "../comm/communicator.h"
#include "nvls.h"

namespace b200ar {

namespace {

// Driver entry points through the runtime (no link-time dependency on libcuda).
template <typename F>
F drv(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  B200AR_CUDA(cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q));
  if (q != cudaDriverEntryPointSuccess || p == nullptr)
    throw std::runtime_error(std::string("driver entry point not available: ") + name);
  return reinterpret_cast<F>(p);
}

void cu_check(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) throw std::runtime_error(std::string(what) + " failed with CUresult " + std::to_string(r));
}

#define CU(fn, ...) cu_check(drv<decltype(&fn)>(#fn)(__VA_ARGS__), #fn)

CUmemAllocationProp phys_prop(int device) {
  CUmemAllocationProp p{};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

CUmulticastObjectProp mc_prop(int world, size_t bytes) {
  CUmulticastObjectProp p{};
  p.numDevices = static_cast<unsigned>(world);
  p.size = bytes;
  p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

size_t round_up(size_t v, size_t g) { return (v + g - 1) / g * g; }

// ------------------------------------------------------------------ kernel

struct NvlsArgs {
  CommCtx ctx;
  char* uc;        // this rank's unicast view of the multicast-bound buffer
  char* mc;        // multicast address of the same buffer
  const char* in;
  char* out;
  int64_t packets;
};

template <typename T>
__device__ __forceinline__ uint4 mm_ld_reduce(const char* addr);

template <>
__device__ __forceinline__ uint4 mm_ld_reduce<__nv_bfloat16>(const char* addr) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(addr)
               : "memory");
  return v;
}
template <>
__device__ __forceinline__ uint4 mm_ld_reduce<__half>(const char* addr) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(addr)
               : "memory");
  return v;
}
template <>
__device__ __forceinline__ uint4 mm_ld_reduce<float>(const char* addr) {
  float a, b, c, d;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(a), "=f"(b), "=f"(c), "=f"(d)
               : "l"(addr)
               : "memory");
  return make_uint4(__float_as_uint(a), __float_as_uint(b), __float_as_uint(c), __float_as_uint(d));
}

__device__ __forceinline__ void mm_st(char* addr, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr),
               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
               "f"(__uint_as_float(v.w))
               : "memory");
}

// CTA j handles sub-range j of every rank's part (as in the two-shot kernel),
// so per-CTA barriers order exactly the data each CTA touches:
//   1. copy own input (sub-range j of every part) into the multicast-bound buffer
//   2. barrier; reduce own part's sub-range through the switch, multicast the sum
//   3. barrier; copy the finished sums (sub-range j of every part) to the output
template <typename T, int N>
__global__ void __launch_bounds__(kArThreads) nvls_kernel(NvlsArgs a) {
  __shared__ uint32_t s_gen;
  const uint32_t gen = read_generation(a.ctx, &s_gen);
  const int r = a.ctx.rank;
  const int64_t P = a.packets;
  const int G = gridDim.x, j = blockIdx.x;
  auto range = [&](int p, int64_t* b, int64_t* e) {
    const int64_t pb = part_begin(P, N, p);
    const int64_t len = part_begin(P, N, p + 1) - pb;
    *b = pb + part_begin(len, G, j);
    *e = pb + part_begin(len, G, j + 1);
  };
  // U packets in flight per thread in every phase (the switch round trip of
  // multimem.ld_reduce is long; one outstanding request per thread starves it).
  constexpr int U = 4;
  const int64_t step = static_cast<int64_t>(U) * blockDim.x;
  int64_t b, e;
#pragma unroll 1
  for (int p = 0; p < N; ++p) {
    range(p, &b, &e);
    for (int64_t i0 = b + threadIdx.x; i0 < e; i0 += step) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i0 + u * blockDim.x < e) v[u] = ld_in(a.in + (i0 + u * blockDim.x) * 16);
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i0 + u * blockDim.x < e) st_cg(a.uc + (i0 + u * blockDim.x) * 16, v[u]);
    }
  }
  bool ok = cta_barrier<N>(a.ctx, j, epoch_of(gen, 0));
  if (ok) {
    range(r, &b, &e);
    for (int64_t i0 = b + threadIdx.x; i0 < e; i0 += step) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i0 + u * blockDim.x < e) v[u] = mm_ld_reduce<T>(a.mc + (i0 + u * blockDim.x) * 16);
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i0 + u * blockDim.x < e) mm_st(a.mc + (i0 + u * blockDim.x) * 16, v[u]);
    }
    __threadfence_system();
  }
  ok = cta_barrier<N>(a.ctx, j, epoch_of(gen, 1)) && ok;
  if (ok) {
#pragma unroll 1
    for (int p = 0; p < N; ++p) {
      range(p, &b, &e);
      for (int64_t i0 = b + threadIdx.x; i0 < e; i0 += step) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (i0 + u * blockDim.x < e) v[u] = ld_cg(a.uc + (i0 + u * blockDim.x) * 16);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (i0 + u * blockDim.x < e) st_out(a.out + (i0 + u * blockDim.x) * 16, v[u]);
      }
    }
  }
  finish_generation(a.ctx, gen);
}

template <typename T>
void launch_t(int world, int ctas, const NvlsArgs& a, cudaStream_t s) {
  switch (world) {
    case 2: nvls_kernel<T, 2><<<ctas, kArThreads, 0, s>>>(a); break;
    case 3: nvls_kernel<T, 3><<<ctas, kArThreads, 0, s>>>(a); break;
    case 4: nvls_kernel<T, 4><<<ctas, kArThreads, 0, s>>>(a); break;
    case 5: nvls_kernel<T, 5><<<ctas, kArThreads, 0, s>>>(a); break;
    case 6: nvls_kernel<T, 6><<<ctas, kArThreads, 0, s>>>(a); break;
    case 7: nvls_kernel<T, 7><<<ctas, kArThreads, 0, s>>>(a); break;
    case 8: nvls_kernel<T, 8><<<ctas, kArThreads, 0, s>>>(a); break;
    default: throw std::invalid_argument("NVLS needs 2..8 ranks");
  }
}

}  // namespace

// ------------------------------------------------------------------ buffer

bool NvlsBuffer::supported(int device) {
  int v = 0;
  CUdevice d;
  try {
    CU(cuDeviceGet, &d, device);
    CU(cuDeviceGetAttribute, &v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, d);
  } catch (const std::exception&) {
    return false;
  }
  return v != 0;
}

NvlsBuffer::NvlsBuffer(int device, int world, int64_t bytes) : device_(device), world_(world) {
  B200AR_CHECK(world >= 2 && world <= kMaxRanks, "NVLS needs 2..8 ranks");
  size_t mc_gran = 0, mem_gran = 0;
  CUmulticastObjectProp mp = mc_prop(world, static_cast<size_t>(bytes));
  CU(cuMulticastGetGranularity, &mc_gran, &mp, CU_MULTICAST_GRANULARITY_MINIMUM);
  CUmemAllocationProp pp = phys_prop(device);
  CU(cuMemGetAllocationGranularity, &mem_gran, &pp, CU_MEM_ALLOC_GRANULARITY_MINIMUM);
  bytes_ = static_cast<int64_t>(round_up(round_up(static_cast<size_t>(bytes), mc_gran), mem_gran));
}

NvlsBuffer::~NvlsBuffer() {
  // Best effort; errors during teardown are ignored.
  try {
    if (mc_va_) {
      drv<decltype(&cuMemUnmap)>("cuMemUnmap")(mc_va_, bytes_);
      drv<decltype(&cuMemAddressFree)>("cuMemAddressFree")(mc_va_, bytes_);
    }
    if (uc_va_) {
      drv<decltype(&cuMemUnmap)>("cuMemUnmap")(uc_va_, bytes_);
      drv<decltype(&cuMemAddressFree)>("cuMemAddressFree")(uc_va_, bytes_);
    }
    if (bound_) {
      CUdevice d;
      drv<decltype(&cuDeviceGet)>("cuDeviceGet")(&d, device_);
      drv<decltype(&cuMulticastUnbind)>("cuMulticastUnbind")(mc_, d, 0, bytes_);
    }
    if (phys_) drv<decltype(&cuMemRelease)>("cuMemRelease")(phys_);
    if (mc_) drv<decltype(&cuMemRelease)>("cuMemRelease")(mc_);
  } catch (...) {
  }
}

int NvlsBuffer::create_and_export() {
  CUmulticastObjectProp mp = mc_prop(world_, static_cast<size_t>(bytes_));
  CUmemGenericAllocationHandle h;
  CU(cuMulticastCreate, &h, &mp);
  mc_ = h;
  int fd = -1;
  CU(cuMemExportToShareableHandle, &fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0ull);
  return fd;
}

void NvlsBuffer::import_handle(int fd) {
  CUmemGenericAllocationHandle h;
  CU(cuMemImportFromShareableHandle, &h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
     CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
  mc_ = h;
}

void NvlsBuffer::add_device() {
  CUdevice d;
  CU(cuDeviceGet, &d, device_);
  CU(cuMulticastAddDevice, mc_, d);
}

void NvlsBuffer::bind_and_map() {
  CUmemAllocationProp pp = phys_prop(device_);
  CUmemGenericAllocationHandle ph;
  CU(cuMemCreate, &ph, static_cast<size_t>(bytes_), &pp, 0ull);
  phys_ = ph;
  CU(cuMulticastBindMem, mc_, 0, ph, 0, static_cast<size_t>(bytes_), 0ull);
  bound_ = true;
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device_;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  size_t gran = 0;
  CU(cuMemGetAllocationGranularity, &gran, &pp, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
  CUdeviceptr va;
  CU(cuMemAddressReserve, &va, static_cast<size_t>(bytes_), gran, 0ull, 0ull);
  uc_va_ = va;
  CU(cuMemMap, va, static_cast<size_t>(bytes_), 0, ph, 0ull);
  CU(cuMemSetAccess, va, static_cast<size_t>(bytes_), &acc, 1);
  CU(cuMemAddressReserve, &va, static_cast<size_t>(bytes_), gran, 0ull, 0ull);
  mc_va_ = va;
  CU(cuMemMap, va, static_cast<size_t>(bytes_), 0, static_cast<CUmemGenericAllocationHandle>(mc_), 0ull);
  CU(cuMemSetAccess, va, static_cast<size_t>(bytes_), &acc, 1);
  B200AR_CUDA(cudaMemset(reinterpret_cast<void*>(uc_va_), 0, static_cast<size_t>(bytes_)));
}

int nvls_blocks_per_sm(DType dt, int world) {
  const void* k = nullptr;
  auto pick = [&](auto tag) {
    using T = decltype(tag);
    switch (world) {
      case 2: k = reinterpret_cast<const void*>(&nvls_kernel<T, 2>); break;
      case 3: k = reinterpret_cast<const void*>(&nvls_kernel<T, 3>); break;
      case 4: k = reinterpret_cast<const void*>(&nvls_kernel<T, 4>); break;
      case 5: k = reinterpret_cast<const void*>(&nvls_kernel<T, 5>); break;
      case 6: k = reinterpret_cast<const void*>(&nvls_kernel<T, 6>); break;
      case 7: k = reinterpret_cast<const void*>(&nvls_kernel<T, 7>); break;
      case 8: k = reinterpret_cast<const void*>(&nvls_kernel<T, 8>); break;
      default: break;
    }
  };
  if (dt == DType::kFloat32) pick(float{});
  else if (dt == DType::kFloat16) pick(__half{});
  else pick(__nv_bfloat16{});
  if (k == nullptr) return kMaxCTAs;
  int n = 0;
  B200AR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kArThreads, 0));
  return n;
}

void nvls_allreduce(Communicator& comm, NvlsBuffer& buf, cudaStream_t stream, const void* in, void* out,
                    int64_t bytes, int dtype, int ctas) {
  comm.check_status();
  B200AR_CHECK(bytes % 16 == 0 && bytes <= buf.bytes(), "NVLS message must be a multiple of 16 bytes and fit the "
                                                        "multicast buffer (" << buf.bytes() << " bytes)");
  B200AR_CHECK(buf.local_ptr() && buf.multicast_ptr(), "NVLS buffer is not mapped");
  if (bytes == 0) return;
  NvlsArgs a{};
  comm.fill_ctx(&a.ctx);
  a.uc = static_cast<char*>(buf.local_ptr());
  a.mc = static_cast<char*>(buf.multicast_ptr());
  a.in = static_cast<const char*>(in);
  a.out = static_cast<char*>(out);
  a.packets = bytes / 16;
  const int world = comm.world();
  const int64_t part = a.packets / world;
  (void)part;
  const int grid = plan_ctas(kNvls, bytes, world, ctas, comm.resident_ctas(kNvls));
  switch (dtype) {
    case 0: launch_t<float>(world, grid, a, stream); break;
    case 1: launch_t<__half>(world, grid, a, stream); break;
    case 2: launch_t<__nv_bfloat16>(world, grid, a, stream); break;
    default: throw std::invalid_argument("NVLS all-reduce supports float32, float16 and bfloat16");
  }
  B200AR_CUDA(cudaGetLastError());
  comm.count_launch();
}

}  // namespace b200ar
