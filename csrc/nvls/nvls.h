// NVLink SHARP (NVLS) multicast buffers and the NVLS all-reduce.
//
// The reference has no switch-side reduction (it targets PCIe, pcie_allreduce.cu:1-3).
// On NVSwitch systems a multicast object lets one instruction reach every
// GPU of the team: `multimem.ld_reduce` returns the sum of one address over
// all GPUs (the reduction happens in the switch), `multimem.st` writes one
// value to every GPU. Per rank this moves about (1 + 1/N) of the message each
// way instead of the 2(N-1)/N of a two-shot.
//
// Set-up is collective and driven from Python (file-descriptor passing between
// the rank processes):
//   rank 0: create() -> POSIX fd of the multicast handle, sent to the others;
//   others: import_handle(fd);
//   all:    add_device(); <barrier>; bind_and_map().
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace b200ar {

class Communicator;

class NvlsBuffer {
 public:
  NvlsBuffer(int device, int world, int64_t bytes);
  ~NvlsBuffer();
  NvlsBuffer(const NvlsBuffer&) = delete;
  NvlsBuffer& operator=(const NvlsBuffer&) = delete;

  // True if `device` reports switch multicast support.
  static bool supported(int device);

  int create_and_export();          // rank 0: returns a POSIX fd (caller closes it)
  void import_handle(int fd);       // other ranks
  void add_device();                // every rank, before any bind
  void bind_and_map();              // every rank, after all add_device calls

  int64_t bytes() const { return bytes_; }
  void* multicast_ptr() const { return reinterpret_cast<void*>(mc_va_); }
  void* local_ptr() const { return reinterpret_cast<void*>(uc_va_); }

 private:
  int device_;
  int world_;
  int64_t bytes_;
  unsigned long long mc_ = 0;    // CUmemGenericAllocationHandle
  unsigned long long phys_ = 0;  // CUmemGenericAllocationHandle
  unsigned long long mc_va_ = 0;
  unsigned long long uc_va_ = 0;
  bool bound_ = false;
};

// Sum all-reduce of `bytes` (multiple of 16, <= buf.bytes()) through `buf`
// with multimem.ld_reduce / multimem.st; barriers use the communicator's
// flags. `dtype`: 0 fp32, 1 fp16, 2 bf16.
void nvls_allreduce(Communicator& comm, NvlsBuffer& buf, cudaStream_t stream, const void* in, void* out,
                    int64_t bytes, int dtype, int ctas);

}  // namespace b200ar
