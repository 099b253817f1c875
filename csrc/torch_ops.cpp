// Dispatcher-registered operators: torch.ops.b200ar.*
//
// The pybind entry points (bindings.cpp, ops/ops.cpp) serve eager Python.
// These registrations expose the same kernels as PyTorch operators so that
// they can be traced: torch.compile sees them as opaque ops (no graph break),
// using the Meta implementations for shape propagation; CUDA-graph capture
// and torch.cuda.graphs work through them unchanged. Outputs are mutated
// arguments (`Tensor(a!)`), like the reference's `all_reduce(fa, inp, out,
// ...)` (pcie_allreduce.cu:504-547): the caller owns every buffer.
//
// A communicator is passed as its native handle (`CustomAllreduce.handle`,
// the address of the Communicator, as the reference passes `fa`). The
// all-reduce op only runs b200ar kernels: a message the selector would hand
// to NCCL runs the two-shot kernel if it fits the slot capacity and raises
// otherwise (the op cannot reach a torch.distributed process group).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "comm/communicator.h"
#include "fused/fused.h"
#include "model/model.h"

namespace b200ar {
namespace {

DType dtype_of(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return DType::kFloat32;
    case at::kHalf: return DType::kFloat16;
    case at::kBFloat16: return DType::kBFloat16;
    default: TORCH_CHECK(false, "b200ar ops take float32, float16 or bfloat16 tensors");
  }
}

cudaStream_t current_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

Communicator& comm_of(int64_t handle) {
  TORCH_CHECK(handle != 0, "b200ar: null communicator handle");
  return *reinterpret_cast<Communicator*>(handle);
}

void all_reduce_cuda(int64_t handle, const at::Tensor& inp, const at::Tensor& out, int64_t variant, int64_t ctas) {
  TORCH_CHECK(inp.is_cuda() && out.is_cuda(), "b200ar::all_reduce takes CUDA tensors");
  TORCH_CHECK(inp.scalar_type() == out.scalar_type() && inp.numel() == out.numel(), "input/output mismatch");
  TORCH_CHECK(inp.is_contiguous() && out.is_contiguous(), "b200ar::all_reduce takes contiguous tensors");
  Communicator& c = comm_of(handle);
  const c10::cuda::CUDAGuard guard(inp.device());
  const int64_t bytes = inp.numel() * inp.element_size();
  LaunchInfo li = c.allreduce(current_stream(), inp.data_ptr(), out.data_ptr(), bytes, dtype_of(inp),
                              static_cast<int>(variant), static_cast<int>(ctas));
  if (li.variant == kNccl) {
    TORCH_CHECK(variant_slot_bytes(kTwoshot, bytes, c.world()) <= c.slot_capacity(),
                "b200ar::all_reduce: message of ", bytes, " bytes is above the NCCL crossover and larger than the "
                "two-shot slot capacity; call CustomAllreduce.all_reduce eagerly or raise max_size");
    c.allreduce(current_stream(), inp.data_ptr(), out.data_ptr(), bytes, dtype_of(inp), kTwoshot, 0);
  }
}

void ar_rmsnorm_cuda(int64_t handle, const at::Tensor& x, const at::Tensor& residual, const at::Tensor& gamma,
                     double eps, const at::Tensor& y, const at::Tensor& residual_out, int64_t variant, int64_t ctas) {
  for (const at::Tensor* t : {&x, &residual, &gamma, &y, &residual_out})
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == at::kBFloat16,
                "b200ar::all_reduce_residual_rmsnorm takes contiguous bf16 CUDA tensors");
  const int64_t hidden = gamma.numel();
  TORCH_CHECK(hidden > 0 && x.numel() % hidden == 0 && residual.numel() == x.numel() && y.numel() == x.numel() &&
                  residual_out.numel() == x.numel(),
              "shape mismatch");
  const c10::cuda::CUDAGuard guard(x.device());
  ar_rmsnorm(comm_of(handle), current_stream(), x.data_ptr(), residual.data_ptr(), gamma.data_ptr(), y.data_ptr(),
             residual_out.data_ptr(), x.numel() / hidden, hidden, static_cast<float>(eps), static_cast<int>(variant),
             static_cast<int>(ctas));
}

void rmsnorm_cuda(const at::Tensor& x, const at::Tensor& gamma, double eps, const at::Tensor& y) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && y.is_contiguous() && x.scalar_type() == at::kBFloat16 &&
                  y.scalar_type() == at::kBFloat16 && gamma.scalar_type() == at::kBFloat16,
              "b200ar::rmsnorm takes contiguous bf16 CUDA tensors");
  TORCH_CHECK(gamma.numel() > 0 && x.numel() % gamma.numel() == 0 && y.numel() == x.numel(), "shape mismatch");
  const c10::cuda::CUDAGuard guard(x.device());
  rmsnorm(x.data_ptr(), gamma.data_ptr(), y.data_ptr(), x.numel() / gamma.numel(), gamma.numel(),
          static_cast<float>(eps), current_stream());
}

void silu_mul_cuda(const at::Tensor& gate_up, const at::Tensor& y, int64_t group) {
  TORCH_CHECK(gate_up.is_cuda() && gate_up.dim() == 2 && gate_up.is_contiguous() && y.is_contiguous() &&
                  gate_up.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16,
              "b200ar::silu_mul takes contiguous bf16 CUDA tensors");
  TORCH_CHECK(gate_up.size(1) % 2 == 0 && y.numel() == gate_up.numel() / 2, "shape mismatch");
  const c10::cuda::CUDAGuard guard(gate_up.device());
  silu_mul(gate_up.data_ptr(), y.data_ptr(), gate_up.size(0), gate_up.size(1) / 2, current_stream(),
           static_cast<int>(group));
}

// Meta (fake) implementations: outputs are caller-provided, nothing to compute.
void all_reduce_meta(int64_t, const at::Tensor& inp, const at::Tensor& out, int64_t, int64_t) {
  TORCH_CHECK(inp.numel() == out.numel() && inp.scalar_type() == out.scalar_type(), "input/output mismatch");
}
void ar_rmsnorm_meta(int64_t, const at::Tensor& x, const at::Tensor& residual, const at::Tensor& gamma, double,
                     const at::Tensor& y, const at::Tensor& residual_out, int64_t, int64_t) {
  TORCH_CHECK(gamma.numel() > 0 && x.numel() % gamma.numel() == 0 && residual.numel() == x.numel() &&
                  y.numel() == x.numel() && residual_out.numel() == x.numel(),
              "shape mismatch");
}
void rmsnorm_meta(const at::Tensor& x, const at::Tensor& gamma, double, const at::Tensor& y) {
  TORCH_CHECK(gamma.numel() > 0 && x.numel() % gamma.numel() == 0 && y.numel() == x.numel(), "shape mismatch");
}
void silu_mul_meta(const at::Tensor& gate_up, const at::Tensor& y, int64_t) {
  TORCH_CHECK(gate_up.dim() == 2 && gate_up.size(1) % 2 == 0 && y.numel() == gate_up.numel() / 2, "shape mismatch");
}

}  // namespace
}  // namespace b200ar

TORCH_LIBRARY(b200ar, m) {
  m.def("all_reduce(int comm, Tensor inp, Tensor(a!) out, int variant=0, int ctas=0) -> ()");
  m.def(
      "all_reduce_residual_rmsnorm(int comm, Tensor x, Tensor residual, Tensor gamma, float eps, Tensor(a!) y, "
      "Tensor(b!) residual_out, int variant=0, int ctas=0) -> ()");
  m.def("rmsnorm(Tensor x, Tensor gamma, float eps, Tensor(a!) y) -> ()");
  m.def("silu_mul(Tensor gate_up, Tensor(a!) y, int group=0) -> ()");
}

TORCH_LIBRARY_IMPL(b200ar, CUDA, m) {
  m.impl("all_reduce", &b200ar::all_reduce_cuda);
  m.impl("all_reduce_residual_rmsnorm", &b200ar::ar_rmsnorm_cuda);
  m.impl("rmsnorm", &b200ar::rmsnorm_cuda);
  m.impl("silu_mul", &b200ar::silu_mul_cuda);
}

TORCH_LIBRARY_IMPL(b200ar, Meta, m) {
  m.impl("all_reduce", &b200ar::all_reduce_meta);
  m.impl("all_reduce_residual_rmsnorm", &b200ar::ar_rmsnorm_meta);
  m.impl("rmsnorm", &b200ar::rmsnorm_meta);
  m.impl("silu_mul", &b200ar::silu_mul_meta);
}
