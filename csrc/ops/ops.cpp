// Binds the single-GPU model kernels (GEMM, norms, RoPE, attention, activation).
#include "ops.h"

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../gemm/gemm_api.h"

namespace py = pybind11;

namespace {

void check_bf16_2d(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.is_contiguous() && t.scalar_type() == at::kBFloat16, name,
              " must be a contiguous 2-D bf16 CUDA tensor");
}

}  // namespace

void register_ops(py::module& m) {
  m.def(
      "gemm_bf16",
      [](const at::Tensor& a, const at::Tensor& b, at::Tensor& c, at::Tensor& err, int max_ctas) {
        check_bf16_2d(a, "A");
        check_bf16_2d(b, "B");
        check_bf16_2d(c, "C");
        TORCH_CHECK(a.size(1) == b.size(1) && c.size(0) == a.size(0) && c.size(1) == b.size(0), "shape mismatch");
        TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt && err.numel() >= 1, "err must be a CUDA int32");
        const at::cuda::OptionalCUDAGuard guard(device_of(a));
        b200ar::gemm_bf16(a.data_ptr(), b.data_ptr(), c.data_ptr(), a.size(0), b.size(0), a.size(1),
                          err.data_ptr<int>(), at::cuda::getCurrentCUDAStream().stream(), max_ctas);
      },
      "C = A @ B^T with the tcgen05 GEMM (bf16 in/out, fp32 accumulate)", py::arg("a"), py::arg("b"), py::arg("c"),
      py::arg("err"), py::arg("max_ctas") = 0);
}
