// Binds the single-GPU model kernels (GEMM, norms, RoPE, attention, activation).
#include "ops.h"

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../gemm/gemm_api.h"
#include "../model/model.h"

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
  m.def(
      "gemm_bf16_2sm",
      [](const at::Tensor& a, const at::Tensor& b, at::Tensor& c, at::Tensor& err, int max_pairs) {
        check_bf16_2d(a, "A");
        check_bf16_2d(b, "B");
        check_bf16_2d(c, "C");
        TORCH_CHECK(a.size(1) == b.size(1) && c.size(0) == a.size(0) && c.size(1) == b.size(0), "shape mismatch");
        TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt && err.numel() >= 1, "err must be a CUDA int32");
        const at::cuda::OptionalCUDAGuard guard(device_of(a));
        b200ar::gemm_bf16_2sm(a.data_ptr(), b.data_ptr(), c.data_ptr(), a.size(0), b.size(0), a.size(1),
                              err.data_ptr<int>(), at::cuda::getCurrentCUDAStream().stream(), max_pairs);
      },
      "C = A @ B^T on CTA pairs (tcgen05 cta_group::2, 256 x 256 tiles)", py::arg("a"), py::arg("b"), py::arg("c"),
      py::arg("err"), py::arg("max_pairs") = 0);
  auto stream = []() { return at::cuda::getCurrentCUDAStream().stream(); };
  m.def(
      "rmsnorm",
      [stream](const at::Tensor& x, const at::Tensor& gamma, at::Tensor& y, double eps) {
        TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && x.scalar_type() == at::kBFloat16, "bf16 contiguous");
        const at::cuda::OptionalCUDAGuard guard(device_of(x));
        b200ar::rmsnorm(x.data_ptr(), gamma.data_ptr(), y.data_ptr(), x.numel() / gamma.numel(), gamma.numel(),
                        static_cast<float>(eps), stream());
      },
      py::arg("x"), py::arg("gamma"), py::arg("y"), py::arg("eps"));
  m.def(
      "rope_kv",
      [stream](const at::Tensor& qkv, const at::Tensor& pos, const at::Tensor& cos_t, const at::Tensor& sin_t,
               at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache, int hq, int hkv, int head_dim) {
        TORCH_CHECK(pos.scalar_type() == at::kInt && cos_t.scalar_type() == at::kFloat, "pos int32, tables fp32");
        TORCH_CHECK(k_cache.dim() == 4, "KV cache is [batch, max_len, kv_heads, head_dim]");
        const at::cuda::OptionalCUDAGuard guard(device_of(qkv));
        b200ar::rope_kv(qkv.data_ptr(), pos.data_ptr<int>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                        q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), qkv.size(0), hq, hkv, head_dim,
                        static_cast<int>(k_cache.size(1)), stream());
      });
  m.def("attention_splits", &b200ar::attention_splits);
  m.def(
      "decode_attention",
      [stream](const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache, const at::Tensor& seq_len,
               at::Tensor& out, at::Tensor& part_acc, at::Tensor& part_ml, at::Tensor& done_count, int hq, int hkv,
               int splits, double scale) {
        const int64_t b = q.size(0);
        TORCH_CHECK(part_acc.numel() >= b * hq * splits * 128 && part_ml.numel() >= b * hq * splits * 2,
                    "attention workspace too small");
        TORCH_CHECK(done_count.scalar_type() == at::kInt && done_count.numel() >= b * hkv,
                    "attention counters must be int32 with one entry per (batch, KV head), zero at first use");
        const at::cuda::OptionalCUDAGuard guard(device_of(q));
        b200ar::decode_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), seq_len.data_ptr<int>(),
                                 out.data_ptr(), part_acc.data_ptr<float>(), part_ml.data_ptr<float>(),
                                 reinterpret_cast<unsigned*>(done_count.data_ptr<int>()), b, hq, hkv,
                                 128, static_cast<int>(k_cache.size(1)), splits, static_cast<float>(scale), stream());
      });
  m.def("attention_tc_splits", &b200ar::attention_tc_splits);
  m.def(
      "decode_attention_tc",
      [stream](const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache, const at::Tensor& seq_len,
               at::Tensor& out, at::Tensor& part_acc, at::Tensor& part_ml, at::Tensor& done_count, at::Tensor& err,
               int hq, int hkv, int splits, double scale) {
        for (const at::Tensor* t : {&q, &k_cache, &v_cache, static_cast<const at::Tensor*>(&out)})
          TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == at::kBFloat16,
                      "decode attention takes contiguous bf16 CUDA tensors");
        TORCH_CHECK(k_cache.dim() == 4 && v_cache.sizes() == k_cache.sizes() && k_cache.size(2) == hkv &&
                        k_cache.size(3) == 128,
                    "KV caches are [batch, max_len, kv_heads, 128]");
        const int64_t b = q.size(0);
        TORCH_CHECK(q.numel() == b * hq * 128 && out.numel() == b * hq * 128 && k_cache.size(0) == b,
                    "q and out are [batch, hq * 128]");
        TORCH_CHECK(seq_len.scalar_type() == at::kInt && seq_len.numel() >= b, "seq_len must be int32 [batch]");
        TORCH_CHECK(part_acc.numel() >= b * hq * splits * 128 && part_ml.numel() >= b * hq * splits * 2,
                    "attention workspace too small");
        TORCH_CHECK(done_count.scalar_type() == at::kInt && done_count.numel() >= b * hkv,
                    "attention counters must be int32 with one entry per (batch, KV head), zero at first use");
        TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt, "err must be a CUDA int32 tensor");
        const at::cuda::OptionalCUDAGuard guard(device_of(q));
        b200ar::decode_attention_tc(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), seq_len.data_ptr<int>(),
                                    out.data_ptr(), part_acc.data_ptr<float>(), part_ml.data_ptr<float>(),
                                    reinterpret_cast<unsigned*>(done_count.data_ptr<int>()), err.data_ptr<int>(), b,
                                    hq, hkv, 128, static_cast<int>(k_cache.size(1)), splits,
                                    static_cast<float>(scale), stream());
      });
  m.def(
      "silu_mul",
      [stream](const at::Tensor& gu, at::Tensor& y, int group) {
        TORCH_CHECK(gu.is_cuda() && gu.dim() == 2 && gu.is_contiguous() && y.is_contiguous() &&
                        gu.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16,
                    "silu_mul takes contiguous bf16 CUDA tensors");
        TORCH_CHECK(gu.size(1) == 2 * y.size(1) && gu.size(0) == y.size(0), "shape mismatch");
        const at::cuda::OptionalCUDAGuard guard(device_of(gu));
        b200ar::silu_mul(gu.data_ptr(), y.data_ptr(), gu.size(0), y.size(1), stream(), group);
      },
      py::arg("gate_up"), py::arg("y"), py::arg("group") = 0);
  m.def("skinny_splits", &b200ar::skinny_splits, py::arg("n"), py::arg("k"), py::arg("sms"));
  m.def(
      "gemm_skinny",
      [](const at::Tensor& x, const at::Tensor& w, at::Tensor& out, at::Tensor& partials, at::Tensor& counters,
         at::Tensor& err, int splits, int epilogue) {
        check_bf16_2d(x, "x");
        check_bf16_2d(w, "W");
        check_bf16_2d(out, "out");
        const int64_t out_cols = epilogue == 1 ? w.size(0) / 2 : w.size(0);
        TORCH_CHECK(x.size(1) == w.size(1) && out.size(0) == x.size(0) && out.size(1) == out_cols, "shape mismatch");
        TORCH_CHECK(partials.is_cuda() && partials.scalar_type() == at::kFloat &&
                        partials.numel() >= (splits > 1 || epilogue ? splits * x.size(0) * w.size(0) : 0),
                    "partials must be a CUDA float32 tensor of splits * M * N elements");
        TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt &&
                        counters.numel() >= (w.size(0) + 127) / 128,
                    "counters must be a zeroed CUDA int32 tensor of ceil(N / 128) elements");
        const at::cuda::OptionalCUDAGuard guard(device_of(x));
        b200ar::gemm_skinny(x.data_ptr(), w.data_ptr(), out.data_ptr(), partials.data_ptr<float>(),
                            reinterpret_cast<unsigned*>(counters.data_ptr<int>()), x.size(0), w.size(0), x.size(1),
                            splits, err.data_ptr<int>(), at::cuda::getCurrentCUDAStream().stream(), epilogue);
      },
      "decode GEMM (M <= 128): out = x @ W^T, swap-AB tcgen05 with split-K; epilogue 1 = SiLU-gate over "
      "64-row gate/up groups",
      py::arg("x"), py::arg("w"), py::arg("out"), py::arg("partials"), py::arg("counters"), py::arg("err"),
      py::arg("splits"), py::arg("epilogue") = 0);
  m.def(
      "gemm_skinny_rope_kv",
      [](const at::Tensor& x, const at::Tensor& w, const at::Tensor& pos, const at::Tensor& cos_t,
         const at::Tensor& sin_t, at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache, at::Tensor& partials,
         at::Tensor& counters, at::Tensor& err, int splits, int hq, int hkv) {
        check_bf16_2d(x, "x");
        check_bf16_2d(w, "W");
        TORCH_CHECK(x.size(1) == w.size(1) && w.size(0) == static_cast<int64_t>(hq + 2 * hkv) * 128,
                    "W must hold (hq + 2 hkv) heads of 128 rows");
        TORCH_CHECK(pos.is_cuda() && pos.scalar_type() == at::kInt && pos.numel() >= x.size(0), "pos: int32 [M]");
        TORCH_CHECK(cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat && cos_t.size(-1) == 64,
                    "rotary tables: fp32 [positions, 64]");
        TORCH_CHECK(q_out.is_contiguous() && q_out.numel() == x.size(0) * hq * 128, "q_out: [M, hq, 128]");
        TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(0) >= x.size(0) && k_cache.size(2) == hkv &&
                        k_cache.size(3) == 128 && v_cache.sizes() == k_cache.sizes() && k_cache.is_contiguous() &&
                        v_cache.is_contiguous(),
                    "KV caches: [batch, max_len, hkv, 128]");
        TORCH_CHECK(partials.is_cuda() && partials.scalar_type() == at::kFloat &&
                        partials.numel() >= splits * x.size(0) * w.size(0),
                    "partials must be a CUDA float32 tensor of splits * M * N elements");
        TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= w.size(0) / 128,
                    "counters must be a zeroed CUDA int32 tensor of N / 128 elements");
        const at::cuda::OptionalCUDAGuard guard(device_of(x));
        b200ar::RopeKvArgs r{};
        r.pos = pos.data_ptr<int>();
        r.cos_t = cos_t.data_ptr<float>();
        r.sin_t = sin_t.data_ptr<float>();
        r.q_out = static_cast<__nv_bfloat16*>(q_out.data_ptr());
        r.k_cache = static_cast<__nv_bfloat16*>(k_cache.data_ptr());
        r.v_cache = static_cast<__nv_bfloat16*>(v_cache.data_ptr());
        r.hq = hq;
        r.hkv = hkv;
        r.max_len = static_cast<int>(k_cache.size(1));
        b200ar::gemm_skinny(x.data_ptr(), w.data_ptr(), nullptr, partials.data_ptr<float>(),
                            reinterpret_cast<unsigned*>(counters.data_ptr<int>()), x.size(0), w.size(0), x.size(1),
                            splits, err.data_ptr<int>(), at::cuda::getCurrentCUDAStream().stream(), 2, &r);
      },
      "decode QKV GEMM (M <= 128) with RoPE and the KV-cache write in its split-K epilogue", py::arg("x"),
      py::arg("w"), py::arg("pos"), py::arg("cos_t"), py::arg("sin_t"), py::arg("q_out"), py::arg("k_cache"),
      py::arg("v_cache"), py::arg("partials"), py::arg("counters"), py::arg("err"), py::arg("splits"),
      py::arg("hq"), py::arg("hkv"));
}
