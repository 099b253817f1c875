// Python bindings of the b200ar native library (module b200ar._C).
//
// Two surfaces:
//  * the idiomatic one used by b200ar.parallel.CustomAllreduce: class `Comm`
//    around the C++ Communicator, the CPU `ShmComm`, and IPC helpers;
//  * the reference-compatible op set (init_custom_ar, all_reduce, dispose,
//    meta_size, register_buffer, register_pcie_buffers,
//    get_graph_buffer_ipc_meta, register_graph_buffers), with the names and
//    argument lists of pcie_allreduce/pcie_allreduce.cu:596-606, so code written
//    against the reference (or sgl_kernel.allreduce) runs unchanged.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include "comm/communicator.h"
#include "cpu/shm_comm.h"
#include "fused/fused.h"
#include "nvls/nvls.h"
#include "ops/ops.h"

namespace py = pybind11;
using namespace b200ar;

namespace {

DType to_dtype(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return DType::kFloat32;
    case at::kHalf: return DType::kFloat16;
    case at::kBFloat16: return DType::kBFloat16;
    default: throw std::invalid_argument("only float32, float16 and bfloat16 are supported");
  }
}

bool weak_contiguous(const at::Tensor& t) {
  return t.is_contiguous() ||
         (t.storage().nbytes() - t.storage_offset() * t.element_size() == t.numel() * t.element_size());
}

void check_pair(const at::Tensor& inp, const at::Tensor& out) {
  TORCH_CHECK(inp.scalar_type() == out.scalar_type(), "input and output dtypes differ");
  TORCH_CHECK(inp.numel() == out.numel(), "input and output sizes differ");
  TORCH_CHECK(weak_contiguous(inp) && weak_contiguous(out), "tensors must be (weakly) contiguous");
}

py::bytes as_bytes(const std::string& s) { return py::bytes(s); }

Communicator* as_comm(int64_t fa) { return reinterpret_cast<Communicator*>(fa); }

// ---- reference-compatible ops -------------------------------------------

int64_t init_custom_ar(const std::vector<int64_t>& fake_ipc_ptrs, at::Tensor& rank_data, int64_t rank) {
  const int world = static_cast<int>(fake_ipc_ptrs.size());
  if (world > kMaxRanks) throw std::invalid_argument("world size > 8 is not supported");
  if (rank < 0 || rank >= world) throw std::invalid_argument("invalid rank");
  TORCH_CHECK(rank_data.is_cuda(), "rank_data must be a CUDA tensor");
  auto* c = new Communicator(fake_ipc_ptrs, rank_data.data_ptr(), rank_data.numel() * rank_data.element_size(),
                             static_cast<int>(rank));
  return reinterpret_cast<int64_t>(c);
}

void compat_all_reduce(int64_t fa, at::Tensor& inp, at::Tensor& out, int64_t reg_buffer, int64_t reg_buffer_sz) {
  Communicator* c = as_comm(fa);
  const at::cuda::OptionalCUDAGuard guard(device_of(inp));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  check_pair(inp, out);
  const int64_t bytes = inp.numel() * inp.element_size();
  const void* src = inp.data_ptr();
  if (!c->slots_registered() && reg_buffer != 0) {
    TORCH_CHECK(bytes <= reg_buffer_sz, "input of ", bytes, " bytes exceeds registered buffer of ", reg_buffer_sz);
    B200AR_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(reg_buffer), src, bytes, cudaMemcpyDeviceToDevice, stream));
    src = reinterpret_cast<const void*>(reg_buffer);
  }
  LaunchInfo li = c->allreduce(stream, src, out.data_ptr(), bytes, to_dtype(inp), kAuto, 0);
  if (li.variant == kNccl)
    throw std::runtime_error("message of " + std::to_string(bytes) +
                             " bytes does not fit the registered buffers and the input is not registered");
}

void dispose(int64_t fa) { delete as_comm(fa); }

int64_t meta_size() { return static_cast<int64_t>(sizeof(Signal)); }

void compat_register_buffer(int64_t fa, const std::vector<int64_t>& ptrs) { as_comm(fa)->register_buffer(ptrs); }

void register_pcie_buffers(int64_t fa, const std::vector<int64_t>& p0, const std::vector<int64_t>& p1,
                           int64_t cap) {
  as_comm(fa)->register_slots(p0, p1, cap);
}

std::tuple<std::vector<int64_t>, std::vector<int64_t>> get_graph_buffer_ipc_meta(int64_t fa) {
  auto [h, off] = as_comm(fa)->graph_buffer_meta();
  std::vector<int64_t> bytes(h.begin(), h.end());
  return {bytes, off};
}

void compat_register_graph_buffers(int64_t fa, const std::vector<std::vector<int64_t>>& handles,
                                   const std::vector<std::vector<int64_t>>& offsets) {
  std::vector<std::string> hs;
  hs.reserve(handles.size());
  for (const auto& h : handles) {
    std::string s(h.size(), '\0');
    for (size_t i = 0; i < h.size(); ++i) s[i] = static_cast<char>(h[i]);
    hs.push_back(std::move(s));
  }
  as_comm(fa)->register_graph_buffers(hs, offsets);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "b200ar native library: NVLink/NVSwitch custom all-reduce and fused TP kernels for sm_100a";

  py::register_exception<CommTimeout>(m, "CommTimeout", PyExc_RuntimeError);

  // ---- constants ----
  m.attr("MAX_RANKS") = kMaxRanks;
  m.attr("MAX_CTAS") = kMaxCTAs;
  m.attr("SIGNAL_BYTES") = static_cast<int64_t>(sizeof(Signal));
  m.attr("IPC_HANDLE_BYTES") = static_cast<int64_t>(sizeof(cudaIpcMemHandle_t));
  py::dict variants;
  variants["auto"] = static_cast<int>(kAuto);
  variants["oneshot_push"] = static_cast<int>(kOneshotPush);
  variants["oneshot_pull"] = static_cast<int>(kOneshotPull);
  variants["twoshot"] = static_cast<int>(kTwoshot);
  variants["nvls"] = static_cast<int>(kNvls);
  variants["registered"] = static_cast<int>(kRegistered);
  variants["nccl"] = static_cast<int>(kNccl);
  variants["copy"] = static_cast<int>(kCopy);
  variants["lamport"] = static_cast<int>(kLamport);
  variants["twoshot_push"] = static_cast<int>(kTwoshotPush);
  m.attr("VARIANTS") = variants;

  m.def("ar_rmsnorm_slot_bytes", &ar_rmsnorm_slot_bytes);
  m.def("gemm_ar_slot_bytes", &gemm_ar_slot_bytes);
  m.def("lamport_bytes", &lamport_bytes);
  m.def("workspace_bytes", &workspace_bytes, "bytes of one rank's workspace for a slot capacity");
  m.def("plan_ctas", &plan_ctas, "CTA count of a collective launch (clamped to the co-resident count)",
        py::arg("variant"), py::arg("bytes"), py::arg("world"), py::arg("requested"), py::arg("resident"));
  m.def("variant_slot_bytes", &variant_slot_bytes, "slot bytes a variant needs", py::arg("variant"),
        py::arg("bytes"), py::arg("world"));

  // ---- IPC helpers ----
  m.def("ipc_malloc", [](int64_t n) { return reinterpret_cast<int64_t>(ipc_malloc(n)); },
        "cudaMalloc + zero-fill (IPC-exportable)");
  m.def("ipc_free", [](int64_t p) { ipc_free(reinterpret_cast<void*>(p)); });
  m.def("ipc_memset", [](int64_t p, int v, int64_t n) {
    B200AR_CUDA(cudaMemset(reinterpret_cast<void*>(p), v, static_cast<size_t>(n)));
  });
  m.def("ipc_get_handle", [](int64_t p) { return as_bytes(ipc_get_handle(reinterpret_cast<void*>(p))); });
  m.def("ipc_open_handle", [](py::bytes h) { return reinterpret_cast<int64_t>(IpcRegistry::get().open(h)); },
        "open a peer's handle (cached, reference counted)");
  m.def("ipc_close_handle", [](int64_t p) { IpcRegistry::get().release(reinterpret_cast<char*>(p)); });
  m.def("ipc_open_count", []() { return IpcRegistry::get().open_count(); });
  m.def("allocation_range", [](int64_t p) {
    auto [b, s] = allocation_range(reinterpret_cast<void*>(p));
    return std::make_tuple(reinterpret_cast<int64_t>(b), s);
  });

  // ---- rank-data arena bookkeeping (host only; exposed for tests) ----
  m.attr("RANK_DATA_BYTES") = static_cast<int64_t>(sizeof(RankData));
  py::class_<RankDataArena>(m, "RankDataArena")
      .def(py::init([](int64_t base, int64_t bytes) { return RankDataArena(reinterpret_cast<void*>(base), bytes); }),
           py::arg("base"), py::arg("bytes"))
      .def_property_readonly("capacity", &RankDataArena::capacity)
      .def_property_readonly("used", &RankDataArena::used)
      .def_property_readonly("remaining", &RankDataArena::remaining)
      .def("fits", &RankDataArena::fits)
      .def("peek", [](const RankDataArena& a, int64_t k) { return reinterpret_cast<int64_t>(a.peek(k)); })
      .def("take", [](RankDataArena& a, int64_t n) { return reinterpret_cast<int64_t>(a.take(n)); });

  // ---- idiomatic communicator ----
  py::class_<Communicator>(m, "Comm")
      .def(py::init([](const std::vector<int64_t>& signals, at::Tensor& rank_data, int rank) {
             TORCH_CHECK(rank_data.is_cuda(), "rank_data must be a CUDA tensor");
             return new Communicator(signals, rank_data.data_ptr(), rank_data.numel() * rank_data.element_size(),
                                     rank);
           }),
           py::arg("signals"), py::arg("rank_data"), py::arg("rank"))
      .def_property_readonly("rank", &Communicator::rank)
      .def_property_readonly("world", &Communicator::world)
      .def_property_readonly("ptr", [](Communicator& c) { return reinterpret_cast<int64_t>(&c); })
      .def_property_readonly("slot_capacity", &Communicator::slot_capacity)
      .def_property_readonly("launches", &Communicator::launches)
      .def("resident_ctas", &Communicator::resident_ctas, py::arg("variant"))
      .def_property_readonly("pending_graph_buffers", &Communicator::pending_graph_buffers)
      .def("open_ipc_handle",
           [](Communicator& c, py::bytes h) { return reinterpret_cast<int64_t>(c.open_ipc_handle(h)); })
      .def("register_slots", &Communicator::register_slots, py::arg("ptrs0"), py::arg("ptrs1"),
           py::arg("capacity"))
      .def("register_buffer", &Communicator::register_buffer)
      .def("register_lamport", &Communicator::register_lamport, py::arg("ptrs"), py::arg("capacity"))
      .def_property_readonly("lamport_capacity", &Communicator::lamport_capacity)
      .def("graph_buffer_meta",
           [](Communicator& c) {
             auto [h, off] = c.graph_buffer_meta();
             return std::make_tuple(py::bytes(h), off);
           })
      .def("register_graph_buffers",
           [](Communicator& c, const std::vector<py::bytes>& handles, const std::vector<std::vector<int64_t>>& off) {
             std::vector<std::string> hs(handles.begin(), handles.end());
             c.register_graph_buffers(hs, off);
           })
      .def("set_timeout_ns", &Communicator::set_timeout_ns)
      .def_property_readonly("timeout_ns", &Communicator::timeout_ns)
      .def("set_selector",
           [](Communicator& c, const std::vector<std::tuple<int64_t, int, int>>& t) {
             std::vector<SelectorEntry> s;
             for (auto& [b, v, k] : t) s.push_back({b, v, k});
             c.set_selector(s);
           })
      .def("selector",
           [](Communicator& c) {
             std::vector<std::tuple<int64_t, int, int>> t;
             for (auto& e : c.selector()) t.emplace_back(e.max_bytes, e.variant, e.ctas);
             return t;
           })
      .def("plan",
           [](Communicator& c, int64_t bytes, int variant, int ctas) {
             LaunchInfo li = c.plan(bytes, variant, ctas, false, false);
             return std::make_tuple(li.variant, li.ctas, li.threads);
           },
           py::arg("bytes"), py::arg("variant") = 0, py::arg("ctas") = 0)
      .def("all_reduce",
           [](Communicator& c, at::Tensor& inp, at::Tensor& out, int variant, int ctas) {
             check_pair(inp, out);
             TORCH_CHECK(inp.is_cuda() && out.is_cuda(), "CUDA tensors required");
             const at::cuda::OptionalCUDAGuard guard(device_of(inp));
             cudaStream_t s = at::cuda::getCurrentCUDAStream().stream();
             LaunchInfo li = c.allreduce(s, inp.data_ptr(), out.data_ptr(), inp.numel() * inp.element_size(),
                                         to_dtype(inp), variant, ctas);
             return li.variant;
           },
           py::arg("inp"), py::arg("out"), py::arg("variant") = 0, py::arg("ctas") = 0)
      // Lean eager entry used by CustomAllreduce.all_reduce for variant "auto":
      // every check in C++, one call from Python. Returns false (nothing
      // launched) when the Python layer must serve the call instead: a dtype,
      // layout or alignment the kernels do not take, or the NCCL range.
      .def("all_reduce_auto",
           [](Communicator& c, const at::Tensor& inp, const at::Tensor& out) {
             const auto st = inp.scalar_type();
             if (st != at::kBFloat16 && st != at::kHalf && st != at::kFloat) return false;
             if (out.scalar_type() != st || out.numel() != inp.numel()) return false;
             const int64_t bytes = inp.numel() * inp.element_size();
             const auto ip = reinterpret_cast<uintptr_t>(inp.data_ptr());
             const auto op = reinterpret_cast<uintptr_t>(out.data_ptr());
             if ((bytes | ip | op) & 15) return false;
             if (!inp.is_cuda() || !inp.is_contiguous() || !out.is_contiguous()) return false;
             const c10::DeviceIndex dev = inp.device().index();
             if (out.device() != inp.device()) return false;
             const at::cuda::OptionalCUDAGuard guard(c10::cuda::current_device() == dev ? std::nullopt
                                                                                        : std::optional<c10::Device>(inp.device()));
             cudaStream_t s = at::cuda::getCurrentCUDAStream(dev).stream();
             LaunchInfo li = c.allreduce(s, inp.data_ptr(), out.data_ptr(), bytes, to_dtype(inp), kAuto, 0);
             return li.variant != kNccl;
           },
           py::arg("inp"), py::arg("out"))
      .def("ar_rmsnorm",
           [](Communicator& c, at::Tensor& x, at::Tensor& residual, at::Tensor& gamma, at::Tensor& y,
              at::Tensor& residual_out, double eps, int variant, int ctas) {
             for (const at::Tensor* t : {&x, &residual, &gamma, &y, &residual_out}) {
               TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == at::kBFloat16,
                           "fused all-reduce + RMSNorm takes contiguous bf16 CUDA tensors");
             }
             const int64_t hidden = gamma.numel();
             TORCH_CHECK(x.numel() % hidden == 0 && residual.numel() == x.numel() && y.numel() == x.numel() &&
                             residual_out.numel() == x.numel(),
                         "shape mismatch");
             const at::cuda::OptionalCUDAGuard guard(device_of(x));
             return ar_rmsnorm(c, at::cuda::getCurrentCUDAStream().stream(), x.data_ptr(), residual.data_ptr(),
                               gamma.data_ptr(), y.data_ptr(), residual_out.data_ptr(), x.numel() / hidden, hidden,
                               static_cast<float>(eps), variant, ctas);
           },
           py::arg("x"), py::arg("residual"), py::arg("gamma"), py::arg("y"), py::arg("residual_out"),
           py::arg("eps"), py::arg("variant") = 0, py::arg("ctas") = 0)
      // The caller keeps `buf` alive and detaches it (set_nvls(None)) before dropping it.
      .def("set_nvls", [](Communicator& c, NvlsBuffer* b) { c.set_nvls(b); }, py::arg("buf").none(true))
      .def_property_readonly("has_nvls", &Communicator::has_nvls)
      .def("gemm_ar_supported", [](Communicator& c, int64_t M, int64_t N) { return gemm_ar_supported(c, M, N); })
      .def("gemm_allreduce",
           [](Communicator& c, at::Tensor& a, at::Tensor& w, at::Tensor& out, at::Tensor& err) {
             for (const at::Tensor* t : {&a, &w, &out})
               TORCH_CHECK(t->is_cuda() && t->dim() == 2 && t->is_contiguous() && t->scalar_type() == at::kBFloat16,
                           "fused GEMM + all-reduce takes contiguous 2-D bf16 CUDA tensors");
             TORCH_CHECK(a.size(1) == w.size(1) && out.size(0) == a.size(0) && out.size(1) == w.size(0),
                         "shape mismatch");
             TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt, "err must be a CUDA int32 tensor");
             const at::cuda::OptionalCUDAGuard guard(device_of(a));
             gemm_allreduce(c, at::cuda::getCurrentCUDAStream().stream(), a.data_ptr(), w.data_ptr(), out.data_ptr(),
                            a.size(0), w.size(0), a.size(1), err.data_ptr<int>());
           })
      .def("ag_gemm_supported",
           [](Communicator& c, int64_t rows, int64_t K) { return ag_gemm_supported(c, rows, K); })
      .def("ag_gemm",
           [](Communicator& c, at::Tensor& x, at::Tensor& w, at::Tensor& y, at::Tensor& err) {
             for (const at::Tensor* t : {&x, &w, &y})
               TORCH_CHECK(t->is_cuda() && t->dim() == 2 && t->is_contiguous() && t->scalar_type() == at::kBFloat16,
                           "all-gather GEMM takes contiguous 2-D bf16 CUDA tensors");
             TORCH_CHECK(x.size(1) == w.size(1) && y.size(0) == x.size(0) * c.world() && y.size(1) == w.size(0),
                         "shape mismatch");
             const at::cuda::OptionalCUDAGuard guard(device_of(x));
             ag_gemm(c, at::cuda::getCurrentCUDAStream().stream(), x.data_ptr(), w.data_ptr(), y.data_ptr(),
                     x.size(0), w.size(0), x.size(1), err.data_ptr<int>());
           })
      .def("check", &Communicator::check_status)
      .def("status",
           [](Communicator& c) {
             Status s = c.status();
             py::dict d;
             d["code"] = s.code;
             d["rank"] = s.rank;
             d["peer"] = s.peer;
             d["cta"] = s.cta;
             d["epoch"] = s.epoch;
             d["seen"] = s.seen;
             d["count"] = s.count;
             return d;
           })
      .def("reset", [](Communicator& c) { c.reset(at::cuda::getCurrentCUDAStream().stream()); });

  // ---- NVLS multicast buffers ----
  py::class_<NvlsBuffer>(m, "NvlsBuffer")
      .def(py::init<int, int, int64_t>(), py::arg("device"), py::arg("world"), py::arg("bytes"))
      .def_static("supported", &NvlsBuffer::supported)
      .def_property_readonly("bytes", &NvlsBuffer::bytes)
      .def("create_and_export", &NvlsBuffer::create_and_export)
      .def("import_handle", &NvlsBuffer::import_handle)
      .def("add_device", &NvlsBuffer::add_device)
      .def("bind_and_map", &NvlsBuffer::bind_and_map);

  // ---- CPU shared-memory backend ----
  py::class_<ShmComm>(m, "ShmComm")
      .def(py::init<const std::string&, int, int, int64_t, int64_t>(), py::arg("prefix"), py::arg("rank"),
           py::arg("world"), py::arg("slot_capacity"), py::arg("lamport_capacity") = 0)
      .def_property_readonly("lamport_capacity", &ShmComm::lamport_capacity)
      .def_property_readonly("segment_name", &ShmComm::segment_name)
      .def_property_readonly("slot_capacity", &ShmComm::slot_capacity)
      .def_property_readonly("generation", &ShmComm::generation)
      .def("connect", &ShmComm::connect)
      .def("set_timeout_ms", &ShmComm::set_timeout_ms)
      .def("inject_skip", &ShmComm::inject_skip)
      .def("inject_flag", &ShmComm::inject_flag, py::arg("cta"), py::arg("src"), py::arg("value"))
      .def("reset", &ShmComm::reset)
      .def("status_code", [](ShmComm& c) { return c.status().code; })
      .def("all_reduce",
           [](ShmComm& c, at::Tensor& inp, at::Tensor& out, int variant, int ctas) {
             check_pair(inp, out);
             TORCH_CHECK(inp.is_cpu() && out.is_cpu(), "CPU tensors required");
             TORCH_CHECK(inp.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
             py::gil_scoped_release nogil;
             c.allreduce(inp.data_ptr(), out.data_ptr(), inp.numel() * inp.element_size(), to_dtype(inp), variant,
                         ctas);
           },
           py::arg("inp"), py::arg("out"), py::arg("variant") = 0, py::arg("ctas") = 0);

  // ---- reference-compatible op set (pcie_allreduce.cu:596-606) ----
  m.def("init_custom_ar", &init_custom_ar, "init custom all-reduce");
  m.def("all_reduce", &compat_all_reduce, "custom all-reduce");
  m.def("dispose", &dispose, "dispose custom all-reduce");
  m.def("meta_size", &meta_size, "signal metadata size");
  m.def("register_buffer", &compat_register_buffer, "register IPC buffer");
  m.def("register_pcie_buffers", &register_pcie_buffers, "register double-buffered IPC buffers", py::arg("fa"),
        py::arg("ptrs0"), py::arg("ptrs1"), py::arg("buf_capacity") = 0);
  m.def("get_graph_buffer_ipc_meta", &get_graph_buffer_ipc_meta, "get graph buffer IPC meta");
  m.def("register_graph_buffers", &compat_register_graph_buffers, "register graph buffers");

  register_ops(m);
}
