// ORACLE — test infrastructure: PyFlame's own Python module with the CUDA
// executor behind it.
//
// The link recipe (Makefile target `pyext`) compiles PyFlame's pybind11
// module exactly as PyFlame ships it (python/bindings.cpp, nn_bindings.cpp and
// the pyflame_core sources, unmodified) into oracle/_ref/py/_pyflame_cpp.so,
// together with this file, which adds what a CUDA backend adds on PyFlame's
// side:
//   - a second module, `_pyflame_cuda`, in the same shared library (so it
//     shares PyFlame's types and thread-local graph; import it before
//     `_pyflame_cpp`, see below): the device functions of
//     the ROCm binding block (bindings.cpp:430-463) as cuda_*, and
//     set_device / get_device accepting "cpu", "cuda" and "cuda:N" as
//     python/pyflame/__init__.py:464-533 does for "rocm[:N]";
//   - TensorImpl::materialize (tensor_impl.cpp:10-36) routed to the CUDA
//     executor while a CUDA device is selected: the whole subgraph of the
//     tensor is evaluated by libpyflame_cuda.so through the PyFlame-side
//     bridge, and the result is stored as the tensor's data.  The link wraps
//     the symbol (-Wl,--wrap), so Tensor::eval / data<T>() / numpy() reach
//     this function first; with the CPU selected it defers to PyFlame's own.
// In PyFlame itself the same routing is a branch at the top of
// TensorImpl::materialize; here it is added without editing PyFlame's files.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "pyflame/core/tensor.hpp"
#include "pyflame/core/tensor_impl.hpp"
#include "pyflame/optim/lr_scheduler.hpp"
#include "pyflame_b200/integration/pyflame_graph_bridge.hpp"

namespace py = pybind11;
using namespace pyflame;

namespace {

// TensorImpl keeps its evaluated bytes in a private member with no setter;
// an explicit instantiation may name a private member (its access is not
// checked there), which gives this harness a pointer to it.
template <typename Tag, typename Tag::type M>
struct Expose {
  friend typename Tag::type member(Tag) { return M; }
};
struct ImplData {
  using type = std::shared_ptr<uint8_t> TensorImpl::*;
  friend type member(ImplData);
};
template struct Expose<ImplData, &TensorImpl::data_>;

// ExecutionResult's fields as PyFlame's executor declares them (executor.cpp:148-160).
struct Result {
  bool success = false;
  std::string error_message;
  double compile_time_ms = 0, transfer_time_ms = 0, compute_time_ms = 0, total_time_ms = 0;
  std::unordered_map<ir::NodeId, std::shared_ptr<uint8_t>> outputs;
};

std::mutex g_mu;
int g_device = -1;  // -1: PyFlame's CPU path
std::unique_ptr<backend::cuda::CudaExecutor> g_ex;
long g_routed = 0;  // tensors evaluated through the CUDA executor

}  // namespace

extern "C" void* __real__ZN7pyflame10TensorImpl11materializeEv(TensorImpl* self);

extern "C" void* __wrap__ZN7pyflame10TensorImpl11materializeEv(TensorImpl* self) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_device < 0 || self->data() || !self->node()->is_operation() || !g_ex) {
      // PyFlame's own path: CPU evaluation, or a constant's payload copy
    } else {
      auto graph = self->graph();
      auto node = self->node();
      Result r = g_ex->execute<Result>(*graph, {node->id()});
      if (!r.success) throw std::runtime_error("CUDA executor: " + r.error_message);
      self->*member(ImplData()) = r.outputs.at(node->id());
      node->mark_evaluated();
      ++g_routed;
      return self->data();
    }
  }
  return __real__ZN7pyflame10TensorImpl11materializeEv(self);
}

PYBIND11_MODULE(_pyflame_cuda, m) {
  m.doc() = "CUDA backend for PyFlame's Python API (B200 executor)";
  // PyFlame's module as shipped cannot be imported: nn_bindings.cpp uses
  // ReduceLROnPlateau::Mode (:470) and OneCycleLR::AnnealStrategy (:491) as
  // default arguments before registering those enums (:480, :496), and
  // pybind11 rejects the conversions at import time.  Module-local
  // registrations here (same shared library, so PyFlame's module sees them)
  // let the defaults convert; PyFlame's own global registrations of the
  // enums are unaffected.  Import this module first.
  py::enum_<optim::ReduceLROnPlateau::Mode>(m, "_ReduceLROnPlateauMode", py::module_local())
      .value("MIN", optim::ReduceLROnPlateau::Mode::MIN)
      .value("MAX", optim::ReduceLROnPlateau::Mode::MAX);
  py::enum_<optim::OneCycleLR::AnnealStrategy>(m, "_AnnealStrategy", py::module_local())
      .value("COS", optim::OneCycleLR::AnnealStrategy::COS)
      .value("LINEAR", optim::OneCycleLR::AnnealStrategy::LINEAR);
  m.def("cuda_is_available", [] { return pfc_cuda_is_available() != 0; });
  m.def("cuda_device_count", [] {
    int n = 0;
    backend::cuda::check(pfc_cuda_get_device_count(&n));
    return n;
  });
  m.def("cuda_get_device", [] {
    int d = -1;
    backend::cuda::check(pfc_cuda_get_device(&d));
    return d;
  });
  m.def("cuda_set_device", [](int d) { backend::cuda::check(pfc_cuda_set_device(d)); });
  m.def("cuda_synchronize", [] { backend::cuda::check(pfc_cuda_synchronize()); });
  m.def("cuda_get_device_info", [](int d) {
    pfc_device_info i;
    backend::cuda::check(pfc_cuda_get_device_info(d, &i));
    py::dict out;
    out["device_id"] = i.device_id;
    out["name"] = std::string(i.name);
    out["architecture"] = std::string(i.architecture);
    out["total_memory"] = i.total_memory;
    out["compute_units"] = i.compute_units;
    return out;
  }, py::arg("device_id") = 0);
  m.def("set_device", [](const std::string& spec) {
    std::string d = spec;
    for (auto& c : d) c = (char)std::tolower((unsigned char)c);
    std::lock_guard<std::mutex> lk(g_mu);
    if (d == "cpu") {
      g_device = -1;
      g_ex.reset();
      return;
    }
    if (d.rfind("cuda", 0) != 0) throw py::value_error("Unknown device: " + spec + ". Valid options: 'cpu', 'cuda', 'cuda:N'");
    if (!pfc_cuda_is_available()) throw std::runtime_error("CUDA backend requested but not available");
    int dev = 0;
    if (d.size() > 4) {
      if (d[4] != ':') throw py::value_error("Invalid CUDA device specification: " + spec);
      dev = std::stoi(d.substr(5));
    }
    int n = 0;
    backend::cuda::check(pfc_cuda_get_device_count(&n));
    if (dev < 0 || dev >= n) throw py::value_error("CUDA device " + std::to_string(dev) + " requested but only " +
                                                   std::to_string(n) + " devices available");
    backend::cuda::check(pfc_cuda_set_device(dev));
    backend::cuda::Config cfg;
    cfg.device_id = dev;
    g_ex = std::make_unique<backend::cuda::CudaExecutor>(cfg);
    g_device = dev;
  }, py::arg("device"));
  m.def("get_device", [] {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_device < 0 ? std::string("cpu") : "cuda:" + std::to_string(g_device);
  });
  m.def("routed_count", [] {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_routed;
  }, "Tensors evaluated by the CUDA executor so far");
}
