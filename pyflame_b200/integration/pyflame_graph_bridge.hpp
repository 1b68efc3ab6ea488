// pyflame_graph_bridge.hpp — PyFlame-side adapter for libpyflame_cuda.so.
//
// Header-only, compiled inside the PyFlame tree (it includes PyFlame's IR
// headers).  It turns a live pyflame::ir::Graph into the C ABI's graph
// description and runs it through the CUDA executor, filling the fields of
// PyFlame's ExecutionResult (src/backend/executor.cpp:148-160).  A
// Backend::CUDA branch of backend::Executor (executor.cpp:171-194) holds a
// cuda::CudaExecutor (below) and calls its execute() where execute_rocm
// (executor.cpp:557-582) calls rocm::ROCmExecutor::execute.
#pragma once

#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "pyflame/core/allocator.hpp"
#include "pyflame/ir/graph.hpp"
#include "pyflame_cuda.h"

namespace pyflame::backend::cuda {

// Attribute names PyFlame's producers write (tensor_impl.cpp:530-533,577-578,
// tensor.cpp:281-283,687,828, conv.cpp:114-117, normalization.cpp:85-89,246-248,
// pooling.cpp:57-59,163-164).
inline const std::vector<std::string>& attribute_names() {
  static const std::vector<std::string> names = {
      "dim", "keepdim", "new_shape", "dim0", "dim1", "start", "end", "stride", "padding", "dilation",
      "groups", "eps", "momentum", "training", "affine", "track_running_stats", "normalized_shape",
      "elementwise_affine", "kernel_size", "output_size"};
  return names;
}

inline void check(int rc) {
  if (rc != PFC_OK) throw std::runtime_error(pfc_last_error());
}

// Cache keys for constant payloads kept on the device across calls.  PyFlame
// node ids restart at 0 in every graph and a freed payload's address is
// reused by later allocations, so neither names a payload on its own.  A key
// here is issued per live node object (tracked through a weak_ptr) and
// payload (address, size, and a fingerprint of 64 sampled words): when the
// node dies or its payload is replaced (Node::set_constant_data,
// node.hpp:175-177), the next lookup issues a fresh key.
class PayloadKeys {
 public:
  uint64_t key(const std::shared_ptr<ir::Node>& n) {
    const auto& d = n->constant_data();
    const uint64_t fp = fingerprint(d.data(), d.size());
    auto it = keys_.find(n.get());
    if (it != keys_.end()) {
      const Entry& e = it->second;
      if (!e.node.expired() && e.node.lock() == n && e.data == d.data() && e.bytes == d.size() && e.fp == fp)
        return e.key;
    }
    if (keys_.size() > 4096) prune();
    Entry e{n, d.data(), d.size(), fp, next_++};
    keys_[n.get()] = e;
    return e.key;
  }

 private:
  struct Entry {
    std::weak_ptr<ir::Node> node;
    const void* data;
    size_t bytes;
    uint64_t fp;
    uint64_t key;
  };
  std::unordered_map<const ir::Node*, Entry> keys_;
  uint64_t next_ = 1;

  static uint64_t fingerprint(const uint8_t* p, size_t n) {
    uint64_t h = 1469598103934665603ull ^ n;
    const size_t words = n / 8;
    for (size_t i = 0; i < 64 && words; ++i) {
      uint64_t w;
      std::memcpy(&w, p + 8 * ((i * words) / 64), 8);
      h = (h ^ w) * 1099511628211ull;
    }
    return h;
  }
  void prune() {
    for (auto it = keys_.begin(); it != keys_.end();)
      it = it->second.node.expired() ? keys_.erase(it) : std::next(it);
  }
};

// Owns a pfc_graph holding every node of `graph` (ids, types, ops, specs,
// edges, typed attributes, constant payloads borrowed from the nodes).
class GraphBridge {
 public:
  GraphBridge(const ir::Graph& graph, PayloadKeys& keys) {
    check(pfc_graph_create(&g_));
    for (const auto& n : graph.topological_order()) add(n, keys);
  }
  ~GraphBridge() { pfc_graph_destroy(g_); }
  GraphBridge(const GraphBridge&) = delete;
  GraphBridge& operator=(const GraphBridge&) = delete;
  pfc_graph* get() const { return g_; }

 private:
  pfc_graph* g_ = nullptr;

  void add(const std::shared_ptr<ir::Node>& np, PayloadKeys& keys) {
    const ir::Node& n = *np;
    std::vector<uint64_t> ins;
    for (const auto& i : n.inputs()) ins.push_back(i->id());
    const auto& shape = n.shape();
    check(pfc_graph_add_node(g_, n.id(), (int)n.type(), (int)n.op_type(), (int)n.dtype(), (int)shape.size(),
                             shape.data(), (int)ins.size(), ins.data()));
    for (const std::string& k : attribute_names()) {
      if (!n.has_attr(k)) continue;
      if (n.has_attr_of_type<int>(k)) {
        int v = n.get_attr<int>(k);
        check(pfc_graph_set_attr(g_, n.id(), k.c_str(), PFC_ATTR_INT32, &v, 1));
      } else if (n.has_attr_of_type<int64_t>(k)) {
        int64_t v = n.get_attr<int64_t>(k);
        check(pfc_graph_set_attr(g_, n.id(), k.c_str(), PFC_ATTR_INT64, &v, 1));
      } else if (n.has_attr_of_type<float>(k)) {
        float v = n.get_attr<float>(k);
        check(pfc_graph_set_attr(g_, n.id(), k.c_str(), PFC_ATTR_FLOAT32, &v, 1));
      } else if (n.has_attr_of_type<double>(k)) {
        double v = n.get_attr<double>(k);
        check(pfc_graph_set_attr(g_, n.id(), k.c_str(), PFC_ATTR_FLOAT64, &v, 1));
      } else if (n.has_attr_of_type<bool>(k)) {
        uint8_t v = n.get_attr<bool>(k) ? 1 : 0;
        check(pfc_graph_set_attr(g_, n.id(), k.c_str(), PFC_ATTR_BOOL, &v, 1));
      } else if (n.has_attr_of_type<std::vector<int64_t>>(k)) {
        auto v = n.get_attr<std::vector<int64_t>>(k);
        check(pfc_graph_set_attr(g_, n.id(), k.c_str(), PFC_ATTR_INT64_VEC, v.data(), (int64_t)v.size()));
      } else if (n.has_attr_of_type<std::vector<int>>(k)) {
        auto v = n.get_attr<std::vector<int>>(k);
        check(pfc_graph_set_attr(g_, n.id(), k.c_str(), PFC_ATTR_INT32_VEC, v.data(), (int64_t)v.size()));
      }
    }
    if (n.has_constant_data()) {
      const auto& d = n.constant_data();
      // CONSTANT and PARAMETER payloads stay on the device across calls; an
      // INPUT node's payload is runtime data (node.hpp:24), uploaded per call
      const bool resident = !n.is_input();
      check(pfc_graph_set_constant(g_, n.id(), d.data(), d.size(), resident ? (uint32_t)PFC_CONST_RESIDENT : 0u,
                                   resident ? keys.key(np) : 0));
    }
  }
};

struct Config {
  int device_id = 0;
  bool enable_profiling = false;
  bool sync_after_launch = false;
  size_t workspace_size_mb = 256;
  int precision = PFC_PRECISION_TF32X3;
  bool use_cuda_graph = true;
};

// Shaped like rocm::ROCmExecutor (rocm_executor.hpp:37-194).  `Result` is
// PyFlame's ExecutionResult (defined in executor.cpp, so passed as a template
// parameter here).
class CudaExecutor {
 public:
  explicit CudaExecutor(const Config& c = Config()) {
    pfc_executor_config cfg;
    pfc_executor_config_default(&cfg);
    cfg.device_id = c.device_id;
    cfg.enable_profiling = c.enable_profiling;
    cfg.sync_after_launch = c.sync_after_launch;
    cfg.workspace_size_mb = c.workspace_size_mb;
    cfg.precision = c.precision;
    cfg.use_cuda_graph = c.use_cuda_graph;
    check(pfc_executor_create(&cfg, &ex_));
  }
  ~CudaExecutor() { pfc_executor_destroy(ex_); }
  CudaExecutor(const CudaExecutor&) = delete;
  CudaExecutor& operator=(const CudaExecutor&) = delete;

  template <class Result>
  Result execute(ir::Graph& graph, const std::vector<ir::NodeId>& output_ids) {
    Result result;
    try {
      GraphBridge bridge(graph, keys_);
      std::vector<uint64_t> ids;
      std::vector<void*> ptrs;
      std::vector<size_t> sizes;
      for (auto id : output_ids) {
        auto node = graph.get_node(id);
        if (!node) continue;  // only ids present in the graph are returned
        size_t bytes = node->output_spec().size_bytes();
        auto buf = std::shared_ptr<uint8_t>(static_cast<uint8_t*>(Allocator::allocate(bytes)),
                                            [](uint8_t* p) { Allocator::deallocate(p); });
        ids.push_back(id);
        ptrs.push_back(buf.get());
        sizes.push_back(bytes);
        result.outputs[id] = buf;
      }
      pfc_execution_result r;
      int rc = pfc_executor_execute(ex_, bridge.get(), ids.data(), (int)ids.size(), ptrs.data(), sizes.data(), &r);
      result.success = rc == PFC_OK;
      result.error_message = rc == PFC_OK ? "" : r.error_message;
      result.compile_time_ms = r.compile_time_ms;
      result.transfer_time_ms = r.transfer_time_ms;
      result.compute_time_ms = r.compute_time_ms;
      result.total_time_ms = r.total_time_ms;
      if (!result.success) result.outputs.clear();
    } catch (const std::exception& e) {
      result.success = false;
      result.error_message = e.what();
      result.outputs.clear();
    }
    return result;
  }

  pfc_memory_stats get_memory_stats() const {
    pfc_memory_stats s;
    check(pfc_executor_get_memory_stats(ex_, &s));
    return s;
  }

 private:
  pfc_executor* ex_ = nullptr;
  PayloadKeys keys_;
};

}  // namespace pyflame::backend::cuda
