// ORACLE — test infrastructure.
//
// Drop-in check of the CUDA executor behind PyFlame's own front end: graphs
// are built by PyFlame's Tensor API and nn modules (compiled from the PyFlame
// sources), handed to libpyflame_cuda.so through the PyFlame-side bridge
// (pyflame_b200/integration/pyflame_graph_bridge.hpp), and compared with the
// oracle restatement (oracle.cpp) on the same graph.  Prints one line per
// case and exits non-zero on any mismatch.  Needs an sm_100 GPU.
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "src/backend/executor.cpp"

#include "pyflame/core/tensor.hpp"
#include "pyflame/core/tensor_impl.hpp"
#include "pyflame/nn/attention.hpp"
#include "pyflame/nn/conv.hpp"
#include "pyflame/nn/linear.hpp"
#include "pyflame/nn/normalization.hpp"
#include "pyflame/nn/pooling.hpp"
#include "pyflame_b200/integration/pyflame_graph_bridge.hpp"

extern "C" {
void* orc_graph_create(void);
void orc_graph_destroy(void*);
int orc_add_node(void*, uint64_t, int, int, int, int, const int64_t*, int, const uint64_t*);
int orc_set_attr(void*, uint64_t, const char*, int, const void*, int64_t);
int orc_set_constant(void*, uint64_t, const void*, size_t);
int orc_execute(void*, const uint64_t*, int, void* const*, int);
const char* orc_last_error(void);
}

using namespace pyflame;

// The same graph in the oracle's description (ids, ops, attrs, payloads).
static std::vector<std::vector<float>> run_oracle(const ir::Graph& g, const std::vector<ir::NodeId>& ids) {
  void* o = orc_graph_create();
  for (const auto& n : g.topological_order()) {
    std::vector<uint64_t> ins;
    for (auto& i : n->inputs()) ins.push_back(i->id());
    orc_add_node(o, n->id(), (int)n->type(), (int)n->op_type(), (int)n->dtype(), n->ndim(), n->shape().data(),
                 (int)ins.size(), ins.data());
    for (const std::string& k : backend::cuda::attribute_names()) {
      if (!n->has_attr(k)) continue;
      if (n->has_attr_of_type<int>(k)) { int v = n->get_attr<int>(k); orc_set_attr(o, n->id(), k.c_str(), 0, &v, 1); }
      else if (n->has_attr_of_type<int64_t>(k)) { int64_t v = n->get_attr<int64_t>(k); orc_set_attr(o, n->id(), k.c_str(), 1, &v, 1); }
      else if (n->has_attr_of_type<float>(k)) { float v = n->get_attr<float>(k); orc_set_attr(o, n->id(), k.c_str(), 2, &v, 1); }
      else if (n->has_attr_of_type<bool>(k)) { uint8_t v = n->get_attr<bool>(k); orc_set_attr(o, n->id(), k.c_str(), 4, &v, 1); }
      else if (n->has_attr_of_type<std::vector<int64_t>>(k)) {
        auto v = n->get_attr<std::vector<int64_t>>(k);
        orc_set_attr(o, n->id(), k.c_str(), 5, v.data(), (int64_t)v.size());
      }
    }
    if (n->has_constant_data()) orc_set_constant(o, n->id(), n->constant_data().data(), n->constant_data().size());
  }
  std::vector<std::vector<float>> outs;
  std::vector<void*> ptrs;
  for (auto id : ids) outs.emplace_back(g.get_node(id)->numel());
  for (auto& v : outs) ptrs.push_back(v.data());
  if (orc_execute(o, ids.data(), (int)ids.size(), ptrs.data(), 0) != 0)
    std::fprintf(stderr, "oracle: %s\n", orc_last_error());
  orc_graph_destroy(o);
  return outs;
}

static int failures = 0;

// max |cuda - oracle| / (rms(oracle) + tiny) over each output
static void compare(const char* name, ir::Graph& g, const std::vector<ir::NodeId>& ids, double tol,
                    backend::cuda::CudaExecutor& ex) {
  auto res = ex.execute<backend::ExecutionResult>(g, ids);
  if (!res.success) {
    std::printf("FAIL %s: %s\n", name, res.error_message.c_str());
    ++failures;
    return;
  }
  auto ref = run_oracle(g, ids);
  double worst = 0;
  for (size_t k = 0; k < ids.size(); ++k) {
    if (!res.outputs.count(ids[k])) {
      std::printf("FAIL %s: output %llu missing\n", name, (unsigned long long)ids[k]);
      ++failures;
      return;
    }
    const float* got = reinterpret_cast<const float*>(res.outputs.at(ids[k]).get());
    double ss = 0;
    for (float v : ref[k]) ss += (double)v * v;
    double rms = std::sqrt(ss / std::max<size_t>(1, ref[k].size())) + 1e-30;
    for (size_t i = 0; i < ref[k].size(); ++i) worst = std::max(worst, std::fabs((double)got[i] - ref[k][i]) / rms);
  }
  bool ok = worst <= tol;
  failures += !ok;
  std::printf("%s %s: max |cuda-oracle|/rms = %.3g (tol %.1g), compute %.3f ms\n", ok ? "PASS" : "FAIL", name, worst,
              tol, res.compute_time_ms);
}

static std::vector<float> randn(size_t n, unsigned seed, float scale = 1.f) {
  std::mt19937 rng(seed);  // seeding as PyFlame's own tests do (test_rocm_kernels.cpp:74)
  std::normal_distribution<float> d(0.f, 1.f);
  std::vector<float> v(n);
  for (auto& x : v) x = d(rng) * scale;
  return v;
}

int main() {
  std::setvbuf(stdout, nullptr, _IONBF, 0);
  if (!pfc_cuda_is_available()) {
    std::printf("SKIP no sm_100 GPU\n");
    return 0;
  }
  backend::cuda::CudaExecutor ex;
  {  // fused elementwise + row reductions + LayerNorm (the headline graph, reduced rows)
    auto graph = std::make_shared<ir::Graph>();
    TensorImpl::set_current_graph(graph);
    auto xd = randn(64 * 4096, 42), yd = randn(64 * 4096, 43);
    auto x = Tensor::from_data(xd.data(), {64, 4096}, DType::Float32, MeshLayout::SinglePE(), xd.size() * 4);
    auto y = Tensor::from_data(yd.data(), {64, 4096}, DType::Float32, MeshLayout::SinglePE(), yd.size() * 4);
    auto z = sigmoid(x * y + 0.5f) - relu(x);
    nn::LayerNorm ln(4096);
    auto s = z.sum(1), m = z.mean(1), mx = z.max(1), l = ln.forward(z);
    compare("fused sigmoid(x*y+0.5)-relu(x) -> sum/mean/max/LayerNorm", *graph,
            {s.node()->id(), m.node()->id(), mx.node()->id(), l.node()->id()}, 1e-5, ex);
  }
  {  // the elementwise part on PyFlame's own CPU executor, which evaluates
     // every node of the graph, so the graph holds only ops it implements
    auto graph = std::make_shared<ir::Graph>();
    TensorImpl::set_current_graph(graph);
    auto xd = randn(64 * 4096, 42), yd = randn(64 * 4096, 43);
    auto x = Tensor::from_data(xd.data(), {64, 4096}, DType::Float32, MeshLayout::SinglePE(), xd.size() * 4);
    auto y = Tensor::from_data(yd.data(), {64, 4096}, DType::Float32, MeshLayout::SinglePE(), yd.size() * 4);
    auto z = sigmoid(x * y + 0.5f) - relu(x);
    backend::Executor cpu;
    auto rc = cpu.execute(*graph, {z.node()->id()});
    auto rg = ex.execute<backend::ExecutionResult>(*graph, {z.node()->id()});
    double worst = 0;
    bool ok = rc.success && rg.success;
    if (ok) {
      // z = sigmoid(.) - relu(x) cancels to ~0 in places, so each difference
      // is held to 1e-5 of the size of the terms plus an absolute 1e-6:
      // ratio = |a-b| / (1e-5 (|sigmoid| + |relu|) + 1e-6) must stay <= 1
      const float* a = reinterpret_cast<const float*>(rc.outputs.at(z.node()->id()).get());
      const float* b = reinterpret_cast<const float*>(rg.outputs.at(z.node()->id()).get());
      for (size_t i = 0; i < xd.size(); ++i) {
        const double terms = std::fabs(a[i] + std::max(0.0f, xd[i])) + std::max(0.0f, xd[i]);
        worst = std::max(worst, (double)std::fabs(a[i] - b[i]) / (1e-5 * terms + 1e-6));
      }
      ok = worst <= 1.0;
    }
    failures += !ok;
    std::printf("%s z vs PyFlame's CPU executor: max |diff|/(1e-5 terms + 1e-6) %.3g%s%s\n", ok ? "PASS" : "FAIL", worst,
                rc.success ? "" : " cpu: ", rc.success ? "" : rc.error_message.c_str());
  }
  {  // MLP: Linear -> ReLU -> Linear -> softmax (PyFlame's nn::Linear emits TRANSPOSE/MATMUL/ADD)
    auto graph = std::make_shared<ir::Graph>();
    TensorImpl::set_current_graph(graph);
    auto xd = randn(64 * 784, 42);
    auto x = Tensor::from_data(xd.data(), {64, 784}, DType::Float32, MeshLayout::SinglePE(), xd.size() * 4);
    nn::Linear l1(784, 256), l2(256, 10);
    auto out = softmax(l2.forward(relu(l1.forward(x))), -1);
    compare("MLP Linear-ReLU-Linear-softmax", *graph, {out.node()->id()}, 1e-4, ex);
  }
  {  // Conv2d + BatchNorm2d(eval) + ReLU + MaxPool2d
    auto graph = std::make_shared<ir::Graph>();
    TensorImpl::set_current_graph(graph);
    auto xd = randn(2 * 3 * 20 * 20, 42);
    auto x = Tensor::from_data(xd.data(), {2, 3, 20, 20}, DType::Float32, MeshLayout::SinglePE(), xd.size() * 4);
    nn::Conv2d conv(3, 8, 3, 1, 1);
    nn::BatchNorm2d bn(8);
    bn.eval();
    nn::MaxPool2d pool(2, 2);
    auto out = pool.forward(relu(bn.forward(conv.forward(x))));
    compare("Conv2d+BatchNorm2d+ReLU+MaxPool2d", *graph, {out.node()->id()}, 1e-4, ex);
  }
  {  // MultiheadAttention (batch_first), PyFlame's attention.cpp graph
    auto graph = std::make_shared<ir::Graph>();
    TensorImpl::set_current_graph(graph);
    auto xd = randn(2 * 8 * 16, 42);
    auto x = Tensor::from_data(xd.data(), {2, 8, 16}, DType::Float32, MeshLayout::SinglePE(), xd.size() * 4);
    nn::MultiheadAttention mha(16, 2, 0.0f, true, false, false, 0, 0, true);
    auto out = mha.forward(x);
    compare("MultiheadAttention", *graph, {out.node()->id()}, 1e-4, ex);
  }
  std::printf("%s (%d failures)\n", failures ? "FAILED" : "ALL PASSED", failures);
  return failures ? 1 : 0;
}
