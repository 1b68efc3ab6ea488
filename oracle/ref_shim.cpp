// ORACLE — test infrastructure, not product code.
//
// C ABI over PyFlame's own C++ code, compiled from the reference sources by
// oracle/Makefile into oracle/_ref/libpyflame_ref.so:
//   * ref_execute_cpu: builds a pyflame::ir::Graph from the flat graph
//     description and runs the reference CPU executor,
//     backend::Executor{Backend::CPU}.execute (src/backend/executor.cpp:171-524);
//   * ref_<op>: the reference's scalar kernels pyflame::ops::*_cpu
//     (src/ops/{elementwise,reduction,matmul}.cpp), which no executor calls;
//   * ref_build: graphs produced by the reference's own Tensor/nn front end
//     (src/core/tensor.cpp, src/nn/*.cpp), serialised as text so the Python
//     front end's IR can be compared node by node.
#include <any>
#include <cstdint>
#include <cstring>
#include <memory>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

// The executor class lives in a .cpp (no header): include it.
#include "src/backend/executor.cpp"

#include "pyflame/autograd/autograd.hpp"
#include "pyflame/core/tensor.hpp"
#include "pyflame/core/tensor_impl.hpp"
#include "pyflame/nn/attention.hpp"
#include "pyflame/nn/conv.hpp"
#include "pyflame/nn/linear.hpp"
#include "pyflame/nn/normalization.hpp"
#include "pyflame/nn/pooling.hpp"

// External-linkage reference kernels without a header.
namespace pyflame::ops {
void add_cpu(const float*, const float*, float*, int64_t);
void sub_cpu(const float*, const float*, float*, int64_t);
void mul_cpu(const float*, const float*, float*, int64_t);
void div_cpu(const float*, const float*, float*, int64_t);
void relu_cpu(const float*, float*, int64_t);
void sigmoid_cpu(const float*, float*, int64_t);
void tanh_cpu(const float*, float*, int64_t);
void gelu_cpu(const float*, float*, int64_t);
void silu_cpu(const float*, float*, int64_t);
void exp_cpu(const float*, float*, int64_t);
void log_cpu(const float*, float*, int64_t);
void sqrt_cpu(const float*, float*, int64_t);
void softmax_cpu(const float*, float*, int64_t, int64_t);
void log_softmax_cpu(const float*, float*, int64_t, int64_t);
void sum_dim_cpu(const float*, float*, int64_t, int64_t, int, bool);
void mean_dim_cpu(const float*, float*, int64_t, int64_t, int, bool);
void max_dim_cpu(const float*, float*, int64_t, int64_t, int, bool);
void min_dim_cpu(const float*, float*, int64_t, int64_t, int, bool);
void matmul_cpu(const float*, const float*, float*, int64_t, int64_t, int64_t);
void batch_matmul_cpu(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t);
void matmul_a_bt_cpu(const float*, const float*, float*, int64_t, int64_t, int64_t);
void transpose_2d_cpu(const float*, float*, int64_t, int64_t);
float sum_all_cpu(const float*, int64_t);
float max_all_cpu(const float*, int64_t);
}  // namespace pyflame::ops

using namespace pyflame;

namespace {

thread_local std::string g_err;

struct FlatNode {
  uint64_t id;
  int type, op, dtype;
  std::vector<int64_t> shape;
  std::vector<uint64_t> inputs;
  std::vector<std::pair<std::string, std::any>> attrs;
  std::vector<uint8_t> data;
};

struct FlatGraph {
  std::vector<FlatNode> nodes;
  std::unordered_map<uint64_t, size_t> index;
};

// Serialise one attribute value (std::any) with its C++ type name.
std::string attr_text(const std::any& a) {
  std::ostringstream o;
  if (a.type() == typeid(int)) o << "int:" << std::any_cast<int>(a);
  else if (a.type() == typeid(int64_t)) o << "int64:" << std::any_cast<int64_t>(a);
  else if (a.type() == typeid(float)) o << "float:" << std::any_cast<float>(a);
  else if (a.type() == typeid(double)) o << "double:" << std::any_cast<double>(a);
  else if (a.type() == typeid(bool)) o << "bool:" << (std::any_cast<bool>(a) ? 1 : 0);
  else if (a.type() == typeid(std::vector<int64_t>)) {
    o << "vec64:";
    for (auto v : std::any_cast<std::vector<int64_t>>(a)) o << v << ",";
  } else if (a.type() == typeid(std::vector<int>)) {
    o << "vec32:";
    for (auto v : std::any_cast<std::vector<int>>(a)) o << v << ",";
  } else o << "other:" << a.type().name();
  return o.str();
}

}  // namespace

// Attribute names a producer may set (tensor_impl.cpp, tensor.cpp, src/nn/*.cpp).
static const char* kAttrNames[] = {"dim", "keepdim", "new_shape", "dim0", "dim1", "start", "end", "stride", "padding",
                                   "dilation", "groups", "eps", "momentum", "training", "affine",
                                   "track_running_stats", "normalized_shape", "elementwise_affine", "kernel_size",
                                   "output_size", "target_shape"};

extern "C" {

const char* ref_last_error(void) { return g_err.c_str(); }

void* ref_graph_create(void) { return new FlatGraph(); }
void ref_graph_destroy(void* g) { delete (FlatGraph*)g; }

int ref_add_node(void* gp, uint64_t id, int type, int op, int dtype, int ndim, const int64_t* shape, int n_in,
                 const uint64_t* inputs) {
  auto& g = *(FlatGraph*)gp;
  FlatNode n{id, type, op, dtype, std::vector<int64_t>(shape, shape + ndim),
             std::vector<uint64_t>(inputs, inputs + n_in), {}, {}};
  g.index[id] = g.nodes.size();
  g.nodes.push_back(std::move(n));
  return 0;
}

int ref_set_attr(void* gp, uint64_t id, const char* key, int type, const void* v, int64_t count) {
  auto& g = *(FlatGraph*)gp;
  auto& n = g.nodes.at(g.index.at(id));
  std::any a;
  switch (type) {
    case 0: a = *(const int*)v; break;
    case 1: a = *(const int64_t*)v; break;
    case 2: a = *(const float*)v; break;
    case 3: a = *(const double*)v; break;
    case 4: a = (*(const uint8_t*)v) != 0; break;
    case 5: a = std::vector<int64_t>((const int64_t*)v, (const int64_t*)v + count); break;
    case 6: a = std::vector<int>((const int*)v, (const int*)v + count); break;
    default: g_err = "bad attr type"; return -1;
  }
  n.attrs.push_back({key, a});
  return 0;
}

int ref_set_constant(void* gp, uint64_t id, const void* data, size_t bytes) {
  auto& g = *(FlatGraph*)gp;
  auto& n = g.nodes.at(g.index.at(id));
  n.data.assign((const uint8_t*)data, (const uint8_t*)data + bytes);
  return 0;
}

// Run backend::Executor{Backend::CPU} on the graph.  Nodes are created in
// the order given (inputs first).  Returns 0 and fills outs, or -1 with the
// executor's error message.
int ref_execute_cpu(void* gp, const uint64_t* ids, int n_out, void* const* outs) {
  try {
    auto& fg = *(FlatGraph*)gp;
    ir::Graph graph;
    std::unordered_map<uint64_t, std::shared_ptr<ir::Node>> map;
    for (const FlatNode& n : fg.nodes) {
      ir::TensorSpec spec(n.shape, (DType)n.dtype);
      std::shared_ptr<ir::Node> node;
      if (n.type == 0) node = graph.create_constant(spec, n.data.empty() ? nullptr : n.data.data());
      else if (n.type == 1) node = graph.create_input(spec);
      else if (n.type == 2) node = graph.create_parameter(spec);
      else {
        std::vector<std::shared_ptr<ir::Node>> ins;
        for (uint64_t i : n.inputs) ins.push_back(map.at(i));
        node = graph.create_op((ir::OpType)n.op, ins, spec);
      }
      if (n.type == 1 || n.type == 2)
        if (!n.data.empty()) node->set_constant_data(n.data);
      for (auto& [k, a] : n.attrs) node->set_attr(k, a);
      map[n.id] = node;
    }
    std::vector<ir::NodeId> rid;
    for (int i = 0; i < n_out; ++i) rid.push_back(map.at(ids[i])->id());
    backend::Executor ex(backend::ExecutorConfig{backend::Backend::CPU});
    auto res = ex.execute(graph, rid);
    if (!res.success) {
      g_err = res.error_message;
      return -1;
    }
    for (int i = 0; i < n_out; ++i) {
      auto it = res.outputs.find(rid[i]);
      if (it == res.outputs.end()) {
        g_err = "output missing";
        return -1;
      }
      std::memcpy(outs[i], it->second.get(), map.at(ids[i])->output_spec().size_bytes());
    }
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

// ---- the reference's scalar kernels ----------------------------------------
void ref_unary(int which, const float* x, float* out, int64_t n) {
  switch (which) {
    case 0: ops::relu_cpu(x, out, n); break;
    case 1: ops::sigmoid_cpu(x, out, n); break;
    case 2: ops::tanh_cpu(x, out, n); break;
    case 3: ops::gelu_cpu(x, out, n); break;
    case 4: ops::silu_cpu(x, out, n); break;
    case 5: ops::exp_cpu(x, out, n); break;
    case 6: ops::log_cpu(x, out, n); break;
    case 7: ops::sqrt_cpu(x, out, n); break;
  }
}
void ref_binary(int which, const float* a, const float* b, float* out, int64_t n) {
  switch (which) {
    case 0: ops::add_cpu(a, b, out, n); break;
    case 1: ops::sub_cpu(a, b, out, n); break;
    case 2: ops::mul_cpu(a, b, out, n); break;
    case 3: ops::div_cpu(a, b, out, n); break;
  }
}
void ref_softmax(const float* x, float* out, int64_t batch, int64_t dim) { ops::softmax_cpu(x, out, batch, dim); }
void ref_log_softmax(const float* x, float* out, int64_t batch, int64_t dim) {
  ops::log_softmax_cpu(x, out, batch, dim);
}
void ref_reduce_dim(int which, const float* x, float* out, int64_t d0, int64_t d1, int rd) {
  switch (which) {
    case 0: ops::sum_dim_cpu(x, out, d0, d1, rd, false); break;
    case 1: ops::mean_dim_cpu(x, out, d0, d1, rd, false); break;
    case 2: ops::max_dim_cpu(x, out, d0, d1, rd, false); break;
    case 3: ops::min_dim_cpu(x, out, d0, d1, rd, false); break;
  }
}
void ref_matmul(const float* a, const float* b, float* c, int64_t M, int64_t K, int64_t N) {
  ops::matmul_cpu(a, b, c, M, K, N);
}
void ref_batch_matmul(const float* a, const float* b, float* c, int64_t B, int64_t M, int64_t K, int64_t N) {
  ops::batch_matmul_cpu(a, b, c, B, M, K, N);
}
void ref_matmul_a_bt(const float* a, const float* b, float* c, int64_t M, int64_t K, int64_t N) {
  ops::matmul_a_bt_cpu(a, b, c, M, K, N);
}

// ---- graphs from the reference's own front end --------------------------------
// kind: 0 Linear(in=8,out=4) on [2,8]; 1 Conv2d(3,4,k3,s2,p1)+BatchNorm2d+ReLU+MaxPool2d(3,2)
// on [2,3,9,9]; 2 LayerNorm([8]) on [2,8] and softmax(dim=-1); 3 MultiheadAttention(8,2,batch_first)
// on [2,5,8]; 4 x*y+0.5 then sum(1), mean(1), max(1); 5 AdaptiveAvgPool2d(1) + AvgPool2d(2)
// Writes one line per node: id|type|op|shape|inputs|attrs.
int ref_build(int kind, char* buf, size_t len) {
  try {
    auto graph = std::make_shared<ir::Graph>();
    TensorImpl::set_current_graph(graph);
    std::vector<float> d(2 * 5 * 8 * 9 * 9, 0.25f);
    Tensor out;
    if (kind == 0) {
      auto x = Tensor::from_data(d.data(), {2, 8}, DType::Float32, MeshLayout::SinglePE(), 2 * 8 * 4);
      nn::Linear lin(8, 4);
      out = lin.forward(x);
    } else if (kind == 1) {
      auto x = Tensor::from_data(d.data(), {2, 3, 9, 9}, DType::Float32, MeshLayout::SinglePE(), 2 * 3 * 81 * 4);
      nn::Conv2d conv(3, 4, 3, 2, 1);
      nn::BatchNorm2d bn(4);
      bn.eval();
      nn::MaxPool2d pool(3, 2);
      out = pool.forward(relu(bn.forward(conv.forward(x))));
    } else if (kind == 2) {
      auto x = Tensor::from_data(d.data(), {2, 8}, DType::Float32, MeshLayout::SinglePE(), 2 * 8 * 4);
      nn::LayerNorm ln(8);
      out = softmax(ln.forward(x), -1);
    } else if (kind == 3) {
      auto x = Tensor::from_data(d.data(), {2, 5, 8}, DType::Float32, MeshLayout::SinglePE(), 2 * 5 * 8 * 4);
      nn::MultiheadAttention mha(8, 2, 0.0f, true, false, false, 0, 0, true);
      out = mha.forward(x);
    } else if (kind == 4) {
      auto x = Tensor::from_data(d.data(), {4, 8}, DType::Float32, MeshLayout::SinglePE(), 4 * 8 * 4);
      auto y = Tensor::from_data(d.data(), {4, 8}, DType::Float32, MeshLayout::SinglePE(), 4 * 8 * 4);
      auto z = sigmoid(x * y + 0.5f) - relu(x);
      auto s = z.sum(1);
      auto m = z.mean(1);
      out = z.max(1);
    } else if (kind == 5) {
      auto x = Tensor::from_data(d.data(), {2, 3, 8, 8}, DType::Float32, MeshLayout::SinglePE(), 2 * 3 * 64 * 4);
      nn::AvgPool2d ap(2);
      nn::AdaptiveAvgPool2d gp(1);
      out = gp.forward(ap.forward(x));
    } else if (kind == 6) {
      // backward graph of an MLP loss (autograd.cpp:421-480)
      auto x = Tensor::from_data(d.data(), {4, 8}, DType::Float32, MeshLayout::SinglePE(), 4 * 8 * 4);
      nn::Linear l1(8, 6), l2(6, 3);
      auto loss = softmax(l2.forward(relu(l1.forward(x))), -1).sum();
      autograd::AutogradEngine::backward(loss.node(), nullptr, graph);
      out = loss;
    } else if (kind == 7) {
      // backward graph of an elementwise chain with a broadcast bias and row reductions
      auto x = Tensor::from_data(d.data(), {4, 8}, DType::Float32, MeshLayout::SinglePE(), 4 * 8 * 4);
      auto y = Tensor::from_data(d.data(), {4, 8}, DType::Float32, MeshLayout::SinglePE(), 4 * 8 * 4);
      auto b = Tensor::from_data(d.data(), {8}, DType::Float32, MeshLayout::SinglePE(), 8 * 4);
      auto a = x * y + b;
      auto h = tanh(a) * sigmoid(x) - exp(y) / (abs(x) + 1.0f);
      auto z = sqrt(h * h + 1.0f).sum(1, true);
      auto loss = (log(z) + sin(x).sum(1, true) * cos(y).mean(1, true)).sum();
      autograd::AutogradEngine::backward(loss.node(), nullptr, graph);
      out = loss;
    } else {
      g_err = "unknown kind";
      return -1;
    }
    std::ostringstream o;
    for (const auto& n : graph->all_nodes()) {
      o << n->id() << "|" << (int)n->type() << "|" << (int)n->op_type() << "|";
      for (auto s : n->shape()) o << s << ",";
      o << "|";
      for (auto& i : n->inputs()) o << i->id() << ",";
      o << "|";
      for (const char* k : kAttrNames)
        if (n->has_attr(k)) {
          // the attribute map is private; find the stored type with
          // Node::has_attr_of_type (node.hpp:154-161), then read it back
          const ir::Node& cn = *n;
          std::any a;
          bool found = true;
          if (cn.has_attr_of_type<int>(k)) a = cn.get_attr<int>(k);
          else if (cn.has_attr_of_type<int64_t>(k)) a = cn.get_attr<int64_t>(k);
          else if (cn.has_attr_of_type<float>(k)) a = cn.get_attr<float>(k);
          else if (cn.has_attr_of_type<double>(k)) a = cn.get_attr<double>(k);
          else if (cn.has_attr_of_type<bool>(k)) a = cn.get_attr<bool>(k);
          else if (cn.has_attr_of_type<std::vector<int64_t>>(k)) a = cn.get_attr<std::vector<int64_t>>(k);
          else if (cn.has_attr_of_type<std::vector<int>>(k)) a = cn.get_attr<std::vector<int>>(k);
          else found = false;
          o << k << "=" << (found ? attr_text(a) : std::string("?")) << ";";
        }
      o << "\n";
    }
    (void)out;
    std::string s = o.str();
    std::snprintf(buf, len, "%s", s.c_str());
    TensorImpl::set_current_graph(std::make_shared<ir::Graph>());
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

}  // extern "C"
