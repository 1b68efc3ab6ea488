#include "graph.hpp"

#include <algorithm>
#include <cstring>
#include <functional>

namespace pfb {

const char* op_name(Op op) {
  switch (op) {
    case Op::ADD: return "add"; case Op::SUB: return "sub"; case Op::MUL: return "mul";
    case Op::DIV: return "div"; case Op::POW: return "pow"; case Op::MAX_BINARY: return "max";
    case Op::MIN_BINARY: return "min"; case Op::NEG: return "neg"; case Op::ABS: return "abs";
    case Op::SQRT: return "sqrt"; case Op::EXP: return "exp"; case Op::LOG: return "log";
    case Op::SIN: return "sin"; case Op::COS: return "cos"; case Op::TANH: return "tanh";
    case Op::RELU: return "relu"; case Op::SIGMOID: return "sigmoid"; case Op::GELU: return "gelu";
    case Op::SILU: return "silu"; case Op::SOFTMAX: return "softmax";
    case Op::LOG_SOFTMAX: return "log_softmax"; case Op::SUM: return "sum";
    case Op::MEAN: return "mean"; case Op::MAX: return "max"; case Op::MIN: return "min";
    case Op::PROD: return "prod"; case Op::MATMUL: return "matmul";
    case Op::TRANSPOSE: return "transpose"; case Op::BATCH_MATMUL: return "batch_matmul";
    case Op::CONV2D: return "conv2d"; case Op::MAX_POOL2D: return "max_pool2d";
    case Op::AVG_POOL2D: return "avg_pool2d"; case Op::ADAPTIVE_AVG_POOL2D: return "adaptive_avg_pool2d";
    case Op::BATCH_NORM: return "batch_norm"; case Op::LAYER_NORM: return "layer_norm";
    case Op::DROPOUT: return "dropout"; case Op::RESHAPE: return "reshape"; case Op::VIEW: return "view";
    case Op::SQUEEZE: return "squeeze"; case Op::UNSQUEEZE: return "unsqueeze";
    case Op::SLICE: return "slice"; case Op::CONCAT: return "concat"; case Op::STACK: return "stack";
    case Op::BROADCAST: return "broadcast"; case Op::COPY: return "copy";
    case Op::CONTIGUOUS: return "contiguous"; case Op::EQ: return "eq"; case Op::NE: return "ne";
    case Op::LT: return "lt"; case Op::LE: return "le"; case Op::GT: return "gt"; case Op::GE: return "ge";
    case Op::LESS: return "less"; case Op::WHERE: return "where"; case Op::MAXIMUM: return "maximum";
    case Op::MINIMUM: return "minimum"; case Op::CLAMP: return "clamp";
    case Op::CONSTANT: return "constant"; case Op::INPUT: return "input";
    case Op::PARAMETER: return "parameter";
    default: return "unknown";
  }
}

bool op_is_elementwise(Op op) {
  uint16_t v = (uint16_t)op;
  if (op == Op::SOFTMAX || op == Op::LOG_SOFTMAX) return false;
  return (v >= 100 && v < 400) || (v >= 800 && v < 900) ;
}

size_t dtype_size(DType d) {
  switch (d) {
    case DType::F32: return 4; case DType::F16: return 2; case DType::BF16: return 2;
    case DType::I32: return 4; case DType::I16: return 2; case DType::I8: return 1;
    case DType::BOOL: return 1; case DType::F64: return 8; case DType::I64: return 8;
  }
  fail(PFC_ERR_INVALID_ARGUMENT, "unknown dtype");
}

const char* dtype_name(DType d) {
  switch (d) {
    case DType::F32: return "float32"; case DType::F16: return "float16";
    case DType::BF16: return "bfloat16"; case DType::I32: return "int32";
    case DType::I16: return "int16"; case DType::I8: return "int8"; case DType::BOOL: return "bool";
    case DType::F64: return "float64"; case DType::I64: return "int64";
  }
  return "unknown";
}

int64_t Node::numel() const {
  int64_t n = 1;
  for (int64_t d : shape) {
    if (d < 0) fail(PFC_ERR_INVALID_ARGUMENT, "negative dimension in node " + std::to_string(id));
    if (d != 0 && n > (int64_t(1) << 62) / d) fail(PFC_ERR_INVALID_ARGUMENT, "numel overflow");
    n *= d;
  }
  return n;
}

static bool attr_is_int(int t) { return t == PFC_ATTR_INT32 || t == PFC_ATTR_INT64 || t == PFC_ATTR_BOOL; }
static bool attr_is_float(int t) { return t == PFC_ATTR_FLOAT32 || t == PFC_ATTR_FLOAT64; }

int64_t Node::attr_int(const std::string& k) const {
  auto it = attrs.find(k);
  if (it == attrs.end()) fail(PFC_ERR_GRAPH, "Attribute not found: " + k + " on node " + std::to_string(id));
  if (!attr_is_int(it->second.type) || it->second.i.empty())
    fail(PFC_ERR_GRAPH, "Type mismatch for attribute '" + k + "' on node " + std::to_string(id));
  return it->second.i[0];
}
int64_t Node::attr_int(const std::string& k, int64_t dflt) const {
  return has_attr(k) ? attr_int(k) : dflt;
}
double Node::attr_float(const std::string& k, double dflt) const {
  auto it = attrs.find(k);
  if (it == attrs.end()) return dflt;
  if (attr_is_float(it->second.type) && !it->second.f.empty()) return it->second.f[0];
  if (attr_is_int(it->second.type) && !it->second.i.empty()) return (double)it->second.i[0];
  fail(PFC_ERR_GRAPH, "Type mismatch for attribute '" + k + "'");
}
bool Node::attr_bool(const std::string& k, bool dflt) const {
  auto it = attrs.find(k);
  if (it == attrs.end()) return dflt;
  if (!attr_is_int(it->second.type) || it->second.i.empty())
    fail(PFC_ERR_GRAPH, "Type mismatch for attribute '" + k + "'");
  return it->second.i[0] != 0;
}
std::vector<int64_t> Node::attr_ints(const std::string& k) const {
  auto it = attrs.find(k);
  if (it == attrs.end()) fail(PFC_ERR_GRAPH, "Attribute not found: " + k + " on node " + std::to_string(id));
  const Attr& a = it->second;
  if (a.type == PFC_ATTR_INT64_VEC || a.type == PFC_ATTR_INT32_VEC || attr_is_int(a.type)) return a.i;
  fail(PFC_ERR_GRAPH, "Type mismatch for attribute '" + k + "'");
}
std::vector<int64_t> Node::attr_ints(const std::string& k, const std::vector<int64_t>& dflt) const {
  return has_attr(k) ? attr_ints(k) : dflt;
}

Node* Graph::find(uint64_t id) {
  auto it = index.find(id);
  return it == index.end() ? nullptr : &nodes[it->second];
}
const Node* Graph::find(uint64_t id) const {
  auto it = index.find(id);
  return it == index.end() ? nullptr : &nodes[it->second];
}
const Node& Graph::at(uint64_t id) const {
  const Node* n = find(id);
  if (!n) fail(PFC_ERR_GRAPH, "Input not found: " + std::to_string(id));
  return *n;
}

// Same limits as executor.cpp:59-60.
static constexpr size_t kMaxGraphNodes = 1000000;
static constexpr size_t kMaxGraphEdges = 10000000;

void validate_graph(const Graph& g) {
  if (g.nodes.size() > kMaxGraphNodes)
    fail(PFC_ERR_GRAPH, "Graph too large: " + std::to_string(g.nodes.size()) +
                            " nodes exceeds maximum of " + std::to_string(kMaxGraphNodes));
  size_t edges = 0;
  for (const Node& n : g.nodes) edges += n.inputs.size();
  if (edges > kMaxGraphEdges)
    fail(PFC_ERR_GRAPH, "Graph too complex: " + std::to_string(edges) + " edges exceeds maximum of " +
                            std::to_string(kMaxGraphEdges));
  // Iterative three-colour DFS: 0 unvisited, 1 on stack, 2 done.
  std::vector<uint8_t> state(g.nodes.size(), 0);
  std::vector<std::pair<size_t, size_t>> stack;
  for (size_t root = 0; root < g.nodes.size(); ++root) {
    if (state[root]) continue;
    stack.push_back({root, 0});
    state[root] = 1;
    while (!stack.empty()) {
      auto& [idx, next] = stack.back();
      const Node& n = g.nodes[idx];
      if (next < n.inputs.size()) {
        uint64_t in = n.inputs[next++];
        auto it = g.index.find(in);
        if (it == g.index.end())
          fail(PFC_ERR_GRAPH, "Node " + std::to_string(n.id) + " references missing input " + std::to_string(in));
        size_t j = it->second;
        if (state[j] == 1)
          fail(PFC_ERR_GRAPH, "Graph validation failed: cycle detected involving node " + std::to_string(in));
        if (state[j] == 0) {
          state[j] = 1;
          stack.push_back({j, 0});
        }
      } else {
        state[idx] = 2;
        stack.pop_back();
      }
    }
  }
}

std::vector<uint64_t> topo_order(const Graph& g, const std::vector<uint64_t>& outputs) {
  std::vector<uint64_t> order;
  std::vector<uint8_t> seen(g.nodes.size(), 0);
  std::vector<std::pair<size_t, size_t>> stack;
  for (uint64_t out : outputs) {
    auto it = g.index.find(out);
    if (it == g.index.end()) fail(PFC_ERR_INVALID_ARGUMENT, "output id not in graph: " + std::to_string(out));
    if (seen[it->second]) continue;
    seen[it->second] = 1;
    stack.push_back({it->second, 0});
    while (!stack.empty()) {
      auto& [idx, next] = stack.back();
      const Node& n = g.nodes[idx];
      if (next < n.inputs.size()) {
        size_t j = g.index.at(n.inputs[next++]);
        if (!seen[j]) {
          seen[j] = 1;
          stack.push_back({j, 0});
        }
      } else {
        order.push_back(n.id);
        stack.pop_back();
      }
    }
  }
  return order;
}

static inline uint64_t mix(uint64_t h, uint64_t v) {
  h ^= v + 0x9e3779b97f4a7c15ULL + (h << 6) + (h >> 2);
  return h * 0xff51afd7ed558ccdULL;
}

uint64_t structural_hash(const Graph& g, const std::vector<uint64_t>& outputs) {
  uint64_t h = 0x12345678abcdefULL;
  for (uint64_t id : outputs) h = mix(h, id);
  for (const Node& n : g.nodes) {
    h = mix(h, n.id);
    h = mix(h, (uint64_t)n.type);
    h = mix(h, (uint64_t)n.op);
    h = mix(h, (uint64_t)n.dtype);
    for (int64_t d : n.shape) h = mix(h, (uint64_t)d);
    h = mix(h, 0xfeed);
    for (uint64_t i : n.inputs) h = mix(h, i);
    for (const auto& [k, a] : n.attrs) {
      for (char c : k) h = mix(h, (uint64_t)c);
      h = mix(h, (uint64_t)a.type);
      for (int64_t v : a.i) h = mix(h, (uint64_t)v);
      for (double v : a.f) {
        uint64_t b;
        std::memcpy(&b, &v, 8);
        h = mix(h, b);
      }
    }
    h = mix(h, n.has_data() ? 1 : 0);
    if (n.data_flags & PFC_CONST_RESIDENT) {
      h = mix(h, n.data_key);
      h = mix(h, (uint64_t)n.data_bytes);
    }
  }
  return h;
}

}  // namespace pfb
