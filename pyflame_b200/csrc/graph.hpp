// Graph description held by the executor: the nodes of one PyFlame ir::Graph
// (include/pyflame/ir/graph.hpp:17-215) in a flat, pointer-free form.
#pragma once

#include <atomic>
#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.hpp"

namespace pfb {

// PyFlame OpType values (include/pyflame/ir/op_type.hpp:9-124).  The numeric
// codes are the interface, so they are kept identical.
enum class Op : uint16_t {
  NONE = 0,
  ADD = 100, SUB = 101, MUL = 102, DIV = 103, POW = 104, MAX_BINARY = 105, MIN_BINARY = 106,
  NEG = 200, ABS = 201, SQRT = 202, EXP = 203, LOG = 204, SIN = 205, COS = 206, TANH = 207,
  RELU = 300, SIGMOID = 301, GELU = 302, SILU = 303, SOFTMAX = 304, LOG_SOFTMAX = 305,
  SUM = 400, MEAN = 401, MAX = 402, MIN = 403, PROD = 404,
  MATMUL = 500, TRANSPOSE = 501, BATCH_MATMUL = 502,
  CONV1D = 510, CONV2D = 511, CONV3D = 512, CONV_TRANSPOSE2D = 513,
  MAX_POOL1D = 520, MAX_POOL2D = 521, MAX_POOL3D = 522, AVG_POOL1D = 523, AVG_POOL2D = 524,
  AVG_POOL3D = 525, ADAPTIVE_AVG_POOL2D = 526, ADAPTIVE_AVG_POOL1D = 527,
  BATCH_NORM = 530, LAYER_NORM = 531, GROUP_NORM = 532, INSTANCE_NORM = 533,
  DROPOUT = 540, EMBEDDING = 545, GATHER = 546,
  RESHAPE = 600, VIEW = 601, SQUEEZE = 602, UNSQUEEZE = 603, SLICE = 604, CONCAT = 605,
  STACK = 606, BROADCAST = 607,
  COPY = 700, CONTIGUOUS = 701, LAYOUT_TRANSFORM = 702,
  EQ = 800, NE = 801, LT = 802, LE = 803, GT = 804, GE = 805, LESS = 806,
  WHERE = 810, MAXIMUM = 811, MINIMUM = 812, CLAMP = 813,
  CONSTANT = 900, INPUT = 901, PARAMETER = 902,
};

const char* op_name(Op op);
// Elementwise per op_type.hpp:216-219 (binary, unary, activations, comparisons,
// conditionals), minus SOFTMAX/LOG_SOFTMAX which are row operations here.
bool op_is_elementwise(Op op);

enum class NodeType : uint8_t { CONSTANT = 0, INPUT = 1, PARAMETER = 2, OPERATION = 3 };

enum class DType : uint8_t {
  F32 = 0, F16 = 1, BF16 = 2, I32 = 3, I16 = 4, I8 = 5, BOOL = 6, F64 = 7, I64 = 8,
};
size_t dtype_size(DType d);
const char* dtype_name(DType d);

struct Attr {
  int type = 0;  // pfc_attr_type
  std::vector<int64_t> i;  // integer and bool payloads
  std::vector<double> f;   // floating payloads
};

struct Node {
  uint64_t id = 0;
  NodeType type = NodeType::OPERATION;
  Op op = Op::NONE;
  DType dtype = DType::F32;
  std::vector<int64_t> shape;
  std::vector<uint64_t> inputs;
  std::map<std::string, Attr> attrs;
  // Constant payload: borrowed pointer or an owned copy.
  const void* data = nullptr;
  size_t data_bytes = 0;
  uint32_t data_flags = 0;
  uint64_t data_key = 0;  // cache key of a resident payload
  std::vector<uint8_t> owned;

  int64_t numel() const;
  size_t size_bytes() const { return (size_t)numel() * dtype_size(dtype); }
  bool has_data() const { return data != nullptr && data_bytes > 0; }

  bool has_attr(const std::string& k) const { return attrs.count(k) != 0; }
  // Typed readers that accept the integer/float widths PyFlame producers use
  // and fail loudly (like Node::get_attr, node.hpp:123-136) on a kind mismatch.
  int64_t attr_int(const std::string& k) const;
  int64_t attr_int(const std::string& k, int64_t dflt) const;
  double attr_float(const std::string& k, double dflt) const;
  bool attr_bool(const std::string& k, bool dflt) const;
  std::vector<int64_t> attr_ints(const std::string& k) const;
  std::vector<int64_t> attr_ints(const std::string& k, const std::vector<int64_t>& dflt) const;
};

struct Graph {
  std::vector<Node> nodes;
  std::unordered_map<uint64_t, size_t> index;
  std::vector<uint64_t> outputs;
  uint64_t version = 0;  // bumped on every mutation
  // process-unique identity (never reused, unlike the object's address)
  const uint64_t uid = next_uid();
  static uint64_t next_uid() {
    static std::atomic<uint64_t> n{1};
    return n.fetch_add(1);
  }

  Node* find(uint64_t id);
  const Node* find(uint64_t id) const;
  const Node& at(uint64_t id) const;
};

// Cycle and size checks in the manner of validate_graph (executor.cpp:58-133).
void validate_graph(const Graph& g);
// Nodes needed for `outputs`, inputs before users (graph.hpp:136-164 visit order).
std::vector<uint64_t> topo_order(const Graph& g, const std::vector<uint64_t>& outputs);
// 64-bit structural hash: ops, shapes, dtypes, edges, attributes, and constant
// identity (pointer+size for resident constants, size otherwise).
uint64_t structural_hash(const Graph& g, const std::vector<uint64_t>& outputs);

}  // namespace pfb
