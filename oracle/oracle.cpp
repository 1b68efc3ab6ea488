// ORACLE — test infrastructure, not product code.
//
// CPU restatement of PyFlame's graph evaluation for the CUDA executor's
// parity tests and the bench's CPU baseline.  Only tests/, the smoke check
// and bench.py's CPU-baseline leg use it.
//
// It evaluates the same flat graph description the executor takes (node ids,
// PyFlame OpType codes, shapes, typed attributes, constant payloads) with
// sequential loops in PyFlame's arithmetic order.  Instantiated for float
// (the reference's fp32 arithmetic) and double (an fp64 shadow used to judge
// conditioning).  Built with -ffp-contract=off so float expressions round
// like the reference build (no fused multiply-add).
//
// Each op cites the PyFlame code it follows.  Ops PyFlame has no CPU code for
// (CONV2D, BATCH_NORM, LAYER_NORM, pooling, per-dim reductions beyond 2-D,
// broadcasting binary ops) follow the attribute contract of their producers
// and PyTorch-compatible semantics.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <limits>
#include <map>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include <cstdlib>
#include <thread>

namespace {

enum Op {
  ADD = 100, SUB = 101, MUL = 102, DIV = 103, POW = 104, MAX_BINARY = 105, MIN_BINARY = 106,
  NEG = 200, ABS = 201, SQRT = 202, EXP = 203, LOG = 204, SIN = 205, COS = 206, TANH = 207,
  RELU = 300, SIGMOID = 301, GELU = 302, SILU = 303, SOFTMAX = 304, LOG_SOFTMAX = 305,
  SUM = 400, MEAN = 401, MAX = 402, MIN = 403, PROD = 404,
  MATMUL = 500, TRANSPOSE = 501, BATCH_MATMUL = 502, CONV2D = 511,
  MAX_POOL2D = 521, AVG_POOL2D = 524, ADAPTIVE_AVG_POOL2D = 526, BATCH_NORM = 530, LAYER_NORM = 531,
  DROPOUT = 540, RESHAPE = 600, VIEW = 601, SQUEEZE = 602, UNSQUEEZE = 603, SLICE = 604, CONCAT = 605,
  STACK = 606, BROADCAST = 607, COPY = 700, CONTIGUOUS = 701, LAYOUT_TRANSFORM = 702,
  EQ = 800, NE = 801, LT = 802, LE = 803, GT = 804, GE = 805, LESS = 806, WHERE = 810, MAXIMUM = 811,
  MINIMUM = 812, CLAMP = 813,
};

struct Attr {
  int type = 0;
  std::vector<int64_t> i;
  std::vector<double> f;
};

struct Node {
  uint64_t id = 0;
  int type = 3, op = 0, dtype = 0;
  std::vector<int64_t> shape;
  std::vector<uint64_t> inputs;
  std::map<std::string, Attr> attrs;
  std::vector<uint8_t> data;
  bool has_data = false;

  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
  bool has(const std::string& k) const { return attrs.count(k) != 0; }
  int64_t geti(const std::string& k, int64_t d) const {
    auto it = attrs.find(k);
    if (it == attrs.end()) return d;
    if (!it->second.i.empty()) return it->second.i[0];
    if (!it->second.f.empty()) return (int64_t)it->second.f[0];
    return d;
  }
  double getf(const std::string& k, double d) const {
    auto it = attrs.find(k);
    if (it == attrs.end()) return d;
    if (!it->second.f.empty()) return it->second.f[0];
    if (!it->second.i.empty()) return (double)it->second.i[0];
    return d;
  }
  std::vector<int64_t> getv(const std::string& k, std::vector<int64_t> d) const {
    auto it = attrs.find(k);
    return it == attrs.end() ? d : it->second.i;
  }
};

struct Graph {
  std::vector<Node> nodes;
  std::unordered_map<uint64_t, size_t> index;
  const Node& at(uint64_t id) const {
    auto it = index.find(id);
    if (it == index.end()) throw std::runtime_error("Input not found: " + std::to_string(id));
    return nodes[it->second];
  }
};

template <class T>
struct Tensor {
  std::vector<int64_t> shape;
  std::vector<T> v;
};

// Worker threads of the calling host thread: set by orc_set_threads (per
// host thread, so concurrent callers can each ask for one), else
// ORACLE_THREADS, else every hardware thread.
thread_local int tl_threads = 0;
int oracle_threads() {
  static int n = [] {
    const char* e = std::getenv("ORACLE_THREADS");
    int v = e ? std::atoi(e) : (int)std::thread::hardware_concurrency();
    return v > 0 ? v : 1;
  }();
  return tl_threads > 0 ? tl_threads : n;
}

// Runs f(i) for i in [0, n) on contiguous chunks; each i runs exactly once,
// so per-element arithmetic is the same as a serial loop.
template <class F>
void parallel_for(int64_t n, F f, int64_t min_par = 2) {
  int nt = (int)std::min<int64_t>(oracle_threads(), n);
  if (nt <= 1 || n < min_par) {
    for (int64_t i = 0; i < n; ++i) f(i);
    return;
  }
  std::vector<std::thread> th;
  int64_t chunk = (n + nt - 1) / nt;
  for (int t = 0; t < nt; ++t) {
    int64_t b = t * chunk, e = std::min(n, b + chunk);
    if (b < e) th.emplace_back([=, &f] { for (int64_t i = b; i < e; ++i) f(i); });
  }
  for (auto& t : th) t.join();
}

std::vector<int64_t> strides_of(const std::vector<int64_t>& s) {
  std::vector<int64_t> st(s.size());
  int64_t a = 1;
  for (int d = (int)s.size() - 1; d >= 0; --d) {
    st[d] = a;
    a *= s[d];
  }
  return st;
}

int64_t prod(const std::vector<int64_t>& s, size_t b = 0, size_t e = SIZE_MAX) {
  int64_t p = 1;
  for (size_t i = b; i < std::min(e, s.size()); ++i) p *= s[i];
  return p;
}

// shape_inference.hpp:16-42
std::vector<int64_t> bcast(const std::vector<int64_t>& a, const std::vector<int64_t>& b) {
  size_t n = std::max(a.size(), b.size());
  std::vector<int64_t> r(n);
  for (size_t i = 0; i < n; ++i) {
    int64_t da = i < a.size() ? a[a.size() - 1 - i] : 1, db = i < b.size() ? b[b.size() - 1 - i] : 1;
    if (da == db || db == 1) r[n - 1 - i] = da;
    else if (da == 1) r[n - 1 - i] = db;
    else throw std::runtime_error("Shapes are not broadcastable");
  }
  return r;
}

// index map: element `lin` of a dense tensor of shape `out` read from `in` (broadcast)
template <class T>
std::vector<int64_t> bcast_index(const std::vector<int64_t>& in, const std::vector<int64_t>& out) {
  std::vector<int64_t> ist = strides_of(in), idx(prod(out));
  size_t off = out.size() - in.size();
  std::vector<int64_t> ost = strides_of(out);
  for (int64_t l = 0; l < (int64_t)idx.size(); ++l) {
    int64_t rem = l, p = 0;
    for (size_t d = 0; d < out.size(); ++d) {
      int64_t c = rem / ost[d];
      rem %= ost[d];
      if (d >= off && in[d - off] != 1) p += c * ist[d - off];
    }
    idx[l] = p;
  }
  return idx;
}

template <class T>
T relu(T x) { return (T(0) < x) ? x : T(0); }  // std::max(0.0f, x), executor.cpp:392-396

template <class T>
T unary(int op, T x) {
  switch (op) {
    case NEG: return -x;                                            // executor.cpp:343-347
    case ABS: return std::abs(x);                                   // :349-353
    case SQRT: return std::sqrt(x);                                 // :355-359
    case EXP: return std::exp(x);                                   // :361-365
    case LOG: return std::log(x);                                   // :367-371
    case SIN: return std::sin(x);                                   // :373-377
    case COS: return std::cos(x);                                   // :379-383
    case TANH: return std::tanh(x);                                 // :385-389
    case RELU: return relu(x);                                      // :392-396
    case SIGMOID: return T(1) / (T(1) + std::exp(-x));              // :398-402
    case GELU: return T(0.5) * x * (T(1) + std::tanh(T(0.7978845608f) * (x + T(0.044715f) * x * x * x)));  // :404-409
    case SILU: return x / (T(1) + std::exp(-x));                    // :411-416
    case DROPOUT: case COPY: case CONTIGUOUS: case LAYOUT_TRANSFORM: return x;  // inference identity (dropout.cpp:26-30)
  }
  throw std::runtime_error("unsupported unary op " + std::to_string(op));
}

template <class T>
T binary(int op, T a, T b) {
  switch (op) {
    case ADD: return a + b;
    case SUB: return a - b;
    case MUL: return a * b;
    case DIV:  // executor.cpp:322-340
      if (b == T(0)) {
        if (a == T(0)) return std::numeric_limits<T>::quiet_NaN();
        return a > T(0) ? std::numeric_limits<T>::infinity() : -std::numeric_limits<T>::infinity();
      }
      return a / b;
    case POW: return std::pow(a, b);
    case MAX_BINARY: case MAXIMUM: return std::fmax(a, b);
    case MIN_BINARY: case MINIMUM: return std::fmin(a, b);
    case EQ: return a == b ? T(1) : T(0);
    case NE: return a != b ? T(1) : T(0);
    case LT: case LESS: return a < b ? T(1) : T(0);
    case LE: return a <= b ? T(1) : T(0);
    case GT: return a > b ? T(1) : T(0);
    case GE: return a >= b ? T(1) : T(0);
  }
  throw std::runtime_error("unsupported binary op " + std::to_string(op));
}

template <class T>
class Eval {
 public:
  explicit Eval(const Graph& g) : g_(g) {}

  const Tensor<T>& value(uint64_t id) {
    auto it = val_.find(id);
    if (it != val_.end()) return it->second;
    // iterative post-order so deep graphs do not overflow the stack
    std::vector<std::pair<uint64_t, size_t>> st{{id, 0}};
    while (!st.empty()) {
      auto& [n, i] = st.back();
      const Node& node = g_.at(n);
      if (val_.count(n)) { st.pop_back(); continue; }
      if (i < node.inputs.size()) {
        uint64_t c = node.inputs[i++];
        if (!val_.count(c)) st.push_back({c, 0});
      } else {
        val_[n] = compute(node);
        st.pop_back();
      }
    }
    return val_.at(id);
  }

 private:
  const Graph& g_;
  std::unordered_map<uint64_t, Tensor<T>> val_;

  const Tensor<T>& in(const Node& n, size_t k) {
    if (k >= n.inputs.size()) throw std::runtime_error("missing input of node " + std::to_string(n.id));
    return val_.at(n.inputs[k]);
  }

  Tensor<T> compute(const Node& n) {
    Tensor<T> out;
    out.shape = n.shape;
    if (n.type != 3) {
      // constants / inputs / parameters: payload or zeros (the ROCm executor zero-fills, rocm_executor.cpp:99-102)
      out.v.assign(n.numel(), T(0));
      if (n.has_data) {
        const int64_t ne = n.numel(), blk = 1 << 16;
        if (n.dtype == 0) {
          const float* p = (const float*)n.data.data();
          parallel_for((ne + blk - 1) / blk, [&](int64_t b) {
            for (int64_t i = b * blk; i < std::min(ne, (b + 1) * blk); ++i) out.v[i] = (T)p[i];
          });
        } else if (n.dtype == 7) {
          const double* p = (const double*)n.data.data();
          parallel_for((ne + blk - 1) / blk, [&](int64_t b) {
            for (int64_t i = b * blk; i < std::min(ne, (b + 1) * blk); ++i) out.v[i] = (T)p[i];
          });
        } else {
          throw std::runtime_error("oracle evaluates float32/float64 payloads only");
        }
      }
      return out;
    }
    const int op = n.op;
    if ((op >= 200 && op < 300) || (op >= 300 && op <= 303) || op == DROPOUT || op == COPY || op == CONTIGUOUS ||
        op == LAYOUT_TRANSFORM) {
      const auto& x = in(n, 0);
      out.v.resize(x.v.size());
      const int64_t ne = (int64_t)x.v.size(), blk = 1 << 14;
      parallel_for((ne + blk - 1) / blk, [&](int64_t b) {
        for (int64_t i = b * blk; i < std::min(ne, (b + 1) * blk); ++i) out.v[i] = unary<T>(op, x.v[i]);
      });
      return out;
    }
    if ((op >= 100 && op < 200) || (op >= 800 && op <= 806) || op == MAXIMUM || op == MINIMUM) {
      // binary with shape_inference broadcasting (shape_inference.hpp:16-42); for
      // trailing-dim broadcasts this equals ops::broadcast_binary_op (elementwise.cpp:399-430)
      const auto& a = in(n, 0);
      const auto& b = in(n, 1);
      auto os = bcast(a.shape, b.shape);
      auto ia = bcast_index<T>(a.shape, os), ib = bcast_index<T>(b.shape, os);
      out.shape = os;
      out.v.resize(prod(os));
      const int64_t ne = (int64_t)out.v.size(), blk = 1 << 14;
      parallel_for((ne + blk - 1) / blk, [&](int64_t bk) {
        for (int64_t i = bk * blk; i < std::min(ne, (bk + 1) * blk); ++i) out.v[i] = binary<T>(op, a.v[ia[i]], b.v[ib[i]]);
      });
      return out;
    }
    switch (op) {
      case WHERE: case CLAMP: {
        const auto& a = in(n, 0);
        const auto& b = in(n, 1);
        const auto& c = in(n, 2);
        auto os = bcast(bcast(a.shape, b.shape), c.shape);
        auto ia = bcast_index<T>(a.shape, os), ib = bcast_index<T>(b.shape, os), ic = bcast_index<T>(c.shape, os);
        out.shape = os;
        out.v.resize(prod(os));
        for (size_t i = 0; i < out.v.size(); ++i)
          out.v[i] = op == WHERE ? (a.v[ia[i]] != T(0) ? b.v[ib[i]] : c.v[ic[i]])
                                 : std::fmin(std::fmax(a.v[ia[i]], b.v[ib[i]]), c.v[ic[i]]);
        return out;
      }
      case SUM: case MEAN: case MAX: case MIN: case PROD: return reduce(n);
      case SOFTMAX: case LOG_SOFTMAX: return softmax(n);
      case LAYER_NORM: return layer_norm(n);
      case BATCH_NORM: return batch_norm(n);
      case MATMUL: case BATCH_MATMUL: return matmul(n);
      case CONV2D: return conv2d(n);
      case MAX_POOL2D: case AVG_POOL2D: case ADAPTIVE_AVG_POOL2D: return pool(n);
      case RESHAPE: case VIEW: case SQUEEZE: case UNSQUEEZE: case BROADCAST: {
        const auto& x = in(n, 0);
        if (op == BROADCAST) {
          auto idx = bcast_index<T>(x.shape, n.shape);
          out.v.resize(idx.size());
          for (size_t i = 0; i < idx.size(); ++i) out.v[i] = x.v[idx[i]];
          return out;
        }
        if ((int64_t)x.v.size() != n.numel()) throw std::runtime_error("reshape: total elements must match");
        out.v = x.v;  // executor.cpp:495-502: contiguous copy
        return out;
      }
      case TRANSPOSE: return transpose(n);
      case SLICE: return slice(n);
      case CONCAT: case STACK: return concat(n);
    }
    throw std::runtime_error("oracle: unsupported operation " + std::to_string(op));
  }

  // Reductions: sequential accumulation in index order along the reduced dim
  // (reduction.cpp:49-121, generalised as reduce_nd_cpu, reduction.cpp:151-220);
  // no `dim` attribute reduces everything (tensor_impl.cpp:214-266).
  Tensor<T> reduce(const Node& n) {
    const auto& x = in(n, 0);
    Tensor<T> out;
    out.shape = n.shape;
    int nd = (int)x.shape.size();
    int64_t O, R, I;
    if (!n.has("dim")) {
      O = 1; R = (int64_t)x.v.size(); I = 1;
    } else {
      int d = (int)n.geti("dim", 0);
      if (d < 0) d += nd;
      if (d < 0 || d >= nd) throw std::runtime_error("Reduction dimension out of range");
      O = prod(x.shape, 0, d); R = x.shape[d]; I = prod(x.shape, d + 1);
    }
    out.v.assign(O * I, T(0));
    parallel_for(O * I, [&](int64_t p) {
      int64_t o = p / I, i = p % I;
      const T* base = x.v.data() + o * R * I + i;
      T acc;
      switch (n.op) {
        case SUM: case MEAN:
          acc = T(0);
          for (int64_t r = 0; r < R; ++r) acc += base[r * I];
          if (n.op == MEAN) acc = acc / (T)R;  // reduction.cpp:78-94
          break;
        case PROD:
          acc = T(1);
          for (int64_t r = 0; r < R; ++r) acc *= base[r * I];
          break;
        case MAX:  // reduction.cpp:96-121: first element, then std::max
          acc = base[0];
          for (int64_t r = 1; r < R; ++r) acc = std::max(acc, base[r * I]);
          break;
        default:  // MIN, reduction.cpp:123-148
          acc = base[0];
          for (int64_t r = 1; r < R; ++r) acc = std::min(acc, base[r * I]);
          break;
      }
      out.v[p] = acc;
    }, 64);
    return out;
  }

  // tensor_impl.cpp:268-352: max (from -inf), exp(x - max), sum, divide; log_softmax
  // returns x - (max + log(sum)).
  Tensor<T> softmax(const Node& n) {
    const auto& x = in(n, 0);
    Tensor<T> out;
    out.shape = x.shape;
    out.v.resize(x.v.size());
    int nd = (int)x.shape.size();
    int d = (int)n.geti("dim", -1);
    if (d < 0) d += nd;
    int64_t O = prod(x.shape, 0, d), R = x.shape[d], I = prod(x.shape, d + 1);
    parallel_for(O * I, [&](int64_t p) {
      int64_t o = p / I, i = p % I;
      const T* xb = x.v.data() + o * R * I + i;
      T* yb = out.v.data() + o * R * I + i;
      T m = -std::numeric_limits<T>::infinity();
      for (int64_t r = 0; r < R; ++r) m = std::max(m, xb[r * I]);
      T s = T(0);
      if (n.op == SOFTMAX) {
        for (int64_t r = 0; r < R; ++r) {
          yb[r * I] = std::exp(xb[r * I] - m);
          s += yb[r * I];
        }
        for (int64_t r = 0; r < R; ++r) yb[r * I] /= s;
      } else {
        for (int64_t r = 0; r < R; ++r) s += std::exp(xb[r * I] - m);
        T lse = m + std::log(s);
        for (int64_t r = 0; r < R; ++r) yb[r * I] = xb[r * I] - lse;
      }
    }, 64);
    return out;
  }

  // LAYER_NORM over the trailing normalized_shape dims (normalization.cpp:224-255):
  // mean, biased variance, (x - mean) * (1 / sqrt(var + eps)) * gamma + beta.
  Tensor<T> layer_norm(const Node& n) {
    const auto& x = in(n, 0);
    auto ns = n.getv("normalized_shape", {x.shape.back()});
    T eps = (T)n.getf("eps", 1e-5);
    int64_t C = prod(ns), R = (int64_t)x.v.size() / C;
    const Tensor<T>* gam = n.inputs.size() >= 3 ? &in(n, 1) : nullptr;
    const Tensor<T>* bet = n.inputs.size() >= 3 ? &in(n, 2) : nullptr;
    Tensor<T> out;
    out.shape = x.shape;
    out.v.resize(x.v.size());
    parallel_for(R, [&](int64_t r) {
      const T* xb = x.v.data() + r * C;
      T* yb = out.v.data() + r * C;
      T s = T(0);
      for (int64_t c = 0; c < C; ++c) s += xb[c];
      T mean = s / (T)C;
      T v = T(0);
      for (int64_t c = 0; c < C; ++c) {
        T dv = xb[c] - mean;
        v += dv * dv;
      }
      T inv = T(1) / std::sqrt(v / (T)C + eps);
      for (int64_t c = 0; c < C; ++c) {
        T t = (xb[c] - mean) * inv;
        if (gam) t = t * gam->v[c];
        if (bet) t = t + bet->v[c];
        yb[c] = t;
      }
    }, 16);
    return out;
  }

  // BATCH_NORM in inference mode (normalization.cpp:53-93): inputs {x, [weight, bias],
  // [running_mean, running_var]}; y = (x - mean[c]) / sqrt(var[c] + eps) * weight[c] + bias[c].
  Tensor<T> batch_norm(const Node& n) {
    const auto& x = in(n, 0);
    bool affine = n.geti("affine", n.inputs.size() == 5) != 0;
    if (n.geti("training", 0)) throw std::runtime_error("oracle: BATCH_NORM training mode");
    size_t k = 1;
    const Tensor<T>* gam = nullptr;
    const Tensor<T>* bet = nullptr;
    if (affine) { gam = &in(n, k++); bet = &in(n, k++); }
    const auto& mean = in(n, k++);
    const auto& var = in(n, k++);
    T eps = (T)n.getf("eps", 1e-5);
    int64_t N = x.shape[0], C = x.shape[1], HW = (int64_t)x.v.size() / (N * C);
    Tensor<T> out;
    out.shape = x.shape;
    out.v.resize(x.v.size());
    for (int64_t i = 0; i < N; ++i)
      for (int64_t c = 0; c < C; ++c)
        for (int64_t p = 0; p < HW; ++p) {
          int64_t idx = (i * C + c) * HW + p;
          T t = (x.v[idx] - mean.v[c]) / std::sqrt(var.v[c] + eps);
          if (gam) t = t * gam->v[c];
          if (bet) t = t + bet->v[c];
          out.v[idx] = t;
        }
    return out;
  }

  // MATMUL: per-element sequential sum over k in the order of executor.cpp:479-487
  // (2-D) / batch_matmul_cpu (matmul.cpp:124-145); shapes per infer_matmul_spec
  // (shape_inference.hpp:146-217) including broadcast batch dims and 1-D operands.
  Tensor<T> matmul(const Node& n) {
    const Tensor<T>& a = in(n, 0);
    const Tensor<T>& b = in(n, 1);
    std::vector<int64_t> as = a.shape, bs = b.shape;
    if (as.size() == 1) as.insert(as.begin(), 1);
    if (bs.size() == 1) bs.push_back(1);
    int64_t M = as[as.size() - 2], K = as.back(), N = bs.back();
    if (bs[bs.size() - 2] != K) throw std::runtime_error("matmul: inner dimensions don't match");
    std::vector<int64_t> ab(as.begin(), as.end() - 2), bb(bs.begin(), bs.end() - 2);
    std::vector<int64_t> batch = bcast(ab, bb);
    int64_t B = prod(batch);
    auto ia = bcast_index<T>(ab.empty() ? std::vector<int64_t>{1} : ab, batch.empty() ? std::vector<int64_t>{1} : batch);
    auto ib = bcast_index<T>(bb.empty() ? std::vector<int64_t>{1} : bb, batch.empty() ? std::vector<int64_t>{1} : batch);
    Tensor<T> out;
    out.shape = n.shape;
    out.v.assign(B * M * N, T(0));
    parallel_for(B * M, [&](int64_t bm) {
        const int64_t bi = bm / M, i = bm % M;
        const T* A = a.v.data() + ia[bi] * M * K + i * K;
        const T* Bm = b.v.data() + ib[bi] * K * N;
        T* Cr = out.v.data() + (bi * M + i) * N;
        // i-k-j order: C[i][j] still accumulates k = 0..K-1 in sequence
        for (int64_t k = 0; k < K; ++k) {
          const T av = A[k];
          const T* Br = Bm + k * N;
          for (int64_t j = 0; j < N; ++j) Cr[j] += av * Br[j];
        }
      }, 4);
    return out;
  }

  // CONV2D (conv.cpp:75-131 attribute contract): cross-correlation with zero
  // padding, sum over (c, kh, kw) in order; groups split channels.
  Tensor<T> conv2d(const Node& n) {
    const auto& x = in(n, 0);
    const auto& w = in(n, 1);
    auto st = n.getv("stride", {1, 1}), pd = n.getv("padding", {0, 0}), dl = n.getv("dilation", {1, 1});
    int64_t G = n.geti("groups", 1);
    int64_t NB = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
    int64_t O = w.shape[0], CG = w.shape[1], KH = w.shape[2], KW = w.shape[3];
    int64_t OH = n.shape[2], OW = n.shape[3];
    (void)C;
    Tensor<T> out;
    out.shape = n.shape;
    out.v.assign(NB * O * OH * OW, T(0));
    parallel_for(NB * O, [&](int64_t bo) {
        const int64_t b = bo / O, o = bo % O;
        int64_t g = o / (O / G);
        for (int64_t oh = 0; oh < OH; ++oh)
          for (int64_t ow = 0; ow < OW; ++ow) {
            T acc = T(0);
            for (int64_t c = 0; c < CG; ++c)
              for (int64_t kh = 0; kh < KH; ++kh) {
                int64_t ih = oh * st[0] - pd[0] + kh * dl[0];
                if (ih < 0 || ih >= H) continue;
                for (int64_t kw = 0; kw < KW; ++kw) {
                  int64_t iw = ow * st[1] - pd[1] + kw * dl[1];
                  if (iw < 0 || iw >= W) continue;
                  acc += x.v[((b * x.shape[1] + g * CG + c) * H + ih) * W + iw] *
                         w.v[((o * CG + c) * KH + kh) * KW + kw];
                }
              }
            out.v[((b * O + o) * OH + oh) * OW + ow] = acc;
          }
      });
    return out;
  }

  // MaxPool2d / AvgPool2d (pooling.cpp:38-63,97-122; output (H + 2p - k)/s + 1),
  // AdaptiveAvgPool2d (pooling.cpp:150-168; window [floor(i*H/OH), ceil((i+1)*H/OH))).
  // Max ignores padding and propagates NaN; average divides by k*k (padding counted).
  Tensor<T> pool(const Node& n) {
    const auto& x = in(n, 0);
    int64_t NB = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
    int64_t OH = n.shape[2], OW = n.shape[3];
    auto ks = n.getv("kernel_size", {1, 1});
    auto st = n.getv("stride", ks), pd = n.getv("padding", {0, 0});
    Tensor<T> out;
    out.shape = n.shape;
    out.v.resize(NB * C * OH * OW);
    parallel_for(NB * C, [&](int64_t bc) {
        const int64_t b = bc / C, c = bc % C;
        const T* xb = x.v.data() + (b * C + c) * H * W;
        for (int64_t oh = 0; oh < OH; ++oh)
          for (int64_t ow = 0; ow < OW; ++ow) {
            T r;
            if (n.op == ADAPTIVE_AVG_POOL2D) {
              int64_t h0 = oh * H / OH, h1 = ((oh + 1) * H + OH - 1) / OH;
              int64_t w0 = ow * W / OW, w1 = ((ow + 1) * W + OW - 1) / OW;
              T s = T(0);
              for (int64_t h = h0; h < h1; ++h)
                for (int64_t w = w0; w < w1; ++w) s += xb[h * W + w];
              r = s / (T)((h1 - h0) * (w1 - w0));
            } else if (n.op == MAX_POOL2D) {
              r = -std::numeric_limits<T>::infinity();
              for (int64_t kh = 0; kh < ks[0]; ++kh) {
                int64_t h = oh * st[0] - pd[0] + kh;
                if (h < 0 || h >= H) continue;
                for (int64_t kw = 0; kw < ks[1]; ++kw) {
                  int64_t w = ow * st[1] - pd[1] + kw;
                  if (w < 0 || w >= W) continue;
                  T v = xb[h * W + w];
                  if (v > r || std::isnan(v)) r = v;
                }
              }
            } else {
              T s = T(0);
              for (int64_t kh = 0; kh < ks[0]; ++kh) {
                int64_t h = oh * st[0] - pd[0] + kh;
                if (h < 0 || h >= H) continue;
                for (int64_t kw = 0; kw < ks[1]; ++kw) {
                  int64_t w = ow * st[1] - pd[1] + kw;
                  if (w < 0 || w >= W) continue;
                  s += xb[h * W + w];
                }
              }
              r = s / (T)(ks[0] * ks[1]);
            }
            out.v[((b * C + c) * OH + oh) * OW + ow] = r;
          }
      });
    return out;
  }

  // TRANSPOSE of any two dims (executor.cpp:505-519 does 2-D; attrs dim0/dim1,
  // tensor_impl.cpp:577-578).
  Tensor<T> transpose(const Node& n) {
    const auto& x = in(n, 0);
    int nd = (int)x.shape.size();
    int d0 = (int)n.geti("dim0", 0), d1 = (int)n.geti("dim1", 1);
    if (d0 < 0) d0 += nd;
    if (d1 < 0) d1 += nd;
    auto ist = strides_of(x.shape);
    Tensor<T> out;
    out.shape = x.shape;
    std::swap(out.shape[d0], out.shape[d1]);
    auto ost = strides_of(out.shape);
    out.v.resize(x.v.size());
    const int64_t ne = (int64_t)out.v.size(), blk = 1 << 14;
    parallel_for((ne + blk - 1) / blk, [&](int64_t b) {
      for (int64_t l = b * blk; l < std::min(ne, (b + 1) * blk); ++l) {
        int64_t rem = l, src = 0;
        for (int d = 0; d < nd; ++d) {
          int64_t c = rem / ost[d];
          rem %= ost[d];
          int sd = d == d0 ? d1 : (d == d1 ? d0 : d);
          src += c * ist[sd];
        }
        out.v[l] = x.v[src];
      }
    });
    return out;
  }

  // SLICE (tensor_impl.cpp:413-457; attrs dim/start/end, normalised by tensor.cpp:262-283)
  Tensor<T> slice(const Node& n) {
    const auto& x = in(n, 0);
    int nd = (int)x.shape.size();
    int d = (int)n.geti("dim", 0);
    if (d < 0) d += nd;
    int64_t size = x.shape[d];
    int64_t s = n.geti("start", 0), e = n.geti("end", size);
    if (s < 0) s += size;
    if (e < 0) e += size;
    s = std::max<int64_t>(0, std::min(s, size));
    e = std::max<int64_t>(0, std::min(e, size));
    int64_t O = prod(x.shape, 0, d), I = prod(x.shape, d + 1);
    Tensor<T> out;
    out.shape = x.shape;
    out.shape[d] = e - s;
    out.v.resize(O * (e - s) * I);
    for (int64_t o = 0; o < O; ++o)
      for (int64_t r = s; r < e; ++r)
        for (int64_t i = 0; i < I; ++i) out.v[(o * (e - s) + (r - s)) * I + i] = x.v[(o * size + r) * I + i];
    return out;
  }

  // CONCAT along `dim` (tensor.cpp:807-831); STACK inserts a new dim.
  Tensor<T> concat(const Node& n) {
    int nd = (int)n.shape.size();
    int d = (int)n.geti("dim", 0);
    if (d < 0) d += nd;
    Tensor<T> out;
    out.shape = n.shape;
    out.v.resize(n.numel());
    int64_t O = prod(n.shape, 0, d), I = prod(n.shape, d + 1), D = n.shape[d];
    int64_t off = 0;
    for (size_t k = 0; k < n.inputs.size(); ++k) {
      const auto& x = in(n, k);
      int64_t len = n.op == STACK ? 1 : x.shape[d];
      for (int64_t o = 0; o < O; ++o)
        for (int64_t r = 0; r < len; ++r)
          for (int64_t i = 0; i < I; ++i) out.v[(o * D + off + r) * I + i] = x.v[(o * len + r) * I + i];
      off += len;
    }
    return out;
  }
};

thread_local std::string g_err;

}  // namespace

extern "C" {

void* orc_graph_create(void) { return new Graph(); }
void orc_graph_destroy(void* g) { delete (Graph*)g; }
const char* orc_last_error(void) { return g_err.c_str(); }

int orc_add_node(void* gp, uint64_t id, int node_type, int op_type, int dtype, int ndim, const int64_t* shape,
                 int n_in, const uint64_t* inputs) {
  Graph& g = *(Graph*)gp;
  if (g.index.count(id)) { g_err = "duplicate id"; return -1; }
  Node n;
  n.id = id;
  n.type = node_type;
  n.op = op_type;
  n.dtype = dtype;
  n.shape.assign(shape, shape + ndim);
  n.inputs.assign(inputs, inputs + n_in);
  g.index[id] = g.nodes.size();
  g.nodes.push_back(std::move(n));
  return 0;
}

int orc_set_attr(void* gp, uint64_t id, const char* key, int type, const void* value, int64_t count) {
  Graph& g = *(Graph*)gp;
  auto it = g.index.find(id);
  if (it == g.index.end()) { g_err = "no node"; return -1; }
  Attr a;
  a.type = type;
  switch (type) {
    case 0: a.i.push_back(*(const int32_t*)value); break;
    case 1: a.i.push_back(*(const int64_t*)value); break;
    case 2: a.f.push_back(*(const float*)value); break;
    case 3: a.f.push_back(*(const double*)value); break;
    case 4: a.i.push_back(*(const uint8_t*)value); break;
    case 5: for (int64_t k = 0; k < count; ++k) a.i.push_back(((const int64_t*)value)[k]); break;
    case 6: for (int64_t k = 0; k < count; ++k) a.i.push_back(((const int32_t*)value)[k]); break;
    case 7: for (int64_t k = 0; k < count; ++k) a.f.push_back(((const float*)value)[k]); break;
    default: g_err = "bad attr type"; return -1;
  }
  g.nodes[it->second].attrs[key] = a;
  return 0;
}

int orc_set_constant(void* gp, uint64_t id, const void* data, size_t bytes) {
  Graph& g = *(Graph*)gp;
  auto it = g.index.find(id);
  if (it == g.index.end()) { g_err = "no node"; return -1; }
  Node& n = g.nodes[it->second];
  n.data.assign((const uint8_t*)data, (const uint8_t*)data + bytes);
  n.has_data = bytes > 0;
  return 0;
}

// precision 0: float arithmetic, outputs float; 1: double arithmetic, outputs double.
int orc_execute(void* gp, const uint64_t* ids, int n, void* const* outs, int precision) {
  try {
    Graph& g = *(Graph*)gp;
    if (precision == 0) {
      Eval<float> ev(g);
      for (int i = 0; i < n; ++i) {
        const auto& t = ev.value(ids[i]);
        std::memcpy(outs[i], t.v.data(), t.v.size() * sizeof(float));
      }
    } else {
      Eval<double> ev(g);
      for (int i = 0; i < n; ++i) {
        const auto& t = ev.value(ids[i]);
        std::memcpy(outs[i], t.v.data(), t.v.size() * sizeof(double));
      }
    }
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

int orc_num_threads(void) { return oracle_threads(); }
// Worker threads for later calls from the calling host thread (0: the default).
void orc_set_threads(int n) { tl_threads = n > 0 ? n : 0; }

}  // extern "C"
