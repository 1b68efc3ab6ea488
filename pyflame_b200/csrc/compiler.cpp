// Graph -> Plan compiler.  See compiler.hpp.
//
// Node semantics follow PyFlame's producers and CPU evaluators; each op's
// reference is cited where it is lowered.  Passes, in order:
//   1. classify nodes (leaf / view / elementwise / row / gemm / conv / pool / concat)
//   2. absorb GEMM and conv epilogues: MATMUL -> *splat -> +bias -> act -> +residual,
//      CONV2D -> +bias[1,C,1,1] -> BATCH_NORM(eval) -> RELU
//   3. grow convex elementwise regions of equal shape
//   4. attach row operations (reductions, softmax, LayerNorm) to the region
//      that produces their input, so the prologue is computed in registers
//   5. decide which values are materialised, build strided views for shape
//      ops, emit steps, plan buffer liveness and the arena.
#include "compiler.hpp"
#include "kernels/kernels.hpp"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <set>
#include <sstream>

#include "jit.hpp"

namespace pfb {

bool View::is_contiguous() const {
  int64_t expect = 1;
  for (int d = (int)shape.size() - 1; d >= 0; --d) {
    if (shape[d] != 1 && strides[d] != expect) return false;
    expect *= shape[d];
  }
  return true;
}

std::vector<int64_t> View::dense_strides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> s(shape.size());
  int64_t acc = 1;
  for (int d = (int)shape.size() - 1; d >= 0; --d) {
    s[d] = acc;
    acc *= shape[d];
  }
  return s;
}

namespace {

enum class Cls : uint8_t { LEAF, VIEW, EW, ROW, GEMM, CONV, POOL, CONCAT };

bool is_view_op(Op op) {
  switch (op) {
    case Op::RESHAPE: case Op::VIEW: case Op::SQUEEZE: case Op::UNSQUEEZE: case Op::TRANSPOSE:
    case Op::SLICE: case Op::BROADCAST: case Op::CONTIGUOUS: case Op::COPY:
    case Op::LAYOUT_TRANSFORM: case Op::DROPOUT:
      return true;
    default:
      return false;
  }
}

bool is_row_op(Op op) {
  switch (op) {
    case Op::SUM: case Op::MEAN: case Op::MAX: case Op::MIN: case Op::PROD:
    case Op::SOFTMAX: case Op::LOG_SOFTMAX: case Op::LAYER_NORM:
      return true;
    default:
      return false;
  }
}

bool is_act(Op op) {
  return op == Op::RELU || op == Op::GELU || op == Op::SIGMOID || op == Op::TANH || op == Op::SILU;
}
int act_code(Op op) {
  switch (op) {
    case Op::RELU: return 1; case Op::GELU: return 2; case Op::SIGMOID: return 3;
    case Op::TANH: return 4; case Op::SILU: return 5; default: return 0;
  }
}

int64_t prod(const std::vector<int64_t>& v, size_t b = 0, size_t e = SIZE_MAX) {
  int64_t p = 1;
  for (size_t i = b; i < std::min(e, v.size()); ++i) p *= v[i];
  return p;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

// Right-aligned broadcast of a view to `shape` (shape_inference.hpp:16-42).
View broadcast_to(const View& v, const std::vector<int64_t>& shape) {
  View r = v;
  size_t nd = shape.size();
  if (v.shape.size() > nd) fail(PFC_ERR_GRAPH, "cannot broadcast " + shape_str(v.shape) + " to " + shape_str(shape));
  r.shape = shape;
  r.strides.assign(nd, 0);
  size_t off = nd - v.shape.size();
  for (size_t d = 0; d < v.shape.size(); ++d) {
    int64_t sz = v.shape[d], tgt = shape[off + d];
    if (sz == tgt) r.strides[off + d] = v.strides.empty() ? 0 : v.strides[d];
    else if (sz == 1) r.strides[off + d] = 0;
    else fail(PFC_ERR_GRAPH, "Shapes are not broadcastable: " + shape_str(v.shape) + " vs " + shape_str(shape));
  }
  return r;
}

// Stride-preserving reshape; false when the new shape cannot view the data.
bool reshape_view(const View& v, const std::vector<int64_t>& ns, View* out) {
  *out = v;
  out->shape = ns;
  int64_t n = v.numel();
  if (n == 0 || n == 1 || v.is_contiguous()) {
    out->strides = View::dense_strides(ns);
    return true;
  }
  const auto& os = v.shape;
  const auto& ost = v.strides;
  std::vector<int64_t> st(ns.size(), 0);
  int vd = (int)ns.size() - 1;
  int64_t base = ost.back(), tn = 1, vn = 1;
  for (int td = (int)os.size() - 1; td >= 0; --td) {
    tn *= os[td];
    if (td == 0 || (os[td - 1] != 1 && ost[td - 1] != tn * base)) {
      while (vd >= 0 && (vn < tn || ns[vd] == 1)) {
        st[vd] = vn * base;
        vn *= ns[vd];
        --vd;
      }
      if (vn != tn) return false;
      if (td > 0) {
        base = ost[td - 1];
        tn = 1;
        vn = 1;
      }
    }
  }
  if (vd != -1) return false;
  out->strides = st;
  return true;
}

// ---------------------------------------------------------------------------
// Kernel specifications
// ---------------------------------------------------------------------------

// One elementwise instruction.  LOAD reads load `load`; the others combine
// earlier instructions (indices in `a`).
enum class EwKind : uint8_t { LOAD, OP, COPY, BN };
struct EwInstr {
  EwKind kind = EwKind::OP;
  Op op = Op::NONE;
  std::vector<int> a;
  int load = -1;
  float p0 = 0.f;  // BN eps
};

struct EwSpec {
  std::vector<int64_t> space;
  std::vector<View> loads;                     // broadcast to `space`
  std::vector<EwInstr> instrs;
  std::vector<std::pair<int, View>> stores;    // instr -> view shaped like `space`
};

struct RowOp {
  Op op;
  int src = -1, gamma = -1, beta = -1;
  float eps = 1e-5f;
  View out;   // reductions: dense [outer*inner]; softmax/LN: view shaped like space
  // softmax/LN feeding GEMMs: the row kernel also writes the tf32x3 operand
  // (hi/lo at the dense offsets of `out`); `out` itself only when read elsewhere
  int op_hi = -1, op_lo = -1;
  bool write_out = true;
};

struct RowSpec {
  EwSpec ew;
  int red_begin = 0, red_end = 0;   // dims [red_begin, red_end) of space are reduced
  std::vector<RowOp> ops;
};

// ---------------------------------------------------------------------------
// Code generation helpers
// ---------------------------------------------------------------------------

const char* kPrelude = R"(
#define PF_INF __int_as_float(0x7f800000)
#define PF_NAN __int_as_float(0x7fffffff)
struct PfArgs { void* p[48]; };
// DIV as the CPU reference evaluates it (executor.cpp:322-340): a zero
// divisor gives NaN for 0/0 and an infinity signed by the dividend.
__device__ __forceinline__ float pf_div(float a, float b) {
  if (b == 0.f) return a == 0.f ? PF_NAN : (a > 0.f ? PF_INF : -PF_INF);
  return a / b;
}
__device__ __forceinline__ float pf_relu(float x) { return (0.f < x) ? x : 0.f; }
// exp(y) from the hardware exp2 (ex2.approx, about 2 ulp over its range)
// with the argument split in the manner of Cody and Waite: p = fl(y*L2E) and
// its rounding error r = (y*L2E - p) + y*L2E_LO (one fma) are kept apart and
// exp(y) = 2^p * 2^r ~= 2^p * (1 + r*ln2), |r| <= 2^-17 for |y| <= 88.8.  A
// plain exp2(fl(y*log2e)) instead loses |y|*2^-24*ln2 of relative accuracy
// (about 4e-6 at |y| = 88).  L2E + L2E_LO = log2(e) to about 2^-50.  Where
// 2^p already saturates (|p| >= 256), infinities or NaN, r is left out.
__device__ __forceinline__ float pf_exp_split(float y) {
  const float L2E = 1.44269502162933349609375f, L2E_LO = 1.925962991e-08f;
  const float p = y * L2E;
  const float r = fabsf(p) < 256.0f ? fmaf(y, L2E, -p) + y * L2E_LO : 0.0f;
  float e;
  asm("ex2.approx.f32 %0, %1;" : "=f"(e) : "f"(p));
  return e * fmaf(r, 0.693147180559945309f, 1.0f);
}
// n / (1 + exp(-x)) with the fast divide (__fdividef, exact to about 2 ulp
// for divisors up to 2^126).  Divisors above 2^126 (x < -87.34, up to the
// infinity of exp's overflow) are scaled by 1/4 on both sides first, so
// results below FLT_MIN still come out as the correctly signed subnormal
// (or zero) that the reference's division gives, and SiLU's normal-range
// outputs for -88.72 < x < -87.34 are kept.
__device__ __forceinline__ float pf_over_1pexp(float n, float x) {
  const float d = 1.0f + pf_exp_split(-x);
  const float s = d > 8.50705917e+37f ? 0.25f : 1.0f;  // 2^126
  return __fdividef(n * s, d * s);
}
// Sigmoid 1/(1+exp(-x)) (executor.cpp:398-403) and SiLU x/(1+exp(-x))
// (executor.cpp:411-416): within a few ulp of the exact value over every
// output at or above FLT_MIN, and exact at the limits (0, 1, NaN).
__device__ __forceinline__ float pf_sigmoid(float x) { return pf_over_1pexp(1.0f, x); }
__device__ __forceinline__ float pf_gelu(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
}
__device__ __forceinline__ float pf_silu(float x) { return pf_over_1pexp(x, x); }
__device__ __forceinline__ float pf_max(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ float pf_min(float a, float b) { return fminf(a, b); }
// The 3xTF32 operand split (identical to the precompiled kernels'): hi keeps
// sign, exponent and the top 10 mantissa bits, lo the exact remainder;
// non-finite values go entirely into hi (NaN canonicalised).
__device__ __forceinline__ void pf_split(float x, float& hi, float& lo) {
  if (!isfinite(x)) { hi = isnan(x) ? __int_as_float(0x7fc00000) : x; lo = 0.f; return; }
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}
)";

// Helpers for kernels that stream rows into shared memory with 1-D TMA bulk
// copies completing on mbarriers.  Waits are bounded by the global timer: on
// expiry the kernel records PFC_ERR_TIMEOUT (-8) in *err and carries on
// without blocking.
const char* kTmaPrelude = R"(
__device__ __forceinline__ unsigned pf_smem(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void pf_mbar_init(unsigned a, unsigned n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(a), "r"(n) : "memory");
}
__device__ __forceinline__ void pf_expect_tx(unsigned a, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void pf_bulk_load(unsigned dst, const void* src, unsigned bytes, unsigned bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ bool pf_mbar_try(unsigned a, unsigned parity) {
  unsigned ok;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(a), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long pf_gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool pf_mbar_wait(unsigned a, unsigned parity, int* err) {
  if (pf_mbar_try(a, parity)) return true;
  const unsigned long long t0 = pf_gtimer();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (pf_mbar_try(a, parity)) return true;
    if (*(volatile int*)err != 0 || pf_gtimer() - t0 > 2000000000ull) {
      atomicCAS(err, 0, -8);
      return false;
    }
  }
}
)";

std::string flit(float f) {
  if (std::isnan(f)) return "PF_NAN";
  if (std::isinf(f)) return f > 0 ? "PF_INF" : "(-PF_INF)";
  uint32_t b;
  std::memcpy(&b, &f, 4);
  char buf[48];
  std::snprintf(buf, sizeof buf, "__int_as_float(0x%08x)", b);
  return buf;
}

std::string op_expr(const EwInstr& in, const std::vector<std::string>& a) {
  auto A = [&](int i) { return a.at(i); };
  switch (in.op) {
    case Op::ADD: return "(" + A(0) + " + " + A(1) + ")";
    case Op::SUB: return "(" + A(0) + " - " + A(1) + ")";
    case Op::MUL: return "(" + A(0) + " * " + A(1) + ")";
    case Op::DIV: return "pf_div(" + A(0) + ", " + A(1) + ")";
    case Op::POW: return "powf(" + A(0) + ", " + A(1) + ")";
    case Op::MAX_BINARY: case Op::MAXIMUM: return "pf_max(" + A(0) + ", " + A(1) + ")";
    case Op::MIN_BINARY: case Op::MINIMUM: return "pf_min(" + A(0) + ", " + A(1) + ")";
    case Op::NEG: return "(-" + A(0) + ")";
    case Op::ABS: return "fabsf(" + A(0) + ")";
    case Op::SQRT: return "sqrtf(" + A(0) + ")";
    case Op::EXP: return "expf(" + A(0) + ")";
    case Op::LOG: return "logf(" + A(0) + ")";
    case Op::SIN: return "sinf(" + A(0) + ")";
    case Op::COS: return "cosf(" + A(0) + ")";
    case Op::TANH: return "tanhf(" + A(0) + ")";
    case Op::RELU: return "pf_relu(" + A(0) + ")";
    case Op::SIGMOID: return "pf_sigmoid(" + A(0) + ")";
    case Op::GELU: return "pf_gelu(" + A(0) + ")";
    case Op::SILU: return "pf_silu(" + A(0) + ")";
    case Op::EQ: return "((" + A(0) + " == " + A(1) + ") ? 1.0f : 0.0f)";
    case Op::NE: return "((" + A(0) + " != " + A(1) + ") ? 1.0f : 0.0f)";
    case Op::LT: case Op::LESS: return "((" + A(0) + " < " + A(1) + ") ? 1.0f : 0.0f)";
    case Op::LE: return "((" + A(0) + " <= " + A(1) + ") ? 1.0f : 0.0f)";
    case Op::GT: return "((" + A(0) + " > " + A(1) + ") ? 1.0f : 0.0f)";
    case Op::GE: return "((" + A(0) + " >= " + A(1) + ") ? 1.0f : 0.0f)";
    case Op::WHERE: return "((" + A(0) + " != 0.0f) ? " + A(1) + " : " + A(2) + ")";
    case Op::CLAMP: return "fminf(fmaxf(" + A(0) + ", " + A(1) + "), " + A(2) + ")";
    default:
      fail(PFC_ERR_UNSUPPORTED, std::string("no elementwise lowering for op ") + op_name(in.op));
  }
}

// Merged iteration dims shared by a set of views: sizes and, per view, strides.
struct Dims {
  std::vector<int64_t> size;
  std::vector<std::vector<int64_t>> stride;  // [view][dim]
};

// Reorder dims by `perm` and merge neighbours that every view walks contiguously.
Dims merge_dims(const std::vector<int64_t>& space, const std::vector<int>& perm,
                const std::vector<const View*>& views) {
  Dims d;
  size_t nv = views.size();
  d.stride.assign(nv, {});
  for (int p : perm) {
    if (space[p] == 1) continue;
    d.size.push_back(space[p]);
    for (size_t v = 0; v < nv; ++v) d.stride[v].push_back(views[v]->strides[p]);
  }
  if (d.size.empty()) {
    d.size.push_back(1);
    for (size_t v = 0; v < nv; ++v) d.stride[v].push_back(0);
  }
  // merge k-1 into k when stride[k-1] == stride[k]*size[k] for all views
  std::vector<int64_t> ms{d.size[0]};
  std::vector<std::vector<int64_t>> mst(nv);
  for (size_t v = 0; v < nv; ++v) mst[v].push_back(d.stride[v][0]);
  for (size_t k = 1; k < d.size.size(); ++k) {
    bool ok = true;
    for (size_t v = 0; v < nv && ok; ++v) ok = mst[v].back() == d.stride[v][k] * d.size[k];
    if (ok) {
      ms.back() *= d.size[k];
      for (size_t v = 0; v < nv; ++v) mst[v].back() = d.stride[v][k];
    } else {
      ms.push_back(d.size[k]);
      for (size_t v = 0; v < nv; ++v) mst[v].push_back(d.stride[v][k]);
    }
  }
  d.size = ms;
  d.stride = mst;
  return d;
}

// Physical order for iterating `space`: follow the first store (or load)
// whose strides are all nonzero, outermost = largest stride.
std::vector<int> pick_perm(const EwSpec& s) {
  std::vector<int> perm(s.space.size());
  for (size_t i = 0; i < perm.size(); ++i) perm[i] = (int)i;
  const View* ref = nullptr;
  if (!s.stores.empty()) ref = &s.stores[0].second;
  if (!ref) {
    for (const View& v : s.loads) {
      bool full = !v.is_splat;
      for (size_t d = 0; d < v.shape.size() && full; ++d) full = v.shape[d] == 1 || v.strides[d] != 0;
      if (full) { ref = &v; break; }
    }
  }
  if (ref) {
    std::stable_sort(perm.begin(), perm.end(), [&](int a, int b) {
      return std::llabs(ref->strides[a]) > std::llabs(ref->strides[b]);
    });
  }
  return perm;
}

std::string ctype_for(DType d) {
  switch (d) {
    case DType::F32: return "float";
    case DType::F64: return "double";
    case DType::I64: return "long long";
    case DType::I32: return "int";
    case DType::I16: case DType::F16: case DType::BF16: return "unsigned short";
    case DType::I8: case DType::BOOL: return "unsigned char";
  }
  return "float";
}

// Emits index arithmetic: coords of linear index `lin` over `sizes`, into c0..cn-1.
std::string emit_coords(const std::string& lin, const std::vector<int64_t>& sizes, const std::string& pfx,
                        const char* ity) {
  std::ostringstream o;
  size_t n = sizes.size();
  if (n == 1) {
    o << ity << " " << pfx << "0 = " << lin << ";\n";
    return o.str();
  }
  o << ity << " " << pfx << "r = " << lin << ";\n";
  for (size_t k = n; k-- > 0;) {
    if (k == 0) {
      o << ity << " " << pfx << "0 = " << pfx << "r;\n";
    } else {
      o << ity << " " << pfx << k << " = " << pfx << "r % (" << ity << ")" << sizes[k] << "; " << pfx
        << "r /= (" << ity << ")" << sizes[k] << ";\n";
    }
  }
  return o.str();
}

std::string emit_offset(const std::vector<int64_t>& strides, const std::string& pfx, size_t ndims,
                        int skip_last, const char* ity) {
  std::ostringstream o;
  o << "(" << ity << ")0";
  for (size_t k = 0; k + skip_last < ndims; ++k)
    if (strides[k] != 0) o << " + " << pfx << k << " * (" << ity << ")" << strides[k];
  return o.str();
}

bool fits_i32(const Dims& d, int64_t extra) {
  int64_t total = prod(d.size) + extra;
  if (total > (int64_t)INT32_MAX / 2) return false;
  for (const auto& st : d.stride) {
    int64_t m = 0;
    for (size_t k = 0; k < st.size(); ++k) m += std::llabs(st[k]) * (d.size[k] - 1);
    if (m > (int64_t)INT32_MAX / 2) return false;
  }
  return true;
}

// --- fused elementwise kernel ---------------------------------------------
std::string gen_ew(const EwSpec& s, const std::string& name, int num_sms, int* grid, int* block) {
  std::vector<int> perm = pick_perm(s);
  std::vector<const View*> views;
  for (const View& v : s.loads) views.push_back(&v);
  for (const auto& st : s.stores) views.push_back(&st.second);
  Dims d = merge_dims(s.space, perm, views);
  size_t nd = d.size.size();
  int64_t total = prod(d.size);
  // Vector width: 4 when the innermost dim is a multiple of 4 and every view
  // walks it with stride 0 or 1 from a 16-byte aligned base.
  int vec = 4;
  if (d.size.back() % 4 != 0) vec = 1;
  for (size_t v = 0; v < views.size() && vec == 4; ++v) {
    if (views[v]->is_splat) continue;
    if (views[v]->dtype != DType::F32) { vec = 1; break; }
    int64_t inner = d.stride[v].back();
    if (inner == 1) {
      if (views[v]->offset % 4 != 0) vec = 1;
      for (size_t k = 0; k + 1 < nd; ++k)
        if (d.stride[v][k] % 4 != 0) vec = 1;
    }
  }
  bool i32 = fits_i32(d, 0);
  const char* ity = i32 ? "int" : "long long";
  // a pure copy of a non-float tensor keeps its element type end to end
  std::string vt = "float";
  {
    bool pure = !s.loads.empty();
    for (const EwInstr& in : s.instrs) pure = pure && (in.kind == EwKind::LOAD || in.kind == EwKind::COPY);
    for (const View& v : s.loads) pure = pure && !v.is_splat && v.dtype == s.loads[0].dtype;
    for (const auto& st : s.stores) pure = pure && st.second.dtype == s.loads[0].dtype;
    if (pure && s.loads[0].dtype != DType::F32) vt = ctype_for(s.loads[0].dtype);
  }
  std::ostringstream o;
  o << kPrelude;
  o << "extern \"C\" __global__ void __launch_bounds__(256) " << name << "(const PfArgs A) {\n";
  size_t nl = s.loads.size(), ns = s.stores.size();
  for (size_t i = 0; i < nl; ++i) {
    if (s.loads[i].is_splat) continue;
    o << "  const " << ctype_for(s.loads[i].dtype) << "* __restrict__ in" << i << " = (const "
      << ctype_for(s.loads[i].dtype) << "*)A.p[" << i << "];\n";
  }
  for (size_t j = 0; j < ns; ++j)
    o << "  " << ctype_for(s.stores[j].second.dtype) << "* __restrict__ out" << j << " = ("
      << ctype_for(s.stores[j].second.dtype) << "*)A.p[" << nl + j << "];\n";
  o << "  const float* __restrict__ scal = (const float*)A.p[" << nl + ns << "];\n";
  for (size_t i = 0; i < nl; ++i)
    if (s.loads[i].is_splat) o << "  const float sp" << i << " = scal[" << s.loads[i].splat_slot << "];\n";
  o << "  const " << ity << " NV = (" << ity << ")" << total / vec << ";\n";
  o << "  for (" << ity << " v = (" << ity << ")blockIdx.x * blockDim.x + threadIdx.x; v < NV; v += (" << ity
    << ")gridDim.x * blockDim.x) {\n";
  o << "    const " << ity << " L = v * " << vec << ";\n";
  o << "    " << emit_coords("L", d.size, "c", ity);
  // loads
  for (size_t i = 0; i < nl; ++i) {
    const View& lv = s.loads[i];
    std::string ct = ctype_for(lv.dtype);
    if (lv.is_splat) {
      o << "    float l" << i << "[" << vec << "]; for (int q = 0; q < " << vec << "; ++q) l" << i << "[q] = sp" << i
        << ";\n";
      continue;
    }
    const auto& st = d.stride[i];
    o << "    " << ct << " l" << i << "[" << vec << "];\n    { const " << ct << "* ptr = in" << i << " + ("
      << emit_offset(st, "c", nd, 0, ity) << ");\n";
    int64_t inner = st.back();
    if (vec == 4 && inner == 1) {
      o << "      float4 t = *(const float4*)ptr; l" << i << "[0]=t.x; l" << i << "[1]=t.y; l" << i << "[2]=t.z; l"
        << i << "[3]=t.w; }\n";
    } else if (inner == 0) {
      o << "      " << ct << " t = ptr[0]; for (int q = 0; q < " << vec << "; ++q) l" << i << "[q] = t; }\n";
    } else {
      o << "      for (int q = 0; q < " << vec << "; ++q) l" << i << "[q] = ptr[q * (" << ity << ")" << inner
        << "]; }\n";
    }
  }
  // compute
  o << "    " << vt << " res[" << std::max<size_t>(ns, 1) << "][" << vec << "];\n";
  o << "#pragma unroll\n    for (int q = 0; q < " << vec << "; ++q) {\n";
  std::vector<std::string> names(s.instrs.size());
  for (size_t k = 0; k < s.instrs.size(); ++k) {
    const EwInstr& in = s.instrs[k];
    names[k] = "t" + std::to_string(k);
    std::string e;
    if (in.kind == EwKind::LOAD) {
      e = "(" + vt + ")l" + std::to_string(in.load) + "[q]";
    } else if (in.kind == EwKind::COPY) {
      e = names[in.a[0]];
    } else if (in.kind == EwKind::BN) {
      // (x - mean) / sqrt(var + eps) * gamma + beta, args: x, mean, var, gamma, beta
      std::string x = names[in.a[0]], m = names[in.a[1]], v = names[in.a[2]];
      e = "((" + x + " - " + m + ") / sqrtf(" + v + " + " + flit(in.p0) + "))";
      if (in.a[3] >= 0) e = "(" + e + " * " + names[in.a[3]] + ")";
      if (in.a[4] >= 0) e = "(" + e + " + " + names[in.a[4]] + ")";
    } else {
      std::vector<std::string> args;
      for (int x : in.a) args.push_back(names[x]);
      e = op_expr(in, args);
    }
    o << "      const " << vt << " " << names[k] << " = " << e << ";\n";
  }
  for (size_t j = 0; j < ns; ++j) o << "      res[" << j << "][q] = " << names[s.stores[j].first] << ";\n";
  o << "    }\n";
  // stores
  for (size_t j = 0; j < ns; ++j) {
    const View& sv = s.stores[j].second;
    std::string ct = ctype_for(sv.dtype);
    const auto& st = d.stride[nl + j];
    o << "    { " << ct << "* ptr = out" << j << " + (" << emit_offset(st, "c", nd, 0, ity) << ");\n";
    if (vec == 4 && st.back() == 1) {
      o << "      *(float4*)ptr = make_float4(res[" << j << "][0], res[" << j << "][1], res[" << j << "][2], res["
        << j << "][3]); }\n";
    } else {
      o << "      for (int q = 0; q < " << vec << "; ++q) ptr[q * (" << ity << ")" << st.back() << "] = (" << ct
        << ")res[" << j << "][q]; }\n";
    }
  }
  o << "  }\n}\n";
  *block = 256;
  int64_t blocks = ceil_div(std::max<int64_t>(total / vec, 1), 256);
  *grid = (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)num_sms * 16));
  return o.str();
}

// --- row kernel: one row (or a few rows) per CTA, values kept in registers ---
struct RowLayout {
  int64_t R = 1, C = 1;
  int tpr = 32, block = 256, rpb = 8, vec = 1, nch = 1;
  bool reg_mode = true;
};

std::string gen_row(const RowSpec& rs, const std::string& name, int num_sms, int* grid, int* block,
                    size_t* smem_bytes) {
  const EwSpec& s = rs.ew;
  std::vector<int64_t> outer_sz(s.space.begin(), s.space.begin() + rs.red_begin);
  std::vector<int64_t> red_sz(s.space.begin() + rs.red_begin, s.space.begin() + rs.red_end);
  RowLayout L;
  L.R = prod(outer_sz);
  L.C = prod(red_sz);
  // Per-view strides split into row dims and column dims.
  std::vector<const View*> views;
  for (const View& v : s.loads) views.push_back(&v);
  for (const auto& st : s.stores) views.push_back(&st.second);
  for (const RowOp& op : rs.ops)
    if (op.op == Op::SOFTMAX || op.op == Op::LOG_SOFTMAX || op.op == Op::LAYER_NORM) views.push_back(&op.out);
  std::vector<int> rperm, cperm;
  for (int k = 0; k < rs.red_begin; ++k) rperm.push_back(k);
  for (int k = rs.red_begin; k < rs.red_end; ++k) cperm.push_back(k);
  Dims rd = merge_dims(s.space, rperm, views);
  Dims cd = merge_dims(s.space, cperm, views);
  size_t nrd = rd.size.size(), ncd = cd.size.size();
  // vector width along the column
  L.vec = (cd.size.back() % 4 == 0) ? 4 : 1;
  for (size_t v = 0; v < views.size() && L.vec == 4; ++v) {
    if (views[v]->is_splat) continue;
    int64_t inner = cd.stride[v].back();
    if (inner == 1) {
      if (views[v]->offset % 4) L.vec = 1;
      for (size_t k = 0; k + 1 < ncd; ++k)
        if (cd.stride[v][k] % 4) L.vec = 1;
      for (size_t k = 0; k < nrd; ++k)
        if (rd.stride[v][k] % 4) L.vec = 1;
    }
  }
  int64_t nvec = ceil_div(L.C, L.vec);
  // threads per row: about four vector chunks per thread.  Measured on the
  // 8192x4096 sum/mean/max/LayerNorm graph: two chunks per thread (512
  // threads) doubled active warps but added 30% instructions and barrier
  // stalls and ran 4% slower than four chunks (256 threads).
  int tpr = 32;
  while (tpr < 1024 && (int64_t)tpr * 4 < nvec) tpr *= 2;
  L.tpr = tpr;
  L.block = std::max(256, tpr);
  L.rpb = L.block / tpr;
  L.nch = (int)ceil_div(nvec, tpr);
  int nsrc = 0;
  {
    std::set<int> srcs;
    for (const RowOp& op : rs.ops) srcs.insert(op.src);
    nsrc = (int)srcs.size();
  }
  L.reg_mode = (int64_t)L.nch * L.vec * std::max(1, nsrc) <= 64;
  bool i32 = fits_i32(rd, 0) && fits_i32(cd, 0) && L.R * L.C < (int64_t)INT32_MAX / 2;
  const char* ity = i32 ? "int" : "long long";
  size_t nl = s.loads.size(), ns = s.stores.size();

  // TMA row streaming: when every per-row input is a contiguous, 16-byte
  // aligned row, a ring of shared-memory stages is filled with 1-D bulk copies
  // for the rows ahead while the CTA computes the current one.  Inputs that
  // do not vary by row (LayerNorm gamma/beta) stay ordinary loads.
  std::vector<int> tma_slot(nl, -1);
  int n_tma = 0;
  bool tma = L.reg_mode && L.rpb == 1 && L.vec == 4 && ncd == 1 && (L.C * 4) % 16 == 0;
  for (size_t i = 0; i < nl && tma; ++i) {
    const View& lv = s.loads[i];
    if (lv.is_splat) continue;
    bool row_const = true;
    for (size_t k = 0; k < nrd; ++k) row_const = row_const && rd.stride[i][k] == 0;
    if (row_const) continue;
    bool contiguous = cd.stride[i][0] == 1 && lv.offset % 4 == 0 && lv.dtype == DType::F32;
    for (size_t k = 0; k < nrd; ++k) contiguous = contiguous && rd.stride[i][k] % 4 == 0;
    if (!contiguous) tma = false;
    else tma_slot[i] = n_tma++;
  }
  const int64_t stage_bytes = (int64_t)n_tma * L.C * 4;
  int stages = 0;
  if (tma && n_tma > 0 && stage_bytes * 2 <= 110 * 1024) {
    stages = (int)std::min<int64_t>(4, (110 * 1024) / stage_bytes);
  } else {
    tma = false;
  }
  *smem_bytes = tma ? (size_t)(stages * stage_bytes + 64) : 0;

  // which instructions feed the row ops / stores; all are computed per element
  std::ostringstream o;
  o << kPrelude;
  if (tma) o << kTmaPrelude;
  o << "extern \"C\" __global__ void __launch_bounds__(" << L.block << ") " << name << "(const PfArgs A) {\n";
  for (size_t i = 0; i < nl; ++i) {
    if (s.loads[i].is_splat) continue;
    o << "  const float* __restrict__ in" << i << " = (const float*)A.p[" << i << "];\n";
  }
  for (size_t j = 0; j < ns; ++j) o << "  float* __restrict__ out" << j << " = (float*)A.p[" << nl + j << "];\n";
  size_t nops = rs.ops.size();
  for (size_t r = 0; r < nops; ++r) o << "  float* __restrict__ ro" << r << " = (float*)A.p[" << nl + ns + r << "];\n";
  o << "  const float* __restrict__ scal = (const float*)A.p[" << nl + ns + nops << "];\n";
  {
    // operand outputs follow the error flag: hi, lo per row op that has them
    size_t k = nl + ns + nops + 2;
    for (size_t r = 0; r < nops; ++r) {
      if (rs.ops[r].op_hi < 0) continue;
      o << "  float* __restrict__ oph" << r << " = (float*)A.p[" << k++ << "];\n";
      o << "  float* __restrict__ opl" << r << " = (float*)A.p[" << k++ << "];\n";
    }
  }
  for (size_t i = 0; i < nl; ++i)
    if (s.loads[i].is_splat) o << "  const float sp" << i << " = scal[" << s.loads[i].splat_slot << "];\n";
  const int TPR = L.tpr, RPB = L.rpb, VEC = L.vec, NCH = L.nch;
  o << "  const int tid = threadIdx.x;\n  const int lr = tid % " << TPR << ";\n  const int rib = tid / " << TPR
    << ";\n";
  if (TPR > 32) o << "  __shared__ float red[" << L.block / 32 << "][8];\n";
  if (tma) {
    o << "  int* err = (int*)A.p[" << nl + ns + rs.ops.size() + 1 << "];\n";
    o << "  extern __shared__ __align__(128) unsigned char pf_dyn[];\n";
    o << "  float* stg = (float*)pf_dyn;\n";
    o << "  unsigned long long* bars = (unsigned long long*)(pf_dyn + " << stages * stage_bytes << ");\n";
    // rows of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...
    o << "  const " << ity << " nmine = (" << ity << ")blockIdx.x < (" << ity << ")" << L.R << " ? ((" << ity << ")"
      << L.R << " - 1 - blockIdx.x) / gridDim.x + 1 : 0;\n";
    o << "  auto issue = [&](" << ity << " it) {\n    const " << ity << " row = (" << ity
      << ")blockIdx.x + it * gridDim.x;\n    const int st = (int)(it % " << stages << ");\n";
    o << "    " << emit_coords("row", rd.size, "q", ity);
    o << "    const unsigned bar = pf_smem(&bars[st]);\n    pf_expect_tx(bar, " << stage_bytes << "u);\n";
    for (size_t i = 0; i < nl; ++i) {
      if (tma_slot[i] < 0) continue;
      o << "    pf_bulk_load(pf_smem(stg + (size_t)st * " << stage_bytes / 4 << " + " << tma_slot[i] * L.C
        << "), in" << i << " + (" << emit_offset(rd.stride[i], "q", nrd, 0, ity) << "), " << L.C * 4 << "u, bar);\n";
    }
    o << "  };\n";
    o << "  if (tid == 0) {\n    for (int s2 = 0; s2 < " << stages << "; ++s2) pf_mbar_init(pf_smem(&bars[s2]), 1);\n"
      << "    asm volatile(\"fence.mbarrier_init.release.cluster;\" ::: \"memory\");\n  }\n  __syncthreads();\n";
    o << "  if (tid == 0)\n    for (" << ity << " it = 0; it < nmine && it < " << stages << "; ++it) issue(it);\n";
  }
  // reduction helpers over the TPR threads of a row
  auto reduce = [&](const std::string& var, const std::string& combine, int slot) {
    std::ostringstream r;
    r << "    for (int off = 16; off > 0; off >>= 1) { float ot = __shfl_xor_sync(0xffffffffu, " << var
      << ", off); " << var << " = " << combine << "; }\n";
    if (TPR > 32) {
      int wpr = TPR / 32;
      r << "    __syncthreads();\n    if ((tid & 31) == 0) red[tid >> 5][" << slot << "] = " << var << ";\n"
        << "    __syncthreads();\n    { const int w0 = rib * " << wpr << "; " << var << " = red[w0][" << slot
        << "];\n      for (int w = 1; w < " << wpr << "; ++w) { float ot = red[w0 + w][" << slot << "]; " << var
        << " = " << combine << "; } }\n";
    }
    return r.str();
  };
  if (tma) {
    o << "  for (" << ity << " it = 0; it < nmine; ++it) {\n    const " << ity << " row = (" << ity
      << ")blockIdx.x + it * gridDim.x;\n    const bool rv = true;\n    const int st = (int)(it % " << stages
      << ");\n    pf_mbar_wait(pf_smem(&bars[st]), (unsigned)((it / " << stages << ") & 1), err);\n"
      << "    const float* stgp = stg + (size_t)st * " << stage_bytes / 4 << ";\n";
  } else {
    o << "  for (" << ity << " rbase = (" << ity << ")blockIdx.x * " << RPB << "; rbase < (" << ity << ")" << L.R
      << "; rbase += (" << ity << ")gridDim.x * " << RPB << ") {\n";
    o << "    const " << ity << " row = rbase + rib;\n    const bool rv = row < (" << ity << ")" << L.R << ";\n";
  }
  o << "    " << emit_coords("(rv ? row : (" + std::string(ity) + ")0)", rd.size, "r", ity);
  // per-view row offsets
  for (size_t v = 0; v < views.size(); ++v)
    o << "    const " << ity << " ro_" << v << " = " << emit_offset(rd.stride[v], "r", nrd, 0, ity) << ";\n";
  // element evaluation macro: computes instr values for column vector chunk `cv` into arrays
  std::vector<int> srcs;
  for (const RowOp& op : rs.ops)
    if (std::find(srcs.begin(), srcs.end(), op.src) == srcs.end()) srcs.push_back(op.src);
  auto src_idx = [&](int instr) { return (int)(std::find(srcs.begin(), srcs.end(), instr) - srcs.begin()); };
  // Instructions needed to produce `roots` (the DAG is in index order).
  auto closure = [&](const std::vector<int>& roots) {
    std::vector<bool> need(s.instrs.size(), false);
    for (int r : roots)
      if (r >= 0) need[r] = true;
    for (int k = (int)s.instrs.size() - 1; k >= 0; --k)
      if (need[k])
        for (int a : s.instrs[k].a)
          if (a >= 0) need[a] = true;
    return need;
  };
  std::vector<bool> all_needed(s.instrs.size(), true);
  // Evaluates the prologue for column chunk `cv`, restricted to `need`.
  auto emit_eval = [&](bool with_stores, const std::vector<bool>& need) {
    std::vector<bool> load_needed(nl, false);
    for (size_t k = 0; k < s.instrs.size(); ++k)
      if (need[k] && s.instrs[k].kind == EwKind::LOAD) load_needed[s.instrs[k].load] = true;
    std::ostringstream e;
    e << "      const " << ity << " cl = cv * " << VEC << ";\n";
    e << "      const bool cok = rv && cl < (" << ity << ")" << L.C << ";\n";
    e << "      " << emit_coords("(cok ? cl : (" + std::string(ity) + ")0)", cd.size, "k", ity);
    for (size_t i = 0; i < nl; ++i) {
      if (!load_needed[i]) continue;
      if (s.loads[i].is_splat) {
        e << "      float l" << i << "[" << VEC << "]; for (int q = 0; q < " << VEC << "; ++q) l" << i << "[q] = sp"
          << i << ";\n";
        continue;
      }
      const auto& st = cd.stride[i];
      if (tma_slot[i] >= 0)  // staged in shared memory by the bulk copy of this row
        e << "      float l" << i << "[" << VEC << "];\n      if (cok) { const float* ptr = stgp + "
          << tma_slot[i] * L.C << " + (" << emit_offset(st, "k", ncd, 0, ity) << ");\n";
      else
        e << "      float l" << i << "[" << VEC << "];\n      if (cok) { const float* ptr = in" << i << " + ro_" << i
          << " + (" << emit_offset(st, "k", ncd, 0, ity) << ");\n";
      if (VEC == 4 && st.back() == 1)
        e << "        float4 t = *(const float4*)ptr; l" << i << "[0]=t.x; l" << i << "[1]=t.y; l" << i
          << "[2]=t.z; l" << i << "[3]=t.w; }\n";
      else if (st.back() == 0)
        e << "        float t = ptr[0]; for (int q = 0; q < " << VEC << "; ++q) l" << i << "[q] = t; }\n";
      else
        e << "        for (int q = 0; q < " << VEC << "; ++q) l" << i << "[q] = ptr[q * (" << ity << ")"
          << st.back() << "]; }\n";
      e << "      else { for (int q = 0; q < " << VEC << "; ++q) l" << i << "[q] = 0.f; }\n";
    }
    e << "      float ev[" << std::max<size_t>(s.instrs.size(), 1) << "][" << VEC << "];\n";
    e << "#pragma unroll\n      for (int q = 0; q < " << VEC << "; ++q) {\n";
    for (size_t k = 0; k < s.instrs.size(); ++k) {
      if (!need[k]) continue;
      const EwInstr& in = s.instrs[k];
      std::string ex;
      auto nm = [&](int x) { return "ev[" + std::to_string(x) + "][q]"; };
      if (in.kind == EwKind::LOAD) ex = "l" + std::to_string(in.load) + "[q]";
      else if (in.kind == EwKind::COPY) ex = nm(in.a[0]);
      else if (in.kind == EwKind::BN) {
        ex = "((" + nm(in.a[0]) + " - " + nm(in.a[1]) + ") / sqrtf(" + nm(in.a[2]) + " + " + flit(in.p0) + "))";
        if (in.a[3] >= 0) ex = "(" + ex + " * " + nm(in.a[3]) + ")";
        if (in.a[4] >= 0) ex = "(" + ex + " + " + nm(in.a[4]) + ")";
      } else {
        std::vector<std::string> args;
        for (int x : in.a) args.push_back(nm(x));
        ex = op_expr(in, args);
      }
      e << "        ev[" << k << "][q] = " << ex << ";\n";
    }
    e << "      }\n";
    if (with_stores) {
      for (size_t j = 0; j < ns; ++j) {
        const auto& st = cd.stride[nl + j];
        e << "      if (cok) { float* ptr = out" << j << " + ro_" << nl + j << " + ("
          << emit_offset(st, "k", ncd, 0, ity) << ");\n";
        int ins = s.stores[j].first;
        if (VEC == 4 && st.back() == 1)
          e << "        *(float4*)ptr = make_float4(ev[" << ins << "][0], ev[" << ins << "][1], ev[" << ins
            << "][2], ev[" << ins << "][3]); }\n";
        else
          e << "        for (int q = 0; q < " << VEC << "; ++q) ptr[q * (" << ity << ")" << st.back() << "] = ev["
            << ins << "][q]; }\n";
      }
    }
    return e.str();
  };
  // Which stats are needed per source
  std::set<int> need_sum, need_max, need_min, need_prod, need_var, need_sexp;
  for (const RowOp& op : rs.ops) {
    int si = src_idx(op.src);
    switch (op.op) {
      case Op::SUM: case Op::MEAN: need_sum.insert(si); break;
      case Op::MAX: need_max.insert(si); break;
      case Op::MIN: need_min.insert(si); break;
      case Op::PROD: need_prod.insert(si); break;
      case Op::LAYER_NORM: need_sum.insert(si); need_var.insert(si); break;
      case Op::SOFTMAX: case Op::LOG_SOFTMAX: need_max.insert(si); need_sexp.insert(si); break;
      default: break;
    }
  }
  // pass 1: evaluate, keep source values (register mode), accumulate sum/max/min/prod
  for (size_t si = 0; si < srcs.size(); ++si) {
    o << "    float s_sum" << si << " = 0.f, s_max" << si << " = -PF_INF, s_min" << si << " = PF_INF, s_prod" << si
      << " = 1.f, s_var" << si << " = 0.f, s_sexp" << si << " = 0.f;\n";
    if (L.reg_mode) o << "    float vals" << si << "[" << NCH << "][" << VEC << "];\n";
  }
  o << (L.reg_mode ? "#pragma unroll\n" : "#pragma unroll 1\n") << "    for (int ch = 0; ch < " << NCH << "; ++ch) {\n      const " << ity
    << " cv = (" << ity << ")ch * " << TPR << " + lr;\n";
  o << emit_eval(true, all_needed);
  for (size_t si = 0; si < srcs.size(); ++si) {
    o << "      for (int q = 0; q < " << VEC << "; ++q) {\n        const bool ok = cok && (cl + q) < (" << ity << ")"
      << L.C << ";\n        const float x = ev[" << srcs[si] << "][q];\n";
    if (L.reg_mode) o << "        vals" << si << "[ch][q] = x;\n";
    if (need_sum.count(si)) o << "        if (ok) s_sum" << si << " += x;\n";
    if (need_max.count(si)) o << "        if (ok) s_max" << si << " = fmaxf(s_max" << si << ", x);\n";
    if (need_min.count(si)) o << "        if (ok) s_min" << si << " = fminf(s_min" << si << ", x);\n";
    if (need_prod.count(si)) o << "        if (ok) s_prod" << si << " *= x;\n";
    o << "      }\n";
  }
  o << "    }\n";
  // One reduction round for several statistics: warp shuffles, then (rows
  // wider than a warp) one shared-memory exchange between two barriers.
  // `between` is emitted after the first barrier, when every thread of the
  // CTA has finished the pass that precedes the round.
  auto reduce_round = [&](const std::vector<std::pair<std::string, std::string>>& vals, const std::string& between) {
    std::ostringstream r;
    for (auto& [v, comb] : vals)
      r << "    for (int off = 16; off > 0; off >>= 1) { float ot = __shfl_xor_sync(0xffffffffu, " << v
        << ", off); " << v << " = " << comb << "; }\n";
    if (TPR > 32) {
      const int wpr = TPR / 32;
      r << "    __syncthreads();\n" << between;
      r << "    if ((tid & 31) == 0) {\n";
      for (size_t k = 0; k < vals.size(); ++k) r << "      red[tid >> 5][" << k << "] = " << vals[k].first << ";\n";
      r << "    }\n    __syncthreads();\n    { const int w0 = rib * " << wpr << ";\n";
      for (size_t k = 0; k < vals.size(); ++k)
        r << "      " << vals[k].first << " = red[w0][" << k << "];\n      for (int w = 1; w < " << wpr
          << "; ++w) { float ot = red[w0 + w][" << k << "]; " << vals[k].first << " = " << vals[k].second
          << "; }\n";
      r << "    }\n";
    } else {
      r << between;
    }
    return r.str();
  };
  (void)reduce;
  {
    std::vector<std::pair<std::string, std::string>> round1;
    for (size_t si = 0; si < srcs.size(); ++si) {
      std::string i = std::to_string(si);
      if (need_sum.count(si)) round1.push_back({"s_sum" + i, "s_sum" + i + " + ot"});
      if (need_max.count(si)) round1.push_back({"s_max" + i, "fmaxf(s_max" + i + ", ot)"});
      if (need_min.count(si)) round1.push_back({"s_min" + i, "fminf(s_min" + i + ", ot)"});
      if (need_prod.count(si)) round1.push_back({"s_prod" + i, "s_prod" + i + " * ot"});
    }
    if (round1.size() > 8) fail(PFC_ERR_UNSUPPORTED, "row group with more than 8 statistics");
    std::string refill = tma ? "    if (tid == 0 && it + " + std::to_string(stages) + " < nmine) issue(it + " +
                                   std::to_string(stages) + ");\n"
                             : "";
    o << reduce_round(round1, refill);
  }
  // pass 2: variance / sum of exp (need pass-1 stats)
  bool need_pass2 = !need_var.empty() || !need_sexp.empty();
  if (need_pass2) {
    for (size_t si = 0; si < srcs.size(); ++si)
      if (need_var.count(si)) o << "    const float mean" << si << " = s_sum" << si << " / " << flit((float)L.C) << ";\n";
    o << (L.reg_mode ? "#pragma unroll\n" : "#pragma unroll 1\n") << "    for (int ch = 0; ch < " << NCH << "; ++ch) {\n      const " << ity << " cv = ("
      << ity << ")ch * " << TPR << " + lr;\n";
    if (!L.reg_mode) o << emit_eval(false, closure(srcs));
    else o << "      const " << ity << " cl = cv * " << VEC << ";\n      const bool cok = rv && cl < (" << ity << ")" << L.C << ";\n";
    for (size_t si = 0; si < srcs.size(); ++si) {
      if (!need_var.count(si) && !need_sexp.count(si)) continue;
      o << "      for (int q = 0; q < " << VEC << "; ++q) {\n        const bool ok = cok && (cl + q) < (" << ity
        << ")" << L.C << ";\n";
      o << "        const float x = " << (L.reg_mode ? "vals" + std::to_string(si) + "[ch][q]" : "ev[" + std::to_string(srcs[si]) + "][q]") << ";\n";
      if (need_var.count(si)) o << "        if (ok) { const float dv = x - mean" << si << "; s_var" << si << " += dv * dv; }\n";
      if (need_sexp.count(si)) o << "        if (ok) s_sexp" << si << " += expf(x - s_max" << si << ");\n";
      o << "      }\n";
    }
    o << "    }\n";
    std::vector<std::pair<std::string, std::string>> round2;
    for (size_t si = 0; si < srcs.size(); ++si) {
      std::string i = std::to_string(si);
      if (need_var.count(si)) round2.push_back({"s_var" + i, "s_var" + i + " + ot"});
      if (need_sexp.count(si)) round2.push_back({"s_sexp" + i, "s_sexp" + i + " + ot"});
    }
    if (round2.size() > 8) fail(PFC_ERR_UNSUPPORTED, "row group with more than 8 statistics");
    o << reduce_round(round2, "");
  }
  // per-row outputs
  bool any_row_out = false;
  for (size_t r = 0; r < nops; ++r) {
    const RowOp& op = rs.ops[r];
    int si = src_idx(op.src);
    std::string v;
    switch (op.op) {
      case Op::SUM: v = "s_sum" + std::to_string(si); break;
      case Op::MEAN: v = "s_sum" + std::to_string(si) + " / " + flit((float)L.C); break;
      case Op::MAX: v = "s_max" + std::to_string(si); break;
      case Op::MIN: v = "s_min" + std::to_string(si); break;
      case Op::PROD: v = "s_prod" + std::to_string(si); break;
      default: continue;
    }
    if (!any_row_out) { o << "    if (rv && lr == 0) {\n"; any_row_out = true; }
    o << "      ro" << r << "[row] = " << v << ";\n";
  }
  if (any_row_out) o << "    }\n";
  // per-element outputs: softmax / log_softmax / layer_norm
  bool any_elem = false;
  for (const RowOp& op : rs.ops)
    if (op.op == Op::SOFTMAX || op.op == Op::LOG_SOFTMAX || op.op == Op::LAYER_NORM) any_elem = true;
  if (any_elem) {
    for (size_t si = 0; si < srcs.size(); ++si) {
      if (need_var.count(si))
        o << "    const float inv" << si << " = 1.0f / sqrtf(s_var" << si << " / " << flit((float)L.C) << " + EPS" << si << ");\n";
      if (need_sexp.count(si)) o << "    const float lse" << si << " = s_max" << si << " + logf(s_sexp" << si << ");\n";
    }
    o << (L.reg_mode ? "#pragma unroll\n" : "#pragma unroll 1\n") << "    for (int ch = 0; ch < " << NCH << "; ++ch) {\n      const " << ity << " cv = ("
      << ity << ")ch * " << TPR << " + lr;\n";
    bool needs_eval = !L.reg_mode;
    std::vector<int> roots = L.reg_mode ? std::vector<int>{} : srcs;
    for (const RowOp& op : rs.ops)
      if (op.op == Op::LAYER_NORM && (op.gamma >= 0 || op.beta >= 0)) {
        needs_eval = true;
        roots.push_back(op.gamma);
        roots.push_back(op.beta);
      }
    if (needs_eval) o << emit_eval(false, closure(roots));
    else o << "      const " << ity << " cl = cv * " << VEC << ";\n      const bool cok = rv && cl < (" << ity << ")" << L.C << ";\n";
    o << "      " << emit_coords("(cok ? cl : (" + std::string(ity) + ")0)", cd.size, "w", ity);
    size_t vbase = nl + ns;
    for (size_t r = 0; r < nops; ++r) {
      const RowOp& op = rs.ops[r];
      if (!(op.op == Op::SOFTMAX || op.op == Op::LOG_SOFTMAX || op.op == Op::LAYER_NORM)) continue;
      int si = src_idx(op.src);
      // view index of this op's output in `views`
      size_t vi = vbase;
      for (size_t r2 = 0; r2 < r; ++r2)
        if (rs.ops[r2].op == Op::SOFTMAX || rs.ops[r2].op == Op::LOG_SOFTMAX || rs.ops[r2].op == Op::LAYER_NORM) ++vi;
      const auto& st = cd.stride[vi];
      o << "      { float y[" << VEC << "];\n        for (int q = 0; q < " << VEC << "; ++q) {\n          const float x = "
        << (L.reg_mode ? "vals" + std::to_string(si) + "[ch][q]" : "ev[" + std::to_string(op.src) + "][q]") << ";\n";
      if (op.op == Op::SOFTMAX)
        o << "          y[q] = expf(x - s_max" << si << ") / s_sexp" << si << ";\n";
      else if (op.op == Op::LOG_SOFTMAX)
        o << "          y[q] = x - lse" << si << ";\n";
      else {
        o << "          float t = (x - mean" << si << ") * inv" << si << ";\n";
        if (op.gamma >= 0) o << "          t = t * ev[" << op.gamma << "][q];\n";
        if (op.beta >= 0) o << "          t = t + ev[" << op.beta << "][q];\n";
        o << "          y[q] = t;\n";
      }
      o << "        }\n        if (cok) { const " << ity << " off = ro_" << vi << " + ("
        << emit_offset(st, "w", ncd, 0, ity) << ");\n";
      if (op.write_out) {
        if (VEC == 4 && st.back() == 1)
          o << "          *(float4*)(ro" << r << " + off) = make_float4(y[0], y[1], y[2], y[3]);\n";
        else
          o << "          for (int q = 0; q < " << VEC << "; ++q) if (cl + q < (" << ity << ")" << L.C << ") ro" << r
            << "[off + q * (" << ity << ")" << st.back() << "] = y[q];\n";
      }
      if (op.op_hi >= 0) {
        // dense row-major `out`: the operand element shares its offset.  With
        // whole, 16-byte aligned 4-element chunks (as the float4 store of `out`
        // above needs) hi and lo go out as one float4 each, not eight scalars.
        if (VEC == 4 && st.back() == 1)
          o << "          { float4 h4, l4;\n            pf_split(y[0], h4.x, l4.x); pf_split(y[1], h4.y, l4.y);\n"
            << "            pf_split(y[2], h4.z, l4.z); pf_split(y[3], h4.w, l4.w);\n            *(float4*)(oph" << r
            << " + off) = h4;\n            *(float4*)(opl" << r << " + off) = l4; }\n";
        else
          o << "          for (int q = 0; q < " << VEC << "; ++q) if (cl + q < (" << ity << ")" << L.C
            << ") { float h, l; pf_split(y[q], h, l); oph" << r << "[off + q] = h; opl" << r << "[off + q] = l; }\n";
      }
      o << "        } }\n";
    }
    o << "    }\n";
  }
  o << "  }\n}\n";
  // substitute eps constants
  std::string src = o.str();
  for (size_t si = 0; si < srcs.size(); ++si) {
    float eps = 1e-5f;
    for (const RowOp& op : rs.ops)
      if (op.op == Op::LAYER_NORM && src_idx(op.src) == (int)si) eps = op.eps;
    std::string key = "EPS" + std::to_string(si);
    size_t p;
    while ((p = src.find(key)) != std::string::npos) src.replace(p, key.size(), flit(eps));
  }
  *block = L.block;
  int64_t blocks = ceil_div(L.R, L.rpb);
  int per_sm = std::max(1, 2048 / L.block);
  *grid = (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)num_sms * per_sm));
  return src;
}

// --- column kernel: reduction over a dim that is not innermost --------------
// Each thread owns one (outer, inner) position and walks the reduced extent.
std::string gen_col(const RowSpec& rs, const std::string& name, int num_sms, int* grid, int* block) {
  const EwSpec& s = rs.ew;
  std::vector<int64_t> outer_sz(s.space.begin(), s.space.begin() + rs.red_begin);
  std::vector<int64_t> inner_sz(s.space.begin() + rs.red_end, s.space.end());
  std::vector<int64_t> red_sz(s.space.begin() + rs.red_begin, s.space.begin() + rs.red_end);
  int64_t O = prod(outer_sz), I = prod(inner_sz), C = prod(red_sz);
  std::vector<const View*> views;
  for (const View& v : s.loads) views.push_back(&v);
  for (const auto& st : s.stores) views.push_back(&st.second);
  for (const RowOp& op : rs.ops)
    if (op.op == Op::SOFTMAX || op.op == Op::LOG_SOFTMAX || op.op == Op::LAYER_NORM) views.push_back(&op.out);
  std::vector<int> operm, iperm, cperm;
  for (int k = 0; k < rs.red_begin; ++k) operm.push_back(k);
  for (int k = rs.red_end; k < (int)s.space.size(); ++k) iperm.push_back(k);
  for (int k = rs.red_begin; k < rs.red_end; ++k) cperm.push_back(k);
  // merge outer and inner as one "position" space (outer-major)
  std::vector<int> pperm = operm;
  pperm.insert(pperm.end(), iperm.begin(), iperm.end());
  Dims pd = merge_dims(s.space, pperm, views);
  Dims cd = merge_dims(s.space, cperm, views);
  size_t npd = pd.size.size(), ncd = cd.size.size();
  const char* ity = "long long";
  std::ostringstream o;
  o << kPrelude;
  o << "extern \"C\" __global__ void __launch_bounds__(256) " << name << "(const PfArgs A) {\n";
  size_t nl = s.loads.size(), ns = s.stores.size(), nops = rs.ops.size();
  for (size_t i = 0; i < nl; ++i)
    if (!s.loads[i].is_splat) o << "  const float* __restrict__ in" << i << " = (const float*)A.p[" << i << "];\n";
  for (size_t j = 0; j < ns; ++j) o << "  float* __restrict__ out" << j << " = (float*)A.p[" << nl + j << "];\n";
  for (size_t r = 0; r < nops; ++r) o << "  float* __restrict__ ro" << r << " = (float*)A.p[" << nl + ns + r << "];\n";
  o << "  const float* __restrict__ scal = (const float*)A.p[" << nl + ns + nops << "];\n";
  for (size_t i = 0; i < nl; ++i)
    if (s.loads[i].is_splat) o << "  const float sp" << i << " = scal[" << s.loads[i].splat_slot << "];\n";
  o << "  for (long long pos = (long long)blockIdx.x * blockDim.x + threadIdx.x; pos < " << O * I
    << "LL; pos += (long long)gridDim.x * blockDim.x) {\n";
  o << "    " << emit_coords("pos", pd.size, "p", ity);
  for (size_t v = 0; v < views.size(); ++v)
    o << "    const long long po_" << v << " = " << emit_offset(pd.stride[v], "p", npd, 0, ity) << ";\n";
  std::vector<int> srcs;
  for (const RowOp& op : rs.ops)
    if (std::find(srcs.begin(), srcs.end(), op.src) == srcs.end()) srcs.push_back(op.src);
  auto src_idx = [&](int instr) { return (int)(std::find(srcs.begin(), srcs.end(), instr) - srcs.begin()); };
  auto emit_eval = [&](bool with_stores) {
    std::ostringstream e;
    e << "      " << emit_coords("cc", cd.size, "k", ity);
    for (size_t i = 0; i < nl; ++i) {
      if (s.loads[i].is_splat) { e << "      const float l" << i << " = sp" << i << ";\n"; continue; }
      e << "      const float l" << i << " = in" << i << "[po_" << i << " + " << emit_offset(cd.stride[i], "k", ncd, 0, ity)
        << "];\n";
    }
    for (size_t k = 0; k < s.instrs.size(); ++k) {
      const EwInstr& in = s.instrs[k];
      std::string ex;
      auto nm = [&](int x) { return "e" + std::to_string(x); };
      if (in.kind == EwKind::LOAD) ex = "l" + std::to_string(in.load);
      else if (in.kind == EwKind::COPY) ex = nm(in.a[0]);
      else if (in.kind == EwKind::BN) {
        ex = "((" + nm(in.a[0]) + " - " + nm(in.a[1]) + ") / sqrtf(" + nm(in.a[2]) + " + " + flit(in.p0) + "))";
        if (in.a[3] >= 0) ex = "(" + ex + " * " + nm(in.a[3]) + ")";
        if (in.a[4] >= 0) ex = "(" + ex + " + " + nm(in.a[4]) + ")";
      } else {
        std::vector<std::string> args;
        for (int x : in.a) args.push_back(nm(x));
        ex = op_expr(in, args);
      }
      e << "      const float e" << k << " = " << ex << ";\n";
    }
    if (with_stores)
      for (size_t j = 0; j < ns; ++j)
        e << "      out" << j << "[po_" << nl + j << " + " << emit_offset(cd.stride[nl + j], "k", ncd, 0, ity)
          << "] = e" << s.stores[j].first << ";\n";
    return e.str();
  };
  for (size_t si = 0; si < srcs.size(); ++si)
    o << "    float s_sum" << si << " = 0.f, s_max" << si << " = -PF_INF, s_min" << si << " = PF_INF, s_prod" << si
      << " = 1.f, s_var" << si << " = 0.f, s_sexp" << si << " = 0.f;\n";
  o << "    for (long long cc = 0; cc < " << C << "LL; ++cc) {\n" << emit_eval(true);
  for (size_t si = 0; si < srcs.size(); ++si)
    o << "      s_sum" << si << " += e" << srcs[si] << "; s_max" << si << " = fmaxf(s_max" << si << ", e" << srcs[si]
      << "); s_min" << si << " = fminf(s_min" << si << ", e" << srcs[si] << "); s_prod" << si << " *= e" << srcs[si]
      << ";\n";
  o << "    }\n";
  bool pass2 = false, elem = false;
  for (const RowOp& op : rs.ops) {
    if (op.op == Op::LAYER_NORM || op.op == Op::SOFTMAX || op.op == Op::LOG_SOFTMAX) pass2 = elem = true;
  }
  if (pass2) {
    for (size_t si = 0; si < srcs.size(); ++si) o << "    const float mean" << si << " = s_sum" << si << " / " << flit((float)C) << ";\n";
    o << "    for (long long cc = 0; cc < " << C << "LL; ++cc) {\n" << emit_eval(false);
    for (size_t si = 0; si < srcs.size(); ++si)
      o << "      { const float dv = e" << srcs[si] << " - mean" << si << "; s_var" << si << " += dv * dv; s_sexp" << si
        << " += expf(e" << srcs[si] << " - s_max" << si << "); }\n";
    o << "    }\n";
  }
  for (size_t r = 0; r < nops; ++r) {
    const RowOp& op = rs.ops[r];
    int si = src_idx(op.src);
    std::string v;
    switch (op.op) {
      case Op::SUM: v = "s_sum" + std::to_string(si); break;
      case Op::MEAN: v = "s_sum" + std::to_string(si) + " / " + flit((float)C); break;
      case Op::MAX: v = "s_max" + std::to_string(si); break;
      case Op::MIN: v = "s_min" + std::to_string(si); break;
      case Op::PROD: v = "s_prod" + std::to_string(si); break;
      default: continue;
    }
    o << "    ro" << r << "[pos] = " << v << ";\n";
  }
  if (elem) {
    o << "    for (long long cc = 0; cc < " << C << "LL; ++cc) {\n" << emit_eval(false);
    size_t vi = nl + ns;
    for (size_t r = 0; r < nops; ++r) {
      const RowOp& op = rs.ops[r];
      if (!(op.op == Op::SOFTMAX || op.op == Op::LOG_SOFTMAX || op.op == Op::LAYER_NORM)) continue;
      int si = src_idx(op.src);
      std::string x = "e" + std::to_string(op.src), y;
      if (op.op == Op::SOFTMAX) y = "expf(" + x + " - s_max" + std::to_string(si) + ") / s_sexp" + std::to_string(si);
      else if (op.op == Op::LOG_SOFTMAX)
        y = x + " - (s_max" + std::to_string(si) + " + logf(s_sexp" + std::to_string(si) + "))";
      else {
        y = "(" + x + " - mean" + std::to_string(si) + ") * (1.0f / sqrtf(s_var" + std::to_string(si) + " / " +
            flit((float)C) + " + " + flit(op.eps) + "))";
        if (op.gamma >= 0) y = "(" + y + ") * e" + std::to_string(op.gamma);
        if (op.beta >= 0) y = "(" + y + ") + e" + std::to_string(op.beta);
      }
      o << "      ro" << r << "[po_" << vi << " + " << emit_offset(cd.stride[vi], "k", ncd, 0, ity) << "] = " << y << ";\n";
      ++vi;
    }
    o << "    }\n";
  }
  o << "  }\n}\n";
  *block = 256;
  *grid = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(O * I, 256), (int64_t)num_sms * 8));
  return o.str();
}

// --- full reduction: two kernels (per-CTA partials, then one CTA) ----------
std::string gen_full(const RowSpec& rs, const std::string& name, int num_sms, int* grid, int nstats_out[1]) {
  const EwSpec& s = rs.ew;
  int64_t N = prod(s.space);
  std::vector<const View*> views;
  for (const View& v : s.loads) views.push_back(&v);
  for (const auto& st : s.stores) views.push_back(&st.second);
  std::vector<int> perm = pick_perm(s);
  Dims d = merge_dims(s.space, perm, views);
  size_t nd = d.size.size();
  const char* ity = "long long";
  size_t nl = s.loads.size(), ns = s.stores.size(), nops = rs.ops.size();
  // stat slots: one per row op
  int G = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(N, 256 * 8), (int64_t)num_sms * 4));
  *grid = G;
  nstats_out[0] = (int)nops;
  std::ostringstream o;
  o << kPrelude;
  auto head = [&](const std::string& kn) {
    o << "extern \"C\" __global__ void __launch_bounds__(256) " << kn << "(const PfArgs A) {\n";
    for (size_t i = 0; i < nl; ++i)
      if (!s.loads[i].is_splat) o << "  const float* __restrict__ in" << i << " = (const float*)A.p[" << i << "];\n";
    for (size_t j = 0; j < ns; ++j) o << "  float* __restrict__ out" << j << " = (float*)A.p[" << nl + j << "];\n";
    for (size_t r = 0; r < nops; ++r) o << "  float* __restrict__ ro" << r << " = (float*)A.p[" << nl + ns + r << "];\n";
    o << "  const float* __restrict__ scal = (const float*)A.p[" << nl + ns + nops << "];\n";
    o << "  float* __restrict__ part = (float*)A.p[" << nl + ns + nops + 1 << "];\n";
    for (size_t i = 0; i < nl; ++i)
      if (s.loads[i].is_splat) o << "  const float sp" << i << " = scal[" << s.loads[i].splat_slot << "];\n";
    o << "  __shared__ float red[8][" << std::max<size_t>(nops, 1) << "];\n";
  };
  auto comb = [&](Op op, const std::string& a, const std::string& b) -> std::string {
    switch (op) {
      case Op::SUM: case Op::MEAN: return a + " + " + b;
      case Op::MAX: return "fmaxf(" + a + ", " + b + ")";
      case Op::MIN: return "fminf(" + a + ", " + b + ")";
      case Op::PROD: return a + " * " + b;
      default: fail(PFC_ERR_UNSUPPORTED, "full reduction supports sum/mean/max/min/prod only");
    }
  };
  auto neutral = [&](Op op) -> std::string {
    switch (op) {
      case Op::MAX: return "-PF_INF";
      case Op::MIN: return "PF_INF";
      case Op::PROD: return "1.f";
      default: return "0.f";
    }
  };
  auto block_reduce = [&]() {
    for (size_t r = 0; r < nops; ++r) {
      o << "  for (int off = 16; off > 0; off >>= 1) { float ot = __shfl_xor_sync(0xffffffffu, acc" << r
        << ", off); acc" << r << " = " << comb(rs.ops[r].op, "acc" + std::to_string(r), "ot") << "; }\n";
      o << "  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][" << r << "] = acc" << r << ";\n";
    }
    o << "  __syncthreads();\n";
    for (size_t r = 0; r < nops; ++r) {
      o << "  acc" << r << " = red[0][" << r << "]; for (int w = 1; w < 8; ++w) acc" << r << " = "
        << comb(rs.ops[r].op, "acc" + std::to_string(r), "red[w][" + std::to_string(r) + "]") << ";\n";
    }
  };
  head(name);
  for (size_t r = 0; r < nops; ++r) o << "  float acc" << r << " = " << neutral(rs.ops[r].op) << ";\n";
  o << "  for (long long L = (long long)blockIdx.x * blockDim.x + threadIdx.x; L < " << N
    << "LL; L += (long long)gridDim.x * blockDim.x) {\n";
  o << "    " << emit_coords("L", d.size, "c", ity);
  for (size_t i = 0; i < nl; ++i) {
    if (s.loads[i].is_splat) { o << "    const float l" << i << " = sp" << i << ";\n"; continue; }
    o << "    const float l" << i << " = in" << i << "[" << emit_offset(d.stride[i], "c", nd, 0, ity) << "];\n";
  }
  for (size_t k = 0; k < s.instrs.size(); ++k) {
    const EwInstr& in = s.instrs[k];
    std::string ex;
    auto nm = [&](int x) { return "e" + std::to_string(x); };
    if (in.kind == EwKind::LOAD) ex = "l" + std::to_string(in.load);
    else if (in.kind == EwKind::COPY) ex = nm(in.a[0]);
    else if (in.kind == EwKind::BN) {
      ex = "((" + nm(in.a[0]) + " - " + nm(in.a[1]) + ") / sqrtf(" + nm(in.a[2]) + " + " + flit(in.p0) + "))";
      if (in.a[3] >= 0) ex = "(" + ex + " * " + nm(in.a[3]) + ")";
      if (in.a[4] >= 0) ex = "(" + ex + " + " + nm(in.a[4]) + ")";
    } else {
      std::vector<std::string> args;
      for (int x : in.a) args.push_back(nm(x));
      ex = op_expr(in, args);
    }
    o << "    const float e" << k << " = " << ex << ";\n";
  }
  for (size_t j = 0; j < ns; ++j)
    o << "    out" << j << "[" << emit_offset(d.stride[nl + j], "c", nd, 0, ity) << "] = e" << s.stores[j].first << ";\n";
  for (size_t r = 0; r < nops; ++r)
    o << "    acc" << r << " = " << comb(rs.ops[r].op, "acc" + std::to_string(r), "e" + std::to_string(rs.ops[r].src))
      << ";\n";
  o << "  }\n";
  block_reduce();
  o << "  if (threadIdx.x == 0) {\n";
  for (size_t r = 0; r < nops; ++r) o << "    part[blockIdx.x * " << nops << " + " << r << "] = acc" << r << ";\n";
  o << "  }\n}\n";
  // finalize
  head(name + "_fin");
  for (size_t r = 0; r < nops; ++r) o << "  float acc" << r << " = " << neutral(rs.ops[r].op) << ";\n";
  o << "  for (int b = threadIdx.x; b < " << G << "; b += blockDim.x) {\n";
  for (size_t r = 0; r < nops; ++r)
    o << "    acc" << r << " = " << comb(rs.ops[r].op, "acc" + std::to_string(r), "part[b * " + std::to_string(nops) + " + " + std::to_string(r) + "]") << ";\n";
  o << "  }\n";
  block_reduce();
  o << "  if (threadIdx.x == 0) {\n";
  for (size_t r = 0; r < nops; ++r) {
    if (rs.ops[r].op == Op::MEAN) o << "    ro" << r << "[0] = acc" << r << " / " << flit((float)N) << ";\n";
    else o << "    ro" << r << "[0] = acc" << r << ";\n";
  }
  o << "  }\n}\n";
  return o.str();
}

// ---------------------------------------------------------------------------
// The compiler
// ---------------------------------------------------------------------------

static bool collapse_batch(const View& v, int nb, int64_t* stride);

struct Region {
  std::vector<uint64_t> nodes;        // topo order
  std::vector<uint64_t> row_ops;      // attached row operations
  std::vector<int64_t> shape;
  int red_begin = -1, red_end = -1;   // shared reduction structure of attached row ops
  bool full = false;
};

struct GemmChain {
  uint64_t mm = 0;                 // MATMUL or CONV2D node
  std::vector<uint64_t> absorbed;  // epilogue nodes in order
  uint64_t result = 0;             // node whose value the step produces
  int alpha_slot = -1;
  float alpha = 1.f;
  uint64_t bias = 0;  bool has_bias = false;
  uint64_t bn = 0;    bool has_bn = false;
  int act = 0;
  uint64_t residual = 0; bool has_residual = false;
};

class Compiler {
 public:
  Compiler(const CompileInput& in, SourceMap* src) : in_(in), g_(*in.g), src_(src) {}

  std::unique_ptr<Plan> run();

 private:
  const CompileInput& in_;
  const Graph& g_;
  SourceMap* src_;
  std::unique_ptr<Plan> P_;
  std::vector<uint64_t> order_;
  std::unordered_map<uint64_t, int> pos_;
  std::unordered_map<uint64_t, std::vector<uint64_t>> users_;
  std::set<uint64_t> is_out_;
  std::unordered_map<uint64_t, Cls> cls_;
  std::unordered_map<uint64_t, View> val_;           // materialised values and views
  std::unordered_map<uint64_t, int> region_of_;
  std::vector<Region> regions_;
  std::unordered_map<uint64_t, int> chain_of_;       // node -> chain index (mm and absorbed)
  std::vector<GemmChain> chains_;
  // attention: chain of the PV matmul -> (chain of the QK^T matmul, softmax node)
  std::unordered_map<int, std::pair<int, uint64_t>> attn_;
  // small-batch Linear layers on the CUDA cores: chain of the (last) layer ->
  // (chain of the first layer or -1, fused softmax/log-softmax node or 0)
  std::unordered_map<int, std::pair<int, uint64_t>> small_;
  std::unordered_map<uint64_t, int> row_region_;     // row op -> region
  std::vector<std::pair<int, Step>> steps_;
  std::unordered_map<uint64_t, int> splat_slot_;
  int kernel_counter_ = 0;
  int cur_pos_ = 0;
  bool depends_on(uint64_t a, uint64_t b);
  bool convex(const std::set<uint64_t>& S);

  const Node& N(uint64_t id) const { return g_.at(id); }

  int new_buffer(size_t bytes, BufKind kind = BufKind::ARENA, uint64_t node = 0) {
    Buffer b;
    b.kind = kind;
    b.bytes = std::max<size_t>(bytes, 4);
    b.node = node;
    P_->buffers.push_back(b);
    return (int)P_->buffers.size() - 1;
  }
  View dense(const std::vector<int64_t>& shape, DType dt) {
    View v;
    v.shape = shape;
    v.strides = View::dense_strides(shape);
    v.dtype = dt;
    int64_t n = prod(shape);
    v.buf = new_buffer((size_t)n * dtype_size(dt));
    return v;
  }
  // Dense view whose dims are laid out in the stride order of `like`.
  View dense_like(const std::vector<int64_t>& shape, const View* like) {
    if (!like || like->is_splat || like->shape.size() != shape.size()) return dense(shape, DType::F32);
    std::vector<int> perm(shape.size());
    for (size_t i = 0; i < perm.size(); ++i) perm[i] = (int)i;
    std::stable_sort(perm.begin(), perm.end(),
                     [&](int a, int b) { return std::llabs(like->strides[a]) > std::llabs(like->strides[b]); });
    View v;
    v.shape = shape;
    v.strides.assign(shape.size(), 0);
    int64_t acc = 1;
    for (int k = (int)perm.size() - 1; k >= 0; --k) {
      v.strides[perm[k]] = acc;
      acc *= shape[perm[k]];
    }
    v.dtype = DType::F32;
    v.buf = new_buffer((size_t)prod(shape) * 4);
    return v;
  }

  const View& value(uint64_t id) {
    auto it = val_.find(id);
    if (it == val_.end()) fail(PFC_ERR_INTERNAL, "value of node " + std::to_string(id) + " not materialised");
    return it->second;
  }

  void add_step(int /*pos*/, Step s) { steps_.push_back({cur_pos_, std::move(s)}); }

  // Tensor-core operand of a view: [rows][kpad] hi/lo fp32 (3xTF32) or bf16.
  struct Operand {
    int hi = -1, lo = -1;
  };
  std::unordered_map<std::string, Operand> operands_;  // view signature -> operand already in the plan
  // operands written by row kernels, keyed (buffer, rows, cols, kpad, precision)
  using OpKey = std::tuple<int, int64_t, int64_t, int64_t, int>;
  std::map<OpKey, Operand> pending_;
  std::set<OpKey> claimed_;
  std::set<OpKey> must_claim_;  // the fp32 value is not written: a GEMM must take the operand

  // A softmax/LayerNorm output that MATMULs read as their A operand is
  // written by its row kernel as a tf32x3 operand too; the fp32 value stays
  // when anything else reads it.
  void plan_row_operand(uint64_t id, RowOp& op) {
    if (in_.precision != PFC_PRECISION_TF32X3) return;
    if (!(op.op == Op::SOFTMAX || op.op == Op::LOG_SOFTMAX || op.op == Op::LAYER_NORM)) return;
    const View& o = op.out;
    if (o.is_splat || o.offset != 0 || o.strides != View::dense_strides(o.shape) || o.shape.size() < 2) return;
    const int64_t C = o.shape.back();
    if (C % 32 != 0) return;
    bool any_mm = false, other = is_out_.count(id) > 0;
    for (uint64_t u : users_[id]) {
      const Node& un = N(u);
      auto ci = cls_.find(u);
      const bool a_operand = un.op == Op::MATMUL && ci != cls_.end() && ci->second == Cls::GEMM &&
                             un.inputs.size() == 2 && un.inputs[0] == id && un.inputs[1] != id &&
                             N(un.inputs[1]).shape.size() <= o.shape.size();
      if (a_operand) any_mm = true;
      else other = true;
    }
    if (!any_mm) return;
    const int64_t rows = o.numel() / C;
    op.op_hi = new_buffer((size_t)rows * C * 4);
    op.op_lo = new_buffer((size_t)rows * C * 4);
    op.write_out = other;
    const OpKey key = std::make_tuple(o.buf, rows, C, C, in_.precision);
    pending_[key] = Operand{op.op_hi, op.op_lo};
    if (!other) must_claim_.insert(key);
  }

  // Emit (or reuse) the preparation of `src` ([rows, cols] logical, any
  // strides) as a GEMM operand.  Values are written once in a plan, so an
  // identical preparation earlier in the plan is reused.  When the source is
  // a resident constant (a weight), the operand is a PREPARED buffer that the
  // executor keeps with the constant, and its step runs only while unfilled.
  // conv_cp > 0: `src` is a Conv2d weight [O,C,KH,KW] laid out for the
  // implicit GEMM (k = (kh*KW + kw)*conv_cp + c).
  Operand prepare_operand(const View& src, int64_t rows, int64_t cols, int64_t kpad, int prec,
                          const std::string& label, int at, int64_t conv_cp = 0, int64_t conv_kwp = 0) {
    if (conv_cp == 0 && !src.is_splat && src.buf >= 0 && src.offset == 0 && src.strides == View::dense_strides(src.shape)) {
      auto pit = pending_.find(std::make_tuple(src.buf, rows, cols, kpad, prec));
      if (pit != pending_.end()) {
        claimed_.insert(pit->first);
        return pit->second;
      }
    }
    std::ostringstream sig;
    sig << src.buf << ':' << src.offset << ':' << (int)src.dtype << ':' << src.is_splat << ':' << src.splat_slot;
    for (size_t d = 0; d < src.shape.size(); ++d) sig << ',' << src.shape[d] << '/' << src.strides[d];
    sig << '|' << rows << ',' << cols << ',' << kpad << ',' << prec << ',' << conv_cp << ',' << conv_kwp;
    auto it = operands_.find(sig.str());
    if (it != operands_.end()) return it->second;
    const size_t esz = prec == PFC_PRECISION_BF16 ? 2 : 4;
    const size_t bytes = (size_t)rows * (size_t)kpad * esz;
    bool resident = false;
    uint64_t pkey = 0;
    if (!src.is_splat && src.buf >= 0 && P_->buffers[src.buf].kind == BufKind::CONST) {
      const Node& cn = N(P_->buffers[src.buf].node);
      if (cn.data_flags & PFC_CONST_RESIDENT) {
        resident = true;
        // FNV-1a over (payload key, payload size, layout signature)
        pkey = 1469598103934665603ull;
        auto mix = [&](uint64_t v) {
          for (int b = 0; b < 8; ++b) pkey = (pkey ^ ((v >> (8 * b)) & 0xFF)) * 1099511628211ull;
        };
        mix(cn.data_key);
        mix(cn.data_bytes);
        for (char ch : sig.str()) mix((uint64_t)(unsigned char)ch);
      }
    }
    Operand op;
    auto make = [&](int part) {
      int b = new_buffer(bytes, resident ? BufKind::PREPARED : BufKind::ARENA,
                         resident ? P_->buffers[src.buf].node : 0);
      if (resident) P_->buffers[b].prep_key = pkey * 2 + (uint64_t)part;
      return b;
    };
    op.hi = make(0);
    op.lo = prec == PFC_PRECISION_BF16 ? -1 : make(1);
    Step s;
    s.kind = StepKind::SPLIT;
    s.once = resident;
    s.label = label + (resident ? " (once per weight)" : "");
    s.split.src = src;
    s.split.precision = prec;
    s.split.rows = rows;
    s.split.cols = cols;
    s.split.kpad = kpad;
    s.split.out_hi = op.hi;
    s.split.out_lo = op.lo;
    s.split.conv_cp = conv_cp;
    s.split.conv_kwp = conv_kwp;
    add_step(at, std::move(s));
    operands_.emplace(sig.str(), op);
    return op;
  }

  std::string kname(const char* kind) {
    return std::string("pf_") + kind + "_" + std::to_string(kernel_counter_++);
  }

  void classify();
  void absorb_epilogues();
  void detect_attention();
  void detect_small();
  bool small_eligible(int ci, int64_t* pm, int64_t* pn, int64_t* pk);
  void build_regions();
  void attach_row_ops();
  void lower();
  void lower_leaf(uint64_t id);
  void lower_view(uint64_t id);
  void lower_region(int r);
  void lower_row_alone(uint64_t id);
  void lower_chain(int c);
  void lower_attention(int c);
  void lower_small(int c);
  void lower_matmul(const GemmChain& ch, int at);
  void lower_conv(const GemmChain& ch, int at);
  void lower_pool(uint64_t id);
  void lower_concat(uint64_t id);
  View materialize_copy(const View& src, int at, const std::string& label);
  void emit_jit(int at, const std::string& label, const std::string& kernel, const std::string& source, int grid,
                int block, const std::vector<std::pair<int, int64_t>>& ptrs, size_t smem = 0);
  void finish();
  void emit_operands_at_producers();

  bool must_materialize(uint64_t id);
  bool row_structure(uint64_t row, const std::vector<int64_t>& in_shape, int* rb, int* re, bool* full);
  View splat_view(uint64_t id, const std::vector<int64_t>& shape);
};

View Compiler::splat_view(uint64_t id, const std::vector<int64_t>& shape) {
  View v;
  v.is_splat = true;
  v.shape = shape;
  v.strides.assign(shape.size(), 0);
  v.dtype = DType::F32;
  auto it = splat_slot_.find(id);
  if (it == splat_slot_.end()) {
    P_->scalars.push_back({id, in_.splats.at(id)});
    it = splat_slot_.emplace(id, (int)P_->scalars.size() - 1).first;
    P_->splat_nodes.push_back(id);
  }
  v.splat_slot = it->second;
  v.splat_value = in_.splats.at(id);
  return v;
}

bool Compiler::depends_on(uint64_t a, uint64_t b) {
  // true when node a (transitively) reads node b
  if (a == b) return true;
  int pb = pos_[b];
  std::vector<uint64_t> stack{a};
  std::set<uint64_t> seen;
  while (!stack.empty()) {
    uint64_t x = stack.back();
    stack.pop_back();
    if (x == b) return true;
    if (!seen.insert(x).second || pos_[x] < pb) continue;
    for (uint64_t in : N(x).inputs) stack.push_back(in);
  }
  return false;
}

void Compiler::classify() {
  for (uint64_t id : order_) {
    const Node& n = N(id);
    Cls c;
    if (n.type != NodeType::OPERATION) c = Cls::LEAF;
    else if (is_view_op(n.op)) c = Cls::VIEW;
    else if (op_is_elementwise(n.op) || n.op == Op::BATCH_NORM) c = Cls::EW;
    else if (is_row_op(n.op)) c = Cls::ROW;
    else if (n.op == Op::MATMUL || n.op == Op::BATCH_MATMUL) c = Cls::GEMM;
    else if (n.op == Op::CONV2D) c = Cls::CONV;
    else if (n.op == Op::MAX_POOL2D || n.op == Op::AVG_POOL2D || n.op == Op::ADAPTIVE_AVG_POOL2D) c = Cls::POOL;
    else if (n.op == Op::CONCAT || n.op == Op::STACK) c = Cls::CONCAT;
    else fail(PFC_ERR_UNSUPPORTED, std::string("Unsupported operation for CUDA execution: ") + op_name(n.op));
    if (c != Cls::LEAF && c != Cls::VIEW && n.dtype != DType::F32)
      fail(PFC_ERR_UNSUPPORTED, std::string("CUDA executor computes float32 only; node ") + std::to_string(id) +
                                    " (" + op_name(n.op) + ") is " + dtype_name(n.dtype));
    if (n.op == Op::BATCH_NORM && (n.attr_bool("training", false) || !n.attr_bool("track_running_stats", true)))
      fail(PFC_ERR_UNSUPPORTED, "BATCH_NORM with batch statistics (training mode) is not supported");
    cls_[id] = c;
  }
}

// Shape-compatible bias: broadcasts along every dim but `ndim_n`.
static bool bias_along(const Node& b, const std::vector<int64_t>& out_shape, int n_dim) {
  if (b.shape.size() > out_shape.size()) return false;
  size_t off = out_shape.size() - b.shape.size();
  bool seen = false;
  for (size_t d = 0; d < b.shape.size(); ++d) {
    int od = (int)(off + d);
    if (od == n_dim) {
      if (b.shape[d] != out_shape[od]) return false;
      seen = true;
    } else if (b.shape[d] != 1) {
      return false;
    }
  }
  return seen || out_shape[n_dim] == 1;
}

void Compiler::absorb_epilogues() {
  for (uint64_t id : order_) {
    Cls c = cls_[id];
    if (c != Cls::GEMM && c != Cls::CONV) continue;
    if (chain_of_.count(id)) continue;  // already absorbed into an earlier chain
    GemmChain ch;
    ch.mm = id;
    uint64_t cur = id;
    const std::vector<int64_t> shape = N(id).shape;
    int n_dim = c == Cls::CONV ? 1 : (int)shape.size() - 1;
    bool stage_alpha = false, stage_bias = false, stage_act = false, stage_res = false;
    while (!is_out_.count(cur) && users_[cur].size() == 1) {
      uint64_t u = users_[cur][0];
      const Node& un = N(u);
      if (cls_[u] != Cls::EW || un.shape != shape) break;
      // the other operand of a binary consumer
      auto other = [&]() -> uint64_t { return un.inputs[0] == cur ? un.inputs[1] : un.inputs[0]; };
      if (un.op == Op::MUL && un.inputs.size() == 2 && un.inputs[0] != un.inputs[1] && !stage_alpha && !stage_bias &&
          !stage_act && !stage_res && c == Cls::GEMM) {
        uint64_t o = other();
        if (!in_.splats.count(o)) {
          // a view chain ending at a splat constant counts too
          const Node* on = &N(o);
          while (on->type == NodeType::OPERATION && is_view_op(on->op) && on->inputs.size() == 1) on = &N(on->inputs[0]);
          if (!in_.splats.count(on->id)) break;
          o = on->id;
        }
        stage_alpha = true;
        splat_view(o, {});
        ch.alpha_slot = splat_slot_.at(o);
        ch.alpha = in_.splats.at(o);
      } else if (un.op == Op::ADD && un.inputs.size() == 2 && un.inputs[0] != un.inputs[1] && !stage_bias &&
                 !stage_act && !stage_res && !ch.has_bn && bias_along(N(other()), shape, n_dim) &&
                 prod(N(other()).shape) == shape[n_dim] && !depends_on(other(), id)) {
        stage_bias = true;
        ch.has_bias = true;
        ch.bias = other();
      } else if (un.op == Op::BATCH_NORM && c == Cls::CONV && un.inputs[0] == cur && !ch.has_bn && !stage_act &&
                 !stage_res) {
        bool ok = true;
        for (size_t i = 1; i < un.inputs.size(); ++i)
          ok = ok && N(un.inputs[i]).shape.size() == 1 && !depends_on(un.inputs[i], id);
        if (!ok) break;
        ch.has_bn = true;
        ch.bn = u;
        stage_bias = true;
      } else if (is_act(un.op) && !stage_act && !stage_res) {
        stage_act = true;
        ch.act = act_code(un.op);
      } else if (un.op == Op::ADD && un.inputs.size() == 2 && un.inputs[0] != un.inputs[1] && !stage_res &&
                 c == Cls::GEMM && N(other()).shape == shape && !depends_on(other(), id) &&
                 !in_.splats.count(other())) {
        stage_res = true;
        ch.has_residual = true;
        ch.residual = other();
      } else {
        break;
      }
      ch.absorbed.push_back(u);
      cur = u;
    }
    ch.result = cur;
    int ci = (int)chains_.size();
    chains_.push_back(ch);
    chain_of_[id] = ci;
    for (uint64_t a : ch.absorbed) {
      chain_of_[a] = ci;
      cls_[a] = cls_[id];  // absorbed nodes no longer form elementwise regions
    }
  }
}

// Attention: MATMUL(Q, K^T) (only a scale absorbed) feeding nothing but a
// softmax over its last dim, which feeds nothing but the A operand of
// MATMUL(P, V) (nothing absorbed), all batched over the same leading dims,
// with head dims <= 64, becomes one unit lowered as the fused attention
// kernel: the scores and probabilities never reach HBM.  This is the core of
// PyFlame's MultiheadAttention::forward (attention.cpp).
void Compiler::detect_attention() {
  if (in_.precision != PFC_PRECISION_TF32X3 && in_.precision != PFC_PRECISION_BF16) return;
  for (int c2 = 0; c2 < (int)chains_.size(); ++c2) {
    const GemmChain& ch2 = chains_[c2];
    if (cls_[ch2.mm] != Cls::GEMM || !ch2.absorbed.empty() || chain_of_.at(ch2.mm) != c2) continue;
    const Node& mm2 = N(ch2.mm);
    if (mm2.op != Op::MATMUL || mm2.inputs.size() != 2 || mm2.inputs[0] == mm2.inputs[1]) continue;
    const uint64_t sm = mm2.inputs[0];
    const Node& smn = N(sm);
    if (smn.op != Op::SOFTMAX || cls_[sm] != Cls::ROW || is_out_.count(sm) || users_[sm].size() != 1) continue;
    const int rank = (int)smn.shape.size();
    if (rank < 3 || rank > 4) continue;  // [slices, M, L] or [B, H, M, L]
    int dim = (int)smn.attr_int("dim", -1);
    if (dim < 0) dim += rank;
    if (dim != rank - 1) continue;
    const uint64_t r1 = smn.inputs.at(0);
    auto it = chain_of_.find(r1);
    if (it == chain_of_.end()) continue;
    const int c1 = it->second;
    const GemmChain& ch1 = chains_[c1];
    if (ch1.result != r1 || is_out_.count(r1) || users_[r1].size() != 1 || cls_[ch1.mm] != Cls::GEMM) continue;
    if (ch1.has_bias || ch1.has_bn || ch1.act || ch1.has_residual || attn_.count(c1)) continue;
    const Node& mm1 = N(ch1.mm);
    if (mm1.op != Op::MATMUL || mm1.inputs.size() != 2) continue;
    bool ok = true;
    for (const Node* x : {&mm1, &mm2})
      for (uint64_t in : x->inputs) {
        const Node& o = N(in);
        ok = ok && o.shape.size() == (size_t)rank && !in_.splats.count(in) && o.dtype == DType::F32;
        for (int k = 0; ok && k < rank - 2; ++k) ok = o.shape[k] == smn.shape[k];
      }
    if (!ok) continue;
    const int64_t d1 = N(mm1.inputs[0]).shape[rank - 1], d2 = N(mm2.inputs[1]).shape[rank - 1];
    if (d1 > 64 || d2 > 64 || mm2.shape[rank - 2] != smn.shape[rank - 2]) continue;
    // every node of the QK^T chain and the softmax join the PV chain's unit
    std::vector<uint64_t> nodes{ch1.mm, sm};
    nodes.insert(nodes.end(), ch1.absorbed.begin(), ch1.absorbed.end());
    for (uint64_t x : nodes) {
      chain_of_[x] = c2;
      cls_[x] = Cls::GEMM;
    }
    attn_.emplace(c2, std::make_pair(c1, sm));
  }
}

// A Linear layer of a small batch, evaluated on the CUDA cores (small_gemm.cu)
// instead of the tensor cores: MATMUL(x, TRANSPOSE(w)) of a 2-D leaf weight
// w [N, K] (PyFlame's Linear, linear.cpp:36-44) with at most kSmallMaxRows
// rows of x and at most 64 MFLOP, optional alpha/bias/activation epilogue.
bool Compiler::small_eligible(int ci, int64_t* pm, int64_t* pn, int64_t* pk) {
  const GemmChain& ch = chains_[ci];
  if (cls_[ch.mm] != Cls::GEMM || chain_of_.at(ch.mm) != ci || attn_.count(ci)) return false;
  if (ch.has_bn || ch.has_residual) return false;
  const Node& mm = N(ch.mm);
  if (mm.op != Op::MATMUL || mm.inputs.size() != 2 || mm.inputs[0] == mm.inputs[1]) return false;
  const Node& a = N(mm.inputs[0]);
  const Node& bt = N(mm.inputs[1]);
  if (a.shape.empty() || bt.shape.size() != 2 || bt.op != Op::TRANSPOSE || bt.inputs.size() != 1) return false;
  const Node& w = N(bt.inputs[0]);
  if (w.type == NodeType::OPERATION || w.shape.size() != 2 || in_.splats.count(bt.inputs[0]) ||
      in_.bindings.count(bt.inputs[0]) || w.dtype != DType::F32 || a.dtype != DType::F32)
    return false;
  const int64_t k = a.shape.back(), n = bt.shape[1];
  if (w.shape[0] != n || w.shape[1] != k || bt.shape[0] != k) return false;  // [K, N] = w^T
  const int64_t m = prod(a.shape) / std::max<int64_t>(k, 1);
  if (m < 1 || m > kSmallMaxRows || k < 1 || n < 1 || 2.0 * m * n * k > 64e6) return false;
  *pm = m;
  *pn = n;
  *pk = k;
  return true;
}

// Linear -> (activation) -> Linear -> (softmax) on a small batch becomes one
// launch (PyFlame's MLP graph, nn/linear.cpp); any other small Linear runs
// alone on the CUDA cores.
void Compiler::detect_small() {
  std::unordered_map<int, std::array<int64_t, 3>> ok;
  for (int ci = 0; ci < (int)chains_.size(); ++ci) {
    int64_t m, n, k;
    if (small_eligible(ci, &m, &n, &k)) ok[ci] = {m, n, k};
  }
  std::set<int> taken;
  for (int c1 = 0; c1 < (int)chains_.size(); ++c1) {
    if (!ok.count(c1) || taken.count(c1)) continue;
    const GemmChain& ch1 = chains_[c1];
    const uint64_t r1 = ch1.result;
    if (is_out_.count(r1) || users_[r1].size() != 1) continue;
    auto it = chain_of_.find(users_[r1][0]);
    if (it == chain_of_.end()) continue;
    const int c2 = it->second;
    const GemmChain& ch2 = chains_[c2];
    if (c2 == c1 || !ok.count(c2) || taken.count(c2) || users_[r1][0] != ch2.mm || N(ch2.mm).inputs[0] != r1) continue;
    const int64_t M = ok[c1][0], N1 = ok[c1][1], N2 = ok[c2][1];
    if (ok[c2][0] != M || N1 > 4096 || 2.0 * M * N1 * N2 > 4e6) continue;
    // an optional row softmax over the last dim, its only reader
    uint64_t sm = 0;
    const uint64_t r2 = ch2.result;
    if (!is_out_.count(r2) && users_[r2].size() == 1) {
      const uint64_t u = users_[r2][0];
      const Node& un = N(u);
      if ((un.op == Op::SOFTMAX || un.op == Op::LOG_SOFTMAX) && cls_[u] == Cls::ROW && un.inputs[0] == r2) {
        int dim = (int)un.attr_int("dim", -1);
        if (dim < 0) dim += (int)un.shape.size();
        if (dim == (int)un.shape.size() - 1) sm = u;
      }
    }
    std::vector<uint64_t> nodes{ch1.mm};
    nodes.insert(nodes.end(), ch1.absorbed.begin(), ch1.absorbed.end());
    if (sm) nodes.push_back(sm);
    for (uint64_t x : nodes) {
      chain_of_[x] = c2;
      cls_[x] = Cls::GEMM;
    }
    small_[c2] = {c1, sm};
    taken.insert(c1);
    taken.insert(c2);
  }
  for (auto& [ci, dims] : ok)
    if (!taken.count(ci)) small_[ci] = {-1, 0};
}

void Compiler::lower_small(int ci) {
  const auto [first, sm] = small_.at(ci);
  const GemmChain& last = chains_[ci];
  const GemmChain& c1 = first >= 0 ? chains_[first] : last;
  const uint64_t result = sm ? sm : last.result;
  const int at = pos_[result];
  Step st;
  st.kind = StepKind::SMALL;
  SmallArgs& S = st.small;
  // rows of x with K contiguous (copied when the view does not have that form)
  View a = value(N(c1.mm).inputs[0]);
  const int64_t K1 = a.shape.back(), M = a.numel() / std::max<int64_t>(K1, 1);
  int64_t lda = K1;
  {
    int64_t rs = K1;
    const bool rows_ok = !a.is_splat && a.strides.back() == 1 &&
                         (a.shape.size() == 1 || collapse_batch(a, (int)a.shape.size() - 1, &rs));
    if (!rows_ok) a = materialize_copy(a, at, "contiguous rows for a small GEMM");
    else lda = a.shape.size() == 1 ? K1 : rs;
    if (a.shape.size() >= 2 && !rows_ok) lda = K1;
  }
  S.a = a;
  S.lda = lda;
  S.M = M;
  auto layer = [&](const GemmChain& ch, SmallLayerArgs& L) {
    const Node& bt = N(N(ch.mm).inputs[1]);
    const View w = value(bt.inputs[0]);  // the [N, K] weight leaf, dense
    if (w.is_splat || w.strides.back() != 1) fail(PFC_ERR_INTERNAL, "small GEMM weight is not dense rows");
    L.w_buf = w.buf;
    L.w_off = w.offset;
    L.N = w.shape[0];
    L.K = w.shape[1];
    L.ldw = w.strides[0];
    L.alpha = ch.alpha;
    L.alpha_slot = ch.alpha_slot;
    L.act = ch.act;
    if (ch.has_bias) {
      View b = value(ch.bias);
      int64_t sn = 0;
      for (size_t d = 0; d < b.shape.size(); ++d)
        if (b.shape[d] != 1) sn = b.strides[d];
      if (b.is_splat) sn = 0;
      L.bias = b;
      L.bstride = sn;
      L.has_bias = true;
    }
  };
  layer(c1, S.l1);
  std::string label = "small gemm [" + std::to_string(M) + "x" + std::to_string(S.l1.N) + "x" + std::to_string(K1) + "]";
  if (first >= 0) {
    S.layers = 2;
    layer(last, S.l2);
    // clusters of 8 CTAs when the rows and weights stage whole in shared
    // memory by 16-byte copies; otherwise one launch whose last CTA runs layer 2
    S.cluster = small_mlp_cluster_fits(M, S.l1.N, K1, S.l2.N) && S.a.offset % 4 == 0 && S.lda % 4 == 0 &&
                S.l1.w_off % 4 == 0 && S.l1.ldw % 4 == 0 && S.l2.w_off % 4 == 0 && S.l2.ldw % 4 == 0;
    if (!S.cluster) {
      S.h_buf = new_buffer((size_t)M * S.l1.N * 4);
      S.counter_buf = new_buffer(8);
      Step ms;
      ms.kind = StepKind::MEMSET;
      ms.label = "zero small-GEMM arrival counter";
      ms.memset_buf = S.counter_buf;
      add_step(at, ms);
    }
    label = "small mlp [" + std::to_string(M) + "x" + std::to_string(S.l1.N) + "x" + std::to_string(K1) + " -> " +
            std::to_string(S.l2.N) + "]";
  }
  if (sm) {
    S.softmax = N(sm).op == Op::SOFTMAX ? 1 : 2;
    label += S.softmax == 1 ? " +softmax" : " +log_softmax";
  }
  if (S.cluster) label += " (clusters)";
  const int64_t nout = S.layers == 2 ? S.l2.N : S.l1.N;
  S.out = dense(N(result).shape, DType::F32);
  S.ldo = nout;
  st.label = label;
  add_step(at, st);
  val_[result] = S.out;
}

void Compiler::lower_attention(int c2) {
  const GemmChain& ch2 = chains_[c2];
  const GemmChain& ch1 = chains_[attn_.at(c2).first];
  const int at = pos_[ch2.result];
  const Node& mm1 = N(ch1.mm);
  const Node& mm2 = N(ch2.mm);
  View q = value(mm1.inputs[0]);   // [batch..., M, d]
  View kt = value(mm1.inputs[1]);  // [batch..., d, L]
  View v = value(mm2.inputs[1]);   // [batch..., L, dv]
  const size_t r = q.shape.size();
  std::vector<int64_t> batch(q.shape.begin(), q.shape.end() - 2);
  const int64_t nbatch = prod(batch);
  const int64_t M = q.shape[r - 2], d = q.shape[r - 1], L = kt.shape[r - 1], dv = v.shape[r - 1];
  if (kt.shape[r - 2] != d || v.shape[r - 2] != L) fail(PFC_ERR_GRAPH, "matmul: inner dimensions don't match");
  const int prec = in_.precision;
  const int64_t kal = prec == PFC_PRECISION_BF16 ? 64 : 32;  // 128-byte rows
  const int64_t kq = round_up(d, kal), kv = round_up(dv, kal);
  // K as [batch..., L, d]: swap the last two dims of K^T (V is used as stored)
  View k = kt;
  std::swap(k.shape[r - 2], k.shape[r - 1]);
  std::swap(k.strides[r - 2], k.strides[r - 1]);
  const Operand oq = prepare_operand(q, nbatch * M, d, kq, prec, "prepare Q " + shape_str(q.shape), at);
  const Operand ok = prepare_operand(k, nbatch * L, d, kq, prec, "prepare K " + shape_str(k.shape), at);
  const Operand ov = prepare_operand(v, nbatch * L, dv, kv, prec, "prepare V " + shape_str(v.shape), at);
  // O [batch..., M, dv], stored with the heads innermost when there is a
  // head dim ([B][M][H][dv] for [B, H, M, dv]): merging the heads back,
  // transpose(1, 2) + reshape, is then a view of a dense [B*M, H*dv] matrix.
  View c = dense(mm2.shape, DType::F32);
  if (r == 4) {
    const int64_t H = mm2.shape[1];
    c.strides = {M * H * dv, dv, H * dv, 1};
  }
  Step st;
  st.kind = StepKind::ATTENTION;
  st.label = "attention " + std::to_string(nbatch) + "x[" + std::to_string(M) + "x" + std::to_string(L) + "x" +
             std::to_string(dv) + "]";
  AttnArgs& A = st.attn;
  A.q_hi = oq.hi; A.q_lo = oq.lo; A.k_hi = ok.hi; A.k_lo = ok.lo; A.v_hi = ov.hi; A.v_lo = ov.lo;
  A.batch = nbatch; A.M = M; A.L = L; A.d = dv; A.kq = kq; A.kv = kv;
  A.alpha = ch1.alpha;
  A.alpha_slot = ch1.alpha_slot;
  A.c = c;
  add_step(at, std::move(st));
  val_[ch2.result] = c;
}

// A set of nodes is convex when no path leaves it and re-enters it; only
// convex sets can run as one kernel.
bool Compiler::convex(const std::set<uint64_t>& S) {
  std::vector<uint64_t> stack;
  std::set<uint64_t> seen;
  for (uint64_t s : S)
    for (uint64_t u : users_[s])
      if (!S.count(u)) stack.push_back(u);
  while (!stack.empty()) {
    uint64_t u = stack.back();
    stack.pop_back();
    if (!seen.insert(u).second) continue;
    if (S.count(u)) return false;
    for (uint64_t v : users_[u]) stack.push_back(v);
  }
  return true;
}

void Compiler::build_regions() {
  // Union-find over elementwise nodes: merge every producer/consumer pair of
  // equal shape while the merged set stays convex.
  std::unordered_map<uint64_t, uint64_t> parent;
  std::unordered_map<uint64_t, std::set<uint64_t>> members;
  std::function<uint64_t(uint64_t)> find = [&](uint64_t x) {
    while (parent[x] != x) {
      parent[x] = parent[parent[x]];
      x = parent[x];
    }
    return x;
  };
  for (uint64_t id : order_)
    if (cls_[id] == Cls::EW && !chain_of_.count(id)) {
      parent[id] = id;
      members[id] = {id};
    }
  for (uint64_t id : order_) {
    if (!parent.count(id)) continue;
    for (uint64_t in : N(id).inputs) {
      if (!parent.count(in) || N(in).shape != N(id).shape) continue;
      uint64_t ra = find(in), rb = find(id);
      if (ra == rb) continue;
      std::set<uint64_t> S = members[ra];
      S.insert(members[rb].begin(), members[rb].end());
      if (!convex(S)) continue;
      parent[ra] = rb;
      members[rb] = std::move(S);
      members.erase(ra);
    }
  }
  std::unordered_map<uint64_t, int> index;
  for (uint64_t id : order_) {
    if (!parent.count(id)) continue;
    uint64_t r = find(id);
    auto it = index.find(r);
    if (it == index.end()) {
      Region rg;
      rg.shape = N(id).shape;
      regions_.push_back(rg);
      it = index.emplace(r, (int)regions_.size() - 1).first;
    }
    regions_[it->second].nodes.push_back(id);
    region_of_[id] = it->second;
  }
}

// Reduction structure of a row op over an input of shape `s`: dims [rb, re) reduced.
bool Compiler::row_structure(uint64_t row, const std::vector<int64_t>& s, int* rb, int* re, bool* full) {
  const Node& n = N(row);
  int nd = (int)s.size();
  *full = false;
  if (n.op == Op::LAYER_NORM) {
    // normalization.cpp:224-255: normalized over the trailing len(normalized_shape) dims
    auto ns = n.attr_ints("normalized_shape");
    int k = (int)ns.size();
    if (k > nd) fail(PFC_ERR_GRAPH, "LAYER_NORM normalized_shape longer than input");
    for (int i = 0; i < k; ++i)
      if (s[nd - k + i] != ns[i]) fail(PFC_ERR_GRAPH, "Input shape doesn't match normalized_shape");
    *rb = nd - k;
    *re = nd;
    return true;
  }
  if (n.op == Op::SOFTMAX || n.op == Op::LOG_SOFTMAX) {
    // tensor_impl.cpp:272-273: attribute `dim` (int), default -1
    int d = (int)n.attr_int("dim", -1);
    if (d < 0) d += nd;
    if (d < 0 || d >= nd) fail(PFC_ERR_GRAPH, "softmax dim out of range");
    *rb = d;
    *re = d + 1;
    return true;
  }
  // reductions: optional int `dim`, bool `keepdim` (tensor_impl.cpp:530-533)
  if (!n.has_attr("dim")) {
    *rb = 0;
    *re = nd;
    *full = true;
    return true;
  }
  int d = (int)n.attr_int("dim");
  if (d < 0) d += nd;
  if (d < 0 || d >= nd) fail(PFC_ERR_GRAPH, "Reduction dimension out of range");
  *rb = d;
  *re = d + 1;
  return true;
}

void Compiler::attach_row_ops() {
  for (uint64_t id : order_) {
    if (cls_[id] != Cls::ROW) continue;
    const Node& n = N(id);
    uint64_t x = n.inputs.at(0);
    int rb, re;
    bool full;
    row_structure(id, N(x).shape, &rb, &re, &full);
    auto r = region_of_.find(x);
    if (r == region_of_.end()) continue;
    Region& rg = regions_[r->second];
    if (rg.shape != N(x).shape) continue;
    if (!rg.row_ops.empty() && (rg.red_begin != rb || rg.red_end != re || rg.full != full)) continue;
    // LN parameters must not depend on the region
    bool ok = true;
    for (size_t i = 1; i < n.inputs.size(); ++i) {
      auto ri = region_of_.find(n.inputs[i]);
      if (ri != region_of_.end() && ri->second == r->second) ok = false;
    }
    if (ok) {
      std::set<uint64_t> S(rg.nodes.begin(), rg.nodes.end());
      S.insert(rg.row_ops.begin(), rg.row_ops.end());
      S.insert(id);
      ok = convex(S);
    }
    if (!ok) continue;
    rg.row_ops.push_back(id);
    rg.red_begin = rb;
    rg.red_end = re;
    rg.full = full;
    row_region_[id] = r->second;
  }
}

bool Compiler::must_materialize(uint64_t id) {
  if (is_out_.count(id)) return true;
  auto r = region_of_.find(id);
  for (uint64_t u : users_[id]) {
    if (r != region_of_.end()) {
      auto ru = region_of_.find(u);
      if (ru != region_of_.end() && ru->second == r->second) continue;
      auto rr = row_region_.find(u);
      if (rr != row_region_.end() && rr->second == r->second && N(u).inputs[0] == id) {
        // feeding an attached row op as its main input; LN params still need a value
        bool also_param = false;
        for (size_t i = 1; i < N(u).inputs.size(); ++i) also_param |= N(u).inputs[i] == id;
        if (!also_param) continue;
      }
    }
    auto c = chain_of_.find(u);
    if (c != chain_of_.end()) {
      const GemmChain& ch = chains_[c->second];
      // the running value of the chain is not materialised
      if (u != ch.mm && (N(u).inputs[0] == id || (N(u).inputs.size() > 1 && N(u).inputs[1] == id))) {
        bool is_chain_value = (id == ch.mm) || std::find(ch.absorbed.begin(), ch.absorbed.end(), id) != ch.absorbed.end();
        if (is_chain_value) continue;
      }
    }
    return true;
  }
  return false;
}

void Compiler::emit_jit(int at, const std::string& label, const std::string& kernel, const std::string& source,
                        int grid, int block, const std::vector<std::pair<int, int64_t>>& ptrs, size_t smem) {
  Step s;
  s.kind = StepKind::JIT;
  s.label = label;
  s.jit.kernel = kernel;
  // kernel names are positional; the key covers the source with a fixed name
  std::string canon = source;
  size_t p;
  while ((p = canon.find(kernel)) != std::string::npos) canon.replace(p, kernel.size(), "pf_kernel");
  s.jit.module_key = hash_hex(canon);
  s.jit.kernel = "pf_kernel";
  s.jit.grid = grid;
  s.jit.block = block;
  s.jit.smem = smem;
  s.jit.ptrs = ptrs;
  (*src_)[s.jit.module_key] = {canon, "pf_kernel"};
  add_step(at, std::move(s));
}

View Compiler::materialize_copy(const View& srcv, int at, const std::string& label) {
  EwSpec s;
  s.space = srcv.shape;
  View out = srcv.is_splat ? dense(srcv.shape, DType::F32) : dense(srcv.shape, srcv.dtype);
  s.loads.push_back(srcv);
  EwInstr ld;
  ld.kind = EwKind::LOAD;
  ld.load = 0;
  s.instrs.push_back(ld);
  s.stores.push_back({0, out});
  std::string name = kname("copy");
  int grid, block;
  std::string code = gen_ew(s, name, in_.num_sms, &grid, &block);
  std::vector<std::pair<int, int64_t>> ptrs;
  ptrs.push_back({srcv.is_splat ? -1 : srcv.buf, srcv.offset * (int64_t)dtype_size(srcv.dtype)});
  ptrs.push_back({out.buf, 0});
  ptrs.push_back({P_->scalar_buf, 0});
  emit_jit(at, label, name, code, grid, block, ptrs);
  return out;
}

void Compiler::lower_leaf(uint64_t id) {
  const Node& n = N(id);
  if (in_.bindings.count(id)) {
    View v;
    v.shape = n.shape;
    v.strides = View::dense_strides(n.shape);
    v.dtype = n.dtype;
    v.buf = new_buffer(n.size_bytes(), BufKind::BINDING, id);
    val_[id] = v;
    return;
  }
  if (in_.splats.count(id)) {
    val_[id] = splat_view(id, n.shape);
    return;
  }
  if (!n.has_data()) {
    // Data-less INPUT/PARAMETER/CONSTANT: zero (the ROCm executor zero-fills, rocm_executor.cpp:99-102).
    if (n.dtype != DType::F32) fail(PFC_ERR_UNSUPPORTED, "data-less non-float32 leaf");
    fail(PFC_ERR_INTERNAL, "data-less leaf should have been classified as a zero splat");
  }
  View v;
  v.shape = n.shape;
  v.strides = View::dense_strides(n.shape);
  v.dtype = n.dtype;
  v.buf = new_buffer(n.size_bytes(), BufKind::CONST, id);
  P_->const_nodes.push_back(id);
  val_[id] = v;
}

void Compiler::lower_view(uint64_t id) {
  const Node& n = N(id);
  const View& x = value(n.inputs.at(0));
  View out;
  switch (n.op) {
    case Op::RESHAPE: case Op::VIEW: case Op::SQUEEZE: case Op::UNSQUEEZE: {
      if (prod(n.shape) != x.numel()) fail(PFC_ERR_GRAPH, "reshape: total elements must match");
      if (x.is_splat) { out = x; out.shape = n.shape; out.strides.assign(n.shape.size(), 0); break; }
      if (!reshape_view(x, n.shape, &out)) {
        View c = materialize_copy(x, pos_[id], std::string("contiguous copy for reshape of %") + std::to_string(id));
        reshape_view(c, n.shape, &out);
      }
      break;
    }
    case Op::TRANSPOSE: {
      // attributes dim0/dim1 (int), tensor_impl.cpp:577-578; spec shape_inference.hpp:220-239
      int nd = (int)x.shape.size();
      int d0 = (int)n.attr_int("dim0"), d1 = (int)n.attr_int("dim1");
      if (d0 < 0) d0 += nd;
      if (d1 < 0) d1 += nd;
      if (d0 < 0 || d0 >= nd || d1 < 0 || d1 >= nd) fail(PFC_ERR_GRAPH, "transpose: dimension out of range");
      out = x;
      std::swap(out.shape[d0], out.shape[d1]);
      std::swap(out.strides[d0], out.strides[d1]);
      break;
    }
    case Op::SLICE: {
      // attributes dim (int), start/end (int64), tensor.cpp:262-283
      int nd = (int)x.shape.size();
      int d = (int)n.attr_int("dim", 0);
      if (d < 0) d += nd;
      if (d < 0 || d >= nd) fail(PFC_ERR_GRAPH, "slice: dimension out of range");
      int64_t size = x.shape[d];
      int64_t st = n.attr_int("start", 0), en = n.attr_int("end", size);
      if (st < 0) st += size;
      if (en < 0) en += size;
      st = std::max<int64_t>(0, std::min(st, size));
      en = std::max<int64_t>(0, std::min(en, size));
      if (en <= st) fail(PFC_ERR_GRAPH, "slice: end must be greater than start");
      out = x;
      out.shape[d] = en - st;
      if (!x.is_splat) out.offset += st * x.strides[d];
      break;
    }
    case Op::BROADCAST:
      out = broadcast_to(x, n.shape);
      break;
    default:  // CONTIGUOUS, COPY, LAYOUT_TRANSFORM, DROPOUT (inference: identity, dropout.cpp:26-30)
      out = x;
      if (n.op == Op::DROPOUT && n.attr_bool("training", false))
        fail(PFC_ERR_UNSUPPORTED, "DROPOUT in training mode is not supported");
      break;
  }
  if (out.shape != n.shape) {
    if (out.numel() != prod(n.shape)) fail(PFC_ERR_GRAPH, "shape op output shape mismatch at node " + std::to_string(id));
    View o2;
    if (out.is_splat) { o2 = out; o2.shape = n.shape; o2.strides.assign(n.shape.size(), 0); }
    else if (!reshape_view(out, n.shape, &o2)) {
      View c = materialize_copy(out, pos_[id], "contiguous copy");
      reshape_view(c, n.shape, &o2);
    }
    out = o2;
  }
  val_[id] = out;
}

// Lower an elementwise region (and its attached row ops).
void Compiler::lower_region(int r) {
  Region& rg = regions_[r];
  RowSpec rs;
  EwSpec& s = rs.ew;
  s.space = rg.shape;
  std::unordered_map<uint64_t, int> instr_of;
  std::unordered_map<uint64_t, int> load_of;  // external node -> load index
  int at = 0;
  const View* layout_ref = nullptr;
  auto operand = [&](uint64_t in) -> int {
    auto it = instr_of.find(in);
    if (it != instr_of.end()) return it->second;
    auto lt = load_of.find(in);
    int li;
    if (lt == load_of.end()) {
      const View& v = value(in);
      View b = broadcast_to(v, s.space);
      s.loads.push_back(b);
      li = (int)s.loads.size() - 1;
      load_of[in] = li;
      if (!layout_ref && !v.is_splat && v.shape == s.space) layout_ref = &value(in);
    } else {
      li = lt->second;
    }
    EwInstr ld;
    ld.kind = EwKind::LOAD;
    ld.load = li;
    s.instrs.push_back(ld);
    int k = (int)s.instrs.size() - 1;
    instr_of[in] = k;
    return k;
  };
  for (uint64_t id : rg.nodes) {
    const Node& n = N(id);
    at = std::max(at, pos_[id]);
    EwInstr e;
    if (n.op == Op::BATCH_NORM) {
      // inputs {x, [weight, bias], [running_mean, running_var]} (normalization.cpp:71-80)
      bool affine = n.attr_bool("affine", n.inputs.size() == 5);
      e.kind = EwKind::BN;
      e.p0 = (float)n.attr_float("eps", 1e-5);
      int x = operand(n.inputs[0]);
      size_t k = 1;
      int gamma = -1, beta = -1;
      // per-channel params broadcast along dim 1 of [N,C,H,W]
      auto chan = [&](uint64_t p) -> int {
        const View& pv = value(p);
        View b;
        b = pv;
        b.shape = s.space;
        b.strides.assign(s.space.size(), 0);
        if (!pv.is_splat) b.strides[1] = pv.strides.empty() ? 1 : pv.strides[0];
        s.loads.push_back(b);
        EwInstr ld;
        ld.kind = EwKind::LOAD;
        ld.load = (int)s.loads.size() - 1;
        s.instrs.push_back(ld);
        return (int)s.instrs.size() - 1;
      };
      if (affine) {
        gamma = chan(n.inputs[k++]);
        beta = chan(n.inputs[k++]);
      }
      if (k + 2 > n.inputs.size()) fail(PFC_ERR_UNSUPPORTED, "BATCH_NORM without running statistics");
      int mean = chan(n.inputs[k++]);
      int var = chan(n.inputs[k++]);
      e.a = {x, mean, var, gamma, beta};
    } else if (n.op == Op::CLAMP) {
      e.op = Op::CLAMP;
      int x = operand(n.inputs[0]);
      if (n.inputs.size() >= 3) {
        e.a = {x, operand(n.inputs[1]), operand(n.inputs[2])};
      } else {
        fail(PFC_ERR_UNSUPPORTED, "CLAMP node needs min and max inputs");
      }
    } else {
      e.op = n.op;
      for (uint64_t in : n.inputs) e.a.push_back(operand(in));
      uint16_t ov = (uint16_t)n.op;
      size_t need = (n.op == Op::WHERE) ? 3 : (ov >= 200 && ov < 400) ? 1 : 2;
      if (e.a.size() != need)
        fail(PFC_ERR_GRAPH, std::string("wrong input count for ") + op_name(n.op) + " at node " + std::to_string(id));
    }
    s.instrs.push_back(e);
    instr_of[id] = (int)s.instrs.size() - 1;
  }
  // stores
  for (uint64_t id : rg.nodes) {
    if (!must_materialize(id)) continue;
    View out = dense_like(s.space, layout_ref);
    s.stores.push_back({instr_of[id], out});
    val_[id] = out;
  }
  std::vector<std::pair<int, int64_t>> ptrs;
  auto push_ptrs = [&]() {
    for (const View& l : s.loads) ptrs.push_back({l.is_splat ? -1 : l.buf, l.offset * (int64_t)dtype_size(l.dtype)});
    for (auto& st : s.stores) ptrs.push_back({st.second.buf, 0});
  };
  if (rg.row_ops.empty()) {
    std::string name = kname("ew");
    int grid, block;
    std::string code = gen_ew(s, name, in_.num_sms, &grid, &block);
    push_ptrs();
    ptrs.push_back({P_->scalar_buf, 0});
    emit_jit(at, "fused elementwise " + shape_str(s.space), name, code, grid, block, ptrs);
    return;
  }
  // row group
  rs.red_begin = rg.red_begin;
  rs.red_end = rg.red_end;
  for (uint64_t rid : rg.row_ops) {
    const Node& rn = N(rid);
    at = std::max(at, pos_[rid]);
    RowOp op;
    op.op = rn.op;
    op.src = instr_of.at(rn.inputs[0]);
    if (rn.op == Op::LAYER_NORM) {
      op.eps = (float)rn.attr_float("eps", 1e-5);
      bool affine = rn.attr_bool("elementwise_affine", rn.inputs.size() >= 3);
      if (affine && rn.inputs.size() >= 3) {
        // gamma/beta have shape normalized_shape: broadcast to the row space
        op.gamma = operand(rn.inputs[1]);
        op.beta = operand(rn.inputs[2]);
      }
    }
    if (rn.op == Op::SOFTMAX || rn.op == Op::LOG_SOFTMAX || rn.op == Op::LAYER_NORM) {
      op.out = dense_like(s.space, layout_ref);
    } else {
      op.out = dense(rn.shape, DType::F32);
    }
    val_[rid] = op.out;
    if (!rg.full && prod(s.space, rg.red_end) == 1) plan_row_operand(rid, op);
    rs.ops.push_back(op);
  }
  push_ptrs();
  for (const RowOp& op : rs.ops) ptrs.push_back({op.write_out ? op.out.buf : -1, 0});
  ptrs.push_back({P_->scalar_buf, 0});
  int64_t outer = prod(s.space, 0, rs.red_begin), inner = prod(s.space, rs.red_end);
  std::string label;
  for (const RowOp& op : rs.ops) label += std::string(op_name(op.op)) + " ";
  if (rg.full) {
    std::string name = kname("full");
    int grid, nst[1];
    std::string code = gen_full(rs, name, in_.num_sms, &grid, nst);
    int part = new_buffer((size_t)grid * std::max(1, nst[0]) * 4);
    ptrs.push_back({part, 0});
    // two kernels share one module: emit as two steps with the same source
    Step s1;
    emit_jit(at, "full reduction (" + label + ") " + shape_str(s.space), name, code, grid, 256, ptrs);
    // second kernel
    Step s2 = steps_.back().second;
    s2.jit.kernel = "pf_kernel_fin";
    s2.jit.grid = 1;
    s2.label = "full reduction finalize";
    add_step(at, s2);
    return;
  }
  std::string name = kname(inner == 1 ? "row" : "col");
  int grid, block;
  size_t smem = 0;
  std::string code = inner == 1 ? gen_row(rs, name, in_.num_sms, &grid, &block, &smem)
                                 : gen_col(rs, name, in_.num_sms, &grid, &block);
  (void)outer;
  ptrs.push_back({kErrorFlagBuffer, 0});
  for (const RowOp& op : rs.ops)
    if (op.op_hi >= 0) ptrs.push_back({op.op_hi, 0}), ptrs.push_back({op.op_lo, 0});
  emit_jit(at, std::string(inner == 1 ? "row kernel (" : "column kernel (") + label + ") " + shape_str(s.space), name,
           code, grid, block, ptrs, smem);
}

void Compiler::lower_row_alone(uint64_t id) {
  // A row op whose input is a materialised value: a region with one load.
  Region rg;
  const Node& n = N(id);
  rg.shape = N(n.inputs[0]).shape;
  int rb, re;
  bool full;
  row_structure(id, rg.shape, &rb, &re, &full);
  rg.red_begin = rb;
  rg.red_end = re;
  rg.full = full;
  rg.row_ops.push_back(id);
  regions_.push_back(rg);
  int r = (int)regions_.size() - 1;
  // the region's prologue is just the load of the input: emulate via a COPY-less region
  // by lowering with zero nodes: operand() creates the load lazily.
  Region& R = regions_[r];
  (void)R;
  // Inline lowering (mirrors lower_region with no elementwise nodes)
  RowSpec rs;
  EwSpec& s = rs.ew;
  s.space = rg.shape;
  auto load_instr = [&](uint64_t in, const std::vector<int64_t>& space) -> int {
    View b = broadcast_to(value(in), space);
    s.loads.push_back(b);
    EwInstr ld;
    ld.kind = EwKind::LOAD;
    ld.load = (int)s.loads.size() - 1;
    s.instrs.push_back(ld);
    return (int)s.instrs.size() - 1;
  };
  RowOp op;
  op.op = n.op;
  op.src = load_instr(n.inputs[0], s.space);
  if (n.op == Op::LAYER_NORM) {
    op.eps = (float)n.attr_float("eps", 1e-5);
    bool affine = n.attr_bool("elementwise_affine", n.inputs.size() >= 3);
    if (affine && n.inputs.size() >= 3) {
      op.gamma = load_instr(n.inputs[1], s.space);
      op.beta = load_instr(n.inputs[2], s.space);
    }
  }
  const View& xin = value(n.inputs[0]);
  if (n.op == Op::SOFTMAX || n.op == Op::LOG_SOFTMAX || n.op == Op::LAYER_NORM)
    op.out = dense_like(s.space, xin.is_splat ? nullptr : &xin);
  else
    op.out = dense(n.shape, DType::F32);
  val_[id] = op.out;
  if (!full && prod(s.space, re) == 1) plan_row_operand(id, op);
  rs.ops.push_back(op);
  rs.red_begin = rb;
  rs.red_end = re;
  std::vector<std::pair<int, int64_t>> ptrs;
  for (const View& l : s.loads) ptrs.push_back({l.is_splat ? -1 : l.buf, l.offset * (int64_t)dtype_size(l.dtype)});
  ptrs.push_back({op.write_out ? op.out.buf : -1, 0});
  ptrs.push_back({P_->scalar_buf, 0});
  int64_t inner = prod(s.space, re);
  if (full) {
    std::string name = kname("full");
    int grid, nst[1];
    std::string code = gen_full(rs, name, in_.num_sms, &grid, nst);
    int part = new_buffer((size_t)grid * std::max(1, nst[0]) * 4);
    ptrs.push_back({part, 0});
    emit_jit(pos_[id], std::string("full reduction (") + op_name(n.op) + ")", name, code, grid, 256, ptrs);
    Step s2 = steps_.back().second;
    s2.jit.kernel = "pf_kernel_fin";
    s2.jit.grid = 1;
    s2.label = "full reduction finalize";
    add_step(pos_[id], s2);
    return;
  }
  std::string name = kname(inner == 1 ? "row" : "col");
  int grid, block;
  size_t smem = 0;
  std::string code = inner == 1 ? gen_row(rs, name, in_.num_sms, &grid, &block, &smem)
                                 : gen_col(rs, name, in_.num_sms, &grid, &block);
  ptrs.push_back({kErrorFlagBuffer, 0});
  if (rs.ops[0].op_hi >= 0) ptrs.push_back({rs.ops[0].op_hi, 0}), ptrs.push_back({rs.ops[0].op_lo, 0});
  emit_jit(pos_[id], std::string(inner == 1 ? "row kernel (" : "column kernel (") + op_name(n.op) + ") " +
                         shape_str(s.space),
           name, code, grid, block, ptrs, smem);
}

// Collapse the batch dims [0, nb) of a view to one stride; false if impossible.
static bool collapse_batch(const View& v, int nb, int64_t* stride) {
  if (nb == 0) { *stride = 0; return true; }
  int64_t st = v.strides[nb - 1];
  int64_t span = v.shape[nb - 1];
  for (int d = nb - 2; d >= 0; --d) {
    if (v.shape[d] == 1) continue;
    if (v.strides[d] != st * span) {
      // allow broadcast (all-zero) batch strides
      bool all0 = true;
      for (int e = 0; e < nb; ++e) all0 = all0 && (v.strides[e] == 0 || v.shape[e] == 1);
      if (all0) { *stride = 0; return true; }
      return false;
    }
    span *= v.shape[d];
  }
  *stride = st;
  return true;
}

void Compiler::lower_matmul(const GemmChain& ch, int at) {
  const Node& mm = N(ch.mm);
  View a = value(mm.inputs.at(0));
  View b = value(mm.inputs.at(1));
  if (a.is_splat) a = materialize_copy(a, at, "materialise splat operand");
  if (b.is_splat) b = materialize_copy(b, at, "materialise splat operand");
  // infer_matmul_spec (shape_inference.hpp:146-217): promote 1-D operands.
  bool a1 = a.shape.size() == 1, b1 = b.shape.size() == 1;
  if (a.shape.empty() || b.shape.empty()) fail(PFC_ERR_GRAPH, "matmul requires non-scalar inputs");
  if (a1) { a.shape.insert(a.shape.begin(), 1); a.strides.insert(a.strides.begin(), 0); }
  if (b1) { b.shape.push_back(1); b.strides.push_back(0); }
  int64_t M = a.shape[a.shape.size() - 2], K = a.shape.back();
  int64_t Kb = b.shape[b.shape.size() - 2], Nn = b.shape.back();
  if (K != Kb) fail(PFC_ERR_GRAPH, "matmul: inner dimensions don't match");
  std::vector<int64_t> ab(a.shape.begin(), a.shape.end() - 2), bb(b.shape.begin(), b.shape.end() - 2);
  // broadcast batch shape
  size_t nb = std::max(ab.size(), bb.size());
  std::vector<int64_t> batch(nb);
  for (size_t i = 0; i < nb; ++i) {
    int64_t da = i < nb - ab.size() ? 1 : ab[i - (nb - ab.size())];
    int64_t db = i < nb - bb.size() ? 1 : bb[i - (nb - bb.size())];
    if (da != db && da != 1 && db != 1) fail(PFC_ERR_GRAPH, "matmul: batch dims not broadcastable");
    batch[i] = std::max(da, db);
  }
  int64_t nbatch = prod(batch);
  int prec = in_.precision;
  int64_t kalign = prec == PFC_PRECISION_BF16 ? 64 : 32;
  int64_t kpad = round_up(std::max<int64_t>(K, 1), kalign);
  // A view broadcast to [batch..., M, K]
  std::vector<int64_t> afull = batch;
  afull.push_back(M);
  afull.push_back(K);
  View av = broadcast_to(a, afull);
  // B as [batch..., N, K]: swap the last two dims of the [.., K, N] view
  std::vector<int64_t> bfull = batch;
  bfull.push_back(K);
  bfull.push_back(Nn);
  bool b_batched = !bb.empty() && prod(bb) > 1;
  View bv = b_batched ? broadcast_to(b, bfull) : b;
  if (!b_batched) {
    // drop size-1 batch dims of b
    View t;
    t = b;
    t.shape = {K, Nn};
    t.strides = {b.strides[b.strides.size() - 2], b.strides.back()};
    bv = t;
  }
  {
    size_t r = bv.shape.size();
    std::swap(bv.shape[r - 2], bv.shape[r - 1]);
    std::swap(bv.strides[r - 2], bv.strides[r - 1]);
  }
  int64_t gbatch = b_batched ? nbatch : 1;
  int64_t gM = b_batched ? M : nbatch * M;
  if (gM == 0 || Nn == 0 || nbatch == 0) {
    // an empty product: nothing to compute, the (empty) output needs no launch
    val_[ch.result] = dense(mm.shape, DType::F32);
    return;
  }
  // prepared operands
  int64_t arows = nbatch * M, brows = (b_batched ? nbatch : 1) * Nn;
  const Operand opa = prepare_operand(av, arows, K, kpad, prec, "prepare A " + shape_str(afull), at);
  const Operand opb = prepare_operand(bv, brows, K, kpad, prec, "prepare B " + shape_str(bv.shape), at);
  // output: node shape of the chain result (same as matmul shape)
  View c = dense(mm.shape, DType::F32);
  Step sg;
  sg.kind = StepKind::GEMM;
  sg.label = "gemm " + std::to_string(gbatch) + "x[" + std::to_string(gM) + "x" + std::to_string(Nn) + "x" +
             std::to_string(K) + "]";
  GemmArgs& G = sg.gemm;
  G.precision = prec;
  G.a_hi = opa.hi;
  G.a_lo = opa.lo;
  G.b_hi = opb.hi;
  G.b_lo = opb.lo;
  G.batch = gbatch;
  G.M = gM;
  G.N = Nn;
  G.K = K;
  G.kpad = kpad;
  G.a_sb = gbatch > 1 ? M * kpad : 0;
  G.b_sb = gbatch > 1 ? Nn * kpad : 0;
  G.c = c;
  G.c_sn = 1;
  G.c_sm = Nn;
  G.c_sb = gbatch > 1 ? M * Nn : 0;
  G.alpha = ch.alpha;
  G.alpha_slot = ch.alpha_slot;
  G.act = ch.act;
  if (ch.has_bias) {
    View bv2 = value(ch.bias);
    // contiguous along n? (a bias of equal values stays a scalar)
    int64_t sn = 0;
    for (size_t d = 0; d < bv2.shape.size(); ++d)
      if (bv2.shape[d] != 1) sn = bv2.strides[d];
    if (!bv2.is_splat && sn != 1 && Nn > 1) bv2 = materialize_copy(bv2, at, "contiguous bias");
    G.bias = bv2;
    G.has_bias = true;
  }
  if (ch.has_residual) {
    View r = broadcast_to(value(ch.residual), mm.shape);
    if (r.is_splat) r = materialize_copy(r, at, "materialise residual");
    size_t rd = r.shape.size();
    int64_t rsb = 0;
    bool ok;
    if (gbatch > 1) {
      ok = collapse_batch(r, (int)rd - 2, &rsb);
      G.r_sm = r.strides[rd - 2];
    } else {
      // rows (batch..., M) must collapse into one stride
      View rr = r;
      int64_t st;
      ok = collapse_batch(rr, (int)rd - 1, &st);
      G.r_sm = rd >= 2 ? st : 0;
      if (rd == 1) G.r_sm = 0;
    }
    if (!ok) {
      r = materialize_copy(r, at, "contiguous residual");
      rsb = gbatch > 1 ? M * Nn : 0;
      G.r_sm = Nn;
    }
    G.residual = r;
    G.r_sb = rsb;
    G.r_sn = r.strides[rd - 1];
    G.has_residual = true;
  }
  add_step(at, sg);
  // result view with the chain result's shape (== mm shape)
  val_[ch.result] = c;
}

void Compiler::lower_conv(const GemmChain& ch, int at) {
  const Node& cv = N(ch.mm);
  View x = value(cv.inputs.at(0));
  View w = value(cv.inputs.at(1));
  if (x.is_splat) x = materialize_copy(x, at, "materialise conv input");
  if (w.is_splat) w = materialize_copy(w, at, "materialise conv weight");
  if (x.shape.size() != 4 || w.shape.size() != 4) fail(PFC_ERR_GRAPH, "Conv2d expects 4D input and weight");
  // attributes stride/padding/dilation (vector<int64_t>), groups (int64_t): conv.cpp:114-117
  auto st = cv.attr_ints("stride", {1, 1}), pd = cv.attr_ints("padding", {0, 0}), dl = cv.attr_ints("dilation", {1, 1});
  int64_t groups = cv.attr_int("groups", 1);
  if (groups != 1) fail(PFC_ERR_UNSUPPORTED, "grouped CONV2D is not supported");
  int64_t Nimg = x.shape[0], Cin = x.shape[1], H = x.shape[2], W = x.shape[3];
  int64_t O = w.shape[0], KH = w.shape[2], KW = w.shape[3];
  if (w.shape[1] != Cin) fail(PFC_ERR_GRAPH, "Input channels mismatch");
  int64_t OH = (H + 2 * pd[0] - dl[0] * (KH - 1) - 1) / st[0] + 1;  // conv.cpp:75-78
  int64_t OW = (W + 2 * pd[1] - dl[1] * (KW - 1) - 1) / st[1] + 1;
  if (cv.shape != std::vector<int64_t>{Nimg, O, OH, OW}) fail(PFC_ERR_GRAPH, "CONV2D output shape mismatch");
  int prec = in_.precision;
  // Implicit GEMM: rows m = (n*OH + oh)*OW + ow, columns k = (kh*KW + kw)*Cp + c
  // over a channels-last copy of the input with Cp channels (C rounded up to
  // a 16-byte chunk), gathered tile by tile inside the GEMM.
  const int64_t chunk = prec == PFC_PRECISION_BF16 ? 8 : 4;
  const int64_t Cp = round_up(Cin, chunk);
  // A filter row of few channels (Cp*KW <= one k-block) is laid out as one
  // k-block of KWp taps (zero weights past KW) over a zero-padded input, so
  // each k-block of A is a 128-byte window of one padded input row (TMA-fed).
  const int64_t bk = prec == PFC_PRECISION_BF16 ? 64 : 32;
  const bool window = Cp * KW <= bk && bk % Cp == 0 && dl[1] == 1;
  // A stride-1 filter over whole k-blocks of channels whose output rows are
  // narrower than the 32-pixel TMA boxes also reads a zero-padded input:
  // numbering output pixels in its padded row space turns every tap into a
  // row offset, so the GEMM stages each tile's input rows (the halo) once per
  // channel block and enters them per tap.  The halo of 128 pixels must fit
  // one 256-row copy.  (At 64 output channels the two TMA-fed forms run at the
  // same rate, and wider rows keep the unpadded input that producers write.)
  const int64_t reach = (KH - 1) * dl[0] * (W + 2 * pd[1]) + (KW - 1) * dl[1];
  const bool halo = !window && st[0] == 1 && st[1] == 1 && Cp % bk == 0 && OW < 32 &&
                    round_up(128 + reach, 8) <= 256;
  const int64_t KWp = window ? bk / Cp : KW;
  int64_t K = KH * KWp * Cp;
  int64_t kpad = round_up(K, bk);
  size_t esz = prec == PFC_PRECISION_BF16 ? 2 : 4;
  int64_t M = Nimg * OH * OW;
  Step si;
  si.kind = StepKind::CONV_INPUT;
  si.label = "conv input (channels-last) " + shape_str(x.shape);
  ConvInputArgs& I = si.convin;
  I.x = x;
  I.cp = Cp;
  I.precision = prec;
  int64_t Hp = 0, Wp = 0;
  if (window || halo) {
    Hp = std::max(H + 2 * pd[0], (OH - 1) * st[0] + (KH - 1) * dl[0] + 1);
    Wp = std::max(W + 2 * pd[1], (OW - 1) * st[1] + (KWp - 1) * dl[1] + 1);
    I.hp = Hp; I.wp = Wp; I.ph = pd[0]; I.pw = pd[1];
    si.label = "conv input (channels-last, padded) " + shape_str(x.shape);
  }
  const size_t xbytes = (size_t)(Nimg * (Hp > 0 ? Hp * Wp : H * W) * Cp) * esz;
  I.out_hi = new_buffer(xbytes);
  I.out_lo = prec == PFC_PRECISION_BF16 ? -1 : new_buffer(xbytes);
  const Operand opw = prepare_operand(w, O, K, kpad, prec, "prepare conv weight", at, Cp, KWp);
  // output NHWC: logical [N,O,OH,OW], strides (OH*OW*O, 1, OW*O, O)
  View c;
  c.shape = {Nimg, O, OH, OW};
  c.strides = {OH * OW * O, 1, OW * O, O};
  c.dtype = DType::F32;
  c.buf = new_buffer((size_t)M * O * 4);
  Step sg;
  sg.kind = StepKind::GEMM;
  sg.label = "conv gemm [" + std::to_string(M) + "x" + std::to_string(O) + "x" + std::to_string(K) + "]";
  GemmArgs& G = sg.gemm;
  G.precision = prec;
  G.b_hi = opw.hi; G.b_lo = opw.lo;
  G.conv = true;
  G.x_hi = I.out_hi; G.x_lo = I.out_lo;
  G.H = H; G.W = W; G.Cp = Cp; G.KH = KH; G.KW = KW; G.sh = st[0]; G.sw = st[1];
  G.ph = pd[0]; G.pw = pd[1]; G.dh = dl[0]; G.dw = dl[1]; G.OH = OH; G.OW = OW;
  G.Nimg = Nimg; G.Hp = Hp; G.Wp = Wp; G.KWp = KWp;
  G.batch = 1; G.M = M; G.N = O; G.K = K; G.kpad = kpad;
  G.c = c; G.c_sm = O; G.c_sn = 1; G.c_sb = 0;
  G.act = ch.act;
  if (ch.has_bias && !ch.has_bn) {
    View bv = value(ch.bias);
    int64_t sn = 0;
    for (size_t d = 0; d < bv.shape.size(); ++d)
      if (bv.shape[d] != 1) sn = bv.strides[d];
    if (!bv.is_splat && sn != 1 && O > 1) bv = materialize_copy(bv, at, "contiguous bias");
    G.bias = bv;
    G.has_bias = true;
  }
  if (ch.has_bn) {
    const Node& bn = N(ch.bn);
    Step sf;
    sf.kind = StepKind::BN_FOLD;
    sf.label = "fold batch_norm";
    BnFoldArgs& F = sf.bnfold;
    F.channels = O;
    F.eps = (float)bn.attr_float("eps", 1e-5);
    bool affine = bn.attr_bool("affine", bn.inputs.size() == 5);
    size_t k = 1;
    if (affine) {
      F.gamma = value(bn.inputs[k++]);
      F.beta = value(bn.inputs[k++]);
      F.has_gamma = F.has_beta = true;
    }
    if (k + 2 > bn.inputs.size()) fail(PFC_ERR_UNSUPPORTED, "BATCH_NORM without running statistics");
    F.mean = value(bn.inputs[k++]);
    F.var = value(bn.inputs[k++]);
    if (ch.has_bias) {
      F.bias = value(ch.bias);
      F.has_bias = true;
    }
    F.out_scale = new_buffer((size_t)O * 4);
    F.out_shift = new_buffer((size_t)O * 4);
    G.scale_buf = F.out_scale;
    G.shift_buf = F.out_shift;
    add_step(at, sf);
  }
  add_step(at, si);
  add_step(at, sg);
  val_[ch.result] = c;
}

void Compiler::lower_chain(int ci) {
  if (attn_.count(ci)) {
    lower_attention(ci);
    return;
  }
  if (small_.count(ci)) {
    lower_small(ci);
    return;
  }
  const GemmChain& ch = chains_[ci];
  int at = pos_[ch.result];
  if (cls_[ch.mm] == Cls::CONV) lower_conv(ch, at);
  else lower_matmul(ch, at);
}

void Compiler::lower_pool(uint64_t id) {
  const Node& n = N(id);
  View x = value(n.inputs.at(0));
  if (x.is_splat) x = materialize_copy(x, pos_[id], "materialise pool input");
  if (x.shape.size() != 4) fail(PFC_ERR_GRAPH, "pooling expects 4D input [N, C, H, W]");
  Step s;
  s.kind = StepKind::POOL;
  PoolArgs& p = s.pool;
  p.x = x;
  if (n.op == Op::ADAPTIVE_AVG_POOL2D) {
    // attribute output_size (vector<int64_t>), pooling.cpp:163-164
    p.mode = 2;
    s.label = "adaptive_avg_pool2d";
  } else {
    // attributes kernel_size/stride/padding (vector<int64_t>), pooling.cpp:57-59
    auto ks = n.attr_ints("kernel_size"), st = n.attr_ints("stride", ks), pd = n.attr_ints("padding", {0, 0});
    p.mode = n.op == Op::MAX_POOL2D ? 0 : 1;
    p.kh = ks[0]; p.kw = ks[1]; p.sh = st[0]; p.sw = st[1]; p.ph = pd[0]; p.pw = pd[1];
    int64_t oh = (x.shape[2] + 2 * p.ph - p.kh) / p.sh + 1, ow = (x.shape[3] + 2 * p.pw - p.kw) / p.sw + 1;
    if (n.shape != std::vector<int64_t>{x.shape[0], x.shape[1], oh, ow}) fail(PFC_ERR_GRAPH, "pool output shape mismatch");
    s.label = n.op == Op::MAX_POOL2D ? "max_pool2d" : "avg_pool2d";
  }
  p.y = dense_like(n.shape, &x);
  val_[id] = p.y;
  add_step(pos_[id], s);
}

void Compiler::lower_concat(uint64_t id) {
  const Node& n = N(id);
  View out = dense(n.shape, n.dtype);
  int nd = (int)n.shape.size();
  int d = (int)n.attr_int("dim", 0);
  bool stack = n.op == Op::STACK;
  if (d < 0) d += nd;
  if (d < 0 || d >= nd) fail(PFC_ERR_GRAPH, "concat: dimension out of range");
  int64_t off = 0;
  for (uint64_t in : n.inputs) {
    View src = value(in);
    View dst = out;
    int64_t len = stack ? 1 : src.shape[d];
    dst.shape[d] = len;
    dst.offset = out.offset + off * out.strides[d];
    if (stack) {
      View s2;
      std::vector<int64_t> sh = src.shape;
      sh.insert(sh.begin() + d, 1);
      if (src.is_splat) { s2 = src; s2.shape = sh; s2.strides.assign(sh.size(), 0); }
      else { s2 = src; s2.shape = sh; s2.strides.insert(s2.strides.begin() + d, 0); }
      src = s2;
    }
    EwSpec s;
    s.space = dst.shape;
    s.loads.push_back(broadcast_to(src, s.space));
    EwInstr ld;
    ld.kind = EwKind::LOAD;
    ld.load = 0;
    s.instrs.push_back(ld);
    View dstv = dst;
    dstv.offset = 0;  // pointer argument carries the offset
    s.stores.push_back({0, dstv});
    std::string name = kname("concat");
    int grid, block;
    std::string code = gen_ew(s, name, in_.num_sms, &grid, &block);
    std::vector<std::pair<int, int64_t>> ptrs;
    ptrs.push_back({src.is_splat ? -1 : src.buf, src.offset * (int64_t)dtype_size(src.dtype)});
    ptrs.push_back({out.buf, dst.offset * (int64_t)dtype_size(out.dtype)});
    ptrs.push_back({P_->scalar_buf, 0});
    emit_jit(pos_[id], "concat part", name, code, grid, block, ptrs);
    off += len;
  }
  val_[id] = out;
}

void Compiler::lower() {
  // Units: an elementwise region (with its attached row ops), an epilogue
  // chain, or a single node.  Regions are convex and chains only absorb
  // operands that do not depend on them, so the unit graph is acyclic.
  std::unordered_map<uint64_t, int> unit_of;
  std::vector<int> kind;  // 0 node, 1 region, 2 chain
  std::vector<int64_t> ref;
  std::unordered_map<int, int> unit_of_region, unit_of_chain;
  for (uint64_t id : order_) {
    int u;
    auto ch = chain_of_.find(id);
    auto rr = row_region_.find(id);
    auto rg = region_of_.find(id);
    if (ch != chain_of_.end()) {
      auto it = unit_of_chain.find(ch->second);
      if (it == unit_of_chain.end()) {
        kind.push_back(2); ref.push_back(ch->second);
        it = unit_of_chain.emplace(ch->second, (int)kind.size() - 1).first;
      }
      u = it->second;
    } else if (rg != region_of_.end() || rr != row_region_.end()) {
      int r = rg != region_of_.end() ? rg->second : rr->second;
      auto it = unit_of_region.find(r);
      if (it == unit_of_region.end()) {
        kind.push_back(1); ref.push_back(r);
        it = unit_of_region.emplace(r, (int)kind.size() - 1).first;
      }
      u = it->second;
    } else {
      kind.push_back(0); ref.push_back((int64_t)id);
      u = (int)kind.size() - 1;
    }
    unit_of[id] = u;
  }
  int nu = (int)kind.size();
  std::vector<std::set<int>> succ(nu);
  std::vector<int> indeg(nu, 0), prio(nu, INT32_MAX);
  for (uint64_t id : order_) {
    int u = unit_of[id];
    prio[u] = std::min(prio[u], pos_[id]);
    for (uint64_t in : N(id).inputs) {
      int v = unit_of.at(in);
      if (v != u && succ[v].insert(u).second) indeg[u]++;
    }
  }
  std::set<std::pair<int, int>> ready;
  for (int u = 0; u < nu; ++u)
    if (!indeg[u]) ready.insert({prio[u], u});
  if (std::getenv("PFB_DEBUG_UNITS"))
    for (uint64_t id : order_) std::fprintf(stderr, "node %llu -> unit %d (indeg %d)\n", (unsigned long long)id, unit_of[id], indeg[unit_of[id]]);
  int step_pos = 0;
  int lowered = 0;
  while (!ready.empty()) {
    int u = ready.begin()->second;
    ready.erase(ready.begin());
    ++lowered;
    cur_pos_ = step_pos++;
    if (std::getenv("PFB_DEBUG_UNITS"))
      std::fprintf(stderr, "unit %d kind %d ref %lld prio %d\n", u, kind[u], (long long)ref[u], prio[u]);
    if (kind[u] == 1) {
      lower_region((int)ref[u]);
    } else if (kind[u] == 2) {
      lower_chain((int)ref[u]);
    } else {
      uint64_t id = (uint64_t)ref[u];
      switch (cls_[id]) {
        case Cls::LEAF: lower_leaf(id); break;
        case Cls::VIEW: lower_view(id); break;
        case Cls::ROW: lower_row_alone(id); break;
        case Cls::POOL: lower_pool(id); break;
        case Cls::CONCAT: lower_concat(id); break;
        default: fail(PFC_ERR_INTERNAL, "unlowered node class");
      }
    }
    for (int v : succ[u])
      if (--indeg[v] == 0) ready.insert({prio[v], v});
  }
  if (lowered != nu) fail(PFC_ERR_INTERNAL, "fusion produced a cyclic unit graph");
  cur_pos_ = step_pos;
}

// Operand preparation moved into the producer.  A SPLIT of a GEMM's output
// (the A operand of the next GEMM: dense rows, K = the producer's N = kpad)
// and a CONV_INPUT of a GEMM's or pool's channels-last output (C = Cp) are
// written by the producer's epilogue directly, and the preparation step is
// dropped; the fp32 value is still written when anything else reads it.
void Compiler::emit_operands_at_producers() {
  std::vector<Step>& S = P_->steps;
  const int nb = (int)P_->buffers.size();
  std::vector<std::vector<int>> refs(nb);  // buffer -> steps referring to it
  auto add = [&](int buf, int i) {
    if (buf >= 0 && buf < nb) refs[buf].push_back(i);
  };
  for (int i = 0; i < (int)S.size(); ++i) {
    const Step& st = S[i];
    switch (st.kind) {
      case StepKind::JIT: for (auto& pr : st.jit.ptrs) add(pr.first, i); break;
      case StepKind::SPLIT: add(st.split.src.buf, i); add(st.split.out_hi, i); add(st.split.out_lo, i); break;
      case StepKind::IM2COL: add(st.im2col.x.buf, i); add(st.im2col.out_hi, i); add(st.im2col.out_lo, i); break;
      case StepKind::CONV_INPUT: add(st.convin.x.buf, i); add(st.convin.out_hi, i); add(st.convin.out_lo, i); break;
      case StepKind::GEMM: {
        const GemmArgs& G = st.gemm;
        add(G.a_hi, i); add(G.a_lo, i); add(G.b_hi, i); add(G.b_lo, i); add(G.c.buf, i);
        if (G.has_bias) add(G.bias.buf, i);
        if (G.has_residual) add(G.residual.buf, i);
        add(G.scale_buf, i); add(G.shift_buf, i); add(G.x_hi, i); add(G.x_lo, i);
        if (G.pool) add(G.pool_y.buf, i);
        add(G.gap_buf, i);
        break;
      }
      case StepKind::POOL: add(st.pool.x.buf, i); add(st.pool.y.buf, i); break;
      case StepKind::BN_FOLD: {
        const BnFoldArgs& F = st.bnfold;
        add(F.gamma.buf, i); add(F.beta.buf, i); add(F.mean.buf, i); add(F.var.buf, i); add(F.bias.buf, i);
        add(F.out_scale, i); add(F.out_shift, i);
        break;
      }
      case StepKind::MEMSET: add(st.memset_buf, i); break;
      case StepKind::ATTENTION: {
        const AttnArgs& A = st.attn;
        add(A.q_hi, i); add(A.q_lo, i); add(A.k_hi, i); add(A.k_lo, i); add(A.v_hi, i); add(A.v_lo, i);
        add(A.c.buf, i); add(A.op_hi, i); add(A.op_lo, i);
        break;
      }
      case StepKind::SMALL: {
        const SmallArgs& Sm = st.small;
        add(Sm.a.buf, i); add(Sm.l1.w_buf, i); add(Sm.l2.w_buf, i); add(Sm.h_buf, i); add(Sm.counter_buf, i);
        add(Sm.out.buf, i);
        if (Sm.l1.has_bias) add(Sm.l1.bias.buf, i);
        if (Sm.l2.has_bias) add(Sm.l2.bias.buf, i);
        break;
      }
    }
  }
  std::unordered_set<int> out_bufs;
  for (const View& v : P_->output_views) out_bufs.insert(v.buf);
  // the step writing buffer b: the GEMM or pool whose output it is
  auto producer = [&](int b) -> int {
    for (int j : refs[b]) {
      const Step& st = S[j];
      if (st.kind == StepKind::GEMM && st.gemm.c.buf == b && st.gemm.write_c) return j;
      if (st.kind == StepKind::POOL && st.pool.y.buf == b && st.pool.write_y) return j;
      if (st.kind == StepKind::ATTENTION && st.attn.c.buf == b && st.attn.write_c) return j;
    }
    return -1;
  };
  std::vector<bool> drop(S.size(), false);
  auto others_read = [&](int b, int j, int i) {
    if (out_bufs.count(b)) return true;
    for (int u : refs[b])
      if (u != j && u != i && !drop[u]) return true;
    return false;
  };
  for (int i = 0; i < (int)S.size(); ++i) {
    Step& st = S[i];
    if (st.kind == StepKind::SPLIT && !st.once && st.split.conv_cp == 0) {
      const View& v = st.split.src;
      if (v.is_splat || v.buf < 0 || v.offset != 0) continue;
      const bool dense_src = v.strides == View::dense_strides(v.shape);
      const int j = producer(v.buf);
      if (j >= 0 && j < i && S[j].kind == StepKind::ATTENTION && dense_src) {
        // the attention's O as a dense [rows, cols] matrix (heads merged)
        AttnArgs& A = S[j].attn;
        const size_t r = A.c.shape.size();
        const int64_t H = r == 4 ? A.c.shape[1] : 1;
        const int64_t cols = H * A.d, rows = A.batch / H * A.M;
        const bool merged = r == 4 ? A.c.strides == std::vector<int64_t>{A.M * cols, A.d, cols, 1}
                                   : A.c.strides == View::dense_strides(A.c.shape);
        if (A.op_hi >= 0 || !merged || A.c.offset != 0 || st.split.cols != cols || st.split.kpad != cols ||
            st.split.rows != rows || cols % 4 != 0)
          continue;
        A.op_hi = st.split.out_hi;
        A.op_lo = st.split.out_lo;
        drop[i] = true;
        A.write_c = others_read(v.buf, j, i);
        S[j].label += " +operand";
        continue;
      }
      if (j < 0 || j > i || S[j].kind != StepKind::GEMM) continue;
      GemmArgs& G = S[j].gemm;
      const bool dense_c = G.c.offset == 0 && G.c_sn == 1 && G.c_sm == G.N && (G.batch == 1 || G.c_sb == G.M * G.N);
      // the per-head split of a projection, [B, H, L, D] over a dense [B*L, H*D]
      // output (what attention reads as Q and K): the epilogue writes it head-split
      if (st.split.src.shape.size() == 4 && !G.conv && G.batch == 1 && dense_c && G.op_hi < 0) {
        const std::vector<int64_t>& sh = st.split.src.shape;
        const int64_t B = sh[0], H = sh[1], L = sh[2], D = sh[3];
        const std::vector<int64_t> want{L * H * D, D, H * D, 1};
        if (st.split.src.strides == want && B * L == G.M && H * D == G.N && st.split.cols == D &&
            st.split.kpad == D && st.split.rows == B * H * L && D % 16 == 0 && L % 32 == 0) {
          G.op_hi = st.split.out_hi;
          G.op_lo = st.split.out_lo;
          G.op_sm = D;
          G.op_heads = H;
          G.op_rows = L;
          drop[i] = true;
          G.write_c = others_read(v.buf, j, i);
          S[j].label += " +heads";
        }
        continue;
      }
      if (!dense_src || G.op_hi >= 0 || !dense_c || st.split.cols != G.N || st.split.kpad != G.N || G.N % 4 != 0 ||
          st.split.rows != G.batch * G.M)
        continue;
      G.op_hi = st.split.out_hi;
      G.op_lo = st.split.out_lo;
      G.op_sm = st.split.kpad;
      drop[i] = true;
      G.write_c = others_read(v.buf, j, i);
      S[j].label += " +operand";
    } else if (st.kind == StepKind::CONV_INPUT) {
      const View& x = st.convin.x;  // [N,C,H,W]
      if (x.is_splat || x.buf < 0 || x.offset != 0 || x.shape.size() != 4 || x.shape[1] != st.convin.cp ||
          st.convin.hp > 0)
        continue;
      const int64_t C = x.shape[1], H = x.shape[2], W = x.shape[3];
      if (x.strides != std::vector<int64_t>{H * W * C, 1, W * C, C}) continue;  // channels-last
      const int j = producer(x.buf);
      if (j < 0 || j > i) continue;
      if (S[j].kind == StepKind::GEMM) {
        GemmArgs& G = S[j].gemm;
        if (G.op_hi >= 0 || G.batch != 1 || G.c.offset != 0 || G.c_sn != 1 || G.c_sm != C || G.N != C || C % 4 != 0)
          continue;
        G.op_hi = st.convin.out_hi;
        G.op_lo = st.convin.out_lo;
        G.op_sm = C;
        drop[i] = true;
        G.write_c = others_read(x.buf, j, i);
        S[j].label += " +operand";
      } else if (S[j].kind == StepKind::POOL) {
        PoolArgs& Pl = S[j].pool;
        if (Pl.op_hi >= 0 || Pl.y.offset != 0 || Pl.y.strides != x.strides || Pl.y.shape != x.shape) continue;
        Pl.op_hi = st.convin.out_hi;
        Pl.op_lo = st.convin.out_lo;
        drop[i] = true;
        Pl.write_y = others_read(x.buf, j, i);
        S[j].label += " +operand";
      }
    }
  }
  // A ReLU convolution read only by a 3x3 / stride 2 max pool (padding 0 or 1)
  // (PyFlame's Conv2d -> BatchNorm -> ReLU -> MaxPool2d stem): the pool runs
  // in the convolution's epilogue and the convolution's output never reaches
  // memory.  The epilogue takes the windowed TMA feed with 64-pixel tiles and
  // 64 output channels (launch_gemm's conv_tma_mode 2, not the halo feed).
  for (int i = 0; i < (int)S.size(); ++i) {
    if (drop[i] || S[i].kind != StepKind::POOL) continue;
    PoolArgs& Pl = S[i].pool;
    if (Pl.mode != 0 || Pl.kh != 3 || Pl.kw != 3 || Pl.sh != 2 || Pl.sw != 2 || Pl.ph != Pl.pw || Pl.ph < 0 ||
        Pl.ph > 1)
      continue;
    const View& x = Pl.x;
    if (x.is_splat || x.buf < 0) continue;
    const int j = producer(x.buf);
    if (j < 0 || j > i || drop[j] || S[j].kind != StepKind::GEMM) continue;
    GemmArgs& G = S[j].gemm;
    if (!G.conv || G.pool || G.act != 1 || G.has_residual || G.N != 64 || G.batch != 1 || G.op_hi >= 0 || !G.write_c)
      continue;

    if (x.offset != G.c.offset || x.shape != G.c.shape || x.strides != G.c.strides || others_read(x.buf, j, i)) continue;
    const int64_t esz = G.precision == PFC_PRECISION_BF16 ? 2 : 4, bk = 128 / esz;
    const int64_t kwp = G.KWp > 0 ? G.KWp : G.KW;
    const bool halo = G.sh == 1 && G.sw == 1 && G.Cp % bk == 0 && kwp == G.KW;
    if (halo || G.Hp == 0 || kwp * G.Cp != bk || G.dw != 1 || (G.sw * G.Cp * esz) % 16 != 0 || G.OW <= 32) continue;
    const View& y = Pl.y;
    if (y.shape.size() != 4 || y.strides[1] != 1 || y.offset % 4 != 0 || y.strides[0] % 4 != 0 ||
        y.strides[2] % 4 != 0 || y.strides[3] % 4 != 0 || y.shape[1] != 64 ||
        y.shape[2] != (G.OH + 2 * Pl.ph - 3) / 2 + 1 || y.shape[3] != (G.OW + 2 * Pl.pw - 3) / 2 + 1 ||
        y.shape[2] < 1 || y.shape[3] < 1)
      continue;
    G.pool = true;
    G.pool_pad = (int)Pl.ph;
    G.pool_y = y;
    G.write_pool_y = Pl.write_y;
    G.op_hi = Pl.op_hi;
    G.op_lo = Pl.op_lo;
    G.write_c = false;
    drop[i] = true;
    S[j].label += Pl.op_hi >= 0 ? " +max_pool2d +operand" : " +max_pool2d";
    // A stride-2 stem whose filter rows are 8 taps of 16-byte pixels reads
    // its padded input as row runs (even columns, then odd ones: a 1 KB run
    // per input row and tile instead of overlapping windows) when nothing
    // else reads the padded copy.
    if (G.Cp * esz == 16 && kwp == 8 && G.sh == 2 && G.sw == 2 && G.dh == 1 && G.KH <= 7 && G.Wp % 2 == 0 &&
        G.Wp / 2 >= G.OW + 3) {
      for (int k = 0; k < j; ++k) {
        if (drop[k] || S[k].kind != StepKind::CONV_INPUT || S[k].convin.out_hi != G.x_hi) continue;
        ConvInputArgs& I = S[k].convin;
        if (I.hp != G.Hp || I.wp != G.Wp || others_read(G.x_hi, k, j) || (G.x_lo >= 0 && others_read(G.x_lo, k, j)))
          break;
        I.deint = true;
        G.deint = true;
        S[k].label += " (de-interleaved rows)";
        S[j].label += " (row runs)";
        break;
      }
    }
  }
  // A convolution (no activation or ReLU) read only by AdaptiveAvgPool2d(1)
  // whose A operand is fed by TMA boxes or windows (output tiles inside one
  // image): the epilogue writes per-tile column sums instead of the output
  // (774400 x 64 fp32 for the conv stack's last convolution), and the pool
  // step adds each image's sums.
  for (int i = 0; i < (int)S.size(); ++i) {
    if (drop[i] || S[i].kind != StepKind::POOL) continue;
    PoolArgs& Pl = S[i].pool;
    if (Pl.mode != 2 || Pl.y.shape.size() != 4 || Pl.y.shape[2] != 1 || Pl.y.shape[3] != 1) continue;
    const View& x = Pl.x;
    if (x.is_splat || x.buf < 0) continue;
    const int j = producer(x.buf);
    if (j < 0 || j > i || drop[j] || S[j].kind != StepKind::GEMM) continue;
    GemmArgs& G = S[j].gemm;
    if (!G.conv || G.pool || G.gap_buf >= 0 || G.has_residual || G.batch != 1 || G.op_hi >= 0 || !G.write_c ||
        G.OW < 32 || (G.act != 0 && G.act != 1))
      continue;
    if (x.offset != G.c.offset || x.shape != G.c.shape || x.strides != G.c.strides || others_read(x.buf, j, i)) continue;
    // the feeds of launch_gemm's conv_tma_mode 1 and 2 (not the halo feed)
    const int64_t esz = G.precision == PFC_PRECISION_BF16 ? 2 : 4, bk = 128 / esz;
    const int64_t kwp = G.KWp > 0 ? G.KWp : G.KW;
    const bool halo = G.Hp > 0 && G.sh == 1 && G.sw == 1 && G.Cp % bk == 0 && kwp == G.KW;
    const bool boxes = G.Hp == 0 && G.Cp % bk == 0 && G.sh == 1 && G.sw == 1 && kwp == G.KW;
    const bool windows = G.Hp > 0 && kwp * G.Cp == bk && G.dw == 1 && (G.sw * G.Cp * esz) % 16 == 0;
    if (halo || !(boxes || windows)) continue;
    const int64_t slots = conv_gap_slots(G.OH, G.OW);
    G.gap_buf = new_buffer((size_t)(G.Nimg * slots * G.N) * 4);
    G.write_c = false;
    View pv;
    pv.buf = G.gap_buf;
    pv.shape = {G.Nimg, G.N, slots, 1};
    pv.strides = {slots * G.N, 1, G.N, G.N};
    Pl.x = pv;
    Pl.mode = 3;
    Pl.count = G.OH * G.OW;
    S[j].label += " +average sums";
    S[i].label = "adaptive_avg_pool2d (from the convolution's sums)";
  }
  std::vector<Step> kept;
  for (int i = 0; i < (int)S.size(); ++i)
    if (!drop[i]) kept.push_back(std::move(S[i]));
  S = std::move(kept);
}

void Compiler::finish() {
  for (const OpKey& k : must_claim_)
    if (!claimed_.count(k))
      fail(PFC_ERR_INTERNAL, "a row kernel's operand output was not taken by its GEMM (buffer " +
                                 std::to_string(std::get<0>(k)) + ")");
  // outputs: dense contiguous views (copies run after everything else)
  for (uint64_t o : in_.outputs) {
    View v = value(o);
    const Node& n = N(o);
    bool dense_ok = !v.is_splat && v.is_contiguous() && v.shape == n.shape && v.offset == 0;
    if (!dense_ok) {
      View c = materialize_copy(v, cur_pos_, "materialise output %" + std::to_string(o));
      c.shape = n.shape;
      c.strides = View::dense_strides(n.shape);
      v = c;
    }
    P_->output_views.push_back(v);
  }
  P_->buffers[P_->scalar_buf].bytes = std::max<size_t>(4, P_->scalars.size() * 4);
  // order steps by position (stable keeps emission order within a position)
  std::stable_sort(steps_.begin(), steps_.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
  for (auto& [pos, s] : steps_) P_->steps.push_back(std::move(s));
  emit_operands_at_producers();
  // liveness
  auto use = [&](int buf, int step) {
    if (buf < 0) return;
    Buffer& b = P_->buffers[buf];
    if (b.first_use < 0 || step < b.first_use) b.first_use = step;
    b.last_use = std::max(b.last_use, step);
  };
  for (int i = 0; i < (int)P_->steps.size(); ++i) {
    const Step& s = P_->steps[i];
    switch (s.kind) {
      case StepKind::JIT: for (auto& p : s.jit.ptrs) use(p.first, i); break;
      case StepKind::SPLIT: use(s.split.src.buf, i); use(s.split.out_hi, i); use(s.split.out_lo, i); break;
      case StepKind::IM2COL: use(s.im2col.x.buf, i); use(s.im2col.out_hi, i); use(s.im2col.out_lo, i); break;
      case StepKind::CONV_INPUT: use(s.convin.x.buf, i); use(s.convin.out_hi, i); use(s.convin.out_lo, i); break;
      case StepKind::GEMM: {
        const GemmArgs& G = s.gemm;
        use(G.a_hi, i); use(G.a_lo, i); use(G.b_hi, i); use(G.b_lo, i);
        if (G.write_c) use(G.c.buf, i);
        if (G.pool && G.write_pool_y) use(G.pool_y.buf, i);
        use(G.op_hi, i); use(G.op_lo, i); use(G.gap_buf, i);
        if (G.conv) { use(G.x_hi, i); use(G.x_lo, i); }
        if (G.has_bias) use(G.bias.buf, i);
        if (G.has_residual) use(G.residual.buf, i);
        use(G.scale_buf, i); use(G.shift_buf, i);
        break;
      }
      case StepKind::POOL:
        use(s.pool.x.buf, i);
        if (s.pool.write_y) use(s.pool.y.buf, i);
        use(s.pool.op_hi, i); use(s.pool.op_lo, i);
        break;
      case StepKind::BN_FOLD: {
        const BnFoldArgs& F = s.bnfold;
        if (F.has_gamma) use(F.gamma.buf, i);
        if (F.has_beta) use(F.beta.buf, i);
        use(F.mean.buf, i); use(F.var.buf, i);
        if (F.has_bias) use(F.bias.buf, i);
        use(F.out_scale, i); use(F.out_shift, i);
        break;
      }
      case StepKind::MEMSET: use(s.memset_buf, i); break;
      case StepKind::ATTENTION: {
        const AttnArgs& A = s.attn;
        use(A.q_hi, i); use(A.q_lo, i); use(A.k_hi, i); use(A.k_lo, i); use(A.v_hi, i); use(A.v_lo, i);
        if (A.write_c) use(A.c.buf, i);
        use(A.op_hi, i); use(A.op_lo, i);
        break;
      }
      case StepKind::SMALL: {
        const SmallArgs& Sm = s.small;
        use(Sm.a.buf, i); use(Sm.l1.w_buf, i); use(Sm.l2.w_buf, i); use(Sm.h_buf, i); use(Sm.counter_buf, i);
        use(Sm.out.buf, i);
        if (Sm.l1.has_bias) use(Sm.l1.bias.buf, i);
        if (Sm.l2.has_bias) use(Sm.l2.bias.buf, i);
        break;
      }
    }
  }
  int nsteps = (int)P_->steps.size();
  for (const View& v : P_->output_views) {
    Buffer& b = P_->buffers[v.buf];
    b.pinned_live = true;
    if (b.first_use < 0) b.first_use = 0;
    b.last_use = nsteps;
  }
  P_->buffers[P_->scalar_buf].pinned_live = true;
  P_->buffers[P_->scalar_buf].first_use = 0;
  P_->buffers[P_->scalar_buf].last_use = nsteps;
  // arena: greedy first-fit by size over liveness intervals, 256-byte aligned
  struct Iv { int b; int s, e; size_t sz; };
  std::vector<Iv> ivs;
  for (int i = 0; i < (int)P_->buffers.size(); ++i) {
    Buffer& b = P_->buffers[i];
    if (b.kind != BufKind::ARENA && b.kind != BufKind::CONST) continue;
    if (b.kind == BufKind::CONST) { b.first_use = 0; b.last_use = nsteps; }
    if (b.first_use < 0) continue;  // unused
    ivs.push_back({i, b.first_use, b.last_use, (size_t)round_up((int64_t)b.bytes, 256)});
  }
  std::sort(ivs.begin(), ivs.end(), [](const Iv& a, const Iv& b) { return a.sz > b.sz; });
  std::vector<std::pair<size_t, Iv>> placed;
  size_t arena = 0;
  for (const Iv& iv : ivs) {
    // collect conflicting placed ranges
    std::vector<std::pair<size_t, size_t>> busy;
    for (auto& [off, p] : placed)
      if (!(p.e < iv.s || iv.e < p.s)) busy.push_back({off, off + p.sz});
    std::sort(busy.begin(), busy.end());
    size_t off = 0;
    for (auto& [b0, b1] : busy) {
      if (off + iv.sz <= b0) break;
      off = std::max(off, b1);
    }
    P_->buffers[iv.b].arena_offset = (int64_t)off;
    placed.push_back({off, iv});
    arena = std::max(arena, off + iv.sz);
  }
  P_->arena_bytes = arena;
  // description
  std::ostringstream d;
  d << "plan: " << P_->steps.size() << " steps, arena " << arena << " bytes, " << P_->scalars.size()
    << " splat constants\n";
  for (size_t i = 0; i < P_->steps.size(); ++i) d << "  [" << i << "] " << P_->steps[i].label << "\n";
  P_->description = d.str();
}

std::unique_ptr<Plan> Compiler::run() {
  P_ = std::make_unique<Plan>();
  P_->precision = in_.precision;
  P_->outputs = in_.outputs;
  order_ = topo_order(g_, in_.outputs);
  for (size_t i = 0; i < order_.size(); ++i) pos_[order_[i]] = (int)i;
  for (uint64_t id : order_)
    for (uint64_t in : N(id).inputs) users_[in].push_back(id);
  for (uint64_t o : in_.outputs) is_out_.insert(o);
  P_->scalar_buf = new_buffer(4 * 64);
  classify();
  absorb_epilogues();
  detect_attention();
  detect_small();
  build_regions();
  attach_row_ops();
  lower();
  finish();
  return std::move(P_);
}

}  // namespace

std::unique_ptr<Plan> compile_plan(const CompileInput& in, SourceMap* sources) {
  Compiler c(in, sources);
  return c.run();
}

}  // namespace pfb
