// Compiled execution plan for one graph structure: buffers, strided views
// over them, and the ordered list of device steps (kernel launches).
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "graph.hpp"

namespace pfb {

// A buffer is a byte range the plan reads or writes.
enum class BufKind : uint8_t {
  ARENA,     // intermediate or output: offset into the plan's arena
  CONST,     // constant payload uploaded from the host (resident or per call)
  BINDING,   // device pointer supplied by the caller (execute_device)
  PREPARED,  // tensor-core operand derived from a resident constant: kept by the
             // executor across calls (keyed by prep_key), filled once
};

struct Buffer {
  BufKind kind = BufKind::ARENA;
  size_t bytes = 0;
  int64_t arena_offset = -1;   // ARENA
  uint64_t node = 0;           // CONST / BINDING / PREPARED: source node id
  uint64_t prep_key = 0;       // PREPARED: constant payload key x operand layout
  int first_use = -1, last_use = -1;  // step indices (liveness)
  bool pinned_live = false;    // keep to the end (graph outputs)
};

// Strided view of a buffer: element (i0..ir) is at
// base + (offset + sum_d i_d*strides[d]) * elem_size.  A buffer index of -1
// with is_splat means every element equals scalar table entry `splat_slot`.
struct View {
  int buf = -1;
  int64_t offset = 0;
  std::vector<int64_t> shape;
  std::vector<int64_t> strides;
  DType dtype = DType::F32;
  bool is_splat = false;
  int splat_slot = -1;
  float splat_value = 0.f;  // value at compile time (the table is refreshed per call)

  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
  bool is_contiguous() const;
  static std::vector<int64_t> dense_strides(const std::vector<int64_t>& shape);
};

enum class StepKind : uint8_t {
  JIT,        // NVRTC-generated kernel (fused elementwise / row / column / full reduction)
  SPLIT,      // pfk_split_tf32 / pfk_convert_bf16 operand preparation
  IM2COL,     // pfk_im2col
  CONV_INPUT, // channels-last hi/lo copy of a Conv2d input (implicit GEMM)
  GEMM,       // pfk_gemm (tcgen05)
  POOL,       // pfk_pool2d
  BN_FOLD,    // fold BatchNorm(eval) into per-channel scale/shift
  MEMSET,     // zero a buffer range
  ATTENTION,  // fused softmax(alpha * Q K^T) V (tcgen05)
  SMALL,      // Linear layers of a small batch on the CUDA cores (one or two layers, optional softmax)
};

// Pointer-argument buffer index that resolves to the executor's device error
// flag (bounded waits record PFC_ERR_TIMEOUT there).
constexpr int kErrorFlagBuffer = -2;

struct JitLaunch {
  std::string module_key;  // hash of the generated source
  std::string kernel;      // kernel symbol
  int grid = 1, block = 256;
  size_t smem = 0;
  std::vector<std::pair<int, int64_t>> ptrs;  // (buffer, byte offset) for each pointer argument
};

struct SplitArgs {
  View src;             // [batch..., rows, cols] logical
  int out_hi = -1, out_lo = -1;  // buffers; lo == -1 for bf16
  int64_t batch = 1, rows = 0, cols = 0, kpad = 0;
  // flattened batch strides (requires the batch dims of src to collapse)
  int64_t sb = 0, sr = 0, sk = 0;
  int precision = 0;
  // conv_cp > 0: src is a Conv2d weight [O,C,KH,KW] laid out for the implicit
  // GEMM, k = (kh*KW + kw)*conv_cp + c
  int64_t conv_cp = 0;
  int64_t conv_kwp = 0;  // taps per filter row in that layout (0 = KW)
};

struct ConvInputArgs {
  View x;  // [N,C,H,W]
  int out_hi = -1, out_lo = -1;  // [N][H][W][cp], or zero-padded [N][hp][wp][cp] when hp > 0
  int64_t cp = 0;
  int64_t hp = 0, wp = 0, ph = 0, pw = 0;
  int precision = 0;
  bool deint = false;  // padded rows stored even columns first, then odd (ConvInputLaunch::deint)
};

struct Im2colArgs {
  View x;  // [N,C,H,W]
  int out_hi = -1, out_lo = -1;
  int64_t kh = 1, kw = 1, sh = 1, sw = 1, ph = 0, pw = 0, dh = 1, dw = 1, oh = 0, ow = 0, kpad = 0;
  int precision = 0;
};

struct GemmArgs {
  int a_hi = -1, a_lo = -1, b_hi = -1, b_lo = -1;
  int64_t a_sb = 0, b_sb = 0, batch = 1, M = 0, N = 0, K = 0, kpad = 0;
  View c;  // output view; strides used for (batch, m, n)
  int64_t c_sb = 0, c_sm = 0, c_sn = 0;
  int precision = 0;
  float alpha = 1.f;
  int alpha_slot = -1;            // splat scale from the scalar table (overrides alpha)
  View bias;  bool has_bias = false;   // [N] view
  int scale_buf = -1, shift_buf = -1;  // folded BatchNorm: per-n scale and shift (replace alpha/bias)
  int act = 0;
  View residual; bool has_residual = false;
  int64_t r_sb = 0, r_sm = 0, r_sn = 0;
  // Operand outputs written by the epilogue for a following GEMM (replacing
  // that GEMM's operand preparation): element (b,m,n) at [(b*M+m)*op_sm + n].
  int op_hi = -1, op_lo = -1;
  int64_t op_sm = 0;
  // op_heads > 0: head-split operand instead, element (m, n) of a batch-1
  // GEMM at [((m / op_rows)*op_heads + n / op_sm)*op_rows + m % op_rows][n % op_sm]
  // (row pitch op_sm): the [B, H, L, D] per-head layout attention reads
  int64_t op_heads = 0, op_rows = 0;
  bool write_c = true;  // false when only the operand outputs are read
  // implicit-GEMM Conv2d: A gathered from the channels-last input x_hi/x_lo
  bool conv = false;
  int x_hi = -1, x_lo = -1;
  int64_t H = 0, W = 0, Cp = 0, KH = 1, KW = 1, sh = 1, sw = 1, ph = 0, pw = 0, dh = 1, dw = 1, OH = 0, OW = 0;
  int64_t Nimg = 1, Hp = 0, Wp = 0, KWp = 0;
  // A 3x3 / stride 2 max pool (padding pool_pad, 0 or 1) of the (ReLU)
  // output, in the epilogue: pooled pool_y (channels-last; written when
  // write_pool_y) and its operand copy (op_hi / op_lo at pool_y's offsets)
  // replace c
  bool pool = false;
  int pool_pad = 0;
  View pool_y;
  bool write_pool_y = true;
  // AdaptiveAvgPool2d(1) of the output in the epilogue: per-tile column sums
  // into gap_buf (conv_gap_slots rows per image), finished by a POOL step of
  // mode 3; replaces c
  int gap_buf = -1;
  // the input copy x_hi / x_lo is de-interleaved (ConvInputArgs::deint): the
  // pooled stem reads it as row runs
  bool deint = false;
};

struct PoolArgs {
  View x;
  View y;
  int mode = 0;
  int64_t kh = 1, kw = 1, sh = 1, sw = 1, ph = 0, pw = 0;
  // channels-last operand copy for a following implicit-GEMM Conv2d
  int op_hi = -1, op_lo = -1;
  bool write_y = true;
  // mode 3 (global average from a convolution's partial sums, x = [n][slots][c]):
  // pixels per image
  int64_t count = 0;
};

struct BnFoldArgs {
  // scale[c] = gamma[c] / sqrt(var[c] + eps); shift[c] = (bias[c] - mean[c]) * scale[c] + beta[c]
  View gamma, beta, mean, var, bias;
  bool has_gamma = false, has_beta = false, has_bias = false;
  float eps = 1e-5f;
  int64_t channels = 0;
  int out_scale = -1, out_shift = -1;
};

// Fused attention over batch slices: Q [batch][M][kq], K [batch][L][kq] and
// V [batch][L][kv] are prepared tf32 hi/lo operands; O is written to the
// view c ([batch..., M, d], rank 3 or 4: slice s = (b, h) of a 4-D view is at
// b*strides[0] + h*strides[1]).  op_hi/op_lo >= 0: O is also written as a
// GEMM operand (hi/lo) at the same element offsets as c (then write_c says
// whether the fp32 value is still needed).
struct AttnArgs {
  int q_hi = -1, q_lo = -1, k_hi = -1, k_lo = -1, v_hi = -1, v_lo = -1;
  int64_t batch = 1, M = 0, L = 0, d = 0, kq = 0, kv = 0;
  float alpha = 1.f;
  int alpha_slot = -1;
  View c;
  int op_hi = -1, op_lo = -1;
  bool write_c = true;
};

// One or two Linear layers of a small batch: a [M, K1] rows (pitch lda) times
// the transposed weights w1 [N1][K1] (pitch ldw1), epilogue alpha/bias/act;
// with two layers, the layer-1 rows go to `h` and the last CTA runs layer 2
// and an optional softmax (1) / log-softmax (2) into `out`.
struct SmallLayerArgs {
  int w_buf = -1;
  int64_t w_off = 0, ldw = 0, N = 0, K = 0;
  View bias;
  bool has_bias = false;
  int64_t bstride = 0;
  float alpha = 1.f;
  int alpha_slot = -1;
  int act = 0;
};
struct SmallArgs {
  View a;
  int64_t lda = 0, M = 0;
  int layers = 1;
  SmallLayerArgs l1, l2;
  int h_buf = -1, counter_buf = -1;
  View out;
  int64_t ldo = 0;
  int softmax = 0;
  bool cluster = false;  // two layers on clusters of 8 CTAs (no h or counter buffer)
};

struct Step {
  StepKind kind = StepKind::JIT;
  bool once = false;           // fills PREPARED buffers: runs only while they are unfilled
  std::string label;           // for describe/profile
  JitLaunch jit;
  SplitArgs split;
  Im2colArgs im2col;
  ConvInputArgs convin;
  GemmArgs gemm;
  PoolArgs pool;
  BnFoldArgs bnfold;
  AttnArgs attn;
  SmallArgs small;
  int memset_buf = -1;
};

struct ScalarSlot {
  uint64_t node;   // splat constant node
  float value;     // value seen when the plan was built
};

struct Plan {
  uint64_t key = 0;
  std::vector<Buffer> buffers;
  std::vector<Step> steps;
  std::vector<ScalarSlot> scalars;   // splat constants; table lives in the arena
  int scalar_buf = -1;
  int error_buf = -1;                // device int for bounded-wait errors
  size_t arena_bytes = 0;
  std::vector<uint64_t> outputs;
  std::vector<View> output_views;    // dense views of requested outputs
  std::vector<uint64_t> const_nodes; // constants with device payload (buffer kind CONST)
  std::vector<uint64_t> splat_nodes; // constants replaced by scalar slots
  std::string description;
  int precision = 0;
};

}  // namespace pfb
