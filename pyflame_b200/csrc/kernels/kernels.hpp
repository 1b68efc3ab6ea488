// Host-side launchers of the precompiled device kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace pfb {

struct GemmLaunch {
  int precision = 0;
  const void* a_hi = nullptr;
  const void* a_lo = nullptr;
  const void* b_hi = nullptr;
  const void* b_lo = nullptr;
  int64_t a_sb = 0, b_sb = 0;  // nonzero: operand has `batch` slices
  int64_t batch = 1, M = 0, N = 0, K = 0, kpad = 0;
  float* c = nullptr;  // may be null when only the operand outputs are wanted
  int64_t c_sb = 0, c_sm = 0, c_sn = 1;
  // Operand outputs: the epilogue also writes its values as the tensor-core
  // operand of a following GEMM (hi/lo split, or bf16 in out_hi): element
  // (b, m, n) at [(b*M + m)*o_sm + n].  Requires N % 4 == 0, o_sm % 4 == 0.
  void* out_hi = nullptr;
  float* out_lo = nullptr;
  int64_t o_sm = 0;
  // o_heads > 0 (batch 1): head-split operand, element (m, n) at
  // [((m / o_rows)*o_heads + n / o_sm)*o_rows + m % o_rows][n % o_sm], row
  // pitch o_sm; needs o_sm % 16 == 0, o_heads*o_sm == N, o_rows % 32 == 0
  int64_t o_heads = 0, o_rows = 0;
  float alpha = 1.f;
  const float* alpha_ptr = nullptr;
  const float* bias = nullptr;
  const float* bias_scalar = nullptr;  // device scalar added to every element (bias of equal values)
  const float* scale = nullptr;  // folded BatchNorm: v = acc*scale[n] + shift[n]
  const float* shift = nullptr;
  int act = 0;
  const float* residual = nullptr;
  int64_t r_sb = 0, r_sm = 0, r_sn = 0;
  int* err = nullptr;
  // Implicit-GEMM Conv2d: when conv is set, A is not a prepared operand; its
  // rows m = (n*OH + oh)*OW + ow and columns k = (kh*KW + kw)*Cp + c are
  // gathered from x_hi/x_lo, a channels-last copy [N][H][W][Cp] of the input
  // (launch_conv_input), with zeros outside the padded image.  K = KH*KW*Cp.
  bool conv = false;
  const void* x_hi = nullptr;
  const void* x_lo = nullptr;
  int64_t H = 0, W = 0, Cp = 0, KH = 1, KW = 1, sh = 1, sw = 1, ph = 0, pw = 0, dh = 1, dw = 1, OH = 0, OW = 0;
  int64_t batch_images = 1;  // N of the convolution (M = N*OH*OW)
  // x is a zero-padded copy [N][Hp][Wp][Cp] when Hp > 0 (padding already
  // applied: padded coordinates are oh*sh + kh*dh, ow*sw + kw*dw)
  int64_t Hp = 0, Wp = 0;
  int64_t KWp = 0;  // taps per filter row in the weight layout (>= KW; 0 = KW)
  bool allow_tma_conv = true;  // TMA-fed A when the geometry allows it
  // pool: a 3x3 / stride 2 max pool (padding pool_pad, 0 or 1) of the ReLU
  // output (N = 64, act 1, the windowed TMA feed) replaces c: pooled
  // [N][PH][PW][64] at pool_y + n*pool_sn + ph*pool_sh + pw*pool_sw + channel
  // (or null), and the operand at the same offsets of out_hi / out_lo (or null)
  bool pool = false;
  int pool_pad = 0;
  float* pool_y = nullptr;
  // deint: x is a de-interleaved padded copy (ConvInputLaunch::deint); a
  // pooled stride-2 stem with 8-tap filter rows of 16-byte pixels then reads
  // it as row runs (conv_rows_pool_kernel)
  bool deint = false;
  int64_t pool_sn = 0, pool_sh = 0, pool_sw = 0, PH = 0, PW = 0;
  // Workspace for a split last wave (plain GEMMs): tail_ws_bytes of fp32
  // slots (one 128 x BN tile per CTA) and tail_cnt_len counters that start
  // at 0 and are left at 0.  Null: whole tiles only.  Launches sharing them
  // must not run at the same time.
  float* tail_ws = nullptr;
  int64_t tail_ws_bytes = 0;
  unsigned* tail_cnt = nullptr;
  int64_t tail_cnt_len = 0;
  // gap: AdaptiveAvgPool2d(1) of the output of a TMA-fed convolution (rows of
  // 32+ output pixels) replaces c: per image conv_gap_slots(OH, OW) rows of
  // N column sums, [N][slots][N] (a PoolLaunch of mode 3 adds them up)
  float* gap = nullptr;
};
void launch_gemm(const GemmLaunch& L, cudaStream_t stream);

// Output tile width (pixels) of a TMA-fed convolution whose output rows are
// ow >= 32 pixels wide; tiles are conv_tile_w x 128 / conv_tile_w pixels.
inline int conv_tile_w(int64_t ow) { return ow > 32 ? 64 : 32; }
// Partial-sum rows per image of a convolution with a fused global average
// pool: four (one per TMEM lane quarter) per output tile.
inline int64_t conv_gap_slots(int64_t oh, int64_t ow) {
  const int64_t tw = conv_tile_w(ow), th = 128 / tw;
  return 4 * ((oh + th - 1) / th) * ((ow + tw - 1) / tw);
}

// Fused attention O = softmax(alpha * Q K^T) V over batch slices (3xTF32
// operands as prepared for the GEMM): Q [batch][M][kq], K [batch][L][kq] and
// V [batch][L][kv] hi/lo, rows of head-dim columns (padded to kq, kv).
// Needs d <= 64 and kq, kv in {32, 64}.  Replaces the QK^T GEMM, softmax
// and PV GEMM that rocm_executor.cpp:278-335 and rocm_kernels.hip run as
// separate passes for PyFlame's MultiheadAttention graphs.
struct AttnLaunch {
  int precision = 0;  // tf32x3 (hi/lo operands) or bf16 (q_hi, k_hi, v_hi, o_hi only; kq = kv = 64)
  int64_t batch = 0, M = 0, L = 0, d = 0, kq = 0, kv = 0;
  const void* q_hi = nullptr;
  const float* q_lo = nullptr;
  const void* k_hi = nullptr;
  const float* k_lo = nullptr;
  const void* v_hi = nullptr;
  const float* v_lo = nullptr;
  float alpha = 1.f;
  const float* alpha_ptr = nullptr;  // device scalar (a splat slot), overrides alpha
  // O of slice s = b*heads + h at c + b*c_sb + h*c_sh + m*c_sm + n*c_sn
  float* c = nullptr;  // may be null when only the operand is written
  int64_t heads = 1, c_sb = 0, c_sh = 0, c_sm = 0, c_sn = 1;
  // O also as the next GEMM's operand at the same element offsets (or null):
  // tf32 hi/lo, or bf16 in o_hi
  float* o_hi = nullptr;
  float* o_lo = nullptr;
  int* err = nullptr;
};
void launch_attention(const AttnLaunch& L, cudaStream_t stream);

// One CTA whose bounded mbarrier wait can never complete: after limit_us it
// records PFC_ERR_TIMEOUT in *err and returns (a test of the failure path).
void launch_wait_check(int* err, int64_t limit_us, cudaStream_t stream);

// Channels-last copy of a Conv2d input for the implicit GEMM: x is a strided
// [N,C,H,W] view; output [N][H][W][Cp] (Cp >= C, zero channels above C) as
// tf32x3 hi/lo fp32 pairs, or bf16 in hi when precision is bf16.
struct ConvInputLaunch {
  const float* x = nullptr;
  int64_t n = 0, c = 0, h = 0, w = 0, sn = 0, sc = 0, sh = 0, sw = 0;
  int64_t cp = 0;
  // zero-padded output [N][hp][wp][cp] with the image at (ph, pw); hp = 0: unpadded
  int64_t hp = 0, wp = 0, ph = 0, pw = 0;
  // deint (padded, wp even): each padded row stores its even columns first,
  // then its odd columns (column w at (w & 1) * wp/2 + w/2)
  bool deint = false;
  int precision = 0;
  void* hi = nullptr;
  float* lo = nullptr;
};
void launch_conv_input(const ConvInputLaunch& L, cudaStream_t stream);

// Conv2d weight [O,C,KH,KW] (strided view) as the implicit GEMM's B operand:
// [O][kpad] with k = (kh*KW + kw)*Cp + c, zero for c >= C and k >= KH*KW*Cp.
struct ConvWeightLaunch {
  const float* w = nullptr;
  int64_t o = 0, c = 0, kh = 0, kw = 0, so = 0, sc = 0, skh = 0, skw = 0;
  int64_t cp = 0, kpad = 0;
  int64_t kwp = 0;  // taps per filter row in the layout (>= kw; 0 = kw): k = (kh*kwp + kw)*cp + c
  int precision = 0;
  void* hi = nullptr;
  float* lo = nullptr;
};
void launch_conv_weight(const ConvWeightLaunch& L, cudaStream_t stream);

// Operand preparation from a strided view of rank <= 6: the last dim is K,
// all leading dims flatten (row-major) into rows.  Output [rows][kpad].
struct PrepLaunch {
  const float* src = nullptr;
  int rank = 2;
  int64_t shape[6] = {0};
  int64_t stride[6] = {0};
  int precision = 0;
  void* hi = nullptr;  // fp32 hi (tf32x3) or bf16 values
  float* lo = nullptr;
  int64_t kpad = 0;
};
void launch_prepare(const PrepLaunch& L, cudaStream_t stream);

struct Im2colLaunch {
  const float* x = nullptr;
  int64_t n = 0, c = 0, h = 0, w = 0, sn = 0, sc = 0, sh = 0, sw = 0;
  int64_t kh = 1, kw = 1, stride_h = 1, stride_w = 1, pad_h = 0, pad_w = 0, dil_h = 1, dil_w = 1;
  int64_t oh = 0, ow = 0, kpad = 0;
  int precision = 0;
  void* hi = nullptr;
  float* lo = nullptr;
};
void launch_im2col(const Im2colLaunch& L, cudaStream_t stream);

struct PoolLaunch {
  const float* x = nullptr;
  float* y = nullptr;
  int mode = 0;
  int64_t n = 0, c = 0, h = 0, w = 0, sn = 0, sc = 0, sh = 0, sw = 0;
  int64_t kh = 1, kw = 1, stride_h = 1, stride_w = 1, pad_h = 0, pad_w = 0;
  int64_t oh = 0, ow = 0, osn = 0, osc = 0, osh = 0, osw = 0;
  // Operand output for an implicit-GEMM Conv2d that reads this pool's
  // result: the channels-last [N][OH][OW][C] copy as tf32x3 hi/lo (or bf16 in
  // out_hi), at the offsets of the channels-last output y (osc == 1).  y
  // itself may then be null.
  void* out_hi = nullptr;
  float* out_lo = nullptr;
  int precision = 0;
  // mode 3: the global average pool finished from a convolution's partial
  // sums (GemmLaunch::gap): x [n][h slots][c] (strides sn, sh, sc), out =
  // the sum of an image's slots in slot order / count
  int64_t count = 0;
};
void launch_pool(const PoolLaunch& L, cudaStream_t stream);

// Linear layers of a small batch (M <= kSmallMaxRows rows) on the CUDA cores:
// layer 1 out1[m][n] = act1(alpha1 * sum_k a[m][k] * w1[n][k] + bias1[n]), with
// w1 rows as Linear stores its weight ([out, in], pitch ldw1).  layers == 2
// adds out[m][n] = act2(alpha2 * sum_j h[m][j] * w2[n][j] + bias2[n]) over
// the layer-1 rows h, and softmax (1) or log-softmax (2) over each output
// row, all in one launch; `counter` (8 bytes) must be zero at the launch.
constexpr int64_t kSmallMaxRows = 256;
struct SmallMlpLaunch {
  int layers = 1;
  const float* a = nullptr;
  int64_t lda = 0, M = 0;
  const float* w1 = nullptr;
  int64_t ldw1 = 0, N1 = 0, K1 = 0;
  const float* bias1 = nullptr;  // bias1[n * bstride1] (stride 0: one value)
  int64_t bstride1 = 0;
  float alpha1 = 1.f;
  const float* alpha1_ptr = nullptr;
  int act1 = 0;
  const float* w2 = nullptr;  // [N2][ldw2], K2 = N1
  int64_t ldw2 = 0, N2 = 0;
  const float* bias2 = nullptr;
  int64_t bstride2 = 0;
  float alpha2 = 1.f;
  const float* alpha2_ptr = nullptr;
  int act2 = 0;
  float* h = nullptr;  // layer-1 rows [M][ldh] (layers == 2)
  int64_t ldh = 0;
  float* out = nullptr;  // final rows [M][ldo]
  int64_t ldo = 0;
  int softmax = 0;
  unsigned long long* counter = nullptr;
  // Two layers on clusters of 8 CTAs (small_mlp_cluster_fits): h, ldh and
  // counter are unused; err receives a timed-out wait.
  bool cluster = false;
  int* err = nullptr;
};
void launch_small_mlp(const SmallMlpLaunch& L, cudaStream_t stream);
// Whether a two-layer chain of these sizes runs on clusters of 8 CTAs, each
// cluster a block of rows and each CTA an eighth of the hidden units: x rows
// and the CTA's weight rows staged whole in shared memory (K % 4 == 0 and
// 16-byte aligned rows, checked again at launch), at most 256 outputs per row.
bool small_mlp_cluster_fits(int64_t M, int64_t N1, int64_t K1, int64_t N2);

struct BnFoldLaunch {
  const float* gamma = nullptr; int64_t gs = 0;  // strides in elements (0 = splat)
  const float* beta = nullptr;  int64_t bs = 0;
  const float* mean = nullptr;  int64_t ms = 0;
  const float* var = nullptr;   int64_t vs = 0;
  const float* bias = nullptr;  int64_t cs = 0;
  float gamma_c = 1.f, beta_c = 0.f, mean_c = 0.f, var_c = 1.f, bias_c = 0.f;  // used when the pointer is null
  float eps = 1e-5f;
  int64_t channels = 0;
  float* scale = nullptr;
  float* shift = nullptr;
};
void launch_bn_fold(const BnFoldLaunch& L, cudaStream_t stream);

}  // namespace pfb
