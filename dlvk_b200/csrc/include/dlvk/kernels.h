// Host-callable launchers of every dlvk_b200 CUDA kernel.  All pointers are
// device pointers; every launcher enqueues on the given stream and never
// synchronises.  Scratch buffers, where needed, are supplied by the caller.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "dlvk/common.h"

namespace dlvk {

// ---- elementwise -----------------------------------------------------------
enum UnaryOp : int {
  UN_RELU = 0, UN_SIGMOID = 1, UN_TANH = 2, UN_SCALE = 3, UN_CLAMP = 4, UN_SQRT = 5, UN_COPY = 6,
  UN_SQUARE = 7, UN_ADD_SCALAR = 8, UN_ABS = 9, UN_EXP = 10, UN_LOG = 11, UN_GELU = 12,
};
enum BinaryOp : int {
  BIN_ADD = 0, BIN_SUB = 1, BIN_MUL = 2, BIN_DIV = 3, BIN_MAX = 4, BIN_MIN = 5,
  BIN_RELU_BWD = 6, BIN_SIGMOID_BWD = 7, BIN_TANH_BWD = 8, BIN_GELU_BWD = 9,
};
void unary(DType dt_in, DType dt_out, const void* x, void* y, int64_t n, int op, float a, float b, cudaStream_t s);
void binary(DType dt, const void* x, const void* y, void* z, int64_t n, int op, cudaStream_t s);
void bias_act(DType dt, DType dt_bias, const void* x, const void* bias, void* out, int64_t rows, int64_t cols, int act,
              cudaStream_t s);

// ---- reductions / layout ---------------------------------------------------
enum ReduceOp : int { RED_SUM = 0, RED_MAX = 1, RED_MIN = 2, RED_SUMSQ = 3, RED_ABSMAX = 4 };
int reduce_scratch_floats();
void reduce(DType dt, const void* x, int64_t n, int op, float scale, float* out, float* scratch, cudaStream_t s);
// out[c] = scale * sum_k partial[k * cols + c] (+ out[c]); fp32, fixed order.
void colsum_partials(const float* partial, int64_t chunks, int64_t cols, float scale, float* out, bool accumulate,
                     cudaStream_t s);
// scratch: colsum_scratch_floats(rows, cols) floats (may be null: single pass)
int64_t colsum_scratch_floats(int64_t rows, int64_t cols);
void colsum(DType dt, DType dt_out, const void* x, int64_t rows, int64_t cols, float scale, void* out, bool accumulate,
            float* scratch, cudaStream_t s);
void rowsum(DType dt, const void* x, int64_t rows, int64_t cols, float scale, float* out, cudaStream_t s);
void transpose2d(DType dt, const void* x, void* y, int64_t batch, int64_t rows, int64_t cols, cudaStream_t s);
void permute4(DType dt, const void* x, void* y, const int* in_dims, const int* perm, cudaStream_t s);

// ---- softmax / losses --------------------------------------------------------
enum LossKind : int { LOSS_MSE = 0, LOSS_BCE = 1 };
void softmax(DType dt, const void* x, void* y, int64_t rows, int64_t cols, bool log_out, cudaStream_t s);
void softmax_bwd(DType dt, const void* y, const void* dy, void* dx, int64_t rows, int64_t cols, cudaStream_t s);
void softmax_cross_entropy(DType dt, const void* logits, const int* labels, const float* probs, float* loss_rows,
                           void* dlogits, int64_t rows, int64_t cols, float grad_scale, cudaStream_t s);
int pointwise_loss_blocks(int64_t n);
void pointwise_loss(DType dt, int kind, const void* p, const float* t, int64_t n, float loss_scale, float grad_scale,
                    void* grad, float* out, float* scratch, cudaStream_t s);
void sum_rows_to_scalar(const float* rows_vals, int64_t n, float scale, float* out, cudaStream_t s);

// ---- GEMM -------------------------------------------------------------------
enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_GELU = 2 };
// C[b](m, n) = act(alpha * sum_k A[b](m, k) * B[b](k, n) + beta * C[b](m, n) + bias[n] + R[b](m, n))
// A(m,k) = A[m*sam + k*sak]; B(k,n) = B[k*sbk + n*sbn]; C(m,n) = C[m*ldc + n].
// Batches are two-level: b = (bo, bi), bo < batch, bi < batch2, with
// independent strides per level (e.g. (batch, head) of an attention tensor).
struct GemmArgs {
  const void* A = nullptr;
  const void* B = nullptr;
  void* C = nullptr;
  int64_t M = 0, N = 0, K = 0;
  int64_t sam = 0, sak = 0, sbk = 0, sbn = 0, ldc = 0;
  int64_t batch = 1, batch_stride_a = 0, batch_stride_b = 0, batch_stride_c = 0;
  int64_t batch2 = 1, batch2_stride_a = 0, batch2_stride_b = 0, batch2_stride_c = 0;
  float alpha = 1.f, beta = 0.f;
  const void* bias = nullptr;
  int bias_dtype = 0;
  int act = ACT_NONE;
  const void* residual = nullptr;  // same dtype as C, added before act
  int64_t ldr = 0, batch_stride_r = 0, batch2_stride_r = 0;
  // Optional mask source (same dtype and shape as C): the output is zeroed
  // where mask <= 0.  Fuses the backward of a preceding ReLU into dX = dY W^T.
  const void* relu_mask = nullptr;
  int64_t ldm = 0, batch_stride_m = 0, batch2_stride_m = 0;
  // Optional column sums of the output (before its rounding to C's dtype):
  // per 32-row block, colsum[(m / 32) * N + n].  Needs gemm_tc_colsum_ok();
  // colsum_partials() then adds the ceil(M / 32) rows.  Fuses a bias
  // gradient db = sum_rows(dY) into the GEMM that produces dY.
  float* colsum = nullptr;
  // Optional fp32 bias per output row (added with the column bias, before
  // the activation): the per-channel bias of a convolution whose output
  // rows are channels (1x1 convolution in NCHW as a batched GEMM).  Tensor-
  // core path only.
  const float* row_bias = nullptr;
  // Optional ReLU bitmask, one bit per output element: bit n % 32 of word
  // [m * ldbits + n / 32].  relu_bits_out is written by a forward GEMM (bit
  // set where the output, after the activation, is > 0); relu_bits zeroes
  // the output where the bit is clear -- the backward of that ReLU, reading
  // 1/16 of the bytes of a bf16 mask.  2-D GEMMs only.
  uint32_t* relu_bits_out = nullptr;
  const uint32_t* relu_bits = nullptr;
  int64_t ldbits = 0;
};
// SIMT GEMM.  With a workspace of gemm_simt_workspace_floats(a) floats, a
// small 2-D GEMM with a plain epilogue splits K across blocks (fp32 partials,
// then a finish kernel; deterministic).
int64_t gemm_simt_workspace_floats(const GemmArgs& a);
void gemm_simt(DType in_dt, DType out_dt, const GemmArgs& a, cudaStream_t s, float* ws = nullptr,
               int64_t ws_floats = 0);
bool gemm_tc_supported(const GemmArgs& a);
// bf16 inputs, bf16 or f32 output, tcgen05 tensor cores.  `err` is the
// device error word; `max_ctas` caps the persistent grid (0 = #SMs).
// Split-K: when the tile grid underfills the GPU, partial sums go to an fp32
// `workspace` of gemm_tc_workspace_floats() floats (0 = none needed) and a
// reduce kernel applies the epilogue.  With a null/small workspace the GEMM
// runs unsplit.  An fp32 C with a linear epilogue (alpha, beta 0 or 1) needs
// no workspace: the partials are added into C by TMA reduces.
int64_t gemm_tc_workspace_floats(const GemmArgs& a, int max_ctas = 0, DType out_dt = DType::BF16,
                                 bool tf32 = false);
// CTA-pair (tcgen05 cta_group::2, 256 x 256 tiles) variant for unsplit bf16
// GEMMs with M >= 256; on by default (DLVK_GEMM_PAIR=0 turns it off).
bool gemm_tc_pair_enabled();
void gemm_tc_set_pair(bool on);
// 256 x 512 CTA-pair tile (two N = 256 MMAs per k-step, one TMEM buffer) for
// long-K GEMMs with few tiles.  Mode 0 never, 1 when the tiling model picks
// it (default; DLVK_GEMM_WIDE sets the initial mode), 2 whenever it applies.
void gemm_tc_set_wide(int mode);
// Forces the tile N (128 / 256 / 512), split-K factor and CTA-pair use of
// later GEMMs (0 / 0 / -1 restore the tiling model); for measurements.
void gemm_tc_set_tiling(int bn, int splits, int pair);
// The tiling the model picks for these operands: tile N (128/256/512), the
// split-K factor, and whether the CTA-pair kernel runs.
void gemm_tc_plan(DType out_dt, const GemmArgs& a, int max_ctas, int* bn, int* splits, int* pair);
bool gemm_tc_colsum_ok(DType out_dt, const GemmArgs& a);
void gemm_tc(DType out_dt, const GemmArgs& a, cudaStream_t s, uint32_t* err, int max_ctas = 0,
             float* workspace = nullptr, int64_t workspace_floats = 0);
// fp32 operands on the tensor cores (tcgen05 kind::tf32: each product uses
// the operands' top 19 bits, fp32 accumulation), single-CTA tiles; A / B
// K-major or M/N-major like gemm_tc, row strides multiples of 4 elements.
bool gemm_tf32_tc_supported(const GemmArgs& a);
void gemm_tf32_tc(DType out_dt, const GemmArgs& a, cudaStream_t s, uint32_t* err, int max_ctas = 0,
                  float* workspace = nullptr, int64_t workspace_floats = 0);
// Splits fp32 x into hi = x rounded to tf32 and lo = x - hi, so that
// A B ~= Ahi Bhi + Ahi Blo + Alo Bhi with every product exact in tf32 up to
// the lo terms' own rounding (relative error ~2^-21): the 3xTF32 scheme.
void tf32_split(const float* x, float* hi, float* lo, int64_t n, cudaStream_t s);

// ---- int8 ----------------------------------------------------------------------
// q[r, :] = round(x[r, :] / s[r]), s[r] = max|x[r, :]| / 127 (symmetric, per row).
void quantize_rows_int8(DType dt, const void* x, int64_t rows, int64_t cols, int64_t ldx, int8_t* q, int64_t ldq,
                        float* scale, cudaStream_t s);
bool gemm_i8_tc_supported(const void* A, const void* Bt, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb);
// C = act(sum_k A[m,k] Bt[n,k] * sa[m] * sb[n] + bias[n]); A [M,K], Bt [N,K] int8.
void gemm_i8_tc(const int8_t* A, const int8_t* Bt, const float* sa, const float* sb, const float* bias, int act,
                void* C, DType out_dt, int64_t ldc, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                cudaStream_t s, uint32_t* err);
void gemm_i8_simt(const int8_t* A, const int8_t* Bt, const float* sa, const float* sb, const float* bias, int act,
                  void* C, DType out_dt, int64_t ldc, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                  cudaStream_t s);

// ---- optimizers --------------------------------------------------------------
enum OptKind : int { OPT_SGD = 0, OPT_ADAM = 1, OPT_RMSPROP = 2 };
// Device-resident optimizer hyper-parameters (one per optimizer instance).
struct OptimHyper {
  float lr;
  float beta1, beta2, eps;
  float weight_decay;
  float momentum;
  float alpha;          // RMSprop smoothing
  float grad_scale;     // multiplies every gradient (e.g. 1/world, 1/loss_scale)
  float bc1, bc2;       // bias corrections, maintained by optim_advance
  int step;
  int bias_correction;  // 1: Adam with 1/(1-beta^t) corrections
  int decoupled_wd;     // 1: AdamW-style decay
  int pad_;
  const float* clip_coef_ptr;  // optional device scalar multiplying the grads
  const int* skip_flag_ptr;    // optional device flag: skip the update when set
};
void optim_advance(OptimHyper* h_dev, cudaStream_t s);
// max_ctas > 0 caps the grid (an update overlapped with other kernels).
void optim_update(int kind, const OptimHyper* h_dev, float* p, const void* g, DType g_dt, float* m, float* v,
                  __nv_bfloat16* p_bf16, int64_t n, float extra_scale, cudaStream_t s, int max_ctas = 0);
int grad_stats_scratch_floats();
void grad_stats(const void* g, DType g_dt, int64_t n, float scale, float max_norm, float* sumsq_out, int* flag,
                float* clip_out, bool accumulate, float* scratch, cudaStream_t s, const float* scale_ptr = nullptr);
// x[i] *= *s (s on the device: a loss scale that a captured graph re-reads).
void scale_by_device_scalar(DType dt, void* x, int64_t n, const float* s, cudaStream_t st);
// Fused L1/L2 regularisation over [n) flat parameters:
//   g += k * (l1 * sign(w) + l2 * w);  *loss_out += ll1 * |w| + 0.5 * ll2 * w^2 (if loss_out),
// with k = *gscale (a loss scale still applied to g) or 1.  The loss
// coefficients differ from the gradient ones for weight decay, which has a
// gradient term and no loss term.
void regularize(const float* w, void* g, DType g_dt, int64_t n, float l1, float l2, float ll1, float ll2,
                float* loss_out, cudaStream_t s, const float* gscale = nullptr);
void scaler_update(float* scale, int* good_steps, const int* found_inf, float growth, float backoff, int interval,
                   float smin, float smax, float* inv_scale, cudaStream_t s);

// ---- convolution / pooling ---------------------------------------------------
struct ConvDesc {
  int N, Cin, H, W, Cout, KH, KW, stride, pad, Ho, Wo;
};
void conv2d_fwd(DType dt, const void* x, const void* w, const float* bias, void* y, const ConvDesc& d, bool relu,
                cudaStream_t s);
// relu_src (optional): the forward input of the preceding ReLU (or its output);
// dx is zeroed where relu_src <= 0, fusing that activation's backward.
void conv2d_dgrad(DType dt, const void* g, const void* w, void* dx, const void* relu_src, const ConvDesc& d,
                  cudaStream_t s);
// Implicit-GEMM tcgen05 convolution (conv_tc.cu), bf16 with channel counts
// that are multiples of 8.  Activations are gathered from NHWC copies; the
// outputs (y, dx) are written NCHW.
bool conv2d_tc_supported(DType dt, const ConvDesc& d);
void conv_tc_set_mode(int mode);  // 0 auto (large convolutions), 1 whenever supported, 2 never
int conv_tc_get_mode();
int64_t conv_pack_cols(int64_t k);  // packed weight row length for K = KH*KW*channels
// [OC][C][KH][KW] -> bf16 [OC][conv_pack_cols(KH*KW*C)] (forward) or
// [C][conv_pack_cols(KH*KW*OC)] (dgrad), taps outer and channels inner.
void conv_pack_weights(DType wdt, const void* w, __nv_bfloat16* out, const ConvDesc& d, bool dgrad, cudaStream_t s);
// forward: src = X (NHWC), out = Y (NCHW); dgrad: src = dY (NHWC), out = dX
// (NCHW), `mask` zeroes dX where the preceding ReLU was inactive.
void conv2d_igemm(const __nv_bfloat16* src_nhwc, const __nv_bfloat16* wpack, const ConvDesc& d, bool dgrad,
                  const float* bias, bool relu, const void* mask, void* out, bool out_f32, cudaStream_t s);
int64_t conv2d_wgrad_tc_ws_floats(const ConvDesc& d);
void conv2d_wgrad_tc(const __nv_bfloat16* x_nhwc, const __nv_bfloat16* dy_nhwc, const ConvDesc& d, float* ws,
                     float* dw, bool accumulate, cudaStream_t s);
int conv2d_wgrad_chunks(const ConvDesc& d);
int64_t conv2d_wgrad_scratch_floats(const ConvDesc& d);
void conv2d_wgrad(DType dt, const void* x, const void* g, float* dw, float* db, bool accumulate, const ConvDesc& d,
                  float* scratch, cudaStream_t s);
void maxpool2d_fwd(DType dt, const void* x, void* y, int32_t* idx, int64_t planes, int H, int W, int k, int stride,
                   cudaStream_t s);
void maxpool2d_bwd(DType dt, const void* g, const int32_t* idx, void* dx, int64_t planes, int H, int W, int k,
                   int stride, cudaStream_t s);
void avgpool2d_fwd(DType dt, const void* x, void* y, int64_t planes, int H, int W, int k, int stride, int pad,
                   cudaStream_t s);
void avgpool2d_bwd(DType dt, const void* g, void* dx, int64_t planes, int H, int W, int k, int stride, int pad,
                   cudaStream_t s);

// ---- normalisation / dropout / embedding -------------------------------------
// Philox dropout stream: key = seed, counter = {element/4, stream, step}.
struct DropoutDesc {
  float p = 0.f;                  // drop probability (0 = disabled)
  uint32_t stream = 0;            // distinct per dropout site
  uint64_t seed = 0;
  uint32_t step = 0;              // used when step_ptr is null
  const int64_t* step_ptr = nullptr;  // device step counter (graph replays)
};
// scratch (both passes): batchnorm_scratch_floats(N, C, S) floats.
int64_t batchnorm_scratch_floats(int N, int C, int S);
void batchnorm_fwd(DType dt, const void* x, const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                   float* run_mean, float* run_var, int N, int C, int S, float momentum, float eps, bool training,
                   bool relu, const DropoutDesc& dd, float* scratch, cudaStream_t s);
void batchnorm_bwd(DType dt, const void* x, const void* dy, const float* mean, const float* rstd, const float* gamma,
                   const float* beta, void* dx, float* dgamma, float* dbeta, bool accumulate, int N, int C, int S,
                   bool relu, const DropoutDesc& dd, float* scratch, cudaStream_t s);
void layernorm_fwd(DType dt, const void* x, const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                   int64_t rows, int D, float eps, cudaStream_t s);
int layernorm_bwd_blocks(int64_t rows);
int64_t layernorm_bwd_scratch_floats(int64_t rows, int D);
// dres (optional, same dtype/shape as dx): a residual-branch gradient added
// to dx, fusing the sum of the two gradients of a pre-norm block input.
// dres_colsum (optional, fp32 [D]): receives (or, with its accumulate flag,
// adds) the column sums of dres -- the bias gradient of the biased GEMM whose
// output gradient dres is.
void layernorm_bwd(DType dt, const void* x, const float* gamma, const float* mean, const float* rstd, const void* dy,
                   void* dx, float* dgamma, float* dbeta, bool accumulate, int64_t rows, int D, float* scratch,
                   cudaStream_t s, const void* dres = nullptr, float* dres_colsum = nullptr,
                   bool dres_colsum_accumulate = false);
void dropout(DType dt, const void* x, void* y, int64_t n, const DropoutDesc& dd, cudaStream_t s);
void embedding_fwd(DType dt, const int32_t* ids, const void* table, void* out, int64_t n, int64_t V, int D,
                   cudaStream_t s);
// dtable must be zeroed (or hold the gradient to accumulate into).
void embedding_bwd(DType dt, const int32_t* ids, const void* dy, float* dtable, int64_t n, int64_t V, int D,
                   cudaStream_t s);

// ---- device error word -------------------------------------------------------
uint32_t* device_error_word();     // per current device, zero-initialised
uint32_t read_device_error(bool clear);
void counter_add(int64_t* c, int64_t delta, cudaStream_t s);

// Per-step training metrics on the device: *loss_sum += *loss * loss_weight and
// *correct += #rows whose logits argmax equals the label (labels: int ids, or
// probs: target rows whose argmax is the class).  Either may be null.
void step_metrics(DType dt, const void* logits, int64_t rows, int cols, const int* labels, const float* probs,
                  const float* loss, float* loss_sum, unsigned long long* correct, float loss_weight, cudaStream_t s);

// ---- fused attention on tcgen05 (attention_tc.cu): head dim 64, S % 128 == 0 --
// qkv: [B, S, 3, H, 64] bf16; out: [B, S, H*64] bf16; lse: [B, H, S] fp32 (log2 units).
bool flash_attention_supported(int64_t B, int64_t S, int64_t H, int64_t D, const void* qkv);
void flash_attention_fwd(const __nv_bfloat16* qkv, __nv_bfloat16* out, float* lse, int B, int S, int H, float scale,
                         cudaStream_t s, uint32_t* err, int max_ctas = 0);
// dqkv: [B, S, 3, H, 64] bf16 (fully written); delta: [B, H, S] and dq_acc:
// [B*S, H*64] fp32 scratch.
void flash_attention_bwd(const __nv_bfloat16* qkv, const __nv_bfloat16* out, const __nv_bfloat16* dout,
                         const float* lse, float* delta, float* dq_acc, __nv_bfloat16* dqkv, int B, int S, int H,
                         float scale, cudaStream_t s, uint32_t* err, int max_ctas = 0);

// ---- recurrent cells (rnn.cu); kind 0 RNN-tanh, 1 LSTM, 2 GRU ---------------
// Every pointer addresses B rows with its own row stride (elements).
struct RnnCellFwd {
  int kind = 0;
  int64_t B = 0;
  int H = 0;
  const void* a = nullptr; int64_t lda = 0;        // pre-activations (GRU: input side) [B, G*H]
  const void* hg = nullptr; int64_t ldhg = 0;      // GRU hidden side h W_hh^T + b_hh [B, 3H]
  const void* h_prev = nullptr; int64_t ldhp = 0;  // GRU h_{t-1}
  const float* c_prev = nullptr; int64_t ldcp = 0; // LSTM c_{t-1} (null = 0)
  void* h_out = nullptr; int64_t ldo = 0;
  void* h_copy = nullptr; int64_t ldcopy = 0;      // optional second copy of h_t
  float* c_out = nullptr; int64_t ldco = 0;        // LSTM c_t
  float* saved = nullptr; int64_t lds = 0;         // LSTM (i,f,g,o) / GRU (r,z,n,hn) [B, 4H]
};
struct RnnCellBwd {
  int kind = 0;
  int64_t B = 0;
  int H = 0;
  const void* dh = nullptr; int64_t lddh = 0;
  const float* dc_next = nullptr; int64_t lddcn = 0;
  const void* h_t = nullptr; int64_t ldht = 0;
  const void* h_prev = nullptr; int64_t ldhp = 0;
  const float* c_t = nullptr; int64_t ldct = 0;
  const float* c_prev = nullptr; int64_t ldcp = 0;
  const float* saved = nullptr; int64_t lds = 0;
  void* dA = nullptr; int64_t ldda = 0;
  void* dAh = nullptr; int64_t lddah = 0;
  float* dc_prev = nullptr; int64_t lddcp = 0;
  const void* dy_prev = nullptr; int64_t lddyp = 0;
  void* resid = nullptr; int64_t ldres = 0;
};
void rnn_cell_fwd(const RnnCellFwd& p, DType dt, cudaStream_t s);
void rnn_cell_bwd(const RnnCellBwd& p, DType dt, cudaStream_t s);

// ---- batched image transforms (augment.cu), fp32 [N, C, H, W] ---------------
// theta: [N, 6] output->input maps (sx = t0*x + t1*y + t2, sy = t3*x + t4*y + t5);
// mode 0 nearest-floor, 1 nearest-round, 2 bilinear.
void image_affine_sample(const float* x, float* y, int N, int C, int H, int W, int OH, int OW, const float* theta,
                         int mode, float fill, cudaStream_t s);
// kind 0 contrast (params [N,2]: factor, -), 1 standardise, 2 min-max (params [N,2]: lo, hi).
void image_per_sample_stats(const float* x, float* y, int64_t N, int64_t len, int kind, const float* params,
                            bool clamp01, cudaStream_t s);
void image_channel_affine(const float* x, float* y, int64_t N, int C, int64_t HW, const float* mean,
                          const float* inv_std, const float* sample_add, bool clamp01, cudaStream_t s);
void image_gaussian_noise(const float* x, float* y, int64_t n, float sigma, uint64_t seed, uint32_t stream,
                          cudaStream_t s);

}  // namespace dlvk
