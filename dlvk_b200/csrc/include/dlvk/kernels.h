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
};
void gemm_simt(DType in_dt, DType out_dt, const GemmArgs& a, cudaStream_t s);
bool gemm_tc_supported(const GemmArgs& a);
// bf16 inputs, bf16 or f32 output, tcgen05 tensor cores.  `err` is the
// device error word; `max_ctas` caps the persistent grid (0 = #SMs).
// Split-K: when the tile grid underfills the GPU, partial sums go to an fp32
// `workspace` of gemm_tc_workspace_floats() floats (0 = no split chosen) and a
// reduce kernel applies the epilogue.  With a null/small workspace the GEMM
// runs unsplit.
int64_t gemm_tc_workspace_floats(const GemmArgs& a, int max_ctas = 0);
void gemm_tc(DType out_dt, const GemmArgs& a, cudaStream_t s, uint32_t* err, int max_ctas = 0,
             float* workspace = nullptr, int64_t workspace_floats = 0);

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
void optim_update(int kind, const OptimHyper* h_dev, float* p, const void* g, DType g_dt, float* m, float* v,
                  __nv_bfloat16* p_bf16, int64_t n, float extra_scale, cudaStream_t s);
int grad_stats_scratch_floats();
void grad_stats(const void* g, DType g_dt, int64_t n, float scale, float max_norm, float* sumsq_out, int* flag,
                float* clip_out, bool accumulate, float* scratch, cudaStream_t s);
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
void batchnorm_fwd(DType dt, const void* x, const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                   float* run_mean, float* run_var, int N, int C, int S, float momentum, float eps, bool training,
                   bool relu, const DropoutDesc& dd, cudaStream_t s);
// scratch: 2*C floats
void batchnorm_bwd(DType dt, const void* x, const void* dy, const float* mean, const float* rstd, const float* gamma,
                   const float* beta, void* dx, float* dgamma, float* dbeta, bool accumulate, int N, int C, int S,
                   bool relu, const DropoutDesc& dd, float* scratch, cudaStream_t s);
void layernorm_fwd(DType dt, const void* x, const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                   int64_t rows, int D, float eps, cudaStream_t s);
int layernorm_bwd_blocks(int64_t rows);
int64_t layernorm_bwd_scratch_floats(int64_t rows, int D);
// dres (optional, same dtype/shape as dx): a residual-branch gradient added
// to dx, fusing the sum of the two gradients of a pre-norm block input.
void layernorm_bwd(DType dt, const void* x, const float* gamma, const float* mean, const float* rstd, const void* dy,
                   void* dx, float* dgamma, float* dbeta, bool accumulate, int64_t rows, int D, float* scratch,
                   cudaStream_t s, const void* dres = nullptr);
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

}  // namespace dlvk
