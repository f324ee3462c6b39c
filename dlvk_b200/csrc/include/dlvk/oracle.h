// CPU oracle (plain C++ restatement of the reference op semantics).  See
// csrc/ref/oracle.cpp for the per-op reference citations.
#pragma once
#include <cstdint>

namespace dlvk {
namespace ref {

struct ConvShape {
  int N, Cin, H, W, Cout, KH, KW, stride, pad;
  int Ho() const { return (H + 2 * pad - KH) / stride + 1; }
  int Wo() const { return (W + 2 * pad - KW) / stride + 1; }
};

void dense_fwd(const float* x, const float* w, const float* b, float* y, int64_t M, int64_t K, int64_t N);
void dense_bwd(const float* x, const float* w, const float* g, float* dx, float* dw, float* db, int64_t M, int64_t K,
               int64_t N);
void relu(const float* x, float* y, int64_t n);
void relu_bwd(const float* g, const float* x, float* dx, int64_t n);
void softmax(const float* x, float* y, int64_t rows, int64_t cols);
float cross_entropy(const float* p, const float* t, int64_t rows, int64_t cols);
void cross_entropy_grad(const float* p, const float* t, float* g, int64_t rows, int64_t cols);
float mse(const float* p, const float* t, float* g, int64_t n);
float bce(const float* p, const float* t, float* g, int64_t n);
void adam(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2, float eps, int step,
          bool bias_correction);
void sgd(float* p, const float* g, float* vel, int64_t n, float lr, float mom);
void rmsprop(float* p, const float* g, float* sq, int64_t n, float lr, float alpha, float eps);
void conv2d_fwd(const float* x, const float* w, const float* b, float* y, const ConvShape& s);
void conv2d_bwd(const float* x, const float* w, const float* g, float* dx, float* dw, float* db, const ConvShape& s);
void maxpool_fwd(const float* x, float* y, int32_t* idx, int N, int C, int H, int W, int k, int stride);
void maxpool_bwd(const float* g, const int32_t* idx, float* dx, int N, int C, int H, int W, int Ho, int Wo);
void avgpool_fwd(const float* x, float* y, int N, int C, int H, int W, int k, int stride, int pad);
void avgpool_bwd(const float* g, float* dx, int N, int C, int H, int W, int k, int stride, int pad);
void batchnorm_fwd(const float* x, const float* gamma, const float* beta, float* y, float* mean, float* rstd,
                   float* run_mean, float* run_var, int N, int C, int S, float momentum, float eps, bool training);
void batchnorm_bwd(const float* x, const float* gamma, const float* mean, const float* rstd, const float* g, float* dx,
                   float* dgamma, float* dbeta, int N, int C, int S);
void layernorm_fwd(const float* x, const float* gamma, const float* beta, float* y, float* mean, float* rstd,
                   int64_t rows, int64_t D, float eps);
void layernorm_bwd(const float* x, const float* gamma, const float* mean, const float* rstd, const float* g, float* dx,
                   float* dgamma, float* dbeta, int64_t rows, int64_t D);
void embedding_fwd(const int32_t* ids, const float* table, float* out, int64_t n, int64_t V, int64_t D);
void embedding_bwd(const int32_t* ids, const float* g, float* dtable, int64_t n, int64_t V, int64_t D);
void dropout_mask(uint8_t* keep, int64_t n, float p, uint64_t seed, uint32_t stream, uint32_t step);
void attention(const float* q, const float* k, const float* v, float* o, int B, int H, int S, int D, bool causal);

}  // namespace ref
}  // namespace dlvk
