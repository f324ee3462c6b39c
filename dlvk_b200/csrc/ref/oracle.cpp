// CPU oracle: plain single-threaded C++ restatement of the reference's op
// semantics, used as the numerical ground truth in tests and as the timed
// CPU baseline.  Every function works on contiguous fp32 arrays.
//
// Semantics (reference file:line):
//  dense        Y = X W + b, W [in,out]           src/layers/dense_layer.cpp:31-42
//  dense bwd    dX = g W^T, dW = X^T g, db = sum0 g src/layers/dense_layer.cpp:44-66
//  softmax      row-wise, max-subtracted          shaders/softmax.comp:32-66
//  CE           -sum t log(p + 1e-8) / B           src/loss/loss_functions.cpp:127-135
//  CE grad      (p - t) / B w.r.t. softmax output  src/loss/loss_functions.cpp:158-160
//  MSE / BCE    src/loss/loss_functions.cpp:59-64,93-96,189-200,230-238
//  Adam         shaders/adam_update.comp:31-61 with bc = 1/(1-beta^t)
//  SGD          v = mu v + g; p -= lr v            src/optimizers/sgd.cpp:55-76
//  conv2d       direct NCHW, W [Cout,Cin,KH,KW]    shaders/conv2d.comp:37-84 (+ bwd shaders)
//  maxpool      first max wins (strict >)         src/layers/pooling_layers.cpp:63-99
//  avgpool      / valid count, count_include_pad=false  shaders/avgpool2d*.comp
//  batchnorm    biased var, running=(1-m)r+m*batch src/layers/batch_norm_layers.cpp:65-116
//  layernorm    shaders/layer_norm.comp:44-91
//  embedding    out-of-range id -> zeros           shaders/embedding_lookup.comp:36-44
//  dropout      Philox4x32-10, key seed, counter {idx/4, stream, step}; keep iff u >= p
#include "dlvk/oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

namespace dlvk {
namespace ref {

void dense_fwd(const float* x, const float* w, const float* b, float* y, int64_t M, int64_t K, int64_t N) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.f;
      for (int64_t k = 0; k < K; ++k) acc += x[m * K + k] * w[k * N + n];
      y[m * N + n] = acc + (b ? b[n] : 0.f);
    }
}

void dense_bwd(const float* x, const float* w, const float* g, float* dx, float* dw, float* db, int64_t M, int64_t K,
               int64_t N) {
  if (dx)
    for (int64_t m = 0; m < M; ++m)
      for (int64_t k = 0; k < K; ++k) {
        float acc = 0.f;
        for (int64_t n = 0; n < N; ++n) acc += g[m * N + n] * w[k * N + n];
        dx[m * K + k] = acc;
      }
  if (dw)
    for (int64_t k = 0; k < K; ++k)
      for (int64_t n = 0; n < N; ++n) {
        float acc = 0.f;
        for (int64_t m = 0; m < M; ++m) acc += x[m * K + k] * g[m * N + n];
        dw[k * N + n] = acc;
      }
  if (db)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.f;
      for (int64_t m = 0; m < M; ++m) acc += g[m * N + n];
      db[n] = acc;
    }
}

void relu(const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = x[i] > 0.f ? x[i] : 0.f;
}
void relu_bwd(const float* g, const float* x, float* dx, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dx[i] = x[i] > 0.f ? g[i] : 0.f;
}

void softmax(const float* x, float* y, int64_t rows, int64_t cols) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * cols;
    float* yr = y + r * cols;
    float mx = xr[0];
    for (int64_t c = 1; c < cols; ++c) mx = std::max(mx, xr[c]);
    float s = 0.f;
    for (int64_t c = 0; c < cols; ++c) {
      yr[c] = std::exp(xr[c] - mx);
      s += yr[c];
    }
    for (int64_t c = 0; c < cols; ++c) yr[c] /= s;
  }
}

float cross_entropy(const float* p, const float* t, int64_t rows, int64_t cols) {
  double acc = 0.0;
  for (int64_t i = 0; i < rows * cols; ++i) acc += -(double)t[i] * std::log((double)p[i] + 1e-8);
  return (float)(acc / rows);
}
void cross_entropy_grad(const float* p, const float* t, float* g, int64_t rows, int64_t cols) {
  for (int64_t i = 0; i < rows * cols; ++i) g[i] = (p[i] - t[i]) / (float)rows;
}

float mse(const float* p, const float* t, float* g, int64_t n) {
  double acc = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    const float d = p[i] - t[i];
    acc += (double)d * d;
    if (g) g[i] = 2.f * d / (float)n;
  }
  return (float)(acc / n);
}
float bce(const float* p, const float* t, float* g, int64_t n) {
  double acc = 0.0;
  const float eps = 1e-7f;
  for (int64_t i = 0; i < n; ++i) {
    const float pc = std::min(std::max(p[i], eps), 1.f - eps);
    acc += -((double)t[i] * std::log((double)pc) + (1.0 - t[i]) * std::log(1.0 - pc));
    if (g) g[i] = (pc - t[i]) / (pc * (1.f - pc)) / (float)n;
  }
  return (float)(acc / n);
}

void adam(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2, float eps, int step,
          bool bias_correction) {
  const float bc1 = bias_correction ? 1.f / (1.f - std::pow(b1, (float)step)) : 1.f;
  const float bc2 = bias_correction ? 1.f / (1.f - std::pow(b2, (float)step)) : 1.f;
  for (int64_t i = 0; i < n; ++i) {
    m[i] = b1 * m[i] + (1.f - b1) * g[i];
    v[i] = b2 * v[i] + (1.f - b2) * g[i] * g[i];
    p[i] -= lr * (m[i] * bc1) / (std::sqrt(v[i] * bc2) + eps);
  }
}
void sgd(float* p, const float* g, float* vel, int64_t n, float lr, float mom) {
  for (int64_t i = 0; i < n; ++i) {
    if (mom != 0.f) {
      vel[i] = mom * vel[i] + g[i];
      p[i] -= lr * vel[i];
    } else {
      p[i] -= lr * g[i];
    }
  }
}
void rmsprop(float* p, const float* g, float* sq, int64_t n, float lr, float alpha, float eps) {
  for (int64_t i = 0; i < n; ++i) {
    sq[i] = alpha * sq[i] + (1.f - alpha) * g[i] * g[i];
    p[i] -= lr * g[i] / (std::sqrt(sq[i]) + eps);
  }
}

void conv2d_fwd(const float* x, const float* w, const float* b, float* y, const ConvShape& s) {
  const int Ho = s.Ho(), Wo = s.Wo();
  for (int n = 0; n < s.N; ++n)
    for (int co = 0; co < s.Cout; ++co)
      for (int oh = 0; oh < Ho; ++oh)
        for (int ow = 0; ow < Wo; ++ow) {
          float acc = b ? b[co] : 0.f;
          for (int ci = 0; ci < s.Cin; ++ci)
            for (int kh = 0; kh < s.KH; ++kh)
              for (int kw = 0; kw < s.KW; ++kw) {
                const int ih = oh * s.stride - s.pad + kh, iw = ow * s.stride - s.pad + kw;
                if (ih < 0 || ih >= s.H || iw < 0 || iw >= s.W) continue;
                acc += x[((int64_t)(n * s.Cin + ci) * s.H + ih) * s.W + iw] *
                       w[((co * s.Cin + ci) * s.KH + kh) * s.KW + kw];
              }
          y[((int64_t)(n * s.Cout + co) * Ho + oh) * Wo + ow] = acc;
        }
}

void conv2d_bwd(const float* x, const float* w, const float* g, float* dx, float* dw, float* db, const ConvShape& s) {
  const int Ho = s.Ho(), Wo = s.Wo();
  if (dx) std::memset(dx, 0, sizeof(float) * (size_t)s.N * s.Cin * s.H * s.W);
  if (dw) std::memset(dw, 0, sizeof(float) * (size_t)s.Cout * s.Cin * s.KH * s.KW);
  if (db) std::memset(db, 0, sizeof(float) * (size_t)s.Cout);
  for (int n = 0; n < s.N; ++n)
    for (int co = 0; co < s.Cout; ++co)
      for (int oh = 0; oh < Ho; ++oh)
        for (int ow = 0; ow < Wo; ++ow) {
          const float gv = g[((int64_t)(n * s.Cout + co) * Ho + oh) * Wo + ow];
          if (db) db[co] += gv;
          for (int ci = 0; ci < s.Cin; ++ci)
            for (int kh = 0; kh < s.KH; ++kh)
              for (int kw = 0; kw < s.KW; ++kw) {
                const int ih = oh * s.stride - s.pad + kh, iw = ow * s.stride - s.pad + kw;
                if (ih < 0 || ih >= s.H || iw < 0 || iw >= s.W) continue;
                const int64_t xi = ((int64_t)(n * s.Cin + ci) * s.H + ih) * s.W + iw;
                const int64_t wi = ((co * s.Cin + ci) * s.KH + kh) * s.KW + kw;
                if (dx) dx[xi] += gv * w[wi];
                if (dw) dw[wi] += gv * x[xi];
              }
        }
}

void maxpool_fwd(const float* x, float* y, int32_t* idx, int N, int C, int H, int W, int k, int stride) {
  const int Ho = (H - k) / stride + 1, Wo = (W - k) / stride + 1;
  for (int nc = 0; nc < N * C; ++nc)
    for (int oh = 0; oh < Ho; ++oh)
      for (int ow = 0; ow < Wo; ++ow) {
        float best = -INFINITY;
        int bi = -1;
        for (int kh = 0; kh < k; ++kh)
          for (int kw = 0; kw < k; ++kw) {
            const int ih = oh * stride + kh, iw = ow * stride + kw;
            const float v = x[((int64_t)nc * H + ih) * W + iw];
            if (bi < 0 || v > best) {  // strict '>': the first maximum wins
              best = v;
              bi = ih * W + iw;
            }
          }
        y[((int64_t)nc * Ho + oh) * Wo + ow] = best;
        if (idx) idx[((int64_t)nc * Ho + oh) * Wo + ow] = bi;
      }
}
void maxpool_bwd(const float* g, const int32_t* idx, float* dx, int N, int C, int H, int W, int Ho, int Wo) {
  std::memset(dx, 0, sizeof(float) * (size_t)N * C * H * W);
  for (int nc = 0; nc < N * C; ++nc)
    for (int o = 0; o < Ho * Wo; ++o) dx[(int64_t)nc * H * W + idx[(int64_t)nc * Ho * Wo + o]] += g[(int64_t)nc * Ho * Wo + o];
}

void avgpool_fwd(const float* x, float* y, int N, int C, int H, int W, int k, int stride, int pad) {
  const int Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
  for (int nc = 0; nc < N * C; ++nc)
    for (int oh = 0; oh < Ho; ++oh)
      for (int ow = 0; ow < Wo; ++ow) {
        float s = 0.f;
        int cnt = 0;
        for (int kh = 0; kh < k; ++kh)
          for (int kw = 0; kw < k; ++kw) {
            const int ih = oh * stride - pad + kh, iw = ow * stride - pad + kw;
            if (ih < 0 || ih >= H || iw < 0 || iw >= W) continue;
            s += x[((int64_t)nc * H + ih) * W + iw];
            ++cnt;
          }
        y[((int64_t)nc * Ho + oh) * Wo + ow] = cnt ? s / cnt : 0.f;
      }
}
void avgpool_bwd(const float* g, float* dx, int N, int C, int H, int W, int k, int stride, int pad) {
  const int Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
  std::memset(dx, 0, sizeof(float) * (size_t)N * C * H * W);
  for (int nc = 0; nc < N * C; ++nc)
    for (int oh = 0; oh < Ho; ++oh)
      for (int ow = 0; ow < Wo; ++ow) {
        int cnt = 0;
        for (int kh = 0; kh < k; ++kh)
          for (int kw = 0; kw < k; ++kw) {
            const int ih = oh * stride - pad + kh, iw = ow * stride - pad + kw;
            if (ih >= 0 && ih < H && iw >= 0 && iw < W) ++cnt;
          }
        if (!cnt) continue;
        const float gv = g[((int64_t)nc * Ho + oh) * Wo + ow] / cnt;
        for (int kh = 0; kh < k; ++kh)
          for (int kw = 0; kw < k; ++kw) {
            const int ih = oh * stride - pad + kh, iw = ow * stride - pad + kw;
            if (ih >= 0 && ih < H && iw >= 0 && iw < W) dx[((int64_t)nc * H + ih) * W + iw] += gv;
          }
      }
}

// Batch norm over [N, C, S] (S = spatial size, 1 for BatchNorm1D).
void batchnorm_fwd(const float* x, const float* gamma, const float* beta, float* y, float* mean, float* rstd,
                   float* run_mean, float* run_var, int N, int C, int S, float momentum, float eps, bool training) {
  for (int c = 0; c < C; ++c) {
    float mu, var;
    if (training) {
      double s = 0.0, s2 = 0.0;
      for (int n = 0; n < N; ++n)
        for (int i = 0; i < S; ++i) {
          const double v = x[((int64_t)n * C + c) * S + i];
          s += v;
          s2 += v * v;
        }
      const double cnt = (double)N * S;
      mu = (float)(s / cnt);
      var = (float)std::max(0.0, s2 / cnt - (s / cnt) * (s / cnt));
      if (run_mean) run_mean[c] = (1.f - momentum) * run_mean[c] + momentum * mu;
      if (run_var) run_var[c] = (1.f - momentum) * run_var[c] + momentum * var;
    } else {
      mu = run_mean[c];
      var = run_var[c];
    }
    const float rs = 1.f / std::sqrt(var + eps);
    if (mean) mean[c] = mu;
    if (rstd) rstd[c] = rs;
    for (int n = 0; n < N; ++n)
      for (int i = 0; i < S; ++i) {
        const int64_t k = ((int64_t)n * C + c) * S + i;
        y[k] = (x[k] - mu) * rs * (gamma ? gamma[c] : 1.f) + (beta ? beta[c] : 0.f);
      }
  }
}
void batchnorm_bwd(const float* x, const float* gamma, const float* mean, const float* rstd, const float* g, float* dx,
                   float* dgamma, float* dbeta, int N, int C, int S) {
  const double cnt = (double)N * S;
  for (int c = 0; c < C; ++c) {
    double sg = 0.0, sgx = 0.0;
    for (int n = 0; n < N; ++n)
      for (int i = 0; i < S; ++i) {
        const int64_t k = ((int64_t)n * C + c) * S + i;
        const double xh = (x[k] - mean[c]) * rstd[c];
        sg += g[k];
        sgx += g[k] * xh;
      }
    if (dgamma) dgamma[c] = (float)sgx;
    if (dbeta) dbeta[c] = (float)sg;
    const float gm = gamma ? gamma[c] : 1.f;
    for (int n = 0; n < N; ++n)
      for (int i = 0; i < S; ++i) {
        const int64_t k = ((int64_t)n * C + c) * S + i;
        const double xh = (x[k] - mean[c]) * rstd[c];
        dx[k] = (float)(gm * rstd[c] * (g[k] - sg / cnt - xh * sgx / cnt));
      }
  }
}

void layernorm_fwd(const float* x, const float* gamma, const float* beta, float* y, float* mean, float* rstd,
                   int64_t rows, int64_t D, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    double s = 0.0, s2 = 0.0;
    for (int64_t d = 0; d < D; ++d) {
      s += x[r * D + d];
      s2 += (double)x[r * D + d] * x[r * D + d];
    }
    const float mu = (float)(s / D);
    const float var = (float)std::max(0.0, s2 / D - (s / D) * (s / D));
    const float rs = 1.f / std::sqrt(var + eps);
    if (mean) mean[r] = mu;
    if (rstd) rstd[r] = rs;
    for (int64_t d = 0; d < D; ++d)
      y[r * D + d] = (x[r * D + d] - mu) * rs * (gamma ? gamma[d] : 1.f) + (beta ? beta[d] : 0.f);
  }
}
void layernorm_bwd(const float* x, const float* gamma, const float* mean, const float* rstd, const float* g, float* dx,
                   float* dgamma, float* dbeta, int64_t rows, int64_t D) {
  if (dgamma) std::fill(dgamma, dgamma + D, 0.f);
  if (dbeta) std::fill(dbeta, dbeta + D, 0.f);
  for (int64_t r = 0; r < rows; ++r) {
    double a = 0.0, b = 0.0;
    for (int64_t d = 0; d < D; ++d) {
      const double xh = (x[r * D + d] - mean[r]) * rstd[r];
      const double gg = g[r * D + d] * (gamma ? gamma[d] : 1.f);
      a += gg;
      b += gg * xh;
      if (dgamma) dgamma[d] += (float)(g[r * D + d] * xh);
      if (dbeta) dbeta[d] += g[r * D + d];
    }
    for (int64_t d = 0; d < D; ++d) {
      const double xh = (x[r * D + d] - mean[r]) * rstd[r];
      const double gg = g[r * D + d] * (gamma ? gamma[d] : 1.f);
      dx[r * D + d] = (float)(rstd[r] * (gg - a / D - xh * b / D));
    }
  }
}

void embedding_fwd(const int32_t* ids, const float* table, float* out, int64_t n, int64_t V, int64_t D) {
  for (int64_t i = 0; i < n; ++i) {
    const int32_t id = ids[i];
    for (int64_t d = 0; d < D; ++d) out[i * D + d] = (id >= 0 && id < V) ? table[(int64_t)id * D + d] : 0.f;
  }
}
void embedding_bwd(const int32_t* ids, const float* g, float* dtable, int64_t n, int64_t V, int64_t D) {
  std::fill(dtable, dtable + V * D, 0.f);
  for (int64_t i = 0; i < n; ++i) {
    const int32_t id = ids[i];
    if (id < 0 || id >= V) continue;
    for (int64_t d = 0; d < D; ++d) dtable[(int64_t)id * D + d] += g[i * D + d];
  }
}

// Philox4x32-10 (Salmon et al., SC'11) -- same stream as the CUDA kernels.
static void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)M0 * c[0], p1 = (uint64_t)M1 * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0, hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += W0;
    k1 += W1;
  }
}

void dropout_mask(uint8_t* keep, int64_t n, float p, uint64_t seed, uint32_t stream, uint32_t step) {
  for (int64_t i = 0; i < n; i += 4) {
    const uint64_t blk = (uint64_t)(i / 4);
    uint32_t c[4] = {(uint32_t)blk, (uint32_t)(blk >> 32), stream, step};
    philox(c, (uint32_t)seed, (uint32_t)(seed >> 32));
    for (int j = 0; j < 4 && i + j < n; ++j) {
      const float u = (float)(c[j] >> 8) * (1.0f / 16777216.0f);
      keep[i + j] = u >= p ? 1 : 0;
    }
  }
}

void attention(const float* q, const float* k, const float* v, float* o, int B, int H, int S, int D, bool causal) {
  const float scale = 1.f / std::sqrt((float)D);
  std::vector<float> row(S);
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h)
      for (int i = 0; i < S; ++i) {
        const float* qi = q + (((int64_t)b * H + h) * S + i) * D;
        float mx = -INFINITY;
        for (int j = 0; j < S; ++j) {
          if (causal && j > i) {
            row[j] = -INFINITY;
            continue;
          }
          const float* kj = k + (((int64_t)b * H + h) * S + j) * D;
          float s = 0.f;
          for (int d = 0; d < D; ++d) s += qi[d] * kj[d];
          row[j] = s * scale;
          mx = std::max(mx, row[j]);
        }
        float sum = 0.f;
        for (int j = 0; j < S; ++j) {
          row[j] = (row[j] == -INFINITY) ? 0.f : std::exp(row[j] - mx);
          sum += row[j];
        }
        float* oi = o + (((int64_t)b * H + h) * S + i) * D;
        for (int d = 0; d < D; ++d) {
          float acc = 0.f;
          for (int j = 0; j < S; ++j) acc += row[j] * v[(((int64_t)b * H + h) * S + j) * D + d];
          oi[d] = acc / sum;
        }
      }
}

}  // namespace ref
}  // namespace dlvk
