/* ORACLE (test infrastructure only): plain-loop double-precision Conv2d / MaxPool / GEMM.
 *
 * Cross-checks the torch-backed pieces of oracle/interp.py on small shapes with code that shares
 * nothing with torch.  Semantics follow ONNX opset 21 Conv / MaxPool as the reference's
 * shape rules state them (src/Shorokoo/Core/Inference/Ops/Conv.cs:34-61): output
 * = floor((in + pad_begin + pad_end - ((k-1)*d + 1)) / s) + 1, pads given explicitly.
 * Built by oracle/Makefile into oracle/_build/libref_small.so; called through ctypes by tests only.
 */
#include <math.h>
#include <stdint.h>

/* x [N,C,H,W], w [M,C/G,KH,KW], b [M] or NULL, y [N,M,OH,OW] */
void ref_conv2d(const double* x, const double* w, const double* b, double* y,
                int64_t N, int64_t C, int64_t H, int64_t W, int64_t M, int64_t KH, int64_t KW,
                int64_t sh, int64_t sw, int64_t dh, int64_t dw,
                int64_t pt, int64_t pl, int64_t pb, int64_t pr, int64_t G) {
  int64_t OH = (H + pt + pb - ((KH - 1) * dh + 1)) / sh + 1;
  int64_t OW = (W + pl + pr - ((KW - 1) * dw + 1)) / sw + 1;
  int64_t cpg = C / G, mpg = M / G;
  for (int64_t n = 0; n < N; ++n)
    for (int64_t m = 0; m < M; ++m) {
      int64_t g = m / mpg;
      for (int64_t oh = 0; oh < OH; ++oh)
        for (int64_t ow = 0; ow < OW; ++ow) {
          double acc = b ? b[m] : 0.0;
          for (int64_t c = 0; c < cpg; ++c)
            for (int64_t kh = 0; kh < KH; ++kh) {
              int64_t ih = oh * sh - pt + kh * dh;
              if (ih < 0 || ih >= H) continue;
              for (int64_t kw = 0; kw < KW; ++kw) {
                int64_t iw = ow * sw - pl + kw * dw;
                if (iw < 0 || iw >= W) continue;
                acc += x[((n * C + g * cpg + c) * H + ih) * W + iw] *
                       w[((m * cpg + c) * KH + kh) * KW + kw];
              }
            }
          y[((n * M + m) * OH + oh) * OW + ow] = acc;
        }
    }
}

/* x [N,C,H,W] -> y [N,C,OH,OW]; OH/OW passed by the caller (ceil_mode handled there). */
void ref_maxpool2d(const double* x, double* y, int64_t N, int64_t C, int64_t H, int64_t W,
                   int64_t OH, int64_t OW, int64_t KH, int64_t KW, int64_t sh, int64_t sw,
                   int64_t dh, int64_t dw, int64_t pt, int64_t pl) {
  for (int64_t nc = 0; nc < N * C; ++nc)
    for (int64_t oh = 0; oh < OH; ++oh)
      for (int64_t ow = 0; ow < OW; ++ow) {
        double m = -INFINITY;
        for (int64_t kh = 0; kh < KH; ++kh) {
          int64_t ih = oh * sh - pt + kh * dh;
          if (ih < 0 || ih >= H) continue;
          for (int64_t kw = 0; kw < KW; ++kw) {
            int64_t iw = ow * sw - pl + kw * dw;
            if (iw < 0 || iw >= W) continue;
            double v = x[(nc * H + ih) * W + iw];
            if (v > m) m = v;
          }
        }
        y[(nc * OH + oh) * OW + ow] = m;
      }
}

/* y[M,N] = a[M,K] * b[K,N] (+ bias[N]) */
void ref_gemm(const double* a, const double* b, const double* bias, double* y,
              int64_t M, int64_t N, int64_t K) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      double acc = bias ? bias[j] : 0.0;
      for (int64_t k = 0; k < K; ++k) acc += a[i * K + k] * b[k * N + j];
      y[i * N + j] = acc;
    }
}
