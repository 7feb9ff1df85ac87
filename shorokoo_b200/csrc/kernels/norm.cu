// Group normalisation over NHWC activations (RetGroupNorm of the GroupNorm RetinaNet heads,
// samples/RetinaNet/RetinaNetDetector.cs:337-372): per (image n, group g) of C/G channels over all
// H x W pixels, y = (x - mean) / sqrt(var + eps) * gamma[c] + beta[c] (biased variance), then an
// optional ReLU, in three memory-bound passes:
//
//  1. gn_stats: blocks own contiguous pixel ranges of one image; each thread keeps one vector of
//     channels (8 bf16 or 4 fp32, 16 bytes) for the whole range, so a warp reads whole pixel rows
//     (coalesced 128-bit loads) and accumulates per channel, in fp32, the sums of (x - K_c) and
//     (x - K_c)^2 with K_c = x[n, pixel 0, c] (a shift that keeps the squares from cancelling when
//     the mean is large against the spread). Threads of one channel vector reduce in shared memory;
//     the block writes its per-channel partial sums.
//  2. gn_finalize: one thread per (n, g) merges the partials of its channels in double
//     (sum (x - mu)^2 = sum (x - K)^2 + 2 (K - mu) sum (x - K) + count (K - mu)^2 per channel) and
//     writes the per-(n, c) affine a = gamma rstd, b = beta - mu gamma rstd.
//  3. gn_apply: the pass-1 geometry again, y = act(x a + b) with a and b in registers, stored
//     bf16, fp32, or fp32 rounded to the TF32 grid for a single-pass TF32 reader.
// Bytes per element: 2 reads + 1 write of the activation (plus the negligible partials).
#include <cuda_bf16.h>

#include <cmath>

#include "kernels.h"

namespace sb {
namespace k {
namespace {

constexpr int kGnThreads = 256;

__device__ __forceinline__ void load_vec(const void* p, int bf16, int64_t off, float* v) {
  if (bf16) {
    const uint4 q = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p) + off);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  } else {
    const float4 q = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + off);
    v[0] = q.x;
    v[1] = q.y;
    v[2] = q.z;
    v[3] = q.w;
  }
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Pixel range [p0, p1) of image n handled by block b of `per_img` blocks.
__device__ __forceinline__ void pixel_range(int64_t HW, int per_img, int b, int64_t& p0, int64_t& p1) {
  const int64_t chunk = (HW + per_img - 1) / per_img;
  p0 = int64_t(b) * chunk;
  p1 = p0 + chunk < HW ? p0 + chunk : HW;
}

// partial layout: [N][per_img][2][C] floats (sum of x - K, sum of (x - K)^2)
__global__ void __launch_bounds__(kGnThreads) gn_stats_kernel(const void* __restrict__ x, int bf16, int N, int64_t HW,
                                                              int C, int64_t ldc, int per_img,
                                                              float* __restrict__ partial) {
  extern __shared__ float sred[];   // [kGnThreads][2 * VEC]
  const int VEC = bf16 ? 8 : 4;
  const int T = C / VEC;                 // threads per pixel (divides kGnThreads)
  const int rows = kGnThreads / T;       // pixels per step
  const int n = blockIdx.x / per_img, b = blockIdx.x - n * per_img;
  const int cv = threadIdx.x % T, r = threadIdx.x / T;
  int64_t p0, p1;
  pixel_range(HW, per_img, b, p0, p1);
  const int64_t base = int64_t(n) * HW * ldc + int64_t(cv) * VEC;
  float k[8], s1[8], s2[8];
  load_vec(x, bf16, base, k);   // pixel 0 of the image: the shift
#pragma unroll
  for (int i = 0; i < 8; ++i) s1[i] = s2[i] = 0.f;
  for (int64_t p = p0 + r; p < p1; p += rows) {
    float v[8];
    load_vec(x, bf16, base + p * ldc, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < VEC) {
        const float d = v[i] - k[i];
        s1[i] += d;
        s2[i] = fmaf(d, d, s2[i]);
      }
    }
  }
  float* mine = sred + threadIdx.x * 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mine[i] = s1[i];
    mine[8 + i] = s2[i];
  }
  __syncthreads();
  // threads cv, cv + T, ... hold the same channels: the first `T` threads sum them
  if (threadIdx.x < T) {
    float a[8], q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = q[i] = 0.f;
    for (int j = 0; j < rows; ++j) {
      const float* o = sred + (j * T + threadIdx.x) * 16;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        a[i] += o[i];
        q[i] += o[8 + i];
      }
    }
    float* out = partial + (int64_t(n) * per_img + b) * 2 * C + int64_t(cv) * VEC;
    for (int i = 0; i < VEC; ++i) {
      out[i] = a[i];
      out[C + i] = q[i];
    }
  }
}

// ab layout: [N][2][C] (a, then b)
__global__ void gn_finalize_kernel(const void* __restrict__ x, int bf16, int N, int64_t HW, int C, int64_t ldc,
                                   int G, int per_img, const float* __restrict__ partial, const float* __restrict__ gamma,
                                   const float* __restrict__ beta, float eps, float* __restrict__ ab) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= N * G) return;
  const int n = t / G, g = t - n * G;
  const int cpg = C / G;
  double tot = 0, sk[64], s1[64], s2[64];   // cpg <= 64
  for (int j = 0; j < cpg; ++j) {
    const int c = g * cpg + j;
    const int64_t off = int64_t(n) * HW * ldc + c;
    const double kc = bf16 ? double(__bfloat162float(static_cast<const __nv_bfloat16*>(x)[off]))
                           : double(static_cast<const float*>(x)[off]);
    double a = 0, q = 0;
    for (int b = 0; b < per_img; ++b) {
      const float* pp = partial + (int64_t(n) * per_img + b) * 2 * C;
      a += double(pp[c]);
      q += double(pp[C + c]);
    }
    sk[j] = kc;
    s1[j] = a;
    s2[j] = q;
    tot += a + double(HW) * kc;
  }
  const double cnt = double(HW) * cpg;
  const double mu = tot / cnt;
  double m2 = 0;
  for (int j = 0; j < cpg; ++j) {
    const double dk = sk[j] - mu;
    m2 += s2[j] + 2.0 * dk * s1[j] + double(HW) * dk * dk;
  }
  const double var = m2 > 0 ? m2 / cnt : 0.0;
  const double rstd = 1.0 / sqrt(var + double(eps));
  for (int j = 0; j < cpg; ++j) {
    const int c = g * cpg + j;
    const double ga = gamma ? double(gamma[c]) : 1.0, be = beta ? double(beta[c]) : 0.0;
    ab[int64_t(n) * 2 * C + c] = float(ga * rstd);
    ab[int64_t(n) * 2 * C + C + c] = float(be - mu * ga * rstd);
  }
}

__global__ void __launch_bounds__(kGnThreads) gn_apply_kernel(const void* __restrict__ x, int xb, int N, int64_t HW, int C,
                                                              int64_t ldc, int per_img, const float* __restrict__ ab,
                                                              void* __restrict__ y, int ymode, int64_t ldy, int relu) {
  const int VEC = xb ? 8 : 4;
  const int T = C / VEC;
  const int rows = kGnThreads / T;
  const int n = blockIdx.x / per_img, b = blockIdx.x - n * per_img;
  const int cv = threadIdx.x % T, r = threadIdx.x / T;
  int64_t p0, p1;
  pixel_range(HW, per_img, b, p0, p1);
  float a[8], bb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    a[i] = i < VEC ? ab[int64_t(n) * 2 * C + cv * VEC + i] : 0.f;
    bb[i] = i < VEC ? ab[int64_t(n) * 2 * C + C + cv * VEC + i] : 0.f;
  }
  const int64_t xbase = int64_t(n) * HW * ldc + int64_t(cv) * VEC;
  const int64_t ybase = int64_t(n) * HW * ldy + int64_t(cv) * VEC;
  for (int64_t p = p0 + r; p < p1; p += rows) {
    float v[8];
    load_vec(x, xb, xbase + p * ldc, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float o = fmaf(v[i], a[i], bb[i]);
      v[i] = relu ? fmaxf(o, 0.f) : o;
    }
    if (ymode == 0) {   // bf16: VEC elements (8 when the input is bf16, 4 otherwise)
      __nv_bfloat16* yp = static_cast<__nv_bfloat16*>(y) + ybase + p * ldy;
      if (VEC == 8) {
        uint4 q;
        uint32_t* w = reinterpret_cast<uint32_t*>(&q);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
          w[i] = *reinterpret_cast<uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(yp) = q;
      } else {
        uint2 q;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
        q.x = *reinterpret_cast<uint32_t*>(&h0);
        q.y = *reinterpret_cast<uint32_t*>(&h1);
        *reinterpret_cast<uint2*>(yp) = q;
      }
    } else {   // fp32 (ymode 2) or fp32 on the TF32 grid (ymode 1)
      float* yp = static_cast<float*>(y) + ybase + p * ldy;
      for (int h = 0; h < VEC; h += 4) {
        float4 q;
        q.x = ymode == 1 ? tf32_rna(v[h]) : v[h];
        q.y = ymode == 1 ? tf32_rna(v[h + 1]) : v[h + 1];
        q.z = ymode == 1 ? tf32_rna(v[h + 2]) : v[h + 2];
        q.w = ymode == 1 ? tf32_rna(v[h + 3]) : v[h + 3];
        *reinterpret_cast<float4*>(yp + h) = q;
      }
    }
  }
}

}  // namespace

bool group_norm_supported(int C, int G, int x_bf16) {
  const int vec = x_bf16 ? 8 : 4;
  if (G < 1 || C % G != 0 || C / G > 64 || C % vec != 0) return false;
  const int T = C / vec;
  return T <= 256 && 256 % T == 0;
}

int group_norm_blocks_per_image(int N, int64_t HW, int num_sms) {
  // about four blocks per SM over the batch, each at least a few pixel steps long
  int64_t per = (int64_t(4) * num_sms + N - 1) / N;
  const int64_t most = (HW + 31) / 32;
  if (per > most) per = most;
  return int(per < 1 ? 1 : per);
}

cudaError_t group_norm(const void* x, int x_bf16, int N, int64_t HW, int C, int64_t ldc, int G, float eps,
                       const float* gamma, const float* beta, void* y, int y_mode, int64_t ldy, int relu, int per_img,
                       float* partial, float* ab, cudaStream_t s) {
  const int vec = x_bf16 ? 8 : 4;
  const int T = C / vec;
  if (!group_norm_supported(C, G, x_bf16) || ldc % vec != 0 || ldy % vec != 0 || per_img < 1)
    return cudaErrorInvalidValue;
  (void)T;
  const int blocks = N * per_img;
  gn_stats_kernel<<<blocks, kGnThreads, kGnThreads * 16 * sizeof(float), s>>>(x, x_bf16, N, HW, C, ldc, per_img,
                                                                             partial);
  const int fin = N * G;
  gn_finalize_kernel<<<(fin + 127) / 128, 128, 0, s>>>(x, x_bf16, N, HW, C, ldc, G, per_img, partial, gamma, beta, eps,
                                                       ab);
  gn_apply_kernel<<<blocks, kGnThreads, 0, s>>>(x, x_bf16, N, HW, C, ldc, per_img, ab, y, y_mode, ldy, relu);
  return cudaGetLastError();
}

}  // namespace k
}  // namespace sb
