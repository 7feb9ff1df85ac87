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
//  2. gn_finalize: one warp per (n, g) merges the partials of its channels in double
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

// 16 bytes of channels: 8 bf16 or 4 fp32 values.
__device__ __forceinline__ uint4 load16(const void* p, int64_t byte_off) {
  return *reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p) + byte_off);
}
template <bool BF16>
__device__ __forceinline__ void unpack16(uint4 q, float* v) {
  if (BF16) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  } else {
    v[0] = __uint_as_float(q.x);
    v[1] = __uint_as_float(q.y);
    v[2] = __uint_as_float(q.z);
    v[3] = __uint_as_float(q.w);
  }
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// VEC values to y at element offset off: bf16 (ymode 0), fp32 on the TF32 grid (1) or fp32 (2).
__device__ __forceinline__ void store_vec(void* y, int ymode, int VEC, int64_t off, const float* v) {
  if (ymode == 0) {
    __nv_bfloat16* yp = static_cast<__nv_bfloat16*>(y) + off;
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    if (VEC == 8)
      *reinterpret_cast<uint4*>(yp) = make_uint4(w[0], w[1], w[2], w[3]);
    else
      *reinterpret_cast<uint2*>(yp) = make_uint2(w[0], w[1]);
  } else {
    float* yp = static_cast<float*>(y) + off;
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

// Pixel range [p0, p1) of image n handled by block b of `per_img` blocks.
__device__ __forceinline__ void pixel_range(int64_t HW, int per_img, int b, int64_t& p0, int64_t& p1) {
  const int64_t chunk = (HW + per_img - 1) / per_img;
  p0 = int64_t(b) * chunk;
  p1 = p0 + chunk < HW ? p0 + chunk : HW;
}

// partial layout: [N][per_img][2][C] floats (sum of x - K, sum of (x - K)^2)
template <bool BF16>
__global__ void __launch_bounds__(kGnThreads, 4) gn_stats_kernel(const void* __restrict__ x, int64_t HW, int C,
                                                                 int64_t ldc, int per_img, float* __restrict__ partial) {
  extern __shared__ float sred[];   // [kGnThreads][16]
  constexpr int VEC = BF16 ? 8 : 4;
  constexpr int ES = BF16 ? 2 : 4;
  const int T = C / VEC;                 // threads per pixel (divides kGnThreads)
  const int rows = kGnThreads / T;       // pixels per step
  const int n = blockIdx.x / per_img, b = blockIdx.x - n * per_img;
  const int cv = threadIdx.x % T, r = threadIdx.x / T;
  int64_t p0, p1;
  pixel_range(HW, per_img, b, p0, p1);
  const int64_t base = (int64_t(n) * HW * ldc + int64_t(cv) * VEC) * ES;
  const int64_t step = ldc * ES;
  float k[VEC], s1[VEC], s2[VEC];
  unpack16<BF16>(load16(x, base), k);   // pixel 0 of the image: the shift
#pragma unroll
  for (int i = 0; i < VEC; ++i) s1[i] = s2[i] = 0.f;
  // four pixels per iteration, their loads issued before any is used (bytes in flight per SM)
  for (int64_t p = p0 + r; p < p1; p += 4 * rows) {
    uint4 q[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (p + u * rows < p1) q[u] = load16(x, base + (p + u * rows) * step);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (p + u * rows >= p1) break;
      float v[VEC];
      unpack16<BF16>(q[u], v);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const float d = v[i] - k[i];
        s1[i] += d;
        s2[i] = fmaf(d, d, s2[i]);
      }
    }
  }
  float* mine = sred + threadIdx.x * 16;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    mine[i] = s1[i];
    mine[8 + i] = s2[i];
  }
  __syncthreads();
  // threads cv, cv + T, ... hold the same channels: the first `T` threads sum them
  if (threadIdx.x < T) {
    float sa[VEC], sq[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) sa[i] = sq[i] = 0.f;
    for (int j = 0; j < rows; ++j) {
      const float* o = sred + (j * T + threadIdx.x) * 16;
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        sa[i] += o[i];
        sq[i] += o[8 + i];
      }
    }
    float* out = partial + (int64_t(n) * per_img + b) * 2 * C + int64_t(cv) * VEC;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      out[i] = sa[i];
      out[C + i] = sq[i];
    }
  }
}

// ab layout: [N][2][C] (a, then b). One warp per (n, g): the warp's lanes first sum the block
// partials of the group's channels (lane = channel j + cpg * block offset, blocks strided by
// 32 / cpg), in double, and reduce across the lanes of one channel with shuffles; lane j then
// holds channel j's sums and the group merge runs across the channel lanes.
__device__ __forceinline__ double shfl_xor_d(double v, int o) { return __shfl_xor_sync(0xFFFFFFFFu, v, o); }

__global__ void __launch_bounds__(128) gn_finalize_kernel(const void* __restrict__ x, int bf16, int N, int64_t HW, int C,
                                                          int64_t ldc, int G, int per_img,
                                                          const float* __restrict__ partial,
                                                          const float* __restrict__ gamma,
                                                          const float* __restrict__ beta, float eps,
                                                          float* __restrict__ ab) {
  const int wid = int((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (wid >= N * G) return;   // (whole warps)
  const int n = wid / G, g = wid - n * G;
  const int cpg = C / G;      // a power of two <= 32 (checked on the host)
  const int j = lane & (cpg - 1), bsub = lane / cpg, bstep = 32 / cpg;
  const int c = g * cpg + j;
  double s1 = 0, s2 = 0;
  for (int b = bsub; b < per_img; b += bstep) {
    const float* pp = partial + (int64_t(n) * per_img + b) * 2 * C;
    s1 += double(pp[c]);
    s2 += double(pp[C + c]);
  }
  for (int o = cpg; o < 32; o <<= 1) {   // over the lanes of this channel
    s1 += shfl_xor_d(s1, o);
    s2 += shfl_xor_d(s2, o);
  }
  const int64_t off = int64_t(n) * HW * ldc + c;
  const double kc = bf16 ? double(__bfloat162float(static_cast<const __nv_bfloat16*>(x)[off]))
                         : double(static_cast<const float*>(x)[off]);
  // group totals over the channel lanes (lanes 0 .. cpg-1 hold one channel each; the others repeat
  // them, so reduce within groups of cpg lanes)
  double tot = s1 + double(HW) * kc;
  for (int o = 1; o < cpg; o <<= 1) tot += shfl_xor_d(tot, o);
  const double cnt = double(HW) * cpg;
  const double mu = tot / cnt;
  const double dk = kc - mu;
  double m2 = s2 + 2.0 * dk * s1 + double(HW) * dk * dk;
  for (int o = 1; o < cpg; o <<= 1) m2 += shfl_xor_d(m2, o);
  const double var = m2 > 0 ? m2 / cnt : 0.0;
  const double rstd = 1.0 / sqrt(var + double(eps));
  if (lane < cpg) {
    const double ga = gamma ? double(gamma[c]) : 1.0, be = beta ? double(beta[c]) : 0.0;
    ab[int64_t(n) * 2 * C + c] = float(ga * rstd);
    ab[int64_t(n) * 2 * C + C + c] = float(be - mu * ga * rstd);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(kGnThreads, 4) gn_apply_kernel(const void* __restrict__ x, int64_t HW, int C,
                                                                 int64_t ldc, int per_img, const float* __restrict__ ab,
                                                                 void* __restrict__ y, int ymode, int64_t ldy, int relu) {
  constexpr int VEC = BF16 ? 8 : 4;
  constexpr int ES = BF16 ? 2 : 4;
  const int T = C / VEC;
  const int rows = kGnThreads / T;
  const int n = blockIdx.x / per_img, b = blockIdx.x - n * per_img;
  const int cv = threadIdx.x % T, r = threadIdx.x / T;
  int64_t p0, p1;
  pixel_range(HW, per_img, b, p0, p1);
  float a[VEC], bb[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    a[i] = ab[int64_t(n) * 2 * C + cv * VEC + i];
    bb[i] = ab[int64_t(n) * 2 * C + C + cv * VEC + i];
  }
  const int64_t xbase = (int64_t(n) * HW * ldc + int64_t(cv) * VEC) * ES;
  const int64_t xstep = ldc * ES;
  const int64_t ybase = int64_t(n) * HW * ldy + int64_t(cv) * VEC;
  for (int64_t p = p0 + r; p < p1; p += 4 * rows) {
    uint4 q[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (p + u * rows < p1) q[u] = load16(x, xbase + (p + u * rows) * xstep);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (p + u * rows >= p1) break;
      float v[8];
      unpack16<BF16>(q[u], v);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const float o = fmaf(v[i], a[i], bb[i]);
        v[i] = relu ? fmaxf(o, 0.f) : o;
      }
      store_vec(y, ymode, VEC, ybase + (p + u * rows) * ldy, v);
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// One warp per row of D features (D a multiple of 4): the mean, then the biased variance from the
// centred values (two passes over the row, which stays in L1), then the affine write.
__global__ void __launch_bounds__(256) layer_norm_kernel(const float* __restrict__ x, int64_t rows, int D, int64_t ldx,
                                                         float eps, const float* __restrict__ gamma,
                                                         const float* __restrict__ beta, void* __restrict__ y,
                                                         int ymode, int64_t ldy) {
  const int lane = threadIdx.x & 31;
  const int64_t wpb = blockDim.x >> 5;
  for (int64_t row = blockIdx.x * wpb + (threadIdx.x >> 5); row < rows; row += int64_t(gridDim.x) * wpb) {
    const float* xr = x + row * ldx;
    float s = 0.f;
    for (int i = lane * 4; i < D; i += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xr + i);
      s += (v.x + v.y) + (v.z + v.w);
    }
    const float mean = warp_sum(s) / float(D);
    float q = 0.f;
    for (int i = lane * 4; i < D; i += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xr + i);
      const float a = v.x - mean, b = v.y - mean, c = v.z - mean, d = v.w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
    const float rstd = 1.f / sqrtf(warp_sum(q) / float(D) + eps);
    for (int i = lane * 4; i < D; i += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xr + i);
      const float4 g = *reinterpret_cast<const float4*>(gamma + i);
      const float4 bt = *reinterpret_cast<const float4*>(beta + i);
      float o[8] = {(v.x - mean) * rstd * g.x + bt.x, (v.y - mean) * rstd * g.y + bt.y,
                    (v.z - mean) * rstd * g.z + bt.z, (v.w - mean) * rstd * g.w + bt.w, 0.f, 0.f, 0.f, 0.f};
      store_vec(y, ymode, 4, row * ldy + i, o);
    }
  }
}

}  // namespace

cudaError_t layer_norm(const float* x, int64_t rows, int D, int64_t ldx, float eps, const float* gamma,
                       const float* beta, void* y, int y_mode, int64_t ldy, cudaStream_t s) {
  if (D % 4 || ldx % 4 || ldy % 4 || (reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(y) & 15u))
    return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  int64_t blocks = (rows + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  layer_norm_kernel<<<int(blocks), 256, 0, s>>>(x, rows, D, ldx, eps, gamma, beta, y, y_mode, ldy);
  return cudaGetLastError();
}

bool group_norm_supported(int C, int G, int x_bf16) {
  const int vec = x_bf16 ? 8 : 4;
  if (G < 1 || C % G != 0 || C % vec != 0) return false;
  const int cpg = C / G;   // channels per group: a power of two up to 32 (one warp merges a group)
  if (cpg > 32 || (cpg & (cpg - 1)) != 0) return false;
  const int T = C / vec;
  return T <= 256 && 256 % T == 0;
}

int group_norm_blocks_per_image(int N, int64_t HW, int num_sms) {
  // one wave of four 256-thread blocks per SM (the register budget of the four-pixel unrolled
  // loops) over the batch, each at least a few pixel steps long
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
  const size_t shm = kGnThreads * 16 * sizeof(float);
  if (x_bf16)
    gn_stats_kernel<true><<<blocks, kGnThreads, shm, s>>>(x, HW, C, ldc, per_img, partial);
  else
    gn_stats_kernel<false><<<blocks, kGnThreads, shm, s>>>(x, HW, C, ldc, per_img, partial);
  const int fin = N * G * 32;   // one warp per (image, group)
  gn_finalize_kernel<<<(fin + 127) / 128, 128, 0, s>>>(x, x_bf16, N, HW, C, ldc, G, per_img, partial, gamma, beta, eps,
                                                       ab);
  if (x_bf16)
    gn_apply_kernel<true><<<blocks, kGnThreads, 0, s>>>(x, HW, C, ldc, per_img, ab, y, y_mode, ldy, relu);
  else
    gn_apply_kernel<false><<<blocks, kGnThreads, 0, s>>>(x, HW, C, ldc, per_img, ab, y, y_mode, ldy, relu);
  return cudaGetLastError();
}

}  // namespace k
}  // namespace sb
