// Memory-bound kernels: layout/dtype conversion, NHWC max pooling, global pooling, generic strided
// elementwise / copy / softmax / reduce / gather. Coalesced along the innermost dimension and
// 128-bit vectorised where the layout allows; grids are sized in multiples of the SM count.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>

#include "kernels.h"

namespace sb {
namespace k {
namespace {

constexpr int kThreads = 256;

inline int grid_for(int64_t n, int threads = kThreads) {
  int64_t g = (n + threads - 1) / threads;
  if (g > 148 * 32) g = 148 * 32;   // grid-stride beyond 32 blocks per SM
  return int(g < 1 ? 1 : g);
}

__device__ __forceinline__ float ld_any(const void* p, int bf16, int64_t i) {
  return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_any(void* p, int bf16, int64_t i, float v) {
  if (bf16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// linear index -> offset under a strided descriptor
__device__ __forceinline__ int64_t offset_of(int64_t lin, const TDesc& d) {
  int64_t off = 0;
#pragma unroll 1
  for (int i = d.rank - 1; i >= 0; --i) {
    const int64_t s = d.shape[i];
    const int64_t q = lin / s;
    off += (lin - q * s) * d.stride[i];
    lin = q;
  }
  return off;
}

// ---- NCHW/any -> NHWC bf16 with channel padding ---------------------------------------------
// One thread per (pixel, 4-channel group): reads are coalesced across pixels of a channel plane.
__global__ void to_nhwc_bf16_kernel(const void* __restrict__ src, int src_bf16, int64_t N, int64_t C, int64_t H,
                                    int64_t W, int64_t s0, int64_t s1, int64_t s2, int64_t s3,
                                    __nv_bfloat16* __restrict__ dst, int Cp) {
  const int groups = Cp / 4;
  const int64_t total = N * H * W * groups;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    // order: pixel fastest within a channel group so that the strided reads coalesce
    const int64_t pix_total = N * H * W;
    const int g = int(i / pix_total);
    const int64_t pix = i - int64_t(g) * pix_total;
    const int64_t n = pix / (H * W);
    const int64_t hw = pix - n * H * W;
    const int64_t h = hw / W, w = hw - (hw / W) * W;
    const int64_t base = n * s0 + h * s2 + w * s3;
    __align__(8) __nv_bfloat16 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = int64_t(g) * 4 + j;
      v[j] = __float2bfloat16_rn(c < C ? ld_any(src, src_bf16, base + c * s1) : 0.f);
    }
    *reinterpret_cast<uint2*>(dst + pix * Cp + g * 4) = *reinterpret_cast<uint2*>(v);
  }
}

// 2x2 space-to-depth into NHWC bf16 with 16 channels: dst[n, hs, ws, (p*2+q)*C + c] =
// src[n, c, 2hs+p, 2ws+q] (zero outside the image; channels 4C..15 zero). One thread per pixel.
__global__ void to_s2d_bf16_kernel(const void* __restrict__ src, int src_bf16, int64_t N, int64_t C, int64_t H,
                                   int64_t W, int64_t s0, int64_t s1, int64_t s2, int64_t s3,
                                   __nv_bfloat16* __restrict__ dst, int64_t Hs, int64_t Ws) {
  const int64_t total = N * Hs * Ws;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t n = i / (Hs * Ws);
    const int64_t r = i - n * Hs * Ws;
    const int64_t hs = r / Ws, ws = r - (r / Ws) * Ws;
    __align__(16) __nv_bfloat16 v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __float2bfloat16_rn(0.f);
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int64_t h = 2 * hs + p, w = 2 * ws + q;
        if (h >= H || w >= W) continue;
        for (int64_t c = 0; c < C; ++c)
          v[(p * 2 + q) * C + c] = __float2bfloat16_rn(ld_any(src, src_bf16, n * s0 + c * s1 + h * s2 + w * s3));
      }
    uint4* d = reinterpret_cast<uint4*>(dst + i * 16);
    d[0] = reinterpret_cast<const uint4*>(v)[0];
    d[1] = reinterpret_cast<const uint4*>(v)[1];
  }
}

// The same for the common case: fp32 NCHW stored contiguously, even width, C (1-4) known at compile
// time. Each thread builds its 16-value pixel in registers from float2 loads of its two input rows
// (consecutive threads read consecutive 8-byte pairs of a row) and stores it as two 16-byte words.
template <int C>
__global__ void to_s2d_bf16_f32_kernel(const float* __restrict__ src, int64_t N, int64_t H, int64_t W,
                                       __nv_bfloat16* __restrict__ dst, int64_t Hs, int64_t Ws) {
  const int64_t total = N * Hs * Ws;
  const int64_t plane = H * W;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t n = i / (Hs * Ws);
    const int64_t r = i - n * Hs * Ws;
    const int64_t hs = r / Ws, ws = r - (r / Ws) * Ws;
    float f[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) f[j] = 0.f;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int64_t h = 2 * hs + p;
      if (h < H) {   // (the width is even: both columns of the pair exist)
#pragma unroll
        for (int c = 0; c < C; ++c) {
          const float2 x = __ldg(reinterpret_cast<const float2*>(src + (n * C + c) * plane + h * W + 2 * ws));
          f[(p * 2) * C + c] = x.x;
          f[(p * 2 + 1) * C + c] = x.y;
        }
      }
    }
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&b);
    }
    uint4* d = reinterpret_cast<uint4*>(dst + i * 16);
    d[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

// fp32 rounded to the TF32 grid (10 explicit mantissa bits, nearest, ties away): the operands the
// TF32 tensor-core path multiplies, rounded once here instead of truncated by the MMA.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// dst (NHWC fp32 [N,H,W,Cp], TF32-rounded) <- src logical [N,C,H,W], 4 channels per thread.
__global__ void to_nhwc_f32_kernel(const void* __restrict__ src, int src_bf16, int64_t N, int64_t C, int64_t H,
                                   int64_t W, int64_t s0, int64_t s1, int64_t s2, int64_t s3, float* __restrict__ dst,
                                   int Cp, int rnd) {
  const int groups = Cp / 4;
  const int64_t total = N * H * W * groups;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t pix_total = N * H * W;
    const int g = int(i / pix_total);
    const int64_t pix = i - int64_t(g) * pix_total;
    const int64_t n = pix / (H * W);
    const int64_t hw = pix - n * H * W;
    const int64_t h = hw / W, w = hw - (hw / W) * W;
    const int64_t base = n * s0 + h * s2 + w * s3;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = int64_t(g) * 4 + j;
      const float x = c < C ? ld_any(src, src_bf16, base + c * s1) : 0.f;
      v[j] = rnd ? tf32_rna(x) : x;
    }
    *reinterpret_cast<float4*>(dst + pix * Cp + g * 4) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

__global__ void to_rows_f32_kernel(const void* __restrict__ src, int src_bf16, int64_t M, int64_t K, int64_t sm,
                                   int64_t sk, float* __restrict__ dst, int64_t Kp, int rnd) {
  const int64_t total = M * Kp;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / Kp, kk = i - m * Kp;
    const float x = kk < K ? ld_any(src, src_bf16, m * sm + kk * sk) : 0.f;
    dst[i] = rnd ? tf32_rna(x) : x;
  }
}

// NHWC fp32 max pooling, 4 channels (16 bytes) per thread (padding never wins).
__global__ void maxpool_nhwc_f32_kernel(const float* __restrict__ x, float* __restrict__ y, int N, int H, int W, int C,
                                        int Ho, int Wo, int kh, int kw, int sh, int sw, int ph, int pw, int dh,
                                        int dw) {
  const int cg = C / 4;
  const int64_t total = int64_t(N) * Ho * Wo * cg;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int g = int(i % cg);
    int64_t pix = i / cg;
    const int wo = int(pix % Wo);
    pix /= Wo;
    const int ho = int(pix % Ho);
    const int n = int(pix / Ho);
    float4 m = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    for (int a = 0; a < kh; ++a) {
      const int hi = ho * sh - ph + a * dh;
      if (hi < 0 || hi >= H) continue;
      for (int b = 0; b < kw; ++b) {
        const int wi = wo * sw - pw + b * dw;
        if (wi < 0 || wi >= W) continue;
        const float4 q = __ldg(reinterpret_cast<const float4*>(x + ((int64_t(n) * H + hi) * W + wi) * C + g * 4));
        m.x = fmaxf(m.x, q.x);
        m.y = fmaxf(m.y, q.y);
        m.z = fmaxf(m.z, q.z);
        m.w = fmaxf(m.w, q.w);
      }
    }
    *reinterpret_cast<float4*>(y + i * 4) = m;
  }
}

__global__ void to_rows_bf16_kernel(const void* __restrict__ src, int src_bf16, int64_t M, int64_t K, int64_t sm,
                                    int64_t sk, __nv_bfloat16* __restrict__ dst, int64_t Kp) {
  const int64_t total = M * Kp;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / Kp, kk = i - m * Kp;
    dst[i] = __float2bfloat16_rn(kk < K ? ld_any(src, src_bf16, m * sm + kk * sk) : 0.f);
  }
}

// ---- NHWC bf16 max pooling, 8 channels (16 bytes) per thread ---------------------------------
__global__ void maxpool_nhwc_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int N, int H,
                                    int W, int C, int Ho, int Wo, int kh, int kw, int sh, int sw, int ph, int pw,
                                    int dh, int dw) {
  const int cg = C / 8;
  const int64_t total = int64_t(N) * Ho * Wo * cg;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int g = int(i % cg);
    int64_t pix = i / cg;
    const int wo = int(pix % Wo);
    pix /= Wo;
    const int ho = int(pix % Ho);
    const int n = int(pix / Ho);
    float m[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) m[j] = -INFINITY;
    for (int a = 0; a < kh; ++a) {
      const int hi = ho * sh - ph + a * dh;
      if (hi < 0 || hi >= H) continue;
      for (int b = 0; b < kw; ++b) {
        const int wi = wo * sw - pw + b * dw;
        if (wi < 0 || wi >= W) continue;
        uint4 q = __ldg(reinterpret_cast<const uint4*>(x + ((int64_t(n) * H + hi) * W + wi) * C + g * 8));
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float2 f = __bfloat1622float2(h[t]);
          m[2 * t] = fmaxf(m[2 * t], f.x);
          m[2 * t + 1] = fmaxf(m[2 * t + 1], f.y);
        }
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int t = 0; t < 4; ++t) oh[t] = __floats2bfloat162_rn(m[2 * t], m[2 * t + 1]);
    *reinterpret_cast<uint4*>(y + i * 8) = o;
  }
}

// K x K window, dilation 1 (the ResNet stem's 3x3/2 pool): all K*K loads of a thread are issued
// before the max chain, so the window's rows are in flight together.
template <int K>
__global__ void maxpool_k_nhwc_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int N,
                                      int H, int W, int C, int Ho, int Wo, int sh, int sw, int ph, int pw) {
  const int cg = C / 8;
  const int64_t total = int64_t(N) * Ho * Wo * cg;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int g = int(i % cg);
    int64_t pix = i / cg;
    const int wo = int(pix % Wo);
    pix /= Wo;
    const int ho = int(pix % Ho);
    const int n = int(pix / Ho);
    const int h0 = ho * sh - ph, w0 = wo * sw - pw;
    const __nv_bfloat16* base = x + int64_t(n) * H * W * C + g * 8;
    uint4 q[K * K];
#pragma unroll
    for (int a = 0; a < K; ++a)
#pragma unroll
      for (int b = 0; b < K; ++b) {
        const int hi = h0 + a, wi = w0 + b;
        const bool ok = hi >= 0 && hi < H && wi >= 0 && wi < W;
        q[a * K + b] = ok ? __ldg(reinterpret_cast<const uint4*>(base + (int64_t(hi) * W + wi) * C))
                          : make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);   // bf16 -inf
      }
    float m[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) m[j] = -INFINITY;
#pragma unroll
    for (int k = 0; k < K * K; ++k) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q[k]);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __bfloat1622float2(h[t]);
        m[2 * t] = fmaxf(m[2 * t], f.x);
        m[2 * t + 1] = fmaxf(m[2 * t + 1], f.y);
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int t = 0; t < 4; ++t) oh[t] = __floats2bfloat162_rn(m[2 * t], m[2 * t + 1]);
    *reinterpret_cast<uint4*>(y + i * 8) = o;
  }
}

// 3x3 stride-2 max pool (the ResNet stem pool), NHWC bf16, C % 8 == 0: one block per output row.
// The block first takes, for every input column its row needs, the max over the window's three input
// rows (16 bytes of channels at a time) into shared memory, then for each output pixel the max over
// three adjacent columns. Each input row is read by 1.5 blocks (instead of each pixel by 2.25
// threads). The max of bf16 values is one of them, so this equals the per-pixel kernel exactly.
__device__ __forceinline__ uint4 bf16x8_max(uint4 a, uint4 b) {
  const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&b);
  uint4 r;
  __nv_bfloat162* z = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int t = 0; t < 4; ++t) z[t] = __hmax2(x[t], y[t]);
  return r;
}
__global__ void maxpool3s2_row_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int H,
                                      int W, int C, int Ho, int Wo, int ph, int pw) {
  extern __shared__ uint4 colmax[];   // [2 * Wo + 1][C / 8]: column w - pw's max over the three rows
  const int cg = C / 8;
  const int Wv = 2 * Wo + 1;
  const int row = blockIdx.x;   // n * Ho + ho
  const int n = row / Ho, ho = row - n * Ho;
  const int h0 = 2 * ho - ph;
  const __nv_bfloat16* img = x + int64_t(n) * H * W * C;
  const uint4 ninf = make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);   // bf16 -inf
  for (int i = threadIdx.x; i < Wv * cg; i += blockDim.x) {
    const int wi = i / cg, g = i - wi * cg;
    const int w = wi - pw;
    uint4 m = ninf;
    if (w >= 0 && w < W) {
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        const int h = h0 + a;
        if (h >= 0 && h < H)
          m = bf16x8_max(m, __ldg(reinterpret_cast<const uint4*>(img + (int64_t(h) * W + w) * C + g * 8)));
      }
    }
    colmax[i] = m;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < Wo * cg; i += blockDim.x) {
    const int wo = i / cg, g = i - wo * cg;
    const uint4 m = bf16x8_max(bf16x8_max(colmax[(2 * wo) * cg + g], colmax[(2 * wo + 1) * cg + g]),
                               colmax[(2 * wo + 2) * cg + g]);
    *reinterpret_cast<uint4*>(y + (int64_t(row) * Wo + wo) * C + g * 8) = m;
  }
}

// Scalar fallback when C is not a multiple of 8.
__global__ void maxpool_nhwc_scalar_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int N,
                                           int H, int W, int C, int Ho, int Wo, int kh, int kw, int sh, int sw, int ph,
                                           int pw, int dh, int dw) {
  const int64_t total = int64_t(N) * Ho * Wo * C;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int c = int(i % C);
    int64_t pix = i / C;
    const int wo = int(pix % Wo);
    pix /= Wo;
    const int ho = int(pix % Ho);
    const int n = int(pix / Ho);
    float m = -INFINITY;
    for (int a = 0; a < kh; ++a) {
      const int hi = ho * sh - ph + a * dh;
      if (hi < 0 || hi >= H) continue;
      for (int b = 0; b < kw; ++b) {
        const int wi = wo * sw - pw + b * dw;
        if (wi < 0 || wi >= W) continue;
        m = fmaxf(m, __bfloat162float(x[((int64_t(n) * H + hi) * W + wi) * C + c]));
      }
    }
    y[i] = __float2bfloat16_rn(m);
  }
}

// ---- global average / max pool over NHWC -------------------------------------------------------
// One block per (image, slab of G x V channels): thread t owns channel group g = t % G (V channels,
// one 128-bit load per pixel) and the pixels p = t / G (mod 256 / G). Each warp's lanes that share a
// channel group are combined with shuffles (lane bits above log2 G), then the block's warps through
// shared memory. A warp's loads of one pixel are G consecutive 16-byte chunks (coalesced).
template <bool BF16>
__global__ void global_pool_vec_kernel(const void* __restrict__ x, int HW, int C, int64_t ldp, void* __restrict__ y,
                                       int y_bf16, int is_max, int G) {
  constexpr int V = BF16 ? 8 : 4;   // channels per 16-byte load
  __shared__ float part[kThreads / 32][32][V];
  const int slabs = (C / V + G - 1) / G;
  const int n = blockIdx.x / slabs, slab = blockIdx.x - n * slabs;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int g = t % G, pslot = t / G, P = kThreads / G;
  const int cg = slab * G + g;   // channel group
  const bool valid = cg < C / V;
  float acc[V];
#pragma unroll
  for (int j = 0; j < V; ++j) acc[j] = is_max ? -INFINITY : 0.f;
  if (valid) {
    const uint8_t* base = reinterpret_cast<const uint8_t*>(x) + (int64_t(n) * HW * ldp + int64_t(cg) * V) * (BF16 ? 2 : 4);
    for (int p = pslot; p < HW; p += P) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(base + int64_t(p) * ldp * (BF16 ? 2 : 4)));
      float v[V];
      if (BF16) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
        for (int j = 0; j < V / 2; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          v[2 * j] = f.x;
          v[2 * j + 1] = f.y;
        }
      } else {
        v[0] = __uint_as_float(q.x);
        v[1] = __uint_as_float(q.y);
        v[2] = __uint_as_float(q.z);
        v[3] = __uint_as_float(q.w);
      }
#pragma unroll
      for (int j = 0; j < V; ++j) acc[j] = is_max ? fmaxf(acc[j], v[j]) : acc[j] + v[j];
    }
  }
  // lanes of one warp with the same channel group differ in the lane bits above log2(G)
  for (int sft = G; sft < 32; sft <<= 1)
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float o = __shfl_xor_sync(0xffffffffu, acc[j], sft);
      acc[j] = is_max ? fmaxf(acc[j], o) : acc[j] + o;
    }
  // (G is a power of two up to 32, so lane l of every warp holds group l % G: after the shuffles
  // lanes 0..G-1 hold the warp's partial result of groups 0..G-1)
  if (lane < G)
#pragma unroll
    for (int j = 0; j < V; ++j) part[warp][lane][j] = acc[j];
  __syncthreads();
  if (t < G && valid) {
    float r[V];
#pragma unroll
    for (int j = 0; j < V; ++j) r[j] = is_max ? -INFINITY : 0.f;
    for (int w = 0; w < kThreads / 32; ++w)
#pragma unroll
      for (int j = 0; j < V; ++j) r[j] = is_max ? fmaxf(r[j], part[w][t][j]) : r[j] + part[w][t][j];
    const int64_t o = int64_t(n) * C + int64_t(cg) * V;
#pragma unroll
    for (int j = 0; j < V; ++j) st_any(y, y_bf16, o + j, is_max ? r[j] : r[j] / float(HW));
  }
}

// Scalar global pool (channel counts or pitches without 16-byte alignment): one thread per (n, c).
__global__ void global_pool_kernel(const void* __restrict__ x, int x_bf16, int N, int HW, int C, int64_t ldp,
                                   void* __restrict__ y, int y_bf16, int is_max) {
  const int64_t total = int64_t(N) * C;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int n = int(i / C), c = int(i - int64_t(i / C) * C);
    const int64_t base = int64_t(n) * HW * ldp + c;
    float acc = is_max ? -INFINITY : 0.f;
    for (int p = 0; p < HW; ++p) {
      const float v = ld_any(x, x_bf16, base + int64_t(p) * ldp);
      acc = is_max ? fmaxf(acc, v) : acc + v;
    }
    st_any(y, y_bf16, i, is_max ? acc : acc / float(HW));
  }
}

__global__ void strided_copy_kernel(const void* __restrict__ src, int src_bf16, TDesc sd, void* __restrict__ dst,
                                    int dst_bf16, TDesc dd, int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x)
    st_any(dst, dst_bf16, offset_of(i, dd), ld_any(src, src_bf16, offset_of(i, sd)));
}

__global__ void f16_to_f32_kernel(const uint4* __restrict__ src, float4* __restrict__ dst, int64_t n8,
                                  const __half* __restrict__ tail_src, float* __restrict__ tail_dst, int tail) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const uint4 q = __ldg(src + i);
    const __half2* h = reinterpret_cast<const __half2*>(&q);
    const float2 a = __half22float2(h[0]), b = __half22float2(h[1]), c = __half22float2(h[2]), d = __half22float2(h[3]);
    dst[2 * i] = make_float4(a.x, a.y, b.x, b.y);
    dst[2 * i + 1] = make_float4(c.x, c.y, d.x, d.y);
  }
  if (blockIdx.x == 0 && int(threadIdx.x) < tail) tail_dst[threadIdx.x] = __half2float(tail_src[threadIdx.x]);
}

__global__ void bf16_to_f32_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t n8,
                                   const uint16_t* __restrict__ tail_src, uint32_t* __restrict__ tail_dst, int tail) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const uint4 q = __ldg(src + i);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {   // bfloat16 bits are the high half of the float32 bits
      f[2 * j] = w[j] << 16;
      f[2 * j + 1] = w[j] & 0xFFFF0000u;
    }
    dst[2 * i] = make_uint4(f[0], f[1], f[2], f[3]);
    dst[2 * i + 1] = make_uint4(f[4], f[5], f[6], f[7]);
  }
  if (blockIdx.x == 0 && int(threadIdx.x) < tail) tail_dst[threadIdx.x] = uint32_t(tail_src[threadIdx.x]) << 16;
}

__global__ void fill_kernel(float* dst, int64_t n, float v) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = v;
}

__device__ __forceinline__ float ew_apply(int op, float a, float b, float alpha, float beta) {
  switch (op) {
    case EW_ADD: return a + b;
    case EW_SUB: return a - b;
    case EW_MUL: return a * b;
    case EW_DIV: return a / b;
    case EW_POW: return powf(a, b);
    case EW_MAX: return fmaxf(a, b);
    case EW_MIN: return fminf(a, b);
    case EW_RELU: return a > 0.f ? a : 0.f;
    case EW_SIGMOID: return 1.f / (1.f + expf(-a));
    case EW_TANH: return tanhf(a);
    case EW_SQRT: return sqrtf(a);
    case EW_NEG: return -a;
    case EW_ABS: return fabsf(a);
    case EW_EXP: return expf(a);
    case EW_LOG: return logf(a);
    case EW_RECIP: return 1.f / a;
    case EW_FLOOR: return floorf(a);
    case EW_CEIL: return ceilf(a);
    case EW_ERF: return erff(a);
    case EW_LEAKY: return a >= 0.f ? a : alpha * a;
    case EW_CLIP: return fminf(fmaxf(a, alpha), beta);
    // GELU (Hendrycks & Gimpel): x Phi(x) with the error function, or its tanh approximation
    case EW_GELU: return 0.5f * a * (1.f + erff(a * 0.70710678118654752f));
    case EW_GELU_TANH: return 0.5f * a * (1.f + tanhf(0.79788456080286536f * (a + 0.044715f * a * a * a)));
    default: return a;
  }
}

__global__ void elementwise_kernel(int op, const void* __restrict__ a, int a_bf16, TDesc ad, const void* __restrict__ b,
                                   int b_bf16, TDesc bd, void* __restrict__ y, int y_bf16, TDesc yd, float alpha,
                                   float beta, int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const float va = ld_any(a, a_bf16, offset_of(i, ad));
    const float vb = b ? ld_any(b, b_bf16, offset_of(i, bd)) : 0.f;
    st_any(y, y_bf16, offset_of(i, yd), ew_apply(op, va, vb, alpha, beta));
  }
}

// Four consecutive elements of the innermost dimension per thread (the dimensions having been
// collapsed on the host so that the innermost one is as long as possible): the outer index is
// divided out once per four elements, and an operand whose innermost stride is 1 is read / written
// with one 16-byte (fp32) or 8-byte (bf16) access; stride 0 (a broadcast operand) is one load.
// L % 4 == 0 and every unit-stride operand is aligned for its vector access.
struct Vec4Op {
  const void* p;
  int bf16;
  int64_t s_in;   // innermost stride (0, 1 or other)
  TDesc outer;    // the outer dimensions
};
__device__ __forceinline__ void vload4(const Vec4Op& o, int64_t off, float (&v)[4]) {
  if (o.s_in == 1) {
    if (o.bf16) {
      const uint2 q = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(o.p) + off));
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
      const float4 q = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(o.p) + off));
      v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    }
  } else if (o.s_in == 0) {
    v[0] = v[1] = v[2] = v[3] = ld_any(o.p, o.bf16, off);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = ld_any(o.p, o.bf16, off + j * o.s_in);
  }
}
__global__ void elementwise_vec4_kernel(int op, Vec4Op a, Vec4Op b, void* __restrict__ y, int y_bf16, int64_t ys_in,
                                        TDesc youter, int64_t L, float alpha, float beta, int64_t nvec) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < nvec; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i * 4;
    const int64_t outer = e / L, in = e - outer * L;
    float va[4], vb[4] = {0.f, 0.f, 0.f, 0.f};
    vload4(a, offset_of(outer, a.outer) + in * a.s_in, va);
    if (b.p) vload4(b, offset_of(outer, b.outer) + in * b.s_in, vb);
    float r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = op < 0 ? va[j] : ew_apply(op, va[j], vb[j], alpha, beta);
    const int64_t yo = offset_of(outer, youter) + in * ys_in;
    if (ys_in == 1 && !y_bf16) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + yo) = make_float4(r[0], r[1], r[2], r[3]);
    } else if (ys_in == 1) {
      uint2 q;
      *reinterpret_cast<__nv_bfloat162*>(&q.x) = __floats2bfloat162_rn(r[0], r[1]);
      *reinterpret_cast<__nv_bfloat162*>(&q.y) = __floats2bfloat162_rn(r[2], r[3]);
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(y) + yo) = q;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) st_any(y, y_bf16, yo + j * ys_in, r[j]);
    }
  }
}

// One warp per softmax row; rows are (outer, inner) pairs, elements `inner` apart.
__global__ void softmax_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t outer, int64_t len,
                               int64_t inner) {
  const int64_t rows = outer * inner;
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; r < rows;
       r += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const int64_t o = r / inner, in = r - o * inner;
    const float* xp = x + o * len * inner + in;
    float* yp = y + o * len * inner + in;
    float m = -INFINITY;
    for (int64_t l = lane; l < len; l += 32) m = fmaxf(m, xp[l * inner]);
#pragma unroll
    for (int s = 16; s; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
    float sum = 0.f;
    for (int64_t l = lane; l < len; l += 32) sum += expf(xp[l * inner] - m);
#pragma unroll
    for (int s = 16; s; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
    const float inv = 1.f / sum;
    for (int64_t l = lane; l < len; l += 32) yp[l * inner] = expf(xp[l * inner] - m) * inv;
  }
}

__global__ void reduce_mid_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t outer, int64_t len,
                                  int64_t inner, int kind) {
  const int64_t total = outer * inner;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t o = i / inner, in = i - o * inner;
    const float* xp = x + o * len * inner + in;
    float acc = kind == 2 ? -INFINITY : 0.f;
    for (int64_t l = 0; l < len; ++l) acc = kind == 2 ? fmaxf(acc, xp[l * inner]) : acc + xp[l * inner];
    y[i] = kind == 1 ? acc / float(len) : acc;
  }
}

__global__ void gather_axes_kernel(const void* __restrict__ x, int x_bf16, TDesc xd, const int64_t* __restrict__ tables,
                                   void* __restrict__ y, int y_bf16, TDesc yd, int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t lin = i, off = 0, tab = 0;
    int64_t tab_off[kMaxRank];
    for (int d = 0; d < yd.rank; ++d) {
      tab_off[d] = tab;
      tab += yd.shape[d];
    }
    for (int d = yd.rank - 1; d >= 0; --d) {
      const int64_t q = lin / yd.shape[d];
      const int64_t idx = lin - q * yd.shape[d];
      off += tables[tab_off[d] + idx] * xd.stride[d];
      lin = q;
    }
    st_any(y, y_bf16, offset_of(i, yd), ld_any(x, x_bf16, off));
  }
}

}  // namespace

cudaError_t to_nhwc_bf16(const void* src, int src_bf16, const int64_t* sh, const int64_t* st, void* dst, int Cp,
                         cudaStream_t s) {
  const int64_t total = sh[0] * sh[2] * sh[3] * (Cp / 4);
  to_nhwc_bf16_kernel<<<grid_for(total), kThreads, 0, s>>>(src, src_bf16, sh[0], sh[1], sh[2], sh[3], st[0], st[1],
                                                           st[2], st[3], reinterpret_cast<__nv_bfloat16*>(dst), Cp);
  return cudaGetLastError();
}

cudaError_t to_nhwc_f32(const void* src, int src_bf16, const int64_t* sh, const int64_t* st, void* dst, int Cp,
                        int round_tf32, cudaStream_t s) {
  if (Cp % 4) return cudaErrorInvalidValue;
  const int64_t total = sh[0] * sh[2] * sh[3] * (Cp / 4);
  to_nhwc_f32_kernel<<<grid_for(total), kThreads, 0, s>>>(src, src_bf16, sh[0], sh[1], sh[2], sh[3], st[0], st[1], st[2],
                                                          st[3], reinterpret_cast<float*>(dst), Cp, round_tf32);
  return cudaGetLastError();
}

cudaError_t to_rows_f32(const void* src, int src_bf16, int64_t M, int64_t K, int64_t sm, int64_t sk, void* dst,
                        int64_t Kp, int round_tf32, cudaStream_t s) {
  to_rows_f32_kernel<<<grid_for(M * Kp), kThreads, 0, s>>>(src, src_bf16, M, K, sm, sk, reinterpret_cast<float*>(dst), Kp,
                                                           round_tf32);
  return cudaGetLastError();
}

cudaError_t maxpool_nhwc_f32(const void* x, void* y, int N, int H, int W, int C, int Ho, int Wo, int kh, int kw, int sh,
                             int sw, int ph, int pw, int dh, int dw, cudaStream_t s) {
  if (C % 4) return cudaErrorInvalidValue;
  maxpool_nhwc_f32_kernel<<<grid_for(int64_t(N) * Ho * Wo * (C / 4)), kThreads, 0, s>>>(
      reinterpret_cast<const float*>(x), reinterpret_cast<float*>(y), N, H, W, C, Ho, Wo, kh, kw, sh, sw, ph, pw, dh, dw);
  return cudaGetLastError();
}

cudaError_t to_s2d_bf16(const void* src, int src_bf16, const int64_t* sh, const int64_t* st, void* dst, int64_t Hs,
                        int64_t Ws, cudaStream_t s) {
  if (sh[1] > 4) return cudaErrorInvalidValue;
  const bool packed = !src_bf16 && st[3] == 1 && st[2] == sh[3] && st[1] == sh[2] * sh[3] &&
                      st[0] == sh[1] * sh[2] * sh[3] && sh[3] % 2 == 0 && 2 * Ws == sh[3] && 2 * Hs >= sh[2] &&
                      2 * Hs <= sh[2] + 1 && (reinterpret_cast<uintptr_t>(src) & 7) == 0;
  if (packed) {
    const float* f = reinterpret_cast<const float*>(src);
    auto d = reinterpret_cast<__nv_bfloat16*>(dst);
    const auto g = grid_for(sh[0] * Hs * Ws);
    switch (sh[1]) {
      case 1: to_s2d_bf16_f32_kernel<1><<<g, kThreads, 0, s>>>(f, sh[0], sh[2], sh[3], d, Hs, Ws); break;
      case 2: to_s2d_bf16_f32_kernel<2><<<g, kThreads, 0, s>>>(f, sh[0], sh[2], sh[3], d, Hs, Ws); break;
      case 3: to_s2d_bf16_f32_kernel<3><<<g, kThreads, 0, s>>>(f, sh[0], sh[2], sh[3], d, Hs, Ws); break;
      default: to_s2d_bf16_f32_kernel<4><<<g, kThreads, 0, s>>>(f, sh[0], sh[2], sh[3], d, Hs, Ws); break;
    }
    return cudaGetLastError();
  }
  to_s2d_bf16_kernel<<<grid_for(sh[0] * Hs * Ws), kThreads, 0, s>>>(src, src_bf16, sh[0], sh[1], sh[2], sh[3], st[0],
                                                                    st[1], st[2], st[3],
                                                                    reinterpret_cast<__nv_bfloat16*>(dst), Hs, Ws);
  return cudaGetLastError();
}

cudaError_t to_rows_bf16(const void* src, int src_bf16, int64_t M, int64_t K, int64_t sm, int64_t sk, void* dst,
                         int64_t Kp, cudaStream_t s) {
  to_rows_bf16_kernel<<<grid_for(M * Kp), kThreads, 0, s>>>(src, src_bf16, M, K, sm, sk,
                                                            reinterpret_cast<__nv_bfloat16*>(dst), Kp);
  return cudaGetLastError();
}

cudaError_t maxpool_nhwc_bf16(const void* x, void* y, int N, int H, int W, int C, int Ho, int Wo, int kh, int kw, int sh,
                              int sw, int ph, int pw, int dh, int dw, cudaStream_t s) {
  auto xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto yb = reinterpret_cast<__nv_bfloat16*>(y);
  const size_t row_smem = size_t(2 * Wo + 1) * (C / 8) * 16;
  if (C % 8 == 0 && kh == 3 && kw == 3 && sh == 2 && sw == 2 && dh == 1 && dw == 1 && row_smem <= 48 * 1024) {
    maxpool3s2_row_kernel<<<int64_t(N) * Ho, 256, row_smem, s>>>(xb, yb, H, W, C, Ho, Wo, ph, pw);
  } else if (C % 8 == 0 && kh == 3 && kw == 3 && dh == 1 && dw == 1) {
    maxpool_k_nhwc_kernel<3><<<grid_for(int64_t(N) * Ho * Wo * (C / 8)), kThreads, 0, s>>>(xb, yb, N, H, W, C, Ho, Wo,
                                                                                           sh, sw, ph, pw);
  } else if (C % 8 == 0) {
    maxpool_nhwc_kernel<<<grid_for(int64_t(N) * Ho * Wo * (C / 8)), kThreads, 0, s>>>(xb, yb, N, H, W, C, Ho, Wo, kh, kw,
                                                                                      sh, sw, ph, pw, dh, dw);
  } else {
    maxpool_nhwc_scalar_kernel<<<grid_for(int64_t(N) * Ho * Wo * C), kThreads, 0, s>>>(xb, yb, N, H, W, C, Ho, Wo, kh,
                                                                                       kw, sh, sw, ph, pw, dh, dw);
  }
  return cudaGetLastError();
}

cudaError_t global_pool_nhwc(const void* x, int x_bf16, int N, int HW, int C, int64_t ldp, void* y, int y_bf16,
                             int is_max, cudaStream_t s) {
  const int V = x_bf16 ? 8 : 4;
  if (C % V == 0 && ldp % V == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && HW > 0) {
    // channel groups per block: all of them up to 32, else 32 (a warp covers 512 contiguous bytes)
    int G = 1;
    while (G < 32 && G < C / V) G <<= 1;
    const int64_t blocks = int64_t(N) * ((C / V + G - 1) / G);
    if (x_bf16)
      global_pool_vec_kernel<true><<<unsigned(blocks), kThreads, 0, s>>>(x, HW, C, ldp, y, y_bf16, is_max, G);
    else
      global_pool_vec_kernel<false><<<unsigned(blocks), kThreads, 0, s>>>(x, HW, C, ldp, y, y_bf16, is_max, G);
    return cudaGetLastError();
  }
  global_pool_kernel<<<grid_for(int64_t(N) * C), kThreads, 0, s>>>(x, x_bf16, N, HW, C, ldp, y, y_bf16, is_max);
  return cudaGetLastError();
}

namespace {

// Merges adjacent dimensions that are contiguous with respect to each other in every descriptor
// (all of the same shape) and drops unit dimensions, so the innermost dimension is as long as
// possible. Returns the rank after collapsing.
int collapse_dims(TDesc** d, int n) {
  const int rank = d[0]->rank;
  int64_t shape[kMaxRank];
  int64_t st[4][kMaxRank];
  int r = 0;
  for (int i = 0; i < rank; ++i) {
    const int64_t sz = d[0]->shape[i];
    if (sz == 1) continue;
    bool merge = r > 0;
    for (int k = 0; k < n && merge; ++k) merge = st[k][r - 1] == d[k]->stride[i] * sz;
    if (merge) {
      shape[r - 1] *= sz;
      for (int k = 0; k < n; ++k) st[k][r - 1] = d[k]->stride[i];
    } else {
      shape[r] = sz;
      for (int k = 0; k < n; ++k) st[k][r] = d[k]->stride[i];
      ++r;
    }
  }
  if (r == 0) {
    shape[0] = 1;
    for (int k = 0; k < n; ++k) st[k][0] = 1;
    r = 1;
  }
  for (int k = 0; k < n; ++k) {
    d[k]->rank = r;
    for (int i = 0; i < r; ++i) {
      d[k]->shape[i] = shape[i];
      d[k]->stride[i] = st[k][i];
    }
  }
  return r;
}

bool aligned_for(const void* p, int bf16, int64_t s_in, const TDesc& outer) {
  if (s_in != 1) return true;
  const int64_t need = 4;   // elements per vector access (8 or 16 bytes)
  if ((reinterpret_cast<uintptr_t>(p) & (bf16 ? 7 : 15)) != 0) return false;
  for (int i = 0; i < outer.rank; ++i)
    if (outer.stride[i] % need) return false;
  return true;
}

// The vectorised path when the collapsed innermost length is a multiple of 4 and the accesses are
// aligned; false to fall back to the per-element kernels.
bool launch_vec4(int op, const void* a, int a_bf16, TDesc ad, const void* b, int b_bf16, TDesc bd, void* y,
                 int y_bf16, TDesc yd, float alpha, float beta, cudaStream_t s) {
  TDesc* ds[3] = {&yd, &ad, &bd};
  const int r = collapse_dims(ds, b ? 3 : 2);
  const int64_t L = yd.shape[r - 1];
  if (L % 4 != 0) return false;
  auto outer_of = [&](const TDesc& d) {
    TDesc o{};
    o.rank = r - 1;
    for (int i = 0; i < r - 1; ++i) {
      o.shape[i] = d.shape[i];
      o.stride[i] = d.stride[i];
    }
    if (o.rank == 0) {   // a single row
      o.rank = 1;
      o.shape[0] = 1;
      o.stride[0] = 0;
    }
    return o;
  };
  Vec4Op va{a, a_bf16, ad.stride[r - 1], outer_of(ad)};
  Vec4Op vb{b, b_bf16, b ? bd.stride[r - 1] : 0, b ? outer_of(bd) : TDesc{}};
  const TDesc yo = outer_of(yd);
  const int64_t ys = yd.stride[r - 1];
  if (!aligned_for(a, a_bf16, va.s_in, va.outer) || (b && !aligned_for(b, b_bf16, vb.s_in, vb.outer)) ||
      !aligned_for(y, y_bf16, ys, yo))
    return false;
  int64_t total = 1;
  for (int i = 0; i < r; ++i) total *= yd.shape[i];
  const int64_t nvec = total / 4;
  elementwise_vec4_kernel<<<grid_for(nvec), kThreads, 0, s>>>(op, va, vb, y, y_bf16, ys, yo, L, alpha, beta, nvec);
  return true;
}

}  // namespace

cudaError_t strided_copy(const void* src, int src_bf16, const TDesc& sd, void* dst, int dst_bf16, const TDesc& dd,
                         cudaStream_t s) {
  int64_t total = 1;
  for (int i = 0; i < dd.rank; ++i) total *= dd.shape[i];
  if (total == 0) return cudaSuccess;
  if (launch_vec4(-1, src, src_bf16, sd, nullptr, 0, TDesc{}, dst, dst_bf16, dd, 0.f, 0.f, s))
    return cudaGetLastError();
  strided_copy_kernel<<<grid_for(total), kThreads, 0, s>>>(src, src_bf16, sd, dst, dst_bf16, dd, total);
  return cudaGetLastError();
}

cudaError_t f16_to_f32(const void* src, void* dst, int64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int64_t n8 = n / 8;
  const int tail = int(n - n8 * 8);
  f16_to_f32_kernel<<<grid_for(std::max<int64_t>(n8, 1)), kThreads, 0, s>>>(
      reinterpret_cast<const uint4*>(src), reinterpret_cast<float4*>(dst), n8,
      reinterpret_cast<const __half*>(src) + n8 * 8, reinterpret_cast<float*>(dst) + n8 * 8, tail);
  return cudaGetLastError();
}

cudaError_t bf16_to_f32(const void* src, void* dst, int64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int64_t n8 = n / 8;
  const int tail = int(n - n8 * 8);
  bf16_to_f32_kernel<<<grid_for(std::max<int64_t>(n8, 1)), kThreads, 0, s>>>(
      reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), n8,
      reinterpret_cast<const uint16_t*>(src) + n8 * 8, reinterpret_cast<uint32_t*>(dst) + n8 * 8, tail);
  return cudaGetLastError();
}

cudaError_t fill_f32(void* dst, int64_t n, float v, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  fill_kernel<<<grid_for(n), kThreads, 0, s>>>(reinterpret_cast<float*>(dst), n, v);
  return cudaGetLastError();
}

cudaError_t elementwise(int op, const void* a, int a_bf16, const TDesc& ad, const void* b, int b_bf16, const TDesc& bd,
                        void* y, int y_bf16, const TDesc& yd, float alpha, float beta, cudaStream_t s) {
  int64_t total = 1;
  for (int i = 0; i < yd.rank; ++i) total *= yd.shape[i];
  if (total == 0) return cudaSuccess;
  if (launch_vec4(op, a, a_bf16, ad, b, b_bf16, bd, y, y_bf16, yd, alpha, beta, s)) return cudaGetLastError();
  elementwise_kernel<<<grid_for(total), kThreads, 0, s>>>(op, a, a_bf16, ad, b, b_bf16, bd, y, y_bf16, yd, alpha, beta,
                                                          total);
  return cudaGetLastError();
}

cudaError_t softmax(const float* x, float* y, int64_t outer, int64_t len, int64_t inner, cudaStream_t s) {
  const int64_t rows = outer * inner;
  if (rows == 0) return cudaSuccess;
  softmax_kernel<<<grid_for(rows * 32), kThreads, 0, s>>>(x, y, outer, len, inner);
  return cudaGetLastError();
}

cudaError_t reduce_mid(const float* x, float* y, int64_t outer, int64_t len, int64_t inner, int kind, cudaStream_t s) {
  if (outer * inner == 0) return cudaSuccess;
  reduce_mid_kernel<<<grid_for(outer * inner), kThreads, 0, s>>>(x, y, outer, len, inner, kind);
  return cudaGetLastError();
}

cudaError_t gather_axes(const void* x, int x_bf16, const TDesc& xd, const int64_t* tables, void* y, int y_bf16,
                        const TDesc& yd, cudaStream_t s) {
  int64_t total = 1;
  for (int i = 0; i < yd.rank; ++i) total *= yd.shape[i];
  if (total == 0) return cudaSuccess;
  gather_axes_kernel<<<grid_for(total), kThreads, 0, s>>>(x, x_bf16, xd, tables, y, y_bf16, yd, total);
  return cudaGetLastError();
}

}  // namespace k
}  // namespace sb
