// Fused scaled dot-product attention on the tcgen05 tensor core (ViTAttention,
// samples/RetinaNet/ViTNet.cs:155-207): y = softmax(scale * q k^T) v per (batch, head), for
// sequences of up to 256 keys and 64-wide heads (ViT-Ti / S / B at 224x224: 197 tokens).
//
// One CTA per (128-query tile, head, batch), 256 threads:
//   1. all threads stage Q [128 x 64], K [256 x 64] and V^T [64 x 256] as bf16 in shared memory in
//      the 128-byte-swizzled K-major layout (q, k, v are strided views of the QKV projection, read
//      with 16-byte loads; V is transposed while staged; rows past the sequence are zero);
//   2. one thread issues S = Q K^T: four tcgen05.mma kind::f16 (M=128, N=256, K=16) into TMEM
//      columns 0-255;
//   3. warps 0-3 (one query row per thread, its TMEM lane) take the row maximum over the valid
//      keys, P = exp(scale (s - max)) rounded to bf16 into shared memory as the next MMA's A
//      operand, and the row sum of the rounded P;
//   4. one thread issues O = P V: sixteen MMAs (M=128, N=64, K=16) into TMEM columns 256-319;
//   5. warps 0-3 divide each row of O by its sum and store it as bf16, fp32 on the TF32 grid or
//      fp32, at out[b, s, h, :] (the [B, S, H, hd] order the following Transpose + Reshape read as
//      a plain row matrix).
// Operands are bf16 in every session precision: checked with the oracle on ViT-B/16, bf16 attention
// operands inside a TF32 session land 6.7e-4 from fp32 (TF32 gate 2e-3).
// Waits on the MMA completions are bounded (global timer); a timeout sets the device error word.
#include <cuda_bf16.h>

#include <atomic>
#include <stdexcept>
#include <string>

#include "kernels.h"
#include "tcgen05.cuh"

namespace sb {
namespace k {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kAttnQ = 128;        // query rows per CTA (TMEM lanes)
constexpr int kAttnKeys = 256;     // keys per CTA (S accumulator columns)
constexpr int kAttnHd = 64;        // head width: one 128-byte k-block of bf16
constexpr uint32_t kSmQ = kAttnQ * 128;                  // 16 KB
constexpr uint32_t kSmK = kAttnKeys * 128;               // 32 KB
constexpr uint32_t kSmVt = (kAttnKeys / 64) * 64 * 128;  // 32 KB: 4 k-blocks of 64 keys x 64 rows
constexpr uint32_t kSmP = (kAttnKeys / 64) * kAttnQ * 128;   // 64 KB: 4 k-blocks x 128 rows
constexpr uint32_t kAttnSmem = kSmQ + kSmK + kSmVt + kSmP + 1024 + 64;

// byte offset of 16-byte chunk `c` (0-7) of row `r` in a K-major 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128_off(int r, int c) { return uint32_t(r) * 128u + (uint32_t(c ^ (r & 7)) << 4); }

// 8 consecutive elements (bf16 or fp32) at element offset `off`, as bf16
__device__ __forceinline__ uint4 load8_bf16(const void* p, int f32, int64_t off) {
  if (!f32) return *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p) + off);
  const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + off);
  const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + off + 4);
  uint4 q;
  __nv_bfloat162 h;
  h = __floats2bfloat162_rn(a.x, a.y);
  q.x = *reinterpret_cast<uint32_t*>(&h);
  h = __floats2bfloat162_rn(a.z, a.w);
  q.y = *reinterpret_cast<uint32_t*>(&h);
  h = __floats2bfloat162_rn(b.x, b.y);
  q.z = *reinterpret_cast<uint32_t*>(&h);
  h = __floats2bfloat162_rn(b.z, b.w);
  q.w = *reinterpret_cast<uint32_t*>(&h);
  return q;
}

__device__ __forceinline__ float tf32_rna_a(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__global__ void __launch_bounds__(kAttnThreads, 1) attention_kernel(const AttentionArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kSmQ;
  uint8_t* sVt = sK + kSmK;
  uint8_t* sP = sVt + kSmVt;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kSmP);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = blockIdx.x * kAttnQ, h = blockIdx.y, b = blockIdx.z;
  const int S = a.S;

  if (tid == 0) {
    mbar_init(&bars[0], 1u);
    mbar_init(&bars[1], 1u);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(tmem_holder, 512);

  // ---- 1. operands into shared memory ----
  const int64_t qb = int64_t(b) * a.qs[0] + int64_t(h) * a.qs[1];
  const int64_t kb = int64_t(b) * a.ks[0] + int64_t(h) * a.ks[1];
  const int64_t vb = int64_t(b) * a.vs[0] + int64_t(h) * a.vs[1];
  for (int i = tid; i < kAttnQ * 8; i += kAttnThreads) {
    const int r = i >> 3, c = i & 7, s = q0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (s < S) v = load8_bf16(a.q, a.in_f32, qb + int64_t(s) * a.qs[2] + c * 8);
    *reinterpret_cast<uint4*>(sQ + sw128_off(r, c)) = v;
  }
  for (int i = tid; i < kAttnKeys * 8; i += kAttnThreads) {
    const int r = i >> 3, c = i & 7;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < S) v = load8_bf16(a.k, a.in_f32, kb + int64_t(r) * a.ks[2] + c * 8);
    *reinterpret_cast<uint4*>(sK + sw128_off(r, c)) = v;
  }
  for (int i = tid; i < kAttnKeys * 8; i += kAttnThreads) {
    const int j = i >> 3, c = i & 7;   // key j, dims 8c .. 8c+7
    uint4 v = make_uint4(0, 0, 0, 0);
    if (j < S) v = load8_bf16(a.v, a.in_f32, vb + int64_t(j) * a.vs[2] + c * 8);
    const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
    const int kblk = j >> 6, jj = j & 63;
    uint8_t* base = sVt + kblk * (64 * 128) + (jj & 7) * 2;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int d = c * 8 + t;
      *reinterpret_cast<uint16_t*>(base + sw128_off(d, jj >> 3)) = e[t];
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // ---- 2. S = Q K^T ----
  if (tid == 0) {
    constexpr uint32_t idS = idesc_mma(kAttnQ, kAttnKeys, false);
    const uint64_t qd = sw128_desc(smem_u32(sQ)), kd = sw128_desc(smem_u32(sK));
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) umma_bf16(tmem, qd + uint64_t(kk * 2), kd + uint64_t(kk * 2), idS, kk > 0 ? 1u : 0u);
    umma_commit(&bars[0]);
  }
  // ---- 3. softmax rows (warps 0-3: TMEM lane quarter = warp) ----
  float rowsum = 1.f;
  bool ok = true;
  if (warp < 4) {
    ok = mbar_wait(&bars[0], 0u, abort_flag, a.err, 1u);
    if (ok) {
      tc_fence_after();
      const int r = warp * 32 + lane;
      const uint32_t taddr = tmem + (uint32_t(warp * 32) << 16);
      const float sl2 = a.scale * 1.4426950408889634f;   // scale * log2(e)
      float m = -INFINITY;
      uint32_t v[32];
      for (int c = 0; c < kAttnKeys / 32; ++c) {
        tmem_ld32(taddr + uint32_t(c * 32), v);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c * 32 + j < S) m = fmaxf(m, __uint_as_float(v[j]) * sl2);
      }
      float l = 0.f;
      for (int c = 0; c < kAttnKeys / 32; ++c) {
        tmem_ld32(taddr + uint32_t(c * 32), v);
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float p0 = c * 32 + j < S ? exp2f(__uint_as_float(v[j]) * sl2 - m) : 0.f;
          const float p1 = c * 32 + j + 1 < S ? exp2f(__uint_as_float(v[j + 1]) * sl2 - m) : 0.f;
          __nv_bfloat162 hp = __floats2bfloat162_rn(p0, p1);
          const float2 back = __bfloat1622float2(hp);   // the row sum of what the MMA reads
          l += back.x + back.y;
          pk[j >> 1] = *reinterpret_cast<uint32_t*>(&hp);
        }
        // columns 32c .. 32c+31: k-block c / 2, 16-byte chunks 4 (c % 2) .. +3
        uint8_t* blk = sP + (c >> 1) * (kAttnQ * 128);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(blk + sw128_off(r, (c & 1) * 4 + q)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
      rowsum = l;
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  // ---- 4. O = P V ----
  if (tid == 0 && !*abort_flag) {
    tc_fence_after();
    constexpr uint32_t idO = idesc_mma(kAttnQ, kAttnHd, false);
#pragma unroll
    for (int kb2 = 0; kb2 < kAttnKeys / 64; ++kb2) {
      const uint64_t pd = sw128_desc(smem_u32(sP + kb2 * (kAttnQ * 128)));
      const uint64_t vd = sw128_desc(smem_u32(sVt + kb2 * (64 * 128)));
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16(tmem + 256u, pd + uint64_t(kk * 2), vd + uint64_t(kk * 2), idO, (kb2 | kk) ? 1u : 0u);
    }
    umma_commit(&bars[1]);
  }
  // ---- 5. normalise and store ----
  if (warp < 4 && ok && !*abort_flag) {
    if (mbar_wait(&bars[1], 0u, abort_flag, a.err, 2u)) {
      tc_fence_after();
      const int r = warp * 32 + lane, s = q0 + r;
      const uint32_t taddr = tmem + (uint32_t(warp * 32) << 16) + 256u;
      const float inv = 1.f / rowsum;
      for (int half = 0; half < 2; ++half) {
        uint32_t v[32];
        tmem_ld32(taddr + uint32_t(half * 32), v);
        if (s < S) {
          const int64_t off = int64_t(b) * a.os[0] + int64_t(h) * a.os[1] + int64_t(s) * a.os[2] + half * 32;
          if (a.out_mode == 0) {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + off);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 hp = __floats2bfloat162_rn(__uint_as_float(v[8 * q + 2 * e]) * inv,
                                                          __uint_as_float(v[8 * q + 2 * e + 1]) * inv);
                w[e] = *reinterpret_cast<uint32_t*>(&hp);
              }
              dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float4 o;
              o.x = __uint_as_float(v[4 * q]) * inv;
              o.y = __uint_as_float(v[4 * q + 1]) * inv;
              o.z = __uint_as_float(v[4 * q + 2]) * inv;
              o.w = __uint_as_float(v[4 * q + 3]) * inv;
              if (a.out_mode == 1) {
                o.x = tf32_rna_a(o.x);
                o.y = tf32_rna_a(o.y);
                o.z = tf32_rna_a(o.z);
                o.w = tf32_rna_a(o.w);
              }
              dst[q] = o;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool attention_supported(int S, int hd) { return S >= 1 && S <= kAttnKeys && hd == kAttnHd; }

void attention_prepare() {
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (done_mask.load() & bit) return;
  cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kAttnSmem));
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaFuncSetAttribute (attention): ") + cudaGetErrorString(e));
  done_mask.fetch_or(bit);
}

cudaError_t attention(const AttentionArgs& a, int B, int H, cudaStream_t s) {
  if (!attention_supported(a.S, a.hd) || B < 1 || H < 1) return cudaErrorInvalidValue;
  const int esz = a.in_f32 ? 4 : 2;
  for (int i = 0; i < 3; ++i)
    if ((a.qs[i] * esz) % 16 || (a.ks[i] * esz) % 16 || (a.vs[i] * esz) % 16) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v) |
       reinterpret_cast<uintptr_t>(a.out)) & 15u)
    return cudaErrorInvalidValue;
  dim3 grid((a.S + kAttnQ - 1) / kAttnQ, H, B);
  attention_kernel<<<grid, kAttnThreads, kAttnSmem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace k
}  // namespace sb
