// tcgen05 / TMEM implicit-GEMM kernel for sm_100a: dense MatMul+bias(+ReLU) and Conv2d (folded
// BatchNorm, fused residual add / nearest-2x upsampled residual, ReLU or Sigmoid epilogue).
//
// Persistent, warp-specialised CTA (one per SM):
//   warp 0      TMA producer: B tiles (weights), A tiles when A is a plain row matrix, and each
//               output tile's residual into a shared-memory ring ahead of its operands
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16 per instr)
//   warps 2-9   epilogue, two warps per TMEM lane quarter: tcgen05.ld accumulator -> bias /
//               residual / activation -> swizzled smem slab -> TMA bulk store
//   warps 10-13 (gather modes only) im2col gather producers: cp.async 16B/8B with zero fill,
//               written into the 128B-swizzled K-major layout the UMMA smem descriptor expects
// Spatial convolutions whose activation channels come in 64s (or 16s) instead take the A operand
// with TMA in im2col mode: one load per k-tile brings 128 consecutive output pixels x 64
// channels of one filter tap, zero-filled outside the image, straight into the swizzled layout.
// Operand tiles are BM=128 rows x 128 bytes (64 bf16, or 32 fp32 in the TF32 accuracy mode: one
// 128-byte swizzle atom per row); the fp32 accumulator
// is double-buffered in TMEM so the epilogue of tile i overlaps the main loop of tile i+1.
// Every mbarrier wait is bounded (global timer); a timeout sets a device error word and the CTA
// drains and frees its TMEM instead of hanging.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <stdexcept>

#include "kernels.h"
#include "tcgen05.cuh"

namespace sb {
namespace k {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;   // bf16 elements per 128-byte k-tile row (32 for TF32 operands)
// fp32 rounded to the TF32 grid (nearest, ties away): activations that feed TF32 MMAs.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Activation of 32 accumulator values; the switch is outside the element loop so each case is one
// straight run. Sigmoid uses the fast reciprocal (a few ulp, far below the bf16 output rounding).
__device__ __forceinline__ void act_apply32(float (&v)[32], int act) {
  if (act == 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = v[j] > 0.f ? v[j] : 0.f;
  } else if (act == 2) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fdividef(1.f, 1.f + __expf(-v[j]));
  } else if (act == 3) {   // GELU, tanh approximation
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.5f * v[j] * (1.f + tanhf(0.79788456080286536f * (v[j] + 0.044715f * v[j] * v[j] * v[j])));
  } else if (act == 4) {   // GELU with the error function
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.5f * v[j] * (1.f + erff(v[j] * 0.70710678118654752f));
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// max(a, 0) and max(b, 0) rounded to bf16 in one conversion (a in the low half).
__device__ __forceinline__ uint32_t pack_bf16x2_relu(float a, float b) {
  uint32_t r;
  asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

// Elementwise max of two groups of 8 bf16 values.
__device__ __forceinline__ uint4 bf16x8_max(uint4 a, uint4 b) {
  const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&b);
  uint4 r;
  __nv_bfloat162* z = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int t = 0; t < 4; ++t) z[t] = __hmax2(x[t], y[t]);
  return r;
}

// Epilogue for one 32-column chunk of one accumulator row.
__device__ __forceinline__ void epilogue_chunk(const ConvGemmArgs& a, const uint32_t (&r)[32], int m, int n0) {
  float v[32];
  const float4* b4 = reinterpret_cast<const float4*>(a.bias + n0);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float4 bb = a.bias_mma ? make_float4(0.f, 0.f, 0.f, 0.f) : __ldg(b4 + j);   // (bias_mma: in the accumulator)
    v[4 * j + 0] = __uint_as_float(r[4 * j + 0]) + bb.x;
    v[4 * j + 1] = __uint_as_float(r[4 * j + 1]) + bb.y;
    v[4 * j + 2] = __uint_as_float(r[4 * j + 2]) + bb.z;
    v[4 * j + 3] = __uint_as_float(r[4 * j + 3]) + bb.w;
  }
  const int ncols = min(32, a.Cout - n0);
  if (a.res && !a.res_mma) {   // (res_mma: the MMA added it)
    int64_t rrow = m;
    if (a.res_mode == 1) {
      int hw = a.Ho * a.Wo;
      int n = m / hw, rem = m - n * hw;
      int ho = rem / a.Wo, wo = rem - ho * a.Wo;
      rrow = (int64_t(n) * a.Hr + (ho >> 1)) * a.Wr + (wo >> 1);
    }
    if (a.res_bf16) {
      const __nv_bfloat16* rp = reinterpret_cast<const __nv_bfloat16*>(a.res) + rrow * a.ldr + n0;
      if (ncols == 32 && (reinterpret_cast<uintptr_t>(rp) & 15) == 0) {
        const uint4* r4 = reinterpret_cast<const uint4*>(rp);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 q = __ldg(r4 + j);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            float2 f = __bfloat1622float2(h[t]);
            v[8 * j + 2 * t] += f.x;
            v[8 * j + 2 * t + 1] += f.y;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < ncols) v[j] += __bfloat162float(rp[j]);
      }
    } else {
      const float* rp = reinterpret_cast<const float*>(a.res) + rrow * a.ldr + n0;
      if (ncols == 32 && (reinterpret_cast<uintptr_t>(rp) & 15) == 0) {
        const float4* r4 = reinterpret_cast<const float4*>(rp);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 q = __ldg(r4 + j);
          v[4 * j] += q.x;
          v[4 * j + 1] += q.y;
          v[4 * j + 2] += q.z;
          v[4 * j + 3] += q.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < ncols) v[j] += rp[j];
      }
    }
  }
  act_apply32(v, a.act);

  int64_t orow = a.group_rows ? (int64_t(m / a.group_rows) * a.group_stride + int64_t(m % a.group_rows) * a.ldo)
                              : int64_t(m) * a.ldo;
  if (a.out_bf16) {
    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(a.out) + orow + n0;
    if (ncols == 32 && (reinterpret_cast<uintptr_t>(op) & 15) == 0) {
      uint4* o4 = reinterpret_cast<uint4*>(op);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 q;
        q.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
        q.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
        q.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
        q.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
        o4[j] = q;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) op[j] = __float2bfloat16_rn(v[j]);
    }
  } else {
    if (a.round_tf32) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = tf32_rna(v[j]);
    }
    float* op = reinterpret_cast<float*>(a.out) + orow + n0;
    if (ncols == 32 && (reinterpret_cast<uintptr_t>(op) & 15) == 0) {
      float4* o4 = reinterpret_cast<float4*>(op);
#pragma unroll
      for (int j = 0; j < 8; ++j) o4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) op[j] = v[j];
    }
  }
}

// Swizzled offset of 16-byte chunk j of row r in a 128-byte-row slab (TMA SWIZZLE_128B layout).
__device__ __forceinline__ uint32_t slab_off(int r, int j) { return uint32_t(r * 128 + ((j ^ (r & 7)) << 4)); }

constexpr int kSmemLimit = 232448;        // opt-in maximum dynamic shared memory per block
constexpr uint32_t kOutSlab = 4096;        // one 32-row x 128-byte output slab
constexpr uint32_t kBiasStage = 8 * 512;   // each epilogue warp's bias columns of the current tile
constexpr int kMaxStages = 8;
constexpr uint32_t kIdBytes = 64 * 128;   // 64x64 bf16 identity, K-major, 128-byte swizzle
constexpr uint32_t kOnesBytes = 128 * 32; // bias_mma: 128 x 16 bf16 A tile, 1.0 at k = 0 and 1, 32-byte swizzle

// 64-byte swizzled slab (32 rows of 64 bytes, the TMA SWIZZLE_64B pattern): 16-byte chunk j of row r.
__device__ __forceinline__ uint32_t slab64_off(int r, int j) { return uint32_t(r * 64 + ((j ^ ((r >> 1) & 3)) << 4)); }

// One output slab (32 rows from row0, 128 bytes of columns from n0) of one epilogue warp:
// accumulator columns [col0, col0 + SC) of the warp's TMEM lanes -> bias (SC floats staged in
// shared memory at bsl) -> residual (from the producer-filled residual slot, or direct rows) ->
// activation -> swizzled smem -> TMA store. With half >= 0 (bf16 output only) the warp does only
// the slab's 32-column half `half` (bias at bsl[0..32)), laid out as a 64-byte swizzled slab and
// stored through a 32x32 box.
template <bool OBF>
__device__ __forceinline__ void epilogue_slab(const ConvGemmArgs& a, const CUtensorMap* tmOut, uint32_t tbase,
                                              int col0, int row0, int n0, uint8_t* sb, const uint8_t* rslab,
                                              const float* bsl, int wait_mode, int parts, int pstride,
                                              int half = -1) {
  constexpr int SC = OBF ? 64 : 32;
  constexpr int EPC = OBF ? 8 : 4;
  constexpr int CH = 32 / EPC;   // 16-byte chunks per 32 columns
  const int lane = threadIdx.x & 31;
  const int m = row0 + lane;
  const int rrow = (row0 & (BM - 1)) + lane;   // row inside the 128-row residual slab
  if (lane == 0 && wait_mode == 1) bulk_wait_read0();   // the last store from this slab has been read
  __syncwarp();
  const int h_begin = half >= 0 ? half : 0;
  const int h_end = half >= 0 ? half + 1 : SC / 32;
  // bias, residual, activation, bf16 / fp32 conversion and the swizzled slab store of half h
  auto finish_half = [&](int h, float(&v)[32]) {
    if (!a.bias_mma) {   // (bias_mma: the accumulator started at the bias)
      const float4* b4 = reinterpret_cast<const float4*>(bsl + (h - h_begin) * 32);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 bb = b4[j];
        add_pair(v, 4 * j, bb.x, bb.y);
        add_pair(v, 4 * j + 2, bb.z, bb.w);
      }
    }
    if (a.res && !a.res_mma) {   // (res_mma: the MMA added it)
      if (rslab) {
#pragma unroll
        for (int j = 0; j < CH; ++j) {
          const uint4 qv = *reinterpret_cast<const uint4*>(rslab + slab_off(rrow, h * CH + j));
          if (OBF) {
            const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&qv);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const float2 f = __bfloat1622float2(hh[t]);
              add_pair(v, 8 * j + 2 * t, f.x, f.y);
            }
          } else {
            add_pair(v, 4 * j, __uint_as_float(qv.x), __uint_as_float(qv.y));
            add_pair(v, 4 * j + 2, __uint_as_float(qv.z), __uint_as_float(qv.w));
          }
        }
      } else if (m < a.M) {
        const int c0 = n0 + h * 32;
        const int ncols = max(0, min(32, a.Cout - c0));
        int64_t rr = m;
        if (a.res_mode == 1) {
          const int hw = a.Ho * a.Wo;
          const int n = m / hw, rem = m - n * hw;
          const int ho = rem / a.Wo, wo = rem - ho * a.Wo;
          rr = (int64_t(n) * a.Hr + (ho >> 1)) * a.Wr + (wo >> 1);
        }
        if (a.res_bf16) {
          const __nv_bfloat16* rp = reinterpret_cast<const __nv_bfloat16*>(a.res) + rr * a.ldr + c0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < ncols) v[j] += __bfloat162float(rp[j]);
        } else {
          const float* rp = reinterpret_cast<const float*>(a.res) + rr * a.ldr + c0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < ncols) v[j] += rp[j];
        }
      }
    }
    // bf16 output folds ReLU into the conversion
    const bool relu_pack = OBF && a.act == 1;
    if (!relu_pack) act_apply32(v, a.act);
    if (!OBF && a.round_tf32) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = tf32_rna(v[j]);
    }
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      uint4 qv;
      if (OBF && relu_pack) {
        qv.x = pack_bf16x2_relu(v[8 * j + 0], v[8 * j + 1]);
        qv.y = pack_bf16x2_relu(v[8 * j + 2], v[8 * j + 3]);
        qv.z = pack_bf16x2_relu(v[8 * j + 4], v[8 * j + 5]);
        qv.w = pack_bf16x2_relu(v[8 * j + 6], v[8 * j + 7]);
      } else if (OBF) {
        qv.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
        qv.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
        qv.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
        qv.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
      } else {
        qv = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]), __float_as_uint(v[4 * j + 2]),
                        __float_as_uint(v[4 * j + 3]));
      }
      *reinterpret_cast<uint4*>(sb + (half >= 0 ? slab64_off(lane, j) : slab_off(lane, h * CH + j))) = qv;
    }
  };
#pragma unroll
  for (int h = h_begin; h < h_end; ++h) {   // unrolled: the halves' independent work interleaves
    float v[32];
    tmem_ld_sum(tbase + uint32_t(col0 + h * 32), parts, pstride, v);
    finish_half(h, v);
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmOut, n0 + h_begin * 32 * (half >= 0), row0, sb);
    bulk_commit();
  }
}

// MODE is a ConvAMode: 0 A rows via TMA; 1 / 2 im2col gather by cp.async in 16 / 8-byte units;
// 3 / 4 im2col by TMA with 64 / 16 channels per pixel.
// Warps: 0 TMA producer, 1 MMA issuer + TMEM owner, 2-9 epilogue (two per TMEM lane quarter,
// splitting the column slabs), then either 10-13 im2col gather (MODE 1/2) or 10-12 more TMA
// producers and 13-15 more MMA issuers. One thread keeps only one TMA load per few hundred cycles
// in flight, and an issuer that waits on a stage barrier per k-tile averages about one tcgen05.mma
// per 160 cycles (back to back, without waits, one thread issues one per ~59 cycles; the tensor core
// retires an M=128 MMA every 48 / 64 / 128 cycles at N = 64 / 128 / 256, N=64 held above its 32 by
// the 6 KB of operands it reads from shared memory at 128 B per cycle), so the k-tiles are
// dealt round-robin to Q producer threads and P MMA-issuing threads (each in its own warp). The stage count is a
// multiple of both, so each stage's full and empty barriers have exactly one producer and one
// consumer, each moving through the stage's phases in order: no waiter can face a barrier two
// phases behind (which a parity wait would mistake for done).
// PREC: 0 bf16 operands (kind::f16); 1 fp32 operands read as TF32 (kind::tf32); 2 error-
// compensated TF32 ("TF32x3"): every operand x = hi + lo with hi its TF32 truncation, three MMAs
// per K slice (hi*hi + hi*lo + lo*hi) give close to fp32 accuracy. The weights' hi / lo matrices
// come from the host (lo rows start at a.w_lo_row); the activation's lo tile is computed per stage
// in shared memory by warps 14-15 once the stage has landed.
template <int MODE, int PREC>
constexpr int kThreads = ((MODE == 1 || MODE == 2) && PREC != 2) ? 448 : 512;

template <int BN, int MODE, int PREC>
__global__ void __launch_bounds__(kThreads<MODE, PREC>, 1)
    conv_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmRes,
                     const ConvGemmArgs a) {
  constexpr bool TF32 = PREC >= 1;
  constexpr bool X3 = PREC == 2;
  constexpr int EB = TF32 ? 4 : 2;        // operand element bytes
  constexpr int BKE = 128 / EB;           // operand elements per 128-byte k-tile row
  constexpr uint32_t A_BYTES = BM * 128;
  constexpr uint32_t B_BYTES = BN * 128;
  constexpr uint32_t A_STAGE = X3 ? 2 * A_BYTES : A_BYTES;   // X3: hi tile, then its lo tile
  constexpr uint32_t B_STAGE = X3 ? 2 * B_BYTES : B_BYTES;
  const int PL = a.mma_lanes;                 // split-K partial accumulators per tile
  const uint32_t TMEM_COLS = uint32_t(2 * PL * BN);
  const int PE = PL;                          // at most KT, so every partial gets a k-tile
  constexpr bool GATHER = MODE == 1 || MODE == 2;
  constexpr bool A_TMA = !GATHER;
  const int STAGES = a.stages;
  const int RS = a.res_slots;
  const uint32_t RSB = uint32_t(a.res_slot_bytes);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int KT = a.Kpad / BKE;
  // split-K: tile t is slice t % KS of output tile t / KS, k-tiles [slice * KTS, slice * KTS + KTS)
  const int KS = a.ksplit > 1 ? a.ksplit : 1;
  const int KTS = KT / KS;
  // residual k-tiles (res_mma): k-tile KT + j adds residual channels [64j, 64j + 64) of the tile
  const bool RESM = A_TMA && MODE != 4 && PREC == 0 && a.res_mma;
  const bool A2 = MODE == 0 && a.a2 != nullptr;   // second A operand (uses the tmRes map)
  const int KTE = KTS + (RESM ? BN / 64 : 0);   // k-tiles per tile (slice)
  const bool BRES = A_TMA && a.b_resident;   // weights loaded once: slot kt holds k-tile kt
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_STAGE;
  uint8_t* sOut = sB + (BRES ? KT * B_BYTES : STAGES * B_STAGE);
  const int OB = a.out_bufs;
  // per-warp output slab: 32 rows x 128 bytes, or 32 x 64 bytes when each warp stores a half
  const uint32_t SLAB = a.epi_half ? kOutSlab / 2 : kOutSlab;
  float* sBias = reinterpret_cast<float*>(sOut + 8 * OB * SLAB);
  uint8_t* sRes = sOut + 8 * OB * SLAB + kBiasStage;
  uint8_t* sId = sRes + RS * RSB;   // RESM: the identity operand
  // bias_mma: the ones tile, then the bias rows of every N tile (hi, lo at k = 0, 1)
  const bool BMMA = PREC == 0 && a.bias_mma;
  uint8_t* sOnes = sId + (RESM ? kIdBytes : 0u);
  uint8_t* sBiasT = sOnes + kOnesBytes;
  const int bias_rows = ((a.Cout + BN - 1) / BN) * BN;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOnes + (BMMA ? kOnesBytes + uint32_t(bias_rows) * 32u : 0u));
  uint64_t* empty = full + kMaxStages;
  uint64_t* accf = empty + kMaxStages;
  uint64_t* acce = accf + 2;
  uint64_t* resf = acce + 2;
  uint64_t* rese = resf + 2;
  uint64_t* bfull = rese + 2;
  uint64_t* split = bfull + 1;   // X3: the stage's activation lo tile is ready
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(split + kMaxStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], GATHER ? 129u : 1u);
      mbar_init(&empty[s], 1u);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], uint32_t(PE));
      mbar_init(&acce[i], 8u);
      mbar_init(&resf[i], 1u);
      mbar_init(&rese[i], 8u);
    }
    mbar_init(bfull, 1u);
    if (X3)
      for (int s = 0; s < STAGES; ++s) mbar_init(&split[s], 64u);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    if (A_TMA) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    if (a.epi == 2) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmOut) : "memory");
    if (RS || RESM || A2) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmRes) : "memory");
  }
  if (RESM) {   // identity rows n: 1.0 at k = n; 16-byte chunk c holds row c / 8, logical chunk (c % 8) ^ (row % 8)
    for (int c = threadIdx.x; c < int(kIdBytes / 16); c += blockDim.x) {
      const int n = c >> 3, lc = (c & 7) ^ (n & 7);
      const int word = (n >> 3) == lc ? (n & 7) >> 1 : -1;   // the 32-bit word holding element n
      const uint32_t one = (n & 1) ? 0x3F800000u : 0x00003F80u;
      reinterpret_cast<uint4*>(sId)[c] =
          make_uint4(word == 0 ? one : 0u, word == 1 ? one : 0u, word == 2 ? one : 0u, word == 3 ? one : 0u);
    }
    fence_async_smem();   // generic writes -> the MMA's async-proxy reads
  }
  if (BMMA) {
    // 32-byte swizzle, K-major: row r's 16-byte chunk c sits at chunk position c ^ ((r / 4) % 2).
    // Ones tile: 1.0 at k = 0, 1 of every row. Bias tile: row n holds hi = bf16(b[n]) at k = 0 and
    // lo = bf16(b[n] - hi) at k = 1, so hi + lo matches the fp32 bias to about 2^-17 of it.
    for (int c = threadIdx.x; c < int(kOnesBytes / 16); c += blockDim.x) {
      const int r = c >> 1, pos = c & 1;
      reinterpret_cast<uint4*>(sOnes)[c] = make_uint4(pos == ((r >> 2) & 1) ? 0x3F803F80u : 0u, 0u, 0u, 0u);
    }
    for (int c = threadIdx.x; c < bias_rows * 2; c += blockDim.x) {
      const int r = c >> 1, pos = c & 1;
      const float b = a.bias[r];
      const __nv_bfloat16 hi = __float2bfloat16_rn(b);
      const __nv_bfloat16 lo = __float2bfloat16_rn(b - __bfloat162float(hi));
      const uint32_t w = uint32_t(__bfloat16_as_ushort(hi)) | (uint32_t(__bfloat16_as_ushort(lo)) << 16);
      reinterpret_cast<uint4*>(sBiasT)[c] = make_uint4(pos == ((r >> 2) & 1) ? w : 0u, 0u, 0u, 0u);
    }
    fence_async_smem();
  }
  if (warp == 1) tmem_alloc(tmem_holder, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (BRES && warp == 0 && lane == 0) {   // this CTA's N tile of the weights (the same for all its tiles), once
    const int nt_cta = int(blockIdx.x) % ((a.Cout + BN - 1) / BN);
    mbar_expect_tx(bfull, uint32_t(KT) * B_BYTES);
    for (int kt = 0; kt < KT; ++kt) tma_load_2d(sB + kt * B_BYTES, &tmB, kt * BKE, nt_cta * BN, bfull);
  }
  pdl_wait();   // the previous kernel's outputs (and the buffers this one overwrites) are settled

  const int tiles_m = (a.M + BM - 1) / BM;
  const int tiles_n = (a.Cout + BN - 1) / BN;
  const int total = tiles_m * tiles_n * KS;
  const int SC = a.out_bf16 ? 64 : 32;   // output columns per 128-byte slab
  const int NS = BN / SC;

  const int NP = GATHER ? 1 : a.producers;      // TMA producer threads
  const int pid = warp == 0 ? 0 : warp - 9;     // producer index of warps 0, 10, 11, 12
  if (warp == 0 || (A_TMA && warp >= 10 && warp <= 12)) {
    if (lane == 0 && pid < NP) {
      int stage = 0;
      uint32_t phase = 0;
      int owner = 0;   // producer of the current k-tile (k-tiles are dealt round-robin)
      const int hw_out = a.Ho * a.Wo;
      const int cblocks = a.Cp / BKE;   // 128-byte channel blocks per filter tap (MODE 3)
      int it = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
        const int tmn = t / KS, kt0 = (t - tmn * KS) * KTS;
        const int mt = tmn / tiles_n, nt = tmn - (tmn / tiles_n) * tiles_n;
        // im2col: image and top-left input corner of the tile's first output pixel
        int img = 0, cw = 0, ch = 0;
        if (MODE == 3 || MODE == 4) {
          const int m0 = mt * BM;
          img = m0 / hw_out;
          const int rem = m0 - img * hw_out;
          const int ho = rem / a.Wo;
          ch = ho * a.sh - a.ph;
          cw = (rem - ho * a.Wo) * a.sw - a.pw;
        }
        if (RS && pid == 0) {   // the tile's residual, into a ring slot, ahead of its operands
          const int slot = it % RS;
          const uint32_t rph = uint32_t(it / RS) & 1u;
          if (!mbar_wait(&rese[slot], rph ^ 1u, abort_flag, a.err, 64u)) goto producer_done;
          int nsl = 0;
          for (int s2 = 0; s2 < NS; ++s2)
            if (nt * BN + s2 * SC < a.Cout) ++nsl;
          mbar_expect_tx(&resf[slot], uint32_t(nsl) * 128u * 128u);
          for (int s2 = 0; s2 < nsl; ++s2)
            tma_load_2d(sRes + slot * RSB + s2 * 128 * 128, &tmRes, nt * BN + s2 * SC, mt * BM, &resf[slot]);
        }
        for (int j = 0; j < KTE; ++j) {
          const int kt = j < KTS ? kt0 + j : KT + (j - KTS);   // (then the residual k-tiles)
          const bool mine = owner == pid;
          if (++owner == NP) owner = 0;
          if (!mine) {
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, a.err, 1u)) goto producer_done;
          if (kt >= KT) {   // residual k-tile: 128 rows x 64 channels of the residual, no weights
            mbar_expect_tx(&full[stage], A_BYTES);
            tma_load_2d(sA + stage * A_STAGE, &tmRes, nt * BN + (kt - KT) * 64, mt * BM, &full[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          mbar_expect_tx(&full[stage], (A_TMA ? A_BYTES : 0u) + (BRES ? 0u : B_STAGE));
          if (MODE == 0) {   // (k-tiles from a2_kt on come from the second operand, through tmRes)
            if (A2 && kt >= a.a2_kt && a.a2_s > 0) {   // strided image: im2col of a 1x1 conv at stride s
              const int m0 = mt * BM;
              const int im = m0 / hw_out, rem = m0 - (m0 / hw_out) * hw_out;
              const int ho = rem / a.Wo, wo = rem - (rem / a.Wo) * a.Wo;
              tma_load_im2col(sA + stage * A_STAGE, &tmRes, (kt - a.a2_kt) * BKE, wo * a.a2_s, ho * a.a2_s, im, 0, 0,
                              &full[stage]);
            } else if (A2 && kt >= a.a2_kt) {
              tma_load_2d(sA + stage * A_STAGE, &tmRes, (kt - a.a2_kt) * BKE, mt * BM, &full[stage]);
            } else {
              tma_load_2d(sA + stage * A_STAGE, &tmA, kt * BKE, mt * BM, &full[stage]);
            }
          }
          if (MODE == 3) {
            const int tap = kt / cblocks, cb = kt - tap * cblocks;
            const int kh = tap / a.KW, kw = tap - (tap / a.KW) * a.KW;
            tma_load_im2col(sA + stage * A_STAGE, &tmA, cb * BKE, cw, ch, img, uint16_t(kw * a.dw),
                            uint16_t(kh * a.dh), &full[stage]);
          }
          if (MODE == 4) {   // four 16-channel taps, one 4 KB sub-tile each
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int tap = kt * 4 + j;
              const int kh = tap / a.KW, kw = tap - (tap / a.KW) * a.KW;
              tma_load_im2col(sA + stage * A_STAGE + j * (BM * 32), &tmA, 0, cw, ch, img, uint16_t(kw * a.dw),
                              uint16_t(kh * a.dh), &full[stage]);
            }
          }
          if (!BRES) tma_load_2d(sB + stage * B_STAGE, &tmB, kt * BKE, nt * BN, &full[stage]);
          if (X3) tma_load_2d(sB + stage * B_STAGE + B_BYTES, &tmB, kt * BKE, a.w_lo_row + nt * BN, &full[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:;
    }
  } else if (X3 && warp >= 14) {
    // ---- X3: activation lo tiles. x = hi + lo with hi = x truncated to TF32 (what the MMA reads
    // from the fp32 tile) and lo = x - hi (exact in fp32), stored rounded to TF32 so the MMA's read
    // of it is exact and the dropped part is unbiased (a truncated lo would bias every product
    // toward zero, an error growing with K). Infinities / NaNs get lo = 0. ----------------------
    const int sid = threadIdx.x - 14 * 32;   // 0..63
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      for (int kt = 0; kt < KTS; ++kt) {
        if (!mbar_wait(&full[stage], phase, abort_flag, a.err, 256u)) goto split_done;
        const uint4* src = reinterpret_cast<const uint4*>(sA + stage * A_STAGE);
        uint4* dst = reinterpret_cast<uint4*>(sA + stage * A_STAGE + A_BYTES);
#pragma unroll 4
        for (int i = sid; i < int(A_BYTES / 16); i += 64) {
          const uint4 u = src[i];
          uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float x = __uint_as_float(w[j]);
            const float hi = __uint_as_float(w[j] & 0xFFFFE000u);
            w[j] = (w[j] & 0x7F800000u) == 0x7F800000u ? 0u : __float_as_uint(tf32_rna(x - hi));
          }
          dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_async_smem();   // generic writes -> the MMA's async-proxy reads
        mbar_arrive(&split[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  split_done:;
  } else if (warp == 1 || (A_TMA && warp >= 13)) {
    // Issuer `mid` (lane 0 of warp 1, 13, 14 or 15) issues the MMAs of the k-tiles with sequence
    // number g = mid (mod PE) into its own partial accumulator: with its per-k-tile barrier waits one
    // thread averages about one tcgen05.mma per 160 cycles, so N=64/128 tiles (48 / 64 cycles of
    // tensor work each) need several issuing threads. Each issuer commits its own k-tiles' stages and
    // arrives once per tile on the accumulator-full barrier.
    const int mid = warp == 1 ? 0 : warp - 12;
    if (lane == 0 && mid < PE) {
      constexpr uint32_t idesc = idesc_mma(BM, BN, TF32);
      constexpr uint32_t idesc64 = idesc_mma(BM, 64, TF32);   // residual k-tiles: 64 columns each
      int it = 0;
      int g0 = 0;   // sequence number of the tile's first k-tile (the producers' numbering)
      // this issuer's next k-tile g (= mid mod PE) and its stage / phase, advanced by PE steps
      int g = mid, stage = mid;
      uint32_t phase = 0;
      if (BRES && !mbar_wait(bfull, 0u, abort_flag, a.err, 128u)) goto mma_done;
      for (int t = blockIdx.x; t < total; t += gridDim.x, ++it, g0 += KTE) {
        const int acc = it & 1;
        const uint32_t aph = uint32_t(it >> 1) & 1u;
        if (!mbar_wait(&acce[acc], aph ^ 1u, abort_flag, a.err, 2u)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t((acc * PL + mid) * BN);
        const int kt0 = (t % KS) * KTS;
        bool ok = true;
        // this issuer's k-tiles of the tile: g0 <= g < g0 + KTE with g = mid (mod PE); the first
        // is always a weight k-tile (PE <= KT), which initialises every column of the partial
        for (bool first = true; g < g0 + KTE; first = false) {
          const int j = g - g0;
          const int kt = j < KTS ? kt0 + j : KT + (j - KTS);
          if (!mbar_wait(&full[stage], phase, abort_flag, a.err, 4u) ||
              (X3 && !mbar_wait(&split[stage], phase, abort_flag, a.err, 512u))) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (GATHER) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          const uint64_t ad = sw128_desc(smem_u32(sA + stage * A_STAGE));
          if (RESM && kt >= KT) {   // residual k-tile: D[:, 64j .. 64j + 64) += R_j * I
            const uint64_t idd = sw128_desc(smem_u32(sId));
            const uint32_t dcol = d_tmem + uint32_t((kt - KT) * 64);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) umma_bf16(dcol, ad + uint64_t(kk * 2), idd + uint64_t(kk * 2), idesc64, 1u);
          } else {
            const uint64_t bd = sw128_desc(smem_u32(BRES ? sB + kt * B_BYTES : sB + stage * B_STAGE));
            // bias_mma: issuer 0 starts the tile's accumulator at the bias (the other issuers'
            // partials start at zero)
            const bool bias_first = BMMA && first && mid == 0;
            if (bias_first)
              umma_bf16(d_tmem, sw32_desc(smem_u32(sOnes)), sw32_desc(smem_u32(sBiasT + ((t / KS) % tiles_n) * BN * 32)),
                        idesc, 0u);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {   // four 32-byte K slices per 128-byte row
              const uint64_t akk = MODE == 4 ? sw32_desc(smem_u32(sA + stage * A_STAGE + kk * (BM * 32)))
                                             : ad + uint64_t(kk * 2);
              const uint32_t accum = (!first || kk != 0 || bias_first) ? 1u : 0u;
              if (X3) {
                const uint64_t alo = sw128_desc(smem_u32(sA + stage * A_STAGE + A_BYTES)) + uint64_t(kk * 2);
                const uint64_t blo = sw128_desc(smem_u32(sB + stage * B_STAGE + B_BYTES)) + uint64_t(kk * 2);
                umma_tf32(d_tmem, akk, bd + uint64_t(kk * 2), idesc, accum);
                umma_tf32(d_tmem, akk, blo, idesc, 1u);
                umma_tf32(d_tmem, alo, bd + uint64_t(kk * 2), idesc, 1u);
              } else if (TF32) {
                umma_tf32(d_tmem, akk, bd + uint64_t(kk * 2), idesc, accum);
              } else {
                umma_bf16(d_tmem, akk, bd + uint64_t(kk * 2), idesc, accum);
              }
            }
          }
          umma_commit(&empty[stage]);
          g += PE;
          stage += PE;
          if (stage >= STAGES) {   // STAGES is a multiple of PE (or PE == 1)
            stage -= STAGES;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&accf[acc]);
      }
    mma_done:;
    }
  } else if (warp < 10) {
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int hsel = (warp - 2) >> 2; // which of the two warps of this quarter
    uint8_t* sb0 = sOut + (warp - 2) * OB * SLAB;
    float* wbias = sBias + (warp - 2) * 128;
    const int HPS = SC / 32;   // 32-column halves per slab
    // Bias of this warp's columns of tile t (slabs hsel, hsel+2, ...; at most 4 x 32 floats),
    // lane-strided into registers one tile ahead of use and staged through wbias. The bias array
    // is padded to a multiple of 256 columns.
    // With epi_half the warp's columns are the tile's 32-column half hsel.
    const bool ehalf = BN == 64 && a.epi_half != 0 && OB != 0;
    auto load_bias = [&](int t, float (&b)[4]) {
      const int nt = (t / KS) % tiles_n;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int s2 = hsel + 2 * (i / HPS);
        if (a.bias_mma) b[i] = 0.f;   // (the accumulator starts at the bias)
        else if (ehalf) b[i] = (t < total && i == 0) ? __ldg(a.bias + nt * BN + hsel * 32 + lane) : 0.f;
        else b[i] = (t < total && s2 < NS) ? __ldg(a.bias + nt * BN + s2 * SC + (i % HPS) * 32 + lane) : 0.f;
      }
    };
    float bpre[4];
    load_bias(blockIdx.x, bpre);
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      const int tmn = t / KS;
      const int mt = tmn / tiles_n, nt = tmn - (tmn / tiles_n) * tiles_n;
      const int acc = it & 1;
      const uint32_t aph = uint32_t(it >> 1) & 1u;
      if (!mbar_wait(&accf[acc], aph, abort_flag, a.err, 8u)) break;
      tc_fence_after();
#pragma unroll
      for (int i = 0; i < 4; ++i) wbias[i * 32 + lane] = bpre[i];
      __syncwarp();
      load_bias(t + gridDim.x, bpre);   // next tile's bias, consumed one tile from now
      const int row0 = mt * BM + q * 32;
      const int srow0 = row0 + (t % KS) * a.Mp;   // (split-K: this slice's rows of the partials)
      const uint32_t tbase = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * PL * BN);
      const int slot = RS ? it % RS : 0;
      if (RS && !mbar_wait(&resf[slot], uint32_t(it / RS) & 1u, abort_flag, a.err, 32u)) break;
      if (row0 < a.M) {   // warp-uniform
        if (a.epi == 2 && ehalf) {   // bf16 output, one 64-column slab: both warps, a half each
          if (nt * BN + hsel * 32 < a.Cout) {
            const uint8_t* rslab = RS ? sRes + slot * RSB : nullptr;
            uint8_t* sb = sb0;
            epilogue_slab<true>(a, &tmOut, tbase, 0, srow0, nt * BN, sb, rslab, wbias, OB, PE, BN, hsel);
          }
        } else if (a.epi == 2) {
          for (int s2 = hsel; s2 < NS; s2 += 2) {
            const int n0 = nt * BN + s2 * SC;
            if (n0 >= a.Cout) break;
            const uint8_t* rslab = RS ? sRes + slot * RSB + s2 * 128 * 128 : nullptr;
            // With a residual ring and no output slabs (OB == 0) the output is written in place
            // over this warp's 32-row band of the residual slab and stored from there; the slot is
            // released once that store has read it. Otherwise the warp's own output slab(s).
            const bool inplace = RS && OB == 0;
            uint8_t* sb = inplace ? sRes + slot * RSB + s2 * 128 * 128 + q * 32 * 128
                                  : sb0;
            const int wm = inplace ? 0 : OB;
            const float* bsl = wbias + ((s2 - hsel) >> 1) * SC;
            if (a.out_bf16 && a.epi_half) {   // two 32-column halves through the warp's 2 KB slab
              for (int hh = 0; hh < 2 && n0 + hh * 32 < a.Cout; ++hh)
                epilogue_slab<true>(a, &tmOut, tbase, s2 * SC, srow0, n0, sb, rslab, bsl + hh * 32, wm, PE, BN, hh);
            } else if (a.out_bf16) epilogue_slab<true>(a, &tmOut, tbase, s2 * SC, srow0, n0, sb, rslab, bsl, wm, PE, BN);
            else epilogue_slab<false>(a, &tmOut, tbase, s2 * SC, srow0, n0, sb, rslab, bsl, wm, PE, BN);
          }
        } else {
          const int m = row0 + lane;
#pragma unroll 1
          for (int c = hsel; c < BN / 32; c += 2) {
            float fv[32];
            tmem_ld_sum(tbase + uint32_t(c * 32), PE, BN, fv);
            uint32_t r[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(fv[j]);
            const int n0 = nt * BN + c * 32;
            if (n0 < a.Cout && m < a.M) epilogue_chunk(a, r, m, n0);
          }
        }
      }
      tc_fence_before();
      __syncwarp();   // also: every lane is done reading wbias before the next tile rewrites it
      if (lane == 0) {
        mbar_arrive(&acce[acc]);
        if (RS) {
          if (OB == 0) bulk_wait_read0();   // in place: this warp's stores have read the slot
          mbar_arrive(&rese[slot]);
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  } else if constexpr (GATHER) {
    // ---- im2col gather producers -------------------------------------------------------------
    const int gt = threadIdx.x - 320;   // 0..127
    constexpr int TPR = MODE == 1 ? 8 : 16;          // threads per 128-byte row
    constexpr int ROWS_PER_PASS = 128 / TPR;         // 16 or 8
    constexpr int PASSES = BM / ROWS_PER_PASS;       // 8 or 16
    const int sub = gt % TPR;
    const int rbase = gt / TPR;
    const uint8_t* xb = reinterpret_cast<const uint8_t*>(a.x);
    const int hw_out = a.Ho * a.Wo;
    const int ktaps = a.KH * a.KW;
    const int kreal = ktaps * a.Cp;
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const int mt = (t / KS) / tiles_n;
      const int kt0 = (t % KS) * KTS;
      int hb[PASSES], wb[PASSES];
      int64_t base[PASSES];
#pragma unroll
      for (int i = 0; i < PASSES; ++i) {
        const int m = mt * BM + rbase + i * ROWS_PER_PASS;
        if (m < a.M) {
          const int n = m / hw_out, rem = m - n * hw_out;
          const int ho = rem / a.Wo, wo = rem - ho * a.Wo;
          hb[i] = ho * a.sh - a.ph;
          wb[i] = wo * a.sw - a.pw;
          base[i] = int64_t(n) * a.H * a.W * a.Cp;
        } else {
          hb[i] = -(1 << 28);   // forces every tap out of range
          wb[i] = 0;
          base[i] = 0;
        }
      }
      for (int kt = kt0; kt < kt0 + KTS; ++kt) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, a.err, 16u)) goto gather_done;
        const uint32_t sbase = smem_u32(sA + stage * A_STAGE);
        if (MODE == 1) {
          const int kidx = kt * BKE + sub * (16 / EB);
          const int tap = kidx / a.Cp;
          const int c = kidx - tap * a.Cp;
          const int kh = tap / a.KW, kw = tap - (tap / a.KW) * a.KW;
          const bool kvalid = kidx < kreal;
          const int dh = kh * a.dh, dw = kw * a.dw;
#pragma unroll
          for (int i = 0; i < PASSES; ++i) {
            const int r = rbase + i * ROWS_PER_PASS;
            const int hi = hb[i] + dh, wi = wb[i] + dw;
            const bool ok = kvalid && hi >= 0 && hi < a.H && wi >= 0 && wi < a.W;
            const uint8_t* src = ok ? xb + (base[i] + (int64_t(hi) * a.W + wi) * a.Cp + c) * EB : xb;
            const uint32_t dst = sbase + uint32_t(r * 128 + ((sub ^ (r & 7)) << 4));
            cp_async_16(dst, src, ok ? 16u : 0u);
          }
        } else {
          const int tap = kt * (BKE / 4) + sub;   // bf16, Cp == 4: one tap per 8-byte unit
          const int kh = tap / a.KW, kw = tap - (tap / a.KW) * a.KW;
          const bool kvalid = tap < ktaps;
          const int dh = kh * a.dh, dw = kw * a.dw;
#pragma unroll
          for (int i = 0; i < PASSES; ++i) {
            const int r = rbase + i * ROWS_PER_PASS;
            const int hi = hb[i] + dh, wi = wb[i] + dw;
            const bool ok = kvalid && hi >= 0 && hi < a.H && wi >= 0 && wi < a.W;
            const uint8_t* src = ok ? xb + (base[i] + (int64_t(hi) * a.W + wi) * 4) * EB : xb;
            const uint32_t dst = sbase + uint32_t(r * 128 + (((sub >> 1) ^ (r & 7)) << 4) + ((sub & 1) << 3));
            cp_async_8(dst, src, ok ? 8u : 0u);
          }
        }
        cp_async_arrive_noinc(&full[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  gather_done:
    cp_async_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---- CTA-pair implicit GEMM (tcgen05.mma.cta_group::2) ----------------------------------------------
// Two CTAs of a cluster compute one 256 x 256 output tile. Each loads its own 128 rows of A and its
// own 128 rows (output channels) of B into the same shared-memory offsets; the even CTA's issuer runs
// M=256, N=256 MMAs that read both CTAs' operands, and each CTA's TMEM holds the accumulator of its
// own 128 rows x all 256 columns. Per SM this halves the B traffic (TMA writes into shared memory, the
// MMAs' operand reads, L2 reads) of a 128 x 256 tile on one SM; each stage is 32 KB instead of 48.
// Barriers sit at the same offsets in both CTAs: full[s] is used in the even CTA (its producer
// expects both CTAs' bytes, the odd CTA's loads complete on it); empty[s] and accf[acc] in both (the
// issuer commits to each CTA's copy separately); acce[acc] in the even CTA (both CTAs' 8 epilogue
// warps arrive, the odd CTA's remotely). Every mbarrier wait is bounded; both CTAs always reach the
// final cluster barrier, before which neither leaves (the issuer reads the odd CTA's shared memory).
// A merged projection shortcut's second A operand comes through tmRes as in the one-SM kernel.
// A bf16 residual is added by the tensor core as in the one-SM kernel: after the weight k-tiles come
// four k-tiles of residual rows (64 channels each) against a 64 x 64 identity, whose rows 32r .. 32r + 31
// CTA r holds (the B operand of an N=64 pair MMA is split between the two CTAs like any other).
// Warps: 0 and 10 TMA producers (A and B), 1 TMEM owner + MMA issuer (even CTA), 2-9 epilogue.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory location in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// the tcgen05 operations of a CTA pair: all of the kernel's use cta_group::2
__device__ __forceinline__ void tmem_alloc2(uint32_t* holder, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma2_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrives on the mbarrier at this shared::cluster address once the issuer's MMAs so far are done
__device__ __forceinline__ void umma2_commit(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}
// TMA loads into this CTA's shared memory whose completion counts on the even CTA's barrier
__device__ __forceinline__ void tma2_load_2d(void* dst, const CUtensorMap* tm, int c0, int c1, uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(tm), "r"(c0), "r"(c1), "r"(leader_bar)
      : "memory");
}
__device__ __forceinline__ void tma2_load_im2col(void* dst, const CUtensorMap* tm, int c, int w, int h, int n, uint16_t ow,
                                                 uint16_t oh, uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.im2col.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], {%7, %8};" ::"r"(smem_u32(dst)),
      "l"(tm), "r"(c), "r"(w), "r"(h), "r"(n), "r"(leader_bar), "h"(ow), "h"(oh)
      : "memory");
}

constexpr uint32_t kPairB = 128 * 128;              // this CTA's 128 weight rows x one 128-byte k-tile
constexpr uint32_t kPairStage = BM * 128 + kPairB;  // 32 KB

template <int MODE>
__global__ void __launch_bounds__(512, 1)
    conv_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmRes,
                     const ConvGemmArgs a) {
  constexpr int BN = 256;
  constexpr uint32_t A_BYTES = BM * 128;
  const int STAGES = a.stages;
  const int OB = a.out_bufs;
  const uint32_t SLAB = a.epi_half ? kOutSlab / 2 : kOutSlab;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sOut = sB + STAGES * kPairB;
  const bool RESM = a.res_mma != 0;
  uint8_t* sId = sOut + 8 * OB * SLAB;   // RESM: this CTA's 32 rows of the identity (1 KB aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(sId + (RESM ? kIdBytes / 2 : 0u));
  uint64_t* empty = full + kMaxStages;
  uint64_t* accf = empty + kMaxStages;
  uint64_t* acce = accf + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1u);
      mbar_init(&empty[s], 1u);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1u);
      mbar_init(&acce[i], 16u);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmOut) : "memory");
    if (RESM || a.a2) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmRes) : "memory");
  }
  if (RESM) {   // local row i is identity row n = 32 rank + i: 1.0 at k = n; chunk c of row i holds
                // logical chunk (c % 8) ^ (i % 8)
    for (int c = threadIdx.x; c < int(kIdBytes / 32); c += blockDim.x) {
      const int i = c >> 3, n = int(rank) * 32 + i, lc = (c & 7) ^ (i & 7);
      const int word = (n >> 3) == lc ? (n & 7) >> 1 : -1;   // the 32-bit word holding element n
      const uint32_t one = (n & 1) ? 0x3F800000u : 0x00003F80u;
      reinterpret_cast<uint4*>(sId)[c] =
          make_uint4(word == 0 ? one : 0u, word == 1 ? one : 0u, word == 2 ? one : 0u, word == 3 ? one : 0u);
    }
    fence_async_smem();   // generic writes -> the MMA's async-proxy reads
  }
  if (warp == 1) tmem_alloc2(tmem_holder, 2 * BN);
  tc_fence_before();
  cluster_sync();   // both CTAs' barriers initialised and TMEM allocated before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_wait();

  const int KT = a.Kpad / BK;
  const int KTE = KT + (RESM ? BN / 64 : 0);   // k-tiles per tile: weights, then residual
  const int tiles_m = (a.M + 2 * BM - 1) / (2 * BM);
  const int tiles_n = (a.Cout + BN - 1) / BN;
  const int total = tiles_m * tiles_n;
  const int pair = int(blockIdx.x >> 1), npairs = int(gridDim.x >> 1);

  if (warp == 0 || warp == 10) {
    // ---- TMA producers (both CTAs): warp 0 loads A (and the residual or second operand) and, in
    // the even CTA, expects the stage's bytes; warp 10 loads this CTA's half of the weights ----
    const bool bprod = warp == 10;
    if (lane == 0) {
      const int hw_out = a.Ho * a.Wo;
      const int cblocks = a.Cp / BK;
      int stage = 0;
      uint32_t phase = 0;
      for (int t = pair; t < total; t += npairs) {
        const int mt = t / tiles_n, nt = t - (t / tiles_n) * tiles_n;
        const int m0 = mt * 2 * BM + int(rank) * BM;
        int img = 0, cw = 0, ch = 0;
        if (MODE == 3) {
          img = m0 / hw_out;
          const int rem = m0 - img * hw_out;
          const int ho = rem / a.Wo;
          ch = ho * a.sh - a.ph;
          cw = (rem - ho * a.Wo) * a.sw - a.pw;
        }
        for (int kt = 0; kt < KTE; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, a.err, 1u)) goto producer_done;
          const uint32_t fb = peer_addr(&full[stage], 0);
          if (bprod) {
            if (kt < KT) tma2_load_2d(sB + stage * kPairB, &tmB, kt * BK, nt * BN + int(rank) * 128, fb);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          if (kt >= KT) {   // residual k-tile: this CTA's 128 rows x 64 residual channels, no weights
            if (leader) mbar_expect_tx(&full[stage], 2 * A_BYTES);
            tma2_load_2d(sA + stage * A_BYTES, &tmRes, nt * BN + (kt - KT) * 64, m0, fb);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          if (leader) mbar_expect_tx(&full[stage], 2 * kPairStage);
          if (MODE == 0) {   // (k-tiles from a2_kt on come from the second operand, through tmRes)
            if (a.a2 && kt >= a.a2_kt && a.a2_s > 0) {   // strided image: im2col of a 1x1 conv at stride s
              const int im = m0 / hw_out, rem = m0 - (m0 / hw_out) * hw_out;
              const int ho = rem / a.Wo, wo = rem - (rem / a.Wo) * a.Wo;
              tma2_load_im2col(sA + stage * A_BYTES, &tmRes, (kt - a.a2_kt) * BK, wo * a.a2_s, ho * a.a2_s, im, 0, 0, fb);
            } else if (a.a2 && kt >= a.a2_kt) {
              tma2_load_2d(sA + stage * A_BYTES, &tmRes, (kt - a.a2_kt) * BK, m0, fb);
            } else {
              tma2_load_2d(sA + stage * A_BYTES, &tmA, kt * BK, m0, fb);
            }
          } else {
            const int tap = kt / cblocks, cb = kt - tap * cblocks;
            const int kh = tap / a.KW, kw = tap - (tap / a.KW) * a.KW;
            tma2_load_im2col(sA + stage * A_BYTES, &tmA, cb * BK, cw, ch, img, uint16_t(kw * a.dw), uint16_t(kh * a.dh),
                             fb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {   // ---- MMA issuer (even CTA) ----
      constexpr uint32_t idesc = idesc_mma(2 * BM, BN, false);
      constexpr uint32_t idesc64 = idesc_mma(2 * BM, 64, false);   // residual k-tiles: 64 columns each
      const uint64_t idd = sw128_desc(smem_u32(sId));
      int stage = 0, it = 0;
      uint32_t phase = 0;
      for (int t = pair; t < total; t += npairs, ++it) {
        const int acc = it & 1;
        if (!mbar_wait(&acce[acc], (uint32_t(it >> 1) & 1u) ^ 1u, abort_flag, a.err, 2u)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        bool ok = true;
        for (int kt = 0; kt < KTE; ++kt) {
          if (!mbar_wait(&full[stage], phase, abort_flag, a.err, 4u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(smem_u32(sA + stage * A_BYTES));
          const uint64_t bd = sw128_desc(smem_u32(sB + stage * kPairB));
          if (kt >= KT) {   // D[:, 64j .. 64j + 64) += R_j * I
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma2_bf16(d_tmem + uint32_t((kt - KT) * 64), ad + uint64_t(kk * 2), idd + uint64_t(kk * 2), idesc64, 1u);
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma2_bf16(d_tmem, ad + uint64_t(kk * 2), bd + uint64_t(kk * 2), idesc, (kt | kk) != 0 ? 1u : 0u);
          }
          umma2_commit(smem_u32(&empty[stage]));
          umma2_commit(peer_addr(&empty[stage], 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma2_commit(smem_u32(&accf[acc]));
        umma2_commit(peer_addr(&accf[acc], 1));
      }
    }
  } else if (warp < 10) {
    // ---- epilogue (both CTAs): this CTA's 128 rows of the tile, all 256 columns ----
    const int q = warp & 3;
    const int hsel = (warp - 2) >> 2;
    uint8_t* sb0 = sOut + (warp - 2) * OB * SLAB;
    const uint32_t acce0 = peer_addr(&acce[0], 0), acce1 = peer_addr(&acce[1], 0);
    int it = 0;
    for (int t = pair; t < total; t += npairs, ++it) {
      const int mt = t / tiles_n, nt = t - (t / tiles_n) * tiles_n;
      const int acc = it & 1;
      if (!mbar_wait(&accf[acc], uint32_t(it >> 1) & 1u, abort_flag, a.err, 8u)) break;
      tc_fence_after();
      const int row0 = mt * 2 * BM + int(rank) * BM + q * 32;
      const uint32_t tbase = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN);
      if (row0 < a.M) {   // warp-uniform
        for (int s2 = hsel; s2 < BN / 64; s2 += 2) {
          const int n0 = nt * BN + s2 * 64;
          if (n0 >= a.Cout) break;
          if (a.epi_half) {
            for (int hh = 0; hh < 2 && n0 + hh * 32 < a.Cout; ++hh)
              epilogue_slab<true>(a, &tmOut, tbase, s2 * 64, row0, n0, sb0, nullptr, a.bias + n0 + hh * 32, OB, 1, BN, hh);
          } else {
            epilogue_slab<true>(a, &tmOut, tbase, s2 * 64, row0, n0, sb0, nullptr, a.bias + n0, OB, 1, BN);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&acce[acc]);
        else remote_arrive(acc ? acce1 : acce0);
      }
    }
    if (lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();   // neither CTA leaves while the other may still touch its shared memory or barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, 2 * BN);
  }
}

// ---- stem convolution + 3x3/2 max pool ----------------------------------------------------------
// The ResNet stem (7x7/2 conv over 3 channels, run as a 4x4 stride-1 conv over the 2x2
// space-to-depth image of 16-channel pixels) with bias, activation and the following MaxPool 3x3 /
// stride 2 / pad 1 in one kernel. A tile is one conv output row (Wo <= 128 pixels; the tile's
// remaining rows are junk, computed and dropped). CTA b walks a contiguous range of pool rows: for
// each it computes conv rows 2po and 2po + 1 (and, at the start of its range, the halo row 2po - 1).
// The conv output (1.6 MB per 224x224 image) never reaches global memory.
// A operand: a ring of space-to-depth input rows, one 2D-like TMA box of 131 pixels x 16 channels
// (32-byte rows, 32-byte swizzle) per row. Conv row r reads input rows r - ph + a (filter row a);
// consecutive conv rows share three of their four input rows, so a row costs one 4 KB load. Filter
// tap (a, b) is the 128-row window of input row a starting b pixels in: the descriptor start moves
// by b x 32 bytes and the swizzle, a function of the address bits, follows it. B: the 64 x 256
// weights, resident. K order (filter column b, filter row a, channel).
// Max pool in registers: epilogue warp (q, h) holds pixels 32q .. 32q + 31 (its TMEM lanes) and
// channels 32h .. 32h + 31. Per pixel it keeps the bf16 values of the last odd conv row (V) and the
// max over the pool row's first two conv rows (M); after the odd row it has the vertical max F, takes
// the horizontal max over pixels 2pw - 1 .. 2pw + 1 with lane shuffles (the pixel left of lane 0
// comes from warp (q - 1, h) through shared memory) and stores pool column 16q + lane / 2 from the
// even lanes. Bias and activation are applied and rounded to bf16 before any max, as the separate
// conv and pool kernels would (rounding is monotonic, so the order of max and rounding is immaterial).
// Warps: 0 TMA producer, 1 and 13-15 MMA issuers (issuer i takes conv rows i mod P, all 16 taps of
// each, into one of eight TMEM accumulators), 2-9 epilogue. Every wait is bounded.
constexpr int kStemKT = 4;                      // filter columns (weight k-tiles)
constexpr uint32_t kStemBBytes = 64 * 128;      // one 64 x 64 bf16 weight k-tile (4 filter rows x 16 channels)
constexpr int kStemRowPx = BM + 3;              // input pixels per ring row: 128 + the three extra filter columns
constexpr uint32_t kStemRowBytes = uint32_t(kStemRowPx) * 32u;
constexpr uint32_t kStemSlot = 5 * 1024;        // ring slot stride (1 KB aligned)
constexpr int kStemRing = 16;                   // input rows in flight
constexpr int kStemAcc = 8;                     // TMEM accumulators (conv rows) of 64 columns

// The conv rows CTA `cta` computes, in order: calls f(n, r, pool) for each, where pool says that the
// row completes pool row r / 2 (r odd, and not the halo row of the range's first pool row).
template <typename F>
__device__ __forceinline__ void stem_rows(const StemPoolArgs& a, int cta, int ctas, F&& f) {
  const int Hp = a.Ho / 2;
  const int64_t total = int64_t(a.N) * Hp;
  const int64_t p0 = total * cta / ctas, p1 = total * (cta + 1) / ctas;
  for (int64_t p = p0; p < p1; ++p) {
    const int n = int(p / Hp), po = int(p - int64_t(n) * Hp);
    if (p == p0 && po > 0)
      if (!f(n, 2 * po - 1, false)) return;
    if (!f(n, 2 * po, false)) return;
    if (!f(n, 2 * po + 1, true)) return;
  }
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* tm, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          smem_u32(dst)),
      "l"(tm), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t bf16x2_max(uint32_t x, uint32_t y) {
  __nv_bfloat162 r = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&x), *reinterpret_cast<const __nv_bfloat162*>(&y));
  return *reinterpret_cast<uint32_t*>(&r);
}

__global__ void __launch_bounds__(512, 1)
    stem_pool_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const StemPoolArgs a) {
  constexpr uint32_t idesc = idesc_mma(BM, 64, false);
  const int PE = a.mma_lanes;         // MMA issuers (1 to 4)
  constexpr uint32_t TMEM_COLS = 512; // kStemAcc accumulators of 64 columns
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;
  uint8_t* ring = sB + kStemKT * kStemBBytes;
  float* sBias = reinterpret_cast<float*>(ring + kStemRing * kStemSlot);
  uint4* xch = reinterpret_cast<uint4*>(sBias + 64);   // [pool-row parity][quarter][half][4 x 16 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(xch + 2 * 4 * 2 * 4);
  uint64_t* empty = full + kStemRing;
  uint64_t* accf = empty + kStemRing;
  uint64_t* acce = accf + kStemAcc;
  uint64_t* bfull = acce + kStemAcc;
  uint64_t* xbar = bfull + 1;   // [2]: the 8 epilogue warps published a pool row's boundary pixels
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(xbar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStemRing; ++s) {
      mbar_init(&full[s], 1u);
      mbar_init(&empty[s], uint32_t(PE));
    }
    for (int i = 0; i < kStemAcc; ++i) {
      mbar_init(&accf[i], 1u);
      mbar_init(&acce[i], 8u);
    }
    mbar_init(bfull, 1u);
    mbar_init(&xbar[0], 8u);
    mbar_init(&xbar[1], 8u);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (threadIdx.x < 64) sBias[threadIdx.x] = a.bias[threadIdx.x];
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
  }
  if (warp == 1) tmem_alloc(tmem_holder, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (warp == 0 && lane == 0) {   // the weights, once
    mbar_expect_tx(bfull, uint32_t(kStemKT) * kStemBBytes);
    for (int kt = 0; kt < kStemKT; ++kt) tma_load_2d(sB + kt * kStemBBytes, &tmB, kt * BK, 0, bfull);
  }
  pdl_wait();

  if (warp == 0) {
    // ---- TMA producer: load s (in conv-row order, one per row, four at an image or range start)
    // goes to ring slot s mod kStemRing once every issuer has released the load before it there ----
    if (lane == 0) {
      int s = 0, pn = -1, pr = -8;
      stem_rows(a, blockIdx.x, gridDim.x, [&](int n, int r, bool) {
        const bool cont = n == pn && r == pr + 1;
        for (int j = cont ? 3 : 0; j < 4; ++j, ++s) {
          const int slot = s % kStemRing;
          if (!mbar_wait(&empty[slot], (uint32_t(s / kStemRing) & 1u) ^ 1u, abort_flag, a.err, 1u)) return false;
          mbar_expect_tx(&full[slot], kStemRowBytes);
          tma_load_4d(ring + slot * kStemSlot, &tmA, 0, -a.pw, r - a.ph + j, n, &full[slot]);
        }
        pn = n;
        pr = r;
        return true;
      });
    }
  } else if (warp == 1 || warp >= 13) {
    // ---- MMA issuers: issuer mid takes the conv rows i = mid (mod PE), all 16 taps of each, into
    // accumulator i mod 8. Loads are released per issuer: at the start of each of its rows an issuer
    // commits the release of every load below that row's first (its earlier rows were its last
    // reads of them; the commit fires once those MMAs are done), so each load gets PE releases ----
    const int mid = warp == 1 ? 0 : warp - 12;
    if (lane == 0 && mid < PE) {
      int row = 0, s_next = 0, rel = 0, pn = -1, pr = -8;
      if (mbar_wait(bfull, 0u, abort_flag, a.err, 128u)) {
        stem_rows(a, blockIdx.x, gridDim.x, [&](int n, int r, bool) {
          const bool cont = n == pn && r == pr + 1;
          pn = n;
          pr = r;
          const int base = cont ? s_next - 3 : s_next;   // this row's input rows: loads base .. base + 3
          s_next = base + 4;
          const int it = row++;
          if (it % PE != mid) return true;
          for (; rel < base; ++rel) umma_commit(&empty[rel % kStemRing]);
          for (int s = base; s < base + 4; ++s)
            if (!mbar_wait(&full[s % kStemRing], uint32_t(s / kStemRing) & 1u, abort_flag, a.err, 4u)) return false;
          const int acc = it % kStemAcc;
          if (!mbar_wait(&acce[acc], (uint32_t(it / kStemAcc) & 1u) ^ 1u, abort_flag, a.err, 2u)) return false;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + uint32_t(acc * 64);
#pragma unroll
          for (int b = 0; b < kStemKT; ++b) {
            const uint64_t bd = sw128_desc(smem_u32(sB + b * kStemBBytes));
#pragma unroll
            for (int fa = 0; fa < 4; ++fa) {
              const uint8_t* rowp = ring + ((base + fa) % kStemRing) * kStemSlot + b * 32;
              umma_bf16(d_tmem, sw32_desc(smem_u32(rowp)), bd + uint64_t(fa * 2), idesc, (b | fa) != 0 ? 1u : 0u);
            }
          }
          umma_commit(&accf[acc]);
          return true;
        });
      }
    }
  } else if (warp >= 2 && warp <= 9) {
    // ---- epilogue warps 2-9: warp w holds pixels 32 (w & 3) .. + 31 and channels 32 h .. + 31 ----
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int Hp = a.Ho / 2, Wp = a.Wo / 2;
    const float* bs = sBias + h * 32;
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    uint32_t V[16], M[16];   // bf16 pairs: last odd conv row; max of the pool row's first two rows
#pragma unroll
    for (int j = 0; j < 16; ++j) V[j] = M[j] = 0u;
    int it = 0, pc = 0;
    stem_rows(a, blockIdx.x, gridDim.x, [&](int n, int r, bool pool) {
      const int acc = it % kStemAcc;
      if (!mbar_wait(&accf[acc], uint32_t(it / kStemAcc) & 1u, abort_flag, a.err, 8u)) return false;
      tc_fence_after();
      uint32_t u[32];
      tmem_ld32(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * 64 + h * 32), u);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[acc]);
      ++it;
      uint32_t c[16];
      const float4* b4 = reinterpret_cast<const float4*>(bs);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 bb = b4[j];
        const float2 x = __fadd2_rn(make_float2(__uint_as_float(u[4 * j]), __uint_as_float(u[4 * j + 1])), make_float2(bb.x, bb.y));
        const float2 y = __fadd2_rn(make_float2(__uint_as_float(u[4 * j + 2]), __uint_as_float(u[4 * j + 3])), make_float2(bb.z, bb.w));
        c[2 * j] = a.act == 1 ? pack_bf16x2_relu(x.x, x.y) : pack_bf16x2(x.x, x.y);
        c[2 * j + 1] = a.act == 1 ? pack_bf16x2_relu(y.x, y.y) : pack_bf16x2(y.x, y.y);
      }
      if (!(r & 1)) {   // conv row 2po: with the row above (none at po = 0: pool padding)
#pragma unroll
        for (int j = 0; j < 16; ++j) M[j] = r > 0 ? bf16x2_max(V[j], c[j]) : c[j];
        return true;
      }
      if (!pool) {   // the range's halo row 2po - 1
#pragma unroll
        for (int j = 0; j < 16; ++j) V[j] = c[j];
        return true;
      }
      // conv row 2po + 1 completes pool row po
      const int po = r >> 1;
      uint32_t F[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        F[j] = bf16x2_max(M[j], c[j]);
        V[j] = c[j];
      }
      uint4* xs = xch + (pc & 1) * 32;   // this pool row's slots: [quarter][half][4]
      if (lane == 31) {
        if (q < 3)
#pragma unroll
          for (int j = 0; j < 4; ++j) xs[(q * 2 + h) * 4 + j] = make_uint4(F[4 * j], F[4 * j + 1], F[4 * j + 2], F[4 * j + 3]);
        mbar_arrive(&xbar[pc & 1]);
      }
      if (!mbar_wait(&xbar[pc & 1], uint32_t(pc >> 1) & 1u, abort_flag, a.err, 16u)) return false;
      uint32_t L[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t lf = __shfl_up_sync(0xffffffffu, F[j], 1);
        const uint32_t rt = __shfl_down_sync(0xffffffffu, F[j], 1);
        L[j] = bf16x2_max(F[j], rt);
        if (lane > 0) L[j] = bf16x2_max(L[j], lf);
      }
      if (lane == 0 && q > 0) {   // pixel 32q - 1, from warp (q - 1, h)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 u = xs[((q - 1) * 2 + h) * 4 + j];
          L[4 * j] = bf16x2_max(L[4 * j], u.x);
          L[4 * j + 1] = bf16x2_max(L[4 * j + 1], u.y);
          L[4 * j + 2] = bf16x2_max(L[4 * j + 2], u.z);
          L[4 * j + 3] = bf16x2_max(L[4 * j + 3], u.w);
        }
      }
      const int pw = q * 16 + (lane >> 1);
      if (!(lane & 1) && pw < Wp) {
        uint4* dst = reinterpret_cast<uint4*>(out + ((int64_t(n) * Hp + po) * Wp + pw) * 64 + h * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[j] = make_uint4(L[4 * j], L[4 * j + 1], L[4 * j + 2], L[4 * j + 3]);
      }
      ++pc;
      return true;
    });
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---- 3x3 / stride 1 / pad 1 convolution from halo tiles ------------------------------------------
// A tile is R output rows x Wp pixels of one image (Wp the power of two >= W + 2, R = 128 / Wp),
// i.e. the 128 accumulator rows are the pixels p = r * Wp + c. One 4D TMA box brings the tile's
// (R + 2) x Wp input halo (64 channels, starting at input row r0 - 1 and column -1, zero outside the
// image) into shared memory in the 128-byte-swizzled K-major layout, and tap (kh, kw) reads it as a
// 128-row window starting kh * Wp + kw rows in: halo row (r + kh) * Wp + c + kw is input pixel
// (r0 + r + kh - 1, c + kw - 1). Pixels c >= W (and rows past H) are junk: computed, never stored
// (their windows may run two rows past the halo, into slack rows of the stage). One load of
// (R + 2) * Wp * 128 bytes per tile replaces nine 16 KB im2col loads; the 64 x 576 weights stay
// resident. Warps: 0 TMA producer, 1 and 13-15 MMA issuers (tap t goes to issuer t mod P, each
// into its own TMEM partial), 2-9 epilogue (TMA stores through a 4D output map that clips the junk).
constexpr uint32_t kHaloBBytes = 64 * 128;   // one 64 x 64 bf16 weight k-tile
constexpr int kHaloTaps = 9;

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* tm, int c0, int c1, int c2, int c3, const void* src) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(tm),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
               : "memory");
}

__host__ __device__ inline uint32_t halo_stage_bytes(int Wp, int R) {
  return (uint32_t((R + 2) * Wp + 2) * 128u + 1023u) & ~1023u;   // + the two slack rows, 1 KB aligned
}

__global__ void __launch_bounds__(512, 1)
    conv3x3_halo_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmOut, const Conv3x3Args a) {
  constexpr uint32_t idesc = idesc_mma(BM, 64, false);
  const int STAGES = a.stages;
  const int PE = a.mma_lanes;
  const uint32_t TMEM_COLS = uint32_t(2 * PE * 64);
  const int Wp = a.Wp, R = a.R;
  const uint32_t HALO_BYTES = uint32_t((R + 2) * Wp) * 128u;
  const uint32_t HALO_STAGE = halo_stage_bytes(Wp, R);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * HALO_STAGE;
  uint8_t* sOut = sB + kHaloTaps * kHaloBBytes;
  float* sBias = reinterpret_cast<float*>(sOut + 8 * (kOutSlab / 2));
  uint64_t* full = reinterpret_cast<uint64_t*>(sBias + 64);
  uint64_t* empty = full + kMaxStages;
  uint64_t* accf = empty + kMaxStages;
  uint64_t* acce = accf + 2;
  uint64_t* bfull = acce + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1u);
      mbar_init(&empty[s], uint32_t(PE));   // every issuer reads every stage
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], uint32_t(PE));
      mbar_init(&acce[i], 8u);
    }
    mbar_init(bfull, 1u);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (threadIdx.x < 64) sBias[threadIdx.x] = a.bias[threadIdx.x];
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmOut) : "memory");
  }
  if (warp == 1) tmem_alloc(tmem_holder, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (warp == 0 && lane == 0) {   // the weights, once
    mbar_expect_tx(bfull, uint32_t(kHaloTaps) * kHaloBBytes);
    for (int t = 0; t < kHaloTaps; ++t) tma_load_2d(sB + t * kHaloBBytes, &tmB, t * BK, 0, bfull);
  }
  pdl_wait();

  const int tpi = (a.H + R - 1) / R;   // tiles per image
  const int total = a.N * tpi;

  if (warp == 0) {
    if (lane == 0) {   // ---- producer: one halo box per tile (the weights came before the wait) ----
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const int n = t / tpi, r0 = (t - n * tpi) * R;
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, a.err, 1u)) break;
        mbar_expect_tx(&full[stage], HALO_BYTES);
        tma_load_4d(sA + stage * HALO_STAGE, &tmA, 0, -1, r0 - 1, n, &full[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1 || warp >= 13) {
    // ---- MMA issuers: issuer mid takes the taps mid, mid + P, ... of every tile ----
    const int mid = warp == 1 ? 0 : warp - 12;
    if (lane == 0 && mid < PE && mbar_wait(bfull, 0u, abort_flag, a.err, 128u)) {
      int stage = 0, it = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t aph = uint32_t(it >> 1) & 1u;
        if (!mbar_wait(&acce[acc], aph ^ 1u, abort_flag, a.err, 2u)) break;
        if (!mbar_wait(&full[stage], phase, abort_flag, a.err, 4u)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t((acc * PE + mid) * 64);
        const uint32_t halo = smem_u32(sA + stage * HALO_STAGE);
        bool first = true;
        for (int tap = mid; tap < kHaloTaps; tap += PE, first = false) {
          const int kh = tap / 3, kw = tap - 3 * (tap / 3);
          const uint32_t win = halo + uint32_t(kh * Wp + kw) * 128u;
          const uint64_t ad = sw128_desc(win);   // the swizzle follows the address bits: no base offset
          const uint64_t bd = sw128_desc(smem_u32(sB + tap * kHaloBBytes));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(d_tmem, ad + uint64_t(kk * 2), bd + uint64_t(kk * 2), idesc, (!first || kk != 0) ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        umma_commit(&accf[acc]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp >= 2 && warp < 10) {
    // ---- epilogue: warp w holds tile pixels 32 (w & 3) .. + 31, channels 32 hsel .. + 31 ----
    const int q = warp & 3, hsel = (warp - 2) >> 2;
    uint8_t* slab = sOut + (warp - 2) * (kOutSlab / 2);
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      const int n = t / tpi, r0 = (t - n * tpi) * R;
      const int acc = it & 1;
      const uint32_t aph = uint32_t(it >> 1) & 1u;
      if (!mbar_wait(&accf[acc], aph, abort_flag, a.err, 8u)) break;
      tc_fence_after();
      float v[32];
      tmem_ld_sum(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * PE * 64 + hsel * 32), PE, 64, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acce[acc]);
        bulk_wait_read0();   // the previous store from this slab has read it
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = v[8 * j + e] + sBias[hsel * 32 + 8 * j + e];
        uint4 qv;
        if (a.act == 1) {
          qv.x = pack_bf16x2_relu(x[0], x[1]);
          qv.y = pack_bf16x2_relu(x[2], x[3]);
          qv.z = pack_bf16x2_relu(x[4], x[5]);
          qv.w = pack_bf16x2_relu(x[6], x[7]);
        } else {
          qv.x = pack_bf16x2(x[0], x[1]);
          qv.y = pack_bf16x2(x[2], x[3]);
          qv.z = pack_bf16x2(x[4], x[5]);
          qv.w = pack_bf16x2(x[6], x[7]);
        }
        *reinterpret_cast<uint4*>(slab + slab64_off(lane, j)) = qv;
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int p0 = q * 32;
        tma_store_4d(&tmOut, hsel * 32, p0 % Wp, r0 + p0 / Wp, n, slab);
        bulk_commit();
      }
    }
    if (lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool encode_2d(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
               uint32_t box_outer, bool f32 = false, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

PFN_cuTensorMapEncodeIm2col_v12000 get_encode_im2col_fn() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
  });
  return fn;
}

// Bounding box of the filter-window corners one output row sweeps: the first corner is -pad, the
// last (Wo-1)*stride - pad; the map encodes the last as an offset from the far edge (W-1).
inline int im2col_upper(int W, int Wo, int s, int pad) { return (Wo - 1) * s - pad - (W - 1); }

// im2col tensor map over the NHWC activation a.x (pitch Cp channels): each load is 128 output
// pixels (traversed W, then H, then N with the conv strides) x `cpp` channels, zero outside.
bool encode_im2col(CUtensorMap* tm, const ConvGemmArgs& a, int cpp) {
  auto fn = get_encode_im2col_fn();
  if (!fn) return false;
  const cuuint64_t eb = a.tf32 ? 4 : 2;
  cuuint64_t dims[4] = {cuuint64_t(a.Cp), cuuint64_t(a.W), cuuint64_t(a.H), cuuint64_t(a.N)};
  cuuint64_t strides[3] = {cuuint64_t(a.Cp) * eb, cuuint64_t(a.W) * a.Cp * eb, cuuint64_t(a.H) * a.W * a.Cp * eb};
  int lower[2] = {-a.pw, -a.ph};
  int upper[2] = {im2col_upper(a.W, a.Wo, a.sw, a.pw), im2col_upper(a.H, a.Ho, a.sh, a.ph)};
  cuuint32_t estr[4] = {1, cuuint32_t(a.sw), cuuint32_t(a.sh), 1};
  CUresult r = fn(tm, a.tf32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                  const_cast<void*>(a.x), dims, strides, lower, upper, cuuint32_t(cpp), cuuint32_t(BM), estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  cpp * eb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The dynamic shared-memory opt-in is a per-device function attribute; it is set while preparing
// a plan (never during stream capture).
template <int BN, int MODE, int PREC>
cudaError_t ensure_attr() {
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (done_mask.load() & bit) return cudaSuccess;
  cudaError_t e =
      cudaFuncSetAttribute(conv_gemm_kernel<BN, MODE, PREC>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  if (e == cudaSuccess) done_mask.fetch_or(bit);
  return e;
}

// Launch with programmatic stream serialisation (the kernel may start before its predecessor in the
// stream has finished; it waits for it after its prologue).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), int grid, int threads, int smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(unsigned(threads));
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <int BN, int MODE, int PREC>
cudaError_t launch_t(const ConvGemmPlan& p, cudaStream_t s) {
  return launch_pdl(conv_gemm_kernel<BN, MODE, PREC>, p.grid, kThreads<MODE, PREC>, p.smem, s, p.tmA, p.tmB, p.tmOut,
                    p.tmRes, p.args);
}

// TF32 / TF32x3 operands use the row-matrix, 16-byte gather and 128-byte im2col modes only.
template <int BN, int PREC>
cudaError_t ensure_attr_f32(int mode) {
  switch (mode) {
    case 0: return ensure_attr<BN, 0, PREC>();
    case 1: return ensure_attr<BN, 1, PREC>();
    case 3: return ensure_attr<BN, 3, PREC>();
    default: return cudaErrorInvalidValue;
  }
}

template <int BN>
cudaError_t ensure_attr_mode(int mode, int prec) {
  if (prec == 1) return ensure_attr_f32<BN, 1>(mode);
  if (prec == 2) return ensure_attr_f32<BN, 2>(mode);
  switch (mode) {
    case 0: return ensure_attr<BN, 0, 0>();
    case 1: return ensure_attr<BN, 1, 0>();
    case 2: return ensure_attr<BN, 2, 0>();
    case 3: return ensure_attr<BN, 3, 0>();
    case 4: return ensure_attr<BN, 4, 0>();
    default: return cudaErrorInvalidValue;
  }
}

template <int BN, int PREC>
cudaError_t launch_f32(const ConvGemmPlan& p, cudaStream_t s) {
  switch (p.mode) {
    case 0: return launch_t<BN, 0, PREC>(p, s);
    case 1: return launch_t<BN, 1, PREC>(p, s);
    case 3: return launch_t<BN, 3, PREC>(p, s);
    default: return cudaErrorInvalidValue;
  }
}

// CTA pairs: clusters of two, with programmatic stream serialisation like the others.
template <int MODE>
cudaLaunchConfig_t pair_config(int grid, int smem, cudaStream_t s, cudaLaunchAttribute (&attr)[2]) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(512u);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cfg;
}

template <int MODE>
cudaError_t launch_pair(const ConvGemmPlan& p, cudaStream_t s) {
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = pair_config<MODE>(p.grid, p.smem, s, attr);
  return cudaLaunchKernelEx(&cfg, conv_pair_kernel<MODE>, p.tmA, p.tmB, p.tmOut, p.tmRes, p.args);
}

// Sets the shared-memory limit of the pair kernel (once per device) and returns how many CTA pairs
// fit on the device at once (0 if the query fails).
template <int MODE>
int pair_setup(int smem, int num_sms) {
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(done_mask.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(conv_pair_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) throw std::runtime_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    done_mask.fetch_or(bit);
  }
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = pair_config<MODE>(2 * (num_sms / 2), smem, nullptr, attr);
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, conv_pair_kernel<MODE>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return clusters;
}

template <int BN>
cudaError_t launch_mode(const ConvGemmPlan& p, cudaStream_t s) {
  if (p.args.tf32) return p.args.x3 ? launch_f32<BN, 2>(p, s) : launch_f32<BN, 1>(p, s);
  switch (p.mode) {
    case 0: return launch_t<BN, 0, 0>(p, s);
    case 1: return launch_t<BN, 1, 0>(p, s);
    case 2: return launch_t<BN, 2, 0>(p, s);
    case 3: return launch_t<BN, 3, 0>(p, s);
    case 4: return launch_t<BN, 4, 0>(p, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int conv_gemm_a_mode(const ConvGemmArgs& a) {
  if (!a.gather) return kARows;
  // TMA im2col: the corner box must fit the map's signed 8-bit corner fields and the tap offsets
  // its 8-bit offset fields; activations under 128 KiB keep the cp.async gather.
  const int up_w = im2col_upper(a.W, a.Wo, a.sw, a.pw), up_h = im2col_upper(a.H, a.Ho, a.sh, a.ph);
  const bool box_ok = a.pw <= 128 && a.ph <= 128 && up_w >= -128 && up_w <= 127 && up_h >= -128 && up_h <= 127 &&
                      (a.KW - 1) * a.dw <= 255 && (a.KH - 1) * a.dh <= 255 && a.sw <= 8 && a.sh <= 8;
  const int eb = a.tf32 ? 4 : 2;
  const bool big = int64_t(a.N) * a.H * a.W * a.Cp * eb >= (int64_t(1) << 17);
  if (box_ok && big) {
    if ((a.Cp * eb) % 128 == 0) return kAIm2col64;   // 128-byte channel blocks
    if (!a.tf32 && a.Cp == 16 && (a.KH * a.KW) % 4 == 0) return kAIm2col16;
  }
  return !a.tf32 && a.Cp == 4 ? kAGather8 : kAGather16;
}

namespace {

__device__ __forceinline__ float act1(float v, int act) {
  switch (act) {
    case 1: return v > 0.f ? v : 0.f;
    case 2: return __fdividef(1.f, 1.f + __expf(-v));
    case 3: return 0.5f * v * (1.f + tanhf(0.79788456080286536f * (v + 0.044715f * v * v * v)));
    case 4: return 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
    default: return v;
  }
}

// One thread per 4 output columns of a row: the slices' partials summed in slice order (a fixed
// order: results do not depend on scheduling), then bias, residual, activation, output type.
__global__ void __launch_bounds__(256) split_reduce_kernel(const float* __restrict__ ws, int ks, int64_t Mp, int64_t M,
                                                           int N, const float* __restrict__ bias,
                                                           const void* __restrict__ res, int res_bf16, int64_t ldr,
                                                           int act, void* __restrict__ out, int out_bf16, int64_t ldo,
                                                           int round_tf32) {
  const int nq = N >> 2;
  const int64_t total = M * nq;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / nq;
    const int n = int(i - m * nq) * 4;
    float4 v = __ldg(reinterpret_cast<const float4*>(bias + n));
    for (int s2 = 0; s2 < ks; ++s2) {
      const float4 p = __ldg(reinterpret_cast<const float4*>(ws + (s2 * Mp + m) * int64_t(N) + n));
      v.x += p.x;
      v.y += p.y;
      v.z += p.z;
      v.w += p.w;
    }
    float o[4] = {v.x, v.y, v.z, v.w};
    if (res) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] += res_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(res)[m * ldr + n + j])
                         : static_cast<const float*>(res)[m * ldr + n + j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[j] = act1(o[j], act);
      if (round_tf32) o[j] = tf32_rna(o[j]);
    }
    if (out_bf16) {
      __nv_bfloat16* op = static_cast<__nv_bfloat16*>(out) + m * ldo + n;
#pragma unroll
      for (int j = 0; j < 4; ++j) op[j] = __float2bfloat16_rn(o[j]);
    } else {
      float* op = static_cast<float*>(out) + m * ldo + n;
#pragma unroll
      for (int j = 0; j < 4; ++j) op[j] = o[j];
    }
  }
}

}  // namespace

cudaError_t conv_gemm_split_reduce(const float* ws, int ks, int64_t Mp, int64_t M, int N, const float* bias,
                                   const void* res, int res_bf16, int64_t ldr, int act, void* out, int out_bf16,
                                   int64_t ldo, int round_tf32, cudaStream_t s) {
  if (N % 4 || (reinterpret_cast<uintptr_t>(ws) & 15u) || (reinterpret_cast<uintptr_t>(bias) & 15u))
    return cudaErrorInvalidValue;
  const int64_t total = M * (N / 4);
  if (total == 0) return cudaSuccess;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  split_reduce_kernel<<<int(blocks), 256, 0, s>>>(ws, ks, Mp, M, N, bias, res, res_bf16, ldr, act, out, out_bf16, ldo,
                                                  round_tf32);
  return cudaGetLastError();
}

int conv_gemm_choose_split(int64_t M, int Cout, int Kpad, int tf32, int x3, int num_sms) {
  const int bke = tf32 ? BK / 2 : BK;
  if (Kpad % bke) return 1;
  const int KT = Kpad / bke;
  // the widest tile conv_gemm_prepare may pick: the fewest tiles, so the split never overfills a wave
  const int bn = Cout <= 64 ? 64 : (Cout <= 128 || x3 ? 128 : 256);
  const int64_t t = ((M + BM - 1) / BM) * ((Cout + bn - 1) / bn);
  // Measured on B200: ResNet-50 bs64's layer-4 convs (50 tiles, 72 or 32 k-tiles) ran no faster in
  // two slices (the CTAs' operand traffic sets the pace) and lost the reduce step (+7 us each);
  // batch-1 ViT-B projections (6-24 tiles) and the bs64 classifier (4 tiles) gained 20-50%. So only
  // tiles filling under a quarter of the SMs are split, into slices of at least four k-tiles.
  if (t * 4 > num_sms || KT < 8 || Cout % 4) return 1;
  int best = 1;
  for (int d = 2; d <= 16 && d <= KT / 4; ++d)
    if (KT % d == 0 && t * d <= num_sms) best = d;
  return best;
}

void conv_gemm_prepare(ConvGemmPlan& p, const void* a_rows, int64_t lda, const void* w, int num_sms) {
  ConvGemmArgs& a = p.args;
  std::memset(&p.tmA, 0, sizeof(p.tmA));
  std::memset(&p.tmB, 0, sizeof(p.tmB));
  std::memset(&p.tmOut, 0, sizeof(p.tmOut));
  std::memset(&p.tmRes, 0, sizeof(p.tmRes));
  // Epilogue: TMA bulk stores when rows and 16-byte chunks are aligned (else direct row stores);
  // a same-dtype, same-shape residual is then streamed into shared memory by the producer warp.
  // split-K (chosen by the caller with conv_gemm_choose_split): the kernel writes raw fp32 partials
  // into `out` [ksplit * Mp, ldo] through the TMA-store epilogue; bias, residual, activation and the
  // output type are conv_gemm_split_reduce's
  const int KSP = a.ksplit > 1 ? a.ksplit : 1;
  if (KSP > 1 && (a.out_bf16 || a.res || a.act || a.round_tf32 || a.group_rows || a.Cout % 4 || a.ldo % 4 ||
                  a.Mp < a.M || a.Mp % BM))
    throw std::runtime_error("conv_gemm: a split-K launch writes plain fp32 partials (caller error)");
  const uint64_t out_rows = KSP > 1 ? uint64_t(KSP) * uint64_t(a.Mp) : uint64_t(a.M);
  const int es = a.out_bf16 ? 2 : 4;
  const int epc = 16 / es;
  const uint32_t sc = a.out_bf16 ? 64 : 32;
  a.epi = 0;
  a.res_slots = 0;
  a.res_slot_bytes = 0;
  const bool out_ok = a.group_rows == 0 && a.Cout % epc == 0 && (a.ldo * es) % 16 == 0 &&
                      (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
  p.mode = conv_gemm_a_mode(a);
  // A bf16 residual of a bf16 conv whose A operand comes by TMA is added by the tensor core (one
  // extra k-tile per 64 channels against an identity operand), which takes the residual off the
  // epilogue's per-element work; otherwise it streams through a shared-memory ring (below) or is
  // read directly by the epilogue.
  const bool res_mma = out_ok && a.res && a.res_mode == 0 && a.res_bf16 && !a.tf32 && !a.x3 &&
                       (p.mode == kARows || p.mode == kAIm2col64) && (a.ldr * 2) % 16 == 0 &&
                       (reinterpret_cast<uintptr_t>(a.res) & 15) == 0;
  a.res_mma = 0;
  const bool res_ring = !res_mma && out_ok && a.res && a.res_mode == 0 && a.res_bf16 == a.out_bf16 &&
                        (a.ldr * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(a.res) & 15) == 0;
  // Tile width: residual convs with a ring use at most 128 columns so two residual tiles fit beside
  // a deep operand pipeline.
  auto tiles = [&](int bn) { return int64_t((a.M + BM - 1) / BM) * ((a.Cout + bn - 1) / bn) * KSP; };
  // (TF32x3 stages hold hi and lo tiles: at most 128 columns so two stages fit)
  int bn = a.Cout <= 64 ? 64 : (a.Cout <= 128 || res_ring || a.x3 ? 128 : 256);
  {
    // The widest tile among those with the fewest waves of persistent CTAs: one tcgen05.mma costs
    // the issuing thread about the same whatever its N (and reads more operand bytes per MAC at a
    // narrower N), so a narrower tile only pays when it cuts
    // the number of waves (measured on ResNet-50 bs64: 1.41 -> 1.39 ms against halving N until
    // every SM has a tile).
    // Among equal wave counts the tile that fills the most SMs wins (ties: the widest): a small batch
    // whose widest tiles occupy a third of the SMs in one wave runs twice as many CTAs at half the
    // width, each also free to use two MMA issuers.
    auto waves = [&](int b) { return (tiles(b) + num_sms - 1) / num_sms; };
    int best = bn;
    for (int b = bn; b >= 64; b /= 2)
      if (waves(b) < waves(best) || (waves(b) == waves(best) && tiles(b) > tiles(best))) best = b;
    bn = best;
  }
  p.bn = bn;
  // Weights stay resident when the conv has one N tile and all its k-tiles fit in 96 KB: every
  // pipeline stage then carries only the activation tile (half the TMA loads for N=64 layers).
  const int bke = a.tf32 ? BK / 2 : BK;   // operand elements per 128-byte k-tile row
  if (a.Kpad % bke) throw std::runtime_error("conv_gemm: reduction length not padded to a whole k-tile");
  const int KT = a.Kpad / bke;
  if (KT % KSP) throw std::runtime_error("conv_gemm: split-K slices must divide the k-tiles");
  // bf16 convs with one or two weight k-tiles (the 1x1 convs from 64 channels, whose epilogue sets
  // the pace) start each accumulator at the bias with one extra MMA, so the epilogue adds none.
  // Measured on ResNet-50 bs512: 1x1 64->64 0.118 -> 0.107 ms, 64->256 -17%, the stage-1 conv with
  // its merged shortcut (two k-tiles) 0.245 -> 0.210 ms; convs with more k-tiles or wider bias tiles
  // lost 1-7% (the extra MMA on the issue path, the bias tile's shared memory).
  const int bias_rows = int((a.Cout + bn - 1) / bn) * bn;
  a.bias_mma = !a.tf32 && !a.x3 && a.bias && KT <= 2 && bias_rows <= 256 && KSP == 1 ? 1 : 0;
  const int64_t w_bytes = int64_t(KT) * bn * 128;
  // ... or when every tile of a CTA has the same N tile (the persistent CTAs step through the tiles
  // by the grid size, so each keeps its N tile when the grid is a multiple of the N-tile count): the
  // CTA's weight columns then stay resident. Measured on ResNet-50 bs512 (A/B on one box): the
  // layer-2 1x1 128->512 convs (two 256-column k-tiles, 64 KB, re-read from L2 for every 128-pixel
  // tile otherwise) 176 -> 156 us; with a 128 KB limit the 512->128 convs lost 15% (three operand
  // stages left) and the layer-3 256->1024 convs did not change, so the limit stays at 96 KB.
  const int tiles_n_est = (a.Cout + bn - 1) / bn;
  const int64_t grid_est = std::min<int64_t>(num_sms, tiles(bn));
  const bool nt_fixed = a.Cout <= bn || (KSP == 1 && grid_est % tiles_n_est == 0);
  const bool bres = !a.x3 && p.mode != kAGather16 && p.mode != kAGather8 && nt_fixed && w_bytes <= 96 * 1024;
  a.b_resident = bres ? 1 : 0;
  // MMA-issuing threads: as many split-K partial accumulators as double-buffered TMEM holds, at
  // most the number of k-tiles.
  const bool gather = p.mode == kAGather16 || p.mode == kAGather8;
  // Measured on ResNet-50: two issuers beat one on N=64/128 im2col tiles (3x3 convs, the stem),
  // four starve on operands, and the row-matrix 1x1 convs lose more to the stage rounding (their
  // residual ring leaves room for only two or three stages) than they gain.
  const bool im2col = p.mode == kAIm2col64 || p.mode == kAIm2col16;
  // Residual convs with a long reduction (>= 8 k-tiles) write their output in place in the residual
  // ring: the output slabs' shared memory becomes a fourth operand stage, which also lets two MMA
  // threads issue. The short ones (HBM-bound) keep separate output slabs, releasing each ring slot
  // without waiting for the stores (measured on ResNet-50: in place there costs 5-6%).
  const bool inplace_hint = res_ring && out_ok && KT >= 8;
  // (the cp.async gather modes have no spare warps: their warps 10-13 gather, so one issuer)
  int pl = !a.x3 && !gather && (im2col || inplace_hint) && bn <= 128 ? 2 : 1;   // X3: warps 13-15 split
  // 64-column im2col convs with 128-byte pixels (ResNet's layer-1 3x3 convs) take four issuers:
  // 0.203 -> 0.196 ms at bs512 (the 16-channel stem lost 10% with four, its epilogue summing them).
  if (pl == 2 && p.mode == kAIm2col64 && bn == 64 && KT >= 4) pl = 4;
  while (pl > 1 && 2 * pl * bn > 512) pl /= 2;
  while (pl > KT / KSP) pl /= 2;   // every issuer's partial gets a k-tile of each slice
  if (gather && pl != 1) throw std::runtime_error("conv_gemm: gather modes have a single MMA issuer");
  a.mma_lanes = pl;
  const int stage_bytes = (BM * 128 + (bres ? 0 : bn * 128)) * (a.x3 ? 2 : 1);
  const int rsb = 128 * bn * es;
  // Output and residual tensor maps first: whether the epilogue stores through TMA and streams the
  // residual through a ring decides the shared-memory plan.
  bool ring = false;
  if (out_ok &&
      encode_2d(&p.tmOut, a.out, uint64_t(a.Cout), out_rows, uint64_t(a.ldo) * es, sc, 32, !a.out_bf16)) {
    a.epi = 2;
    if (res_mma)   // residual k-tiles: 128 rows x 64 channels, the A operand's layout
      a.res_mma = encode_2d(&p.tmRes, a.res, uint64_t(a.Cout), uint64_t(a.M), uint64_t(a.ldr) * 2, 64, 128) ? 1 : 0;
    ring = res_ring && encode_2d(&p.tmRes, a.res, uint64_t(a.Cout), uint64_t(a.M), uint64_t(a.ldr) * es, sc, 128,
                                 !a.out_bf16);
  }
  // Shared memory: operand stages + output slabs + bias + residual ring (two slots when two
  // operand stages still fit beside them). In-place residual convs have no output slabs;
  // otherwise one slab per epilogue warp (a second slab per warp, letting a store drain while the
  // next slab is computed, measured slower on ResNet-50: the operand stages it costs are worth more).
  // bf16 output of 64-column tiles is one 128-byte slab per 32 rows, which would leave one of each
  // TMEM quarter's two epilogue warps idle: it is split into two 32-column halves, one per warp,
  // each stored from its own 64-byte slab through a 32x32 box (not for in-place output, whose slab
  // is the residual ring's 128-byte layout). The halved slabs also leave room for more stages, so
  // wider bf16 tiles take them too when that buys a stage (each warp then stores its 64-column
  // slabs as two 32-column halves through the one 2 KB slab).
  bool wide_half = false;
  auto half_for = [&](int ob) { return a.epi == 2 && a.out_bf16 && ob != 0 && (bn == 64 || wide_half); };
  auto fixed_for = [&](int ob) {
    return int(8 * ob * (half_for(ob) ? kOutSlab / 2 : kOutSlab) + kBiasStage) + 1024 + 512 + (bres ? int(w_bytes) : 0) + (a.res_mma ? int(kIdBytes) : 0) +
           (a.bias_mma ? int(kOnesBytes) + bias_rows * 32 : 0);
  };
  auto ring_for = [&](int ob) {   // residual slots that still leave two operand stages (0: direct reads)
    if (!ring) return 0;
    if ((kSmemLimit - fixed_for(ob) - 2 * rsb) / stage_bytes >= 2) return 2;
    return (kSmemLimit - fixed_for(ob) - rsb) / stage_bytes >= 2 ? 1 : 0;
  };
  auto stages_for = [&](int ob, int rs) { return std::min(kMaxStages, (kSmemLimit - fixed_for(ob) - rs * rsb) / stage_bytes); };
  int ob = ring && KT >= 8 ? 0 : 1;
  int rs = ring_for(ob);
  if (rs == 0 && ob == 0) ob = 1;   // writing in place needs a residual ring
  // Producers and stages. With one MMA issuer the stages are consumed in order, and at least as
  // many stages as producers keeps every barrier wait within one phase. With several issuers the
  // stage count must be a multiple of both counts (one producer and one consumer per stage).
  // Prefer three or four producers (TMA issue rate), then the deepest ring.
  auto lcm = [](int x, int y) { int g = x, h = y; while (h) { int r = g % h; g = h; h = r; } return x / g * y; };
  auto split_stages = [&](int smax, int& np, int& stages) {
    np = 1;
    stages = (smax / pl) * pl;
    if (!gather && pl == 1) {
      np = std::min(3, smax);
      stages = smax;
    } else if (!gather) {
      int best_np = 0, best_s = 0;
      for (int q : {3, 4, 2, 1}) {
        const int l = lcm(q, pl);
        const int s_q = (smax / l) * l;
        if (s_q < std::max(2, l)) continue;
        if (best_np == 0 || (std::min(q, 3) > std::min(best_np, 3)) ||
            (std::min(q, 3) == std::min(best_np, 3) && s_q > best_s)) {
          best_np = q;
          best_s = s_q;
        }
      }
      if (best_np == 0) throw std::runtime_error("conv_gemm: no producer/stage split fits shared memory");
      np = best_np;
      stages = best_s;
    }
  };
  int np = 1, stages = 0;
  split_stages(stages_for(ob, rs), np, stages);
  // Half slabs for wider bf16 tiles when the pipeline is shallow and they buy a stage. Measured on
  // ResNet-50 bs512 (A/B on one box): 3 -> 4 stages (the 256-column layer-3/4 convs) -7 to -10%, the
  // layer-2 3x3 convs (4 stages of 4 producers -> 6 of 3) -12%; where five or more stages fit already
  // the extra stage gains nothing and the four half stores per tile cost up to 25%.
  if (bn > 64 && a.epi == 2 && a.out_bf16 && ob != 0 && stages < 5) {
    wide_half = true;
    int np2 = 0, st2 = 0;
    if (ring_for(ob) == rs) split_stages(stages_for(ob, rs), np2, st2);
    if (st2 > stages) {
      np = np2;
      stages = st2;
    } else {
      wide_half = false;
    }
  }
  a.producers = np;
  if (stages < 2) throw std::runtime_error("conv_gemm: shared-memory plan leaves fewer than 2 stages");
  const int fixed = fixed_for(ob);
  a.out_bufs = ob;
  a.epi_half = 0;
  if (half_for(ob)) {
    if (!encode_2d(&p.tmOut, a.out, uint64_t(a.Cout), out_rows, uint64_t(a.ldo) * es, 32, 32, false,
                   CU_TENSOR_MAP_SWIZZLE_64B))
      throw std::runtime_error("conv_gemm: output tensor map (32x32 box) rejected");
    a.epi_half = 1;
  }
  if (KSP > 1 && a.epi != 2) throw std::runtime_error("conv_gemm: split-K partials need the TMA-store epilogue");
  a.stages = stages;
  p.smem = stages * stage_bytes + fixed + rs * rsb;
  int64_t t = tiles(bn);
  p.grid = int(t < num_sms ? t : num_sms);
  const int eb = a.tf32 ? 4 : 2;
  if (a.x3 && (a.w_lo_row < a.Cout || a.w_lo_row % bn))
    throw std::runtime_error("conv_gemm: TF32x3 weights need their lo rows after a BN-padded hi block");
  bool ok = encode_2d(&p.tmB, w, uint64_t(a.Kpad), uint64_t(a.x3 ? 2 * a.w_lo_row : a.Cout), uint64_t(a.Kpad) * eb,
                      uint32_t(bke), uint32_t(bn), a.tf32 != 0);
  if (p.mode == kARows)
    ok = ok && encode_2d(&p.tmA, a_rows, uint64_t(lda), uint64_t(a.M), uint64_t(lda) * eb, uint32_t(bke), BM, a.tf32 != 0);
  if (a.a2) {   // second A operand: a row matrix like the first, through the (then unused) tmRes map
    if (p.mode != kARows || a.res || a.a2_kt <= 0 || a.a2_kt >= KT)
      throw std::runtime_error("conv_gemm: a second A operand needs row-matrix A, no residual, a split inside K");
    if (a.a2_s > 0) {   // an NHWC image read at stride a2_s: im2col map of a 1x1 conv, no padding
      ConvGemmArgs t = a;
      t.x = a.a2;
      t.H = a.a2_H;
      t.W = a.a2_W;
      t.Cp = int(a.lda2);
      t.KH = t.KW = 1;
      t.sh = t.sw = a.a2_s;
      t.ph = t.pw = 0;
      t.dh = t.dw = 1;
      if (!encode_im2col(&p.tmRes, t, bke))
        throw std::runtime_error("cuTensorMapEncodeIm2col failed for the second A operand");
    } else {
      ok = ok && encode_2d(&p.tmRes, a.a2, uint64_t(a.lda2), uint64_t(a.M), uint64_t(a.lda2) * eb, uint32_t(bke), BM,
                           a.tf32 != 0);
    }
  }
  if (!ok) throw std::runtime_error("cuTensorMapEncodeTiled failed (driver entry point missing or bad layout)");
  if ((p.mode == kAIm2col64 || p.mode == kAIm2col16) && !encode_im2col(&p.tmA, a, p.mode == kAIm2col64 ? bke : 16))
    throw std::runtime_error("cuTensorMapEncodeIm2col failed (driver entry point missing or bad layout)");
  a.res_slots = rs;
  a.res_slot_bytes = rs ? rsb : 0;
  const int mode = p.mode;
  const int prec = a.tf32 ? (a.x3 ? 2 : 1) : 0;
  cudaError_t e = bn == 64 ? ensure_attr_mode<64>(mode, prec)
                           : (bn == 128 ? ensure_attr_mode<128>(mode, prec) : ensure_attr_mode<256>(mode, prec));
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  // CTA pairs for the 256-column bf16 tiles that stream their weights (no residual or one the tensor
  // core adds, a merged projection shortcut's second operand or none, no split): each SM loads and
  // reads half of every weight k-tile.
  p.pair = 0;
  const int64_t pair_tiles = int64_t((a.M + 2 * BM - 1) / (2 * BM)) * ((a.Cout + 255) / 256);
  if (bn == 256 && !a.tf32 && (p.mode == kARows || p.mode == kAIm2col64) && (!a.res || a.res_mma) &&
      KSP == 1 && a.epi == 2 && a.out_bf16 && a.group_rows == 0 && !a.bias_mma && !bres && num_sms >= 2) {
    const int fixed_pair = int(8 * (a.epi_half ? kOutSlab / 2 : kOutSlab)) + (a.res_mma ? int(kIdBytes / 2) : 0) + 1024 + 512;
    const int st = std::min(kMaxStages, (kSmemLimit - fixed_pair) / int(kPairStage));
    const int smem_pair = st * int(kPairStage) + fixed_pair;
    const int clusters = st >= 2 ? (p.mode == kARows ? pair_setup<0>(smem_pair, num_sms) : pair_setup<3>(smem_pair, num_sms)) : 0;
    if (clusters >= 1 && encode_2d(&p.tmB, w, uint64_t(a.Kpad), uint64_t(a.Cout), uint64_t(a.Kpad) * 2, uint32_t(bke),
                                   128, false)) {
      p.pair = 1;
      a.stages = st;
      a.producers = 1;
      a.mma_lanes = 1;
      a.out_bufs = 1;
      p.smem = smem_pair;
      p.grid = int(2 * std::min<int64_t>(std::min(clusters, num_sms / 2), pair_tiles));
    }
  }
}

int conv3x3_tile_width(int H, int W) {
  int Wp = 1;
  while (Wp < W + 2) Wp <<= 1;
  if (Wp > BM) return 0;
  const int R = BM / Wp;
  const int tiles = (H + R - 1) / R;
  // at least 70% of the computed pixels are real ones (a 7-row map in 8-row tiles is not worth it)
  if (double(H) * W < 0.7 * double(tiles) * R * Wp) return 0;
  return Wp;
}

void conv3x3_prepare(Conv3x3Plan& p, const void* w, int num_sms) {
  Conv3x3Args& a = p.args;
  std::memset(&p.tmA, 0, sizeof(p.tmA));
  std::memset(&p.tmB, 0, sizeof(p.tmB));
  std::memset(&p.tmOut, 0, sizeof(p.tmOut));
  auto fn = get_encode_fn();
  if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled entry point missing");
  cuuint64_t dims[4] = {64, cuuint64_t(a.W), cuuint64_t(a.H), cuuint64_t(a.N)};
  cuuint64_t strides[3] = {128, cuuint64_t(a.W) * 128, cuuint64_t(a.H) * a.W * 128};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  cuuint32_t box_in[4] = {64, cuuint32_t(a.Wp), cuuint32_t(a.R + 2), 1};
  CUresult r = fn(&p.tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(a.x), dims, strides, box_in, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed for the 3x3 halo input");
  const cuuint32_t spx = cuuint32_t(std::min(a.Wp, 32));
  cuuint32_t box_out[4] = {32, spx, 32 / spx, 1};
  r = fn(&p.tmOut, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a.out, dims, strides, box_out, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed for the 3x3 halo output");
  if (!encode_2d(&p.tmB, w, uint64_t(kHaloTaps) * BK, 64, uint64_t(kHaloTaps) * BK * 2, BK, 64))
    throw std::runtime_error("cuTensorMapEncodeTiled failed for the 3x3 weights");
  a.mma_lanes = 4;
  const int fixed = int(kHaloTaps * kHaloBBytes + 8 * (kOutSlab / 2)) + 256 + 1024 + 512;
  const int stage = int(halo_stage_bytes(a.Wp, a.R));
  int stages = std::min(kMaxStages, (kSmemLimit - fixed) / stage);
  if (stages < 2) throw std::runtime_error("conv3x3: shared-memory plan leaves fewer than 2 stages");
  a.stages = stages;
  p.smem = stages * stage + fixed;
  const int64_t tiles = int64_t(a.N) * ((a.H + a.R - 1) / a.R);
  p.grid = int(std::min<int64_t>(num_sms, tiles));
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(done_mask.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(conv3x3_halo_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) throw std::runtime_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    done_mask.fetch_or(bit);
  }
}

cudaError_t conv3x3_launch(const Conv3x3Plan& p, cudaStream_t s) {
  return launch_pdl(conv3x3_halo_kernel, p.grid, 512, p.smem, s, p.tmA, p.tmB, p.tmOut, p.args);
}

bool stem_pool_supported(int Cout, int Ho, int Wo, int KH, int KW) {
  return Cout == 64 && Wo <= BM && Ho % 2 == 0 && Wo % 2 == 0 && KH == 4 && KW == 4;
}

void stem_pool_prepare(StemPoolPlan& p, const void* w, int num_sms) {
  StemPoolArgs& a = p.args;
  std::memset(&p.tmA, 0, sizeof(p.tmA));
  std::memset(&p.tmB, 0, sizeof(p.tmB));
  auto fn = get_encode_fn();
  if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled entry point missing");
  // the space-to-depth image as a 4D tensor (channel, x, y, image); one box = one input row of
  // 131 pixels x 16 channels, 32-byte rows swizzled as the K=16 MMA sub-tiles expect
  cuuint64_t dims[4] = {16, cuuint64_t(a.Ws), cuuint64_t(a.Hs), cuuint64_t(a.N)};
  cuuint64_t strides[3] = {32, cuuint64_t(a.Ws) * 32, cuuint64_t(a.Hs) * a.Ws * 32};
  cuuint32_t box[4] = {16, uint32_t(kStemRowPx), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(&p.tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(a.x), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed for the stem input");
  if (!encode_2d(&p.tmB, w, uint64_t(kStemKT) * BK, 64, uint64_t(kStemKT) * BK * 2, BK, 64))
    throw std::runtime_error("cuTensorMapEncodeTiled failed for the stem weights");
  // four MMA issuers taking every fourth conv row (ResNet-50 bs512: 457 us with two, 320 with four;
  // an issuer waits on its row's loads and accumulator between rows); one TMA producer (a 4 KB input
  // row per conv row)
  a.mma_lanes = 4;
  a.producers = 1;
  a.stages = kStemRing;
  p.smem = int(kStemKT * kStemBBytes + kStemRing * kStemSlot) + 256 + 1024 + 512 + 1024;
  const int64_t pool_rows = int64_t(a.N) * (a.Ho / 2);
  p.grid = int(std::min<int64_t>(num_sms, pool_rows));
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(done_mask.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(stem_pool_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) throw std::runtime_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    done_mask.fetch_or(bit);
  }
}

cudaError_t stem_pool_launch(const StemPoolPlan& p, cudaStream_t s) {
  return launch_pdl(stem_pool_kernel, p.grid, 512, p.smem, s, p.tmA, p.tmB, p.args);
}

std::string conv_gemm_describe(const ConvGemmPlan& p) {
  static const char* kModes[] = {"tma", "gather", "gather8", "im2col", "im2col16"};
  const ConvGemmArgs& a = p.args;
  const char* res = !a.res ? "none" : a.res_mma ? "mma" : a.res_slots ? "ring" : "direct";
  char buf[320];
  std::snprintf(buf, sizeof(buf),
                "M=%d N=%d K=%d mode=%s%s bn=%d%s grid=%d stages=%d producers=%d issuers=%d residual=%s%s "
                "out_slabs=%d%s weights=%s bias=%s split=%d smem=%d",
                a.M, a.Cout, a.Kpad, kModes[p.mode], a.x3 ? " tf32x3" : (a.tf32 ? " tf32" : ""), p.bn,
                p.pair ? " (CTA pairs)" : "", p.grid, a.stages,
                a.producers, a.mma_lanes, res, a.res_slots ? (a.res_slots == 2 ? " x2" : " x1") : "", a.out_bufs,
                a.epi_half ? " (half slabs)" : "", a.b_resident ? "resident" : "streamed", a.bias_mma ? "mma" : "epilogue",
                a.ksplit > 1 ? a.ksplit : 1, p.smem);
  return buf;
}

cudaError_t conv_gemm_launch(const ConvGemmPlan& p, cudaStream_t s) {
  if (p.pair) return p.mode == kARows ? launch_pair<0>(p, s) : launch_pair<3>(p, s);
  switch (p.bn) {
    case 64: return launch_mode<64>(p, s);
    case 128: return launch_mode<128>(p, s);
    case 256: return launch_mode<256>(p, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace k
}  // namespace sb
