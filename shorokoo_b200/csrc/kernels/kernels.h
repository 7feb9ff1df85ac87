// Launch interface of the sm_100a kernels. Plain pointers and sizes only; every launcher takes the
// stream to run on. Implementations: conv_gemm.cu (tcgen05 tensor-core path), misc.cu (memory-bound).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <string>

namespace sb {
namespace k {

// ---- tensor-core implicit GEMM --------------------------------------------------------------
// D[m, n] = act( sum_k A[m, k] * B[n, k] + bias[n] (+ residual[m, n]) )
//   A = rows of a bf16 matrix (mode TMA) or the im2col of an NHWC bf16 activation (mode GATHER);
//   B = bf16 weights [Cout, Kpad], K-major, K ordered (kh, kw, c) to match NHWC im2col.
struct ConvGemmArgs {
  // geometry of the A operand
  int gather;              // 0: A rows via TMA (lda = Kpad elements); 1: im2col from NHWC
  const void* x;           // NHWC bf16 [N, H, W, Cp] (im2col)
  int N, H, W, Cp;
  int Ho, Wo, KH, KW, sh, sw, ph, pw, dh, dw;
  int M;                   // rows of D (N*Ho*Wo for convs)
  int Cout;                // columns of D
  int Kpad;                // padded reduction length (multiple of 64)
  const float* bias;       // [round_up(Cout, BN)] f32, zero padded (never null)
  // residual operand
  const void* res;         // null if none
  int res_bf16;            // 1: bf16, 0: f32
  int64_t ldr;             // elements between residual rows
  int res_mode;            // 0: row m; 1: nearest-2x upsample source (Hr = Ho/2, Wr = Wo/2 rounded up)
  int Hr, Wr;
  // output
  void* out;
  int out_bf16;
  int64_t ldo;             // elements between output rows
  int64_t group_rows;      // rows per output group (0 = contiguous rows)
  int64_t group_stride;    // elements between output groups
  int act;                 // 0 none, 1 relu, 2 sigmoid
  unsigned int* err;       // device error word (bounded-wait timeouts)
  // set by conv_gemm_prepare:
  int epi;                 // epilogue: 0 direct row stores, 2 TMA bulk stores from smem slabs
  int stages;              // operand pipeline depth
  int res_slots;           // residual ring slots filled by the producer warp (0: direct residual reads)
  int res_slot_bytes;
  int out_bufs;            // output slabs per epilogue warp: 1, or 0 when the output is written in
                           // place over the residual ring
  const void* a2;          // second A operand (a row matrix like the first, row mode only) supplying
                           // k-tiles a2_kt.. (a merged projection shortcut's input), or null
  int64_t lda2;            // its row pitch in elements
  int a2_kt;               // first k-tile read from a2 (k-tile kt reads its k-tile kt - a2_kt)
  int a2_s;                // 0: a2 is a row matrix [M, lda2]; s > 0: a2 is an NHWC image
                           // [N, a2_H, a2_W, lda2] read at stride s (output pixel (ho, wo) -> (s ho, s wo))
  int a2_H, a2_W;
  int res_mma;             // 1: the tensor core adds the bf16 residual: after the tile's k-tiles come
                           // one k-tile per 64 residual channels, A = the residual rows (TMA), B = a
                           // 64x64 identity in shared memory, accumulated into those 64 columns
  int bias_mma;            // 1: the tensor core starts every accumulator at the bias: one K=16 MMA of
                           // a ones tile (A) and the bias split into bf16 hi + lo (B) per tile
  int epi_half;            // 1: bf16 output of 64-column tiles; each of a TMEM quarter's two epilogue
                           // warps stores its own 32-column half (64-byte swizzled slab, 32x32 box)
  int b_resident;          // 1: every weight k-tile is loaded once and stays in shared memory
  int mma_lanes;           // MMA-issuing threads P (1, 2 or 4, one per warp): issuer p accumulates
                           // the k-tiles g = p mod P into its own partial accumulator
  int tf32;                // 0: bf16 operands (kind::f16, 64 per k-tile row); 1: fp32 operands
                           // multiplied as TF32 (kind::tf32, 32 per 128-byte k-tile row)
  int round_tf32;          // fp32 output rounded to the TF32 grid (it feeds TF32 MMAs)
  int x3;                  // with tf32: error-compensated TF32 (hi*hi + hi*lo + lo*hi per K slice)
  int w_lo_row;            // x3: row of the weights' lo matrix (hi rows 0..Cout-1, zero to w_lo_row)
  int producers;           // TMA producer threads Q (1-4): thread q loads k-tiles g = q mod Q
                           // (stages is a multiple of P and Q, so every stage has one producer
                           // and one consumer, each in order)
  int ksplit;              // > 1: split-K over CTAs. Tile (m, n) is computed as ksplit slices of
                           // Kpad / ksplit each; slice s writes its raw fp32 partial (no bias,
                           // residual or activation) to rows s * Mp + m of `out` [ksplit * Mp, ldo]
                           // and conv_gemm_split_reduce finishes the output. 0 or 1: no split.
  int Mp;                  // ksplit > 1: rows per slice in `out` (M rounded up to 128)
};

// Slices for split-K: the largest divisor of the k-tile count that keeps the (estimated) tiles in
// one wave of the SMs, or 1 when the tiles already fill half the SMs or K is short.
int conv_gemm_choose_split(int64_t M, int Cout, int Kpad, int tf32, int x3, int num_sms);
// y[m, n] = act(sum_s ws[s * Mp + m, n] + bias[n] (+ res[m, n])) for m < M, n < N (N a multiple of
// 4), stored as bf16, fp32 or fp32 on the TF32 grid with row pitch ldo (res: bf16 or fp32, pitch ldr).
cudaError_t conv_gemm_split_reduce(const float* ws, int ks, int64_t Mp, int64_t M, int N, const float* bias,
                                   const void* res, int res_bf16, int64_t ldr, int act, void* out, int out_bf16,
                                   int64_t ldo, int round_tf32, cudaStream_t s);

// How the kernel fetches its A operand (chosen from the geometry by conv_gemm_a_mode):
//   0  A is a row matrix: 2D TMA tiles
//   1  im2col by cp.async in 16-byte units (Cp % 8 == 0)
//   2  im2col by cp.async in 8-byte units (Cp == 4)
//   3  im2col by TMA (im2col tensor map, 64 channels x 128 output pixels per load; Cp % 64 == 0)
//   4  im2col by TMA, 16 channels x 128 pixels per load, four taps per k-tile (Cp == 16)
enum ConvAMode { kARows = 0, kAGather16 = 1, kAGather8 = 2, kAIm2col64 = 3, kAIm2col16 = 4 };
int conv_gemm_a_mode(const ConvGemmArgs& a);

struct ConvGemmPlan {
  CUtensorMap tmA;   // 2D tiles (mode 0) or im2col map (modes 3, 4)
  CUtensorMap tmB;
  CUtensorMap tmOut;   // valid when args.epi == 2
  CUtensorMap tmRes;   // valid when args.res_slots > 0
  int bn;            // 64, 128 or 256
  int pair;          // 1: CTA pairs (clusters of two) compute 256 x 256 tiles with cta_group::2 MMAs
  int mode;          // ConvAMode
  int grid;
  int smem;
  ConvGemmArgs args;
};

// Builds tensor maps and the launch shape. `a_rows` is the A matrix base (TMA mode) with leading
// dimension `lda` elements; `w` the weight matrix [Cout_rows >= Cout, Kpad]. Returns false when the
// driver entry point for tensor-map encoding is unavailable.
void conv_gemm_prepare(ConvGemmPlan& p, const void* a_rows, int64_t lda, const void* w, int num_sms);
cudaError_t conv_gemm_launch(const ConvGemmPlan& p, cudaStream_t s);
// One line with the launch shape and pipeline choices of a prepared plan (debug output).
std::string conv_gemm_describe(const ConvGemmPlan& p);

// ---- stem convolution with its 3x3/2 max pool fused into the epilogue (conv_gemm.cu) ----------
// y = maxpool3x3/2,pad1( act( conv(x) + bias ) ) for the ResNet stem run as a 4x4 stride-1 conv over
// the 2x2 space-to-depth image x (NHWC bf16 [N, Hs, Ws, 16]); weights bf16 [64, 256] with K ordered
// (filter column b, filter row a, channel c); y NHWC bf16 [N, Ho/2, Wo/2, 64]. Requires Cout = 64,
// Wo <= 128, Ho and Wo even. The conv output itself is never written to global memory.
struct StemPoolArgs {
  const void* x;
  int N, Hs, Ws;           // space-to-depth image
  int Ho, Wo;              // conv output (before pooling)
  int ph, pw;              // conv padding in space-to-depth pixels
  const float* bias;       // [64] f32
  void* out;               // [N, Ho/2, Wo/2, 64] bf16
  int act;                 // 0 none, 1 relu
  unsigned int* err;
  // set by stem_pool_prepare:
  int stages, producers, mma_lanes;
};
struct StemPoolPlan {
  CUtensorMap tmA;   // 4D tiled map of x: box 16 channels x 131 pixels x 1 row
  CUtensorMap tmB;   // weights, 64 x 64 boxes (one k-tile)
  int grid, smem;
  StemPoolArgs args;
};
bool stem_pool_supported(int Cout, int Ho, int Wo, int KH, int KW);
void stem_pool_prepare(StemPoolPlan& p, const void* w, int num_sms);
cudaError_t stem_pool_launch(const StemPoolPlan& p, cudaStream_t s);

// ---- 3x3 / stride 1 / pad 1 convolution from halo tiles (conv_gemm.cu) ---------------------------
// y = act(conv3x3(x) + bias) over NHWC bf16 x [N, H, W, 64] with 64 output channels, y NHWC bf16.
// A tile is R output rows x Wp pixels (Wp the power of two >= W + 2, R = 128 / Wp; pixels past W and
// rows past H are computed and dropped): one 4D TMA box loads the tile's (R + 2) x Wp input halo
// (zero outside the image) and the nine taps read it through shared-memory descriptors shifted by
// kh * Wp + kw rows, instead of nine im2col loads. Weights bf16 [64, 576], K ordered (kh, kw, c).
struct Conv3x3Args {
  const void* x;
  int N, H, W;
  int Wp, R;               // tile geometry
  const float* bias;       // [64]
  void* out;
  int act;                 // 0 none, 1 relu
  unsigned int* err;
  // set by conv3x3_prepare:
  int stages, mma_lanes;
};
struct Conv3x3Plan {
  CUtensorMap tmA;   // 4D tiled map of x, box 64 channels x Wp pixels x (R + 2) rows
  CUtensorMap tmB;   // weights, 64 x 64 boxes
  CUtensorMap tmOut; // 4D tiled map of y, box 32 channels x min(32, Wp) pixels x rows
  int grid, smem;
  Conv3x3Args args;
};
// The tile width for an output width W (0 when none fits: W + 2 > 128 or too few valid pixels).
int conv3x3_tile_width(int H, int W);
void conv3x3_prepare(Conv3x3Plan& p, const void* w, int num_sms);
cudaError_t conv3x3_launch(const Conv3x3Plan& p, cudaStream_t s);

// ---- memory-bound kernels (misc.cu) ------------------------------------------------------------
constexpr int kMaxRank = 8;
struct TDesc {
  int rank;
  int64_t shape[kMaxRank];
  int64_t stride[kMaxRank];   // elements
};

// dst (NHWC bf16 [N,H,W,Cp]) <- src logical [N,C,H,W] with arbitrary strides, f32 or bf16; channels
// C..Cp-1 are zero.
cudaError_t to_nhwc_bf16(const void* src, int src_bf16, const int64_t* shape4, const int64_t* stride4,
                         void* dst, int Cp, cudaStream_t s);
// 2x2 space-to-depth: dst (NHWC bf16 [N, Hs, Ws, 16]) <- src logical [N, C<=4, H, W] (any strides):
// dst[n, hs, ws, (p*2+q)*C + c] = src[n, c, 2hs+p, 2ws+q], zero outside the image and in channels 4C..15.
cudaError_t to_s2d_bf16(const void* src, int src_bf16, const int64_t* shape4, const int64_t* stride4, void* dst,
                        int64_t Hs, int64_t Ws, cudaStream_t s);
// The same conversions into fp32 operands for the TF32 paths: NHWC fp32 [N,H,W,Cp] (Cp % 4 == 0)
// and rows fp32 [M, Kp]; values rounded to the TF32 grid when round_tf32 (single-pass TF32), kept
// exact for TF32x3.
cudaError_t to_nhwc_f32(const void* src, int src_bf16, const int64_t* shape4, const int64_t* stride4, void* dst,
                        int Cp, int round_tf32, cudaStream_t s);
cudaError_t to_rows_f32(const void* src, int src_bf16, int64_t M, int64_t K, int64_t sm, int64_t sk, void* dst,
                        int64_t Kp, int round_tf32, cudaStream_t s);
// NHWC fp32 max pooling (C % 4 == 0).
cudaError_t maxpool_nhwc_f32(const void* x, void* y, int N, int H, int W, int C, int Ho, int Wo, int kh, int kw,
                             int sh, int sw, int ph, int pw, int dh, int dw, cudaStream_t s);
// dst (bf16 [M, Kp]) <- src logical [M, K] with arbitrary strides; columns K..Kp-1 zero.
cudaError_t to_rows_bf16(const void* src, int src_bf16, int64_t M, int64_t K, int64_t sm, int64_t sk,
                         void* dst, int64_t Kp, cudaStream_t s);
// NHWC bf16 max pooling (padding never wins: out-of-range taps are skipped).
cudaError_t maxpool_nhwc_bf16(const void* x, void* y, int N, int H, int W, int C, int Ho, int Wo, int kh,
                              int kw, int sh, int sw, int ph, int pw, int dh, int dw, cudaStream_t s);
// NHWC (bf16 or f32 with C contiguous, pixel stride ldp) -> [N, C] mean or max, bf16 or f32 output.
// Fused attention (attention.cu): y[b, h, s, :] = softmax(scale q k^T) v over q, k, v
// [B, H, S, hd] strided views (head dim contiguous, 16-byte aligned rows), bf16 or fp32 (read as
// bf16), S <= 256 and hd = 64; y written at out + b os[0] + h os[1] + s os[2] as bf16 (out_mode 0),
// fp32 on the TF32 grid (1) or fp32 (2).
struct AttentionArgs {
  const void* q;
  const void* k;
  const void* v;
  int64_t qs[3], ks[3], vs[3];   // element strides of the batch, head and sequence axes
  int in_f32;
  int S, hd;
  float scale;
  void* out;
  int64_t os[3];
  int out_mode;
  unsigned int* err;
};
bool attention_supported(int S, int hd);
void attention_prepare();   // once per device, before the first launch (shared-memory attribute)
cudaError_t attention(const AttentionArgs& a, int B, int H, cudaStream_t s);

// Row-wise layer normalisation (norm.cu): y[r, :] = (x[r, :] - mean) / sqrt(var + eps) * gamma +
// beta over the last axis of D features, x fp32 rows of pitch ldx, y with pitch ldy as bf16
// (y_mode 0), fp32 on the TF32 grid (1) or fp32 (2).
cudaError_t layer_norm(const float* x, int64_t rows, int D, int64_t ldx, float eps, const float* gamma,
                       const float* beta, void* y, int y_mode, int64_t ldy, cudaStream_t s);

// Group normalisation over NHWC x [N, HW, ldc] (bf16 or fp32; C channels in G groups, C / G <= 64,
// C a multiple of the 16-byte vector with C / vector dividing 256): y = act(((x - mean) * rstd) *
// gamma + beta) per (n, group), stored with pitch ldy as bf16 (y_mode 0), fp32 on the TF32 grid (1)
// or fp32 (2). Scratch: partial [N * per_img * 2 * C] and ab [N * 2 * C] floats (norm.cu).
bool group_norm_supported(int C, int G, int x_bf16);
int group_norm_blocks_per_image(int N, int64_t HW, int num_sms);
cudaError_t group_norm(const void* x, int x_bf16, int N, int64_t HW, int C, int64_t ldc, int G, float eps,
                       const float* gamma, const float* beta, void* y, int y_mode, int64_t ldy, int relu, int per_img,
                       float* partial, float* ab, cudaStream_t s);
cudaError_t global_pool_nhwc(const void* x, int x_bf16, int N, int HW, int C, int64_t ldp, void* y, int y_bf16,
                             int is_max, cudaStream_t s);
// Generic strided copy with dtype conversion: dst[idx] = src[idx] over `shape`.
cudaError_t strided_copy(const void* src, int src_bf16, const TDesc& sd, void* dst, int dst_bf16, const TDesc& dd,
                         cudaStream_t s);
cudaError_t fill_f32(void* dst, int64_t n, float v, cudaStream_t s);
// dst f32 [n] <- src IEEE half [n] (16-byte aligned buffers: 8 halves per thread and step).
cudaError_t f16_to_f32(const void* src, void* dst, int64_t n, cudaStream_t s);
// dst f32 [n] <- src bfloat16 [n] (exact widening; 16-byte aligned buffers).
cudaError_t bf16_to_f32(const void* src, void* dst, int64_t n, cudaStream_t s);
// Elementwise: y (f32 contiguous over out shape) = f(a [, b]) with broadcasting strides.
enum EwOp : int {
  EW_ADD = 0, EW_SUB, EW_MUL, EW_DIV, EW_POW, EW_MAX, EW_MIN,
  EW_RELU = 16, EW_SIGMOID, EW_TANH, EW_SQRT, EW_NEG, EW_ABS, EW_EXP, EW_LOG, EW_RECIP, EW_FLOOR, EW_CEIL,
  EW_ERF, EW_LEAKY, EW_CLIP, EW_IDENT, EW_GELU, EW_GELU_TANH
};
cudaError_t elementwise(int op, const void* a, int a_bf16, const TDesc& ad, const void* b, int b_bf16,
                        const TDesc& bd, void* y, int y_bf16, const TDesc& yd, float alpha, float beta,
                        cudaStream_t s);
// Softmax over `len` elements spaced `inner` apart, for outer*inner independent rows; f32 in/out
// contiguous.
cudaError_t softmax(const float* x, float* y, int64_t outer, int64_t len, int64_t inner, cudaStream_t s);
// Reduce over the middle axis of a contiguous [outer, len, inner] f32 view. kind: 0 sum, 1 mean, 2 max.
cudaError_t reduce_mid(const float* x, float* y, int64_t outer, int64_t len, int64_t inner, int kind, cudaStream_t s);
// Gather along every axis with per-axis index tables (nearest Resize):
// y[o] = x[sum_d table_d[o_d] * xd.stride[d]]; `tables` holds the per-axis tables back to back
// (table_d has yd.shape[d] entries).
cudaError_t gather_axes(const void* x, int x_bf16, const TDesc& xd, const int64_t* tables, void* y, int y_bf16,
                        const TDesc& yd, cudaStream_t s);

}  // namespace k
}  // namespace sb
