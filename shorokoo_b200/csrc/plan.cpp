// Plan construction: layout / dtype selection, conversion insertion, weight packing, arena
// allocation (liveness + best fit), launch closures and CUDA-graph capture.
//
// Layout policy: activations that feed tensor-core or pooling kernels are stored NHWC bf16 (channel
// contiguous, so an im2col row of one filter tap is a contiguous 128-byte run), or NHWC fp32 rounded
// to the TF32 grid in the TF32 accuracy mode; everything a generic op or a graph output reads is
// fp32. Reshape / Transpose / Slice / Expand are stride views when the
// memory permits (the NHWC conv output of a RetinaNet head makes its Reshape->Transpose chain a pure
// view), otherwise a strided copy materialises them.
#include "plan.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <cstdio>
#include <map>
#include <numeric>
#include <optional>

namespace sb {

namespace {

constexpr size_t kAlign = 256;

std::vector<int64_t> contig_strides(const std::vector<int64_t>& s) {
  std::vector<int64_t> st(s.size());
  int64_t acc = 1;
  for (int i = int(s.size()) - 1; i >= 0; --i) {
    st[size_t(i)] = acc;
    acc *= std::max<int64_t>(s[size_t(i)], 1);
  }
  return st;
}

bool is_contig(const DevTensor& t) {
  auto c = contig_strides(t.shape);
  for (size_t i = 0; i < t.shape.size(); ++i)
    if (t.shape[i] != 1 && t.strides[i] != c[i]) return false;
  return true;
}

// Strides for viewing (shape, strides) as new_shape without copying, if possible (the stride
// bookkeeping of a reshape over non-contiguous memory: dims are grouped into runs that are
// contiguous with respect to each other, and every run must split/merge exactly).
std::optional<std::vector<int64_t>> view_strides(const std::vector<int64_t>& shape, const std::vector<int64_t>& strides,
                                                 const std::vector<int64_t>& new_shape) {
  if (numel(shape) == 0) return contig_strides(new_shape);
  // drop size-1 dims of the source; they do not constrain the view
  std::vector<int64_t> s, st;
  for (size_t i = 0; i < shape.size(); ++i)
    if (shape[i] != 1) {
      s.push_back(shape[i]);
      st.push_back(strides[i]);
    }
  std::vector<int64_t> out(new_shape.size(), 0);
  int vi = int(new_shape.size()) - 1;
  int i = int(s.size()) - 1;
  while (i >= 0) {
    // gather a maximal contiguous run of source dims [j..i]
    int j = i;
    int64_t run = s[size_t(i)];
    while (j > 0 && st[size_t(j - 1)] == st[size_t(j)] * s[size_t(j)]) {
      --j;
      run *= s[size_t(j)];
    }
    // consume new dims covering exactly `run` elements, innermost first
    int64_t acc = 1;
    const int64_t base = st[size_t(i)];
    while (vi >= 0 && (acc < run || new_shape[size_t(vi)] == 1)) {
      if (new_shape[size_t(vi)] == 1) {
        out[size_t(vi)] = acc * base;
        --vi;
        continue;
      }
      out[size_t(vi)] = acc * base;
      acc *= new_shape[size_t(vi)];
      --vi;
    }
    if (acc != run) return std::nullopt;
    i = j - 1;
  }
  while (vi >= 0) {
    if (new_shape[size_t(vi)] != 1) return std::nullopt;
    out[size_t(vi)] = 1;
    --vi;
  }
  return out;
}

k::TDesc tdesc(const DevTensor& t) {
  k::TDesc d{};
  SB_CHECK(t.shape.size() <= size_t(k::kMaxRank), SB_UNSUPPORTED, "tensor rank above 8 is not supported on device");
  d.rank = int(t.shape.size());
  for (size_t i = 0; i < t.shape.size(); ++i) {
    d.shape[i] = t.shape[i];
    d.stride[i] = t.strides[i];
  }
  if (d.rank == 0) {   // scalars: rank-1 of length 1
    d.rank = 1;
    d.shape[0] = 1;
    d.stride[0] = 1;
  }
  return d;
}

// Broadcast view of `t` to `out_shape` (stride 0 on broadcast dims).
DevTensor broadcast_to(const DevTensor& t, const std::vector<int64_t>& out_shape) {
  DevTensor r = t;
  r.shape = out_shape;
  r.strides.assign(out_shape.size(), 0);
  size_t off = out_shape.size() - t.shape.size();
  for (size_t i = 0; i < t.shape.size(); ++i) {
    if (t.shape[i] == out_shape[i + off]) r.strides[i + off] = t.strides[i];
    else SB_CHECK(t.shape[i] == 1, SB_SHAPE_ERROR, "broadcast mismatch");
  }
  return r;
}

bool is_view_op(const std::string& t) {
  return t == "Reshape" || t == "Transpose" || t == "Identity" || t == "Slice" || t == "Expand";
}

int ew_code(const std::string& t) {
  static const std::map<std::string, int> m = {
      {"Add", k::EW_ADD}, {"Sub", k::EW_SUB}, {"Mul", k::EW_MUL}, {"Div", k::EW_DIV}, {"Pow", k::EW_POW},
      {"Max", k::EW_MAX}, {"Min", k::EW_MIN}, {"Relu", k::EW_RELU}, {"Sigmoid", k::EW_SIGMOID},
      {"Tanh", k::EW_TANH}, {"Sqrt", k::EW_SQRT}, {"Neg", k::EW_NEG}, {"Abs", k::EW_ABS}, {"Exp", k::EW_EXP},
      {"Log", k::EW_LOG}, {"Reciprocal", k::EW_RECIP}, {"Floor", k::EW_FLOOR}, {"Ceil", k::EW_CEIL},
      {"Erf", k::EW_ERF}, {"LeakyRelu", k::EW_LEAKY}, {"Clip", k::EW_CLIP}, {"Gelu", k::EW_GELU}};
  auto it = m.find(t);
  return it == m.end() ? -1 : it->second;
}

inline void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    if (e == cudaErrorMemoryAllocation) fail(SB_OUT_OF_MEMORY, std::string(what) + ": " + cudaGetErrorString(e));
    fail(SB_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

}  // namespace

// ---------------------------------------------------------------------------------------------
Plan::Plan(LGraph g, int device, int num_sms, int precision)
    : g_(std::move(g)), device_(device), num_sms_(num_sms) {
  fuse(g_);
  assign_precision(g_, precision);
  build();
  allocate_and_finalize();
}

Plan::~Plan() {
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device_);
  if (exec_) cudaGraphExecDestroy(exec_);
  if (graph_) cudaGraphDestroy(graph_);
  if (arena_) cudaFree(arena_);
  if (weights_) cudaFree(weights_);
  if (err_) cudaFree(err_);
  if (prev >= 0) cudaSetDevice(prev);
}

int Plan::new_buffer(size_t bytes) {
  Buffer b;
  b.bytes = (bytes + kAlign - 1) / kAlign * kAlign;
  if (b.bytes == 0) b.bytes = kAlign;
  bufs_.push_back(b);
  return int(bufs_.size()) - 1;
}

DevTensor Plan::alloc_contig(const std::vector<int64_t>& shape, bool bf16) {
  DevTensor t;
  t.bf16 = bf16;
  t.shape = shape;
  t.strides = contig_strides(shape);
  t.buf = new_buffer(size_t(numel(shape)) * (bf16 ? 2 : 4));
  return t;
}

// NHWC storage for a logical NCHW tensor, channel stride 1 and `cstride` elements per pixel.
DevTensor Plan::alloc_nhwc(const std::vector<int64_t>& s, bool bf16, int64_t cstride) {
  DevTensor t;
  t.bf16 = bf16;
  t.shape = s;
  t.strides = {s[2] * s[3] * cstride, 1, s[3] * cstride, cstride};
  t.buf = new_buffer(size_t(s[0] * s[2] * s[3] * cstride) * (bf16 ? 2 : 4));
  return t;
}

// Tensor-core weights [rows, K] in the operand dtype: bf16 (round to nearest even), or fp32
// rounded to the TF32 grid (10 explicit mantissa bits, nearest even) so the MMA's read of them is
// exact. TF32x3: the TF32-rounded hi matrix, zero rows up to *lo_row (rows rounded up to 256),
// then the lo matrix w - hi rounded to TF32 (unbiased, and read exactly by the MMA).
int64_t Plan::add_operand_weights(const std::vector<float>& w, int64_t rows, int64_t* lo_row, int prec) {
  if (lo_row) *lo_row = 0;
  if (prec == 0) {
    std::vector<uint16_t> b(w.size());
    for (size_t i = 0; i < w.size(); ++i) b[i] = f32_to_bf16_rne(w[i]);
    return add_weight_bytes(b.data(), b.size() * 2);
  }
  auto tf32_rne = [](float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0xFFFu + ((u >> 13) & 1u)) & ~0x1FFFu;   // finite values only
    float r;
    std::memcpy(&r, &u, 4);
    return r;
  };
  if (prec == 1) {
    std::vector<float> f(w.size());
    for (size_t i = 0; i < w.size(); ++i) f[i] = tf32_rne(w[i]);
    return add_weight_bytes(f.data(), f.size() * 4);
  }
  const int64_t K = rows ? int64_t(w.size()) / rows : 0;
  const int64_t lo = round_up(rows, 256);
  std::vector<float> f(size_t(2 * lo * K), 0.f);
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t k = 0; k < K; ++k) {
      const float x = w[size_t(r * K + k)];
      const float hi = tf32_rne(x);
      f[size_t(r * K + k)] = hi;
      f[size_t((lo + r) * K + k)] = std::isfinite(x) ? tf32_rne(x - hi) : 0.f;   // lo, itself on the TF32 grid
    }
  if (lo_row) *lo_row = lo;
  return add_weight_bytes(f.data(), f.size() * 4);
}

int64_t Plan::add_weight_bytes(const void* data, size_t bytes) {
  size_t off = (wblob_.size() + kAlign - 1) / kAlign * kAlign;
  wblob_.resize(off + std::max<size_t>(bytes, 1));
  if (bytes) std::memcpy(wblob_.data() + off, data, bytes);
  return int64_t(off);
}

void* Plan::buffer_ptr(int buf) const { return static_cast<uint8_t*>(arena_) + bufs_[size_t(buf)].offset; }

void* Plan::ptr(const DevTensor& t) const {
  SB_CHECK(t.valid(), SB_INTERNAL, "plan: invalid tensor reference");
  uint8_t* base = t.buf == -1 ? static_cast<uint8_t*>(weights_) : static_cast<uint8_t*>(arena_) + bufs_[size_t(t.buf)].offset;
  return base + t.off;
}

void Plan::add_step(const std::string& kind, std::vector<DevTensor> reads, std::vector<DevTensor> writes,
                    std::function<std::function<cudaError_t(cudaStream_t)>()> b) {
  const int idx = int(pending_.size());
  for (auto* lst : {&reads, &writes})
    for (auto& t : *lst)
      if (t.buf >= 0) {
        bufs_[size_t(t.buf)].first = std::min(bufs_[size_t(t.buf)].first, idx);
        bufs_[size_t(t.buf)].last = std::max(bufs_[size_t(t.buf)].last, idx);
      }
  pending_.push_back({kind, std::move(b), std::move(reads), std::move(writes)});
  stats_.kernels++;
}

// The dtype v is stored in, from what its readers (through views and max pools) take:
//   kStoreBf16   every reader is a bf16-operand contraction (operand, residual or second operand);
//   kStoreTf32   every reader is a single-pass TF32 contraction: fp32 rounded to the TF32 grid;
//   kStoreF32    anything else (generic ops, graph outputs, TF32x3 readers, mixed precisions).
// Global pools, group norms and attention read either dtype and add no constraint; a value whose
// readers add none takes `pref`, the class of its producer's operands.
int Plan::storage_class(int v, int pref) const {
  if (is_output_[size_t(v)]) return kStoreF32;
  int cls = -1;
  auto meet = [&](int c) {
    if (c < 0) return;
    cls = cls < 0 ? c : (cls == c ? c : kStoreF32);
  };
  for (int oi : consumers_[size_t(v)]) {
    const Op& op = g_.ops[size_t(oi)];
    if (op.type == "FusedConv" || op.type == "FusedGemm") {
      meet(op.prec == 0 ? kStoreBf16 : (op.prec == 1 ? kStoreTf32 : kStoreF32));
    } else if (op.type == "GlobalAveragePool" || op.type == "GlobalMaxPool" || op.type == "GroupNorm" ||
               op.type == "Attention") {
      continue;
    } else if (op.type == "MaxPool" || (is_view_op(op.type) && op.in[0] == v)) {
      const int c = storage_class(op.out[0], -1);
      meet(c);
    } else {
      meet(kStoreF32);
    }
  }
  if (cls < 0) cls = pref < 0 ? -1 : pref;
  return cls;
}

DevTensor Plan::materialize(const DevTensor& src, bool bf16) {
  DevTensor dst = alloc_contig(src.shape, bf16);
  add_step("copy", {src}, {dst}, [this, src, dst]() {
    void* sp = ptr(src);
    void* dp = ptr(dst);
    k::TDesc sd = tdesc(src), dd = tdesc(dst);
    int sb = src.bf16, db = dst.bf16;
    return std::function<cudaError_t(cudaStream_t)>(
        [=](cudaStream_t s) { return k::strided_copy(sp, sb, sd, dp, db, dd, s); });
  });
  return dst;
}

DevTensor Plan::as_f32_contig(int v) {
  const DevTensor& t = vt_[size_t(v)];
  if (!t.bf16 && is_contig(t)) return t;
  return materialize(t, false);
}

// NHWC copy of v in the operand dtype of a precision-`prec` contraction (bf16, or fp32 rounded to
// the TF32 grid for single-pass TF32, exact fp32 for TF32x3) with Cp channels per pixel. An fp32
// tensor that is not on the TF32 grid is read as is by a TF32 contraction (the MMA truncates it).
DevTensor Plan::as_nhwc_op(int v, int Cp, int prec) {
  const DevTensor& t = vt_[size_t(v)];
  SB_CHECK(t.shape.size() == 4, SB_SHAPE_ERROR, "expected a rank-4 activation");
  const int64_t N = t.shape[0], C = t.shape[1], H = t.shape[2], W = t.shape[3];
  if (t.bf16 == (prec == 0) && C == Cp && t.strides[1] == 1 && t.strides[3] == Cp && (t.strides[2] == W * Cp || H == 1) &&
      (t.strides[0] == H * W * Cp || N == 1) && t.off % 16 == 0)
    return t;
  auto key = std::make_pair(v, Cp * 4 + prec);
  auto it = conv_cache_.find(key);
  if (it != conv_cache_.end()) return it->second;
  DevTensor dst = alloc_nhwc({N, C, H, W}, prec == 0, Cp);
  const bool f32 = prec != 0;
  const int rnd = prec == 1;
  add_step(f32 ? "to_nhwc_f32" : "to_nhwc_bf16", {t}, {dst}, [this, t, dst, Cp, f32, rnd]() {
    const void* sp = ptr(t);
    void* dp = ptr(dst);
    int64_t sh[4] = {t.shape[0], t.shape[1], t.shape[2], t.shape[3]};
    int64_t st[4] = {t.strides[0], t.strides[1], t.strides[2], t.strides[3]};
    int sb = t.bf16;
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return f32 ? k::to_nhwc_f32(sp, sb, sh, st, dp, Cp, rnd, s) : k::to_nhwc_bf16(sp, sb, sh, st, dp, Cp, s);
    });
  });
  conv_cache_[key] = dst;
  return dst;
}

// Row matrix [M, Kp] of v in the operand dtype of a precision-`prec` contraction, rows 16-byte
// aligned.
DevTensor Plan::as_rows_op(int v, int64_t M, int64_t K, int prec) {
  const bool tf32 = prec != 0;
  DevTensor t = vt_[size_t(v)];
  auto vs = view_strides(t.shape, t.strides, {M, K});
  if (vs) {
    DevTensor r = t;
    r.shape = {M, K};
    r.strides = *vs;
    if (t.bf16 == !tf32 && r.strides[1] == 1 && (r.strides[0] == K || M == 1) && K % (tf32 ? 4 : 8) == 0 &&
        t.off % 16 == 0) {
      r.strides[0] = K;
      return r;
    }
    t = r;
  } else {
    t = materialize(t, false);
    t.shape = {M, K};
    t.strides = {K, 1};
  }
  auto it = rows_cache_.find(std::make_pair(v, prec));
  if (it != rows_cache_.end()) return it->second;
  const int64_t Kp = round_up(K, tf32 ? 4 : 8);
  DevTensor dst = alloc_contig({M, Kp}, !tf32);
  const bool f32 = tf32;
  const int rnd = prec == 1;
  add_step(f32 ? "to_rows_f32" : "to_rows_bf16", {t}, {dst}, [this, t, dst, M, K, Kp, f32, rnd]() {
    const void* sp = ptr(t);
    void* dp = ptr(dst);
    int64_t sm = t.strides[0], sk = t.strides[1];
    int sb = t.bf16;
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return f32 ? k::to_rows_f32(sp, sb, M, K, sm, sk, dp, Kp, rnd, s) : k::to_rows_bf16(sp, sb, M, K, sm, sk, dp, Kp, s);
    });
  });
  rows_cache_[std::make_pair(v, prec)] = dst;
  return dst;
}

// Storage of conv output v inside the buffer of the Concat it reaches through single-reader views
// (the RetinaNet heads: NHWC conv output -> Reshape [B,A,K,H,W] -> Transpose(0,3,4,1,2) ->
// Reshape [B,H*W*A,K] -> Concat on axis 1, RetinaNetDetector.cs:539-571): when those views of NHWC
// rows placed in the concat's buffer land exactly on the concat's slice for this input, the conv
// writes its rows there (grouped per image: the image stride is the concat's) and the concat copies
// nothing. Returns an invalid tensor when the layouts do not line up.
DevTensor Plan::concat_home(int v, int64_t Cout) {
  const Value& yv = g_.vals[size_t(v)];
  if (yv.shape.size() != 4) return {};
  std::vector<const Op*> chain;
  const Op* cat = nullptr;
  int cur = v;
  while (true) {
    if (is_output_[size_t(cur)] || consumers_[size_t(cur)].size() != 1) return {};
    const Op& o = g_.ops[size_t(consumers_[size_t(cur)][0])];
    if (o.type == "Concat") {
      cat = &o;
      break;
    }
    if (!((o.type == "Reshape" || o.type == "Transpose" || o.type == "Identity") && o.in[0] == cur)) return {};
    chain.push_back(&o);
    cur = o.out[0];
  }
  const int cid = cat->out[0];
  const Value& cv = g_.vals[size_t(cid)];
  if (cv.shape.empty() || cv.shape[0] != yv.shape[0]) return {};
  DevTensor& y = concat_out_[cid];
  if (!y.valid()) y = alloc_contig(cv.shape, false);
  int64_t off = 0;
  for (int id : cat->in) {
    if (id == cur) break;
    off += g_.vals[size_t(id)].shape[size_t(cat->axis)];
  }
  DevTensor dst = y;
  dst.shape = g_.vals[size_t(cur)].shape;
  dst.off = off * y.strides[size_t(cat->axis)] * 4;
  const int64_t W = yv.shape[3];
  DevTensor t = y;
  t.shape = yv.shape;
  t.strides = {y.strides[0], 1, W * Cout, Cout};
  t.off = dst.off;
  DevTensor r = t;
  for (const Op* o : chain) {
    const Value& ov = g_.vals[size_t(o->out[0])];
    if (o->type == "Transpose") {
      DevTensor q = r;
      q.shape.clear();
      q.strides.clear();
      for (auto pp : o->perm) {
        q.shape.push_back(r.shape[size_t(pp)]);
        q.strides.push_back(r.strides[size_t(pp)]);
      }
      r = q;
    } else if (o->type == "Reshape") {
      auto vs = view_strides(r.shape, r.strides, ov.shape);
      if (!vs) return {};
      r.shape = ov.shape;
      r.strides = *vs;
    }
  }
  if (r.shape != dst.shape || r.off != dst.off) return {};
  for (size_t d = 0; d < r.shape.size(); ++d)
    if (r.shape[d] != 1 && r.strides[d] != dst.strides[d]) return {};
  if (y.strides[0] < yv.shape[2] * W * Cout) return {};
  return t;
}

// The ResNet stem pattern the fused stem + max-pool kernel runs: a bf16 7x7/2-style conv over at
// most 4 channels (space-to-depth eligible, a 4x4 kernel after the transform) to 64 channels, no
// residual, whose only reader is a MaxPool 3x3 / stride 2 / pad 1 (floor mode) with an even, at most
// 128 pixel wide input and a bf16-stored output.
void Plan::find_stem_pools() {
  for (size_t i = 0; i < g_.ops.size(); ++i) {
    const Op& op = g_.ops[i];
    if (op.dead || op.type != "FusedConv" || op.prec != 0 || op.residual >= 0 || op.concat >= 0 || op.act > 1)
      continue;
    const Value& xv = g_.vals[size_t(op.in[0])];
    const Value& yv = g_.vals[size_t(op.out[0])];
    const auto& w = op.weight->shape;
    if (xv.shape.size() != 4 || w.size() != 4 || xv.shape[1] > 4 || op.group != 1) continue;
    if (op.strides[0] != 2 || op.strides[1] != 2 || op.dilations[0] != 1 || op.dilations[1] != 1 || w[2] < 3 || w[3] < 3)
      continue;
    const int64_t gkh = ceil_div(w[2] + op.pads[0] % 2, 2), gkw = ceil_div(w[3] + op.pads[1] % 2, 2);
    if (!k::stem_pool_supported(int(w[0]), int(yv.shape[2]), int(yv.shape[3]), int(gkh), int(gkw))) continue;
    if (is_output_[size_t(op.out[0])] || consumers_[size_t(op.out[0])].size() != 1) continue;
    const int pi = consumers_[size_t(op.out[0])][0];
    const Op& mp = g_.ops[size_t(pi)];
    if (mp.type != "MaxPool" || mp.in[0] != op.out[0] || mp.kernel != std::vector<int64_t>{3, 3} ||
        mp.strides != std::vector<int64_t>{2, 2} || mp.pads != std::vector<int64_t>{1, 1, 1, 1} || mp.ceil_mode ||
        (!mp.dilations.empty() && mp.dilations != std::vector<int64_t>{1, 1}))
      continue;
    const Value& pv = g_.vals[size_t(mp.out[0])];
    if (pv.shape.size() != 4 || pv.shape[2] * 2 != yv.shape[2] || pv.shape[3] * 2 != yv.shape[3]) continue;
    if (storage_class(mp.out[0], kStoreBf16) != kStoreBf16) continue;
    stem_pool_[int(i)] = pi;
    pooled_by_conv_.insert(pi);
  }
}

// Space-to-depth NHWC bf16 image [N, ceil(H/2), ceil(W/2), 16] of a stride-2 conv's input (shared by
// every conv that reads the same value this way).
DevTensor Plan::s2d_input(int v) {
  auto key = std::make_pair(v, -16);
  auto it = conv_cache_.find(key);
  if (it != conv_cache_.end()) return it->second;
  const DevTensor t = vt_[size_t(v)];
  const int64_t N = t.shape[0], H = t.shape[2], W = t.shape[3];
  const int64_t Hs = ceil_div(H, 2), Ws = ceil_div(W, 2);
  DevTensor x = alloc_nhwc({N, 16, Hs, Ws}, true, 16);
  add_step("to_s2d_bf16", {t}, {x}, [this, t, x, Hs, Ws]() {
    const void* sp = ptr(t);
    void* dp = ptr(x);
    int64_t sh[4] = {t.shape[0], t.shape[1], t.shape[2], t.shape[3]};
    int64_t st[4] = {t.strides[0], t.strides[1], t.strides[2], t.strides[3]};
    int sb = t.bf16;
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return k::to_s2d_bf16(sp, sb, sh, st, dp, Hs, Ws, s);
    });
  });
  conv_cache_[key] = x;
  return x;
}

// The stem conv and the max pool reading it as one kernel (k::stem_pool_*): the space-to-depth 4x4
// conv whose K is ordered (filter column, filter row, channel) so that one 4D TMA box of 4 image rows
// holds a whole k-tile; output = the pool's output, NHWC bf16.
void Plan::plan_stem_pool(const Op& op, const Op& pool) {
  const Value& xv = g_.vals[size_t(op.in[0])];
  const Value& yv = g_.vals[size_t(op.out[0])];
  const Value& pv = g_.vals[size_t(pool.out[0])];
  const HostTensor& Wt = *op.weight;
  const int64_t N = xv.shape[0], C = xv.shape[1], H = xv.shape[2], W = xv.shape[3];
  const int64_t Cout = Wt.shape[0], KH = Wt.shape[2], KW = Wt.shape[3];
  const int64_t Ho = yv.shape[2], Wo = yv.shape[3];
  const int64_t et = op.pads[0] % 2, el = op.pads[1] % 2;
  const int64_t gKH = ceil_div(KH + et, 2), gKW = ceil_div(KW + el, 2);
  const int64_t gph = (op.pads[0] + et) / 2, gpw = (op.pads[1] + el) / 2;
  DevTensor x = s2d_input(op.in[0]);
  const int64_t Kpad = gKH * gKW * 16;   // 256
  std::vector<float> wf(size_t(Cout * Kpad), 0.f);
  const float* wp = Wt.ptr<float>();
  for (int64_t m = 0; m < Cout; ++m)
    for (int64_t c = 0; c < C; ++c)
      for (int64_t a = 0; a < KH; ++a)
        for (int64_t b = 0; b < KW; ++b) {
          const int64_t u = a + et, v = b + el;   // u = 2 a' + p, v = 2 b' + q
          const int64_t kidx = ((v / 2) * gKH + (u / 2)) * 16 + ((u % 2) * 2 + (v % 2)) * C + c;
          wf[size_t(m * Kpad + kidx)] = wp[((m * C + c) * KH + a) * KW + b];
        }
  DevTensor wt;
  wt.buf = -1;
  wt.off = add_operand_weights(wf, Cout, nullptr, 0);
  std::vector<float> bias(size_t(round_up(Cout, 256)), 0.f);
  for (int64_t m = 0; m < Cout; ++m) bias[size_t(m)] = op.bias ? op.bias->ptr<float>()[m] : 0.f;
  DevTensor bt;
  bt.buf = -1;
  bt.off = add_weight_bytes(bias.data(), bias.size() * 4);
  DevTensor y = alloc_nhwc(pv.shape, true, Cout);
  vt_[size_t(pool.out[0])] = y;
  const double macs = double(N * Ho * Wo) * double(Cout) * double(C * KH * KW);
  stats_.macs += macs;
  stats_.macs_by_prec[0] += macs;
  stats_.tc_kernels++;
  const int sms = num_sms_;
  const std::string kind = "conv " + std::to_string(KH) + "x" + std::to_string(KW) + "/2 " + std::to_string(C) + "->" +
                           std::to_string(Cout) + " M=" + std::to_string(N * Ho * Wo) + " s2d +maxpool3x3/2";
  add_step(kind, {x}, {y}, [=]() {
    auto p = std::make_shared<k::StemPoolPlan>();
    k::StemPoolArgs& a = p->args;
    std::memset(&a, 0, sizeof(a));
    a.x = ptr(x);
    a.N = int(N);
    a.Hs = int(x.shape[2]);
    a.Ws = int(x.shape[3]);
    a.Ho = int(Ho);
    a.Wo = int(Wo);
    a.ph = int(gph);
    a.pw = int(gpw);
    a.bias = static_cast<const float*>(ptr(bt));
    a.out = ptr(y);
    a.act = op.act;
    a.err = err_;
    k::stem_pool_prepare(*p, ptr(wt), sms);
    return std::function<cudaError_t(cudaStream_t)>([p](cudaStream_t s) { return k::stem_pool_launch(*p, s); });
  });
}

// ---------------------------------------------------------------------------------------------
void Plan::plan_conv(const Op& op) {
  const Value& xv = g_.vals[size_t(op.in[0])];
  const Value& yv = g_.vals[size_t(op.out[0])];
  SB_CHECK(op.group == 1, SB_UNSUPPORTED, "Conv: group > 1 is not supported");
  const HostTensor& Wt = *op.weight;
  const int64_t N = xv.shape[0], C = xv.shape[1], H = xv.shape[2], W = xv.shape[3];
  const int64_t Cout = Wt.shape[0], KH = Wt.shape[2], KW = Wt.shape[3];
  const int prec = op.prec;
  const bool tf32 = prec != 0;
  const int64_t Ho = yv.shape[2], Wo = yv.shape[3];
  // Strided convs on at most 4 input channels (the ResNet stem) run as a stride-1 conv over the 2x2
  // space-to-depth image: out(ho) reads original rows i = 2*ho - pt + kh; with e = pt % 2 and
  // u = kh + e = 2a + p this is s2d row ho - (pt+e)/2 + a, parity p, so the kernel becomes
  // ceil((KH+e)/2) taps over 16 channels (p, q, c) with zero weights where kh falls outside [0, KH).
  const bool s2d = !tf32 && op.strides[0] == 2 && op.strides[1] == 2 && op.dilations[0] == 1 &&
                   op.dilations[1] == 1 && C <= 4 && KH >= 3 && KW >= 3;
  int64_t gH = H, gW = W, gKH = KH, gKW = KW, gsh = op.strides[0], gsw = op.strides[1];
  int64_t gph = op.pads[0], gpw = op.pads[1], gdh = op.dilations[0], gdw = op.dilations[1];
  int Cp = int(tf32 ? round_up(C, 4) : (C % 8 == 0 ? C : (C <= 4 ? 4 : round_up(C, 8))));
  int64_t et = 0, el = 0;
  if (s2d) {
    et = op.pads[0] % 2;
    el = op.pads[1] % 2;
    gH = ceil_div(H, 2);
    gW = ceil_div(W, 2);
    gKH = ceil_div(KH + et, 2);
    gKW = ceil_div(KW + el, 2);
    gsh = gsw = 1;
    gph = (op.pads[0] + et) / 2;
    gpw = (op.pads[1] + el) / 2;
    gdh = gdw = 1;
    Cp = 16;
  }
  const bool one_by_one = !s2d && KH == 1 && KW == 1 && op.strides[0] == 1 && op.strides[1] == 1 && op.pads[0] == 0 &&
                          op.pads[1] == 0 && op.pads[2] == 0 && op.pads[3] == 0 && Cp % (tf32 ? 4 : 8) == 0;
  DevTensor x;
  if (s2d) {
    x = s2d_input(op.in[0]);
  } else {
    x = as_nhwc_op(op.in[0], Cp, prec);
  }
  // A merged projection shortcut's input (op.concat): its C2 channels follow X's in the reduction,
  // read by the kernel from its own row matrix (k-tiles from Cp / k-tile width on).
  DevTensor x2;
  int64_t C2 = 0;
  if (op.concat >= 0) {
    C2 = Wt.shape[1] - C;
    const Value& cv = g_.vals[size_t(op.concat)];
    const int64_t cs = op.concat_stride;
    SB_CHECK(one_by_one && Cp == C && C % 64 == 0 && C2 > 0 && C2 % 64 == 0 && cv.shape.size() == 4 &&
                 cv.shape[0] == N && cv.shape[1] == C2 && (cs == 1 || cs == 2) && (cv.shape[2] - 1) / cs + 1 == H &&
                 (cv.shape[3] - 1) / cs + 1 == W,
             SB_UNSUPPORTED, "Conv: concatenated operand layout");
    x2 = as_nhwc_op(op.concat, int(C2), prec);
  }
  const int64_t K = gKH * gKW * Cp + C2;
  const int64_t Kpad = round_up(K, tf32 ? 32 : 64);   // whole 128-byte k-tile rows
  SB_CHECK(N * Ho * Wo < (int64_t(1) << 31) && N * gH * gW * Cp < (int64_t(1) << 40), SB_UNSUPPORTED,
           "Conv: problem too large for 32-bit row indexing");
  // weights [Cout, Kpad] bf16 (or TF32-rounded fp32), K ordered (kh, kw, c) of the kernel as run
  std::vector<float> wf(size_t(Cout * Kpad), 0.f);
  const float* wp = Wt.ptr<float>();
  if (op.concat >= 0)   // 1x1 over [X, X2]: k = channel
    for (int64_t m = 0; m < Cout; ++m)
      for (int64_t c = 0; c < C + C2; ++c) wf[size_t(m * Kpad + c)] = wp[m * (C + C2) + c];
  for (int64_t m = 0; m < Cout && op.concat < 0; ++m)
    for (int64_t c = 0; c < C; ++c)
      for (int64_t a = 0; a < KH; ++a)
        for (int64_t b = 0; b < KW; ++b) {
          int64_t kidx;
          if (s2d) {
            const int64_t u = a + et, v = b + el;   // u = 2*a' + p, v = 2*b' + q
            kidx = ((u / 2) * gKW + (v / 2)) * Cp + ((u % 2) * 2 + (v % 2)) * C + c;
          } else {
            kidx = (a * KW + b) * Cp + c;
          }
          wf[size_t(m * Kpad + kidx)] = wp[((m * C + c) * KH + a) * KW + b];
        }
  DevTensor wt;
  wt.buf = -1;
  int64_t w_lo_row = 0;
  wt.off = add_operand_weights(wf, Cout, &w_lo_row, prec);
  std::vector<float> bias(size_t(round_up(Cout, 256)), 0.f);
  for (int64_t m = 0; m < Cout; ++m) bias[size_t(m)] = op.bias ? op.bias->ptr<float>()[m] : 0.f;
  DevTensor bt;
  bt.buf = -1;
  bt.off = add_weight_bytes(bias.data(), bias.size() * 4);

  const int out_cls = storage_class(op.out[0], prec == 0 ? kStoreBf16 : (prec == 1 ? kStoreTf32 : kStoreF32));
  const bool out_bf16 = out_cls == kStoreBf16;
  DevTensor y;
  int64_t grp_rows = 0, grp_stride = 0;   // rows per image and image stride when writing into a concat
  if (!out_bf16) {
    y = concat_home(op.out[0], Cout);
    if (y.valid() && N > 1) {
      grp_rows = Ho * Wo;
      grp_stride = y.strides[0];
    }
  }
  if (!y.valid()) y = alloc_nhwc(yv.shape, out_bf16, Cout);
  vt_[size_t(op.out[0])] = y;

  DevTensor r;
  int64_t ldr = 0;
  int Hr = 0, Wr = 0;
  if (op.residual >= 0) {
    const DevTensor& rt = vt_[size_t(op.residual)];
    SB_CHECK(rt.shape.size() == 4 && rt.shape[1] == Cout && rt.shape[0] == N, SB_SHAPE_ERROR, "Conv: residual shape");
    const int64_t rh = rt.shape[2], rw = rt.shape[3];
    if (op.residual_mode == 0) SB_CHECK(rh == Ho && rw == Wo, SB_SHAPE_ERROR, "Conv: residual shape");
    else SB_CHECK(rh * 2 == Ho && rw * 2 == Wo, SB_SHAPE_ERROR, "Conv: upsampled residual shape");
    const int64_t cs = rt.strides[3];
    if (rt.strides[1] == 1 && (rt.strides[2] == rw * cs || rh == 1) && (rt.strides[0] == rh * rw * cs || N == 1) &&
        cs >= Cout) {
      r = rt;
      ldr = cs;
    } else {
      r = as_nhwc_op(op.residual, int(round_up(Cout, 4)), out_bf16 ? 0 : 2);
      ldr = round_up(Cout, 4);
    }
    Hr = int(rh);
    Wr = int(rw);
  }
  const double macs = double(N * Ho * Wo) * double(Cout) * double(C * KH * KW + C2);
  stats_.macs += macs;
  stats_.macs_by_prec[prec] += macs;
  stats_.tc_kernels++;
  std::vector<DevTensor> reads{x};
  if (r.valid()) reads.push_back(r);
  if (x2.valid()) reads.push_back(x2);
  const int sms = num_sms_;
  const bool f32 = tf32;
  const bool round_out = out_cls == kStoreTf32;   // the next MMA reads it as TF32
  const int x3 = prec == 2;
  k::ConvGemmArgs geo;   // geometry only: how the kernel will fetch A (for the step's label)
  std::memset(&geo, 0, sizeof(geo));
  geo.gather = one_by_one ? 0 : 1;
  geo.N = int(N);
  geo.H = int(gH);
  geo.W = int(gW);
  geo.Cp = Cp;
  geo.Ho = int(Ho);
  geo.Wo = int(Wo);
  geo.KH = int(gKH);
  geo.KW = int(gKW);
  geo.sh = int(gsh);
  geo.sw = int(gsw);
  geo.ph = int(gph);
  geo.pw = int(gpw);
  geo.dh = int(gdh);
  geo.dw = int(gdw);
  // 3x3 / stride 1 / pad 1 convs from 64 to 64 channels with a bf16 output and no residual run from
  // halo tiles (one TMA box of input rows per tile instead of nine im2col boxes).
  const int halo_wp = (prec == 0 && !s2d && KH == 3 && KW == 3 && op.strides[0] == 1 && op.strides[1] == 1 &&
                       op.dilations[0] == 1 && op.dilations[1] == 1 && op.pads[0] == 1 && op.pads[1] == 1 &&
                       op.pads[2] == 1 && op.pads[3] == 1 && C == 64 && Cp == 64 && Cout == 64 && op.residual < 0 &&
                       op.concat < 0 && out_bf16 && grp_rows == 0 && op.act <= 1 && x.strides[3] == 64 && x.off % 16 == 0)
                          ? k::conv3x3_tile_width(int(H), int(W))
                          : 0;
  if (halo_wp) {
    const std::string hkind = "conv 3x3/1 64->64 M=" + std::to_string(N * Ho * Wo) + " halo";
    add_step(hkind, reads, {y}, [=]() {
      auto p = std::make_shared<k::Conv3x3Plan>();
      k::Conv3x3Args& a = p->args;
      std::memset(&a, 0, sizeof(a));
      a.x = ptr(x);
      a.N = int(N);
      a.H = int(H);
      a.W = int(W);
      a.Wp = halo_wp;
      a.R = 128 / halo_wp;
      a.bias = static_cast<const float*>(ptr(bt));
      a.out = ptr(y);
      a.act = op.act;
      a.err = err_;
      k::conv3x3_prepare(*p, ptr(wt), sms);
      return std::function<cudaError_t(cudaStream_t)>([p](cudaStream_t s) { return k::conv3x3_launch(*p, s); });
    });
    return;
  }
  static const char* kAModeName[] = {"tma", "gather", "gather8", "im2col", "im2col16"};
  const std::string kind = "conv " + std::to_string(KH) + "x" + std::to_string(KW) + "/" +
                           std::to_string(op.strides[0]) + " " + std::to_string(C) + "->" + std::to_string(Cout) +
                           " M=" + std::to_string(N * Ho * Wo) + " " + kAModeName[k::conv_gemm_a_mode(geo)] +
                           (s2d ? " s2d" : "") + (op.residual >= 0 ? " +res" : "") +
                           (op.concat >= 0 ? " +proj " + std::to_string(C2) : "") +
                           (prec == 1 ? " tf32" : (prec == 2 ? " tf32x3" : ""));
  // Split-K when the output tiles leave most SMs idle (small batches, the deep layers): slices of
  // the reduction run on separate CTAs into fp32 partials, a reduce step finishes the output.
  const int64_t Mrows = N * Ho * Wo;
  const int ksplit = grp_rows == 0 && op.residual_mode == 0
                         ? k::conv_gemm_choose_split(Mrows, int(Cout), int(Kpad), f32, x3, sms)
                         : 1;
  const int64_t Mp = round_up(Mrows, 128);
  DevTensor ws, zb;
  if (ksplit > 1) {
    ws = alloc_contig({ksplit * Mp, Cout}, false);
    std::vector<float> z(size_t(round_up(Cout, 256)), 0.f);
    zb.buf = -1;
    zb.off = add_weight_bytes(z.data(), z.size() * 4);
  }
  add_step(kind + (ksplit > 1 ? " split" + std::to_string(ksplit) : ""), reads, {ksplit > 1 ? ws : y}, [=]() {
    auto p = std::make_shared<k::ConvGemmPlan>();
    k::ConvGemmArgs& a = p->args;
    std::memset(&a, 0, sizeof(a));
    a.gather = one_by_one ? 0 : 1;
    a.x = ptr(x);
    a.N = int(N);
    a.H = int(gH);
    a.W = int(gW);
    a.Cp = Cp;
    a.Ho = int(Ho);
    a.Wo = int(Wo);
    a.KH = int(gKH);
    a.KW = int(gKW);
    a.sh = int(gsh);
    a.sw = int(gsw);
    a.ph = int(gph);
    a.pw = int(gpw);
    a.dh = int(gdh);
    a.dw = int(gdw);
    a.M = int(N * Ho * Wo);
    a.Cout = int(Cout);
    a.Kpad = int(Kpad);
    a.bias = static_cast<const float*>(ptr(bt));
    a.res = r.valid() ? ptr(r) : nullptr;
    a.res_bf16 = r.valid() ? int(r.bf16) : 0;
    a.ldr = ldr;
    a.res_mode = op.residual_mode;
    a.Hr = Hr;
    a.Wr = Wr;
    a.out = ptr(y);
    a.out_bf16 = int(y.bf16);
    a.ldo = Cout;
    a.group_rows = grp_rows;
    a.group_stride = grp_stride;
    a.act = op.act;
    a.err = err_;
    a.tf32 = f32;
    a.round_tf32 = round_out;
    a.x3 = x3;
    a.w_lo_row = int(w_lo_row);
    if (x2.valid()) {
      a.a2 = ptr(x2);
      a.lda2 = C2;
      a.a2_kt = int(Cp / (f32 ? 32 : 64));
      a.a2_s = op.concat_stride > 1 ? int(op.concat_stride) : 0;
      a.a2_H = int(x2.shape[2]);
      a.a2_W = int(x2.shape[3]);
    }
    if (ksplit > 1) {   // raw partials; bias, residual, activation and output type in the reduce
      a.ksplit = ksplit;
      a.Mp = int(Mp);
      a.out = ptr(ws);
      a.out_bf16 = 0;
      a.ldo = Cout;
      a.bias = static_cast<const float*>(ptr(zb));
      a.res = nullptr;
      a.res_bf16 = 0;
      a.act = 0;
      a.round_tf32 = 0;
    }
    k::conv_gemm_prepare(*p, ptr(x), Cp, ptr(wt), sms);
    if (debug_level() >= 2) std::fprintf(stderr, "[shorokoo_b200] conv_gemm %s\n", k::conv_gemm_describe(*p).c_str());
    return std::function<cudaError_t(cudaStream_t)>([p](cudaStream_t s) { return k::conv_gemm_launch(*p, s); });
  });
  if (ksplit > 1) add_split_reduce(ws, ksplit, Mp, Mrows, Cout, bt, r, ldr, op.act, y, round_out);
}

// The reduce step of a split-K contraction: y = act(sum of the slices' partials + bias (+ residual)).
void Plan::add_split_reduce(const DevTensor& ws, int ksplit, int64_t Mp, int64_t M, int64_t Cout, const DevTensor& bias,
                            const DevTensor& res, int64_t ldr, int act, const DevTensor& y, bool round_tf32) {
  std::vector<DevTensor> reads{ws};
  if (res.valid()) reads.push_back(res);
  add_step("split_reduce " + std::to_string(ksplit) + "x" + std::to_string(M) + "x" + std::to_string(Cout), reads, {y},
           [=]() {
             const float* wp = static_cast<const float*>(ptr(ws));
             const float* bp = static_cast<const float*>(ptr(bias));
             const void* rp = res.valid() ? ptr(res) : nullptr;
             const int rb = res.valid() ? int(res.bf16) : 0;
             void* yp = ptr(y);
             const int yb = int(y.bf16);
             const int rt = round_tf32 ? 1 : 0;
             return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
               return k::conv_gemm_split_reduce(wp, ksplit, Mp, M, int(Cout), bp, rp, rb, ldr, act, yp, yb, Cout, rt, s);
             });
           });
}

void Plan::plan_gemm(const Op& op) {
  const Value& xv = g_.vals[size_t(op.in[0])];
  const Value& yv = g_.vals[size_t(op.out[0])];
  const HostTensor& Wt = *op.weight;
  const int64_t Nn = Wt.shape[0], K = Wt.shape[1];
  SB_CHECK(!xv.shape.empty() && xv.shape.back() == K, SB_SHAPE_ERROR, "Gemm: inner dimension mismatch");
  const int64_t M = numel(xv.shape) / std::max<int64_t>(K, 1);
  SB_CHECK(M < (int64_t(1) << 31), SB_UNSUPPORTED, "Gemm: too many rows");
  const int prec = op.prec;
  const bool tf32 = prec != 0;
  DevTensor x = as_rows_op(op.in[0], M, K, prec);
  const int64_t lda = x.strides[0];
  const int64_t Kpad = round_up(K, tf32 ? 32 : 64);
  std::vector<float> wf(size_t(Nn * Kpad), 0.f);
  const float* wp = Wt.ptr<float>();
  for (int64_t n = 0; n < Nn; ++n)
    for (int64_t kk = 0; kk < K; ++kk) wf[size_t(n * Kpad + kk)] = wp[n * K + kk];
  DevTensor wt;
  wt.buf = -1;
  int64_t w_lo_row = 0;
  wt.off = add_operand_weights(wf, Nn, &w_lo_row, prec);
  std::vector<float> bias(size_t(round_up(Nn, 256)), 0.f);
  for (int64_t n = 0; n < Nn; ++n) bias[size_t(n)] = op.bias ? op.bias->ptr<float>()[n] : 0.f;
  DevTensor bt;
  bt.buf = -1;
  bt.off = add_weight_bytes(bias.data(), bias.size() * 4);
  const int out_cls = storage_class(op.out[0], prec == 0 ? kStoreBf16 : (prec == 1 ? kStoreTf32 : kStoreF32));
  const bool out_bf16 = out_cls == kStoreBf16;
  DevTensor y = alloc_contig(yv.shape, out_bf16);
  vt_[size_t(op.out[0])] = y;
  DevTensor r;
  if (op.residual >= 0) {
    r = vt_[size_t(op.residual)];
    if (!is_contig(r)) r = materialize(r, false);
  }
  const double macs = double(M) * double(Nn) * double(K);
  stats_.macs += macs;
  stats_.macs_by_prec[prec] += macs;
  stats_.tc_kernels++;
  std::vector<DevTensor> reads{x};
  if (r.valid()) reads.push_back(r);
  const int sms = num_sms_;
  const bool f32 = tf32;
  const bool round_out = out_cls == kStoreTf32;   // the next MMA reads it as TF32
  const int x3 = prec == 2;
  const int ksplit = k::conv_gemm_choose_split(M, int(Nn), int(Kpad), f32 ? 1 : 0, x3, sms);
  const int64_t Mp = round_up(M, 128);
  DevTensor ws, zb;
  if (ksplit > 1) {
    ws = alloc_contig({ksplit * Mp, Nn}, false);
    std::vector<float> z(size_t(round_up(Nn, 256)), 0.f);
    zb.buf = -1;
    zb.off = add_weight_bytes(z.data(), z.size() * 4);
  }
  add_step("gemm " + std::to_string(M) + "x" + std::to_string(K) + "->" + std::to_string(Nn) +
               (prec == 1 ? " tf32" : (prec == 2 ? " tf32x3" : "")) + (ksplit > 1 ? " split" + std::to_string(ksplit) : ""),
           reads, {ksplit > 1 ? ws : y}, [=]() {
    auto p = std::make_shared<k::ConvGemmPlan>();
    k::ConvGemmArgs& a = p->args;
    std::memset(&a, 0, sizeof(a));
    a.gather = 0;
    a.N = 1;
    a.H = a.W = 1;
    a.Ho = 1;
    a.Wo = 1;
    a.KH = a.KW = 1;
    a.sh = a.sw = 1;
    a.dh = a.dw = 1;
    a.Cp = int(K);
    a.M = int(M);
    a.Cout = int(Nn);
    a.Kpad = int(Kpad);
    a.bias = static_cast<const float*>(ptr(bt));
    a.res = r.valid() ? ptr(r) : nullptr;
    a.res_bf16 = r.valid() ? int(r.bf16) : 0;
    a.ldr = Nn;
    a.out = ptr(y);
    a.out_bf16 = int(y.bf16);
    a.ldo = Nn;
    a.act = op.act;
    a.err = err_;
    a.tf32 = f32;
    a.round_tf32 = round_out;
    a.x3 = x3;
    a.w_lo_row = int(w_lo_row);
    if (ksplit > 1) {   // raw partials; bias, residual, activation and output type in the reduce
      a.ksplit = ksplit;
      a.Mp = int(Mp);
      a.out = ptr(ws);
      a.out_bf16 = 0;
      a.ldo = Nn;
      a.bias = static_cast<const float*>(ptr(zb));
      a.res = nullptr;
      a.res_bf16 = 0;
      a.act = 0;
      a.round_tf32 = 0;
    }
    k::conv_gemm_prepare(*p, ptr(x), lda, ptr(wt), sms);
    if (debug_level() >= 2) std::fprintf(stderr, "[shorokoo_b200] conv_gemm %s\n", k::conv_gemm_describe(*p).c_str());
    return std::function<cudaError_t(cudaStream_t)>([p](cudaStream_t s) { return k::conv_gemm_launch(*p, s); });
  });
  if (ksplit > 1) add_split_reduce(ws, ksplit, Mp, M, Nn, bt, r, Nn, op.act, y, round_out);
}

void Plan::plan_maxpool(const Op& op) {
  const Value& xv = g_.vals[size_t(op.in[0])];
  const Value& yv = g_.vals[size_t(op.out[0])];
  const DevTensor& t = vt_[size_t(op.in[0])];
  const int64_t C = xv.shape[1];
  DevTensor x;
  int64_t cs = t.strides.size() == 4 ? t.strides[3] : 0;
  // The pool keeps the dtype its input is stored in (converting to what its readers take if the
  // input is in no operand layout).
  if (t.strides[1] == 1 && cs >= C && t.strides[2] == xv.shape[3] * cs &&
      t.strides[0] == xv.shape[2] * xv.shape[3] * cs && t.off % 16 == 0 && cs % 4 == 0) {
    x = t;
  } else {
    cs = round_up(C, 4);
    const int cls = storage_class(op.out[0], kStoreF32);
    x = as_nhwc_op(op.in[0], int(cs), cls == kStoreBf16 ? 0 : (cls == kStoreTf32 ? 1 : 2));
  }
  DevTensor y = alloc_nhwc(yv.shape, x.bf16, cs);
  vt_[size_t(op.out[0])] = y;
  const int N = int(xv.shape[0]), H = int(xv.shape[2]), W = int(xv.shape[3]);
  const int Ho = int(yv.shape[2]), Wo = int(yv.shape[3]);
  const int Cs = int(cs);
  const bool f32 = !x.bf16;
  add_step("maxpool", {x}, {y}, [=]() {
    const void* xp = ptr(x);
    void* yp = ptr(y);
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      auto fn = f32 ? k::maxpool_nhwc_f32 : k::maxpool_nhwc_bf16;
      return fn(xp, yp, N, H, W, Cs, Ho, Wo, int(op.kernel[0]), int(op.kernel[1]), int(op.strides[0]),
                int(op.strides[1]), int(op.pads[0]), int(op.pads[1]), int(op.dilations[0]), int(op.dilations[1]), s);
    });
  });
}

void Plan::plan_global_pool(const Op& op) {
  const Value& xv = g_.vals[size_t(op.in[0])];
  const Value& yv = g_.vals[size_t(op.out[0])];
  SB_CHECK(xv.shape.size() == 4, SB_UNSUPPORTED, "GlobalPool: rank-4 input required");
  const DevTensor& t = vt_[size_t(op.in[0])];
  const int64_t N = xv.shape[0], C = xv.shape[1], H = xv.shape[2], W = xv.shape[3];
  DevTensor x = t;
  int64_t ldp = t.strides[3];
  bool nhwc = t.strides[1] == 1 && (t.strides[2] == W * ldp || H == 1) && (t.strides[0] == H * W * ldp || N == 1);
  if (!nhwc) {
    ldp = round_up(C, 4);
    x = as_nhwc_op(op.in[0], int(ldp), 2);
  }
  const bool out_bf16 = storage_class(op.out[0], kStoreF32) == kStoreBf16;
  DevTensor y = alloc_contig(yv.shape, out_bf16);
  vt_[size_t(op.out[0])] = y;
  const int is_max = op.type == "GlobalMaxPool";
  add_step("global_pool", {x}, {y}, [=]() {
    const void* xp = ptr(x);
    void* yp = ptr(y);
    int xb = x.bf16, yb = y.bf16;
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return k::global_pool_nhwc(xp, xb, int(N), int(H * W), int(C), ldp, yp, yb, is_max, s);
    });
  });
}

// GroupNorm (fused from its primitives): reads its input NHWC in the dtype it is stored in (a conv
// output: bf16, or fp32 for TF32 / TF32x3 convs) and writes what its readers take, so the
// normalisation sits between two contractions at one read for the statistics and one read and one
// write for the affine + ReLU pass.
void Plan::plan_group_norm(const Op& op) {
  const Value& xv = g_.vals[size_t(op.in[0])];
  const Value& yv = g_.vals[size_t(op.out[0])];
  SB_CHECK(xv.shape.size() == 4, SB_UNSUPPORTED, "GroupNorm: rank-4 input required");
  const int64_t N = xv.shape[0], C = xv.shape[1], H = xv.shape[2], W = xv.shape[3];
  const int G = int(op.group);
  const DevTensor& t = vt_[size_t(op.in[0])];
  DevTensor x = t;
  int64_t ldc = t.strides.size() == 4 ? t.strides[3] : 0;
  const int vec = t.bf16 ? 8 : 4;
  const bool nhwc = t.strides.size() == 4 && t.strides[1] == 1 && ldc >= C && (t.strides[2] == W * ldc || H == 1) &&
                    (t.strides[0] == H * W * ldc || N == 1) && t.off % 16 == 0 && ldc % vec == 0 &&
                    k::group_norm_supported(int(C), G, t.bf16);
  if (!nhwc) {
    ldc = round_up(C, 4);
    x = as_nhwc_op(op.in[0], int(ldc), 2);
  }
  SB_CHECK(k::group_norm_supported(int(C), G, x.bf16) && ldc % (x.bf16 ? 8 : 4) == 0, SB_UNSUPPORTED,
           "GroupNorm: " + std::to_string(C) + " channels in " + std::to_string(G) + " groups");
  const int cls = storage_class(op.out[0], x.bf16 ? kStoreBf16 : kStoreF32);
  const int ymode = cls == kStoreBf16 ? 0 : (cls == kStoreTf32 ? 1 : 2);
  const int64_t ldy = round_up(C, 8);
  DevTensor y = alloc_nhwc(yv.shape, ymode == 0, ldy);
  vt_[size_t(op.out[0])] = y;
  std::vector<float> gb(size_t(2 * C));
  for (int64_t c = 0; c < C; ++c) {
    gb[size_t(c)] = op.weight->ptr<float>()[c];
    gb[size_t(C + c)] = op.bias->ptr<float>()[c];
  }
  DevTensor gbt;
  gbt.buf = -1;
  gbt.off = add_weight_bytes(gb.data(), gb.size() * 4);
  const int per_img = k::group_norm_blocks_per_image(int(N), H * W, num_sms_);
  DevTensor partial = alloc_contig({N * per_img * 2 * C}, false);
  DevTensor ab = alloc_contig({N * 2 * C}, false);
  const float eps = op.alpha;
  const int relu = op.act == 1;
  stats_.kernels += 2;   // (three launches: statistics, their merge, the normalisation)
  add_step("group_norm " + std::to_string(C) + "/" + std::to_string(G), {x}, {y, partial, ab}, [=]() {
    const void* xp = ptr(x);
    const float* gp = static_cast<const float*>(ptr(gbt));
    void* yp = ptr(y);
    float* pp = static_cast<float*>(ptr(partial));
    float* abp = static_cast<float*>(ptr(ab));
    const int xb = x.bf16;
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return k::group_norm(xp, xb, int(N), H * W, int(C), ldc, G, eps, gp, gp + C, yp, ymode, ldy, relu, per_img, pp,
                           abp, s);
    });
  });
}

// LayerNorm over the last axis (fused from its primitives): fp32 rows in, the readers' operand
// type out (bf16 rows for a bf16 projection), one warp per row.
void Plan::plan_layer_norm(const Op& op) {
  const Value& xv = g_.vals[size_t(op.in[0])];
  const Value& yv = g_.vals[size_t(op.out[0])];
  const int64_t D = xv.shape.back();
  const int64_t rows = numel(xv.shape) / std::max<int64_t>(D, 1);
  DevTensor x = as_f32_contig(op.in[0]);
  SB_CHECK(D % 4 == 0 && x.off % 16 == 0, SB_UNSUPPORTED, "LayerNorm: " + std::to_string(D) + " features");
  const int cls = storage_class(op.out[0], kStoreF32);
  const int ymode = cls == kStoreBf16 ? 0 : (cls == kStoreTf32 ? 1 : 2);
  DevTensor y = alloc_contig(yv.shape, ymode == 0);
  vt_[size_t(op.out[0])] = y;
  std::vector<float> gb(size_t(2 * D));
  for (int64_t c = 0; c < D; ++c) {
    gb[size_t(c)] = op.weight->ptr<float>()[c];
    gb[size_t(D + c)] = op.bias->ptr<float>()[c];
  }
  DevTensor gbt;
  gbt.buf = -1;
  gbt.off = add_weight_bytes(gb.data(), gb.size() * 4);
  const float eps = op.alpha;
  add_step("layer_norm " + std::to_string(D), {x}, {y}, [=]() {
    const float* xp = static_cast<const float*>(ptr(x));
    const float* gp = static_cast<const float*>(ptr(gbt));
    void* yp = ptr(y);
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return k::layer_norm(xp, rows, int(D), D, eps, gp, gp + D, yp, ymode, D, s);
    });
  });
}

// Attention (fused q k^T -> scale -> softmax -> v): q, k, v are read where they are (strided views
// of the QKV projection); the output is laid out [B, S, H, hd], so the Transpose(0, 2, 1, 3) and
// Reshape to [B, S, H hd] that follow are a plain row matrix for the output projection.
void Plan::plan_attention(const Op& op) {
  const Value& qv = g_.vals[size_t(op.in[0])];
  const size_t r = qv.shape.size();
  SB_CHECK(r == 3 || r == 4, SB_UNSUPPORTED, "Attention: rank-3 or rank-4 operands required");
  const int64_t B = qv.shape[0], H = r == 4 ? qv.shape[1] : 1, S = qv.shape[r - 2], hd = qv.shape[r - 1];
  SB_CHECK(k::attention_supported(int(S), int(hd)), SB_UNSUPPORTED,
           "Attention: sequences of up to 256 and heads of 64 are supported (got " + std::to_string(S) + " x " +
               std::to_string(hd) + ")");
  DevTensor in[3];
  for (int i = 0; i < 3; ++i) in[i] = vt_[size_t(op.in[size_t(i)])];
  auto usable = [&](const DevTensor& t) {
    const int es = t.bf16 ? 2 : 4;
    if (t.strides.back() != 1 || (t.off % 16) != 0) return false;
    for (size_t d = 0; d + 1 < r; ++d)
      if ((t.strides[d] * es) % 16 != 0) return false;
    return true;
  };
  const bool same = in[0].bf16 == in[1].bf16 && in[1].bf16 == in[2].bf16;
  for (int i = 0; i < 3; ++i)
    if (!same || !usable(in[i])) in[i] = as_f32_contig(op.in[size_t(i)]);
  const int cls = storage_class(op.out[0], kStoreF32);
  const int ymode = cls == kStoreBf16 ? 0 : (cls == kStoreTf32 ? 1 : 2);
  DevTensor y = alloc_contig({B, S, H, hd}, ymode == 0);
  DevTensor yl = y;   // the logical [B, H, S, hd] (or [B, S, hd]) view
  if (r == 4) {
    yl.shape = {B, H, S, hd};
    yl.strides = {S * H * hd, hd, H * hd, 1};
  } else {
    yl.shape = {B, S, hd};
    yl.strides = {S * hd, hd, 1};
  }
  vt_[size_t(op.out[0])] = yl;
  auto st3 = [&](const DevTensor& t, int64_t* o) {
    o[0] = t.strides[0];
    o[1] = r == 4 ? t.strides[1] : 0;
    o[2] = t.strides[r - 2];
  };
  k::AttentionArgs a;
  std::memset(&a, 0, sizeof(a));
  st3(in[0], a.qs);
  st3(in[1], a.ks);
  st3(in[2], a.vs);
  a.in_f32 = in[0].bf16 ? 0 : 1;
  a.S = int(S);
  a.hd = int(hd);
  a.scale = op.alpha;
  a.os[0] = S * H * hd;
  a.os[1] = hd;
  a.os[2] = H * hd;
  a.out_mode = ymode;
  a.err = err_;
  const double macs = 2.0 * double(B * H) * double(S) * double(S) * double(hd);
  stats_.macs += macs;
  stats_.macs_by_prec[0] += macs;
  stats_.tc_kernels++;
  const DevTensor q = in[0], kk = in[1], v = in[2];
  add_step("attention " + std::to_string(B * H) + "x" + std::to_string(S) + "x" + std::to_string(hd), {q, kk, v}, {y},
           [=]() {
             k::AttentionArgs aa = a;
             aa.q = ptr(q);
             aa.k = ptr(kk);
             aa.v = ptr(v);
             aa.out = ptr(y);
             k::attention_prepare();
             const int nb = int(B), nh = int(H);
             return std::function<cudaError_t(cudaStream_t)>(
                 [=](cudaStream_t s) { return k::attention(aa, nb, nh, s); });
           });
}

void Plan::plan_elementwise(const Op& op) {
  const Value& yv = g_.vals[size_t(op.out[0])];
  const int code = op.type == "Gelu" && op.mode == "tanh" ? int(k::EW_GELU_TANH) : ew_code(op.type);
  SB_CHECK(code >= 0, SB_UNSUPPORTED, "no device kernel for " + op.type);
  std::vector<DevTensor> ins;
  for (int id : op.in) {
    if (id < 0) continue;
    const Value& v = g_.vals[size_t(id)];
    if (v.is_host) {
      std::vector<float> f(size_t(v.host->numel()));
      for (int64_t i = 0; i < v.host->numel(); ++i) f[size_t(i)] = float(v.host->get_f64(i));
      DevTensor h;
      h.buf = -1;
      h.off = add_weight_bytes(f.data(), f.size() * 4);
      h.shape = v.shape;
      h.strides = contig_strides(v.shape);
      ins.push_back(h);
    } else {
      ins.push_back(vt_[size_t(id)]);
    }
  }
  // Output follows the physical order of the first same-shape dense input (keeps NHWC as NHWC).
  DevTensor y;
  const DevTensor* like = nullptr;
  for (auto& t : ins)
    if (t.shape == yv.shape && t.buf >= 0) {
      like = &t;
      break;
    }
  if (like && yv.shape.size() == 4 && like->strides[1] == 1 && !is_contig(*like)) {
    const int64_t cs = yv.shape[1];
    y = alloc_nhwc(yv.shape, false, cs);
  } else {
    y = alloc_contig(yv.shape, false);
  }
  vt_[size_t(op.out[0])] = y;
  DevTensor a = broadcast_to(ins[0], yv.shape);
  DevTensor b;
  if (ins.size() > 1) b = broadcast_to(ins[1], yv.shape);
  float alpha = op.alpha, beta = 0.f;
  if (op.type == "Clip") {
    alpha = op.fmin;
    beta = op.fmax;
  }
  std::vector<DevTensor> reads{ins[0]};
  if (ins.size() > 1) reads.push_back(ins[1]);
  add_step("elementwise:" + op.type, reads, {y}, [=]() {
    const void* ap = ptr(a);
    const void* bp = b.valid() ? ptr(b) : nullptr;
    void* yp = ptr(y);
    k::TDesc ad = tdesc(a), bd = b.valid() ? tdesc(b) : k::TDesc{}, yd = tdesc(y);
    int ab = a.bf16, bb = b.valid() ? int(b.bf16) : 0;
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return k::elementwise(code, ap, ab, ad, bp, bb, bd, yp, 0, yd, alpha, beta, s);
    });
  });
}

void Plan::plan_view(const Op& op) {
  const Value& yv = g_.vals[size_t(op.out[0])];
  DevTensor t = vt_[size_t(op.in[0])];
  SB_CHECK(t.valid(), SB_INTERNAL, "view of an unplanned value");
  if (op.type == "Identity") {
    vt_[size_t(op.out[0])] = t;
    return;
  }
  if (op.type == "Transpose") {
    DevTensor r = t;
    r.shape.clear();
    r.strides.clear();
    for (auto p : op.perm) {
      r.shape.push_back(t.shape[size_t(p)]);
      r.strides.push_back(t.strides[size_t(p)]);
    }
    vt_[size_t(op.out[0])] = r;
    return;
  }
  if (op.type == "Slice") {
    DevTensor r = t;
    int64_t es = t.bf16 ? 2 : 4;
    for (size_t d = 0; d < t.shape.size(); ++d) {
      r.off += op.axes[d] * t.strides[d] * es;
      r.strides[d] = t.strides[d] * op.strides[d];
    }
    r.shape = yv.shape;
    vt_[size_t(op.out[0])] = r;
    return;
  }
  if (op.type == "Expand") {
    vt_[size_t(op.out[0])] = broadcast_to(t, yv.shape);
    return;
  }
  // Reshape
  auto vs = view_strides(t.shape, t.strides, yv.shape);
  if (!vs) {
    t = materialize(t, t.bf16);
    vs = contig_strides(yv.shape);
  }
  DevTensor r = t;
  r.shape = yv.shape;
  r.strides = *vs;
  vt_[size_t(op.out[0])] = r;
}

void Plan::plan_concat(const Op& op) {
  const Value& yv = g_.vals[size_t(op.out[0])];
  auto home = concat_out_.find(op.out[0]);   // inputs written in place by their convs
  DevTensor y = home != concat_out_.end() ? home->second : alloc_contig(yv.shape, false);
  vt_[size_t(op.out[0])] = y;
  int64_t off = 0;
  for (int id : op.in) {
    const Value& v = g_.vals[size_t(id)];
    DevTensor src;
    if (v.is_host) {
      std::vector<float> f(size_t(v.host->numel()));
      for (int64_t i = 0; i < v.host->numel(); ++i) f[size_t(i)] = float(v.host->get_f64(i));
      src.buf = -1;
      src.off = add_weight_bytes(f.data(), f.size() * 4);
      src.shape = v.shape;
      src.strides = contig_strides(v.shape);
    } else {
      src = vt_[size_t(id)];
    }
    DevTensor dst = y;
    dst.shape = v.shape;
    dst.off = off * y.strides[size_t(op.axis)] * 4;
    off += v.shape[size_t(op.axis)];
    if (numel(v.shape) == 0) continue;
    if (src.buf == dst.buf && src.off == dst.off && src.shape == dst.shape && !src.bf16) {
      bool same = true;
      for (size_t d = 0; d < dst.shape.size(); ++d)
        if (dst.shape[d] != 1 && src.strides[d] != dst.strides[d]) same = false;
      if (same) continue;   // already in place
    }
    add_step("concat_copy", {src}, {y}, [this, src, dst]() {
      const void* sp = ptr(src);
      void* dp = ptr(dst);
      k::TDesc sd = tdesc(src), dd = tdesc(dst);
      int sb = src.bf16;
      return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
        return k::strided_copy(sp, sb, sd, dp, 0, dd, s);
      });
    });
  }
}

void Plan::plan_softmax(const Op& op) {
  const Value& yv = g_.vals[size_t(op.out[0])];
  DevTensor x = as_f32_contig(op.in[0]);
  DevTensor y = alloc_contig(yv.shape, false);
  vt_[size_t(op.out[0])] = y;
  int64_t outer = 1, inner = 1;
  for (int64_t d = 0; d < op.axis; ++d) outer *= yv.shape[size_t(d)];
  for (size_t d = size_t(op.axis) + 1; d < yv.shape.size(); ++d) inner *= yv.shape[d];
  const int64_t len = yv.shape.empty() ? 1 : yv.shape[size_t(op.axis)];
  add_step("softmax", {x}, {y}, [=]() {
    const float* xp = static_cast<const float*>(ptr(x));
    float* yp = static_cast<float*>(ptr(y));
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return k::softmax(xp, yp, outer, len, inner, s);
    });
  });
}

void Plan::plan_reduce(const Op& op) {
  const Value& xv = g_.vals[size_t(op.in[0])];
  const Value& yv = g_.vals[size_t(op.out[0])];
  const int kind = op.type == "ReduceMax" ? 2 : 0;
  DevTensor cur = as_f32_contig(op.in[0]);
  std::vector<int64_t> shape = xv.shape;
  int64_t count = 1;
  // reduce one axis at a time from the innermost (keepdims), then a mean scale if needed
  std::vector<int64_t> axes = op.axes;
  std::sort(axes.rbegin(), axes.rend());
  for (int64_t a : axes) {
    int64_t outer = 1, inner = 1;
    for (int64_t d = 0; d < a; ++d) outer *= shape[size_t(d)];
    for (size_t d = size_t(a) + 1; d < shape.size(); ++d) inner *= shape[d];
    const int64_t len = shape[size_t(a)];
    count *= len;
    shape[size_t(a)] = 1;
    DevTensor nx = alloc_contig(shape, false);
    DevTensor src = cur;
    add_step("reduce", {src}, {nx}, [=]() {
      const float* xp = static_cast<const float*>(ptr(src));
      float* yp = static_cast<float*>(ptr(nx));
      return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
        return k::reduce_mid(xp, yp, outer, len, inner, kind, s);
      });
    });
    cur = nx;
  }
  if (op.type == "ReduceMean" && count > 1) {
    DevTensor nx = alloc_contig(shape, false);
    DevTensor src = cur;
    const float inv = 1.f / float(count);
    std::vector<float> c{inv};
    DevTensor ct;
    ct.buf = -1;
    ct.off = add_weight_bytes(c.data(), 4);
    ct.shape = {};
    ct.strides = {};
    DevTensor cb = broadcast_to(ct, shape);
    add_step("reduce_scale", {src}, {nx}, [=]() {
      const void* xp = ptr(src);
      const void* cp = ptr(cb);
      void* yp = ptr(nx);
      k::TDesc d = tdesc(src), cd = tdesc(cb), yd = tdesc(nx);
      return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
        return k::elementwise(k::EW_MUL, xp, 0, d, cp, 0, cd, yp, 0, yd, 0.f, 0.f, s);
      });
    });
    cur = nx;
  }
  cur.shape = yv.shape;
  cur.strides = contig_strides(yv.shape);
  vt_[size_t(op.out[0])] = cur;
}

void Plan::plan_pad(const Op& op) {
  const Value& yv = g_.vals[size_t(op.out[0])];
  DevTensor x = vt_[size_t(op.in[0])];
  DevTensor y = alloc_contig(yv.shape, false);
  vt_[size_t(op.out[0])] = y;
  const int64_t n = numel(yv.shape);
  const float val = op.alpha;
  add_step("pad_fill", {}, {y}, [=]() {
    void* yp = ptr(y);
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) { return k::fill_f32(yp, n, val, s); });
  });
  DevTensor dst = y;
  const size_t r = yv.shape.size();
  dst.shape = x.shape;
  for (size_t d = 0; d < r; ++d) dst.off += op.pads[d] * y.strides[d] * 4;
  add_step("pad_copy", {x}, {y}, [=]() {
    const void* xp = ptr(x);
    void* dp = ptr(dst);
    k::TDesc xd = tdesc(x), dd = tdesc(dst);
    int xb = x.bf16;
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return k::strided_copy(xp, xb, xd, dp, 0, dd, s);
    });
  });
}

void Plan::plan_resize(const Op& op) {
  const Value& xv = g_.vals[size_t(op.in[0])];
  const Value& yv = g_.vals[size_t(op.out[0])];
  DevTensor x = vt_[size_t(op.in[0])];
  DevTensor y = alloc_contig(yv.shape, false);
  vt_[size_t(op.out[0])] = y;
  // per-axis nearest index tables (ONNX Resize, mode=nearest)
  std::vector<int64_t> tables;
  for (size_t d = 0; d < yv.shape.size(); ++d) {
    const int64_t in_len = xv.shape[d], out_len = yv.shape[d];
    const double scale = double(op.scales[d]);
    for (int64_t o = 0; o < out_len; ++o) {
      double xo;
      if (op.coord_mode == "asymmetric") xo = double(o) / scale;
      else if (op.coord_mode == "align_corners") xo = out_len > 1 ? double(o) * double(in_len - 1) / double(out_len - 1) : 0.0;
      else if (op.coord_mode == "pytorch_half_pixel") xo = out_len > 1 ? (double(o) + 0.5) / scale - 0.5 : 0.0;
      else if (op.coord_mode == "half_pixel") xo = (double(o) + 0.5) / scale - 0.5;
      else fail(SB_UNSUPPORTED, "Resize: coordinate_transformation_mode " + op.coord_mode);
      double idx;
      const double fl = std::floor(xo);
      if (op.nearest_mode == "floor") idx = fl;
      else if (op.nearest_mode == "ceil") idx = std::ceil(xo);
      else if (op.nearest_mode == "round_prefer_ceil") idx = (xo - fl == 0.5) ? fl + 1 : std::nearbyint(xo);
      else idx = (xo - fl == 0.5) ? fl : std::round(xo);
      tables.push_back(std::clamp<int64_t>(int64_t(idx), 0, in_len - 1));
    }
  }
  DevTensor tt;
  tt.buf = -1;
  tt.off = add_weight_bytes(tables.data(), tables.size() * 8);
  add_step("resize_nearest", {x}, {y}, [=]() {
    const void* xp = ptr(x);
    const int64_t* tp = static_cast<const int64_t*>(ptr(tt));
    void* yp = ptr(y);
    k::TDesc xd = tdesc(x), yd = tdesc(y);
    int xb = x.bf16;
    return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) {
      return k::gather_axes(xp, xb, xd, tp, yp, 0, yd, s);
    });
  });
}

// ---------------------------------------------------------------------------------------------
void Plan::build() {
  vt_.assign(g_.vals.size(), DevTensor{});
  consumers_.assign(g_.vals.size(), {});
  is_output_.assign(g_.vals.size(), false);
  for (size_t i = 0; i < g_.ops.size(); ++i) {
    const Op& op = g_.ops[i];
    if (op.dead) continue;
    for (int id : op.in)
      if (id >= 0) consumers_[size_t(id)].push_back(int(i));
    if (op.residual >= 0) consumers_[size_t(op.residual)].push_back(int(i));
    if (op.concat >= 0) consumers_[size_t(op.concat)].push_back(int(i));
  }
  for (int id : g_.outputs) is_output_[size_t(id)] = true;

  // Host-known operands read by device ops (plan-time inputs, folded constants) live in the
  // weights blob as f32 contiguous tensors.
  for (const Op& op : g_.ops) {
    if (op.dead) continue;
    std::vector<int> ids = op.in;
    if (op.residual >= 0) ids.push_back(op.residual);
    if (op.concat >= 0) ids.push_back(op.concat);
    for (int id : ids) {
      if (id < 0 || vt_[size_t(id)].valid()) continue;
      const Value& v = g_.vals[size_t(id)];
      if (!v.is_host) continue;
      std::vector<float> f(size_t(v.host->numel()));
      for (int64_t i = 0; i < v.host->numel(); ++i) f[size_t(i)] = float(v.host->get_f64(i));
      DevTensor h;
      h.buf = -1;
      h.off = add_weight_bytes(f.data(), f.size() * 4);
      h.shape = v.shape;
      h.strides = contig_strides(v.shape);
      vt_[size_t(id)] = h;
    }
  }

  // graph inputs: contiguous buffers filled by H2D in the caller's element type. bfloat16 inputs are
  // read as they are by every kernel (half the transfer of float32); float16 ones are widened to
  // float32 on the device first.
  for (size_t k = 0; k < g_.inputs.size(); ++k) {
    const Value& v = g_.vals[size_t(g_.inputs[k])];
    if (v.is_host) continue;
    DevTensor t = alloc_contig(v.shape, v.dtype == DT_BFLOAT16);
    if (v.dtype == DT_FLOAT16) {
      DevTensor h = alloc_contig(v.shape, true);   // raw 16-bit storage of the transfer
      bufs_[size_t(h.buf)].first = -1;
      inputs_.push_back({int(k), h.buf, size_t(numel(v.shape)) * 2});
      const int64_t n = numel(v.shape);
      add_step("f16_to_f32", {h}, {t}, [this, h, t, n]() {
        const void* sp = ptr(h);
        void* dp = ptr(t);
        return std::function<cudaError_t(cudaStream_t)>([=](cudaStream_t s) { return k::f16_to_f32(sp, dp, n, s); });
      });
    } else {
      bufs_[size_t(t.buf)].first = -1;
      InputBinding ib{int(k), t.buf, size_t(numel(v.shape)) * dtype_size(v.dtype)};
      ib.bf16_ok = v.dtype == DT_FLOAT && storage_class(g_.inputs[k], kStoreF32) == kStoreBf16;
      inputs_.push_back(ib);
    }
    vt_[size_t(g_.inputs[k])] = t;
  }

  find_stem_pools();
  for (size_t i = 0; i < g_.ops.size(); ++i) {
    const Op& op = g_.ops[i];
    if (op.dead) continue;
    const std::string& t = op.type;
    auto sp = stem_pool_.find(int(i));
    if (sp != stem_pool_.end()) {
      plan_stem_pool(op, g_.ops[size_t(sp->second)]);
      continue;
    }
    if (t == "MaxPool" && pooled_by_conv_.count(int(i))) continue;   // done by the stem kernel
    if (t == "FusedConv") plan_conv(op);
    else if (t == "FusedGemm") plan_gemm(op);
    else if (t == "MaxPool") plan_maxpool(op);
    else if (t == "GlobalAveragePool" || t == "GlobalMaxPool") plan_global_pool(op);
    else if (t == "GroupNorm") plan_group_norm(op);
    else if (t == "LayerNorm") plan_layer_norm(op);
    else if (t == "Attention") plan_attention(op);
    else if (is_view_op(t)) plan_view(op);
    else if (t == "Concat") plan_concat(op);
    else if (t == "Softmax") plan_softmax(op);
    else if (t == "ReduceMean" || t == "ReduceSum" || t == "ReduceMax") plan_reduce(op);
    else if (t == "Pad") plan_pad(op);
    else if (t == "Resize") plan_resize(op);
    else if (ew_code(t) >= 0) plan_elementwise(op);
    else if (t == "Conv") fail(SB_INTERNAL, "Conv was not fused");
    else if (t == "MatMul" || t == "Gemm")
      fail(SB_UNSUPPORTED, t + " with a non-constant weight operand is not supported");
    else fail(SB_UNSUPPORTED, "no device plan for operator " + t);
  }

  for (size_t j = 0; j < g_.outputs.size(); ++j) {
    const int id = g_.outputs[j];
    const Value& v = g_.vals[size_t(id)];
    OutputBinding ob;
    ob.shape = v.shape;
    if (v.is_host) {
      ob.host = true;
      ob.value = v.host;
    } else {
      DevTensor t = vt_[size_t(id)];
      SB_CHECK(t.valid(), SB_INTERNAL, "graph output was not planned");
      if (t.bf16 || !is_contig(t) || t.buf < 0) t = materialize(t, false);
      bufs_[size_t(t.buf)].last = 1 << 30;
      ob.dev = t;
    }
    outputs_.push_back(ob);
  }
}

void Plan::allocate_and_finalize() {
  // Best-fit offsets by decreasing size; two buffers may share memory only if their step ranges
  // [first, last] do not overlap.
  std::vector<int> order(bufs_.size());
  std::iota(order.begin(), order.end(), 0);
  std::sort(order.begin(), order.end(), [&](int a, int b) { return bufs_[size_t(a)].bytes > bufs_[size_t(b)].bytes; });
  std::vector<int> placed;
  size_t total = 0;
  for (int bi : order) {
    Buffer& b = bufs_[size_t(bi)];
    if (b.last < b.first) {   // never used (e.g. dead view); still give it a slot at the end
      b.first = b.last = 1 << 29;
    }
    std::vector<std::pair<size_t, size_t>> busy;
    for (int pj : placed) {
      const Buffer& o = bufs_[size_t(pj)];
      if (o.first <= b.last && b.first <= o.last) busy.push_back({o.offset, o.offset + o.bytes});
    }
    std::sort(busy.begin(), busy.end());
    size_t off = 0;
    size_t best = SIZE_MAX, best_gap = SIZE_MAX;
    for (auto& iv : busy) {
      if (iv.first >= off + b.bytes) {
        size_t gap = iv.first - off;
        if (gap < best_gap) {
          best_gap = gap;
          best = off;
        }
      }
      off = std::max(off, iv.second);
    }
    if (best == SIZE_MAX) best = off;
    b.offset = best;
    total = std::max(total, best + b.bytes);
    placed.push_back(bi);
  }
  stats_.arena_bytes = total;
  stats_.weight_bytes = wblob_.size();

  ck(cudaSetDevice(device_), "cudaSetDevice");
  ck(cudaMalloc(&arena_, std::max<size_t>(total, kAlign)), "arena allocation");
  ck(cudaMalloc(&weights_, std::max<size_t>(wblob_.size(), kAlign)), "weight allocation");
  if (!wblob_.empty()) ck(cudaMemcpy(weights_, wblob_.data(), wblob_.size(), cudaMemcpyHostToDevice), "weight upload");
  wblob_.clear();
  wblob_.shrink_to_fit();
  ck(cudaMalloc(&err_, sizeof(unsigned int)), "error word allocation");
  ck(cudaMemset(err_, 0, sizeof(unsigned int)), "error word init");

  for (auto& p : pending_) {
    kinds_.push_back(p.kind);
    steps_.push_back(p.build());
  }
  pending_.clear();

  // Capture the kernel sequence once.
  cudaStream_t s;
  ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream create");
  bool ok = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
  if (ok) {
    for (auto& st : steps_)
      if (st(s) != cudaSuccess) ok = false;
    cudaGraph_t gph = nullptr;
    cudaError_t e = cudaStreamEndCapture(s, &gph);
    if (ok && e == cudaSuccess && gph) {
      graph_ = gph;
      if (cudaGraphInstantiate(&exec_, graph_, 0) != cudaSuccess) {
        exec_ = nullptr;
      }
    } else if (gph) {
      cudaGraphDestroy(gph);
    }
  }
  cudaGetLastError();   // clear capture errors; steps are replayed directly below if needed
  cudaStreamDestroy(s);
  if (debug_level() >= 1)
    std::fprintf(stderr, "[shorokoo_b200] plan dev%d: %zu launches (%lld tensor-core), arena %.1f MB, weights %.1f MB, %s\n",
                 device_, steps_.size(), (long long)stats_.tc_kernels, double(stats_.arena_bytes) / 1e6,
                 double(stats_.weight_bytes) / 1e6, exec_ ? "cuda graph" : "direct launches");
}

void Plan::enqueue_kernels(cudaStream_t stream) {
  if (exec_) {
    ck(cudaGraphLaunch(exec_, stream), "graph launch");
  } else {
    for (auto& st : steps_) ck(st(stream), "kernel launch");
  }
}

double Plan::time_kernels(cudaStream_t stream, int iters) {
  cudaEvent_t e0, e1;
  ck(cudaEventCreate(&e0), "event");
  ck(cudaEventCreate(&e1), "event");
  enqueue_kernels(stream);
  ck(cudaEventRecord(e0, stream), "event record");
  for (int i = 0; i < iters; ++i) enqueue_kernels(stream);
  ck(cudaEventRecord(e1, stream), "event record");
  ck(cudaEventSynchronize(e1), "event sync");
  float t = 0;
  ck(cudaEventElapsedTime(&t, e0, e1), "elapsed");
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  check_device_error();
  return double(t) / std::max(iters, 1);
}

void Plan::enqueue(cudaStream_t stream, const std::vector<const void*>& host_in, const std::vector<void*>& host_out) {
  for (auto& ib : inputs_) {
    SB_CHECK(size_t(ib.index) < host_in.size() && host_in[size_t(ib.index)], SB_INVALID_ARGUMENT, "missing input data");
    // (host or device-resident source: the runtime picks the direction)
    ck(cudaMemcpyAsync(buffer_ptr(ib.buf), host_in[size_t(ib.index)], ib.bytes, cudaMemcpyDefault, stream), "H2D");
  }
  enqueue_kernels(stream);
  enqueue_outputs(stream, host_out);
}

void Plan::enqueue_outputs(cudaStream_t stream, const std::vector<void*>& host_out) {
  for (size_t j = 0; j < outputs_.size(); ++j) {
    const OutputBinding& ob = outputs_[j];
    if (ob.host || j >= host_out.size() || !host_out[j]) continue;
    ck(cudaMemcpyAsync(host_out[j], ptr(ob.dev), size_t(numel(ob.shape)) * 4, cudaMemcpyDefault, stream), "D2H");
  }
}

std::vector<std::pair<std::string, double>> Plan::profile(cudaStream_t stream, int iters) {
  std::vector<std::pair<std::string, double>> out;
  cudaEvent_t e0, e1;
  ck(cudaEventCreate(&e0), "event");
  ck(cudaEventCreate(&e1), "event");
  for (size_t i = 0; i < steps_.size(); ++i) {
    ck(steps_[i](stream), "kernel launch");   // warm
    ck(cudaEventRecord(e0, stream), "event record");
    for (int r = 0; r < iters; ++r) ck(steps_[i](stream), "kernel launch");
    ck(cudaEventRecord(e1, stream), "event record");
    ck(cudaEventSynchronize(e1), "event sync");
    float t = 0;
    ck(cudaEventElapsedTime(&t, e0, e1), "elapsed");
    out.push_back({kinds_[i], double(t) / std::max(iters, 1)});
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return out;
}

void Plan::check_device_error() {
  unsigned int e = 0;
  ck(cudaMemcpy(&e, err_, sizeof(e), cudaMemcpyDeviceToHost), "error word read");
  if (e) {
    cudaMemset(err_, 0, sizeof(unsigned int));
    fail(SB_CUDA_ERROR, "device pipeline wait timed out (error word " + std::to_string(e) + ")");
  }
}

}  // namespace sb
