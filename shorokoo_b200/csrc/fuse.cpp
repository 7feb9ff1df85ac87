// Pattern fusion on the lowered graph.
//
//  Conv  [Pad folded into pads]  -> (Mul|Add|Sub|Div by per-channel constants)*  -> [Add residual]
//        -> [Relu|Sigmoid]                                          => FusedConv
//    The per-channel chain is the reference's inference-mode FrozenBatchNorm, emitted as primitive
//    ops over initializers (samples/RetinaNet/ResNet.cs:177-201): y = x*scale + shift with
//    scale = w / sqrt(var + eps), shift = b - mean*scale. It is folded into the conv weights and
//    bias in double precision: W' = W*scale, b' = b*scale + shift.
//    The residual may be a same-shape tensor (ResNet.cs:280-329) or the nearest-2x Resize of a
//    coarser map (FPN top-down add, RetinaNetDetector.cs:375-384,401-450).
//  MatMul(x, W^T constant) / Gemm -> (+bias) -> [Relu|Sigmoid]  => FusedGemm
//    (Linear, src/Shorokoo.Modules/Layers/Linear.cs:25-39; DenseBasic, ResNet.cs:102-125).
//  Reshape -> ReduceMean -> Sub / Mul / ReduceMean / Add(eps) / Sqrt / Div -> Reshape
//    -> (per-channel Mul|Add) -> [Relu]                           => GroupNorm (fuse_group_norms)
//  ReduceMean(last axis) -> Sub / Pow|Mul / ReduceMean / Add(eps) / Sqrt / Div -> (Mul|Add)
//                                                                 => LayerNorm (fuse_layer_norms)
//  MatMul(q, Transpose(k)) -> [scale] -> Softmax -> MatMul(., v)  => Attention (fuse_attention)
//
// A fused op takes the slot of the last op it absorbed, so operands that the original graph
// computes later (e.g. the projection shortcut of a bottleneck) are ready when it runs.
#include <algorithm>
#include <cmath>

#include "ir.h"

namespace sb {

namespace {

struct Consumers {
  std::vector<std::vector<int>> ops;   // per value: live consumer op indices
  std::vector<bool> is_output;
};

Consumers consumers(const LGraph& g) {
  Consumers c;
  c.ops.assign(g.vals.size(), {});
  c.is_output.assign(g.vals.size(), false);
  for (size_t i = 0; i < g.ops.size(); ++i) {
    const Op& op = g.ops[i];
    if (op.dead) continue;
    for (int id : op.in)
      if (id >= 0) c.ops[size_t(id)].push_back(int(i));
    if (op.residual >= 0) c.ops[size_t(op.residual)].push_back(int(i));
    if (op.concat >= 0) c.ops[size_t(op.concat)].push_back(int(i));
  }
  for (int id : g.outputs) c.is_output[size_t(id)] = true;
  return c;
}

// A FusedConv that is a plain 1x1, unpadded, ungrouped conv with stride 1 (or `stride` in both
// dimensions) and no second operand yet.
bool pointwise_conv(const Op& o, int64_t stride = 1) {
  if (o.dead || o.type != "FusedConv" || o.group != 1 || o.concat >= 0 || !o.weight) return false;
  const auto& w = o.weight->shape;
  if (w.size() != 4 || w[2] != 1 || w[3] != 1) return false;
  for (int64_t s : o.strides)
    if (s != stride) return false;
  for (int64_t d : o.dilations)
    if (d != 1) return false;
  for (int64_t p : o.pads)
    if (p != 0) return false;
  return true;
}

// Projection shortcut merged into the conv that adds it (the first bottleneck of a ResNet stage,
// ResNet.cs:280-329): y = act(X1*W1 + b1 + (X0*Ws + bs)) is one GEMM over X1's and X0's channels
// side by side, y = act([X1 X0] * [W1; Ws] + (b1 + bs)), so the shortcut's output is neither
// written nor read back. The shortcut may be strided (1x1 stride 2: X0 is then read at every other
// pixel). Both channel counts must be multiples of 64, so each operand fills whole k-tiles in
// every precision.
void merge_projection_shortcuts(LGraph& g) {
  const Consumers cons = consumers(g);
  auto uniform_stride = [](const Op& o) -> int64_t {
    if (o.strides.empty()) return 1;
    for (int64_t s : o.strides)
      if (s != o.strides[0]) return 0;
    return o.strides[0];
  };
  for (size_t i = 0; i < g.ops.size(); ++i) {
    Op& f = g.ops[i];   // the conv that absorbed the Add (its residual is the other conv's output)
    const int64_t sf = f.dead ? 0 : uniform_stride(f);
    if ((sf != 1 && sf != 2) || !pointwise_conv(f, sf) || f.residual < 0 || f.residual_mode != 0) continue;
    const int r = f.residual;
    const int pi = g.vals[size_t(r)].producer;
    if (pi < 0 || pi >= int(g.ops.size())) continue;
    Op& p = g.ops[size_t(pi)];
    const int64_t sp = p.dead ? 0 : uniform_stride(p);
    if ((sp != 1 && sp != 2) || !pointwise_conv(p, sp) || p.act != 0 || p.residual >= 0 || p.out.size() != 1 ||
        p.out[0] != r)
      continue;
    if (cons.is_output[size_t(r)] || cons.ops[size_t(r)].size() != 1) continue;
    // main: the stride-1 conv (its input X1 is the GEMM's first operand); shortcut: the other (X0,
    // read at its stride). Either may be the one that absorbed the Add, depending on node order.
    if (sf != 1 && sp != 1) continue;
    const bool f_main = sf == 1;
    const Op& mo = f_main ? f : p;
    const Op& so = f_main ? p : f;
    const int64_t ss = f_main ? sp : sf;
    const int x1id = mo.in[0], x0id = so.in[0];
    const Value& x1 = g.vals[size_t(x1id)];
    const Value& x0 = g.vals[size_t(x0id)];
    if (x1.is_host || x0.is_host || x1.shape.size() != 4 || x0.shape.size() != 4) continue;
    if (x1.shape[0] != x0.shape[0] || (x0.shape[2] - 1) / ss + 1 != x1.shape[2] ||
        (x0.shape[3] - 1) / ss + 1 != x1.shape[3])
      continue;
    const int64_t M = mo.weight->shape[0], C1 = mo.weight->shape[1], C0 = so.weight->shape[1];
    if (so.weight->shape[0] != M || C1 != x1.shape[1] || C0 != x0.shape[1] || C1 % 64 || C0 % 64) continue;
    auto w = std::make_shared<HostTensor>(DT_FLOAT, std::vector<int64_t>{M, C1 + C0, 1, 1});
    const float* w1 = mo.weight->ptr<float>();
    const float* w0 = so.weight->ptr<float>();
    float* wp = w->mptr<float>();
    for (int64_t m = 0; m < M; ++m) {
      for (int64_t c = 0; c < C1; ++c) wp[m * (C1 + C0) + c] = w1[m * C1 + c];
      for (int64_t c = 0; c < C0; ++c) wp[m * (C1 + C0) + C1 + c] = w0[m * C0 + c];
    }
    auto b = std::make_shared<HostTensor>(DT_FLOAT, std::vector<int64_t>{M});
    float* bp = b->mptr<float>();
    for (int64_t m = 0; m < M; ++m)
      bp[m] = (f.bias ? f.bias->ptr<float>()[m] : 0.f) + (p.bias ? p.bias->ptr<float>()[m] : 0.f);
    // the merged conv keeps f's slot, output and activation
    f.in[0] = x1id;
    f.strides.assign(f.strides.size(), 1);
    f.weight = w;
    f.bias = b;
    f.concat = x0id;
    f.concat_stride = int(ss);
    f.residual = -1;
    p.dead = true;
  }
}

// Host tensor that broadcasts against an output of `rank` dims and varies at most along `axis`
// (size `len`); returns the per-index values (length len).
bool per_axis_values(const HostTensor& h, size_t rank, size_t axis, int64_t len, std::vector<double>& out) {
  if (h.shape.size() > rank) return false;
  size_t off = rank - h.shape.size();
  int64_t along = 1;
  for (size_t i = 0; i < h.shape.size(); ++i) {
    size_t d = i + off;
    if (d == axis) {
      along = h.shape[i];
      if (along != 1 && along != len) return false;
    } else if (h.shape[i] != 1) {
      return false;
    }
  }
  out.resize(size_t(len));
  for (int64_t m = 0; m < len; ++m) out[size_t(m)] = h.get_f64(along == 1 ? 0 : m);
  return true;
}

std::shared_ptr<HostTensor> to_f32(const HostTensor& h) {
  auto o = std::make_shared<HostTensor>(DT_FLOAT, h.shape);
  if (h.dtype == DT_FLOAT) {
    std::memcpy(o->mutable_data(), h.data(), h.nbytes());
  } else {
    float* p = o->mptr<float>();
    for (int64_t i = 0; i < h.numel(); ++i) p[i] = float(h.get_f64(i));
  }
  return o;
}

// Resize that maps output index o to floor(o/2) on the two spatial axes and is identity elsewhere.
bool is_nearest_up2(const Op& r, const LGraph& g) {
  if (r.type != "Resize" || r.dead) return false;
  if (r.scales.size() != 4 || r.scales[0] != 1.f || r.scales[1] != 1.f || r.scales[2] != 2.f || r.scales[3] != 2.f)
    return false;
  const auto& xs = g.vals[size_t(r.in[0])].shape;
  const auto& ys = g.vals[size_t(r.out[0])].shape;
  if (xs.size() != 4 || ys[2] != 2 * xs[2] || ys[3] != 2 * xs[3]) return false;
  bool hp = r.coord_mode == "half_pixel" || r.coord_mode == "pytorch_half_pixel";
  bool asym = r.coord_mode == "asymmetric";
  if (hp) return r.nearest_mode == "round_prefer_floor";
  if (asym) return r.nearest_mode == "floor" || r.nearest_mode == "round_prefer_floor";
  return false;
}

}  // namespace

// Sigmoid / Relu of a value that only rearranges the outputs of activation-free contractions
// (views and concatenations, e.g. the RetinaNet heads' Reshape -> Transpose(0,3,4,1,2) -> Reshape
// -> Concat over the pyramid levels followed by the class Sigmoid, RetinaNetDetector.cs:539-571)
// is applied per element in those contractions' epilogues; the elementwise op becomes an Identity.
// Every value on the way must have that single reader and be no graph output.
static void push_activation_into_producers(LGraph& g) {
  Consumers C = consumers(g);
  for (Op& e : g.ops) {
    if (e.dead || (e.type != "Sigmoid" && e.type != "Relu") || e.in.size() != 1 || e.in[0] < 0) continue;
    std::vector<int> producers;
    bool ok = true;
    std::vector<int> todo{e.in[0]};
    while (ok && !todo.empty()) {
      const int v = todo.back();
      todo.pop_back();
      const Value& val = g.vals[size_t(v)];
      if (val.is_host || C.is_output[size_t(v)] || C.ops[size_t(v)].size() != 1 || val.producer < 0) {
        ok = false;
        break;
      }
      const Op& p = g.ops[size_t(val.producer)];
      if (p.dead) {
        ok = false;
      } else if (p.type == "FusedConv" || p.type == "FusedGemm") {
        if (p.act != 0) ok = false;
        else producers.push_back(val.producer);
      } else if (p.type == "Reshape" || p.type == "Transpose" || p.type == "Identity") {
        todo.push_back(p.in[0]);
      } else if (p.type == "Concat") {
        for (int id : p.in) todo.push_back(id);
      } else {
        ok = false;
      }
    }
    if (!ok || producers.empty()) continue;
    for (int pi : producers) g.ops[size_t(pi)].act = e.type == "Sigmoid" ? 2 : 1;
    e.type = "Identity";
  }
}

// GroupNorm written out in primitives, as the exporter emits RetGroupNorm
// (samples/RetinaNet/RetinaNetDetector.cs:337-372) and the GroupNorm layer
// (src/Shorokoo.Modules/Layers/Normalization.cs:278-310):
//   xr  = Reshape(x [N, C, H, W] -> [N, G, ...])       (a split of the channel axis)
//   mu  = ReduceMean(xr, axes 2.., keepdims)
//   d_i = Sub(xr, mu)                                   (one or more such nodes)
//   var = ReduceMean(Mul(d_a, d_b), axes 2.., keepdims)
//   y   = Reshape(Div(d_c, Sqrt(Add(var, eps))) -> [N, C, H, W])
//   then per-channel Mul / Add / Sub / Div by constants (gamma, beta) and an optional Relu
// => GroupNorm(x): group = G, alpha = eps, weight / bias = the per-channel scale and shift, act.
static void fuse_group_norms(LGraph& g) {
  for (size_t mi = 0; mi < g.ops.size(); ++mi) {
    if (g.ops[mi].dead || g.ops[mi].type != "ReduceMean" || !g.ops[mi].keepdims) continue;
    Consumers C = consumers(g);
    const Op m1 = g.ops[mi];
    const int xr = m1.in[0];
    const Value& xrv = g.vals[size_t(xr)];
    if (xrv.producer < 0 || C.is_output[size_t(xr)]) continue;
    const int r1i = xrv.producer;
    const Op& r1 = g.ops[size_t(r1i)];
    if (r1.dead || r1.type != "Reshape") continue;
    const int x = r1.in[0];
    const Value& xv = g.vals[size_t(x)];
    if (xv.is_host || xv.shape.size() != 4) continue;
    const int64_t N = xv.shape[0], Ch = xv.shape[1], H = xv.shape[2], W = xv.shape[3];
    const auto& rs = xrv.shape;
    if (rs.size() < 3 || rs[0] != N || rs[1] < 1 || Ch % rs[1] != 0) continue;
    const int64_t G = rs[1];
    // the kernel's shapes: channel groups of a power of two up to 32, channels in 16-byte vectors
    // (other shapes keep the primitives)
    const int64_t cpg = Ch / G;
    if (cpg > 32 || (cpg & (cpg - 1)) != 0 || Ch % 8 != 0) continue;
    int64_t rest = 1;
    for (size_t i = 2; i < rs.size(); ++i) rest *= rs[i];
    if (rest != (Ch / G) * H * W) continue;
    // the reduced axes are exactly 2 .. rank-1
    bool ok = m1.axes.size() == rs.size() - 2;
    for (size_t i = 0; ok && i < m1.axes.size(); ++i) ok = m1.axes[i] == int64_t(i + 2);
    if (!ok) continue;
    const int mu = m1.out[0];
    if (C.is_output[size_t(mu)]) continue;
    // mu feeds only Sub(xr, mu) nodes; xr feeds only m1 and those
    std::vector<int> subs, sub_outs;
    for (int oi : C.ops[size_t(mu)]) {
      const Op& o = g.ops[size_t(oi)];
      if (o.type != "Sub" || o.in.size() != 2 || o.in[0] != xr || o.in[1] != mu) ok = false;
      subs.push_back(oi);
      sub_outs.push_back(o.out[0]);
    }
    if (!ok || subs.empty() || C.ops[size_t(xr)].size() != subs.size() + 1) continue;
    auto is_sub_out = [&](int v) { return std::find(sub_outs.begin(), sub_outs.end(), v) != sub_outs.end(); };
    // the square and the normalising division, reading only sub outputs
    int sq = -1, dv = -1;
    for (int so : sub_outs) {
      if (C.is_output[size_t(so)]) ok = false;
      for (int oi : C.ops[size_t(so)]) {
        const Op& o = g.ops[size_t(oi)];
        if (o.type == "Mul" && o.in.size() == 2 && is_sub_out(o.in[0]) && is_sub_out(o.in[1]) && (sq < 0 || sq == oi))
          sq = oi;
        else if (o.type == "Div" && o.in.size() == 2 && is_sub_out(o.in[0]) && (dv < 0 || dv == oi))
          dv = oi;
        else
          ok = false;
      }
    }
    if (!ok || sq < 0 || dv < 0) continue;
    auto single = [&](int v) -> int {   // the one consumer of v (-1 when none, several or an output)
      if (C.is_output[size_t(v)] || C.ops[size_t(v)].size() != 1) return -1;
      return C.ops[size_t(v)][0];
    };
    const int m2 = single(g.ops[size_t(sq)].out[0]);
    if (m2 < 0 || g.ops[size_t(m2)].type != "ReduceMean" || g.ops[size_t(m2)].axes != m1.axes ||
        !g.ops[size_t(m2)].keepdims)
      continue;
    const int ad = single(g.ops[size_t(m2)].out[0]);
    if (ad < 0 || g.ops[size_t(ad)].type != "Add" || g.ops[size_t(ad)].in.size() != 2) continue;
    const Op& add = g.ops[size_t(ad)];
    const int ev = add.in[0] == g.ops[size_t(m2)].out[0] ? add.in[1] : add.in[0];
    if (!g.vals[size_t(ev)].is_host || g.vals[size_t(ev)].host->numel() != 1) continue;
    const double eps = g.vals[size_t(ev)].host->get_f64(0);
    const int sr = single(add.out[0]);
    if (sr < 0 || g.ops[size_t(sr)].type != "Sqrt") continue;
    if (single(g.ops[size_t(sr)].out[0]) != dv || g.ops[size_t(dv)].in[1] != g.ops[size_t(sr)].out[0]) continue;
    const int r2 = single(g.ops[size_t(dv)].out[0]);
    if (r2 < 0 || g.ops[size_t(r2)].type != "Reshape" || g.vals[size_t(g.ops[size_t(r2)].out[0])].shape != xv.shape)
      continue;
    // per-channel affine and activation after the normalisation
    std::vector<double> scale(size_t(Ch), 1.0), shift(size_t(Ch), 0.0);
    int cur = g.ops[size_t(r2)].out[0];
    int slot = r2;
    std::vector<int> absorbed = {r1i, int(mi), sq, m2, ad, sr, dv, r2};
    absorbed.insert(absorbed.end(), subs.begin(), subs.end());
    int act = 0;
    while (true) {
      const int oi = single(cur);
      if (oi < 0) break;
      const Op& o = g.ops[size_t(oi)];
      if ((o.type == "Mul" || o.type == "Add" || o.type == "Sub" || o.type == "Div") && o.in.size() == 2 && act == 0) {
        const bool cur_first = o.in[0] == cur;
        const Value& ov = g.vals[size_t(cur_first ? o.in[1] : o.in[0])];
        std::vector<double> v;
        if (!ov.is_host || !per_axis_values(*ov.host, 4, 1, Ch, v) || g.vals[size_t(o.out[0])].shape != xv.shape) break;
        if ((o.type == "Sub" || o.type == "Div") && !cur_first) break;
        for (int64_t c = 0; c < Ch; ++c) {
          const double k = v[size_t(c)];
          if (o.type == "Mul") {
            scale[size_t(c)] *= k;
            shift[size_t(c)] *= k;
          } else if (o.type == "Add") {
            shift[size_t(c)] += k;
          } else if (o.type == "Sub") {
            shift[size_t(c)] -= k;
          } else {
            scale[size_t(c)] /= k;
            shift[size_t(c)] /= k;
          }
        }
      } else if (o.type == "Relu" && act == 0) {
        act = 1;
      } else {
        break;
      }
      absorbed.push_back(oi);
      cur = o.out[0];
      slot = oi;
    }
    Op f;
    f.type = "GroupNorm";
    f.name = m1.name;
    f.in = {x};
    f.out = {cur};
    f.group = G;
    f.alpha = float(eps);
    f.act = act;
    f.weight = std::make_shared<HostTensor>(DT_FLOAT, std::vector<int64_t>{Ch});
    f.bias = std::make_shared<HostTensor>(DT_FLOAT, std::vector<int64_t>{Ch});
    for (int64_t c = 0; c < Ch; ++c) {
      f.weight->mptr<float>()[c] = float(scale[size_t(c)]);
      f.bias->mptr<float>()[c] = float(shift[size_t(c)]);
    }
    for (int a : absorbed) g.ops[size_t(a)].dead = true;
    g.vals[size_t(cur)].producer = slot;
    g.ops[size_t(slot)] = f;
  }
}

// LayerNorm written out in primitives (ViTLayerNorm, samples/RetinaNet/ViTNet.cs:51-72):
//   mu = ReduceMean(x, last axis, keepdims); d_i = Sub(x, mu); var = ReduceMean(Pow(d, 2) or
//   Mul(d_a, d_b), last axis, keepdims); y = Div(d_c, Sqrt(Add(var, eps))); then Mul / Add / Sub /
//   Div by constants varying along the last axis (gamma, beta)
// => LayerNorm(x): alpha = eps, weight / bias = the per-feature scale and shift.
static void fuse_layer_norms(LGraph& g) {
  for (size_t mi = 0; mi < g.ops.size(); ++mi) {
    if (g.ops[mi].dead || g.ops[mi].type != "ReduceMean" || !g.ops[mi].keepdims) continue;
    Consumers C = consumers(g);
    const Op m1 = g.ops[mi];
    const int x = m1.in[0];
    const Value& xv = g.vals[size_t(x)];
    if (xv.is_host || xv.shape.size() < 2) continue;
    const int64_t r = int64_t(xv.shape.size()), D = xv.shape.back();
    if (m1.axes.size() != 1 || m1.axes[0] != r - 1) continue;
    const int mu = m1.out[0];
    if (C.is_output[size_t(mu)]) continue;
    bool ok = true;
    std::vector<int> subs, sub_outs;
    for (int oi : C.ops[size_t(mu)]) {
      const Op& o = g.ops[size_t(oi)];
      if (o.type != "Sub" || o.in.size() != 2 || o.in[0] != x || o.in[1] != mu) ok = false;
      subs.push_back(oi);
      sub_outs.push_back(o.out[0]);
    }
    if (!ok || subs.empty()) continue;
    auto is_sub_out = [&](int v) { return std::find(sub_outs.begin(), sub_outs.end(), v) != sub_outs.end(); };
    int sq = -1, dv = -1;
    for (int so : sub_outs) {
      if (C.is_output[size_t(so)]) ok = false;
      for (int oi : C.ops[size_t(so)]) {
        const Op& o = g.ops[size_t(oi)];
        const bool square = (o.type == "Mul" && o.in.size() == 2 && is_sub_out(o.in[0]) && is_sub_out(o.in[1])) ||
                            (o.type == "Pow" && o.in.size() == 2 && is_sub_out(o.in[0]) && g.vals[size_t(o.in[1])].is_host &&
                             g.vals[size_t(o.in[1])].host->numel() == 1 && g.vals[size_t(o.in[1])].host->get_f64(0) == 2.0);
        if (square && (sq < 0 || sq == oi))
          sq = oi;
        else if (o.type == "Div" && o.in.size() == 2 && is_sub_out(o.in[0]) && (dv < 0 || dv == oi))
          dv = oi;
        else
          ok = false;
      }
    }
    if (!ok || sq < 0 || dv < 0) continue;
    auto single = [&](int v) -> int {
      if (C.is_output[size_t(v)] || C.ops[size_t(v)].size() != 1) return -1;
      return C.ops[size_t(v)][0];
    };
    const int m2 = single(g.ops[size_t(sq)].out[0]);
    if (m2 < 0 || g.ops[size_t(m2)].type != "ReduceMean" || g.ops[size_t(m2)].axes != m1.axes ||
        !g.ops[size_t(m2)].keepdims)
      continue;
    const int ad = single(g.ops[size_t(m2)].out[0]);
    if (ad < 0 || g.ops[size_t(ad)].type != "Add" || g.ops[size_t(ad)].in.size() != 2) continue;
    const Op& add = g.ops[size_t(ad)];
    const int ev = add.in[0] == g.ops[size_t(m2)].out[0] ? add.in[1] : add.in[0];
    if (!g.vals[size_t(ev)].is_host || g.vals[size_t(ev)].host->numel() != 1) continue;
    const double eps = g.vals[size_t(ev)].host->get_f64(0);
    const int sr = single(add.out[0]);
    if (sr < 0 || g.ops[size_t(sr)].type != "Sqrt") continue;
    if (single(g.ops[size_t(sr)].out[0]) != dv || g.ops[size_t(dv)].in[1] != g.ops[size_t(sr)].out[0]) continue;
    std::vector<double> scale(size_t(D), 1.0), shift(size_t(D), 0.0);
    int cur = g.ops[size_t(dv)].out[0];
    int slot = dv;
    std::vector<int> absorbed = {int(mi), sq, m2, ad, sr, dv};
    absorbed.insert(absorbed.end(), subs.begin(), subs.end());
    while (true) {
      const int oi = single(cur);
      if (oi < 0) break;
      const Op& o = g.ops[size_t(oi)];
      if (!((o.type == "Mul" || o.type == "Add" || o.type == "Sub" || o.type == "Div") && o.in.size() == 2)) break;
      const bool cur_first = o.in[0] == cur;
      const Value& ov = g.vals[size_t(cur_first ? o.in[1] : o.in[0])];
      std::vector<double> v;
      if (!ov.is_host || !per_axis_values(*ov.host, size_t(r), size_t(r - 1), D, v) ||
          g.vals[size_t(o.out[0])].shape != xv.shape)
        break;
      if ((o.type == "Sub" || o.type == "Div") && !cur_first) break;
      for (int64_t c = 0; c < D; ++c) {
        const double k = v[size_t(c)];
        if (o.type == "Mul") {
          scale[size_t(c)] *= k;
          shift[size_t(c)] *= k;
        } else if (o.type == "Add") {
          shift[size_t(c)] += k;
        } else if (o.type == "Sub") {
          shift[size_t(c)] -= k;
        } else {
          scale[size_t(c)] /= k;
          shift[size_t(c)] /= k;
        }
      }
      absorbed.push_back(oi);
      cur = o.out[0];
      slot = oi;
    }
    Op f;
    f.type = "LayerNorm";
    f.name = m1.name;
    f.in = {x};
    f.out = {cur};
    f.alpha = float(eps);
    f.weight = std::make_shared<HostTensor>(DT_FLOAT, std::vector<int64_t>{D});
    f.bias = std::make_shared<HostTensor>(DT_FLOAT, std::vector<int64_t>{D});
    for (int64_t c = 0; c < D; ++c) {
      f.weight->mptr<float>()[c] = float(scale[size_t(c)]);
      f.bias->mptr<float>()[c] = float(shift[size_t(c)]);
    }
    for (int a : absorbed) g.ops[size_t(a)].dead = true;
    g.vals[size_t(cur)].producer = slot;
    g.ops[size_t(slot)] = f;
  }
}

// Scaled dot-product attention written out in primitives (ViTAttention, ViTNet.cs:155-207):
//   s = MatMul(q, Transpose(k, last two axes)) [* or / a scalar]; p = Softmax(s, last axis);
//   y = MatMul(p, v), with q, k, v [..., S, hd] device tensors
// => Attention(q, k, v): alpha = the scale on the scores.
static void fuse_attention(LGraph& g) {
  for (size_t mi = 0; mi < g.ops.size(); ++mi) {
    if (g.ops[mi].dead || g.ops[mi].type != "MatMul" || g.ops[mi].in.size() != 2) continue;
    Consumers C = consumers(g);
    const Op mm1 = g.ops[mi];
    const int q = mm1.in[0], kt = mm1.in[1];
    const Value& qv = g.vals[size_t(q)];
    const Value& ktv = g.vals[size_t(kt)];
    if (qv.is_host || ktv.is_host || qv.shape.size() < 3 || ktv.producer < 0) continue;
    const int ti = ktv.producer;
    const Op& tr = g.ops[size_t(ti)];
    if (tr.dead || tr.type != "Transpose") continue;
    const size_t r = qv.shape.size();
    bool ok = tr.perm.size() == r;
    for (size_t i = 0; ok && i < r; ++i)
      ok = tr.perm[i] == int64_t(i + 2 == r ? r - 1 : (i + 1 == r ? r - 2 : i));
    if (!ok) continue;
    const int k = tr.in[0];
    if (g.vals[size_t(k)].shape != qv.shape) continue;
    auto single = [&](int v) -> int {
      if (C.is_output[size_t(v)] || C.ops[size_t(v)].size() != 1) return -1;
      return C.ops[size_t(v)][0];
    };
    int cur = mm1.out[0];
    double scale = 1.0;
    std::vector<int> absorbed = {int(mi)};
    int oi = single(cur);
    if (oi >= 0 && (g.ops[size_t(oi)].type == "Mul" || g.ops[size_t(oi)].type == "Div") && g.ops[size_t(oi)].in.size() == 2) {
      const Op& o = g.ops[size_t(oi)];
      const bool cur_first = o.in[0] == cur;
      const Value& sv = g.vals[size_t(cur_first ? o.in[1] : o.in[0])];
      if (sv.is_host && sv.host->numel() == 1 && (o.type == "Mul" || cur_first)) {
        scale = o.type == "Mul" ? sv.host->get_f64(0) : 1.0 / sv.host->get_f64(0);
        absorbed.push_back(oi);
        cur = o.out[0];
        oi = single(cur);
      }
    }
    if (oi < 0 || g.ops[size_t(oi)].type != "Softmax" || g.ops[size_t(oi)].axis != int64_t(r - 1)) continue;
    absorbed.push_back(oi);
    cur = g.ops[size_t(oi)].out[0];
    const int m2 = single(cur);
    if (m2 < 0 || g.ops[size_t(m2)].type != "MatMul" || g.ops[size_t(m2)].in[0] != cur) continue;
    const int v = g.ops[size_t(m2)].in[1];
    const Value& vv = g.vals[size_t(v)];
    if (vv.is_host || vv.shape != qv.shape) continue;
    absorbed.push_back(m2);
    Op f;
    f.type = "Attention";
    f.name = mm1.name;
    f.in = {q, k, v};
    f.out = g.ops[size_t(m2)].out;
    f.alpha = float(scale);
    for (int a : absorbed) g.ops[size_t(a)].dead = true;
    if (C.ops[size_t(kt)].size() == 1 && !C.is_output[size_t(kt)]) g.ops[size_t(ti)].dead = true;
    g.vals[size_t(f.out[0])].producer = m2;
    g.ops[size_t(m2)] = f;
  }
}

void fuse(LGraph& g) {
  // ---------------- Conv chains ----------------
  for (size_t ci = 0; ci < g.ops.size(); ++ci) {
    if (g.ops[ci].dead || g.ops[ci].type != "Conv") continue;
    Consumers C = consumers(g);
    Op conv = g.ops[ci];
    int x = conv.in[0];
    // Fold a zero constant Pad on the spatial axes into the conv padding (ResNet stem, ResNet.cs:364).
    const Value& xv = g.vals[size_t(x)];
    if (xv.producer >= 0) {
      const Op& p = g.ops[size_t(xv.producer)];
      if (!p.dead && p.type == "Pad" && p.alpha == 0.f && p.pads.size() == 8 && p.pads[0] == 0 && p.pads[1] == 0 &&
          p.pads[4] == 0 && p.pads[5] == 0 && C.ops[size_t(x)].size() == 1 && !C.is_output[size_t(x)]) {
        conv.pads[0] += p.pads[2];
        conv.pads[1] += p.pads[3];
        conv.pads[2] += p.pads[6];
        conv.pads[3] += p.pads[7];
        g.ops[size_t(xv.producer)].dead = true;
        x = p.in[0];
      }
    }
    const HostTensor& W = *g.vals[size_t(conv.in[1])].host;
    const int64_t M = W.shape[0];
    Op f;
    f.type = "FusedConv";
    f.name = conv.name;
    f.in = {x};
    f.kernel = conv.kernel;
    f.strides = conv.strides;
    f.pads = conv.pads;
    f.dilations = conv.dilations;
    f.group = conv.group;
    f.weight = to_f32(W);
    f.bias = std::make_shared<HostTensor>(DT_FLOAT, std::vector<int64_t>{M});
    std::vector<double> scale(size_t(M), 1.0), shift(size_t(M), 0.0);
    if (conv.in.size() > 2 && conv.in[2] >= 0) {
      const HostTensor& b = *g.vals[size_t(conv.in[2])].host;
      SB_CHECK(b.numel() == M, SB_SHAPE_ERROR, "Conv: bias length mismatch");
      for (int64_t m = 0; m < M; ++m) shift[size_t(m)] = b.get_f64(m);
    }
    int cur = conv.out[0];
    int slot = int(ci);
    std::vector<int> absorbed;
    while (true) {
      if (C.is_output[size_t(cur)] || C.ops[size_t(cur)].size() != 1) break;
      int oi = C.ops[size_t(cur)][0];
      const Op& o = g.ops[size_t(oi)];
      if (o.residual >= 0) break;
      auto other_of = [&](const Op& op) { return op.in[0] == cur ? op.in[1] : op.in[0]; };
      bool done = false;
      if ((o.type == "Mul" || o.type == "Add" || o.type == "Sub" || o.type == "Div") && o.in.size() == 2 &&
          f.residual < 0 && f.act == 0) {
        int other = other_of(o);
        const Value& ov = g.vals[size_t(other)];
        std::vector<double> v;
        if (ov.is_host && per_axis_values(*ov.host, 4, 1, M, v) &&
            g.vals[size_t(o.out[0])].shape == g.vals[size_t(cur)].shape) {
          bool cur_first = o.in[0] == cur;
          for (int64_t m = 0; m < M; ++m) {
            double k = v[size_t(m)];
            if (o.type == "Mul") {
              scale[size_t(m)] *= k;
              shift[size_t(m)] *= k;
            } else if (o.type == "Add") {
              shift[size_t(m)] += k;
            } else if (o.type == "Sub") {
              if (cur_first) {
                shift[size_t(m)] -= k;
              } else {
                scale[size_t(m)] = -scale[size_t(m)];
                shift[size_t(m)] = k - shift[size_t(m)];
              }
            } else {   // Div
              if (!cur_first) { done = true; break; }
              scale[size_t(m)] /= k;
              shift[size_t(m)] /= k;
            }
          }
          if (done) break;
          absorbed.push_back(oi);
          cur = o.out[0];
          slot = oi;
          continue;
        }
        if (o.type == "Add" && !ov.is_host && f.residual < 0) {
          // Nearest-2x upsampled operand: read the coarse map directly in the epilogue.
          if (ov.producer >= 0 && is_nearest_up2(g.ops[size_t(ov.producer)], g) &&
              g.vals[size_t(o.out[0])].shape == g.vals[size_t(cur)].shape) {
            const Op& rz = g.ops[size_t(ov.producer)];
            f.residual = rz.in[0];
            f.residual_mode = 1;
            absorbed.push_back(oi);
            cur = o.out[0];
            slot = oi;
            continue;
          }
          if (ov.shape == g.vals[size_t(cur)].shape) {
            f.residual = other;
            f.residual_mode = 0;
            absorbed.push_back(oi);
            cur = o.out[0];
            slot = oi;
            continue;
          }
        }
        break;
      }
      if ((o.type == "Relu" || o.type == "Sigmoid" || o.type == "Gelu") && f.act == 0) {
        f.act = o.type == "Relu" ? 1 : (o.type == "Sigmoid" ? 2 : (o.mode == "tanh" ? 3 : 4));
        absorbed.push_back(oi);
        cur = o.out[0];
        slot = oi;
        continue;
      }
      break;
    }
    // Fold scale/shift into weights and bias.
    const int64_t per = f.weight->numel() / std::max<int64_t>(M, 1);
    float* wp = f.weight->mptr<float>();
    float* bp = f.bias->mptr<float>();
    for (int64_t m = 0; m < M; ++m) {
      const double s = scale[size_t(m)];
      if (s != 1.0)
        for (int64_t j = 0; j < per; ++j) wp[m * per + j] = float(double(wp[m * per + j]) * s);
      bp[m] = float(shift[size_t(m)]);
    }
    f.out = {cur};
    g.ops[ci].dead = true;
    for (int a : absorbed) g.ops[size_t(a)].dead = true;
    g.vals[size_t(cur)].producer = slot;
    g.ops[size_t(slot)] = f;
  }

  // ---------------- MatMul / Gemm chains ----------------
  for (size_t mi = 0; mi < g.ops.size(); ++mi) {
    Op& mm0 = g.ops[mi];
    if (mm0.dead || (mm0.type != "MatMul" && mm0.type != "Gemm")) continue;
    int bid = mm0.in[1];
    if (bid < 0 || !g.vals[size_t(bid)].is_host) continue;   // device x device: planned as a generic GEMM
    if (mm0.type == "Gemm" && mm0.axes[0] != 0) continue;        // transA: planned generically
    Consumers C = consumers(g);
    Op mm = mm0;
    const HostTensor& B = *g.vals[size_t(bid)].host;
    Op f;
    f.type = "FusedGemm";
    f.name = mm.name;
    f.in = {mm.in[0]};
    // W = [N, K]
    bool b_is_nk = mm.type == "Gemm" && mm.axes[1] != 0;
    if (!b_is_nk && B.transpose_src && !B.buf) {
      f.weight = to_f32(*B.transpose_src);   // MatMul(x, Transpose(W)): use W directly
    } else if (b_is_nk) {
      f.weight = to_f32(B);
    } else {
      HostTensor bt = B;
      auto t = std::make_shared<HostTensor>(B.dtype, std::vector<int64_t>{B.shape[1], B.shape[0]});
      size_t es = dtype_size(B.dtype);
      const uint8_t* s = bt.data();
      uint8_t* d = t->mutable_data();
      for (int64_t i = 0; i < B.shape[0]; ++i)
        for (int64_t j = 0; j < B.shape[1]; ++j) std::memcpy(d + (j * B.shape[0] + i) * es, s + (i * B.shape[1] + j) * es, es);
      f.weight = to_f32(*t);
    }
    const int64_t N = f.weight->shape[0];
    f.bias = std::make_shared<HostTensor>(DT_FLOAT, std::vector<int64_t>{N});
    std::vector<double> shift(size_t(N), 0.0), scale(size_t(N), 1.0);
    if (mm.type == "Gemm") {
      if (mm.alpha != 1.f)
        for (auto& s : scale) s = mm.alpha;
      if (mm.in.size() > 2 && mm.in[2] >= 0) {
        const Value& cv = g.vals[size_t(mm.in[2])];
        std::vector<double> v;
        SB_CHECK(cv.is_host && per_axis_values(*cv.host, 2, 1, N, v), SB_UNSUPPORTED,
                 "Gemm: bias must be a plan-time constant broadcast along columns");
        for (int64_t n = 0; n < N; ++n) shift[size_t(n)] = double(mm.beta) * v[size_t(n)];
      }
    }
    int cur = mm.out[0];
    const size_t rank = g.vals[size_t(cur)].shape.size();
    int slot = int(mi);
    std::vector<int> absorbed;
    while (true) {
      if (C.is_output[size_t(cur)] || C.ops[size_t(cur)].size() != 1) break;
      int oi = C.ops[size_t(cur)][0];
      const Op& o = g.ops[size_t(oi)];
      if (o.residual >= 0) break;
      if ((o.type == "Add" || o.type == "Mul") && o.in.size() == 2 && f.act == 0 && f.residual < 0) {
        int other = o.in[0] == cur ? o.in[1] : o.in[0];
        const Value& ov = g.vals[size_t(other)];
        std::vector<double> v;
        if (ov.is_host && per_axis_values(*ov.host, rank, rank - 1, N, v) &&
            g.vals[size_t(o.out[0])].shape == g.vals[size_t(cur)].shape) {
          for (int64_t n = 0; n < N; ++n) {
            if (o.type == "Add") {
              shift[size_t(n)] += v[size_t(n)];
            } else {
              scale[size_t(n)] *= v[size_t(n)];
              shift[size_t(n)] *= v[size_t(n)];
            }
          }
          absorbed.push_back(oi);
          cur = o.out[0];
          slot = oi;
          continue;
        }
        if (o.type == "Add" && !ov.is_host && ov.shape == g.vals[size_t(cur)].shape) {
          f.residual = other;
          absorbed.push_back(oi);
          cur = o.out[0];
          slot = oi;
          continue;
        }
        break;
      }
      if ((o.type == "Relu" || o.type == "Sigmoid" || o.type == "Gelu") && f.act == 0) {
        f.act = o.type == "Relu" ? 1 : (o.type == "Sigmoid" ? 2 : (o.mode == "tanh" ? 3 : 4));
        absorbed.push_back(oi);
        cur = o.out[0];
        slot = oi;
        continue;
      }
      break;
    }
    const int64_t K = f.weight->shape[1];
    float* wp = f.weight->mptr<float>();
    float* bp = f.bias->mptr<float>();
    for (int64_t n = 0; n < N; ++n) {
      if (scale[size_t(n)] != 1.0)
        for (int64_t k = 0; k < K; ++k) wp[n * K + k] = float(double(wp[n * K + k]) * scale[size_t(n)]);
      bp[n] = float(shift[size_t(n)]);
    }
    f.out = {cur};
    g.ops[mi].dead = true;
    for (int a : absorbed) g.ops[size_t(a)].dead = true;
    g.vals[size_t(cur)].producer = slot;
    g.ops[size_t(slot)] = f;
  }
  merge_projection_shortcuts(g);
  fuse_group_norms(g);
  fuse_layer_norms(g);
  fuse_attention(g);
  push_activation_into_producers(g);
  g.dce();
}

}  // namespace sb
