// Plan-time specialisation of an ONNX model:
//  * inlines model-local functions (FastOnnxModelBuilder.cs:1116-1190 emits them in domain
//    "Functions"),
//  * folds everything computable from initializers, Constant nodes, input shapes and plan-time
//    input values on the host (the runtime shape chains of FastProcessors.cs:4691),
//  * resolves If with a host-known condition and unrolls Loop with a host-known trip count
//    (the live-[Hyper] control flow of FastOnnxModelBuilder.cs:1199-1300),
//  * infers shapes of the remaining device ops.
#include <algorithm>
#include <cmath>
#include <functional>
#include <set>
#include <unordered_map>

#include "ir.h"

namespace sb {

namespace {

const std::set<std::string> kDeviceOps = {
    "Conv", "MaxPool", "AveragePool", "GlobalAveragePool", "GlobalMaxPool", "MatMul", "Gemm",
    "Relu", "Sigmoid", "Tanh", "Sqrt", "Neg", "Abs", "Exp", "Log", "Reciprocal", "Floor", "Ceil", "Erf",
    "LeakyRelu", "Clip", "Identity", "Add", "Sub", "Mul", "Div", "Pow", "Max", "Min", "Softmax",
    "Reshape", "Flatten", "Squeeze", "Unsqueeze", "Transpose", "Concat", "Slice", "Pad", "Resize",
    "ReduceMean", "ReduceSum", "ReduceMax", "Expand", "Shape", "Size", "Cast", "Dropout", "Gelu"};

bool is_std_domain(const std::string& d) { return d.empty() || d == "ai.onnx"; }

struct Scope {
  std::unordered_map<std::string, int> map;
  const Scope* parent = nullptr;
  int find(const std::string& n) const {
    for (const Scope* s = this; s; s = s->parent) {
      auto it = s->map.find(n);
      if (it != s->map.end()) return it->second;
    }
    return -2;
  }
};

int64_t norm_axis(int64_t a, int64_t r) {
  int64_t x = a < 0 ? a + r : a;
  SB_CHECK(x >= 0 && x < std::max<int64_t>(r, 1), SB_SHAPE_ERROR, "axis " + std::to_string(a) + " out of range");
  return x;
}

class Lowerer {
 public:
  Lowerer(const OnnxModel& m, LGraph& g) : m_(m), g_(g) {
    auto it = m.opsets.find("");
    opset_ = it != m.opsets.end() ? it->second : 21;
  }

  void run(const std::vector<InputSpec>& specs) {
    Scope root;
    std::set<std::string> init_names;
    for (auto& t : m_.graph.initializers) {
      init_names.insert(t.name);
      root.map[t.name] = g_.add_host(HostTensor::from_onnx(t), t.name);
    }
    size_t k = 0;
    for (auto& vi : m_.graph.inputs) {
      if (init_names.count(vi.name)) continue;
      SB_CHECK(k < specs.size(), SB_INVALID_ARGUMENT, "missing value for graph input '" + vi.name + "'");
      const InputSpec& s = specs[k];
      int id;
      if (s.value) {
        id = g_.add_host(*s.value, vi.name);
      } else {
        Value v;
        v.dtype = s.dtype;
        v.shape = s.shape;
        v.input_index = int(k);
        v.name = vi.name;
        // device inputs: float32, or the 16-bit float types a caller creates with CreateTensor<BFloat16 /
        // Float16> (OrtSessionFactory.cs:46-55), which reach float math through a Cast to float32
        SB_CHECK(s.dtype == DT_FLOAT || s.dtype == DT_BFLOAT16 || s.dtype == DT_FLOAT16, SB_UNSUPPORTED,
                 std::string("graph input '") + vi.name + "' of type " + dtype_name(s.dtype) +
                     " must be small enough to be a plan-time value; device inputs are float32, bfloat16 or float16");
        id = g_.add_value(std::move(v));
      }
      root.map[vi.name] = id;
      g_.inputs.push_back(id);
      ++k;
    }
    lower_nodes(m_.graph.nodes, root, 0);
    for (auto& o : m_.graph.outputs) {
      int id = root.find(o.name);
      SB_CHECK(id >= 0, SB_INVALID_ARGUMENT, "graph output '" + o.name + "' is never produced");
      g_.outputs.push_back(id);
      g_.output_names.push_back(o.name);
    }
  }

 private:
  const OnnxModel& m_;
  LGraph& g_;
  int64_t opset_ = 21;
  int64_t budget_ = 2000000;   // guards runaway Loop unrolling

  const Value& V(int id) const { return g_.vals[size_t(id)]; }

  void lower_nodes(const std::vector<OnnxNode>& nodes, Scope& sc, int depth) {
    SB_CHECK(depth < 64, SB_UNSUPPORTED, "subgraph nesting too deep");
    for (const OnnxNode& n : nodes) {
      SB_CHECK(--budget_ > 0, SB_UNSUPPORTED, "graph too large after Loop unrolling");
      std::vector<int> in;
      for (auto& name : n.inputs) {
        if (name.empty()) {
          in.push_back(-1);
        } else {
          int id = sc.find(name);
          SB_CHECK(id >= 0, SB_INVALID_ARGUMENT, "node '" + n.name + "' (" + n.op_type + ") reads undefined value '" + name + "'");
          in.push_back(id);
        }
      }
      std::vector<int> out = lower_node(n, in, sc, depth);
      SB_CHECK(out.size() >= n.outputs.size() || n.op_type == "Dropout" || n.op_type == "MaxPool", SB_INTERNAL,
               "lowering produced too few outputs for " + n.op_type);
      for (size_t i = 0; i < n.outputs.size() && i < out.size(); ++i)
        if (!n.outputs[i].empty()) {
          sc.map[n.outputs[i]] = out[i];
          if (g_.vals[size_t(out[i])].name.empty()) g_.vals[size_t(out[i])].name = n.outputs[i];
        }
    }
  }

  std::vector<int> lower_node(const OnnxNode& n, const std::vector<int>& in, Scope& sc, int depth) {
    if (!is_std_domain(n.domain)) return inline_function(n, in, sc, depth);
    if (n.op_type == "If") return lower_if(n, in, sc, depth);
    if (n.op_type == "Loop") return lower_loop(n, in, sc, depth);

    bool all_host = true;
    for (int id : in)
      if (id >= 0 && !V(id).is_host) all_host = false;
    if (all_host && host_eval_supported(n.op_type)) {
      std::vector<const HostTensor*> hin;
      for (int id : in) hin.push_back(id >= 0 ? V(id).host.get() : nullptr);
      std::vector<HostTensor> hout;
      SB_CHECK(host_eval(n, hin, hout, opset_), SB_UNSUPPORTED, "no host implementation of " + n.op_type);
      std::vector<int> ids;
      for (auto& h : hout) ids.push_back(g_.add_host(std::move(h)));
      return ids;
    }
    // Ops that read only metadata of a device value.
    if (n.op_type == "Shape" || n.op_type == "Size") {
      std::vector<HostTensor> hout;
      HostTensor shape_only;
      shape_only.dtype = DT_FLOAT;
      shape_only.shape = V(in[0]).shape;
      shape_only.buf = std::make_shared<std::vector<uint8_t>>();
      // host_eval for Shape/Size only inspects .shape
      if (n.op_type == "Size") return {g_.add_host(HostTensor::scalar_i64(numel(V(in[0]).shape)))};
      std::vector<const HostTensor*> hin{&shape_only};
      host_eval(n, hin, hout, opset_);
      return {g_.add_host(std::move(hout[0]))};
    }
    SB_CHECK(kDeviceOps.count(n.op_type), SB_UNSUPPORTED,
             "operator '" + n.op_type + "' (node '" + n.name + "') has no B200 device implementation");
    return device_op(n, in);
  }

  // ------------------------------------------------------------------------------------------
  std::vector<int> inline_function(const OnnxNode& n, const std::vector<int>& in, Scope& sc, int depth) {
    const OnnxFunction* fn = nullptr;
    for (auto& f : m_.functions)
      if (f.name == n.op_type && f.domain == n.domain) fn = &f;
    SB_CHECK(fn != nullptr, SB_UNSUPPORTED, "unknown function " + n.domain + "." + n.op_type);
    for (auto& fnode : fn->nodes)
      for (auto& a : fnode.attrs)
        SB_CHECK(a.ref_attr_name.empty(), SB_UNSUPPORTED, "function attribute references are not supported");
    Scope child;
    child.parent = nullptr;   // functions see only their formal inputs
    for (size_t i = 0; i < fn->inputs.size(); ++i) child.map[fn->inputs[i]] = i < in.size() ? in[i] : -1;
    lower_nodes(fn->nodes, child, depth + 1);
    std::vector<int> out;
    for (auto& o : fn->outputs) {
      int id = child.find(o);
      SB_CHECK(id >= 0, SB_INVALID_ARGUMENT, "function output '" + o + "' not produced");
      out.push_back(id);
    }
    return out;
  }

  std::vector<int> run_subgraph(const OnnxGraph& g, Scope& parent, const std::vector<int>& bound, int depth) {
    Scope child;
    child.parent = &parent;
    for (auto& t : g.initializers) child.map[t.name] = g_.add_host(HostTensor::from_onnx(t), t.name);
    for (size_t i = 0; i < g.inputs.size() && i < bound.size(); ++i) child.map[g.inputs[i].name] = bound[i];
    lower_nodes(g.nodes, child, depth + 1);
    std::vector<int> out;
    for (auto& o : g.outputs) {
      int id = child.find(o.name);
      SB_CHECK(id >= 0, SB_INVALID_ARGUMENT, "subgraph output '" + o.name + "' not produced");
      out.push_back(id);
    }
    return out;
  }

  bool host_bool(int id, const char* what) {
    SB_CHECK(id >= 0 && V(id).is_host, SB_UNSUPPORTED,
             std::string(what) + " depends on tensor data; only conditions computable at plan time "
                                 "(constants, shapes, scalar inputs) are supported");
    SB_CHECK(V(id).host->numel() >= 1, SB_INVALID_ARGUMENT, std::string(what) + " is empty");
    return V(id).host->get_f64(0) != 0.0;
  }

  std::vector<int> lower_if(const OnnxNode& n, const std::vector<int>& in, Scope& sc, int depth) {
    bool c = host_bool(in.at(0), "If condition");
    const OnnxAttr* br = n.attr(c ? "then_branch" : "else_branch");
    SB_CHECK(br && br->g, SB_INVALID_ARGUMENT, "If without branch graph");
    return run_subgraph(*br->g, sc, {}, depth);
  }

  std::vector<int> lower_loop(const OnnxNode& n, const std::vector<int>& in, Scope& sc, int depth) {
    const OnnxAttr* b = n.attr("body");
    SB_CHECK(b && b->g, SB_INVALID_ARGUMENT, "Loop without body");
    const OnnxGraph& body = *b->g;
    int64_t trip = INT64_MAX;
    if (in.size() > 0 && in[0] >= 0) {
      SB_CHECK(V(in[0]).is_host, SB_UNSUPPORTED, "Loop trip count depends on tensor data");
      trip = V(in[0]).host->get_i64(0);
    }
    bool keep = true;
    if (in.size() > 1 && in[1] >= 0) keep = host_bool(in[1], "Loop condition");
    std::vector<int> carried(in.begin() + std::min<size_t>(2, in.size()), in.end());
    size_t nc = carried.size();
    size_t nscan = body.outputs.size() - 1 - nc;
    std::vector<std::vector<int>> scans(nscan);
    int64_t i = 0;
    while (i < trip && keep) {
      SB_CHECK(i < 100000, SB_UNSUPPORTED, "Loop with more than 100000 iterations");
      std::vector<int> bound{g_.add_host(HostTensor::scalar_i64(i))};
      HostTensor cb(DT_BOOL, {});
      cb.set_i64(0, 1);
      bound.push_back(g_.add_host(cb));
      bound.insert(bound.end(), carried.begin(), carried.end());
      auto outs = run_subgraph(body, sc, bound, depth);
      keep = host_bool(outs[0], "Loop continue condition");
      for (size_t j = 0; j < nc; ++j) carried[j] = outs[1 + j];
      for (size_t j = 0; j < nscan; ++j) scans[j].push_back(outs[1 + nc + j]);
      ++i;
    }
    std::vector<int> out = carried;
    for (auto& s : scans) {
      // Scan outputs: stack along a new leading axis (host values only).
      for (int id : s) SB_CHECK(V(id).is_host, SB_UNSUPPORTED, "Loop scan outputs of device tensors are not supported");
      if (s.empty()) {
        out.push_back(g_.add_host(HostTensor(DT_FLOAT, {0})));
        continue;
      }
      const HostTensor& f = *V(s[0]).host;
      std::vector<int64_t> shp = f.shape;
      shp.insert(shp.begin(), int64_t(s.size()));
      HostTensor st(f.dtype, shp);
      size_t bytes = f.nbytes();
      for (size_t k = 0; k < s.size(); ++k) std::memcpy(st.mutable_data() + k * bytes, V(s[k]).host->data(), bytes);
      out.push_back(g_.add_host(std::move(st)));
    }
    return out;
  }

  // ------------------------------------------------------------------------------------------
  int new_dev(const std::vector<int64_t>& shape, int producer) {
    Value v;
    v.dtype = DT_FLOAT;
    v.shape = shape;
    v.producer = producer;
    return g_.add_value(std::move(v));
  }

  const HostTensor& need_host(int id, const std::string& what) {
    SB_CHECK(id >= 0 && V(id).is_host, SB_UNSUPPORTED, what + " must be known at plan time");
    return *V(id).host;
  }

  static std::vector<int64_t> resolve_pads(const OnnxNode& n, const std::vector<int64_t>& in_sp,
                                           const std::vector<int64_t>& k, const std::vector<int64_t>& s,
                                           const std::vector<int64_t>& d) {
    // explicit pads vs SAME_UPPER / SAME_LOWER / VALID (src/Shorokoo/Core/Inference/Ops/Conv.cs:34-61)
    size_t nd = in_sp.size();
    std::string ap = n.attr_s("auto_pad", "NOTSET");
    std::vector<int64_t> pads(2 * nd, 0);
    if (ap == "SAME_UPPER" || ap == "SAME_LOWER") {
      for (size_t i = 0; i < nd; ++i) {
        int64_t out = ceil_div(in_sp[i], s[i]);
        int64_t total = std::max<int64_t>((out - 1) * s[i] + (k[i] - 1) * d[i] + 1 - in_sp[i], 0);
        int64_t small = total / 2, big = total - small;
        pads[i] = ap == "SAME_UPPER" ? small : big;
        pads[i + nd] = ap == "SAME_UPPER" ? big : small;
      }
    } else if (ap == "VALID") {
      // zeros
    } else {
      auto p = n.attr_ints("pads");
      if (!p.empty()) {
        SB_CHECK(p.size() == 2 * nd, SB_INVALID_ARGUMENT, n.op_type + ": pads has wrong length");
        pads = p;
      }
    }
    return pads;
  }

  std::vector<int> device_op(const OnnxNode& n, const std::vector<int>& in) {
    const std::string& t = n.op_type;
    Op op;
    op.type = t;
    op.in = in;
    op.name = n.name;
    int opi = int(g_.ops.size());
    auto X = [&](size_t i) -> const Value& {
      SB_CHECK(i < in.size() && in[i] >= 0, SB_INVALID_ARGUMENT, t + ": missing input " + std::to_string(i));
      return V(in[i]);
    };
    for (int id : in)
      if (id >= 0 && !V(id).is_host)
        SB_CHECK(V(id).dtype == DT_FLOAT || (t == "Cast" && (V(id).dtype == DT_BFLOAT16 || V(id).dtype == DT_FLOAT16)),
                 SB_UNSUPPORTED, t + ": device tensors of type " + dtype_name(V(id).dtype) + " are not supported");
    std::vector<std::vector<int64_t>> oshapes;

    if (t == "Conv") {
      const Value& x = X(0);
      SB_CHECK(x.shape.size() == 4, SB_UNSUPPORTED, "Conv: only 2-D convolution (rank-4 input) is supported");
      const HostTensor& w = need_host(in.at(1), "Conv weight");
      SB_CHECK(w.shape.size() == 4, SB_SHAPE_ERROR, "Conv: weight must be rank 4");
      op.group = n.attr_i("group", 1);
      op.kernel = n.attr_ints("kernel_shape");
      if (op.kernel.empty()) op.kernel = {w.shape[2], w.shape[3]};
      op.strides = n.attr_ints("strides");
      if (op.strides.empty()) op.strides = {1, 1};
      op.dilations = n.attr_ints("dilations");
      if (op.dilations.empty()) op.dilations = {1, 1};
      SB_CHECK(w.shape[1] * op.group == x.shape[1], SB_SHAPE_ERROR,
               "Conv: input channels " + std::to_string(x.shape[1]) + " do not match weight " + shape_str(w.shape));
      SB_CHECK(op.kernel[0] == w.shape[2] && op.kernel[1] == w.shape[3], SB_SHAPE_ERROR, "Conv: kernel_shape mismatch");
      op.pads = resolve_pads(n, {x.shape[2], x.shape[3]}, op.kernel, op.strides, op.dilations);
      if (in.size() > 2 && in[2] >= 0) need_host(in[2], "Conv bias");
      int64_t ho = (x.shape[2] + op.pads[0] + op.pads[2] - ((op.kernel[0] - 1) * op.dilations[0] + 1)) / op.strides[0] + 1;
      int64_t wo = (x.shape[3] + op.pads[1] + op.pads[3] - ((op.kernel[1] - 1) * op.dilations[1] + 1)) / op.strides[1] + 1;
      SB_CHECK(ho > 0 && wo > 0, SB_SHAPE_ERROR, "Conv: empty output");
      oshapes.push_back({x.shape[0], w.shape[0], ho, wo});
    } else if (t == "MaxPool" || t == "AveragePool") {
      const Value& x = X(0);
      SB_CHECK(x.shape.size() == 4, SB_UNSUPPORTED, t + ": only 2-D pooling is supported");
      SB_CHECK(n.outputs.size() < 2 || n.outputs[1].empty(), SB_UNSUPPORTED, "MaxPool: Indices output is not supported");
      op.kernel = n.attr_ints("kernel_shape");
      op.strides = n.attr_ints("strides");
      if (op.strides.empty()) op.strides = {1, 1};
      op.dilations = n.attr_ints("dilations");
      if (op.dilations.empty()) op.dilations = {1, 1};
      op.ceil_mode = n.attr_i("ceil_mode", 0);
      op.keepdims = n.attr_i("count_include_pad", 0);
      op.pads = resolve_pads(n, {x.shape[2], x.shape[3]}, op.kernel, op.strides, op.dilations);
      std::vector<int64_t> os = {x.shape[0], x.shape[1]};
      for (int i = 0; i < 2; ++i) {
        int64_t eff = (op.kernel[size_t(i)] - 1) * op.dilations[size_t(i)] + 1;
        int64_t num = x.shape[size_t(2 + i)] + op.pads[size_t(i)] + op.pads[size_t(i + 2)] - eff;
        int64_t o = (op.ceil_mode ? ceil_div(num, op.strides[size_t(i)]) : num / op.strides[size_t(i)]) + 1;
        if (op.ceil_mode && (o - 1) * op.strides[size_t(i)] >= x.shape[size_t(2 + i)] + op.pads[size_t(i)]) --o;
        SB_CHECK(o > 0, SB_SHAPE_ERROR, t + ": empty output");
        os.push_back(o);
      }
      oshapes.push_back(os);
    } else if (t == "GlobalAveragePool" || t == "GlobalMaxPool") {
      const Value& x = X(0);
      SB_CHECK(x.shape.size() >= 3, SB_SHAPE_ERROR, t + ": rank < 3");
      std::vector<int64_t> os = {x.shape[0], x.shape[1]};
      for (size_t i = 2; i < x.shape.size(); ++i) os.push_back(1);
      oshapes.push_back(os);
    } else if (t == "MatMul") {
      const Value& a = X(0);
      const Value& b = X(1);
      SB_CHECK(a.shape.size() >= 2 && b.shape.size() >= 2, SB_UNSUPPORTED,
               "MatMul: supported forms are [...,M,K] x [...,K,N]");
      const size_t ra = a.shape.size(), rb = b.shape.size();
      SB_CHECK(a.shape[ra - 1] == b.shape[rb - 2], SB_SHAPE_ERROR,
               "MatMul: inner dimensions differ " + shape_str(a.shape) + " x " + shape_str(b.shape));
      // batch dimensions broadcast (a device x device product runs only inside a fused attention)
      std::vector<int64_t> os = broadcast_shapes(std::vector<int64_t>(a.shape.begin(), a.shape.end() - 2),
                                                 std::vector<int64_t>(b.shape.begin(), b.shape.end() - 2));
      os.push_back(a.shape[ra - 2]);
      os.push_back(b.shape[rb - 1]);
      oshapes.push_back(os);
    } else if (t == "Gemm") {
      const Value& a = X(0);
      const Value& b = X(1);
      SB_CHECK(a.shape.size() == 2 && b.shape.size() == 2, SB_SHAPE_ERROR, "Gemm: rank-2 operands required");
      op.axes = {n.attr_i("transA", 0), n.attr_i("transB", 0)};
      op.alpha = n.attr_f("alpha", 1.f);
      op.beta = n.attr_f("beta", 1.f);
      int64_t M = op.axes[0] ? a.shape[1] : a.shape[0];
      int64_t K = op.axes[0] ? a.shape[0] : a.shape[1];
      int64_t K2 = op.axes[1] ? b.shape[1] : b.shape[0];
      int64_t N = op.axes[1] ? b.shape[0] : b.shape[1];
      SB_CHECK(K == K2, SB_SHAPE_ERROR, "Gemm: inner dimensions differ");
      if (in.size() > 2 && in[2] >= 0) broadcast_shapes(V(in[2]).shape, {M, N});
      oshapes.push_back({M, N});
    } else if (t == "Relu" || t == "Sigmoid" || t == "Tanh" || t == "Sqrt" || t == "Neg" || t == "Abs" ||
               t == "Exp" || t == "Log" || t == "Reciprocal" || t == "Floor" || t == "Ceil" || t == "Erf" ||
               t == "Identity" || t == "Dropout") {
      if (t == "Dropout") op.type = "Identity";
      oshapes.push_back(X(0).shape);
    } else if (t == "Gelu") {   // approximate: "none" (erf) or "tanh"
      op.mode = n.attr_s("approximate", "none");
      SB_CHECK(op.mode == "none" || op.mode == "tanh", SB_UNSUPPORTED, "Gelu: approximate=" + op.mode);
      oshapes.push_back(X(0).shape);
    } else if (t == "LeakyRelu") {
      op.alpha = n.attr_f("alpha", 0.01f);
      oshapes.push_back(X(0).shape);
    } else if (t == "Clip") {
      op.fmin = -INFINITY;
      op.fmax = INFINITY;
      if (in.size() > 1 && in[1] >= 0) op.fmin = float(need_host(in[1], "Clip min").get_f64(0));
      if (in.size() > 2 && in[2] >= 0) op.fmax = float(need_host(in[2], "Clip max").get_f64(0));
      op.in.resize(1);
      oshapes.push_back(X(0).shape);
    } else if (t == "Cast") {
      int64_t to = n.attr_i("to", DT_FLOAT);
      SB_CHECK(to == DT_FLOAT, SB_UNSUPPORTED, "Cast of a device tensor to a non-float32 type is not supported");
      op.type = "Identity";
      oshapes.push_back(X(0).shape);
    } else if (t == "Add" || t == "Sub" || t == "Mul" || t == "Div" || t == "Pow" || t == "Max" || t == "Min") {
      SB_CHECK(in.size() == 2, SB_UNSUPPORTED, t + " with more than two inputs is not supported on device");
      for (int id : in) SB_CHECK(V(id).is_host ? V(id).host->is_float() : true, SB_UNSUPPORTED, t + ": mixed int/float operands");
      oshapes.push_back(broadcast_shapes(X(0).shape, X(1).shape));
    } else if (t == "Softmax") {
      op.axis = norm_axis(n.attr_i("axis", -1), int64_t(X(0).shape.size()));
      oshapes.push_back(X(0).shape);
    } else if (t == "Reshape") {
      const Value& x = X(0);
      auto shp = need_host(in.at(1), "Reshape shape").to_i64_vec();
      bool allowzero = n.attr_i("allowzero", 0) != 0;
      int64_t known = 1, neg = -1;
      for (size_t i = 0; i < shp.size(); ++i) {
        if (shp[i] == 0 && !allowzero) {
          SB_CHECK(i < x.shape.size(), SB_SHAPE_ERROR, "Reshape: 0 refers past input rank");
          shp[i] = x.shape[i];
        }
        if (shp[i] == -1) {
          SB_CHECK(neg < 0, SB_SHAPE_ERROR, "Reshape: more than one -1");
          neg = int64_t(i);
        } else {
          known *= shp[i];
        }
      }
      if (neg >= 0) {
        SB_CHECK(known > 0 && numel(x.shape) % known == 0, SB_SHAPE_ERROR, "Reshape: cannot infer -1");
        shp[size_t(neg)] = numel(x.shape) / known;
      }
      SB_CHECK(numel(shp) == numel(x.shape), SB_SHAPE_ERROR,
               "Reshape: cannot reshape " + shape_str(x.shape) + " to " + shape_str(shp));
      op.in = {in[0]};
      oshapes.push_back(shp);
    } else if (t == "Flatten") {
      const Value& x = X(0);
      int64_t r = int64_t(x.shape.size());
      int64_t a = n.attr_i("axis", 1);
      if (a < 0) a += r;
      int64_t o = 1;
      for (int64_t i = 0; i < a; ++i) o *= x.shape[size_t(i)];
      op.type = "Reshape";
      oshapes.push_back({o, numel(x.shape) / std::max<int64_t>(o, 1)});
    } else if (t == "Squeeze" || t == "Unsqueeze") {
      const Value& x = X(0);
      std::vector<int64_t> axes = (in.size() > 1 && in[1] >= 0) ? need_host(in[1], t + " axes").to_i64_vec()
                                                                 : n.attr_ints("axes");
      std::vector<int64_t> s = x.shape;
      if (t == "Unsqueeze") {
        int64_t r = int64_t(s.size() + axes.size());
        std::vector<int64_t> na;
        for (auto a : axes) na.push_back(norm_axis(a, r));
        std::sort(na.begin(), na.end());
        for (auto a : na) s.insert(s.begin() + a, 1);
      } else {
        int64_t r = int64_t(s.size());
        std::vector<bool> drop(size_t(r), false);
        if (axes.empty()) {
          for (int64_t i = 0; i < r; ++i) drop[size_t(i)] = s[size_t(i)] == 1;
        } else {
          for (auto a : axes) drop[size_t(norm_axis(a, r))] = true;
        }
        std::vector<int64_t> ns;
        for (int64_t i = 0; i < r; ++i) {
          if (drop[size_t(i)]) SB_CHECK(s[size_t(i)] == 1, SB_SHAPE_ERROR, "Squeeze: dim is not 1");
          else ns.push_back(s[size_t(i)]);
        }
        s = ns;
      }
      op.type = "Reshape";
      op.in = {in[0]};
      oshapes.push_back(s);
    } else if (t == "Transpose") {
      const Value& x = X(0);
      int64_t r = int64_t(x.shape.size());
      op.perm = n.attr_ints("perm");
      if (op.perm.empty())
        for (int64_t i = r - 1; i >= 0; --i) op.perm.push_back(i);
      SB_CHECK(int64_t(op.perm.size()) == r, SB_SHAPE_ERROR, "Transpose: perm length != rank");
      std::vector<int64_t> s;
      for (auto p : op.perm) s.push_back(x.shape[size_t(norm_axis(p, r))]);
      oshapes.push_back(s);
    } else if (t == "Concat") {
      int64_t r = int64_t(X(0).shape.size());
      op.axis = norm_axis(n.attr_i("axis", 0), r);
      std::vector<int64_t> s = X(0).shape;
      s[size_t(op.axis)] = 0;
      for (int id : in) {
        SB_CHECK(id >= 0, SB_INVALID_ARGUMENT, "Concat: missing input");
        const Value& v = V(id);
        SB_CHECK(int64_t(v.shape.size()) == r, SB_SHAPE_ERROR, "Concat: rank mismatch");
        for (int64_t d = 0; d < r; ++d)
          if (d != op.axis) SB_CHECK(v.shape[size_t(d)] == s[size_t(d)], SB_SHAPE_ERROR, "Concat: shape mismatch");
        s[size_t(op.axis)] += v.shape[size_t(op.axis)];
      }
      oshapes.push_back(s);
    } else if (t == "Slice") {
      const Value& x = X(0);
      int64_t r = int64_t(x.shape.size());
      auto starts = need_host(in.at(1), "Slice starts").to_i64_vec();
      auto ends = need_host(in.at(2), "Slice ends").to_i64_vec();
      std::vector<int64_t> axes, steps;
      if (in.size() > 3 && in[3] >= 0) axes = need_host(in[3], "Slice axes").to_i64_vec();
      else for (size_t i = 0; i < starts.size(); ++i) axes.push_back(int64_t(i));
      if (in.size() > 4 && in[4] >= 0) steps = need_host(in[4], "Slice steps").to_i64_vec();
      else steps.assign(starts.size(), 1);
      op.axes.assign(size_t(r), 0);    // per-dim start
      op.strides.assign(size_t(r), 1); // per-dim step
      std::vector<int64_t> s = x.shape;
      for (size_t i = 0; i < starts.size(); ++i) {
        int64_t a = norm_axis(axes[i], r);
        int64_t d = x.shape[size_t(a)];
        int64_t st = starts[i], en = ends[i], sp = steps[i];
        SB_CHECK(sp != 0, SB_INVALID_ARGUMENT, "Slice: zero step");
        if (st < 0) st += d;
        if (en < 0) en += d;
        if (sp > 0) {
          st = std::clamp<int64_t>(st, 0, d);
          en = std::clamp<int64_t>(en, 0, d);
          s[size_t(a)] = std::max<int64_t>(0, ceil_div(en - st, sp));
        } else {
          st = std::clamp<int64_t>(st, -1, d - 1);
          en = std::clamp<int64_t>(en, -1, d - 1);
          s[size_t(a)] = std::max<int64_t>(0, ceil_div(st - en, -sp));
        }
        op.axes[size_t(a)] = st;
        op.strides[size_t(a)] = sp;
      }
      op.in = {in[0]};
      oshapes.push_back(s);
    } else if (t == "Pad") {
      const Value& x = X(0);
      std::string mode = n.attr_s("mode", "constant");
      SB_CHECK(mode == "constant", SB_UNSUPPORTED, "Pad: only constant mode is supported on device");
      auto pads = need_host(in.at(1), "Pad pads").to_i64_vec();
      int64_t r = int64_t(x.shape.size());
      std::vector<int64_t> axes;
      if (in.size() > 3 && in[3] >= 0) axes = need_host(in[3], "Pad axes").to_i64_vec();
      else for (int64_t i = 0; i < r; ++i) axes.push_back(i);
      SB_CHECK(pads.size() == 2 * axes.size(), SB_INVALID_ARGUMENT, "Pad: pads length mismatch");
      op.pads.assign(size_t(2 * r), 0);
      for (size_t j = 0; j < axes.size(); ++j) {
        int64_t a = norm_axis(axes[j], r);
        op.pads[size_t(a)] = pads[j];
        op.pads[size_t(a + r)] = pads[j + axes.size()];
      }
      for (auto p : op.pads) SB_CHECK(p >= 0, SB_UNSUPPORTED, "Pad: negative pads are not supported");
      op.alpha = 0.f;
      if (in.size() > 2 && in[2] >= 0 && V(in[2]).is_host && V(in[2]).host->numel() > 0)
        op.alpha = float(V(in[2]).host->get_f64(0));
      std::vector<int64_t> s = x.shape;
      for (int64_t i = 0; i < r; ++i) s[size_t(i)] += op.pads[size_t(i)] + op.pads[size_t(i + r)];
      op.in = {in[0]};
      oshapes.push_back(s);
    } else if (t == "Resize") {
      const Value& x = X(0);
      op.mode = n.attr_s("mode", "nearest");
      SB_CHECK(op.mode == "nearest", SB_UNSUPPORTED, "Resize: only mode=nearest is supported");
      op.coord_mode = n.attr_s("coordinate_transformation_mode", "half_pixel");
      op.nearest_mode = n.attr_s("nearest_mode", "round_prefer_floor");
      SB_CHECK(n.attr_ints("axes").empty(), SB_UNSUPPORTED, "Resize: axes attribute not supported");
      std::vector<int64_t> s = x.shape;
      bool have_scales = in.size() > 2 && in[2] >= 0 && V(in[2]).is_host && V(in[2]).host->numel() > 0;
      bool have_sizes = in.size() > 3 && in[3] >= 0 && V(in[3]).is_host && V(in[3]).host->numel() > 0;
      if (have_sizes) {
        auto sz = V(in[3]).host->to_i64_vec();
        SB_CHECK(sz.size() == s.size(), SB_SHAPE_ERROR, "Resize: sizes length mismatch");
        for (size_t i = 0; i < s.size(); ++i) op.scales.push_back(float(double(sz[i]) / double(s[i])));
        s = sz;
      } else {
        SB_CHECK(have_scales, SB_UNSUPPORTED, "Resize: scales or sizes must be known at plan time");
        auto sc = V(in[2]).host->to_f64_vec();
        SB_CHECK(sc.size() == s.size(), SB_SHAPE_ERROR, "Resize: scales length mismatch");
        for (size_t i = 0; i < s.size(); ++i) {
          op.scales.push_back(float(sc[i]));
          s[i] = int64_t(std::floor(double(s[i]) * double(float(sc[i]))));
        }
      }
      op.in = {in[0]};
      oshapes.push_back(s);
    } else if (t == "ReduceMean" || t == "ReduceSum" || t == "ReduceMax") {
      const Value& x = X(0);
      int64_t r = int64_t(x.shape.size());
      std::vector<int64_t> axes = (in.size() > 1 && in[1] >= 0) ? need_host(in[1], t + " axes").to_i64_vec()
                                                                 : n.attr_ints("axes");
      op.keepdims = n.attr_i("keepdims", 1);
      if (axes.empty()) {
        SB_CHECK(!n.attr_i("noop_with_empty_axes", 0), SB_UNSUPPORTED, t + ": noop_with_empty_axes");
        for (int64_t i = 0; i < r; ++i) axes.push_back(i);
      }
      for (auto& a : axes) a = norm_axis(a, r);
      std::sort(axes.begin(), axes.end());
      op.axes = axes;
      std::vector<int64_t> s;
      for (int64_t i = 0; i < r; ++i) {
        bool red = std::find(axes.begin(), axes.end(), i) != axes.end();
        if (!red) s.push_back(x.shape[size_t(i)]);
        else if (op.keepdims) s.push_back(1);
      }
      op.in = {in[0]};
      oshapes.push_back(s);
    } else if (t == "Expand") {
      auto shp = need_host(in.at(1), "Expand shape").to_i64_vec();
      op.in = {in[0]};
      oshapes.push_back(broadcast_shapes(X(0).shape, shp));
    } else {
      fail(SB_UNSUPPORTED, "operator '" + t + "' has no B200 device implementation");
    }
    for (auto& s : oshapes) op.out.push_back(new_dev(s, opi));
    g_.ops.push_back(std::move(op));
    return g_.ops.back().out;
  }
};

}  // namespace

std::vector<int> LGraph::use_counts() const {
  std::vector<int> c(vals.size(), 0);
  for (auto& op : ops) {
    if (op.dead) continue;
    for (int id : op.in)
      if (id >= 0) c[size_t(id)]++;
    if (op.residual >= 0) c[size_t(op.residual)]++;
    if (op.concat >= 0) c[size_t(op.concat)]++;
  }
  for (int id : outputs) c[size_t(id)]++;
  return c;
}

void LGraph::dce() {
  std::vector<bool> live(vals.size(), false);
  for (int id : outputs) live[size_t(id)] = true;
  for (int i = int(ops.size()) - 1; i >= 0; --i) {
    Op& op = ops[size_t(i)];
    if (op.dead) continue;
    bool any = false;
    for (int o : op.out)
      if (live[size_t(o)]) any = true;
    if (!any) {
      op.dead = true;
      continue;
    }
    for (int id : op.in)
      if (id >= 0) live[size_t(id)] = true;
    if (op.residual >= 0) live[size_t(op.residual)] = true;
    if (op.concat >= 0) live[size_t(op.concat)] = true;
  }
}

ModelInfo model_info(const OnnxModel& m) {
  ModelInfo info;
  std::set<std::string> inits;
  for (auto& t : m.graph.initializers) inits.insert(t.name);
  for (auto& vi : m.graph.inputs) {
    if (inits.count(vi.name)) continue;
    info.input_names.push_back(vi.name);
    info.input_dtypes.push_back(vi.elem_type ? vi.elem_type : DT_FLOAT);
    info.input_ranks.push_back(vi.has_shape ? int(vi.dims.size()) : -1);
  }
  for (auto& o : m.graph.outputs) info.output_names.push_back(o.name);
  return info;
}

namespace {
void check_nodes(const std::vector<OnnxNode>& nodes, const OnnxModel& m, int depth) {
  for (auto& n : nodes) {
    if (!is_std_domain(n.domain)) {
      bool found = false;
      for (auto& f : m.functions)
        if (f.name == n.op_type && f.domain == n.domain) {
          found = true;
          if (depth < 16) check_nodes(f.nodes, m, depth + 1);
        }
      SB_CHECK(found, SB_UNSUPPORTED, "unknown operator " + n.domain + "." + n.op_type + " (node '" + n.name + "')");
      continue;
    }
    if (n.op_type == "If" || n.op_type == "Loop") {
      for (auto& a : n.attrs)
        if (a.g) check_nodes(a.g->nodes, m, depth + 1);
      continue;
    }
    SB_CHECK(host_eval_supported(n.op_type) || kDeviceOps.count(n.op_type), SB_UNSUPPORTED,
             "operator '" + n.op_type + "' (node '" + n.name + "') is not supported by the B200 backend");
  }
}
}  // namespace

void check_supported_ops(const OnnxModel& m) { check_nodes(m.graph.nodes, m, 0); }

LGraph lower(const OnnxModel& m, const std::vector<InputSpec>& inputs) {
  LGraph g;
  Lowerer L(m, g);
  L.run(inputs);
  g.dce();
  return g;
}

}  // namespace sb
