// Host evaluator for plan-time folding. Elementwise arithmetic on floats is done in double and
// rounded once to the output type, which equals the IEEE single-precision result for each of
// + - * / sqrt (double carries more than 2*24+2 significand bits).
#include "host_tensor.h"

#include <algorithm>
#include <cmath>
#include <numeric>

namespace sb {

// ---------------------------------------------------------------------------------------------
// half / bfloat16 helpers (bit-level, from the IEEE-754 binary16 / bfloat16 layouts)
// ---------------------------------------------------------------------------------------------
uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);   // quiet NaN
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return uint16_t(u >> 16);
}

float bf16_to_f32(uint16_t h) {
  uint32_t u = uint32_t(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

float f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h >> 15) << 31;
  int exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else {   // subnormal: value = man * 2^-24
      float f = std::ldexp(float(man), -24);
      std::memcpy(&u, &f, 4);
      u |= sign;
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (man << 13);
  } else {
    u = sign | (uint32_t(exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

uint16_t f32_to_f16(float f) {
  // Round-to-nearest-even via double arithmetic on the exact value.
  if (std::isnan(f)) return 0x7e00;
  uint16_t sign = std::signbit(f) ? 0x8000 : 0;
  double a = std::fabs(double(f));
  if (a >= 65520.0) return sign | 0x7c00;
  if (a < std::ldexp(1.0, -14)) {   // subnormal range: quantum 2^-24
    double q = std::nearbyint(a * std::ldexp(1.0, 24));
    return sign | uint16_t(q);
  }
  int e;
  double m = std::frexp(a, &e);          // a = m * 2^e, m in [0.5, 1)
  double q = std::nearbyint(m * 2048.0);  // 11 significant bits
  if (q >= 2048.0) { q /= 2; e += 1; }
  int exp = e - 1 + 15;
  uint16_t man = uint16_t(int64_t(q) - 1024);
  return sign | uint16_t(exp << 10) | man;
}

// ---------------------------------------------------------------------------------------------
HostTensor::HostTensor(int32_t dt, std::vector<int64_t> s) : dtype(dt), shape(std::move(s)) {
  buf = std::make_shared<std::vector<uint8_t>>(nbytes());
}

const uint8_t* HostTensor::data() const {
  if (!buf && transpose_src) {
    auto* self = const_cast<HostTensor*>(this);
    const HostTensor& src = *transpose_src;
    size_t es = dtype_size(dtype);
    int64_t r = src.shape[0], c = src.shape[1];
    self->buf = std::make_shared<std::vector<uint8_t>>(size_t(r * c) * es);
    const uint8_t* s = src.data();
    uint8_t* d = self->buf->data();
    const int64_t B = 64;
    for (int64_t i0 = 0; i0 < r; i0 += B)
      for (int64_t j0 = 0; j0 < c; j0 += B)
        for (int64_t i = i0; i < std::min(r, i0 + B); ++i)
          for (int64_t j = j0; j < std::min(c, j0 + B); ++j)
            std::memcpy(d + (j * r + i) * es, s + (i * c + j) * es, es);
    self->transpose_src.reset();
  }
  static const uint8_t empty = 0;
  return buf ? buf->data() : &empty;
}

uint8_t* HostTensor::mutable_data() {
  data();
  if (buf.use_count() > 1) buf = std::make_shared<std::vector<uint8_t>>(*buf);   // copy on write
  return buf->data();
}

double HostTensor::get_f64(int64_t i) const {
  const uint8_t* p = data();
  switch (dtype) {
    case DT_FLOAT: return double(reinterpret_cast<const float*>(p)[i]);
    case DT_DOUBLE: return reinterpret_cast<const double*>(p)[i];
    case DT_INT64: return double(reinterpret_cast<const int64_t*>(p)[i]);
    case DT_INT32: return double(reinterpret_cast<const int32_t*>(p)[i]);
    case DT_INT16: return double(reinterpret_cast<const int16_t*>(p)[i]);
    case DT_INT8: return double(reinterpret_cast<const int8_t*>(p)[i]);
    case DT_UINT8: case DT_BOOL: return double(p[i]);
    case DT_UINT16: return double(reinterpret_cast<const uint16_t*>(p)[i]);
    case DT_UINT32: return double(reinterpret_cast<const uint32_t*>(p)[i]);
    case DT_UINT64: return double(reinterpret_cast<const uint64_t*>(p)[i]);
    case DT_FLOAT16: return double(f16_to_f32(reinterpret_cast<const uint16_t*>(p)[i]));
    case DT_BFLOAT16: return double(bf16_to_f32(reinterpret_cast<const uint16_t*>(p)[i]));
    default: fail(SB_UNSUPPORTED, std::string("host: dtype ") + dtype_name(dtype));
  }
}

int64_t HostTensor::get_i64(int64_t i) const {
  const uint8_t* p = data();
  switch (dtype) {
    case DT_INT64: return reinterpret_cast<const int64_t*>(p)[i];
    case DT_INT32: return reinterpret_cast<const int32_t*>(p)[i];
    case DT_INT16: return reinterpret_cast<const int16_t*>(p)[i];
    case DT_INT8: return reinterpret_cast<const int8_t*>(p)[i];
    case DT_UINT8: case DT_BOOL: return p[i];
    case DT_UINT16: return reinterpret_cast<const uint16_t*>(p)[i];
    case DT_UINT32: return reinterpret_cast<const uint32_t*>(p)[i];
    case DT_UINT64: return int64_t(reinterpret_cast<const uint64_t*>(p)[i]);
    default: return int64_t(get_f64(i));
  }
}

void HostTensor::set_f64(int64_t i, double v) {
  uint8_t* p = mutable_data();
  switch (dtype) {
    case DT_FLOAT: reinterpret_cast<float*>(p)[i] = float(v); break;
    case DT_DOUBLE: reinterpret_cast<double*>(p)[i] = v; break;
    case DT_FLOAT16: reinterpret_cast<uint16_t*>(p)[i] = f32_to_f16(float(v)); break;
    case DT_BFLOAT16: reinterpret_cast<uint16_t*>(p)[i] = f32_to_bf16_rne(float(v)); break;
    case DT_BOOL: p[i] = v != 0.0; break;
    default: set_i64(i, int64_t(v));
  }
}

void HostTensor::set_i64(int64_t i, int64_t v) {
  uint8_t* p = mutable_data();
  switch (dtype) {
    case DT_INT64: reinterpret_cast<int64_t*>(p)[i] = v; break;
    case DT_INT32: reinterpret_cast<int32_t*>(p)[i] = int32_t(v); break;
    case DT_INT16: reinterpret_cast<int16_t*>(p)[i] = int16_t(v); break;
    case DT_INT8: reinterpret_cast<int8_t*>(p)[i] = int8_t(v); break;
    case DT_UINT8: p[i] = uint8_t(v); break;
    case DT_BOOL: p[i] = v != 0; break;
    case DT_UINT16: reinterpret_cast<uint16_t*>(p)[i] = uint16_t(v); break;
    case DT_UINT32: reinterpret_cast<uint32_t*>(p)[i] = uint32_t(v); break;
    case DT_UINT64: reinterpret_cast<uint64_t*>(p)[i] = uint64_t(v); break;
    default: set_f64(i, double(v));
  }
}

std::vector<int64_t> HostTensor::to_i64_vec() const {
  std::vector<int64_t> v(static_cast<size_t>(numel()));
  for (int64_t i = 0; i < numel(); ++i) v[size_t(i)] = get_i64(i);
  return v;
}

std::vector<double> HostTensor::to_f64_vec() const {
  std::vector<double> v(static_cast<size_t>(numel()));
  for (int64_t i = 0; i < numel(); ++i) v[size_t(i)] = get_f64(i);
  return v;
}

HostTensor HostTensor::from_onnx(const OnnxTensor& t) {
  SB_CHECK(t.data_type != DT_STRING, SB_UNSUPPORTED, "host: string tensors are not supported in graphs");
  SB_CHECK(dtype_size(t.data_type) != 0, SB_UNSUPPORTED,
           "host: tensor dtype " + std::to_string(t.data_type) + " not supported");
  HostTensor h;
  h.dtype = t.data_type;
  h.shape = t.dims;
  h.buf = std::make_shared<std::vector<uint8_t>>(t.data);
  SB_CHECK(int64_t(h.buf->size()) == h.numel() * int64_t(dtype_size(h.dtype)), SB_INVALID_ARGUMENT,
           "onnx: tensor '" + t.name + "' has no or short data");
  return h;
}

HostTensor HostTensor::scalar_i64(int64_t v) {
  HostTensor h(DT_INT64, {});
  h.set_i64(0, v);
  return h;
}

HostTensor HostTensor::vec_i64(const std::vector<int64_t>& v) {
  HostTensor h(DT_INT64, {int64_t(v.size())});
  if (!v.empty()) std::memcpy(h.mutable_data(), v.data(), v.size() * 8);
  return h;
}

HostTensor HostTensor::scalar_f32(float v) {
  HostTensor h(DT_FLOAT, {});
  h.set_f64(0, v);
  return h;
}

HostTensor HostTensor::reshaped(const std::vector<int64_t>& s) const {
  HostTensor h = *this;
  data();   // force materialisation of lazy views (shape changes would break the transpose)
  h.buf = buf;
  h.transpose_src.reset();
  h.shape = s;
  return h;
}

std::vector<int64_t> broadcast_shapes(const std::vector<int64_t>& a, const std::vector<int64_t>& b) {
  size_t r = std::max(a.size(), b.size());
  std::vector<int64_t> out(r);
  for (size_t i = 0; i < r; ++i) {
    int64_t da = i < r - a.size() ? 1 : a[i - (r - a.size())];
    int64_t db = i < r - b.size() ? 1 : b[i - (r - b.size())];
    SB_CHECK(da == db || da == 1 || db == 1, SB_SHAPE_ERROR,
             "broadcast: incompatible shapes " + shape_str(a) + " and " + shape_str(b));
    out[i] = da == 1 ? db : da;
  }
  return out;
}

namespace {

// strides (in elements) of `s` broadcast to `out` rank; broadcast dims get 0
std::vector<int64_t> bstrides(const std::vector<int64_t>& s, const std::vector<int64_t>& out) {
  std::vector<int64_t> st(out.size(), 0);
  int64_t acc = 1;
  for (int i = int(s.size()) - 1; i >= 0; --i) {
    size_t oi = out.size() - s.size() + size_t(i);
    st[oi] = s[size_t(i)] == 1 ? 0 : acc;
    acc *= s[size_t(i)];
  }
  return st;
}

template <typename F>
void for_each_index(const std::vector<int64_t>& shape, F f) {
  int64_t n = numel(shape);
  std::vector<int64_t> idx(shape.size(), 0);
  for (int64_t lin = 0; lin < n; ++lin) {
    f(lin, idx);
    for (int d = int(shape.size()) - 1; d >= 0; --d) {
      if (++idx[size_t(d)] < shape[size_t(d)]) break;
      idx[size_t(d)] = 0;
    }
  }
}

int64_t norm_axis(int64_t a, int64_t r) {
  int64_t x = a < 0 ? a + r : a;
  SB_CHECK(x >= 0 && x < std::max<int64_t>(r, 1), SB_SHAPE_ERROR, "axis " + std::to_string(a) + " out of range");
  return x;
}

bool is_int_type(int32_t dt) {
  return dt == DT_INT64 || dt == DT_INT32 || dt == DT_INT16 || dt == DT_INT8 || dt == DT_UINT8 ||
         dt == DT_UINT16 || dt == DT_UINT32 || dt == DT_UINT64;
}

HostTensor binary(const HostTensor& a, const HostTensor& b, int32_t out_dt,
                  const std::function<double(double, double)>& ff,
                  const std::function<int64_t(int64_t, int64_t)>& fi) {
  auto shape = broadcast_shapes(a.shape, b.shape);
  HostTensor o(out_dt, shape);
  auto sa = bstrides(a.shape, shape), sb_ = bstrides(b.shape, shape);
  bool ints = is_int_type(a.dtype) && is_int_type(b.dtype) && fi;
  for_each_index(shape, [&](int64_t lin, const std::vector<int64_t>& idx) {
    int64_t ia = 0, ib = 0;
    for (size_t d = 0; d < idx.size(); ++d) {
      ia += idx[d] * sa[d];
      ib += idx[d] * sb_[d];
    }
    if (ints) o.set_i64(lin, fi(a.get_i64(ia), b.get_i64(ib)));
    else o.set_f64(lin, ff(a.get_f64(ia), b.get_f64(ib)));
  });
  return o;
}

HostTensor unary(const HostTensor& a, const std::function<double(double)>& f) {
  HostTensor o(a.dtype, a.shape);
  for (int64_t i = 0; i < a.numel(); ++i) o.set_f64(i, f(a.get_f64(i)));
  return o;
}

HostTensor gather_bytes(const HostTensor& x, const std::vector<int64_t>& out_shape,
                        const std::function<int64_t(const std::vector<int64_t>&)>& src_index) {
  HostTensor o(x.dtype, out_shape);
  size_t es = dtype_size(x.dtype);
  const uint8_t* s = x.data();
  uint8_t* d = o.mutable_data();
  for_each_index(out_shape, [&](int64_t lin, const std::vector<int64_t>& idx) {
    std::memcpy(d + size_t(lin) * es, s + size_t(src_index(idx)) * es, es);
  });
  return o;
}

std::vector<int64_t> contiguous_strides(const std::vector<int64_t>& s) {
  std::vector<int64_t> st(s.size());
  int64_t acc = 1;
  for (int i = int(s.size()) - 1; i >= 0; --i) {
    st[size_t(i)] = acc;
    acc *= s[size_t(i)];
  }
  return st;
}

HostTensor reduce(const HostTensor& x, std::vector<int64_t> axes, bool keep, const std::string& kind) {
  int64_t r = int64_t(x.shape.size());
  if (axes.empty())
    for (int64_t i = 0; i < r; ++i) axes.push_back(i);
  std::vector<bool> red(size_t(r), false);
  for (auto a : axes) red[size_t(norm_axis(a, r))] = true;
  std::vector<int64_t> oshape, kshape;
  for (int64_t i = 0; i < r; ++i) {
    if (red[size_t(i)]) {
      kshape.push_back(1);
      if (keep) oshape.push_back(1);
    } else {
      kshape.push_back(x.shape[size_t(i)]);
      oshape.push_back(x.shape[size_t(i)]);
    }
  }
  int64_t on = numel(kshape);
  std::vector<double> acc(size_t(on), kind == "prod" ? 1.0 : (kind == "max" ? -INFINITY : (kind == "min" ? INFINITY : 0.0)));
  std::vector<int64_t> acci(size_t(on), kind == "prod" ? 1 : 0);
  std::vector<int64_t> cnt(size_t(on), 0);
  auto kst = contiguous_strides(kshape);
  bool ints = is_int_type(x.dtype);
  for_each_index(x.shape, [&](int64_t lin, const std::vector<int64_t>& idx) {
    int64_t o = 0;
    for (size_t d = 0; d < idx.size(); ++d)
      if (!red[d]) o += idx[d] * kst[d];
    if (ints && (kind == "prod" || kind == "sum")) {
      int64_t v = x.get_i64(lin);
      acci[size_t(o)] = kind == "prod" ? acci[size_t(o)] * v : acci[size_t(o)] + v;
    }
    double v = x.get_f64(lin);
    if (kind == "prod") acc[size_t(o)] *= v;
    else if (kind == "max") acc[size_t(o)] = std::max(acc[size_t(o)], v);
    else if (kind == "min") acc[size_t(o)] = std::min(acc[size_t(o)], v);
    else acc[size_t(o)] += v;
    cnt[size_t(o)]++;
  });
  HostTensor out(x.dtype, oshape);
  for (int64_t i = 0; i < on; ++i) {
    if (ints && (kind == "prod" || kind == "sum")) out.set_i64(i, acci[size_t(i)]);
    else if (kind == "mean") out.set_f64(i, acc[size_t(i)] / double(std::max<int64_t>(cnt[size_t(i)], 1)));
    else out.set_f64(i, acc[size_t(i)]);
  }
  return out;
}

int32_t promote(int32_t a, int32_t b) { return a == b ? a : (a == DT_DOUBLE || b == DT_DOUBLE ? DT_DOUBLE : a); }

}  // namespace

static const char* kHostOps[] = {
    "Constant", "ConstantOfShape", "Identity", "Shape", "Size", "Gather", "Slice", "Unsqueeze", "Squeeze",
    "Concat", "Reshape", "Flatten", "Transpose", "Expand", "Cast", "Range", "ReduceProd", "ReduceSum",
    "ReduceMean", "ReduceMax", "ReduceMin", "Add", "Sub", "Mul", "Div", "Pow", "Max", "Min", "Equal", "Less",
    "Greater", "LessOrEqual", "GreaterOrEqual", "Not", "And", "Or", "Where", "Sqrt", "Neg", "Abs", "Exp",
    "Log", "Reciprocal", "Relu", "Sigmoid", "Tanh", "Floor", "Ceil", "MatMul", "Softmax", "Pad",
    "SequenceConstruct", "SequenceAt", "SequenceLength", "Tile"};

bool host_eval_supported(const std::string& op) {
  for (const char* s : kHostOps)
    if (op == s) return true;
  return false;
}

bool host_eval(const OnnxNode& n, const std::vector<const HostTensor*>& in, std::vector<HostTensor>& out,
               int64_t /*opset*/) {
  const std::string& op = n.op_type;
  auto I = [&](size_t i) -> const HostTensor& {
    SB_CHECK(i < in.size() && in[i], SB_INVALID_ARGUMENT, op + ": missing input " + std::to_string(i));
    return *in[i];
  };
  auto has = [&](size_t i) { return i < in.size() && in[i] != nullptr; };
  out.clear();

  if (op == "Constant") {
    if (auto* a = n.attr("value")) {
      out.push_back(HostTensor::from_onnx(*a->t));
    } else if (auto* a2 = n.attr("value_float")) {
      out.push_back(HostTensor::scalar_f32(a2->f));
    } else if (auto* a3 = n.attr("value_int")) {
      out.push_back(HostTensor::scalar_i64(a3->i));
    } else if (auto* a4 = n.attr("value_ints")) {
      out.push_back(HostTensor::vec_i64(a4->ints));
    } else if (auto* a5 = n.attr("value_floats")) {
      HostTensor h(DT_FLOAT, {int64_t(a5->floats.size())});
      for (size_t i = 0; i < a5->floats.size(); ++i) h.set_f64(int64_t(i), a5->floats[i]);
      out.push_back(h);
    } else {
      fail(SB_UNSUPPORTED, "Constant: unsupported value attribute");
    }
    return true;
  }
  if (op == "ConstantOfShape") {
    auto shape = I(0).to_i64_vec();
    HostTensor v = HostTensor::scalar_f32(0.f);
    if (auto* a = n.attr("value")) v = HostTensor::from_onnx(*a->t);
    HostTensor o(v.dtype, shape);
    size_t es = dtype_size(v.dtype);
    uint8_t* d = o.mutable_data();
    for (int64_t i = 0; i < o.numel(); ++i) std::memcpy(d + size_t(i) * es, v.data(), es);
    out.push_back(o);
    return true;
  }
  if (op == "Identity") { out.push_back(I(0)); return true; }
  // Sequences (the reference's module-stage graphs hold a module's parameters in one and pick them
  // by computed index: SequenceConstruct -> SequenceAt, FastOnnxModelBuilder.cs:1116-1190).
  if (op == "SequenceConstruct") {
    HostTensor s;
    s.seq = std::make_shared<std::vector<HostTensor>>();
    for (size_t i = 0; i < in.size(); ++i) {
      SB_CHECK(in[i] && !in[i]->seq, SB_INVALID_ARGUMENT, "SequenceConstruct: tensor inputs expected");
      s.seq->push_back(*in[i]);
    }
    out.push_back(s);
    return true;
  }
  if (op == "SequenceAt" || op == "SequenceLength") {
    SB_CHECK(I(0).seq != nullptr, SB_INVALID_ARGUMENT, op + ": input 0 is not a sequence");
    const auto& items = *I(0).seq;
    if (op == "SequenceLength") {
      out.push_back(HostTensor::scalar_i64(int64_t(items.size())));
      return true;
    }
    int64_t k = I(1).get_i64(0);
    if (k < 0) k += int64_t(items.size());
    SB_CHECK(k >= 0 && k < int64_t(items.size()), SB_INVALID_ARGUMENT, "SequenceAt: index out of range");
    out.push_back(items[size_t(k)]);
    return true;
  }
  if (op == "Pad") {   // constant mode only (the mode the reference emits)
    std::string mode = n.attr_s("mode", "constant");
    SB_CHECK(mode == "constant", SB_UNSUPPORTED, "Pad: only constant mode on the host");
    const HostTensor& x = I(0);
    const int64_t r = int64_t(x.shape.size());
    auto pads = I(1).to_i64_vec();
    std::vector<int64_t> axes;
    if (has(3)) {
      for (int64_t a : I(3).to_i64_vec()) axes.push_back(a < 0 ? a + r : a);
    } else {
      for (int64_t a = 0; a < r; ++a) axes.push_back(a);
    }
    SB_CHECK(pads.size() == 2 * axes.size(), SB_SHAPE_ERROR, "Pad: pads length");
    std::vector<int64_t> lo(static_cast<size_t>(r), 0), hi(static_cast<size_t>(r), 0);
    for (size_t j = 0; j < axes.size(); ++j) {
      lo[size_t(axes[j])] = pads[j];
      hi[size_t(axes[j])] = pads[j + axes.size()];
      SB_CHECK(pads[j] >= 0 && pads[j + axes.size()] >= 0, SB_UNSUPPORTED, "Pad: negative pads");
    }
    std::vector<int64_t> os(static_cast<size_t>(r), 0);
    for (int64_t d = 0; d < r; ++d) os[size_t(d)] = x.shape[size_t(d)] + lo[size_t(d)] + hi[size_t(d)];
    HostTensor o(x.dtype, os);
    const double cv = has(2) && I(2).numel() ? I(2).get_f64(0) : 0.0;
    const bool fl = x.is_float();
    for (int64_t i = 0; i < o.numel(); ++i) {   // every output element: copy or fill
      int64_t rem = i, src = 0, stride = 1;
      bool inside = true;
      for (int64_t d = r - 1; d >= 0; --d) {
        const int64_t c = rem % os[size_t(d)] - lo[size_t(d)];
        rem /= os[size_t(d)];
        if (c < 0 || c >= x.shape[size_t(d)]) inside = false;
        src += c * stride;
        stride *= x.shape[size_t(d)];
      }
      if (fl) o.set_f64(i, inside ? x.get_f64(src) : cv);
      else o.set_i64(i, inside ? x.get_i64(src) : int64_t(cv));
    }
    out.push_back(o);
    return true;
  }
  if (op == "Shape") {
    auto s = I(0).shape;
    int64_t r = int64_t(s.size());
    int64_t st = n.attr_i("start", 0), en = n.attr_i("end", r);
    if (st < 0) st += r;
    if (en < 0) en += r;
    st = std::clamp<int64_t>(st, 0, r);
    en = std::clamp<int64_t>(en, 0, r);
    out.push_back(HostTensor::vec_i64(std::vector<int64_t>(s.begin() + st, s.begin() + std::max(st, en))));
    return true;
  }
  if (op == "Size") { out.push_back(HostTensor::scalar_i64(I(0).numel())); return true; }
  if (op == "Gather") {
    const HostTensor& x = I(0);
    const HostTensor& ind = I(1);
    int64_t r = int64_t(x.shape.size());
    int64_t ax = norm_axis(n.attr_i("axis", 0), r);
    std::vector<int64_t> oshape(x.shape.begin(), x.shape.begin() + ax);
    oshape.insert(oshape.end(), ind.shape.begin(), ind.shape.end());
    oshape.insert(oshape.end(), x.shape.begin() + ax + 1, x.shape.end());
    auto xs = contiguous_strides(x.shape);
    auto idxv = ind.to_i64_vec();
    auto ist = contiguous_strides(ind.shape);
    int64_t dim = x.shape[size_t(ax)];
    int64_t ir = int64_t(ind.shape.size());
    out.push_back(gather_bytes(x, oshape, [&](const std::vector<int64_t>& idx) {
      int64_t s = 0;
      for (int64_t d = 0; d < ax; ++d) s += idx[size_t(d)] * xs[size_t(d)];
      int64_t li = 0;
      for (int64_t d = 0; d < ir; ++d) li += idx[size_t(ax + d)] * ist[size_t(d)];
      int64_t g = idxv[size_t(li)];
      if (g < 0) g += dim;
      SB_CHECK(g >= 0 && g < dim, SB_INVALID_ARGUMENT, "Gather: index out of range");
      s += g * xs[size_t(ax)];
      for (int64_t d = ax + 1; d < r; ++d) s += idx[size_t(d + ir - 1)] * xs[size_t(d)];
      return s;
    }));
    return true;
  }
  if (op == "Slice") {
    const HostTensor& x = I(0);
    int64_t r = int64_t(x.shape.size());
    auto starts = I(1).to_i64_vec(), ends = I(2).to_i64_vec();
    std::vector<int64_t> axes, steps;
    if (has(3)) axes = I(3).to_i64_vec();
    else for (size_t i = 0; i < starts.size(); ++i) axes.push_back(int64_t(i));
    if (has(4)) steps = I(4).to_i64_vec();
    else steps.assign(starts.size(), 1);
    std::vector<int64_t> st(size_t(r), 0), sp(size_t(r), 1), oshape = x.shape;
    for (size_t i = 0; i < starts.size(); ++i) {
      int64_t a = norm_axis(axes[i], r);
      int64_t d = x.shape[size_t(a)];
      int64_t s = starts[i], e = ends[i], stp = steps[i];
      SB_CHECK(stp != 0, SB_INVALID_ARGUMENT, "Slice: zero step");
      if (s < 0) s += d;
      if (e < 0) e += d;
      if (stp > 0) {
        s = std::clamp<int64_t>(s, 0, d);
        e = std::clamp<int64_t>(e, 0, d);
        oshape[size_t(a)] = std::max<int64_t>(0, ceil_div(e - s, stp));
      } else {
        s = std::clamp<int64_t>(s, -1, d - 1);
        e = std::clamp<int64_t>(e, -1, d - 1);
        oshape[size_t(a)] = std::max<int64_t>(0, ceil_div(s - e, -stp));
      }
      st[size_t(a)] = s;
      sp[size_t(a)] = stp;
    }
    auto xs = contiguous_strides(x.shape);
    out.push_back(gather_bytes(x, oshape, [&](const std::vector<int64_t>& idx) {
      int64_t s = 0;
      for (int64_t d = 0; d < r; ++d) s += (st[size_t(d)] + idx[size_t(d)] * sp[size_t(d)]) * xs[size_t(d)];
      return s;
    }));
    return true;
  }
  if (op == "Unsqueeze" || op == "Squeeze") {
    const HostTensor& x = I(0);
    std::vector<int64_t> axes = has(1) ? I(1).to_i64_vec() : n.attr_ints("axes");
    std::vector<int64_t> s = x.shape;
    if (op == "Unsqueeze") {
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
        for (auto a : axes) {
          int64_t aa = norm_axis(a, r);
          SB_CHECK(s[size_t(aa)] == 1, SB_SHAPE_ERROR, "Squeeze: dim is not 1");
          drop[size_t(aa)] = true;
        }
      }
      std::vector<int64_t> ns;
      for (int64_t i = 0; i < r; ++i)
        if (!drop[size_t(i)]) ns.push_back(s[size_t(i)]);
      s = ns;
    }
    out.push_back(x.reshaped(s));
    return true;
  }
  if (op == "Concat") {
    std::vector<const HostTensor*> xs;
    for (size_t i = 0; i < in.size(); ++i)
      if (in[i]) xs.push_back(in[i]);
    SB_CHECK(!xs.empty(), SB_INVALID_ARGUMENT, "Concat: no inputs");
    int64_t r = int64_t(xs[0]->shape.size());
    int64_t ax = norm_axis(n.attr_i("axis", 0), r);
    std::vector<int64_t> oshape = xs[0]->shape;
    oshape[size_t(ax)] = 0;
    for (auto* x : xs) oshape[size_t(ax)] += x->shape[size_t(ax)];
    HostTensor o(xs[0]->dtype, oshape);
    size_t es = dtype_size(o.dtype);
    int64_t outer = 1;
    for (int64_t d = 0; d < ax; ++d) outer *= oshape[size_t(d)];
    int64_t inner = 1;
    for (int64_t d = ax + 1; d < r; ++d) inner *= oshape[size_t(d)];
    uint8_t* dst = o.mutable_data();
    int64_t off = 0;
    for (auto* x : xs) {
      SB_CHECK(x->dtype == o.dtype, SB_INVALID_ARGUMENT, "Concat: dtype mismatch");
      int64_t w = x->shape[size_t(ax)] * inner;
      const uint8_t* s = x->data();
      for (int64_t i = 0; i < outer; ++i)
        std::memcpy(dst + size_t(i * oshape[size_t(ax)] * inner + off) * es, s + size_t(i * w) * es, size_t(w) * es);
      off += w;
    }
    out.push_back(o);
    return true;
  }
  if (op == "Reshape") {
    const HostTensor& x = I(0);
    auto shp = I(1).to_i64_vec();
    bool allowzero = n.attr_i("allowzero", 0) != 0;
    int64_t known = 1, neg = -1;
    for (size_t i = 0; i < shp.size(); ++i) {
      if (shp[i] == 0 && !allowzero) shp[i] = x.shape.at(i);
      if (shp[i] == -1) {
        SB_CHECK(neg < 0, SB_SHAPE_ERROR, "Reshape: more than one -1");
        neg = int64_t(i);
      } else {
        known *= shp[i];
      }
    }
    if (neg >= 0) shp[size_t(neg)] = known ? x.numel() / known : 0;
    SB_CHECK(numel(shp) == x.numel(), SB_SHAPE_ERROR,
             "Reshape: cannot reshape " + shape_str(x.shape) + " to " + shape_str(shp));
    out.push_back(x.reshaped(shp));
    return true;
  }
  if (op == "Flatten") {
    const HostTensor& x = I(0);
    int64_t r = int64_t(x.shape.size());
    int64_t a = n.attr_i("axis", 1);
    if (a < 0) a += r;
    int64_t o = 1;
    for (int64_t i = 0; i < a; ++i) o *= x.shape[size_t(i)];
    out.push_back(x.reshaped({o, o ? x.numel() / o : 0}));
    return true;
  }
  if (op == "Transpose") {
    const HostTensor& x = I(0);
    int64_t r = int64_t(x.shape.size());
    auto perm = n.attr_ints("perm");
    if (perm.empty())
      for (int64_t i = r - 1; i >= 0; --i) perm.push_back(i);
    std::vector<int64_t> oshape;
    for (auto p : perm) oshape.push_back(x.shape[size_t(p)]);
    if (r == 2 && perm[0] == 1 && perm[1] == 0 && x.numel() > 4096) {   // lazy
      HostTensor h;
      h.dtype = x.dtype;
      h.shape = oshape;
      h.transpose_src = std::make_shared<HostTensor>(x);
      out.push_back(h);
      return true;
    }
    auto xs = contiguous_strides(x.shape);
    out.push_back(gather_bytes(x, oshape, [&](const std::vector<int64_t>& idx) {
      int64_t s = 0;
      for (int64_t d = 0; d < r; ++d) s += idx[size_t(d)] * xs[size_t(perm[size_t(d)])];
      return s;
    }));
    return true;
  }
  if (op == "Expand") {
    const HostTensor& x = I(0);
    auto shape = broadcast_shapes(x.shape, I(1).to_i64_vec());
    auto st = bstrides(x.shape, shape);
    out.push_back(gather_bytes(x, shape, [&](const std::vector<int64_t>& idx) {
      int64_t s = 0;
      for (size_t d = 0; d < idx.size(); ++d) s += idx[d] * st[d];
      return s;
    }));
    return true;
  }
  if (op == "Tile") {   // out[i] = x[i mod x.shape] with out.shape = x.shape * repeats
    const HostTensor& x = I(0);
    auto rep = I(1).to_i64_vec();
    SB_CHECK(rep.size() == x.shape.size(), SB_SHAPE_ERROR, "Tile: repeats length != rank");
    std::vector<int64_t> shape(x.shape.size());
    for (size_t d = 0; d < shape.size(); ++d) {
      SB_CHECK(rep[d] >= 0, SB_SHAPE_ERROR, "Tile: negative repeat");
      shape[d] = x.shape[d] * rep[d];
    }
    auto st = bstrides(x.shape, x.shape);   // (size-1 dims: stride 0, index 0 anyway)
    out.push_back(gather_bytes(x, shape, [&](const std::vector<int64_t>& idx) {
      int64_t s = 0;
      for (size_t d = 0; d < idx.size(); ++d) s += (idx[d] % x.shape[d]) * st[d];
      return s;
    }));
    return true;
  }
  if (op == "Cast") {
    const HostTensor& x = I(0);
    int32_t to = int32_t(n.attr_i("to", DT_FLOAT));
    HostTensor o(to, x.shape);
    for (int64_t i = 0; i < x.numel(); ++i) {
      if (is_int_type(to) && is_int_type(x.dtype)) o.set_i64(i, x.get_i64(i));
      else if (to == DT_BOOL) o.set_i64(i, x.get_f64(i) != 0.0);
      else o.set_f64(i, x.get_f64(i));
    }
    out.push_back(o);
    return true;
  }
  if (op == "Range") {
    const HostTensor& s = I(0);
    if (is_int_type(s.dtype)) {
      int64_t a = s.get_i64(0), b = I(1).get_i64(0), d = I(2).get_i64(0);
      SB_CHECK(d != 0, SB_INVALID_ARGUMENT, "Range: zero delta");
      int64_t cnt = d > 0 ? (b > a ? (b - a + d - 1) / d : 0) : (a > b ? (a - b - d - 1) / (-d) : 0);
      HostTensor o(s.dtype, {cnt});
      for (int64_t i = 0; i < cnt; ++i) o.set_i64(i, a + i * d);
      out.push_back(o);
    } else {
      double a = s.get_f64(0), b = I(1).get_f64(0), d = I(2).get_f64(0);
      int64_t cnt = std::max<int64_t>(0, int64_t(std::ceil((b - a) / d)));
      HostTensor o(s.dtype, {cnt});
      for (int64_t i = 0; i < cnt; ++i) o.set_f64(i, a + double(i) * d);
      out.push_back(o);
    }
    return true;
  }
  if (op.rfind("Reduce", 0) == 0) {
    std::string kind = op == "ReduceProd" ? "prod" : op == "ReduceSum" ? "sum" : op == "ReduceMean" ? "mean"
                     : op == "ReduceMax" ? "max" : "min";
    std::vector<int64_t> axes = has(1) ? I(1).to_i64_vec() : n.attr_ints("axes");
    if (axes.empty() && n.attr_i("noop_with_empty_axes", 0)) { out.push_back(I(0)); return true; }
    out.push_back(reduce(I(0), axes, n.attr_i("keepdims", 1) != 0, kind));
    return true;
  }
  auto cmp_dt = [&](const HostTensor& a, const HostTensor& b) { return promote(a.dtype, b.dtype); };
  if (op == "Add") { out.push_back(binary(I(0), I(1), cmp_dt(I(0), I(1)), [](double a, double b) { return a + b; }, [](int64_t a, int64_t b) { return a + b; })); return true; }
  if (op == "Sub") { out.push_back(binary(I(0), I(1), cmp_dt(I(0), I(1)), [](double a, double b) { return a - b; }, [](int64_t a, int64_t b) { return a - b; })); return true; }
  if (op == "Mul") { out.push_back(binary(I(0), I(1), cmp_dt(I(0), I(1)), [](double a, double b) { return a * b; }, [](int64_t a, int64_t b) { return a * b; })); return true; }
  if (op == "Div") {
    out.push_back(binary(I(0), I(1), cmp_dt(I(0), I(1)), [](double a, double b) { return a / b; },
                         [](int64_t a, int64_t b) {
                           SB_CHECK(b != 0, SB_INVALID_ARGUMENT, "Div: integer division by zero");
                           return a / b;
                         }));
    return true;
  }
  if (op == "Pow") { out.push_back(binary(I(0), I(1), I(0).dtype, [](double a, double b) { return std::pow(a, b); }, nullptr)); return true; }
  if (op == "Max" || op == "Min") {
    HostTensor acc = I(0);
    for (size_t i = 1; i < in.size(); ++i)
      acc = binary(acc, I(i), acc.dtype,
                   op == "Max" ? std::function<double(double, double)>([](double a, double b) { return std::max(a, b); })
                               : std::function<double(double, double)>([](double a, double b) { return std::min(a, b); }),
                   op == "Max" ? std::function<int64_t(int64_t, int64_t)>([](int64_t a, int64_t b) { return std::max(a, b); })
                               : std::function<int64_t(int64_t, int64_t)>([](int64_t a, int64_t b) { return std::min(a, b); }));
    out.push_back(acc);
    return true;
  }
  if (op == "Equal") { out.push_back(binary(I(0), I(1), DT_BOOL, [](double a, double b) { return double(a == b); }, [](int64_t a, int64_t b) { return int64_t(a == b); })); return true; }
  if (op == "Less") { out.push_back(binary(I(0), I(1), DT_BOOL, [](double a, double b) { return double(a < b); }, [](int64_t a, int64_t b) { return int64_t(a < b); })); return true; }
  if (op == "Greater") { out.push_back(binary(I(0), I(1), DT_BOOL, [](double a, double b) { return double(a > b); }, [](int64_t a, int64_t b) { return int64_t(a > b); })); return true; }
  if (op == "LessOrEqual") { out.push_back(binary(I(0), I(1), DT_BOOL, [](double a, double b) { return double(a <= b); }, [](int64_t a, int64_t b) { return int64_t(a <= b); })); return true; }
  if (op == "GreaterOrEqual") { out.push_back(binary(I(0), I(1), DT_BOOL, [](double a, double b) { return double(a >= b); }, [](int64_t a, int64_t b) { return int64_t(a >= b); })); return true; }
  if (op == "And") { out.push_back(binary(I(0), I(1), DT_BOOL, [](double a, double b) { return double(a != 0 && b != 0); }, [](int64_t a, int64_t b) { return int64_t(a && b); })); return true; }
  if (op == "Or") { out.push_back(binary(I(0), I(1), DT_BOOL, [](double a, double b) { return double(a != 0 || b != 0); }, [](int64_t a, int64_t b) { return int64_t(a || b); })); return true; }
  if (op == "Not") {
    HostTensor o(DT_BOOL, I(0).shape);
    for (int64_t i = 0; i < o.numel(); ++i) o.set_i64(i, I(0).get_i64(i) == 0);
    out.push_back(o);
    return true;
  }
  if (op == "Where") {
    const HostTensor &c = I(0), &a = I(1), &b = I(2);
    auto shape = broadcast_shapes(broadcast_shapes(c.shape, a.shape), b.shape);
    auto sc = bstrides(c.shape, shape), sa = bstrides(a.shape, shape), sbb = bstrides(b.shape, shape);
    HostTensor o(a.dtype, shape);
    size_t es = dtype_size(a.dtype);
    for_each_index(shape, [&](int64_t lin, const std::vector<int64_t>& idx) {
      int64_t ic = 0, ia = 0, ib = 0;
      for (size_t d = 0; d < idx.size(); ++d) { ic += idx[d] * sc[d]; ia += idx[d] * sa[d]; ib += idx[d] * sbb[d]; }
      const HostTensor& src = c.get_i64(ic) ? a : b;
      std::memcpy(o.mutable_data() + size_t(lin) * es, src.data() + size_t(c.get_i64(ic) ? ia : ib) * es, es);
    });
    out.push_back(o);
    return true;
  }
  if (op == "Sqrt") { out.push_back(unary(I(0), [](double v) { return std::sqrt(v); })); return true; }
  if (op == "Neg") {
    if (is_int_type(I(0).dtype)) {
      HostTensor o(I(0).dtype, I(0).shape);
      for (int64_t i = 0; i < o.numel(); ++i) o.set_i64(i, -I(0).get_i64(i));
      out.push_back(o);
    } else {
      out.push_back(unary(I(0), [](double v) { return -v; }));
    }
    return true;
  }
  if (op == "Abs") { out.push_back(unary(I(0), [](double v) { return std::fabs(v); })); return true; }
  if (op == "Exp") { out.push_back(unary(I(0), [](double v) { return std::exp(v); })); return true; }
  if (op == "Log") { out.push_back(unary(I(0), [](double v) { return std::log(v); })); return true; }
  if (op == "Reciprocal") { out.push_back(unary(I(0), [](double v) { return 1.0 / v; })); return true; }
  if (op == "Relu") { out.push_back(unary(I(0), [](double v) { return v > 0 ? v : 0.0; })); return true; }
  if (op == "Sigmoid") { out.push_back(unary(I(0), [](double v) { return 1.0 / (1.0 + std::exp(-v)); })); return true; }
  if (op == "Tanh") { out.push_back(unary(I(0), [](double v) { return std::tanh(v); })); return true; }
  if (op == "Floor") { out.push_back(unary(I(0), [](double v) { return std::floor(v); })); return true; }
  if (op == "Ceil") { out.push_back(unary(I(0), [](double v) { return std::ceil(v); })); return true; }
  if (op == "MatMul") {
    const HostTensor &a = I(0), &b = I(1);
    // rank 2 x rank 2; a rank-1 operand is a row (left) or a column (right) vector whose unit
    // dimension is dropped from the result (numpy matmul)
    SB_CHECK(a.shape.size() >= 1 && a.shape.size() <= 2 && b.shape.size() >= 1 && b.shape.size() <= 2, SB_UNSUPPORTED,
             "host MatMul: operands of rank 1 or 2 only");
    const bool av = a.shape.size() == 1, bv = b.shape.size() == 1;
    int64_t M = av ? 1 : a.shape[0], K = av ? a.shape[0] : a.shape[1], N = bv ? 1 : b.shape[1];
    SB_CHECK((bv ? b.shape[0] : b.shape[0]) == K, SB_SHAPE_ERROR, "MatMul: inner dims differ");
    std::vector<int64_t> os;
    if (!av) os.push_back(M);
    if (!bv) os.push_back(N);
    HostTensor o(a.dtype, os);
    for (int64_t i = 0; i < M; ++i)
      for (int64_t j = 0; j < N; ++j) {
        double acc = 0;
        for (int64_t k = 0; k < K; ++k) acc += a.get_f64(i * K + k) * b.get_f64(k * N + j);
        o.set_f64(i * N + j, acc);
      }
    out.push_back(o);
    return true;
  }
  if (op == "Softmax") {
    const HostTensor& x = I(0);
    int64_t r = int64_t(x.shape.size());
    int64_t ax = norm_axis(n.attr_i("axis", -1), r);
    int64_t inner = 1;
    for (int64_t d = ax + 1; d < r; ++d) inner *= x.shape[size_t(d)];
    int64_t len = x.shape[size_t(ax)];
    int64_t outer = x.numel() / std::max<int64_t>(1, len * inner);
    HostTensor o(x.dtype, x.shape);
    for (int64_t a = 0; a < outer; ++a)
      for (int64_t c = 0; c < inner; ++c) {
        double m = -INFINITY, s = 0;
        for (int64_t l = 0; l < len; ++l) m = std::max(m, x.get_f64((a * len + l) * inner + c));
        for (int64_t l = 0; l < len; ++l) s += std::exp(x.get_f64((a * len + l) * inner + c) - m);
        for (int64_t l = 0; l < len; ++l)
          o.set_f64((a * len + l) * inner + c, std::exp(x.get_f64((a * len + l) * inner + c) - m) / s);
      }
    out.push_back(o);
    return true;
  }
  return false;
}

}  // namespace sb
