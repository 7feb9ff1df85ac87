// Protobuf wire-format decoder for ONNX (field numbers from the public onnx.proto).
#include "onnx.h"

#include <cstring>

namespace sb {
namespace {

struct Reader {
  const uint8_t* p;
  const uint8_t* end;

  bool done() const { return p >= end; }

  uint64_t varint() {
    uint64_t r = 0;
    int shift = 0;
    while (true) {
      SB_CHECK(p < end, SB_INVALID_ARGUMENT, "onnx: truncated varint");
      uint8_t b = *p++;
      r |= uint64_t(b & 0x7f) << shift;
      if (!(b & 0x80)) return r;
      shift += 7;
      SB_CHECK(shift < 70, SB_INVALID_ARGUMENT, "onnx: varint too long");
    }
  }
  Reader sub() {
    uint64_t n = varint();
    SB_CHECK(n <= uint64_t(end - p), SB_INVALID_ARGUMENT, "onnx: truncated length-delimited field");
    Reader r{p, p + n};
    p += n;
    return r;
  }
  std::string str() {
    Reader r = sub();
    return std::string(reinterpret_cast<const char*>(r.p), r.end - r.p);
  }
  uint32_t fixed32() {
    SB_CHECK(end - p >= 4, SB_INVALID_ARGUMENT, "onnx: truncated fixed32");
    uint32_t v;
    std::memcpy(&v, p, 4);
    p += 4;
    return v;
  }
  uint64_t fixed64() {
    SB_CHECK(end - p >= 8, SB_INVALID_ARGUMENT, "onnx: truncated fixed64");
    uint64_t v;
    std::memcpy(&v, p, 8);
    p += 8;
    return v;
  }
  void skip(int wt) {
    switch (wt) {
      case 0: varint(); break;
      case 1: fixed64(); break;
      case 2: sub(); break;
      case 5: fixed32(); break;
      default: fail(SB_INVALID_ARGUMENT, "onnx: unsupported wire type " + std::to_string(wt));
    }
  }
  // next field key; returns false at end
  bool key(int& no, int& wt) {
    if (done()) return false;
    uint64_t k = varint();
    no = int(k >> 3);
    wt = int(k & 7);
    return true;
  }
};

// repeated int64/int32 (packed or not)
void read_ints(Reader& r, int wt, std::vector<int64_t>& out) {
  if (wt == 2) {
    Reader s = r.sub();
    while (!s.done()) out.push_back(int64_t(s.varint()));
  } else {
    out.push_back(int64_t(r.varint()));
  }
}

template <typename T, typename U>
void read_fixed(Reader& r, int wt, std::vector<uint8_t>& out) {
  auto push = [&](U v) {
    T t;
    std::memcpy(&t, &v, sizeof(T));
    size_t o = out.size();
    out.resize(o + sizeof(T));
    std::memcpy(out.data() + o, &t, sizeof(T));
  };
  if (wt == 2) {
    Reader s = r.sub();
    while (!s.done()) push(sizeof(U) == 4 ? U(s.fixed32()) : U(s.fixed64()));
  } else {
    push(sizeof(U) == 4 ? U(r.fixed32()) : U(r.fixed64()));
  }
}

OnnxGraph parse_graph(Reader r);

OnnxTensor parse_tensor(Reader r) {
  OnnxTensor t;
  std::vector<int64_t> i32s, i64s;
  std::vector<uint8_t> fdata, ddata, u64data;
  bool have_raw = false;
  int no, wt;
  while (r.key(no, wt)) {
    switch (no) {
      case 1: read_ints(r, wt, t.dims); break;
      case 2: t.data_type = int32_t(r.varint()); break;
      case 8: t.name = r.str(); break;
      case 9: {
        Reader s = r.sub();
        t.data.assign(s.p, s.end);
        have_raw = true;
        break;
      }
      case 4: read_fixed<uint32_t, uint32_t>(r, wt, fdata); break;
      case 10: read_fixed<uint64_t, uint64_t>(r, wt, ddata); break;
      case 5: read_ints(r, wt, i32s); break;
      case 7: read_ints(r, wt, i64s); break;
      case 11: {
        std::vector<int64_t> tmp;
        read_ints(r, wt, tmp);
        for (int64_t v : tmp) {
          size_t o = u64data.size();
          u64data.resize(o + 8);
          std::memcpy(u64data.data() + o, &v, 8);
        }
        break;
      }
      case 13: case 14:
        if (no == 14) {
          uint64_t loc = r.varint();
          SB_CHECK(loc == 0, SB_UNSUPPORTED, "onnx: external tensor data is not supported");
        } else {
          fail(SB_UNSUPPORTED, "onnx: external tensor data is not supported");
        }
        break;
      default: r.skip(wt);
    }
  }
  if (have_raw) {
    t.has_data = true;
  } else {
    size_t es = dtype_size(t.data_type);
    switch (t.data_type) {
      case DT_FLOAT: t.data = fdata; t.has_data = !fdata.empty(); break;
      case DT_DOUBLE: t.data = ddata; t.has_data = !ddata.empty(); break;
      case DT_UINT64: t.data = u64data; t.has_data = !u64data.empty(); break;
      case DT_INT64:
        t.data.resize(i64s.size() * 8);
        if (!i64s.empty()) std::memcpy(t.data.data(), i64s.data(), i64s.size() * 8);
        t.has_data = !i64s.empty();
        break;
      case DT_UINT32: {
        t.data.resize(i64s.size() * 4);
        for (size_t k = 0; k < i64s.size(); ++k) {
          uint32_t v = uint32_t(i64s[k]);
          std::memcpy(t.data.data() + 4 * k, &v, 4);
        }
        t.has_data = !i64s.empty();
        break;
      }
      default:
        // int32_data carries INT32/INT16/INT8/UINT16/UINT8/BOOL/FLOAT16/BFLOAT16 bit patterns.
        if (es) {
          t.data.resize(i32s.size() * es);
          for (size_t k = 0; k < i32s.size(); ++k) {
            int64_t v = i32s[k];
            std::memcpy(t.data.data() + es * k, &v, es);
          }
          t.has_data = !i32s.empty();
        }
    }
    int64_t n = numel(t.dims);
    if (!t.has_data && n == 0) t.has_data = true;   // empty tensor
  }
  if (t.has_data && t.data_type != DT_STRING) {
    size_t es = dtype_size(t.data_type);
    SB_CHECK(es != 0, SB_UNSUPPORTED, std::string("onnx: tensor dtype ") + std::to_string(t.data_type) + " not supported");
    SB_CHECK(int64_t(t.data.size()) == numel(t.dims) * int64_t(es), SB_INVALID_ARGUMENT,
             "onnx: tensor '" + t.name + "' payload size " + std::to_string(t.data.size()) +
                 " does not match dims " + shape_str(t.dims));
  }
  return t;
}

OnnxAttr parse_attr(Reader r) {
  OnnxAttr a;
  int no, wt;
  while (r.key(no, wt)) {
    switch (no) {
      case 1: a.name = r.str(); break;
      case 21: a.ref_attr_name = r.str(); break;
      case 20: a.kind = int(r.varint()); break;
      case 2: { uint32_t v = r.fixed32(); std::memcpy(&a.f, &v, 4); break; }
      case 3: a.i = int64_t(r.varint()); break;
      case 4: a.s = r.str(); break;
      case 5: a.t = std::make_shared<OnnxTensor>(parse_tensor(r.sub())); break;
      case 6: a.g = std::make_shared<OnnxGraph>(parse_graph(r.sub())); break;
      case 7: {
        std::vector<uint8_t> tmp;
        read_fixed<uint32_t, uint32_t>(r, wt, tmp);
        size_t n = tmp.size() / 4;
        size_t o = a.floats.size();
        a.floats.resize(o + n);
        std::memcpy(a.floats.data() + o, tmp.data(), n * 4);
        break;
      }
      case 8: read_ints(r, wt, a.ints); break;
      case 9: a.strings.push_back(r.str()); break;
      default: r.skip(wt);
    }
  }
  if (a.kind == OnnxAttr::UNDEF) {   // older writers may omit the type field
    if (a.g) a.kind = OnnxAttr::GRAPH;
    else if (a.t) a.kind = OnnxAttr::TENSOR;
    else if (!a.ints.empty()) a.kind = OnnxAttr::INTS;
    else if (!a.floats.empty()) a.kind = OnnxAttr::FLOATS;
    else if (!a.s.empty()) a.kind = OnnxAttr::STRING;
  }
  return a;
}

OnnxNode parse_node(Reader r) {
  OnnxNode n;
  int no, wt;
  while (r.key(no, wt)) {
    switch (no) {
      case 1: n.inputs.push_back(r.str()); break;
      case 2: n.outputs.push_back(r.str()); break;
      case 3: n.name = r.str(); break;
      case 4: n.op_type = r.str(); break;
      case 7: n.domain = r.str(); break;
      case 5: n.attrs.push_back(parse_attr(r.sub())); break;
      default: r.skip(wt);
    }
  }
  SB_CHECK(!n.op_type.empty(), SB_INVALID_ARGUMENT, "onnx: node '" + n.name + "' has no op_type");
  return n;
}

OnnxValueInfo parse_value_info(Reader r) {
  OnnxValueInfo v;
  int no, wt;
  while (r.key(no, wt)) {
    if (no == 1) {
      v.name = r.str();
    } else if (no == 2) {
      Reader tp = r.sub();
      int n2, w2;
      while (tp.key(n2, w2)) {
        if (n2 == 1) {   // tensor_type
          Reader tt = tp.sub();
          int n3, w3;
          while (tt.key(n3, w3)) {
            if (n3 == 1) {
              v.elem_type = int32_t(tt.varint());
            } else if (n3 == 2) {
              v.has_shape = true;
              Reader sh = tt.sub();
              int n4, w4;
              while (sh.key(n4, w4)) {
                if (n4 == 1) {
                  Reader dm = sh.sub();
                  int64_t d = -1;
                  int n5, w5;
                  while (dm.key(n5, w5)) {
                    if (n5 == 1) d = int64_t(dm.varint());
                    else dm.skip(w5);
                  }
                  v.dims.push_back(d);
                } else {
                  sh.skip(w4);
                }
              }
            } else {
              tt.skip(w3);
            }
          }
        } else {
          tp.skip(w2);
        }
      }
    } else {
      r.skip(wt);
    }
  }
  return v;
}

OnnxGraph parse_graph(Reader r) {
  OnnxGraph g;
  int no, wt;
  while (r.key(no, wt)) {
    switch (no) {
      case 1: g.nodes.push_back(parse_node(r.sub())); break;
      case 2: g.name = r.str(); break;
      case 5: g.initializers.push_back(parse_tensor(r.sub())); break;
      case 11: g.inputs.push_back(parse_value_info(r.sub())); break;
      case 12: g.outputs.push_back(parse_value_info(r.sub())); break;
      case 15: fail(SB_UNSUPPORTED, "onnx: sparse initializers are not supported");
      default: r.skip(wt);
    }
  }
  return g;
}

OnnxFunction parse_function(Reader r) {
  OnnxFunction f;
  int no, wt;
  while (r.key(no, wt)) {
    switch (no) {
      case 1: f.name = r.str(); break;
      case 10: f.domain = r.str(); break;
      case 4: f.inputs.push_back(r.str()); break;
      case 5: f.outputs.push_back(r.str()); break;
      case 6: f.attributes.push_back(r.str()); break;
      case 7: f.nodes.push_back(parse_node(r.sub())); break;
      default: r.skip(wt);
    }
  }
  return f;
}

}  // namespace

OnnxModel parse_onnx(const uint8_t* data, size_t len) {
  SB_CHECK(data != nullptr && len > 0, SB_INVALID_ARGUMENT, "onnx: empty model bytes");
  Reader r{data, data + len};
  OnnxModel m;
  bool have_graph = false;
  int no, wt;
  while (r.key(no, wt)) {
    switch (no) {
      case 1: m.ir_version = int64_t(r.varint()); break;
      case 7: m.graph = parse_graph(r.sub()); have_graph = true; break;
      case 8: {
        Reader s = r.sub();
        std::string dom;
        int64_t ver = 0;
        int n2, w2;
        while (s.key(n2, w2)) {
          if (n2 == 1) dom = s.str();
          else if (n2 == 2) ver = int64_t(s.varint());
          else s.skip(w2);
        }
        m.opsets[dom] = ver;
        break;
      }
      case 25: m.functions.push_back(parse_function(r.sub())); break;
      default: r.skip(wt);
    }
  }
  SB_CHECK(have_graph, SB_INVALID_ARGUMENT, "onnx: ModelProto has no graph");
  return m;
}

}  // namespace sb
