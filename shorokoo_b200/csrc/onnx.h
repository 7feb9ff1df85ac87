// ONNX ModelProto reader: a hand-written protobuf wire-format decoder (no libprotobuf in the image).
// Covers the message types the reference's FastOnnxModelBuilder emits
// (src/Shorokoo/Core/Factory/IR/onnx_IR10.cs): Model, Graph, Node, Attribute, Tensor, ValueInfo,
// Function.
#pragma once

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"

namespace sb {

struct OnnxTensor {
  std::string name;
  std::vector<int64_t> dims;
  int32_t data_type = 0;
  std::vector<uint8_t> data;   // little-endian element bytes (raw_data or decoded typed fields)
  bool has_data = false;
};

struct OnnxGraph;

struct OnnxAttr {
  enum Kind { UNDEF = 0, FLOAT = 1, INT = 2, STRING = 3, TENSOR = 4, GRAPH = 5, FLOATS = 6, INTS = 7, STRINGS = 8 };
  std::string name;
  std::string ref_attr_name;
  int kind = UNDEF;
  float f = 0;
  int64_t i = 0;
  std::string s;
  std::shared_ptr<OnnxTensor> t;
  std::shared_ptr<OnnxGraph> g;
  std::vector<float> floats;
  std::vector<int64_t> ints;
  std::vector<std::string> strings;
};

struct OnnxNode {
  std::string name, op_type, domain;
  std::vector<std::string> inputs, outputs;
  std::vector<OnnxAttr> attrs;

  const OnnxAttr* attr(const std::string& n) const {
    for (auto& a : attrs)
      if (a.name == n) return &a;
    return nullptr;
  }
  int64_t attr_i(const std::string& n, int64_t def) const {
    auto* a = attr(n);
    return a ? a->i : def;
  }
  float attr_f(const std::string& n, float def) const {
    auto* a = attr(n);
    return a ? a->f : def;
  }
  std::string attr_s(const std::string& n, const std::string& def) const {
    auto* a = attr(n);
    return a ? a->s : def;
  }
  std::vector<int64_t> attr_ints(const std::string& n) const {
    auto* a = attr(n);
    return a ? a->ints : std::vector<int64_t>{};
  }
};

struct OnnxValueInfo {
  std::string name;
  int32_t elem_type = 0;
  bool has_shape = false;
  std::vector<int64_t> dims;   // -1 for symbolic
};

struct OnnxGraph {
  std::string name;
  std::vector<OnnxNode> nodes;
  std::vector<OnnxTensor> initializers;
  std::vector<OnnxValueInfo> inputs, outputs;
};

struct OnnxFunction {
  std::string name, domain;
  std::vector<std::string> inputs, outputs, attributes;
  std::vector<OnnxNode> nodes;
};

struct OnnxModel {
  int64_t ir_version = 0;
  std::map<std::string, int64_t> opsets;
  OnnxGraph graph;
  std::vector<OnnxFunction> functions;
};

// Throws sb::Error(SB_INVALID_ARGUMENT) on malformed or truncated input.
OnnxModel parse_onnx(const uint8_t* data, size_t len);

}  // namespace sb
