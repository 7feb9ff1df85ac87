// Lowered graph: what remains after plan-time specialisation of the ONNX model for one set of
// input shapes and plan-time input values. Host values are folded constants; device values are
// float tensors produced by device ops.
#pragma once

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "host_tensor.h"
#include "onnx.h"

namespace sb {

struct Value {
  int32_t dtype = DT_UNDEFINED;
  std::vector<int64_t> shape;
  bool is_host = false;
  std::shared_ptr<HostTensor> host;   // valid when is_host
  int producer = -1;                  // op index (device values)
  int input_index = -1;               // session input index (device graph inputs)
  std::string name;
};

struct Op {
  std::string type;              // ONNX op type, or a fused kind ("FusedConv", "FusedGemm", ...)
  std::vector<int> in;           // value ids, -1 for absent optional inputs
  std::vector<int> out;
  std::string name;              // originating ONNX node name (diagnostics)
  bool dead = false;
  // Normalised attributes (meaning depends on type).
  std::vector<int64_t> kernel, strides, pads, dilations, perm, axes;
  int64_t axis = 0, group = 1, ceil_mode = 0, keepdims = 1;
  float alpha = 0.f, beta = 0.f, fmin = 0.f, fmax = 0.f;
  std::string mode, coord_mode, nearest_mode;
  std::vector<float> scales;
  // Fused-op payload
  int act = 0;                   // 0 none, 1 relu, 2 sigmoid
  int residual = -1;             // value id of a residual operand (FusedConv/FusedGemm)
  int residual_mode = 0;         // 0 same shape, 1 nearest-2x upsampled source
  int concat = -1;               // FusedConv 1x1/s1: value id of a second activation whose channels
                                 // follow in[0]'s in the reduction (weight holds both blocks)
  int concat_stride = 1;         // stride at which the second activation is sampled (1 or 2)
  std::shared_ptr<HostTensor> weight;   // folded weights (FusedConv: [M,C,KH,KW] f32; FusedGemm: [N,K] f32)
  std::shared_ptr<HostTensor> bias;     // folded bias [M] f32 (may be null)
  int prec = 0;                  // FusedConv/FusedGemm operand precision: 0 bf16, 1 TF32, 2 TF32x3
                                 // (set per op by assign_precision)
};

struct LGraph {
  std::vector<Value> vals;
  std::vector<Op> ops;
  std::vector<int> inputs;    // value id per session input
  std::vector<int> outputs;   // value id per graph output
  std::vector<std::string> output_names;

  int add_value(Value v) {
    vals.push_back(std::move(v));
    return int(vals.size()) - 1;
  }
  int add_host(HostTensor h, const std::string& name = "") {
    Value v;
    v.dtype = h.dtype;
    v.shape = h.shape;
    v.is_host = true;
    v.host = std::make_shared<HostTensor>(std::move(h));
    v.name = name;
    return add_value(std::move(v));
  }
  // Number of live (non-dead) ops reading value `id`, plus graph-output references.
  std::vector<int> use_counts() const;
  void dce();
};

struct InputSpec {
  int32_t dtype = DT_FLOAT;
  std::vector<int64_t> shape;
  std::shared_ptr<HostTensor> value;   // set for plan-time (small) inputs
};

// Session-level view of the model: graph inputs that must be fed (initializers excluded).
struct ModelInfo {
  std::vector<std::string> input_names;
  std::vector<int32_t> input_dtypes;
  std::vector<int> input_ranks;   // -1 unknown
  std::vector<std::string> output_names;
};

ModelInfo model_info(const OnnxModel& m);

// Rejects models that use an operator the backend has neither a host nor a device
// implementation for (hard error at session creation).
void check_supported_ops(const OnnxModel& m);

LGraph lower(const OnnxModel& m, const std::vector<InputSpec>& inputs);

// Sets Op::prec of every contraction from the session precision (0 bf16, 1 TF32, 2 TF32x3): dense
// chains of contractions too long for the session's operand precision to meet its accuracy gate
// get a more precise operand type for part of the chain (precision.cpp).
void assign_precision(LGraph& g, int session_precision);

// Inputs with at most this many elements are treated as plan-time constants (hyper scalars such
// as bnEps / includeTop / Loop trip counts); their values key the plan cache.
constexpr int64_t kPlanTimeInputMaxElems = 16;

}  // namespace sb
