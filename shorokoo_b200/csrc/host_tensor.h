// Host-side tensors and the host evaluator used at plan time: shape arithmetic on graph inputs
// (Shape/Gather/Unsqueeze/Concat/ReduceProd chains), constant folding over initializers
// (e.g. the FrozenBatchNorm Div/Sqrt/Mul/Sub chain) and scalar control-flow conditions.
#pragma once

#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "onnx.h"

namespace sb {

struct HostTensor {
  int32_t dtype = DT_UNDEFINED;
  std::vector<int64_t> shape;
  // Materialised bytes. For a lazy 2-D transpose (see below) this stays null until data() is asked.
  std::shared_ptr<std::vector<uint8_t>> buf;
  // Lazy transpose of a rank-2 host tensor: lets MatMul(x, Transpose(W)) use W [N,K] directly
  // without copying a large weight twice.
  std::shared_ptr<HostTensor> transpose_src;
  // A sequence of tensors (SequenceConstruct; dtype undefined, no shape) when set.
  std::shared_ptr<std::vector<HostTensor>> seq;

  HostTensor() = default;
  HostTensor(int32_t dt, std::vector<int64_t> s);

  int64_t numel() const { return sb::numel(shape); }
  size_t nbytes() const { return size_t(numel()) * dtype_size(dtype); }
  const uint8_t* data() const;
  uint8_t* mutable_data();
  template <typename T> const T* ptr() const { return reinterpret_cast<const T*>(data()); }
  template <typename T> T* mptr() { return reinterpret_cast<T*>(mutable_data()); }

  double get_f64(int64_t i) const;
  int64_t get_i64(int64_t i) const;
  void set_f64(int64_t i, double v);
  void set_i64(int64_t i, int64_t v);
  std::vector<int64_t> to_i64_vec() const;
  std::vector<double> to_f64_vec() const;
  bool is_float() const { return dtype == DT_FLOAT || dtype == DT_DOUBLE || dtype == DT_FLOAT16 || dtype == DT_BFLOAT16; }

  static HostTensor from_onnx(const OnnxTensor& t);
  static HostTensor scalar_i64(int64_t v);
  static HostTensor vec_i64(const std::vector<int64_t>& v);
  static HostTensor scalar_f32(float v);
  HostTensor reshaped(const std::vector<int64_t>& s) const;   // shares bytes
};

// Evaluates one ONNX node whose inputs are all host values. Returns false if the op has no
// host implementation (the caller then treats it as a device op or rejects it).
bool host_eval(const OnnxNode& node, const std::vector<const HostTensor*>& in, std::vector<HostTensor>& out,
               int64_t opset);

// True if host_eval implements this op type.
bool host_eval_supported(const std::string& op_type);

// Numpy-style broadcast of two shapes; throws SB_SHAPE_ERROR when incompatible.
std::vector<int64_t> broadcast_shapes(const std::vector<int64_t>& a, const std::vector<int64_t>& b);

uint16_t f32_to_bf16_rne(float f);
float bf16_to_f32(uint16_t h);
float f16_to_f32(uint16_t h);
uint16_t f32_to_f16(float f);

}  // namespace sb
