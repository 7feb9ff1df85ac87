// Shared definitions for the B200 inference backend: status codes, element types, errors.
#pragma once

#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace sb {

// Status codes returned through the C ABI (include/shorokoo_b200.h).
enum Status : int32_t {
  SB_OK = 0,
  SB_INVALID_ARGUMENT = 1,
  SB_UNSUPPORTED = 2,
  SB_SHAPE_ERROR = 3,
  SB_CUDA_ERROR = 4,
  SB_OUT_OF_MEMORY = 5,
  SB_INTERNAL = 6,
};

// ONNX TensorProto.DataType numbering == ShorokooTensorElementType
// (src/Shorokoo/Core/Inference/Abstractions/ShorokooTensorElementType.cs:6-31).
enum DType : int32_t {
  DT_UNDEFINED = 0,
  DT_FLOAT = 1,
  DT_UINT8 = 2,
  DT_INT8 = 3,
  DT_UINT16 = 4,
  DT_INT16 = 5,
  DT_INT32 = 6,
  DT_INT64 = 7,
  DT_STRING = 8,
  DT_BOOL = 9,
  DT_FLOAT16 = 10,
  DT_DOUBLE = 11,
  DT_UINT32 = 12,
  DT_UINT64 = 13,
  DT_BFLOAT16 = 16,
};

inline size_t dtype_size(int32_t dt) {
  switch (dt) {
    case DT_FLOAT: case DT_INT32: case DT_UINT32: return 4;
    case DT_UINT8: case DT_INT8: case DT_BOOL: return 1;
    case DT_UINT16: case DT_INT16: case DT_FLOAT16: case DT_BFLOAT16: return 2;
    case DT_INT64: case DT_DOUBLE: case DT_UINT64: return 8;
    default: return 0;
  }
}

inline const char* dtype_name(int32_t dt) {
  switch (dt) {
    case DT_FLOAT: return "float32"; case DT_UINT8: return "uint8"; case DT_INT8: return "int8";
    case DT_UINT16: return "uint16"; case DT_INT16: return "int16"; case DT_INT32: return "int32";
    case DT_INT64: return "int64"; case DT_STRING: return "string"; case DT_BOOL: return "bool";
    case DT_FLOAT16: return "float16"; case DT_DOUBLE: return "float64"; case DT_UINT32: return "uint32";
    case DT_UINT64: return "uint64"; case DT_BFLOAT16: return "bfloat16"; default: return "undefined";
  }
}

struct Error : std::runtime_error {
  int32_t code;
  Error(int32_t c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(int32_t code, const std::string& msg) { throw Error(code, msg); }

#define SB_CHECK(cond, code, msg)                 \
  do {                                            \
    if (!(cond)) ::sb::fail((code), (msg));       \
  } while (0)

inline int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (int64_t d : s) n *= d;
  return n;
}

inline std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

// Debug logging gated by SHOROKOO_B200_DEBUG (0 = off, 1 = plan summary, 2 = per-op).
int debug_level();

}  // namespace sb
