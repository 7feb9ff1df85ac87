// Execution plan for one device: every live op of the fused graph becomes one or more kernel
// launches over a static activation arena; weights live in one packed device blob. The launch
// sequence is captured once into a CUDA graph and replayed per run.
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "ir.h"
#include "kernels/kernels.h"

namespace sb {

void fuse(LGraph& g);

struct DevTensor {
  int buf = -2;            // arena buffer id; -1 = weights blob; -2 = invalid
  int64_t off = 0;         // bytes from the buffer start
  bool bf16 = false;
  std::vector<int64_t> shape, strides;   // logical shape, element strides
  bool valid() const { return buf != -2; }
};

struct PlanStats {
  int64_t kernels = 0;          // kernel launches per run
  int64_t tc_kernels = 0;       // tensor-core (tcgen05) launches per run
  double macs = 0;              // algorithmic multiply-accumulates (Conv/MatMul) per run
  double macs_by_prec[3] = {0, 0, 0};   // the same split by operand precision (bf16, TF32, TF32x3)
  size_t arena_bytes = 0, weight_bytes = 0;
};

struct InputBinding {
  int index;               // session input index
  int buf;                 // arena buffer receiving the H2D copy
  size_t bytes;
  bool bf16_ok = false;    // float32 input whose every reader rounds it to bfloat16 first: its values
                           // may arrive as bfloat16 (exact after widening back)
};

struct OutputBinding {
  bool host = false;                 // value folded at plan time
  std::shared_ptr<HostTensor> value; // when host
  DevTensor dev;                     // f32 contiguous when !host
  std::vector<int64_t> shape;
};

class Plan {
 public:
  // precision: the session's operand precision (0 bf16; 1 fp32 read as TF32; 2 TF32x3,
  // error-compensated), turned into one precision per contraction by assign_precision.
  Plan(LGraph g, int device, int num_sms, int precision = 0);
  ~Plan();
  Plan(const Plan&) = delete;
  Plan& operator=(const Plan&) = delete;

  // Enqueues H2D of inputs, the captured kernel graph and D2H of outputs on `stream`.
  // host_in[i] points at session input i (nullptr for plan-time inputs); host_out[j] receives
  // output j (device outputs only; host outputs are copied by the caller).
  void enqueue(cudaStream_t stream, const std::vector<const void*>& host_in, const std::vector<void*>& host_out);
  // Runs only the kernel sequence (inputs already resident); used for device-side timing.
  void enqueue_kernels(cudaStream_t stream);
  // Device milliseconds per replay of the kernel sequence (after one warm replay), CUDA events on
  // `stream`; whatever the input buffers hold (timing only).
  double time_kernels(cudaStream_t stream, int iters);
  // Enqueues only the D2H copies of the device outputs (host_out[j] as in enqueue).
  void enqueue_outputs(cudaStream_t stream, const std::vector<void*>& host_out);
  // Checks and clears the device error word written by bounded waits.
  void check_device_error();
  // Times every launch of the sequence on its own (`iters` repetitions each, CUDA events on
  // `stream`); returns (kind, milliseconds per launch) in launch order.
  std::vector<std::pair<std::string, double>> profile(cudaStream_t stream, int iters);

  const std::vector<OutputBinding>& outputs() const { return outputs_; }
  const std::vector<InputBinding>& inputs() const { return inputs_; }
  const PlanStats& stats() const { return stats_; }
  int device() const { return device_; }
  void* buffer_ptr(int buf) const;
  // Device address of output j (f32 contiguous; device outputs only).
  void* output_ptr(size_t j) const { return ptr(outputs_[j].dev); }

 private:
  struct Buffer {
    size_t bytes = 0;
    int first = 1 << 30, last = -1;
    size_t offset = 0;
  };
  struct PendingStep {
    std::string kind;
    std::function<std::function<cudaError_t(cudaStream_t)>()> build;   // run after allocation
    std::vector<DevTensor> reads, writes;
  };

  LGraph g_;
  int device_;
  int num_sms_;
  std::vector<DevTensor> vt_;       // per value id
  std::vector<Buffer> bufs_;
  std::vector<PendingStep> pending_;
  std::vector<std::function<cudaError_t(cudaStream_t)>> steps_;
  std::vector<std::string> kinds_;
  std::vector<uint8_t> wblob_;      // host staging of the weights blob
  std::vector<InputBinding> inputs_;
  std::vector<OutputBinding> outputs_;
  PlanStats stats_;
  void* arena_ = nullptr;
  void* weights_ = nullptr;
  unsigned int* err_ = nullptr;
  cudaGraph_t graph_ = nullptr;
  cudaGraphExec_t exec_ = nullptr;
  std::vector<std::vector<int>> consumers_;
  std::vector<bool> is_output_;
  std::map<std::pair<int, int>, DevTensor> conv_cache_;   // (value, 4 Cp + prec) -> NHWC operand copy
  std::map<std::pair<int, int>, DevTensor> rows_cache_;   // (value, prec) -> rows operand copy
  std::map<int, DevTensor> concat_out_;                    // Concat output value -> its buffer, when
                                                           // producers write their slices in place

  void build();
  void allocate_and_finalize();
  int new_buffer(size_t bytes);
  DevTensor alloc_contig(const std::vector<int64_t>& shape, bool bf16);
  DevTensor alloc_nhwc(const std::vector<int64_t>& shape_nchw, bool bf16, int64_t cstride);
  int64_t add_operand_weights(const std::vector<float>& w, int64_t rows, int64_t* lo_row, int prec);
  int64_t add_weight_bytes(const void* data, size_t bytes);
  void* ptr(const DevTensor& t) const;
  void add_step(const std::string& kind, std::vector<DevTensor> reads, std::vector<DevTensor> writes,
                std::function<std::function<cudaError_t(cudaStream_t)>()> build);

  static constexpr int kStoreBf16 = 0, kStoreTf32 = 1, kStoreF32 = 2;
  int storage_class(int v, int pref) const;
  DevTensor as_nhwc_op(int v, int Cp, int prec);
  DevTensor as_rows_op(int v, int64_t M, int64_t K, int prec);
  DevTensor as_f32_contig(int v);
  DevTensor materialize(const DevTensor& src, bool bf16);
  DevTensor concat_home(int v, int64_t Cout);
  DevTensor s2d_input(int v);
  void find_stem_pools();
  void plan_stem_pool(const Op& conv, const Op& pool);
  std::map<int, int> stem_pool_;      // stem conv op -> the MaxPool op it absorbs (fused kernel)
  std::set<int> pooled_by_conv_;      // MaxPool ops done by a fused stem kernel

  void plan_conv(const Op& op);
  void plan_gemm(const Op& op);
  void plan_maxpool(const Op& op);
  void plan_global_pool(const Op& op);
  void plan_group_norm(const Op& op);
  void plan_layer_norm(const Op& op);
  void add_split_reduce(const DevTensor& ws, int ksplit, int64_t Mp, int64_t M, int64_t Cout, const DevTensor& bias,
                        const DevTensor& res, int64_t ldr, int act, const DevTensor& y, bool round_tf32);
  void plan_attention(const Op& op);
  void plan_elementwise(const Op& op);
  void plan_view(const Op& op);
  void plan_concat(const Op& op);
  void plan_softmax(const Op& op);
  void plan_reduce(const Op& op);
  void plan_pad(const Op& op);
  void plan_resize(const Op& op);
  void plan_avgpool(const Op& op);
};

}  // namespace sb
