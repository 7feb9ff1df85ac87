// Session runtime behind the C ABI: the native side of IShorokooInferenceSession
// (src/Shorokoo/Core/Inference/Abstractions/IShorokooInferenceSession.cs:3-13) and of the host
// tensor values of IShorokooTensorValue (IShorokooTensorValue.cs:8-31).
#pragma once

#include <atomic>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "ir.h"
#include "plan.h"

namespace sb {

// Host value: tensor (any byte-stride element type), string tensor, or sequence of values.
struct HostValue {
  enum Kind { TENSOR = 1, SEQUENCE = 2 };   // ShorokooOnnxValueType numbering
  int kind = TENSOR;
  int32_t elem_type = DT_FLOAT;
  std::vector<int64_t> shape;
  // tensor bytes
  void* data = nullptr;
  size_t nbytes = 0;
  bool owned = true;       // false: borrowed caller memory
  bool pinned = false;
  // Device-resident tensor (an output of a run that kept its outputs on the device): `dev` holds
  // the nbytes on device `dev_id`; `data` stays null until host_data() copies them to the host.
  void* dev = nullptr;
  int dev_id = -1;
  std::mutex host_mu;
  void* host_data();       // data, copying a device-resident tensor to host memory on first use
  std::vector<std::string> strings;
  std::vector<std::shared_ptr<HostValue>> items;   // sequence elements
  ~HostValue();
  // pin: page-locked even below the pool's size threshold (outputs of a pipelined Run, whose
  // per-chunk device->host copies must not block the host)
  static std::shared_ptr<HostValue> alloc_tensor(int32_t elem_type, const std::vector<int64_t>& shape,
                                                 bool pin = false);
};

struct SessionOptions {
  int num_devices = 0;   // 0: SHOROKOO_B200_DEVICES or all visible devices
  int first_device = 0;
  int precision = -1;    // -1: SHOROKOO_B200_PRECISION (bf16 | tf32 | tf32x3, default bf16); 0, 1, 2
};

class Session {
 public:
  Session(const uint8_t* model, size_t len, const SessionOptions& opt);
  ~Session();

  const std::vector<std::string>& input_names() const { return info_.input_names; }
  const std::vector<std::string>& output_names() const { return info_.output_names; }

  // Run with inputs in session input order; returns outputs in the order of `out_idx`. With
  // keep_on_device the device outputs stay in device memory (no device->host copy); inputs that are
  // device-resident are copied device to device.
  std::vector<std::shared_ptr<HostValue>> run(const std::vector<std::shared_ptr<HostValue>>& inputs,
                                              const std::vector<int>& out_idx, bool keep_on_device = false);
  // Device-only timing: uploads inputs once and times `iters` replays of the kernel sequence on
  // every device; returns per-device milliseconds per run (CUDA events on each device's stream).
  std::vector<double> time_device(const std::vector<std::shared_ptr<HostValue>>& inputs, int warmup, int iters);
  // Times each launch of device 0's plan individually (no graph); returns (kind, ms) pairs.
  std::vector<std::pair<std::string, double>> profile_steps(const std::vector<std::shared_ptr<HostValue>>& inputs,
                                                            int iters);
  PlanStats stats(const std::vector<std::shared_ptr<HostValue>>& inputs);
  // Bytes a run() of these inputs moves host->device and device->host (float32 inputs staged as
  // bfloat16 count as such).
  std::pair<int64_t, int64_t> transfer_bytes(const std::vector<std::shared_ptr<HostValue>>& inputs);
  int devices_used(const std::vector<std::shared_ptr<HostValue>>& inputs);

 private:
  struct Shard {
    int device;
    int64_t begin, count;   // batch rows
    std::shared_ptr<Plan> plan;
  };
  // Micro-batch pipeline of one shard for run() (every shard has its own, on its own device): the
  // shard's rows are cut into small head chunks and larger body chunks (rows), each running
  // through a plan built for its size. Chunk c is copied host->device on the copy stream into
  // staging slot c % 2 while chunk c-1 computes; the compute stream then moves it into the plan's
  // input buffers (device->device), runs the kernels and copies the chunk's outputs back. The small
  // head keeps the one copy that nothing overlaps short. A one-chunk pipeline (rows = {shard rows},
  // the shard's own plan) is what a run with inputs in pageable memory takes when cutting does not
  // pay: it still stages them through page-locked memory (and narrows float32 read as bf16).
  struct Pipeline {
    int device = 0;                            // CUDA device ordinal
    unsigned host_threads = 16;                // threads of the host staging copies
    std::vector<int64_t> rows;                 // chunk sizes, in batch order
    std::vector<std::shared_ptr<Plan>> plans;  // plan of each chunk (chunks of one size share it)
    std::vector<void*> staging[2];                // per plan input binding
    cudaEvent_t h2d_done[2] = {nullptr, nullptr};  // staging slot filled
    cudaEvent_t consumed[2] = {nullptr, nullptr};  // staging slot read by the compute stream
    cudaStream_t copy = nullptr;
    // outputs: the compute stream copies chunk c's outputs into slot c mod 2 (per output, sized for
    // the largest chunk); the d2h stream copies the slot to the host while later chunks compute
    std::vector<void*> out_staging[2];
    cudaEvent_t out_ready[2] = {nullptr, nullptr};   // slot filled by the compute stream
    cudaEvent_t out_free[2] = {nullptr, nullptr};    // slot copied to the host
    cudaStream_t d2h = nullptr;
    // Inputs in borrowed pageable memory (sb_value_wrap_tensor over a caller's array, the way the
    // reference's CreateTensor<T> aliases a managed array) go through page-locked host slots: the
    // host copies chunk c into slot c % 2 while chunk c - 1 is still being transferred, so the
    // transfer stays asynchronous (a transfer straight from pageable memory blocks the host).
    std::vector<void*> host_staging[2];             // per plan input binding (allocated on first use)
    std::vector<size_t> host_staging_bytes;
    ~Pipeline();
  };
  struct PlanSet {
    std::vector<Shard> shards;
    std::vector<std::vector<int64_t>> out_shapes;
    std::vector<bool> out_host;
    std::vector<std::shared_ptr<HostTensor>> out_values;
    bool sharded = false;
    int64_t batch = -1;        // common leading dimension of the device inputs (-1 none, -2 mixed)
    bool separable = false;    // the graph treats batch rows independently
    bool pipe_checked[2] = {false, false};
    // one per shard, or none: [0] for inputs in page-locked (or device) memory, [1] for inputs in
    // pageable memory, whose host staging is a pipeline stage of its own
    std::vector<std::shared_ptr<Pipeline>> pipes[2];
  };

  OnnxModel model_;
  ModelInfo info_;
  SessionOptions opt_;
  int precision_ = 0;   // 0 bf16 operands, 1 TF32, 2 TF32x3 (the accuracy modes)
  std::vector<int> devices_;
  std::vector<int> sm_counts_;
  std::vector<cudaStream_t> streams_;
  std::mutex mu_;
  std::map<std::string, std::shared_ptr<PlanSet>> cache_;

  std::shared_ptr<PlanSet> get_plans(const std::vector<std::shared_ptr<HostValue>>& inputs);
  void maybe_build_pipeline(PlanSet& ps, const std::vector<std::shared_ptr<HostValue>>& inputs);
  std::shared_ptr<Pipeline> build_pipeline(PlanSet& ps, size_t si, const std::vector<std::shared_ptr<HostValue>>& inputs,
                                           bool may_cut, unsigned host_threads, bool pageable);
  // 1 when an input the plan copies lies in pageable host memory, else 0
  static int staging_mode(const std::vector<std::shared_ptr<HostValue>>& inputs);
  bool use_pipelines(const PlanSet& ps, const std::vector<std::shared_ptr<HostValue>>& inputs) const;
  void run_shards(PlanSet& ps, const std::vector<std::shared_ptr<HostValue>>& inputs,
                  const std::vector<std::shared_ptr<HostValue>>& outs);
  void run_pipelined(PlanSet& ps, int mode, size_t si, const std::vector<std::shared_ptr<HostValue>>& inputs,
                     const std::vector<std::shared_ptr<HostValue>>& outs);
  std::vector<InputSpec> specs_for(const std::vector<std::shared_ptr<HostValue>>& inputs, int64_t batch_begin,
                                   int64_t batch_count, bool shard) const;
};

bool batch_separable(const LGraph& g);
// SB_PRECISION_DEFAULT (-1) -> SHOROKOO_B200_PRECISION (bf16 | tf32 | tf32x3, default bf16);
// 0 bf16; 1 tf32; 2 tf32x3.
int resolve_precision(int requested);

}  // namespace sb
