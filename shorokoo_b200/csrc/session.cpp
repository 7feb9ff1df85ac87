// Session: model parsing at creation (unsupported operators are a hard error here, as the
// reference's CreateSession contract requires), a plan cache keyed by input shapes and plan-time
// input values, and batch sharding across devices with replicated weights and no collective.
#include "session.h"

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <set>
#include <thread>

#include <immintrin.h>

namespace sb {

int debug_level() {
  static int lvl = [] {
    const char* e = std::getenv("SHOROKOO_B200_DEBUG");
    return e ? std::atoi(e) : 0;
  }();
  return lvl;
}

namespace {

inline void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    if (e == cudaErrorMemoryAllocation) fail(SB_OUT_OF_MEMORY, std::string(what) + ": " + cudaGetErrorString(e));
    fail(SB_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

// ---- host memory: pinned (page-locked) when a CUDA device exists, pooled for reuse ------------
constexpr size_t kPinnedMin = size_t(1) << 20;
constexpr size_t kPoolMaxBytes = size_t(16) << 30;

struct HostPool {
  std::mutex mu;
  std::multimap<size_t, void*> free_blocks;
  size_t pooled = 0;
  int cuda_ok = -1;

  bool have_cuda() {
    if (cuda_ok < 0) {
      int n = 0;
      cuda_ok = (cudaGetDeviceCount(&n) == cudaSuccess && n > 0) ? 1 : 0;
      cudaGetLastError();
    }
    return cuda_ok == 1;
  }

  void* alloc(size_t bytes, bool& pinned, bool force_pin = false) {
    pinned = false;
    if (bytes >= kPinnedMin || force_pin) {
      size_t sz = (bytes + kPinnedMin - 1) / kPinnedMin * kPinnedMin;
      {
        std::lock_guard<std::mutex> l(mu);
        auto it = free_blocks.lower_bound(sz);
        if (it != free_blocks.end() && it->first <= sz + sz / 4) {
          void* p = it->second;
          pooled -= it->first;
          free_blocks.erase(it);
          pinned = true;
          return p;
        }
      }
      if (have_cuda()) {
        void* p = nullptr;
        if (cudaHostAlloc(&p, sz, cudaHostAllocPortable) == cudaSuccess) {
          pinned = true;
          return p;
        }
        cudaGetLastError();
      }
    }
    void* p = std::aligned_alloc(64, std::max<size_t>((bytes + 63) / 64 * 64, 64));
    SB_CHECK(p != nullptr, SB_OUT_OF_MEMORY, "host allocation failed");
    return p;
  }

  void release(void* p, size_t bytes, bool pinned) {
    if (!p) return;
    if (!pinned) {
      std::free(p);
      return;
    }
    size_t sz = (bytes + kPinnedMin - 1) / kPinnedMin * kPinnedMin;
    std::lock_guard<std::mutex> l(mu);
    if (pooled + sz <= kPoolMaxBytes) {
      free_blocks.emplace(sz, p);
      pooled += sz;
    } else {
      cudaFreeHost(p);
    }
  }
};

HostPool& pool() {
  static HostPool* p = new HostPool();   // intentionally leaked: outlives static destructors
  return *p;
}

// Parallel memcpy for large host copies: one piece of at least 4 MiB per thread, up to 16 threads
// (one thread copies at ~14 GB/s on the B200 host; the staging copies of a pipelined Run, running
// beside host->device transfers, measured 34 GB/s with 8 threads and 45 GB/s with 16).
void par_memcpy(void* dst, const void* src, size_t n, unsigned max_threads = 16) {
  const size_t piece = size_t(4) << 20;
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const unsigned nt = unsigned(std::min<size_t>(std::min(std::max(1u, max_threads), hw), n / piece));
  if (nt <= 1) {
    std::memcpy(dst, src, n);
    return;
  }
  std::vector<std::thread> th;
  const size_t per = (n / nt + 63) / 64 * 64;
  for (unsigned i = 1; i < nt; ++i) {
    const size_t b = i * per, e = std::min(n, b + per);
    if (b >= e) break;
    th.emplace_back([=] { std::memcpy(static_cast<uint8_t*>(dst) + b, static_cast<const uint8_t*>(src) + b, e - b); });
  }
  std::memcpy(dst, src, std::min(n, per));
  for (auto& t : th) t.join();
}

// float32 -> bfloat16 (round to nearest even; NaN stays NaN, quieted), n elements: the rounding the
// device applies when it reads a float32 operand as bfloat16, so narrowing on the host is exact.
void f32_to_bf16_scalar(uint16_t* __restrict__ dst, const float* __restrict__ src, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    uint32_t u;
    std::memcpy(&u, src + i, 4);
    const bool nan = (u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu);
    const uint32_t r = u + 0x7FFFu + ((u >> 16) & 1u);
    dst[i] = uint16_t(nan ? (u >> 16) | 0x40u : r >> 16);
  }
}

// The same, 16 elements per step with AVX2, written with non-temporal stores: the destination is a
// page-locked staging slot the copy engine reads next, so its lines are not read for ownership or
// kept in the host caches (the narrowing of a 308 MB batch is bound by host memory traffic).
__attribute__((target("avx2"))) inline __m256i bf16_round8(__m256i u) {
  const __m256i r = _mm256_srli_epi32(_mm256_add_epi32(_mm256_add_epi32(u, _mm256_set1_epi32(0x7FFF)),
                                                       _mm256_and_si256(_mm256_srli_epi32(u, 16), _mm256_set1_epi32(1))),
                                      16);
  const __m256i nan = _mm256_cmpgt_epi32(_mm256_and_si256(u, _mm256_set1_epi32(0x7FFFFFFF)), _mm256_set1_epi32(0x7F800000));
  return _mm256_blendv_epi8(r, _mm256_or_si256(_mm256_srli_epi32(u, 16), _mm256_set1_epi32(0x40)), nan);
}

__attribute__((target("avx2"))) void f32_to_bf16_avx2(uint16_t* __restrict__ dst, const float* __restrict__ src,
                                                       size_t n) {
  size_t i = 0;
  while (i < n && (reinterpret_cast<uintptr_t>(dst + i) & 31u)) {   // to a 32-byte destination boundary
    f32_to_bf16_scalar(dst + i, src + i, 1);
    ++i;
  }
  for (; i + 16 <= n; i += 16) {
    const __m256i a = bf16_round8(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i)));
    const __m256i b = bf16_round8(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i + 8)));
    // packus interleaves the 128-bit halves: a0-3 b0-3 a4-7 b4-7 -> a0-7 b0-7
    const __m256i p = _mm256_permute4x64_epi64(_mm256_packus_epi32(a, b), 0xD8);
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i), p);
  }
  _mm_sfence();
  if (i < n) f32_to_bf16_scalar(dst + i, src + i, n - i);
}

void f32_to_bf16_span(uint16_t* dst, const float* src, size_t n) {
  static const bool avx2 = __builtin_cpu_supports("avx2");
  if (avx2)
    f32_to_bf16_avx2(dst, src, n);
  else
    f32_to_bf16_scalar(dst, src, n);
}

// The same over up to max_threads threads (pieces of at least 1 Mi elements).
void par_f32_to_bf16(uint16_t* dst, const float* src, size_t n, unsigned max_threads = 16) {
  const size_t piece = size_t(1) << 20;
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const unsigned nt =
      unsigned(std::max<size_t>(1, std::min<size_t>(std::min(std::max(1u, max_threads), hw), n / piece)));
  const size_t per = (n / nt + 63) / 64 * 64;
  std::vector<std::thread> th;
  for (unsigned i = 1; i < nt; ++i) {
    const size_t b = i * per, e = std::min(n, b + per);
    if (b >= e) break;
    th.emplace_back([=] { f32_to_bf16_span(dst + b, src + b, e - b); });
  }
  f32_to_bf16_span(dst, src, std::min(n, per));
  for (auto& t : th) t.join();
}

}  // namespace

void* host_alloc(size_t bytes, bool& pinned) { return pool().alloc(bytes, pinned); }
void host_release(void* p, size_t bytes, bool pinned) { pool().release(p, bytes, pinned); }
void host_copy(void* dst, const void* src, size_t n) { par_memcpy(dst, src, n); }
void host_narrow_bf16(uint16_t* dst, const float* src, size_t n, unsigned threads) {
  par_f32_to_bf16(dst, src, n, threads);
}
// True when p lies in page-locked host memory the CUDA runtime knows (cudaHostAlloc'd or
// cudaHostRegister'ed), so a device transfer from it is asynchronous.
bool host_is_page_locked(const void* p) {
  if (!p || !pool().have_cuda()) return false;
  cudaPointerAttributes at;
  const bool ok = cudaPointerGetAttributes(&at, p) == cudaSuccess && at.type == cudaMemoryTypeHost;
  cudaGetLastError();
  return ok;
}

HostValue::~HostValue() {
  if (owned && data) pool().release(data, nbytes, pinned);
  if (dev) {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(dev_id);
    cudaFree(dev);
    if (prev >= 0) cudaSetDevice(prev);
  }
}

void* HostValue::host_data() {
  if (!dev || data || !nbytes) return data;
  std::lock_guard<std::mutex> l(host_mu);
  if (!data) {
    bool pin = false;
    void* h = pool().alloc(nbytes, pin);
    cudaError_t e = cudaMemcpy(h, dev, nbytes, cudaMemcpyDefault);
    if (e != cudaSuccess) {
      pool().release(h, nbytes, pin);
      fail(SB_CUDA_ERROR, std::string("copy of a device-resident value to the host: ") + cudaGetErrorString(e));
    }
    pinned = pin;
    owned = true;
    data = h;
  }
  return data;
}

std::shared_ptr<HostValue> HostValue::alloc_tensor(int32_t elem_type, const std::vector<int64_t>& shape, bool pin) {
  auto v = std::make_shared<HostValue>();
  v->kind = TENSOR;
  v->elem_type = elem_type;
  v->shape = shape;
  v->nbytes = size_t(numel(shape)) * dtype_size(elem_type);
  bool pinned = false;
  v->data = pool().alloc(std::max<size_t>(v->nbytes, 1), pinned, pin);
  v->pinned = pinned;
  v->owned = true;
  return v;
}

// ---- batch separability --------------------------------------------------------------------
// Every device value gets the axis that carries the batch (-1: no batch dependence, -2: mixed).
// A graph shards cleanly when every op keeps samples independent and every output carries the
// batch on axis 0.
bool batch_separable(const LGraph& g) {
  std::vector<int> ax(g.vals.size(), -1);
  for (int id : g.inputs) {
    const Value& v = g.vals[size_t(id)];
    if (!v.is_host) {
      if (v.shape.empty()) return false;
      ax[size_t(id)] = 0;
    }
  }
  auto host_ok = [&](int id, int axis, size_t out_rank) {
    // a plan-time constant must not vary along the batch axis of the output
    const Value& v = g.vals[size_t(id)];
    if (axis < 0) return true;
    size_t off = out_rank - v.shape.size();
    if (size_t(axis) < off) return true;
    return v.shape[size_t(axis) - off] == 1;
  };
  for (const Op& op : g.ops) {
    if (op.dead) continue;
    const Value& y = g.vals[size_t(op.out[0])];
    int a0 = op.in.empty() || op.in[0] < 0 ? -1 : ax[size_t(op.in[0])];
    if (a0 == -2) return false;
    int out = -2;
    const std::string& t = op.type;
    if (t == "FusedConv" || t == "MaxPool" || t == "GlobalAveragePool" || t == "GlobalMaxPool" ||
        t == "AveragePool" || t == "GroupNorm") {
      if (a0 != 0) return false;
      if (op.residual >= 0 && ax[size_t(op.residual)] != 0) return false;
      if (op.concat >= 0 && ax[size_t(op.concat)] != 0) return false;
      out = 0;
    } else if (t == "FusedGemm") {
      if (a0 != 0 || g.vals[size_t(op.in[0])].shape.size() < 2) return false;
      if (op.residual >= 0 && ax[size_t(op.residual)] != 0) return false;
      out = 0;
    } else if (t == "LayerNorm") {   // per row over the last axis
      if (a0 != 0 || g.vals[size_t(op.in[0])].shape.size() < 2) return false;
      out = 0;
    } else if (t == "Attention") {   // per (batch, head): q, k and v sharded alike
      for (int id : op.in)
        if (ax[size_t(id)] != 0) return false;
      out = 0;
    } else if (t == "Identity") {
      out = a0;
    } else if (t == "Transpose") {
      out = -1;
      for (size_t i = 0; i < op.perm.size(); ++i)
        if (op.perm[i] == a0) out = int(i);
      if (a0 >= 0 && out < 0) return false;
    } else if (t == "Reshape") {
      const auto& xs = g.vals[size_t(op.in[0])].shape;
      if (a0 < 0) out = -1;
      else if (a0 == 0 && !y.shape.empty() && y.shape[0] == xs[0]) out = 0;
      else return false;
    } else if (t == "Slice") {
      if (a0 >= 0 && (op.axes[size_t(a0)] != 0 || op.strides[size_t(a0)] != 1 ||
                      y.shape[size_t(a0)] != g.vals[size_t(op.in[0])].shape[size_t(a0)]))
        return false;
      out = a0;
    } else if (t == "Expand") {
      out = a0 >= 0 ? a0 + int(y.shape.size() - g.vals[size_t(op.in[0])].shape.size()) : -1;
    } else if (t == "Concat" || t == "Softmax") {
      out = -1;
      for (int id : op.in) {
        if (id < 0) continue;
        int ai = ax[size_t(id)];
        if (ai == -2) return false;
        if (ai >= 0) {
          if (out >= 0 && out != ai) return false;
          out = ai;
        }
      }
      if (out >= 0 && out == int(op.axis)) return false;
      for (int id : op.in)
        if (id >= 0 && ax[size_t(id)] < 0 && out >= 0 && !g.vals[size_t(id)].is_host) return false;
    } else if (t == "Pad") {
      if (a0 >= 0 && (op.pads[size_t(a0)] != 0 || op.pads[size_t(a0) + y.shape.size()] != 0)) return false;
      out = a0;
    } else if (t == "Resize") {
      if (a0 >= 0 && op.scales[size_t(a0)] != 1.f) return false;
      out = a0;
    } else if (t == "ReduceMean" || t == "ReduceSum" || t == "ReduceMax") {
      if (a0 >= 0 && std::find(op.axes.begin(), op.axes.end(), a0) != op.axes.end()) return false;
      int removed = 0;
      if (!op.keepdims)
        for (auto a : op.axes)
          if (a < a0) ++removed;
      out = a0 >= 0 ? a0 - removed : -1;
    } else {
      // elementwise (broadcasting)
      out = -1;
      for (int id : op.in) {
        if (id < 0) continue;
        const Value& v = g.vals[size_t(id)];
        int ai = ax[size_t(id)];
        if (ai == -2) return false;
        if (ai >= 0) {
          int aligned = ai + int(y.shape.size() - v.shape.size());
          if (out >= 0 && out != aligned) return false;
          out = aligned;
        }
      }
      for (int id : op.in)
        if (id >= 0 && ax[size_t(id)] < 0 && !host_ok(id, out, y.shape.size())) return false;
    }
    for (int o : op.out) ax[size_t(o)] = out;
  }
  for (int id : g.outputs)
    if (g.vals[size_t(id)].is_host || ax[size_t(id)] != 0) return false;
  return true;
}

// ---- Session -------------------------------------------------------------------------------
Session::Session(const uint8_t* model, size_t len, const SessionOptions& opt) : opt_(opt) {
  model_ = parse_onnx(model, len);
  check_supported_ops(model_);
  info_ = model_info(model_);
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    fail(SB_CUDA_ERROR, "no CUDA device is available for the B200 backend");
  }
  precision_ = resolve_precision(opt.precision);
  int want = opt.num_devices;
  if (want <= 0) {
    const char* e = std::getenv("SHOROKOO_B200_DEVICES");
    want = e ? std::atoi(e) : count;
  }
  want = std::max(1, std::min(want, count - opt.first_device));
  SB_CHECK(opt.first_device >= 0 && opt.first_device < count, SB_INVALID_ARGUMENT, "first_device out of range");
  for (int d = 0; d < want; ++d) {
    const int dev = opt.first_device + d;
    cudaDeviceProp prop;
    ck(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
    SB_CHECK(prop.major == 10 && prop.minor == 0, SB_UNSUPPORTED,
             std::string("device ") + std::to_string(dev) + " (" + prop.name +
                 ") is not sm_100; this backend ships sm_100a kernels only");
    devices_.push_back(dev);
    sm_counts_.push_back(prop.multiProcessorCount);
    ck(cudaSetDevice(dev), "cudaSetDevice");
    cudaStream_t s;
    ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
    streams_.push_back(s);
  }
}

int resolve_precision(int requested) {
  if (requested >= 0) return requested;
  const char* e = std::getenv("SHOROKOO_B200_PRECISION");
  const std::string v = e ? e : "bf16";
  SB_CHECK(v == "bf16" || v == "tf32" || v == "tf32x3", SB_INVALID_ARGUMENT,
           "SHOROKOO_B200_PRECISION must be bf16, tf32 or tf32x3");
  return v == "tf32" ? 1 : (v == "tf32x3" ? 2 : 0);
}

Session::~Session() {
  cache_.clear();
  for (size_t i = 0; i < streams_.size(); ++i) {
    cudaSetDevice(devices_[i]);
    cudaStreamDestroy(streams_[i]);
  }
}

std::vector<InputSpec> Session::specs_for(const std::vector<std::shared_ptr<HostValue>>& inputs, int64_t b0,
                                          int64_t cnt, bool shard) const {
  std::vector<InputSpec> specs;
  for (size_t i = 0; i < inputs.size(); ++i) {
    const HostValue& v = *inputs[i];
    InputSpec s;
    s.dtype = v.elem_type;
    s.shape = v.shape;
    if (numel(v.shape) <= kPlanTimeInputMaxElems) {
      auto h = std::make_shared<HostTensor>(v.elem_type, v.shape);
      if (v.nbytes) std::memcpy(h->mutable_data(), const_cast<HostValue&>(v).host_data(), v.nbytes);
      s.value = h;
    } else if (shard) {
      s.shape[0] = cnt;
      (void)b0;
    }
    specs.push_back(std::move(s));
  }
  return specs;
}

std::shared_ptr<Session::PlanSet> Session::get_plans(const std::vector<std::shared_ptr<HostValue>>& inputs) {
  SB_CHECK(inputs.size() == info_.input_names.size(), SB_INVALID_ARGUMENT,
           "expected " + std::to_string(info_.input_names.size()) + " inputs, got " + std::to_string(inputs.size()));
  std::string key;
  for (size_t i = 0; i < inputs.size(); ++i) {
    const HostValue& v = *inputs[i];
    SB_CHECK(v.kind == HostValue::TENSOR, SB_UNSUPPORTED, "input '" + info_.input_names[i] + "': sequences are not supported");
    SB_CHECK(v.elem_type != DT_STRING, SB_UNSUPPORTED, "input '" + info_.input_names[i] + "': string tensors are not supported");
    if (info_.input_dtypes[i] != DT_UNDEFINED)
      SB_CHECK(v.elem_type == info_.input_dtypes[i], SB_INVALID_ARGUMENT,
               "input '" + info_.input_names[i] + "' expects " + dtype_name(info_.input_dtypes[i]) + ", got " +
                   dtype_name(v.elem_type));
    if (info_.input_ranks[i] >= 0)
      SB_CHECK(int(v.shape.size()) == info_.input_ranks[i], SB_INVALID_ARGUMENT,
               "input '" + info_.input_names[i] + "' expects rank " + std::to_string(info_.input_ranks[i]) +
                   ", got " + shape_str(v.shape));
    key += std::to_string(v.elem_type) + shape_str(v.shape);
    if (numel(v.shape) <= kPlanTimeInputMaxElems)
      key += "=" + std::string(static_cast<const char*>(const_cast<HostValue&>(v).host_data()), v.nbytes);
    key += ";";
  }
  auto it = cache_.find(key);
  if (it != cache_.end()) return it->second;

  auto ps = std::make_shared<PlanSet>();
  LGraph full = lower(model_, specs_for(inputs, 0, 0, false));
  fuse(full);
  for (size_t j = 0; j < full.outputs.size(); ++j) {
    const Value& v = full.vals[size_t(full.outputs[j])];
    ps->out_shapes.push_back(v.shape);
    ps->out_host.push_back(v.is_host);
    ps->out_values.push_back(v.is_host ? v.host : nullptr);
  }
  int64_t batch = -1;
  for (size_t i = 0; i < inputs.size(); ++i)
    if (numel(inputs[i]->shape) > kPlanTimeInputMaxElems) {
      if (batch < 0) batch = inputs[i]->shape[0];
      else if (inputs[i]->shape[0] != batch) batch = -2;
    }
  const int nd = int(devices_.size());
  ps->batch = batch;
  ps->separable = batch >= 2 && batch_separable(full);
  bool shard = nd > 1 && ps->separable;
  if (nd > 1 && !shard && debug_level() >= 1)
    std::fprintf(stderr, "[shorokoo_b200] graph does not shard on the batch axis; running on one device\n");
  if (!shard) {
    ck(cudaSetDevice(devices_[0]), "cudaSetDevice");
    ps->shards.push_back({0, 0, batch > 0 ? batch : 0, std::make_shared<Plan>(std::move(full), devices_[0], sm_counts_[0], precision_)});
  } else {
    ps->sharded = true;
    const int parts = int(std::min<int64_t>(nd, batch));
    int64_t b0 = 0;
    for (int d = 0; d < parts; ++d) {
      int64_t cnt = batch / parts + (d < batch % parts ? 1 : 0);
      ps->shards.push_back({d, b0, cnt, nullptr});
      b0 += cnt;
    }
    std::vector<std::thread> th;
    std::vector<std::string> errs(ps->shards.size());
    std::vector<int32_t> codes(ps->shards.size(), 0);
    for (size_t si = 0; si < ps->shards.size(); ++si) {
      th.emplace_back([&, si] {
        Shard& sh = ps->shards[si];
        try {
          cudaSetDevice(devices_[size_t(sh.device)]);
          LGraph g = lower(model_, specs_for(inputs, sh.begin, sh.count, true));
          sh.plan = std::make_shared<Plan>(std::move(g), devices_[size_t(sh.device)], sm_counts_[size_t(sh.device)], precision_);
        } catch (const Error& e) {
          errs[si] = e.what();
          codes[si] = e.code;
        } catch (const std::exception& e) {
          errs[si] = e.what();
          codes[si] = SB_INTERNAL;
        }
      });
    }
    for (auto& t : th) t.join();
    for (size_t si = 0; si < errs.size(); ++si)
      if (codes[si]) fail(codes[si], "device " + std::to_string(devices_[size_t(ps->shards[si].device)]) + ": " + errs[si]);
  }
  cache_[key] = ps;
  return ps;
}

// Milliseconds per byte of a host->device copy from page-locked memory, measured once per device
// (one 64 MiB transfer on stream s).
static double copy_ms_per_byte(cudaStream_t s) {
  static std::mutex mu;
  static std::map<int, double> cache;
  int dev = 0;
  ck(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> l(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  const size_t n = size_t(64) << 20;
  void* h = nullptr;
  void* d = nullptr;
  ck(cudaHostAlloc(&h, n, cudaHostAllocPortable), "cudaHostAlloc");
  cudaError_t e = cudaMalloc(&d, n);
  double r = 1.0 / 50e6;   // 50 GB/s if the measurement cannot run
  if (e == cudaSuccess) {
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaMemcpyAsync(d, h, n, cudaMemcpyHostToDevice, s);   // warm
    cudaEventRecord(e0, s);
    cudaMemcpyAsync(d, h, n, cudaMemcpyHostToDevice, s);
    cudaEventRecord(e1, s);
    if (cudaEventSynchronize(e1) == cudaSuccess) {
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      if (ms > 0) r = double(ms) / double(n);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(d);
  }
  cudaGetLastError();
  cudaFreeHost(h);
  cache[dev] = r;
  return r;
}

Session::Pipeline::~Pipeline() {
  cudaSetDevice(device);
  for (auto& slot : host_staging)
    for (void* p : slot)
      if (p) cudaFreeHost(p);
  for (auto& slot : staging)
    for (void* p : slot) cudaFree(p);
  for (auto& slot : out_staging)
    for (void* p : slot) cudaFree(p);
  for (int i = 0; i < 2; ++i) {
    if (h2d_done[i]) cudaEventDestroy(h2d_done[i]);
    if (consumed[i]) cudaEventDestroy(consumed[i]);
    if (out_ready[i]) cudaEventDestroy(out_ready[i]);
    if (out_free[i]) cudaEventDestroy(out_free[i]);
  }
  if (copy) cudaStreamDestroy(copy);
  if (d2h) cudaStreamDestroy(d2h);
}

// Host threads for the staging copies of one session: SHOROKOO_B200_HOST_THREADS, else 16 (the
// narrowing of a large batch saturates the host's memory bandwidth at about 16). Processes that share
// the host (one per GPU) divide them.
static unsigned host_staging_threads() {
  static const unsigned n = [] {
    if (const char* e = std::getenv("SHOROKOO_B200_HOST_THREADS")) {
      const int v = std::atoi(e);
      if (v >= 1 && v <= 256) return unsigned(v);
    }
    return 16u;
  }();
  return n;
}

int Session::staging_mode(const std::vector<std::shared_ptr<HostValue>>& inputs) {
  for (const auto& v : inputs)
    if (numel(v->shape) > kPlanTimeInputMaxElems && !v->pinned && !v->dev) return 1;
  return 0;
}

// Milliseconds per source byte of the host staging of a pageable input into a page-locked slot
// (narrowed float32 -> bfloat16, or copied), on `threads` host threads; measured once per process.
static double host_stage_ms_per_byte(unsigned threads, bool narrow) {
  static std::mutex mu;
  static std::map<std::pair<unsigned, bool>, double> cache;
  std::lock_guard<std::mutex> l(mu);
  auto key = std::make_pair(threads, narrow);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  const size_t n = size_t(16) << 20;   // floats (64 MB)
  std::vector<float> src(n, 1.f);
  void* dst = nullptr;
  double r = 1.0 / 20e6;   // 20 GB/s if the measurement cannot run
  if (cudaHostAlloc(&dst, n * 4, cudaHostAllocPortable) == cudaSuccess) {
    double best = 1e30;
    for (int rep = 0; rep < 2; ++rep) {
      const auto t0 = std::chrono::steady_clock::now();
      if (narrow)
        par_f32_to_bf16(static_cast<uint16_t*>(dst), src.data(), n, threads);
      else
        par_memcpy(dst, src.data(), n * 4, threads);
      best = std::min(best, std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
    }
    r = best / double(n * 4);
    cudaFreeHost(dst);
  }
  cudaGetLastError();
  cache[key] = r;
  return r;
}

void Session::maybe_build_pipeline(PlanSet& ps, const std::vector<std::shared_ptr<HostValue>>& inputs) {
  const int mode = staging_mode(inputs);
  if (ps.pipe_checked[mode]) return;
  ps.pipe_checked[mode] = true;
  if (!ps.separable || ps.batch < 2) return;
  bool may_cut = true;
  if (const char* e = std::getenv("SHOROKOO_B200_PIPELINE"))
    if (e[0] == '0') may_cut = false;
  // Every shard builds its pipeline on its own device (in parallel, like the shards' plans); the
  // host staging copies of concurrent shards share the host's threads.
  const size_t n = ps.shards.size();
  const unsigned threads = std::max(2u, host_staging_threads() / unsigned(n));
  std::vector<std::shared_ptr<Pipeline>> pipes(n);
  if (n == 1) {
    pipes[0] = build_pipeline(ps, 0, inputs, may_cut, threads, mode == 1);
  } else {
    std::vector<std::thread> th;
    for (size_t si = 0; si < n; ++si)
      th.emplace_back([&, si] { pipes[si] = build_pipeline(ps, si, inputs, may_cut, threads, mode == 1); });
    for (auto& t : th) t.join();
  }
  for (const auto& p : pipes)
    if (!p) return;   // (a shard whose pipeline could not be set up: every shard runs unstaged)
  ps.pipes[mode] = std::move(pipes);
}

std::shared_ptr<Session::Pipeline> Session::build_pipeline(PlanSet& ps, size_t si,
                                                           const std::vector<std::shared_ptr<HostValue>>& inputs,
                                                           bool may_cut, unsigned host_threads, bool pageable) {
  const Shard& sh = ps.shards[si];
  const int64_t rows_total = ps.sharded ? sh.count : ps.batch;
  // Below kPipeMinBytes of copies (in + out) they are too short to be worth hiding (at 32 MiB the
  // 8192-row MLP gains 30% end to end, 2.22 -> 1.71 ms per run). Chunks: two head
  // chunks of an eighth of the rows, then two body chunks of the rest. The first chunk's copy is
  // the one nothing overlaps, so it is small; each chunk's compute must outlast the next chunk's
  // copy, so sizes grow. Measured for ResNet-50 bs512 on B200 (device ms at batch 32 / 64 / 160 /
  // 192: 1.01 / 1.38 / 2.68 / 3.02; PCIe 10.85 us per image): 64 + 64 + 192 + 192 models 9.6 ms
  // per run against 10.2 ms for the earlier 32 + 3 x 160.
  constexpr size_t kPipeMinBytes = size_t(32) << 20;
  // (input and output copies both overlap the chunks' kernels: outputs such as a detector's dense
  // per-anchor maps can outweigh the inputs)
  size_t in_bytes = 0, out_bytes = 0;
  for (const auto& v : inputs)
    if (numel(v->shape) > kPlanTimeInputMaxElems) in_bytes += v->nbytes;
  for (size_t j = 0; j < ps.out_shapes.size(); ++j)
    if (!ps.out_host[j]) out_bytes += size_t(numel(ps.out_shapes[j])) * 4;
  in_bytes = size_t(double(in_bytes) * double(rows_total) / double(ps.batch));   // this shard's share
  out_bytes = size_t(double(out_bytes) * double(rows_total) / double(ps.batch));
  auto P = std::make_shared<Pipeline>();
  P->device = devices_[size_t(sh.device)];
  P->host_threads = host_threads;
  const int64_t head = std::max<int64_t>(1, rows_total / 8);
  if (may_cut && in_bytes + out_bytes >= kPipeMinBytes && rows_total >= 8) {
    if (out_bytes > in_bytes) {
      // Output-bound (device->host copies outlast the kernels): once the first chunk's outputs start
      // copying back the copy stream should never wait, and the last chunk's copy is the one nothing
      // overlaps, so after two small chunks the rest goes in quarters (RetinaNet bs16: 2 + 2 + 4 +
      // 4 + 4 took 825 MB of outputs back in about the time of the copy alone).
      const int64_t quarter = std::max<int64_t>(1, rows_total / 4);
      const int64_t last = rows_total - 2 * head - 2 * quarter;
      if (last >= 1) P->rows = {head, head, quarter, quarter, last};
    } else {
      const int64_t body = (rows_total - 2 * head) / 2;
      if (body >= head && body >= 2) P->rows = {head, head, body, rows_total - 2 * head - body};
    }
  }
  cudaStream_t cs = streams_[size_t(sh.device)];
  try {
    ck(cudaSetDevice(P->device), "cudaSetDevice");
    ck(cudaStreamCreateWithFlags(&P->copy, cudaStreamNonBlocking), "cudaStreamCreate");
    ck(cudaStreamCreateWithFlags(&P->d2h, cudaStreamNonBlocking), "cudaStreamCreate");
    for (int slot = 0; slot < 2; ++slot) {
      ck(cudaEventCreateWithFlags(&P->h2d_done[slot], cudaEventDisableTiming), "event");
      ck(cudaEventCreateWithFlags(&P->consumed[slot], cudaEventDisableTiming), "event");
      ck(cudaEventCreateWithFlags(&P->out_ready[slot], cudaEventDisableTiming), "event");
      ck(cudaEventCreateWithFlags(&P->out_free[slot], cudaEventDisableTiming), "event");
    }
    if (!P->rows.empty()) {
      auto build = [&](int64_t n) {
        LGraph g = lower(model_, specs_for(inputs, 0, n, true));
        auto plan = std::make_shared<Plan>(std::move(g), P->device, sm_counts_[size_t(sh.device)], precision_);
        const auto& outs = plan->outputs();
        for (size_t j = 0; j < outs.size(); ++j)
          if (!outs[j].host && (outs[j].shape.empty() || outs[j].shape[0] != n || ps.out_shapes[j].empty() ||
                                ps.out_shapes[j][0] != ps.batch))
            return std::shared_ptr<Plan>();   // an output is not cut along the batch
        return plan;
      };
      std::vector<std::pair<int64_t, std::shared_ptr<Plan>>> built;   // one plan per distinct size
      for (int64_t n : P->rows) {
        std::shared_ptr<Plan> plan;
        for (const auto& kv : built)
          if (kv.first == n) plan = kv.second;
        if (!plan) {
          plan = build(n);
          if (!plan) break;
          built.emplace_back(n, plan);
        }
        P->plans.push_back(plan);
      }
      if (P->plans.size() != P->rows.size()) {
        P->rows.clear();
        P->plans.clear();
      }
    }
    if (!P->rows.empty()) {
      // Keep the cut only where it pays: small chunks leave SMs idle (a 64-image ResNet-50 batch
      // cut into 8 + 8 + 24 + 24 ran 2.70 ms end to end against 2.03 ms unpipelined), so the
      // schedule is simulated with measured chunk kernel times and the measured copy rate against
      // one copy in, the whole shard's kernels and one copy out.
      const double t_full = sh.plan->time_kernels(cs, 3);
      std::vector<double> t_chunk;
      for (size_t c = 0; c < P->rows.size(); ++c) {
        double t = -1;
        for (size_t c2 = 0; c2 < c; ++c2)
          if (P->plans[c2] == P->plans[c]) t = t_chunk[c2];
        t_chunk.push_back(t >= 0 ? t : P->plans[c]->time_kernels(cs, 3));
      }
      const double ms_per_byte = copy_ms_per_byte(P->copy);
      // Inputs in pageable memory are staged by the host first (narrowed to bf16 where the plan
      // reads them as bf16, halving the transfer): a pipeline stage of its own, so the host's pass
      // over chunk c overlaps the transfer and kernels of the chunks before it.
      double xfer_bytes = 0, host_ms = 0;
      for (const auto& b : sh.plan->inputs()) {
        const HostValue& v = *inputs[size_t(b.index)];
        const bool narrow = pageable && b.bf16_ok && v.elem_type == DT_FLOAT;
        xfer_bytes += narrow ? double(b.bytes) / 2 : double(b.bytes);
        if (pageable) host_ms += double(b.bytes) * host_stage_ms_per_byte(host_threads, narrow);
      }
      const double rows = double(rows_total);
      double host_end = 0, copy_end = 0, comp_end = 0, back_end = 0;
      std::vector<double> copy_ends, comp_ends;
      for (size_t c = 0; c < P->rows.size(); ++c) {
        const double share = double(P->rows[c]) / rows;
        // host slot c % 2 is free once chunk c - 2's transfer out of it is done
        host_end = std::max(host_end, c >= 2 ? copy_ends[c - 2] : 0.0) + share * host_ms;
        double start = std::max(copy_end, host_end);
        if (c >= 2) start = std::max(start, comp_ends[c - 2]);   // its device staging slot is free
        copy_end = start + share * xfer_bytes * ms_per_byte;
        copy_ends.push_back(copy_end);
        comp_end = std::max(comp_end, copy_end) + t_chunk[c];
        comp_ends.push_back(comp_end);
        back_end = std::max(back_end, comp_end) + share * double(out_bytes) * ms_per_byte;
      }
      const double t_seq = host_ms + (xfer_bytes + double(out_bytes)) * ms_per_byte + t_full;
      if (debug_level() >= 1)
        std::fprintf(stderr, "[shorokoo_b200] pipeline model: %.3f ms pipelined vs %.3f ms in one piece (device %d%s)\n",
                     back_end, t_seq, P->device, pageable ? ", pageable inputs" : "");
      if (back_end >= 0.97 * t_seq) {
        P->rows.clear();
        P->plans.clear();
      }
    }
    if (P->rows.empty()) {   // one chunk: the shard's own plan
      P->rows = {rows_total};
      P->plans = {sh.plan};
    }
    // device staging: per chunk slot and input binding (a one-chunk pipeline copies straight into
    // the plan's buffers and stages only inputs that may travel as bf16, at their bf16 size)
    const bool one = P->rows.size() == 1;
    size_t big = 0;   // the largest chunk: its plan's bindings size the staging slots
    for (size_t c = 1; c < P->rows.size(); ++c)
      if (P->rows[c] > P->rows[big]) big = c;
    for (int slot = 0; slot < (one ? 1 : 2); ++slot) {
      for (const auto& b : P->plans[big]->inputs()) {
        void* d = nullptr;
        const size_t bytes = one ? (b.bf16_ok ? b.bytes / 2 : 0) : b.bytes;
        if (bytes) ck(cudaMalloc(&d, std::max<size_t>(bytes, 16)), "cudaMalloc (pipeline staging)");
        P->staging[slot].push_back(d);
      }
      const auto& louts = P->plans[big]->outputs();
      for (size_t j = 0; j < louts.size(); ++j) {
        void* d = nullptr;
        if (!louts[j].host && !one)
          ck(cudaMalloc(&d, std::max<size_t>(size_t(numel(louts[j].shape)) * 4, 16)), "cudaMalloc (output staging)");
        P->out_staging[slot].push_back(d);
      }
    }
  } catch (const Error& e) {
    if (debug_level() >= 1) std::fprintf(stderr, "[shorokoo_b200] no micro-batch pipeline: %s\n", e.what());
    return nullptr;
  }
  if (debug_level() >= 1) {
    std::string sched;
    for (size_t c = 0; c < P->rows.size(); ++c) sched += (c ? " + " : "") + std::to_string(P->rows[c]);
    if (P->rows.size() > 1)
      std::fprintf(stderr, "[shorokoo_b200] run pipeline: %zu chunks of %s rows (device %d)\n", P->rows.size(),
                   sched.c_str(), P->device);
    else
      std::fprintf(stderr, "[shorokoo_b200] run staging: one piece of %s rows (device %d)\n", sched.c_str(), P->device);
  }
  return P;
}

// The pipelines run when they cut a shard into chunks, or when an input sits in pageable memory
// (staged through page-locked memory either way).
bool Session::use_pipelines(const PlanSet& ps, const std::vector<std::shared_ptr<HostValue>>& inputs) const {
  const int mode = staging_mode(inputs);
  if (ps.pipes[mode].empty()) return false;
  if (mode == 1) return true;   // pageable inputs: always staged
  for (const auto& p : ps.pipes[mode])
    if (p->rows.size() > 1) return true;
  return false;
}

void Session::run_pipelined(PlanSet& ps, int mode, size_t si, const std::vector<std::shared_ptr<HostValue>>& inputs,
                            const std::vector<std::shared_ptr<HostValue>>& outs) {
  Pipeline& P = *ps.pipes[mode][si];
  const Shard& sh = ps.shards[si];
  ck(cudaSetDevice(P.device), "cudaSetDevice");
  cudaStream_t cs = streams_[size_t(sh.device)];
  const bool one = P.rows.size() == 1;
  using clk = std::chrono::steady_clock;
  const auto t_run = clk::now();
  double ms_copy = 0, ms_wait = 0;   // host time in staging copies / waiting for staging slots
  std::vector<void*> hout(outs.size(), nullptr);
  int64_t r0 = ps.sharded ? sh.begin : 0;   // first batch row of the chunk
  for (size_t c = 0; c < P.rows.size(); r0 += P.rows[c], ++c) {
    Plan& plan = *P.plans[c];
    const auto& binds = plan.inputs();
    const int slot = int(c & 1);
    if (c >= 2) ck(cudaStreamWaitEvent(P.copy, P.consumed[slot], 0), "stream wait");
    bool host_slot_free = c < 2;
    std::vector<bool> narrowed(binds.size(), false);
    for (size_t bi = 0; bi < binds.size(); ++bi) {
      const HostValue& v = *inputs[size_t(binds[bi].index)];
      const size_t row = v.nbytes / size_t(std::max<int64_t>(v.shape[0], 1));
      const uint8_t* src = static_cast<const uint8_t*>(v.data) + size_t(r0) * row;
      // A float32 input read only as bfloat16 by the plan travels as bfloat16 when it has to be staged
      // anyway (half the transfer; widened back on the device, where the plan rounds it to bfloat16
      // again: the same values).
      const bool narrow = !v.pinned && binds[bi].bf16_ok && v.elem_type == DT_FLOAT;
      narrowed[bi] = narrow;
      const size_t xfer = narrow ? binds[bi].bytes / 2 : binds[bi].bytes;
      if (!v.pinned) {   // borrowed pageable memory: through page-locked host slot `slot`
        if (!host_slot_free) {   // chunk c - 2's transfer out of this slot has finished
          const auto t0 = clk::now();
          ck(cudaEventSynchronize(P.h2d_done[slot]), "event synchronize");
          ms_wait += std::chrono::duration<double, std::milli>(clk::now() - t0).count();
          host_slot_free = true;
        }
        if (P.host_staging_bytes.size() < binds.size()) P.host_staging_bytes.assign(binds.size(), 0);
        for (auto& hs : P.host_staging) hs.resize(binds.size(), nullptr);
        if (!P.host_staging[slot][bi]) {
          size_t most = 0;   // the largest chunk's bytes of this binding
          for (size_t c2 = 0; c2 < P.plans.size(); ++c2) most = std::max(most, P.plans[c2]->inputs()[bi].bytes);
          ck(cudaHostAlloc(&P.host_staging[slot][bi], most, cudaHostAllocPortable), "cudaHostAlloc (input staging)");
          P.host_staging_bytes[bi] = most;
        }
        const auto t0 = clk::now();
        if (narrow)
          par_f32_to_bf16(static_cast<uint16_t*>(P.host_staging[slot][bi]), reinterpret_cast<const float*>(src),
                          binds[bi].bytes / 4, P.host_threads);
        else
          par_memcpy(P.host_staging[slot][bi], src, binds[bi].bytes, P.host_threads);
        ms_copy += std::chrono::duration<double, std::milli>(clk::now() - t0).count();
        src = static_cast<const uint8_t*>(P.host_staging[slot][bi]);
      }
      void* dst = (one && !narrow) ? plan.buffer_ptr(binds[bi].buf) : P.staging[slot][bi];
      ck(cudaMemcpyAsync(dst, src, xfer, cudaMemcpyHostToDevice, P.copy), "H2D");
    }
    ck(cudaEventRecord(P.h2d_done[slot], P.copy), "event record");
    ck(cudaStreamWaitEvent(cs, P.h2d_done[slot], 0), "stream wait");
    for (size_t bi = 0; bi < binds.size(); ++bi) {
      if (narrowed[bi])
        ck(k::bf16_to_f32(P.staging[slot][bi], plan.buffer_ptr(binds[bi].buf), int64_t(binds[bi].bytes / 4), cs),
           "bf16 widening");
      else if (!one)
        ck(cudaMemcpyAsync(plan.buffer_ptr(binds[bi].buf), P.staging[slot][bi], binds[bi].bytes,
                           cudaMemcpyDeviceToDevice, cs),
           "D2D");
    }
    ck(cudaEventRecord(P.consumed[slot], cs), "event record");
    plan.enqueue_kernels(cs);
    // outputs: into output slot `slot` on the compute stream (once its previous host copy is done),
    // then to the host on the d2h stream, overlapping the next chunks (one chunk: straight from the
    // plan's output buffers)
    if (c >= 2) ck(cudaStreamWaitEvent(cs, P.out_free[slot], 0), "stream wait");
    for (size_t j = 0; j < outs.size(); ++j) {
      hout[j] = nullptr;
      if (!outs[j] || ps.out_host[j]) continue;
      const size_t row = outs[j]->nbytes / size_t(std::max<int64_t>(ps.out_shapes[j][0], 1));
      hout[j] = static_cast<uint8_t*>(outs[j]->data) + size_t(r0) * row;
      if (!one)
        ck(cudaMemcpyAsync(P.out_staging[slot][j], plan.output_ptr(j), row * size_t(P.rows[c]),
                           cudaMemcpyDeviceToDevice, cs),
           "D2D (outputs)");
    }
    ck(cudaEventRecord(P.out_ready[slot], cs), "event record");
    ck(cudaStreamWaitEvent(P.d2h, P.out_ready[slot], 0), "stream wait");
    for (size_t j = 0; j < outs.size(); ++j)
      if (hout[j])
        ck(cudaMemcpyAsync(hout[j], one ? plan.output_ptr(j) : P.out_staging[slot][j],
                           outs[j]->nbytes / size_t(std::max<int64_t>(ps.out_shapes[j][0], 1)) * size_t(P.rows[c]),
                           cudaMemcpyDeviceToHost, P.d2h),
           "D2H");
    ck(cudaEventRecord(P.out_free[slot], P.d2h), "event record");
  }
  const double ms_enqueued = std::chrono::duration<double, std::milli>(clk::now() - t_run).count();
  ck(cudaStreamSynchronize(cs), "stream synchronize");
  ck(cudaStreamSynchronize(P.copy), "stream synchronize");
  ck(cudaStreamSynchronize(P.d2h), "stream synchronize");
  if (debug_level() >= 2)
    std::fprintf(stderr, "[shorokoo_b200] pipelined run (device %d): %.3f ms (all enqueued at %.3f ms; host staging "
                 "copies %.3f ms, waits for staging slots %.3f ms)\n",
                 P.device, std::chrono::duration<double, std::milli>(clk::now() - t_run).count(), ms_enqueued, ms_copy,
                 ms_wait);
  for (size_t c = 0; c < P.plans.size(); ++c)
    if (c == 0 || P.plans[c] != P.plans[c - 1]) P.plans[c]->check_device_error();
}

// Runs every shard's plan on its device (one host thread per device when sharded): copies of the
// inputs in, the kernels, copies of the outputs out; input and output pointers may be host memory or
// device memory (cudaMemcpyDefault picks the direction).
void Session::run_shards(PlanSet& ps, const std::vector<std::shared_ptr<HostValue>>& inputs,
                         const std::vector<std::shared_ptr<HostValue>>& outs) {
  const size_t nout = ps.out_shapes.size();
  std::vector<std::string> errs(ps.shards.size());
  std::vector<int32_t> codes(ps.shards.size(), 0);
  auto work = [&](size_t si) {
    const Shard& sh = ps.shards[si];
    try {
      ck(cudaSetDevice(devices_[size_t(sh.device)]), "cudaSetDevice");
      std::vector<const void*> hin(inputs.size(), nullptr);
      for (size_t i = 0; i < inputs.size(); ++i) {
        const HostValue& v = *inputs[i];
        if (numel(v.shape) <= kPlanTimeInputMaxElems) continue;
        size_t row = v.shape.empty() ? 0 : v.nbytes / size_t(std::max<int64_t>(v.shape[0], 1));
        const void* base = v.dev ? v.dev : v.data;   // device-resident: copied device to device
        hin[i] = static_cast<const uint8_t*>(base) + (ps.sharded ? size_t(sh.begin) * row : 0);
      }
      std::vector<void*> hout(nout, nullptr);
      for (size_t j = 0; j < nout; ++j) {
        if (!outs[j] || ps.out_host[j]) continue;
        size_t row = ps.out_shapes[j].empty() ? 0
                                                : outs[j]->nbytes / size_t(std::max<int64_t>(ps.out_shapes[j][0], 1));
        void* base = outs[j]->dev ? outs[j]->dev : outs[j]->data;
        hout[j] = static_cast<uint8_t*>(base) + (ps.sharded ? size_t(sh.begin) * row : 0);
      }
      cudaStream_t s = streams_[size_t(sh.device)];
      sh.plan->enqueue(s, hin, hout);
      ck(cudaStreamSynchronize(s), "stream synchronize");
      sh.plan->check_device_error();
    } catch (const Error& e) {
      errs[si] = e.what();
      codes[si] = e.code;
    } catch (const std::exception& e) {
      errs[si] = e.what();
      codes[si] = SB_INTERNAL;
    }
  };
  if (ps.shards.size() == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (size_t si = 0; si < ps.shards.size(); ++si) th.emplace_back(work, si);
    for (auto& t : th) t.join();
  }
  for (size_t si = 0; si < errs.size(); ++si)
    if (codes[si]) fail(codes[si], errs[si]);
}

std::vector<std::shared_ptr<HostValue>> Session::run(const std::vector<std::shared_ptr<HostValue>>& inputs,
                                                     const std::vector<int>& out_idx, bool keep_on_device) {
  std::lock_guard<std::mutex> lock(mu_);
  auto ps = get_plans(inputs);
  const size_t nout = ps->out_shapes.size();
  std::vector<std::shared_ptr<HostValue>> outs(nout);
  std::vector<bool> wanted(nout, false);
  for (int j : out_idx) wanted[size_t(j)] = true;
  bool dev_inputs = false;
  for (const auto& v : inputs) dev_inputs = dev_inputs || v->dev != nullptr;
  if (keep_on_device || dev_inputs) {   // chained runs: no host copies to hide, no micro-batch pipeline
    for (size_t j = 0; j < nout; ++j) {
      if (!wanted[j]) continue;
      if (ps->out_host[j]) {
        const HostTensor& h = *ps->out_values[j];
        outs[j] = HostValue::alloc_tensor(h.dtype, h.shape);
        if (h.nbytes()) std::memcpy(outs[j]->data, h.data(), h.nbytes());
      } else if (keep_on_device) {
        auto v = std::make_shared<HostValue>();
        v->elem_type = DT_FLOAT;
        v->shape = ps->out_shapes[j];
        v->nbytes = size_t(numel(v->shape)) * 4;
        v->dev_id = devices_[0];
        ck(cudaSetDevice(v->dev_id), "cudaSetDevice");
        ck(cudaMalloc(&v->dev, std::max<size_t>(v->nbytes, 16)), "cudaMalloc (device-resident output)");
        outs[j] = v;
      } else {
        outs[j] = HostValue::alloc_tensor(DT_FLOAT, ps->out_shapes[j]);
      }
    }
  } else {
    maybe_build_pipeline(*ps, inputs);
  }
  if (keep_on_device || dev_inputs) {
    run_shards(*ps, inputs, outs);
    std::vector<std::shared_ptr<HostValue>> res;
    for (int j : out_idx) res.push_back(outs[size_t(j)]);
    return res;
  }
  // A pipelined run copies each chunk's outputs back while later chunks still copy in and compute:
  // a copy into pageable memory would block the host until the chunk is done, serialising the
  // pipeline, so those outputs are page-locked whatever their size.
  const bool pipes = use_pipelines(*ps, inputs);
  const bool pin_outputs = pipes;
  for (size_t j = 0; j < nout; ++j) {
    if (!wanted[j]) continue;
    if (ps->out_host[j]) {
      const HostTensor& h = *ps->out_values[j];
      outs[j] = HostValue::alloc_tensor(h.dtype, h.shape);
      if (h.nbytes()) std::memcpy(outs[j]->data, h.data(), h.nbytes());
    } else {
      outs[j] = HostValue::alloc_tensor(DT_FLOAT, ps->out_shapes[j], pin_outputs);
    }
  }
  if (pipes) {
    const int mode = staging_mode(inputs);
    const auto& pl = ps->pipes[mode];
    if (pl.size() == 1) {
      run_pipelined(*ps, mode, 0, inputs, outs);
    } else {   // one host thread per device
      std::vector<std::string> errs(pl.size());
      std::vector<int32_t> codes(pl.size(), 0);
      std::vector<std::thread> th;
      for (size_t si = 0; si < pl.size(); ++si)
        th.emplace_back([&, si] {
          try {
            run_pipelined(*ps, mode, si, inputs, outs);
          } catch (const Error& e) {
            errs[si] = e.what();
            codes[si] = e.code;
          } catch (const std::exception& e) {
            errs[si] = e.what();
            codes[si] = SB_INTERNAL;
          }
        });
      for (auto& t : th) t.join();
      for (size_t si = 0; si < errs.size(); ++si)
        if (codes[si]) fail(codes[si], errs[si]);
    }
    std::vector<std::shared_ptr<HostValue>> res;
    for (int j : out_idx) res.push_back(outs[size_t(j)]);
    return res;
  }
  run_shards(*ps, inputs, outs);
  std::vector<std::shared_ptr<HostValue>> res;
  for (int j : out_idx) res.push_back(outs[size_t(j)]);
  return res;
}

std::vector<double> Session::time_device(const std::vector<std::shared_ptr<HostValue>>& inputs, int warmup, int iters) {
  std::lock_guard<std::mutex> lock(mu_);
  auto ps = get_plans(inputs);
  std::vector<double> ms(ps->shards.size(), 0.0);
  std::vector<std::string> errs(ps->shards.size());
  std::vector<int32_t> codes(ps->shards.size(), 0);
  auto work = [&](size_t si) {
    const Shard& sh = ps->shards[si];
    try {
      ck(cudaSetDevice(devices_[size_t(sh.device)]), "cudaSetDevice");
      cudaStream_t s = streams_[size_t(sh.device)];
      std::vector<const void*> hin(inputs.size(), nullptr);
      for (size_t i = 0; i < inputs.size(); ++i) {
        const HostValue& v = *inputs[i];
        if (numel(v.shape) <= kPlanTimeInputMaxElems) continue;
        size_t row = v.shape.empty() ? 0 : v.nbytes / size_t(std::max<int64_t>(v.shape[0], 1));
        hin[i] = static_cast<const uint8_t*>(v.dev ? v.dev : v.data) + (ps->sharded ? size_t(sh.begin) * row : 0);
      }
      std::vector<void*> hout(ps->out_shapes.size(), nullptr);
      sh.plan->enqueue(s, hin, hout);   // inputs resident in HBM from here on
      for (int w = 0; w < warmup; ++w) sh.plan->enqueue_kernels(s);
      cudaEvent_t e0, e1;
      ck(cudaEventCreate(&e0), "event");
      ck(cudaEventCreate(&e1), "event");
      ck(cudaStreamSynchronize(s), "sync");
      ck(cudaEventRecord(e0, s), "event record");
      for (int i = 0; i < iters; ++i) sh.plan->enqueue_kernels(s);
      ck(cudaEventRecord(e1, s), "event record");
      ck(cudaEventSynchronize(e1), "event sync");
      float t = 0;
      ck(cudaEventElapsedTime(&t, e0, e1), "elapsed");
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      ms[si] = double(t) / std::max(iters, 1);
      sh.plan->check_device_error();
    } catch (const Error& e) {
      errs[si] = e.what();
      codes[si] = e.code;
    }
  };
  std::vector<std::thread> th;
  for (size_t si = 0; si < ps->shards.size(); ++si) th.emplace_back(work, si);
  for (auto& t : th) t.join();
  for (size_t si = 0; si < errs.size(); ++si)
    if (codes[si]) fail(codes[si], errs[si]);
  return ms;
}

std::vector<std::pair<std::string, double>> Session::profile_steps(const std::vector<std::shared_ptr<HostValue>>& inputs,
                                                                   int iters) {
  std::lock_guard<std::mutex> lock(mu_);
  auto ps = get_plans(inputs);
  const Shard& sh = ps->shards[0];
  ck(cudaSetDevice(devices_[size_t(sh.device)]), "cudaSetDevice");
  cudaStream_t s = streams_[size_t(sh.device)];
  std::vector<const void*> hin(inputs.size(), nullptr);
  for (size_t i = 0; i < inputs.size(); ++i)
    if (numel(inputs[i]->shape) > kPlanTimeInputMaxElems) hin[i] = inputs[i]->dev ? inputs[i]->dev : inputs[i]->data;
  std::vector<void*> hout(ps->out_shapes.size(), nullptr);
  sh.plan->enqueue(s, hin, hout);
  ck(cudaStreamSynchronize(s), "sync");
  auto r = sh.plan->profile(s, iters);
  sh.plan->check_device_error();
  return r;
}

PlanStats Session::stats(const std::vector<std::shared_ptr<HostValue>>& inputs) {
  std::lock_guard<std::mutex> lock(mu_);
  auto ps = get_plans(inputs);
  PlanStats t;
  for (auto& sh : ps->shards) {
    const PlanStats& s = sh.plan->stats();
    t.kernels += s.kernels;
    t.tc_kernels += s.tc_kernels;
    t.macs += s.macs;
    t.arena_bytes += s.arena_bytes;
    t.weight_bytes += s.weight_bytes;
  }
  return t;
}

std::pair<int64_t, int64_t> Session::transfer_bytes(const std::vector<std::shared_ptr<HostValue>>& inputs) {
  std::lock_guard<std::mutex> lock(mu_);
  auto ps = get_plans(inputs);
  maybe_build_pipeline(*ps, inputs);
  int64_t h2d = 0, d2h = 0;
  for (const auto& sh : ps->shards)
    for (const auto& b : sh.plan->inputs()) {
      const HostValue& v = *inputs[size_t(b.index)];
      const bool narrow = !ps->pipes[1].empty() && !v.pinned && !v.dev && b.bf16_ok && v.elem_type == DT_FLOAT;
      h2d += int64_t(narrow ? b.bytes / 2 : b.bytes);
    }
  for (size_t j = 0; j < ps->out_shapes.size(); ++j)
    if (!ps->out_host[j]) d2h += numel(ps->out_shapes[j]) * 4;
  return {h2d, d2h};
}

int Session::devices_used(const std::vector<std::shared_ptr<HostValue>>& inputs) {
  std::lock_guard<std::mutex> lock(mu_);
  return int(get_plans(inputs)->shards.size());
}

}  // namespace sb
