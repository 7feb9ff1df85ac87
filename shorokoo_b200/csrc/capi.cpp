// extern "C" entry points declared in include/shorokoo_b200.h.
#include "../../include/shorokoo_b200.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <list>
#include <memory>
#include <mutex>
#include <string>

#include "session.h"

extern char** environ;

namespace sb {
void* host_alloc(size_t bytes, bool& pinned);
bool host_is_page_locked(const void* p);
void host_copy(void* dst, const void* src, size_t n);
void host_narrow_bf16(uint16_t* dst, const float* src, size_t n, unsigned threads);
}  // namespace sb

using sb::HostValue;

struct sb_session {
  std::shared_ptr<sb::Session> s;   // shared with the session cache and other handles on the same model
  std::vector<std::string> profile_kinds;
};

struct sb_value {
  std::shared_ptr<HostValue> v;
};

namespace {

thread_local std::string g_last_error;

int32_t set_error(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

template <typename F>
int32_t guarded(F&& f) {
  try {
    g_last_error.clear();
    return f();
  } catch (const sb::Error& e) {
    return set_error(e.code, e.what());
  } catch (const std::bad_alloc&) {
    return set_error(SB_STATUS_OUT_OF_MEMORY, "host out of memory");
  } catch (const std::exception& e) {
    return set_error(SB_STATUS_INTERNAL, e.what());
  }
}

std::vector<int64_t> shape_of(const int64_t* shape, int32_t rank) {
  SB_CHECK(rank >= 0 && rank <= 16, sb::SB_INVALID_ARGUMENT, "rank out of range");
  SB_CHECK(rank == 0 || shape != nullptr, sb::SB_INVALID_ARGUMENT, "shape is null");
  std::vector<int64_t> s(shape, shape + rank);
  for (int64_t d : s) SB_CHECK(d >= 0, sb::SB_INVALID_ARGUMENT, "negative dimension");
  return s;
}

std::vector<std::shared_ptr<HostValue>> ordered_inputs(const sb::Session& s, int32_t n, const char* const* names,
                                                       sb_value* const* vals) {
  const auto& want = s.input_names();
  SB_CHECK(n >= 0 && (n == 0 || (names && vals)), sb::SB_INVALID_ARGUMENT, "null input arrays");
  std::vector<std::shared_ptr<HostValue>> out(want.size());
  for (int32_t i = 0; i < n; ++i) {
    SB_CHECK(names[i] && vals[i], sb::SB_INVALID_ARGUMENT, "null input name or value");
    size_t k = 0;
    while (k < want.size() && want[k] != names[i]) ++k;
    SB_CHECK(k < want.size(), sb::SB_INVALID_ARGUMENT, std::string("unknown input '") + names[i] + "'");
    SB_CHECK(!out[k], sb::SB_INVALID_ARGUMENT, std::string("input '") + names[i] + "' given twice");
    out[k] = vals[i]->v;
  }
  for (size_t k = 0; k < want.size(); ++k)
    SB_CHECK(out[k] != nullptr, sb::SB_INVALID_ARGUMENT, "missing input '" + want[k] + "'");
  return out;
}

// Process-wide session cache: ComputeContext.Execute creates a new session per call
// (ComputeContext.cs:318-359), so a handle created for model bytes already seen (same 128-bit
// content hash and length, device range, precision and SHOROKOO_B200_* settings, which plans
// read when they are built) shares the existing session and with it every plan built so far. The bytes themselves are not retained. The last
// SHOROKOO_B200_SESSION_CACHE (default 2, 0 disables) distinct sessions stay cached after their
// handles are destroyed; sb_session_cache_clear releases them.
struct CacheKey {
  uint64_t h1, h2;
  size_t len;
  int32_t num_devices, first_device, precision;
  std::string env;   // SHOROKOO_B200_* settings in effect
  bool operator==(const CacheKey& o) const {
    return h1 == o.h1 && h2 == o.h2 && len == o.len && num_devices == o.num_devices &&
           first_device == o.first_device && precision == o.precision && env == o.env;
  }
};

// Two independent 64-bit multiply-xorshift hashes over 8-byte words (with the tail zero-padded).
void content_hash(const uint8_t* p, size_t n, uint64_t& h1, uint64_t& h2) {
  uint64_t a = 0x243F6A8885A308D3ull ^ n, b = 0x13198A2E03707344ull + n;
  size_t i = 0;
  auto mix = [](uint64_t h, uint64_t w, uint64_t k) {
    h ^= w * k;
    h = (h << 27) | (h >> 37);
    return h * 0x9E3779B97F4A7C15ull + 0x632BE59BD9B4E019ull;
  };
  for (; i + 8 <= n; i += 8) {
    uint64_t w;
    std::memcpy(&w, p + i, 8);
    a = mix(a, w, 0xC2B2AE3D27D4EB4Full);
    b = mix(b, w ^ 0xA0761D6478BD642Full, 0x165667B19E3779F9ull);
  }
  uint64_t w = 0;
  if (i < n) std::memcpy(&w, p + i, n - i);
  a = mix(a, w, 0xC2B2AE3D27D4EB4Full);
  b = mix(b, w ^ 0xA0761D6478BD642Full, 0x165667B19E3779F9ull);
  a ^= a >> 33;
  b ^= b >> 29;
  h1 = a * 0xFF51AFD7ED558CCDull;
  h2 = b * 0xC4CEB9FE1A85EC53ull;
}

std::mutex g_cache_mu;
std::list<std::pair<CacheKey, std::shared_ptr<sb::Session>>> g_cache;   // most recent first

std::string backend_env() {
  std::string r;
  for (char** e = environ; e && *e; ++e)
    if (std::strncmp(*e, "SHOROKOO_B200_", 14) == 0 && std::strncmp(*e, "SHOROKOO_B200_SESSION_CACHE=", 28) != 0) {
      r += *e;
      r += '\n';
    }
  return r;
}

size_t cache_capacity() {
  const char* e = std::getenv("SHOROKOO_B200_SESSION_CACHE");
  return e ? size_t(std::max(0, std::atoi(e))) : 2;
}

}  // namespace

namespace sb {
void set_thread_error(const std::string& msg) { g_last_error = msg; }
}  // namespace sb

extern "C" {

int32_t sb_version(void) { return 100; }

const char* sb_last_error(void) { return g_last_error.c_str(); }

int32_t sb_session_create_ex(const uint8_t* model, size_t len, int32_t, int32_t, int32_t num_devices,
                             int32_t first_device, int32_t precision, sb_session** out) {
  return guarded([&] {
    SB_CHECK(out != nullptr, sb::SB_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    SB_CHECK(precision >= SB_PRECISION_DEFAULT && precision <= SB_PRECISION_TF32X3, sb::SB_INVALID_ARGUMENT,
             "precision must be SB_PRECISION_DEFAULT, _BF16, _TF32 or _TF32X3");
    SB_CHECK(model != nullptr || len == 0, sb::SB_INVALID_ARGUMENT, "model is null");
    sb::SessionOptions o;
    o.num_devices = num_devices;
    o.first_device = first_device;
    o.precision = sb::resolve_precision(precision);
    CacheKey key;
    content_hash(model, len, key.h1, key.h2);
    key.len = len;
    key.num_devices = num_devices;
    key.first_device = first_device;
    key.precision = o.precision;
    key.env = backend_env();
    auto s = std::make_unique<sb_session>();
    const size_t cap = cache_capacity();
    if (cap > 0) {
      std::lock_guard<std::mutex> l(g_cache_mu);
      for (auto it = g_cache.begin(); it != g_cache.end(); ++it)
        if (it->first == key) {
          s->s = it->second;
          g_cache.splice(g_cache.begin(), g_cache, it);
          break;
        }
    }
    if (!s->s) {
      s->s = std::make_shared<sb::Session>(model, len, o);
      if (cap > 0) {
        std::lock_guard<std::mutex> l(g_cache_mu);
        g_cache.emplace_front(key, s->s);
        while (g_cache.size() > cap) g_cache.pop_back();
      }
    }
    *out = s.release();
    return SB_STATUS_OK;
  });
}

int32_t sb_session_create(const uint8_t* model, size_t len, int32_t opt, int32_t sev, sb_session** out) {
  return sb_session_create_ex(model, len, opt, sev, 0, 0, SB_PRECISION_DEFAULT, out);
}

void sb_session_destroy(sb_session* s) { delete s; }

int32_t sb_session_cache_clear(void) {
  std::list<std::pair<CacheKey, std::shared_ptr<sb::Session>>> drop;
  {
    std::lock_guard<std::mutex> l(g_cache_mu);
    drop.swap(g_cache);
  }
  return int32_t(drop.size());   // the sessions are released here unless a handle still holds one
}

int32_t sb_session_input_count(const sb_session* s) { return s ? int32_t(s->s->input_names().size()) : 0; }
const char* sb_session_input_name(const sb_session* s, int32_t i) {
  if (!s || i < 0 || size_t(i) >= s->s->input_names().size()) return nullptr;
  return s->s->input_names()[size_t(i)].c_str();
}
int32_t sb_session_output_count(const sb_session* s) { return s ? int32_t(s->s->output_names().size()) : 0; }
const char* sb_session_output_name(const sb_session* s, int32_t i) {
  if (!s || i < 0 || size_t(i) >= s->s->output_names().size()) return nullptr;
  return s->s->output_names()[size_t(i)].c_str();
}

static int32_t run_impl(sb_session* s, int32_t n_in, const char* const* in_names, sb_value* const* in_values,
                        int32_t n_out, const char* const* out_names, sb_value** out_values, bool keep_on_device) {
  return guarded([&] {
    SB_CHECK(s != nullptr, sb::SB_INVALID_ARGUMENT, "session is null");
    SB_CHECK(n_out >= 0 && (n_out == 0 || (out_names && out_values)), sb::SB_INVALID_ARGUMENT, "null output arrays");
    for (int32_t j = 0; j < n_out; ++j) out_values[j] = nullptr;
    auto ins = ordered_inputs(*s->s, n_in, in_names, in_values);
    const auto& onames = s->s->output_names();
    std::vector<int> idx;
    for (int32_t j = 0; j < n_out; ++j) {
      SB_CHECK(out_names[j] != nullptr, sb::SB_INVALID_ARGUMENT, "null output name");
      size_t k = 0;
      while (k < onames.size() && onames[k] != out_names[j]) ++k;
      SB_CHECK(k < onames.size(), sb::SB_INVALID_ARGUMENT, std::string("unknown output '") + out_names[j] + "'");
      idx.push_back(int(k));
    }
    auto outs = s->s->run(ins, idx, keep_on_device);
    for (int32_t j = 0; j < n_out; ++j) out_values[j] = new sb_value{outs[size_t(j)]};
    return SB_STATUS_OK;
  });
}

int32_t sb_session_run(sb_session* s, int32_t n_in, const char* const* in_names, sb_value* const* in_values,
                       int32_t n_out, const char* const* out_names, sb_value** out_values) {
  return run_impl(s, n_in, in_names, in_values, n_out, out_names, out_values, false);
}

int32_t sb_session_run_device(sb_session* s, int32_t n_in, const char* const* in_names, sb_value* const* in_values,
                              int32_t n_out, const char* const* out_names, sb_value** out_values) {
  return run_impl(s, n_in, in_names, in_values, n_out, out_names, out_values, true);
}

int32_t sb_value_device_ptr(const sb_value* v, void** ptr, int32_t* device) {
  return guarded([&] {
    SB_CHECK(v && ptr && device, sb::SB_INVALID_ARGUMENT, "null argument");
    *ptr = v->v->dev;
    *device = v->v->dev ? v->v->dev_id : -1;
    return SB_STATUS_OK;
  });
}

int32_t sb_value_create_tensor(int32_t et, const int64_t* shape, int32_t rank, const void* data, size_t nbytes,
                               sb_value** out) {
  return guarded([&] {
    SB_CHECK(out != nullptr, sb::SB_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    SB_CHECK(et != sb::DT_STRING, sb::SB_INVALID_ARGUMENT,
             "String tensors are variable-length and not byte-stride; use sb_value_create_string_tensor");
    SB_CHECK(sb::dtype_size(et) != 0, sb::SB_UNSUPPORTED, "element type " + std::to_string(et) + " is not supported");
    auto s = shape_of(shape, rank);
    auto v = HostValue::alloc_tensor(et, s);
    SB_CHECK(nbytes == v->nbytes, sb::SB_INVALID_ARGUMENT,
             "data is " + std::to_string(nbytes) + " bytes but shape " + sb::shape_str(s) + " needs " +
                 std::to_string(v->nbytes));
    SB_CHECK(nbytes == 0 || data != nullptr, sb::SB_INVALID_ARGUMENT, "data is null");
    if (nbytes) sb::host_copy(v->data, data, nbytes);
    *out = new sb_value{v};
    return SB_STATUS_OK;
  });
}

int32_t sb_value_wrap_tensor(int32_t et, const int64_t* shape, int32_t rank, void* data, size_t nbytes, sb_value** out) {
  return guarded([&] {
    SB_CHECK(out != nullptr, sb::SB_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    SB_CHECK(sb::dtype_size(et) != 0 && et != sb::DT_STRING, sb::SB_UNSUPPORTED,
             "element type " + std::to_string(et) + " is not supported");
    auto s = shape_of(shape, rank);
    auto v = std::make_shared<HostValue>();
    v->elem_type = et;
    v->shape = s;
    v->nbytes = size_t(sb::numel(s)) * sb::dtype_size(et);
    SB_CHECK(nbytes == v->nbytes, sb::SB_INVALID_ARGUMENT, "data size does not match shape " + sb::shape_str(s));
    SB_CHECK(nbytes == 0 || data != nullptr, sb::SB_INVALID_ARGUMENT, "data is null");
    v->data = data;
    v->owned = false;
    v->pinned = sb::host_is_page_locked(data);
    *out = new sb_value{v};
    return SB_STATUS_OK;
  });
}

int32_t sb_value_create_string_tensor(const char* const* strings, size_t count, const int64_t* shape, int32_t rank,
                                      sb_value** out) {
  return guarded([&] {
    SB_CHECK(out != nullptr, sb::SB_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    auto s = shape_of(shape, rank);
    SB_CHECK(int64_t(count) == sb::numel(s), sb::SB_INVALID_ARGUMENT, "string count does not match shape");
    auto v = std::make_shared<HostValue>();
    v->elem_type = sb::DT_STRING;
    v->shape = s;
    for (size_t i = 0; i < count; ++i) {
      SB_CHECK(strings && strings[i], sb::SB_INVALID_ARGUMENT, "null string");
      v->strings.emplace_back(strings[i]);
    }
    *out = new sb_value{v};
    return SB_STATUS_OK;
  });
}

int32_t sb_value_create_sequence(sb_value* const* values, size_t count, sb_value** out) {
  return guarded([&] {
    SB_CHECK(out != nullptr, sb::SB_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    auto v = std::make_shared<HostValue>();
    v->kind = HostValue::SEQUENCE;
    for (size_t i = 0; i < count; ++i) {
      SB_CHECK(values && values[i], sb::SB_INVALID_ARGUMENT, "null sequence element");
      SB_CHECK(values[i]->v->kind == HostValue::TENSOR, sb::SB_UNSUPPORTED, "sequences of sequences are not supported");
      if (i) SB_CHECK(values[i]->v->elem_type == v->items[0]->elem_type, sb::SB_INVALID_ARGUMENT,
                      "sequence elements must share an element type");
      v->items.push_back(values[i]->v);
    }
    v->elem_type = v->items.empty() ? sb::DT_UNDEFINED : v->items[0]->elem_type;
    *out = new sb_value{v};
    return SB_STATUS_OK;
  });
}

void sb_value_release(sb_value* v) { delete v; }

int32_t sb_value_type(const sb_value* v) { return v ? v->v->kind : 0; }
int32_t sb_value_elem_type(const sb_value* v) { return v ? v->v->elem_type : 0; }
int32_t sb_value_rank(const sb_value* v) { return v ? int32_t(v->v->shape.size()) : 0; }
const int64_t* sb_value_shape(const sb_value* v) { return v ? v->v->shape.data() : nullptr; }
void* sb_value_data(sb_value* v) {
  if (!v) return nullptr;
  try {
    return v->v->host_data();   // (a device-resident value is copied to the host on first use)
  } catch (const std::exception& e) {
    sb::set_thread_error(e.what());
    return nullptr;
  }
}
size_t sb_value_nbytes(const sb_value* v) { return v ? v->v->nbytes : 0; }
size_t sb_value_string_count(const sb_value* v) { return v ? v->v->strings.size() : 0; }
const char* sb_value_string_at(const sb_value* v, size_t i) {
  if (!v || i >= v->v->strings.size()) return nullptr;
  return v->v->strings[i].c_str();
}
int32_t sb_value_count(const sb_value* v) { return v ? int32_t(v->v->items.size()) : 0; }
int32_t sb_value_at(const sb_value* v, int32_t i, sb_value** out) {
  return guarded([&] {
    SB_CHECK(v && out && i >= 0 && size_t(i) < v->v->items.size(), sb::SB_INVALID_ARGUMENT, "index out of range");
    *out = new sb_value{v->v->items[size_t(i)]};
    return SB_STATUS_OK;
  });
}
int32_t sb_value_sequence_elem_type(const sb_value* v) {
  return v && v->v->kind == HostValue::SEQUENCE ? v->v->elem_type : 0;
}

int32_t sb_session_time_device(sb_session* s, int32_t n_in, const char* const* in_names, sb_value* const* in_values,
                               int32_t warmup, int32_t iters, double* ms, int32_t capacity, int32_t* n_dev) {
  return guarded([&] {
    SB_CHECK(s && ms && n_dev && iters > 0, sb::SB_INVALID_ARGUMENT, "bad arguments");
    auto ins = ordered_inputs(*s->s, n_in, in_names, in_values);
    auto r = s->s->time_device(ins, warmup, iters);
    *n_dev = int32_t(r.size());
    for (size_t i = 0; i < r.size() && int32_t(i) < capacity; ++i) ms[i] = r[i];
    return SB_STATUS_OK;
  });
}

int32_t sb_session_profile(sb_session* s, int32_t n_in, const char* const* in_names, sb_value* const* in_values,
                           int32_t iters, const char** kinds, double* ms, int32_t capacity, int32_t* n_steps) {
  return guarded([&] {
    SB_CHECK(s && kinds && ms && n_steps && iters > 0, sb::SB_INVALID_ARGUMENT, "bad arguments");
    auto ins = ordered_inputs(*s->s, n_in, in_names, in_values);
    auto r = s->s->profile_steps(ins, iters);
    s->profile_kinds.clear();
    for (auto& p : r) s->profile_kinds.push_back(p.first);
    *n_steps = int32_t(r.size());
    for (size_t i = 0; i < r.size() && int32_t(i) < capacity; ++i) {
      kinds[i] = s->profile_kinds[i].c_str();
      ms[i] = r[i].second;
    }
    return SB_STATUS_OK;
  });
}

int32_t sb_session_stats(sb_session* s, int32_t n_in, const char* const* in_names, sb_value* const* in_values,
                         int64_t* launches, int64_t* tc, double* macs, int64_t* dev_bytes, int32_t* devices) {
  return guarded([&] {
    SB_CHECK(s != nullptr, sb::SB_INVALID_ARGUMENT, "session is null");
    auto ins = ordered_inputs(*s->s, n_in, in_names, in_values);
    auto st = s->s->stats(ins);
    if (launches) *launches = st.kernels;
    if (tc) *tc = st.tc_kernels;
    if (macs) *macs = st.macs;
    if (dev_bytes) *dev_bytes = int64_t(st.arena_bytes + st.weight_bytes);
    if (devices) *devices = s->s->devices_used(ins);
    return SB_STATUS_OK;
  });
}

int32_t sb_session_transfer_bytes(sb_session* s, int32_t n_in, const char* const* in_names, sb_value* const* in_values,
                                  int64_t* h2d, int64_t* d2h) {
  return guarded([&] {
    SB_CHECK(s != nullptr && h2d && d2h, sb::SB_INVALID_ARGUMENT, "null argument");
    auto ins = ordered_inputs(*s->s, n_in, in_names, in_values);
    auto r = s->s->transfer_bytes(ins);
    *h2d = r.first;
    *d2h = r.second;
    return SB_STATUS_OK;
  });
}

int32_t sb_debug_lower(const uint8_t* model, size_t len, int32_t n_in, sb_value* const* in_values, char* buf,
                       size_t cap, size_t* needed) {
  return guarded([&] {
    sb::OnnxModel m = sb::parse_onnx(model, len);
    sb::check_supported_ops(m);
    std::vector<sb::InputSpec> specs;
    for (int32_t i = 0; i < n_in; ++i) {
      SB_CHECK(in_values && in_values[i], sb::SB_INVALID_ARGUMENT, "null input value");
      const HostValue& v = *in_values[i]->v;
      sb::InputSpec s;
      s.dtype = v.elem_type;
      s.shape = v.shape;
      if (sb::numel(v.shape) <= sb::kPlanTimeInputMaxElems) {
        auto h = std::make_shared<sb::HostTensor>(v.elem_type, v.shape);
        if (v.nbytes) std::memcpy(h->mutable_data(), v.data, v.nbytes);
        s.value = h;
      }
      specs.push_back(s);
    }
    sb::LGraph g = sb::lower(m, specs);
    sb::fuse(g);
    // each contraction's operand precision in a bf16 / TF32 / TF32x3 session
    std::vector<std::vector<int>> precs(3);
    for (int p = 0; p < 3; ++p) {
      sb::assign_precision(g, p);
      for (const sb::Op& op : g.ops) precs[size_t(p)].push_back(op.prec);
    }
    static const char* kPrecName[] = {"bf16", "tf32", "tf32x3"};
    std::string out;
    for (size_t oi = 0; oi < g.ops.size(); ++oi) {
      const sb::Op& op = g.ops[oi];
      if (op.dead) continue;
      out += op.type;
      for (int id : op.in)
        if (id >= 0) out += " " + sb::shape_str(g.vals[size_t(id)].shape) + (g.vals[size_t(id)].is_host ? "h" : "");
      out += " ->";
      for (int id : op.out) out += " " + sb::shape_str(g.vals[size_t(id)].shape);
      if (op.type == "FusedConv")
        out += " k=" + std::to_string(op.kernel[0]) + "x" + std::to_string(op.kernel[1]) + " s=" +
               std::to_string(op.strides[0]) + " pads=" + sb::shape_str(op.pads);
      if (op.act) out += " act=" + std::to_string(op.act);
      if (op.residual >= 0) out += " residual=" + std::to_string(op.residual_mode);
      if (op.concat >= 0) out += " concat/" + std::to_string(op.concat_stride);
      if (op.type == "FusedConv" || op.type == "FusedGemm")
        out += std::string(" prec=") + kPrecName[precs[0][oi]] + "/" + kPrecName[precs[1][oi]] + "/" +
               kPrecName[precs[2][oi]];
      out += "\n";
    }
    for (size_t j = 0; j < g.outputs.size(); ++j) {
      const sb::Value& v = g.vals[size_t(g.outputs[j])];
      out += "output " + sb::shape_str(v.shape) + (v.is_host ? " host" : " device") + "\n";
    }
    out += std::string("separable=") + (sb::batch_separable(g) ? "1" : "0") + "\n";
    if (needed) *needed = out.size() + 1;
    if (buf && cap) {
      size_t n = std::min(cap - 1, out.size());
      std::memcpy(buf, out.data(), n);
      buf[n] = 0;
    }
    return SB_STATUS_OK;
  });
}

int32_t sb_debug_narrow_bf16(const float* src, uint16_t* dst, size_t n, int32_t threads) {
  return guarded([&] {
    SB_CHECK((src && dst) || n == 0, sb::SB_INVALID_ARGUMENT, "null buffer");
    sb::host_narrow_bf16(dst, src, n, unsigned(std::max(1, threads)));
    return SB_STATUS_OK;
  });
}

}  // extern "C"
