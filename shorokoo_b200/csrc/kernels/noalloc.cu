// sb_linear_noalloc: the dense Linear kernel path (fp32 -> bf16 operand conversion + tcgen05 GEMM
// with bias / ReLU epilogue) for callers that must not allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is not allowed or not safe to call — a host
// application whose memory is fully budgeted up front, a plugin that lives inside another
// runtime's allocator, or a latency-critical loop that must not hit the driver's allocator. Such a
// caller owns its input and output buffers already; the only extra memory the kernel path needs is
// scratch for the bf16 copies of the operands, the padded bias and the device error word.
//
// That scratch is one file-scope device array of kNoAllocScratchBytes (16 MiB), present on every
// GPU that loads this library until the process exits. Host code cannot use the array's name as a
// device address (it names a host-side stand-in), so each device's address is looked up once with
// cudaGetSymbolAddress while that device is current, on the first call for the device. The address
// is cached per device ordinal, which holds for the CUDA runtime's primary context of that device
// (the context every runtime-API caller uses); a caller that makes its own driver-API context
// current gets a different per-context address from the lookup, which this cache does not track.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <string>

#include "shorokoo_b200.h"
#include "kernels.h"

namespace sb {
void set_thread_error(const std::string& msg);
}

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::atomic<void*> g_scratch_ptr[kMaxDevices];   // device address of the array, per device
std::atomic<int> g_sm_count[kMaxDevices];         // multiprocessors, per device (0: not looked up)
std::mutex g_setup_mu;

size_t up256(size_t n) { return (n + 255) / 256 * 256; }

int32_t fail(int32_t code, const std::string& msg) {
  sb::set_thread_error(msg);
  return code;
}

}  // namespace

extern "C" int32_t sb_linear_noalloc(const float* x, const float* w, const float* bias, float* y, int64_t M,
                                     int64_t K, int64_t N, int32_t relu, void* stream) {
  if (!x || !w || !y || M <= 0 || K <= 0 || N <= 0)
    return fail(SB_STATUS_INVALID_ARGUMENT, "sb_linear_noalloc: null pointer or non-positive size");
  const int64_t Kp = (K + 7) / 8 * 8;          // bf16 row pitch of x (16-byte rows for TMA)
  const int64_t Kpad = (K + 63) / 64 * 64;     // reduction length of the weights
  const int64_t Nb = (N + 255) / 256 * 256;    // padded bias length
  const size_t x_bytes = up256(size_t(M) * size_t(Kp) * 2);
  const size_t w_bytes = up256(size_t(N) * size_t(Kpad) * 2);
  const size_t b_bytes = up256(size_t(Nb) * 4);
  const size_t need = x_bytes + w_bytes + b_bytes + 256;
  if (M >= (int64_t(1) << 31) || need > kNoAllocScratchBytes)
    return fail(SB_STATUS_INVALID_ARGUMENT,
                "sb_linear_noalloc: M=" + std::to_string(M) + " K=" + std::to_string(K) + " N=" + std::to_string(N) +
                    " needs " + std::to_string(need) + " scratch bytes; the fixed scratch holds " +
                    std::to_string(kNoAllocScratchBytes));
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(SB_STATUS_CUDA_ERROR, "sb_linear_noalloc: no current CUDA device");
  void* base = g_scratch_ptr[dev].load();
  int sms = g_sm_count[dev].load();
  if (!base || sms <= 0) {   // first call on this device: the scratch array's address, the SM count
    std::lock_guard<std::mutex> l(g_setup_mu);
    base = g_scratch_ptr[dev].load();
    sms = g_sm_count[dev].load();
    if (!base) {
      cudaError_t e = cudaGetSymbolAddress(&base, g_noalloc_scratch);
      if (e != cudaSuccess || !base)
        return fail(SB_STATUS_CUDA_ERROR, std::string("sb_linear_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      g_scratch_ptr[dev].store(base);
    }
    if (sms <= 0) {
      if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        return fail(SB_STATUS_CUDA_ERROR, "sb_linear_noalloc: cannot read the multiprocessor count");
      g_sm_count[dev].store(sms);
    }
  }
  uint8_t* p = static_cast<uint8_t*>(base);
  void* xs = p;
  void* ws = p + x_bytes;
  float* bs = reinterpret_cast<float*>(p + x_bytes + w_bytes);
  unsigned int* err = reinterpret_cast<unsigned int*>(p + x_bytes + w_bytes + b_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // The scratch keeps the previous call's contents: clear the padded bias and the error word.
  cudaError_t e = cudaMemsetAsync(bs, 0, b_bytes + 256, s);
  if (e == cudaSuccess && bias) e = cudaMemcpyAsync(bs, bias, size_t(N) * 4, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess) e = sb::k::to_rows_bf16(x, 0, M, K, K, 1, xs, Kp, s);
  if (e == cudaSuccess) e = sb::k::to_rows_bf16(w, 0, N, K, K, 1, ws, Kpad, s);
  if (e != cudaSuccess) return fail(SB_STATUS_CUDA_ERROR, std::string("sb_linear_noalloc: ") + cudaGetErrorString(e));

  sb::k::ConvGemmPlan plan;
  std::memset(&plan, 0, sizeof(plan));
  sb::k::ConvGemmArgs& a = plan.args;
  a.gather = 0;
  a.N = a.H = a.W = 1;
  a.Ho = a.Wo = 1;
  a.KH = a.KW = 1;
  a.sh = a.sw = a.dh = a.dw = 1;
  a.Cp = int(K);
  a.M = int(M);
  a.Cout = int(N);
  a.Kpad = int(Kpad);
  a.bias = bs;
  a.out = y;
  a.out_bf16 = 0;
  a.ldo = N;
  a.act = relu ? 1 : 0;
  a.err = err;
  try {
    sb::k::conv_gemm_prepare(plan, xs, Kp, ws, sms);
  } catch (const std::exception& ex) {
    return fail(SB_STATUS_CUDA_ERROR, std::string("sb_linear_noalloc: ") + ex.what());
  }
  e = sb::k::conv_gemm_launch(plan, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(SB_STATUS_CUDA_ERROR, std::string("sb_linear_noalloc: ") + cudaGetErrorString(e));
  unsigned int werr = 0;
  if (cudaMemcpy(&werr, err, sizeof(werr), cudaMemcpyDeviceToHost) != cudaSuccess || werr != 0)
    return fail(SB_STATUS_CUDA_ERROR, "sb_linear_noalloc: tensor-core pipeline wait timed out");
  return SB_STATUS_OK;
}
