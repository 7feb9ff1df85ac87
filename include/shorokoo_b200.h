/* shorokoo_b200 — C ABI of the B200 inference backend for Shorokoo.
 *
 * This is the native surface a Shorokoo backend plugin binds (through [LibraryImport] from C#, or
 * ctypes from Python). It replaces the ONNX Runtime calls behind the reference's backend plugin
 * interface:
 *   IShorokooInferenceSessionFactory  src/Shorokoo/Core/Inference/Abstractions/IShorokooInferenceSessionFactory.cs:5-24
 *   IShorokooInferenceSession         src/Shorokoo/Core/Inference/Abstractions/IShorokooInferenceSession.cs:3-13
 *   IShorokooTensorValue              src/Shorokoo/Core/Inference/Abstractions/IShorokooTensorValue.cs:8-31
 * whose ORT implementation is src/Backend/OnnxRuntime/Shorokoo.OnnxRuntime/{OrtSessionFactory,
 * OrtInferenceSession,OrtTensorValue}.cs and whose GPU slot is
 * src/Backend/OnnxRuntime/Shorokoo.LinuxGPU/LinuxGpuInferenceFactory.cs:5-8.
 *
 * Conventions: every function returning int32_t returns a status (SB_STATUS_*); on failure
 * sb_last_error() gives a message for the calling thread. Element types use the ONNX
 * TensorProto.DataType numbering (== ShorokooTensorElementType). All tensor data is HOST memory.
 * Values are reference counted; every sb_value* handed out must be released exactly once.
 */
#ifndef SHOROKOO_B200_H_
#define SHOROKOO_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SB_API __attribute__((visibility("default")))
#else
#define SB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SB_STATUS_OK 0
#define SB_STATUS_INVALID_ARGUMENT 1 /* -> ArgumentException */
#define SB_STATUS_UNSUPPORTED 2      /* -> NotSupportedException (unsupported op/dtype: hard error) */
#define SB_STATUS_SHAPE_ERROR 3      /* -> ArgumentException */
#define SB_STATUS_CUDA_ERROR 4       /* -> InvalidOperationException */
#define SB_STATUS_OUT_OF_MEMORY 5    /* -> OutOfMemoryException */
#define SB_STATUS_INTERNAL 6         /* -> InvalidOperationException */

/* ShorokooOnnxValueType (src/Shorokoo/Core/Inference/Abstractions/ShorokooOnnxValueType.cs) */
#define SB_VALUE_TENSOR 1
#define SB_VALUE_SEQUENCE 2

typedef struct sb_session sb_session;
typedef struct sb_value sb_value;

/* Library version (major*10000 + minor*100 + patch). */
SB_API int32_t sb_version(void);
/* Message of the last failing call on this thread ("" if none). Valid until the next call. */
SB_API const char* sb_last_error(void);

/* ---- IShorokooInferenceSessionFactory.CreateSession(modelBytes, graphOptimization, logSeverity)
 * (IShorokooInferenceSessionFactory.cs:7-10; ORT: OrtSessionFactory.cs:23-42).
 * Parses the ONNX ModelProto bytes (not retained) and rejects any operator without a B200
 * implementation. graph_optimization (ShorokooGraphOptimization) and log_severity
 * (ShorokooLogSeverity) are accepted for interface parity; plans are always fully optimised.
 * Devices: SHOROKOO_B200_DEVICES (default: all visible CUDA devices); batches shard across them. */
SB_API int32_t sb_session_create(const uint8_t* model, size_t model_len, int32_t graph_optimization,
                          int32_t log_severity, sb_session** out);
/* Same, with an explicit device range [first_device, first_device + num_devices) and the
 * tensor-core precision: SB_PRECISION_BF16 (bf16 operands, fp32 accumulation; the throughput mode,
 * normwise error <= 1e-2), SB_PRECISION_TF32 (fp32 operands read as TF32; <= 2e-3 except where
 * deep per-pixel outputs sit at the TF32 floor), SB_PRECISION_TF32X3 (error-compensated TF32:
 * three MMAs per K slice, close to fp32 accuracy, at a third of the TF32 rate), or
 * SB_PRECISION_DEFAULT (SHOROKOO_B200_PRECISION=bf16|tf32|tf32x3, else bf16).
 * sb_session_create uses SB_PRECISION_DEFAULT. No counterpart in the reference, whose ORT CUDA
 * provider computes in fp32 (OrtSessionFactory.cs:23-42). */
#define SB_PRECISION_DEFAULT (-1)
#define SB_PRECISION_BF16 0
#define SB_PRECISION_TF32 1
#define SB_PRECISION_TF32X3 2
SB_API int32_t sb_session_create_ex(const uint8_t* model, size_t model_len, int32_t graph_optimization,
                             int32_t log_severity, int32_t num_devices, int32_t first_device,
                             int32_t precision, sb_session** out);
/* IShorokooInferenceSession.Dispose (IDisposable). */
SB_API void sb_session_destroy(sb_session* session);
/* Sessions are cached per process by model content (128-bit hash of the bytes, which are not
 * retained), device range and precision, so ComputeContext.Execute's session-per-call pattern
 * (ComputeContext.cs:318-359) reuses plans already built. Up to SHOROKOO_B200_SESSION_CACHE
 * (default 2; 0 disables) sessions stay cached after their last handle is destroyed. This
 * releases them and returns how many were cached. No counterpart in the reference. */
SB_API int32_t sb_session_cache_clear(void);

/* IShorokooInferenceSession.InputNames / OutputNames (IShorokooInferenceSession.cs:5-6).
 * Inputs are reported in graph-input order (ComputeContext.cs:209-211 maps them positionally). */
SB_API int32_t sb_session_input_count(const sb_session* session);
SB_API const char* sb_session_input_name(const sb_session* session, int32_t index);
SB_API int32_t sb_session_output_count(const sb_session* session);
SB_API const char* sb_session_output_name(const sb_session* session, int32_t index);

/* IShorokooInferenceSession.Run(inputs, outputNames) (IShorokooInferenceSession.cs:10-12;
 * ORT: OrtInferenceSession.cs:15-36). Inputs by name; outputs in the order of out_names, written
 * to out_values as new references owned by the caller (they outlive the session). */
SB_API int32_t sb_session_run(sb_session* session, int32_t n_inputs, const char* const* in_names,
                       sb_value* const* in_values, int32_t n_outputs, const char* const* out_names,
                       sb_value** out_values);
/* Run for chained inference (no counterpart in the reference interface, whose Run returns host
 * tensors): the same as sb_session_run except that the outputs stay in device memory of the
 * session's first device, with no device->host copy. sb_value_data copies such a value to host
 * memory on first use; passed as an input of a later run (of this or another session), it is copied
 * device to device. Inputs that are device-resident are accepted by sb_session_run as well. Runs
 * with device-resident inputs or outputs do not use the micro-batch pipeline. */
SB_API int32_t sb_session_run_device(sb_session* session, int32_t n_inputs, const char* const* in_names,
                              sb_value* const* in_values, int32_t n_outputs, const char* const* out_names,
                              sb_value** out_values);

/* ---- IShorokooInferenceSessionFactory.CreateTensor<T> / CreateTensorFromRawBytes
 * (IShorokooInferenceSessionFactory.cs:12-18; ORT: OrtSessionFactory.cs:44-91).
 * Copies `nbytes` of element data (page-locked host memory when large). */
SB_API int32_t sb_value_create_tensor(int32_t elem_type, const int64_t* shape, int32_t rank, const void* data,
                               size_t nbytes, sb_value** out);
/* Wraps caller memory without copying (ORT aliases managed arrays the same way,
 * OrtSessionFactory.cs:56). The memory must stay valid and unchanged until the value is released.
 * Page-locked memory is transferred to the device directly; pageable memory (a pinned managed
 * array, say) is staged by Run through page-locked slots, chunk by chunk, overlapped with the
 * transfers and kernels of the previous chunks. */
SB_API int32_t sb_value_wrap_tensor(int32_t elem_type, const int64_t* shape, int32_t rank, void* data,
                             size_t nbytes, sb_value** out);
/* IShorokooInferenceSessionFactory.CreateStringTensor (IShorokooInferenceSessionFactory.cs:20-22). */
SB_API int32_t sb_value_create_string_tensor(const char* const* strings, size_t count, const int64_t* shape,
                                      int32_t rank, sb_value** out);
/* IShorokooInferenceSessionFactory.CreateSequence (IShorokooInferenceSessionFactory.cs:23). */
SB_API int32_t sb_value_create_sequence(sb_value* const* values, size_t count, sb_value** out);
/* IShorokooTensorValue.Dispose. */
SB_API void sb_value_release(sb_value* value);

/* ---- IShorokooTensorValue accessors (IShorokooTensorValue.cs:10-30; ORT: OrtTensorValue.cs:11-56) */
SB_API int32_t sb_value_type(const sb_value* value);      /* ValueType: SB_VALUE_TENSOR / SB_VALUE_SEQUENCE */
SB_API int32_t sb_value_elem_type(const sb_value* value); /* ElementType */
SB_API int32_t sb_value_rank(const sb_value* value);
SB_API const int64_t* sb_value_shape(const sb_value* value); /* Shape */
SB_API void* sb_value_data(sb_value* value);               /* GetTensor(Mutable)DataAsSpan: host memory
                                                            * (NULL and sb_last_error on a failed copy of
                                                            * a device-resident value) */
/* Device address of a device-resident value (an output of sb_session_run_device) and its device;
 * NULL and -1 for host values. No counterpart in the reference interface. */
SB_API int32_t sb_value_device_ptr(const sb_value* value, void** ptr, int32_t* device);
SB_API size_t sb_value_nbytes(const sb_value* value);
SB_API size_t sb_value_string_count(const sb_value* value);           /* GetStringTensorData */
SB_API const char* sb_value_string_at(const sb_value* value, size_t index);
SB_API int32_t sb_value_count(const sb_value* value);                 /* GetValueCount */
SB_API int32_t sb_value_at(const sb_value* value, int32_t index, sb_value** out); /* GetValue: new reference */
SB_API int32_t sb_value_sequence_elem_type(const sb_value* value);    /* GetSequenceElementType */

/* ---- Measurement (no counterpart in the reference interface) ------------------------------ */
/* Uploads the inputs once, replays the captured kernel sequence `iters` times after `warmup`
 * replays, and writes the device time per run (ms, CUDA events) for each device used into
 * ms_per_device[0..*n_devices). */
SB_API int32_t sb_session_time_device(sb_session* session, int32_t n_inputs, const char* const* in_names,
                               sb_value* const* in_values, int32_t warmup, int32_t iters,
                               double* ms_per_device, int32_t capacity, int32_t* n_devices);
/* Times every launch of device 0's plan separately; writes up to `capacity` entries. kinds receive
 * pointers valid until the next call on this session. */
SB_API int32_t sb_session_profile(sb_session* session, int32_t n_inputs, const char* const* in_names,
                           sb_value* const* in_values, int32_t iters, const char** kinds, double* ms,
                           int32_t capacity, int32_t* n_steps);
/* Plan statistics for these inputs: kernel launches per run, tensor-core launches, algorithmic
 * multiply-accumulates, device bytes (arena + weights), devices used. */
SB_API int32_t sb_session_stats(sb_session* session, int32_t n_inputs, const char* const* in_names,
                         sb_value* const* in_values, int64_t* launches, int64_t* tc_launches, double* macs,
                         int64_t* device_bytes, int32_t* devices_used);

/* Bytes a Run of these inputs copies host->device and device->host (a float32 input that the plan
 * only reads as bfloat16 and that Run has to stage from pageable memory travels as bfloat16). */
SB_API int32_t sb_session_transfer_bytes(sb_session* session, int32_t n_inputs, const char* const* in_names,
                                  sb_value* const* in_values, int64_t* h2d_bytes, int64_t* d2h_bytes);

/* ---- Allocation-free dense layer (no counterpart in the reference interface) -------------------
 * y[M,N] = x[M,K] * w[N,K]^T + bias[N] (ReLU when relu != 0): fp32 device buffers in and out, bf16
 * tensor-core arithmetic with fp32 accumulation, the same kernels a session uses for Linear layers.
 * For callers that cannot call cudaMalloc (pre-budgeted device memory, a host runtime that owns the
 * allocator, allocation-free hot loops): it allocates nothing. Its scratch (bf16 operand copies,
 * padded bias, error word) is one fixed 16 MiB device array that every GPU loading this library
 * holds until exit; sizes whose scratch exceeds it (M*round8(K)*2 + N*round64(K)*2 + ~1 KiB) are
 * rejected with SB_STATUS_INVALID_ARGUMENT. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) and caches it per device for the runtime's primary context (a
 * caller that makes its own driver-API context current is not supported), so make that first call
 * before any stream capture. All calls share
 * the array and the previous call's contents remain in it; calls that overlap on the GPU (other
 * streams, other threads) race on it. The call runs on `stream` (cudaStream_t, NULL = default) and
 * returns after it completes. bias may be NULL. */
SB_API int32_t sb_linear_noalloc(const float* x, const float* w, const float* bias, float* y, int64_t M, int64_t K,
                                 int64_t N, int32_t relu, void* stream);

/* ---- Diagnostics (no counterpart in the reference interface) ------------------------------- */
/* Lowers and fuses the model on the host only (no device needed) for inputs given in session input
 * order, and writes a summary (one line per device op, then "separable=0|1") into buf as a
 * NUL-terminated string; *needed receives the full length + 1. Each contraction's line ends with
 * "prec=A/B/C": its operand precision in a bf16 / TF32 / TF32x3 session. */
SB_API int32_t sb_debug_lower(const uint8_t* model, size_t model_len, int32_t n_inputs, sb_value* const* in_values,
                              char* buf, size_t capacity, size_t* needed);

/* The host narrowing a Run applies to a float32 input in pageable memory that the plan only reads
 * as bfloat16 (round to nearest even, NaN kept as a quiet NaN; the device's own rounding of a float32
 * operand, so the narrowed batch gives the same results): n values, up to `threads` host threads. */
SB_API int32_t sb_debug_narrow_bf16(const float* src, uint16_t* dst, size_t n, int32_t threads);

#ifdef __cplusplus
}
#endif

#endif /* SHOROKOO_B200_H_ */
