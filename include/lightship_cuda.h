/*
 * lightship_cuda.h -- C ABI of the B200 (sm_100a) CUDA backend for LightShip.
 *
 * The backend sits behind LightShip's `Backend` trait
 * (lightship-core/src/backend/backend.rs:128-163).  A Rust `backend/cuda.rs` binds the
 * functions below with an `extern "C"` block and implements the trait on top of them;
 * each declaration names the reference interface it replaces.  Status codes extend the
 * public LightShip C API's error enum (c-api/include/lightship.h:36-59) with the
 * backend error kinds of `BackendErrorCode` (backend.rs:9-23) and
 * `BackendError` (lightship-core/src/common/error.rs:79-103).
 *
 * Conventions
 *  - Plain pointers and sizes only.  `lsc_stream` is a cudaStream_t (NULL = legacy
 *    default stream).  Device pointers must belong to the calling thread's current
 *    device unless a backend handle says otherwise.
 *  - Every function is thread-safe and re-entrant.  None aborts, traps or waits without a
 *    bound: device-side waits give up after 2 s and raise LSC_ERROR_TIMEOUT.
 *  - On failure a function returns a non-zero lsc_status and stores a message that
 *    lsc_last_error() returns (per calling thread).
 *  - Kernel-level entry points (lsc_gemm_i8, lsc_quantize_f32, ...) are stream-ordered and
 *    return after the launch; errors raised on the device are reported by the next
 *    lsc_check_device / lsc_synchronize.
 */
#ifndef LIGHTSHIP_CUDA_H
#define LIGHTSHIP_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LSC_ABI_VERSION 1
#define LSC_MAX_DIMS 8

/* ---- status codes (lightship.h:36-59 + backend.rs:9-23) ----------------------------- */
typedef enum lsc_status {
  LSC_SUCCESS = 0,                     /* LIGHTSHIP_SUCCESS */
  LSC_ERROR = 1,                       /* LIGHTSHIP_ERROR */
  LSC_ERROR_INVALID_ARGUMENT = 2,      /* LIGHTSHIP_ERROR_INVALID_ARGUMENT / InvalidParameter */
  LSC_ERROR_OUT_OF_MEMORY = 3,         /* LIGHTSHIP_ERROR_OUT_OF_MEMORY / OutOfMemory */
  LSC_ERROR_BACKEND_NOT_AVAILABLE = 6, /* LIGHTSHIP_ERROR_BACKEND_NOT_AVAILABLE / NotAvailable */
  LSC_ERROR_SHAPE_MISMATCH = 7,        /* LIGHTSHIP_ERROR_SHAPE_MISMATCH */
  LSC_ERROR_UNSUPPORTED_DATATYPE = 8,  /* LIGHTSHIP_ERROR_UNSUPPORTED_DATATYPE */
  LSC_ERROR_DEVICE_ERROR = 9,          /* LIGHTSHIP_ERROR_DEVICE_ERROR */
  LSC_ERROR_NOT_IMPLEMENTED = 10,      /* LIGHTSHIP_ERROR_NOT_IMPLEMENTED */
  LSC_ERROR_UNSUPPORTED_OPERATOR = 11, /* BackendErrorCode::UnsupportedOperator */
  LSC_ERROR_COMPILATION_FAILED = 12,   /* BackendErrorCode::CompilationFailed */
  LSC_ERROR_EXECUTION_FAILED = 13,     /* BackendErrorCode::ExecutionFailed */
  LSC_ERROR_UNSUPPORTED_LAYOUT = 14,   /* BackendError::UnsupportedLayout */
  LSC_ERROR_TIMEOUT = 15               /* LightShipError::Timeout: a device wait ran out */
} lsc_status;

/* ---- data types (lightship.h:66-87, DataType in common/types.rs:5-44) --------------- */
typedef enum lsc_dtype {
  LSC_DTYPE_F32 = 0,
  LSC_DTYPE_F16 = 1,
  LSC_DTYPE_F64 = 2,
  LSC_DTYPE_I8 = 3,
  LSC_DTYPE_I16 = 4,
  LSC_DTYPE_I32 = 5,
  LSC_DTYPE_I64 = 6,
  LSC_DTYPE_U8 = 7,
  LSC_DTYPE_QUINT8 = 8,
  LSC_DTYPE_QINT8 = 9,
  LSC_DTYPE_QINT32 = 10
} lsc_dtype;

/* StorageLayout (lightship.h:90-97; common/types.rs) */
typedef enum lsc_layout {
  LSC_LAYOUT_NCHW = 0,
  LSC_LAYOUT_NHWC = 1,
  LSC_LAYOUT_OIHW = 2,
  LSC_LAYOUT_OHWI = 3, /* conv weight [Cout, KH, KW, Cin/groups] for NHWC kernels */
  LSC_LAYOUT_DEFAULT = 4
} lsc_layout;

/* Operators on the dense-contraction path (OperatorType, ir/operator.rs:9-100) */
typedef enum lsc_op_type {
  LSC_OP_CONV2D = 0,
  LSC_OP_FULLY_CONNECTED = 1,
  LSC_OP_MATMUL = 2,
  LSC_OP_BATCHNORM = 3,
  LSC_OP_RELU = 4,
  LSC_OP_RELU6 = 5,
  LSC_OP_SILU = 6,
  LSC_OP_QUANTIZE = 7,   /* quantize_tensor (quantization/helpers.rs:11-50) */
  LSC_OP_DEQUANTIZE = 8, /* dequantize_tensor (quantization/helpers.rs:53-94) */
  LSC_OP_QGEMM = 9,      /* quantized_gemm_int8 + requant/dequant (cpu/quantized_ops.rs:13-48) */
  LSC_OP_MAXPOOL2D = 10, /* MaxPool2d on int8 NHWC or f32 NCHW (operator/pooling.rs:383-455) */
  LSC_OP_GLOBAL_AVGPOOL2D = 11, /* GlobalAvgPool2d on int8 NHWC ([N, C] out) or f32 NCHW
                                   ([N, C, 1, 1] out, operator/pooling.rs:457-530) */
  LSC_OP_GELU = 12,      /* Gelu::compute, tanh form (operator/gelu.rs:77-103) */
  LSC_OP_LAYERNORM = 13, /* LayerNorm over the last axis (operator/layernorm.rs:140-205) */
  LSC_OP_SOFTMAX = 14,   /* Softmax over the last axis (operator/softmax.rs:106-169) */
  LSC_OP_ADD = 15        /* elementwise f32 Add (ir/operator.rs OperatorType::Add), with
                            FusionType::AddReLU (ir/fusion.rs:20) as activation ReLU */
} lsc_op_type;

/* FusionType (ir/fusion.rs:8-23); LSC_FUSION_NONE = no FusionInfo */
typedef enum lsc_fusion_type {
  LSC_FUSION_NONE = -1,
  LSC_FUSION_CONV_RELU = 0,
  LSC_FUSION_CONV_RELU6 = 1,
  LSC_FUSION_CONV_SIGMOID = 2,
  LSC_FUSION_CONV_BATCHNORM = 3,
  LSC_FUSION_BATCHNORM_RELU = 4,
  LSC_FUSION_ADD_RELU = 5,
  LSC_FUSION_MUL_RELU = 6
} lsc_fusion_type;

/* epilogue activations */
#define LSC_ACT_NONE 0
#define LSC_ACT_RELU 1  /* x > 0 ? x : 0           platform/simd.rs:552-556 */
#define LSC_ACT_RELU6 2 /* f32::clamp(x, 0, 6)     platform/simd.rs:558-562 */
#define LSC_ACT_SILU 3  /* x / (1 + exp(-x)), +-20 cut-offs  operator/silu.rs:47-61 */
#define LSC_ACT_GELU 4  /* 0.5x(1 + t(0.79788456(x + 0.044715x^3))), t the reference's polynomial
                           tanh (x - x^3/3 + x^5/5 - x^7/7, +-1 past +-5)  operator/gelu.rs:77-103 */

/* rounding of the requantize step */
#define LSC_ROUND_HALF_AWAY 0 /* Rust f32::round (cpu/quantized_ops.rs:45, helpers.rs:153) */
#define LSC_ROUND_HALF_EVEN 1

/* FP32 contraction mode */
#define LSC_FP32_3XTF32 0 /* split-TF32, three tensor-core products: ~fp32 accuracy */
#define LSC_FP32_TF32 1   /* single TF32 product: 10-bit mantissa inputs */
#define LSC_FP32_WINOGRAD 2 /* as LSC_FP32_3XTF32, with 3x3 stride-1 dilation-1 FP32 convolutions
                               run as Winograd F(2x2, 3x3) (cpu/winograd_conv2d.rs:50-397) */

/* tensor memory location */
#define LSC_MEM_HOST 0
#define LSC_MEM_DEVICE 1

typedef void* lsc_stream;
typedef struct lsc_backend lsc_backend;
typedef struct lsc_op lsc_op;

/* GpuBackendConfig (backend/backend.rs:81-96) plus the CUDA backend's extensions */
typedef struct lsc_config {
  int32_t device_id;    /* GpuBackendConfig::device_id */
  int32_t enable_fp16;  /* GpuBackendConfig::enable_fp16 (accepted, FP16 paths not used) */
  int32_t rounding;     /* default requantize rounding: LSC_ROUND_* */
  int32_t fp32_mode;    /* LSC_FP32_* */
  uint64_t arena_bytes; /* device arena size; 0 = 1 GiB */
} lsc_config;

/* BackendCapabilities subset (backend/capabilities.rs:46-67) */
typedef struct lsc_caps {
  int32_t backend_type; /* BackendType::GPU = 1 (lightship.h:104) */
  int32_t device_id;
  int32_t sm_count;
  int32_t cc_major, cc_minor;
  uint64_t total_memory;
  uint32_t memory_alignment;
  uint32_t supported_ops_mask; /* bit (1 << lsc_op_type) per supported operator */
} lsc_caps;

/* Quantization (ir/tensor.rs:9-18); count = 0 means "not quantized" */
typedef struct lsc_quant {
  const float* scale;
  const int32_t* zero_point;
  int32_t count;
  int32_t bit_width;
} lsc_quant;

/* Tensor (ir/tensor.rs:39-54) with its data either in host memory (TensorData::Owned bytes)
 * or on the device (the TensorData::Device variant this backend adds). */
typedef struct lsc_tensor {
  const char* name;
  int32_t ndim;
  int64_t shape[LSC_MAX_DIMS];
  int32_t dtype;    /* lsc_dtype */
  int32_t layout;   /* lsc_layout */
  int32_t location; /* LSC_MEM_HOST | LSC_MEM_DEVICE */
  int32_t device;
  void* data;
  uint64_t nbytes;
  lsc_quant quant;
} lsc_tensor;

/* OperatorDef (ir/operator.rs:200-226) with the attributes the dense path reads, plus
 * FusionInfo::fusion_type (ir/fusion.rs:41-49). */
typedef struct lsc_op_desc {
  int32_t op_type; /* lsc_op_type */
  int32_t fusion;  /* lsc_fusion_type */
  int32_t stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w, groups;
  int32_t activation;  /* extra epilogue activation, LSC_ACT_* */
  int32_t rounding;    /* LSC_ROUND_*, -1 = backend default */
  int32_t fp32_mode;   /* LSC_FP32_*, -1 = backend default */
  float bn_epsilon;    /* BatchNorm epsilon; 0 selects the reference default 1e-5
                          (operator/batchnorm.rs:49) */
  float output_scale;  /* s_out of a requantized int8 output */
  int32_t output_dtype; /* dtype of outputs[0] for QGEMM / quantized Conv2d */
  int32_t kernel_h, kernel_w; /* pooling window (Pool2dConfig, operator/pooling.rs) */
  /* Conv2d end padding relative to pad_h / pad_w: bottom = pad_h + pad_h_end_delta, right =
     pad_w + pad_w_end_delta (0 = symmetric, as Conv2dConfig's padding; a negative total crops).
     No counterpart in the reference: lets an INT8 input carry a row pitch padded for the
     pixel-grouped convolution. */
  int32_t pad_h_end_delta, pad_w_end_delta;
} lsc_op_desc;

/* Backend::allocate result (backend/memory.rs:32-45) */
typedef struct lsc_memory_block {
  uint64_t id;
  void* ptr;
  uint64_t size;
  uint64_t alignment;
  int32_t location; /* StorageLocation::GPU */
} lsc_memory_block;

/* ---- library ----------------------------------------------------------------------------- */
const char* lsc_version(void);               /* LightShip_GetVersion (lightship.h:29) */
const char* lsc_last_error(void);            /* per-thread; capi/handle.rs:593 pattern */
const char* lsc_status_string(int32_t code); /* LightShipError_GetMessage (lightship.h:62) */
int32_t lsc_device_count(void);

/* ---- Backend trait (backend/backend.rs:128-163) ------------------------------------------ */
lsc_status lsc_backend_create(const lsc_config* config, lsc_backend** out); /* GpuBackend ctor */
void lsc_backend_destroy(lsc_backend* backend);                             /* Drop */
int32_t lsc_backend_is_available(const lsc_backend* backend);               /* is_available */
lsc_status lsc_backend_capabilities(const lsc_backend* backend, lsc_caps* caps); /* capabilities */
/* compile_operator(def, fusion, inputs, outputs): weights/static inputs that carry data are
 * prepacked on the device now (BN fold, per-channel INT8 quantization, layout change).
 * Conv2d with groups > 1 takes the reference's grouped filter [Cout, Cin/groups, KH, KW]
 * (convolution.rs:105-122) and runs it as the dense convolution whose filter is zero outside
 * each output channel's group: exact, at groups x the MACs. */
lsc_status lsc_compile_operator(lsc_backend* backend, const lsc_op_desc* def,
                                const lsc_tensor* inputs, int32_t n_inputs,
                                const lsc_tensor* outputs, int32_t n_outputs, lsc_op** out);
/* execute(op, inputs, outputs): host or device tensors; sets outputs[i].shape/ndim. */
lsc_status lsc_execute(lsc_backend* backend, const lsc_op* op, const lsc_tensor* inputs,
                       int32_t n_inputs, lsc_tensor* outputs, int32_t n_outputs,
                       lsc_stream stream);
void lsc_op_destroy(lsc_op* op);
lsc_status lsc_allocate(lsc_backend* backend, uint64_t size, uint64_t alignment,
                        lsc_memory_block* block);                 /* allocate */
void lsc_deallocate(lsc_backend* backend, lsc_memory_block* block); /* deallocate */
lsc_status lsc_synchronize(lsc_backend* backend);                   /* synchronize */
/* arena statistics (memory/stats.rs:7-110): current and peak bytes in use */
lsc_status lsc_memory_stats(const lsc_backend* backend, uint64_t* current, uint64_t* peak,
                            uint64_t* capacity);
lsc_status lsc_memcpy_h2d(void* dst, const void* src, uint64_t bytes, lsc_stream stream);
lsc_status lsc_memcpy_d2h(void* dst, const void* src, uint64_t bytes, lsc_stream stream);

/* Reads (and clears) the current device's sticky device-error word: 0 = no error.  Returns
 * LSC_ERROR_TIMEOUT when a kernel gave up on a bounded wait. */
lsc_status lsc_check_device(uint32_t* word);

/* ---- kernel-level entry points (device pointers, stream-ordered) ------------------------- */

/* INT8 chain (cpu/quantized_ops.rs:13-48 with quantization/helpers.rs:139-160):
 *   acc[m,n] = sum_k A[m,k] * W[n,k]           (A [M,K] and W [N,K] row-major int8, exact i32)
 *   acc     += bias[n]                         (bias may be NULL)
 *   y        = (f32)acc * scale[n]             (scale has N entries)
 *   y        = act(y)                          (LSC_ACT_*)
 *   out_f32  = y ; out_i8 = (i8)clamp(R(y / s_out), -128, 127) ; out_i32 = acc
 * Any of out_i8 / out_f32 / out_i32 may be NULL (at least one must be given); each output
 * is row-major [M, N].  Needs K % 16 == 0 and 16-byte aligned A and W. */
lsc_status lsc_gemm_i8(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                       const int32_t* bias, const float* scale, float s_out, int32_t act,
                       int32_t rounding, int8_t* out_i8, float* out_f32, int32_t* out_i32,
                       lsc_stream stream);

/* INT8 convolution on NHWC activations, as an implicit GEMM with the INT8 chain's epilogue
 * (the quantized form of Conv2d::forward, operator/convolution.rs:90-267, with
 * Conv2dConfig's stride/padding/dilation, convolution.rs:12-62; groups = 1):
 *   x [N, H, W, C] int8 with C a multiple of 16 (pad channels with zeros),
 *   w [Cout, KH, KW, C] int8 (K ordered kh, kw, c), scale [Cout], bias [Cout] or NULL,
 *   outputs NHWC [N, OH, OW, Cout] with OH = (H + 2 ph - dh (KH-1) - 1) / sh + 1 (same for W).
 * `residual` (optional) is an int8 NHWC tensor shaped like the outputs, added before the
 * activation as (f32)r * residual_scale -- a ResNet block's Add+ReLU (FusionType::AddReLU,
 * ir/fusion.rs:20) fused into the second convolution.
 * Limits of the im2col load unit: stride <= 8, padding <= 127. */
lsc_status lsc_conv2d_i8_nhwc(const int8_t* x, const int8_t* w, int64_t n, int64_t h, int64_t wd,
                              int64_t c, int64_t c_out, int64_t kh, int64_t kw, int64_t sh,
                              int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw,
                              const int32_t* bias, const float* scale, float s_out, int32_t act,
                              int32_t rounding, int8_t* out_i8, float* out_f32, int32_t* out_i32,
                              const int8_t* residual, float residual_scale, lsc_stream stream);

/* quantize_tensor, per-tensor (quantization/helpers.rs:11-50 with quantize_value :139-155):
 *   q = clamp(sat_i32(R(x / scale)) + zero_point, qmin, qmax)   (i32 add wraps)
 * qdtype sets the storage: LSC_DTYPE_QINT8/I8 -> int8 out, QUINT8/U8 -> uint8, QINT32/I32 ->
 * int32.  The clamp range follows quantize_value: QINT8 [-128, 127], QINT32 the i32 range,
 * every other dtype (QUINT8, and plain I8 / U8 / I32 by the reference's `_` arm) [0, 255];
 * with I8 storage a code above 127 wraps as Rust's `as i8`.
 * R = LSC_ROUND_HALF_AWAY reproduces the reference; HALF_EVEN is offered as a variant. */
lsc_status lsc_quantize_f32(const float* x, void* out, int64_t n, int32_t qdtype, float scale,
                            int32_t zero_point, int32_t rounding, lsc_stream stream);
/* per-channel form (QuantizationParameters::new_per_channel, quantization/scheme.rs:75-90):
 * element i uses channel c = (i / inner) % channels; scales/zero_points are device arrays
 * (zero_points may be NULL = all zero). */
lsc_status lsc_quantize_f32_per_channel(const float* x, void* out, int64_t n, int32_t qdtype,
                                        const float* scales, const int32_t* zero_points,
                                        int32_t channels, int64_t inner, int32_t rounding,
                                        lsc_stream stream);
/* dequantize_tensor (quantization/helpers.rs:53-94, dequantize_value :158-160):
 *   x = ((f32)q - (f32)zero_point) * scale */
lsc_status lsc_dequantize(const void* q, int32_t qdtype, float* out, int64_t n, float scale,
                          int32_t zero_point, lsc_stream stream);
lsc_status lsc_dequantize_per_channel(const void* q, int32_t qdtype, float* out, int64_t n,
                                      const float* scales, const int32_t* zero_points,
                                      int32_t channels, int64_t inner, lsc_stream stream);
/* find_scale_zp (quantization/helpers.rs:101-136) over a device f32 array.  qdtype is any
 * lsc_dtype; (qmin, qmax) = QINT8 (-128, 127), QINT32 (INT32_MIN, INT32_MAX), any other
 * (0, 255) as the reference's `_` arm.  Writes the scale
 * and zero point to device memory.  `workspace` is caller-provided device scratch of at
 * least lsc_find_scale_zp_workspace_size() bytes (4-byte aligned); calls that share a
 * workspace must be ordered on one stream. */
uint64_t lsc_find_scale_zp_workspace_size(void);
lsc_status lsc_find_scale_zp_f32(const float* x, int64_t n, int32_t qdtype, int32_t symmetric,
                                 void* workspace, uint64_t workspace_bytes, float* scale_out,
                                 int32_t* zero_point_out, lsc_stream stream);
/* find_scale_zp applied per channel (the per-channel QuantizationParameters of
 * quantization/scheme.rs:75-90 calibrated with helpers.rs:101-136): x is [channels,
 * per_channel] row-major (a weight [Cout, K]); writes channels scales and zero points to
 * device memory.  `workspace`: caller-provided device scratch of at least
 * lsc_find_scale_zp_per_channel_workspace_size(channels) bytes (12 per channel). */
uint64_t lsc_find_scale_zp_per_channel_workspace_size(int64_t channels);
lsc_status lsc_find_scale_zp_per_channel_f32(const float* x, int64_t channels, int64_t per_channel,
                                             int32_t qdtype, int32_t symmetric, void* workspace,
                                             uint64_t workspace_bytes, float* scales_out,
                                             int32_t* zero_points_out, lsc_stream stream);
/* No counterpart in the reference.  lsc_find_scale_zp_per_channel_f32 for callers that
 * cannot allocate device memory -- code running inside a host runtime that owns the GPU's
 * memory (a framework's caching allocator, a serving process with a fixed budget), where a
 * cudaMalloc would synchronise the device and fail once the owner holds the memory.  It
 * takes no workspace and allocates nothing: its scratch is a static device array sized for
 * at most 16384 channels (192 KiB, held on every GPU that loads the library until exit);
 * more channels are rejected with LSC_ERROR_INVALID_ARGUMENT.  The array is reserved when
 * the library's CUDA module is loaded on a device; under lazy module loading (the CUDA 12
 * default) that is the first call, so make one call per device early, before the owner of
 * the memory has reserved the GPU, and before any stream capture (the first call also looks
 * up the array's address).  All calls share the array: calls that overlap on the GPU race
 * with each other; sequential calls do not. */
lsc_status lsc_find_scale_zp_per_channel_f32_noalloc(const float* x, int64_t channels,
                                                     int64_t per_channel, int32_t qdtype,
                                                     int32_t symmetric, float* scales_out,
                                                     int32_t* zero_points_out, lsc_stream stream);

/* ---- test hook of the bounded device waits ----------------------------------------------
 * No counterpart in the reference, which has no device waits; it tests the path that reports
 * LightShipError::Timeout (common/error.rs:32-34).  The next `launches` lsc_gemm_i8 calls made
 * by this thread that run on single CTAs (not CTA pairs) leave one operand copy of their first
 * tile unissued and give each device wait `wait_limit_ns` (1 ms .. 2 s) instead of 2 s: the
 * waits on that copy run out, the kernel drains what it issued, frees its tensor memory and
 * returns, the outputs are incomplete, and the next lsc_check_device / lsc_synchronize returns
 * LSC_ERROR_TIMEOUT.  Nothing faults; the device stays usable.  0 launches cancels. */
lsc_status lsc_debug_withhold_copy(int32_t launches, uint64_t wait_limit_ns);

/* ---- measurement -----------------------------------------------------------------------
 * No counterpart in the reference.  The tensor pipe's issue rate on operands resident in
 * shared memory: on `ctas` SMs at once (one CTA, or one CTA pair with cta_pair = 1, per SM),
 * one thread issues `iters` tcgen05.mma instructions of M = 128 (256 for a pair) x N (64, 128
 * or 256) x 32 bytes of K (kind 0: kind::i8; kind 1: kind::f16) and waits for them; returns
 * the median over CTAs of clock cycles and nanoseconds per instruction.  `mode` selects the
 * shape of the issue loop: 0 a flat loop; 1 the flat loop with an optional commit every
 * `commit_every` instructions and a wait for the commit `wait_lag` (0..7) back; 2 k-blocks of
 * four instructions with a commit per k-block and a bounded wait `wait_lag` k-blocks back; 3
 * as 2 with the whole warp looping and one elected lane issuing; 4 as 2 with a plain spin in
 * place of the timed wait.  The ceiling the contraction kernels' roofline fractions are read
 * against.  Allocates a few bytes of device memory for the results and synchronises. */
lsc_status lsc_probe_tensor_rate(int32_t kind, int32_t n, int32_t cta_pair, int32_t iters, int32_t ctas,
                                 int32_t mode, int32_t commit_every, int32_t wait_lag,
                                 double* cycles_per_mma, double* ns_per_mma);
/* No counterpart in the reference.  Operand delivery into shared memory: on `ctas` SMs, one
 * thread per CTA keeps `depth` (1..3) TMA tile loads of box_rows (64/128/256) x 128 bytes x
 * `chunks` (1, 2 or 4 consecutive 128-byte column blocks, a 3-D box, at most 64 KB) in flight
 * from the device buffer `src` (`bytes` long, rows `row_pitch` bytes apart, 128-byte
 * aligned), all slots within 192 KB; `same` = 1 makes every CTA read the same rows.  The
 * producers are lane 0 of as many warps (mode 0: waits as the kernels do, bounded and timed;
 * mode 1: a non-suspending spin) or lanes of one warp (mode 2).  Returns bytes per SM
 * clock (median
 * CTA) and the whole GPU's GB/s.  With the issue-loop modes above, the two probes separate
 * the MMA pipe, the stage-release cadence and operand delivery.  Synchronises the device. */
/* No counterpart in the reference.  The same for im2col loads, the convolutions' A operand:
 * `src` is an NHWC int8 tensor [n, h, w, 128] (128-byte aligned); every load brings 128 output
 * pixels x 128 channels of one tap of a 3x3, padding-1 filter (16 KB); `producers` (1..4)
 * warps keep `depth` loads each in flight. */
lsc_status lsc_probe_im2col_rate(const void* src, int64_t n, int64_t h, int64_t w, int32_t depth,
                                 int32_t producers, int32_t iters, int32_t ctas, double* bytes_per_clock,
                                 double* gbytes_per_s);
lsc_status lsc_probe_tma_rate(const void* src, uint64_t bytes, int64_t row_pitch, int32_t box_rows,
                              int32_t chunks, int32_t depth, int32_t producers, int32_t same, int32_t iters,
                              int32_t ctas, int32_t mode, double* bytes_per_clock, double* gbytes_per_s);

/* ---- FP16 attention products (transformer block) ---------------------------------------
 * Batched C[bb][m][n] = alpha * sum_k A[bb][m][k] * B[bb][n][k] on the tensor cores (f16
 * operands, f32 accumulation), bb = b * heads + h.  Operand element (bb, row, k) is at
 * a + b*as_batch + (h + a_head0)*as_head + row*as_row + k (f16 elements; k contiguous; strides
 * multiples of 8; base 16-byte aligned; K a multiple of 8), likewise for b; C element
 * (bb, m, n) is at c + b*cs_batch + h*cs_head + m*cs_row + n, c_dtype LSC_DTYPE_F16 or F32.
 * Serves scores = Q K^T / sqrt(d) and O = P V of the reference's attention
 * (core/operator/attention.rs) on the FP16 path of the BERT-shaped workload; the reference's
 * CPU backend has no FP16 kernel of its own. */
lsc_status lsc_gemm_f16_batched(const void* a, int64_t as_row, int64_t as_head, int64_t as_batch,
                                int64_t a_head0, const void* b, int64_t bs_row, int64_t bs_head,
                                int64_t bs_batch, int64_t b_head0, int64_t batch, int64_t heads,
                                int64_t m, int64_t n, int64_t k, float alpha, void* c,
                                int32_t c_dtype, int64_t cs_row, int64_t cs_head, int64_t cs_batch,
                                lsc_stream stream);
/* y[b][h][c][r] = x[b][h + head0][r][c] (f16; x strides in elements), the K-major layout of V
 * for O = P V.  No counterpart in the reference. */
lsc_status lsc_transpose_heads_f16(const void* x, void* y, int64_t x_batch_stride,
                                   int64_t x_head_stride, int64_t x_row_stride, int64_t head0,
                                   int64_t batch, int64_t heads, int64_t rows, int64_t cols,
                                   lsc_stream stream);

/* Fused multi-head attention of an encoder block: for each batch b, head h and query q,
 *   out[b, q, h, :] = sum_k P[q, k] V[b, k, h, :],  P = f16(softmax_k(f16(alpha * Q[b,q,h,:] . K[b,k,h,:])))
 * with f32 accumulation -- what lsc_gemm_f16_batched (scores), the Softmax operator and
 * lsc_gemm_f16_batched (P V) compute in sequence, without the [batch, heads, seq, seq] scores
 * in memory.  qkv is the f16 QKV projection [batch, seq, 3, heads, 64] (Q, K, V head-major),
 * 16-byte aligned.  Outputs
 * [batch, seq, heads, 64]: out_f32 (32-byte aligned) and/or out_i8, the latter quantized
 * per tensor with s_out (quantize_value's arithmetic, `rounding` as lsc_rounding).  seq a
 * multiple of 128 up to 384, head dim 64.  Replaces the attention the reference declares
 * (core/ir/operator.rs:54-58, core/operator/attention.rs), whose CPU backend has no kernel;
 * the softmax is operator/softmax.rs:106-146.  A row whose scores hold an infinity or NaN
 * yields NaN outputs. */
lsc_status lsc_attention_f16(const void* qkv, int64_t batch, int64_t seq, int64_t heads, float alpha,
                             float* out_f32, int8_t* out_i8, float s_out, int32_t rounding, lsc_stream stream);

/* ---- models and sessions (ONNX; FP32 NCHW graphs) ----------------------------------------
 * An ONNX model loaded from memory (LightShipEngine_LoadModelFromMemory, lightship.h:186-198;
 * OnnxLoader, model/onnx.rs).  Node attributes (strides, pads, dilations, group, epsilon,
 * kernel_shape, transB, axis) are read; the reference's parser skips them (onnx.rs:613).
 * Loading runs the graph optimizer's fusion pass (FusionPass, ir/optimizer.rs:505-890, with
 * its single-consumer rule): Conv->BatchNormalization->Relu|Clip(0,6) becomes one Conv with
 * FusionType::ConvBatchNorm and the activation, Conv->Relu ConvReLU, Add->Relu AddReLU,
 * BatchNormalization->Relu BatchNormReLU.  Supported ONNX operators: Conv, BatchNormalization,
 * Relu, Clip(0, 6), Add, MaxPool, GlobalAveragePool, Flatten, Reshape (constant shape), Gemm /
 * MatMul (constant right operand -> FullyConnected), Softmax, LayerNormalization, Gelu; any
 * other operator fails the load with LSC_ERROR_UNSUPPORTED_OPERATOR. */
typedef struct lsc_model lsc_model;
typedef struct lsc_session lsc_session;
lsc_status lsc_model_load_onnx(const uint8_t* data, uint64_t size, lsc_model** out);
void lsc_model_destroy(lsc_model* model);                  /* LightShipModel_Destroy */
/* LightShipModel_GetMetadata (lightship.h:208-214): counts after fusion */
lsc_status lsc_model_info(const lsc_model* model, uint32_t* n_inputs, uint32_t* n_outputs,
                          uint32_t* n_nodes);
/* LightShipModel_GetInputInfo / GetOutputInfo (lightship.h:226-258); shape needs
 * LSC_MAX_DIMS entries; -1 marks a symbolic dimension */
lsc_status lsc_model_io(const lsc_model* model, int32_t is_output, uint32_t index, const char** name,
                        int32_t* dtype, int64_t* shape, uint32_t* ndim);
/* The Backend operator node `index` of the fused graph lowers to (op_type -1: a view such as
 * Flatten, no kernel), its name and its ONNX operator. */
lsc_status lsc_model_node(const lsc_model* model, uint32_t index, lsc_op_desc* desc,
                          const char** name, const char** onnx_op);
/* LightShipEngine_CreateSession (lightship.h:283-297): compiles every node on `backend` (weights
 * prepacked once) and takes one arena buffer per intermediate tensor; the model's inputs need
 * static shapes.  The session keeps `model` and `backend` in use until it is destroyed. */
lsc_status lsc_session_create(lsc_backend* backend, const lsc_model* model, lsc_session** out);
void lsc_session_destroy(lsc_session* session); /* LightShipSession_Destroy */
/* LightShipSession_Run (lightship.h:319-331): inputs and outputs in the model's order, f32,
 * host or device memory; runs every node on `stream` (host outputs are complete on return). */
lsc_status lsc_session_run(lsc_session* session, const lsc_tensor* inputs, uint32_t n_inputs,
                           lsc_tensor* outputs, uint32_t n_outputs, lsc_stream stream);

/* ---- INT8 sessions ---------------------------------------------------------------------
 * LightShipEngine_CreateSession (lightship.h:283-297) with the backend's precision choice.
 * precision LSC_PRECISION_F32 is lsc_session_create.  LSC_PRECISION_INT8 compiles an ONNX CNN
 * (Conv with BatchNormalization / Relu / Clip fused, residual Add(+Relu), MaxPool,
 * GlobalAveragePool, Flatten / Reshape, a final Gemm / MatMul classifier; one f32 NCHW input
 * of static shape) into the INT8 chain: per-output-channel INT8 filters with BN folded, the
 * residual Add fused into the convolution that feeds it, per-tensor activation scales
 * calibrated with find_scale_zp (quantization/helpers.rs:101-136) on `calibration` (an f32
 * batch of the input's shape, host or device), int8 NHWC activations carved from one arena
 * block by live range (plan_memory = 1) or one buffer each (0), and the whole network captured
 * by the library as a CUDA graph, with a convolution that reads the same tensor as the one
 * before it on a second stream (concurrent = 1).  The output is the classifier's f32 logits. */
#define LSC_PRECISION_F32 0
#define LSC_PRECISION_INT8 1
typedef struct lsc_session_options {
  int32_t precision;             /* LSC_PRECISION_* */
  int32_t rounding;              /* INT8 requantize rounding LSC_ROUND_*, -1 = the backend's default */
  int32_t concurrent;            /* 1 = independent sibling convolutions on a second stream */
  int32_t plan_memory;           /* 1 = activations share one block by live range */
  const lsc_tensor* calibration; /* INT8: the calibration batch */
} lsc_session_options;
lsc_status lsc_session_create_ex(lsc_backend* backend, const lsc_model* model, const lsc_session_options* options,
                                 lsc_session** out);
/* LightShipSession_Run, pipelined (INT8 sessions): enqueues one run on `stream` and returns.
 * Host inputs are uploaded on the session's own copy stream into one of two input slots, so
 * the next call's upload overlaps this call's network; the output is written when the stream
 * reaches it (a host output should be pinned memory).  Host inputs must stay unchanged until
 * the stream has passed this call.  Calls on one session must use one stream. */
lsc_status lsc_session_run_async(lsc_session* session, const lsc_tensor* inputs, uint32_t n_inputs,
                                 lsc_tensor* outputs, uint32_t n_outputs, lsc_stream stream);
/* The device buffer behind input slot 0 (is_output = 0) or the output (1) of an INT8 session.
 * An lsc_session_run whose input data is this buffer, or whose output data is the output
 * buffer, copies nothing for it.  No counterpart in the reference (its tensors are host bytes). */
lsc_status lsc_session_io_buffer(lsc_session* session, int32_t is_output, uint32_t index, void** device_ptr,
                                 uint64_t* bytes);
/* The INT8 session's activation memory: the planned block (peak, MemoryPlan::peak_memory in
 * executor/plan.rs:67-118) against the sum of one buffer per activation (total_memory), and
 * the number of activations. */
lsc_status lsc_session_memory_plan(const lsc_session* session, uint64_t* planned_bytes, uint64_t* unplanned_bytes,
                                   uint32_t* values);
/* An INT8 session's activation `tensor_name` (an ONNX tensor name; the quantized input is the
 * input's name + ":q"): its calibrated scale, its device buffer and an NHWC int8 description.
 * With plan_memory = 1 the buffer may hold a later activation once the run has moved on. */
lsc_status lsc_session_value(const lsc_session* session, const char* tensor_name, float* scale, void** device_ptr,
                             lsc_tensor* desc);

#ifdef __cplusplus
}
#endif
#endif /* LIGHTSHIP_CUDA_H */
