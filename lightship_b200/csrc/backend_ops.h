// backend_ops.h -- internal types of the Backend implementation: the backend and
// compiled-operator objects behind the opaque C handles, host/device staging of tensors,
// and the per-operator compile/execute entry points (backend_ops.cpp).
#pragma once
#include <atomic>
#include <initializer_list>
#include <vector>

#include "arena.h"
#include "lsc_internal.h"

// The backend object is reference counted: every compiled operator holds a reference, so
// destroying the backend before its operators (in any order) is safe.
struct lsc_backend {
  int device = 0;
  lsc_config cfg{};
  lsc::DeviceState* ds = nullptr;
  lsc::Arena arena;
  std::atomic<uint64_t> next_id{1};
  std::atomic<int> refs{1};
  void retain() { refs.fetch_add(1); }
  void release();
};

// What a compiled operator runs.
enum class OpKind {
  kQGemm,          // INT8 chain, weight [N, Kp] K-major
  kConvI8,         // INT8 NHWC implicit-GEMM convolution
  kQuantize,       // f32 -> q
  kDequantize,     // q -> f32
  kMatMulF32,      // C = A[M,K] B[K,N]
  kFcF32,          // Y = X W^T (+ bias)
  kLayerNorm,      // LayerNorm over the last axis (f32 / f16)
  kSoftmax,        // Softmax over the last axis (f32 / f16)
  kConvF32,        // NCHW convolution (+ folded BN, bias, activation)
  kBatchNormF32,   // per-channel affine (+ ReLU)
  kActF32,         // ReLU / ReLU6 / SiLU
  kMaxPoolI8,      // MaxPool2d on int8 NHWC
  kAvgPoolI8,      // GlobalAvgPool2d on int8 NHWC
  kMaxPoolF32,     // MaxPool2d on f32 NCHW
  kAvgPoolF32,     // GlobalAvgPool2d on f32 NCHW
  kAddF32,         // elementwise Add (+ ReLU)
};

struct lsc_op {
  lsc_backend* be = nullptr;
  lsc_op_desc desc{};
  OpKind kind = OpKind::kQGemm;
  int rounding = LSC_ROUND_HALF_AWAY;
  int fp32_mode = LSC_FP32_3XTF32;
  int act = LSC_ACT_NONE;

  // contraction operands prepacked at compile time (arena memory owned by the op)
  int64_t n = 0, k = 0, kp = 0;  // output channels, reduction length, padded reduction
  void* w = nullptr;             // weights in the kernel's layout
  void* w_lo = nullptr;          // low part of split-TF32 weights
  int32_t* bias_i32 = nullptr;
  float* bias_f32 = nullptr;
  float* scale = nullptr;        // per-output-channel dequant scale (s_a * s_w[n])
  float s_out = 1.0f;

  // convolution geometry
  int64_t c_in = 0, kh = 1, kw = 1;
  int32_t sh = 1, sw = 1, ph = 0, pw = 0, dh = 1, dw = 1, groups = 1;
  int32_t ph_end = 0, pw_end = 0;  // bottom / right padding
  // FP32 Winograd F(2x2, 3x3) form (fp32_mode LSC_FP32_WINOGRAD on a 3x3 stride-1 dilation-1
  // convolution with symmetric padding): w / w_lo then hold the transformed filter
  // U = G g G^T as [16][Cout][kp] split-TF32 halves.
  bool winograd = false;

  // pixel-grouped form of a stride-1 INT8 convolution (group_px > 1): the NHWC input viewed
  // as [N, H, W/G, G*C] and the filter expanded to [G*Cout, KH, kw_g, G*C], so that each
  // im2col request moves G pixels; output column (g, o) is pixel G*x + g, channel o, which
  // is the NHWC output's own layout.  Used when W and OW are multiples of G at execute time.
  int32_t group_px = 1, kw_g = 0, pw_g = 0;
  void* w_grouped = nullptr;
  int32_t* bias_grouped = nullptr;
  float* scale_grouped = nullptr;

  // quantize / dequantize / batchnorm parameters
  int32_t qdtype = LSC_DTYPE_QINT8;
  int32_t q_channels = 0;            // 0 = per tensor
  float q_scale0 = 1.0f;
  int32_t q_zp0 = 0;
  float* q_scales = nullptr;         // device, per channel
  int32_t* q_zps = nullptr;          // device, per channel
  int32_t q_axis = 1;

  std::vector<void*> owned;  // arena blocks released with the op
  ~lsc_op();
};

namespace lsc {

int64_t dtype_size(int32_t dt);
bool is_int8(int32_t dt);
int64_t numel(const lsc_tensor& t);
void set_shape(lsc_tensor& t, std::initializer_list<int64_t> dims);
lsc_status read_tensor_bytes(const lsc_tensor& t, int64_t bytes, std::vector<uint8_t>& out);
lsc_status upload(lsc_backend* be, const void* host, int64_t bytes, void** dptr);
uint32_t supported_ops_mask();

class DeviceGuard {
 public:
  explicit DeviceGuard(int dev);
  ~DeviceGuard();
  bool ok() const { return ok_; }

 private:
  int prev_ = -1;
  bool ok_ = true;
};

// Gives kernels device pointers for host or device tensors of one execute call.
struct Staging {
  lsc_backend* be = nullptr;
  cudaStream_t st = nullptr;
  bool touched_host = false;
  struct Down {
    void* host;
    void* dev;
    int64_t bytes;
  };
  std::vector<void*> temps;
  std::vector<Down> downs;
  lsc_status input(const lsc_tensor& t, int64_t bytes, const void** dptr);
  lsc_status output(lsc_tensor& t, int64_t bytes, void** dptr);
  void* scratch(int64_t bytes);
  // Downloads host outputs, synchronises when host memory was involved, releases scratch.
  lsc_status finish(lsc_status st_in);
};

// backend_conv.cpp
lsc_status compile_conv(lsc_op* op, const lsc_tensor* in, int n_in, const lsc_tensor* out, int n_out);
lsc_status execute_conv(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out, int n_out,
                        Staging& s);
// The INT8 session's fused stem: compiled pixel-grouped ReLU convolution `op` and the 3x3 / 2
// max pool of padding 1 after it, in one launch, into the pooled int8 NHWC y (device tensors).
// LSC_ERROR_UNSUPPORTED_OPERATOR (nothing launched) when the convolution does not qualify.
lsc_status execute_conv_pool(const lsc_op* op, const lsc_tensor& x, lsc_tensor& y, cudaStream_t st);
lsc_status compile_matmul_f32(lsc_op* op, const lsc_tensor* in, int n_in, int n_out);
lsc_status execute_matmul_f32(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                              int n_out, Staging& s);
lsc_status compile_fc_f32(lsc_op* op, const lsc_tensor* in, int n_in, int n_out);
lsc_status execute_fc_f32(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                          int n_out, Staging& s);
lsc_status compile_batchnorm(lsc_op* op, const lsc_tensor* in, int n_in, int n_out);
lsc_status execute_batchnorm(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                             int n_out, Staging& s);
lsc_status compile_pool(lsc_op* op, const lsc_tensor* in, int n_in, int n_out, bool global);
lsc_status execute_pool(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out, int n_out,
                        Staging& s);
lsc_status compile_activation(lsc_op* op, const lsc_tensor* in, int n_in, int n_out, int act);
lsc_status compile_add(lsc_op* op, const lsc_tensor* in, int n_in, int n_out);
lsc_status execute_add(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out, int n_out, Staging& s);
lsc_status compile_layernorm(lsc_op* op, const lsc_tensor* in, int n_in, const lsc_tensor* out, int n_out);
lsc_status compile_softmax(lsc_op* op, const lsc_tensor* in, int n_in, int n_out);
lsc_status execute_rownorm(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out, int n_out,
                           Staging& s);
lsc_status execute_activation(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                              int n_out, Staging& s);

lsc_status compile_op(lsc_backend* be, lsc_op* op, const lsc_tensor* in, int n_in,
                      const lsc_tensor* out, int n_out);
lsc_status execute_op(lsc_backend* be, const lsc_op* op, const lsc_tensor* in, int n_in,
                      lsc_tensor* out, int n_out, Staging& s);

}  // namespace lsc
