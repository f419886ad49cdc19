// runtime.cu -- error reporting, per-device state, tensor-map encoding and the
// stateless kernel-level C entry points.
#include <stdarg.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "lsc_internal.h"
#include "sm100.cuh"

namespace lsc {

namespace {
thread_local char t_last_error[1024] = "";

// Sticky per-device error word.  Kernels receive its device address (taken once per
// device in device_state) and atomically OR LSC_DEVERR_* bits into it.
__device__ uint32_t g_device_error_word;

constexpr int kMaxDevices = 64;
std::mutex g_state_mu;
DeviceState g_states[kMaxDevices];
bool g_state_ready[kMaxDevices] = {};
}  // namespace

lsc_status set_error(lsc_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

lsc_status cuda_error(cudaError_t e, const char* what) {
  const lsc_status code =
      e == cudaErrorMemoryAllocation ? LSC_ERROR_OUT_OF_MEMORY : LSC_ERROR_DEVICE_ERROR;
  return set_error(code, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

DeviceState* device_state(int device) {
  if (device < 0 || device >= kMaxDevices) {
    set_error(LSC_ERROR_INVALID_ARGUMENT, "device %d out of range", device);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_state_mu);
  if (g_state_ready[device]) return &g_states[device];
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) {
    cuda_error(e, "cudaGetDevice");
    return nullptr;
  }
  if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess) {
    cuda_error(e, "cudaSetDevice");
    return nullptr;
  }
  DeviceState s;
  s.device = device;
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e == cudaSuccess) {
    s.sm_count = prop.multiProcessorCount;
    s.cc_major = prop.major;
    s.cc_minor = prop.minor;
    s.smem_optin = prop.sharedMemPerBlockOptin;
    s.total_memory = prop.totalGlobalMem;
    const char* ov = getenv("LSC_OVERLAP_LAUNCHES");
    s.overlap_launches = !(ov && ov[0] == '0');
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_device_error_word);
    s.err_word = static_cast<uint32_t*>(addr);
  }
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    cuda_error(e, "device set-up");
    return nullptr;
  }
  g_states[device] = s;
  g_state_ready[device] = true;
  return &g_states[device];
}

DeviceState* current_device_state() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cuda_error(e, "cudaGetDevice");
    return nullptr;
  }
  return device_state(dev);
}

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

lsc_status encode(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, const void* base,
                  const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                  const cuuint32_t* estr, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(LSC_ERROR_DEVICE_ERROR, "cuTensorMapEncodeTiled unavailable");
  const CUresult r = fn(map, dtype, rank, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (CUresult %d)",
                     static_cast<int>(r));
  return LSC_SUCCESS;
}
typedef CUresult (*EncodeIm2colFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const int*, const int*,
                                   cuuint32_t, cuuint32_t, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeIm2colFn encode_im2col_fn() {
  static std::once_flag once;
  static EncodeIm2colFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeIm2colFn>(p);
  });
  return fn;
}
}  // namespace

lsc_status encode_tmap_im2col(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                              const uint64_t dims[4], const uint64_t strides_bytes[3],
                              const int lower[2], const int upper[2], uint32_t channels_per_pixel,
                              uint32_t pixels_per_column, const uint32_t elem_strides[4],
                              CUtensorMapSwizzle swizzle) {
  EncodeIm2colFn fn = encode_im2col_fn();
  if (!fn) return set_error(LSC_ERROR_DEVICE_ERROR, "cuTensorMapEncodeIm2col unavailable");
  const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t s[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  const cuuint32_t e[4] = {elem_strides[0], elem_strides[1], elem_strides[2], elem_strides[3]};
  const CUresult r = fn(map, dtype, 4, const_cast<void*>(base), d, s, lower, upper,
                        channels_per_pixel, pixels_per_column, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "cuTensorMapEncodeIm2col failed (CUresult %d)",
                     static_cast<int>(r));
  return LSC_SUCCESS;
}

lsc_status encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                          uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                          uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, dtype, 2, base, dims, strides, box, estr, swizzle);
}

lsc_status encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                          const uint64_t dims[3], const uint64_t strides_bytes[2],
                          const uint32_t box[3], const uint32_t elem_strides[3],
                          CUtensorMapSwizzle swizzle) {
  const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  const cuuint64_t s[2] = {strides_bytes[0], strides_bytes[1]};
  const cuuint32_t b[3] = {box[0], box[1], box[2]};
  const cuuint32_t e[3] = {elem_strides[0], elem_strides[1], elem_strides[2]};
  return encode(map, dtype, 3, base, d, s, b, e, swizzle);
}

lsc_status encode_tmap_4d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                          const uint64_t dims[4], const uint64_t strides_bytes[3],
                          const uint32_t box[4], const uint32_t elem_strides[4],
                          CUtensorMapSwizzle swizzle) {
  const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t s[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  const cuuint32_t b[4] = {box[0], box[1], box[2], box[3]};
  const cuuint32_t e[4] = {elem_strides[0], elem_strides[1], elem_strides[2], elem_strides[3]};
  return encode(map, dtype, 4, base, d, s, b, e, swizzle);
}

}  // namespace lsc

using namespace lsc;

extern "C" {

const char* lsc_version(void) { return "lightship-b200 0.1.0 (sm_100a)"; }

const char* lsc_last_error(void) { return t_last_error; }

const char* lsc_status_string(int32_t code) {
  switch (code) {
    case LSC_SUCCESS: return "success";
    case LSC_ERROR: return "error";
    case LSC_ERROR_INVALID_ARGUMENT: return "invalid argument";
    case LSC_ERROR_OUT_OF_MEMORY: return "out of memory";
    case LSC_ERROR_BACKEND_NOT_AVAILABLE: return "backend not available";
    case LSC_ERROR_SHAPE_MISMATCH: return "tensor shape mismatch";
    case LSC_ERROR_UNSUPPORTED_DATATYPE: return "data type not supported";
    case LSC_ERROR_DEVICE_ERROR: return "device error";
    case LSC_ERROR_NOT_IMPLEMENTED: return "not implemented";
    case LSC_ERROR_UNSUPPORTED_OPERATOR: return "operator not supported";
    case LSC_ERROR_COMPILATION_FAILED: return "compilation failed";
    case LSC_ERROR_EXECUTION_FAILED: return "execution failed";
    case LSC_ERROR_UNSUPPORTED_LAYOUT: return "layout not supported";
    case LSC_ERROR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

int32_t lsc_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

lsc_status lsc_check_device(uint32_t* word) {
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  LSC_CUDA_TRY(cudaDeviceSynchronize());
  uint32_t w = 0;
  LSC_CUDA_TRY(cudaMemcpy(&w, ds->err_word, sizeof(w), cudaMemcpyDeviceToHost));
  if (w) {
    const uint32_t zero = 0;
    LSC_CUDA_TRY(cudaMemcpy(ds->err_word, &zero, sizeof(zero), cudaMemcpyHostToDevice));
  }
  if (word) *word = w;
  if (w & LSC_DEVERR_TIMEOUT)
    return set_error(LSC_ERROR_TIMEOUT, "a kernel gave up on a bounded device wait");
  if (w) return set_error(LSC_ERROR_EXECUTION_FAILED, "device error word 0x%x", w);
  return LSC_SUCCESS;
}

lsc_status lsc_memcpy_h2d(void* dst, const void* src, uint64_t bytes, lsc_stream stream) {
  if (bytes == 0) return LSC_SUCCESS;
  if (!dst || !src) return set_error(LSC_ERROR_INVALID_ARGUMENT, "memcpy_h2d: null pointer");
  LSC_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice,
                               static_cast<cudaStream_t>(stream)));
  return LSC_SUCCESS;
}

lsc_status lsc_memcpy_d2h(void* dst, const void* src, uint64_t bytes, lsc_stream stream) {
  if (bytes == 0) return LSC_SUCCESS;
  if (!dst || !src) return set_error(LSC_ERROR_INVALID_ARGUMENT, "memcpy_d2h: null pointer");
  LSC_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost,
                               static_cast<cudaStream_t>(stream)));
  return LSC_SUCCESS;
}

lsc_status lsc_gemm_i8(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                       const int32_t* bias, const float* scale, float s_out, int32_t act,
                       int32_t rounding, int8_t* out_i8, float* out_f32, int32_t* out_i32,
                       lsc_stream stream) {
  return launch_gemm_i8(a, w, m, n, k, bias, scale, s_out, act, rounding, out_i8, out_f32,
                        out_i32, n, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
