// backend.cpp -- the CUDA backend behind LightShip's `Backend` trait
// (lightship-core/src/backend/backend.rs:128-163), exported through the C ABI of
// include/lightship_cuda.h.
//
//   lsc_backend_create        GpuBackend construction (GpuBackendConfig, backend.rs:81-96)
//   lsc_compile_operator      Backend::compile_operator: validates shapes, prepacks weights
//                             on the device (BN fold, per-channel INT8 quantization,
//                             transposes and K padding) -- work the CPU backend redoes on
//                             every execute (cpu.rs:161-174 compiles nothing)
//   lsc_execute               Backend::execute: host (TensorData::Owned) or device tensors;
//                             sets the output shapes (the executor passes [1] placeholders,
//                             executor/graph_executor.rs:148)
//   lsc_allocate/deallocate   Backend::allocate/deallocate from the device arena
//   lsc_synchronize           Backend::synchronize
// Unlike CpuBackend::execute (cpu.rs:205-211), an operator this backend cannot run is an
// error (LSC_ERROR_UNSUPPORTED_OPERATOR), never a silent Ok.
#include <math.h>
#include <string.h>

#include <atomic>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <vector>

#include "arena.h"
#include "backend_ops.h"
#include "lsc_internal.h"

using namespace lsc;

namespace lsc {

int64_t dtype_size(int32_t dt) {
  switch (dt) {
    case LSC_DTYPE_F32:
    case LSC_DTYPE_I32:
    case LSC_DTYPE_QINT32: return 4;
    case LSC_DTYPE_F16:
    case LSC_DTYPE_I16: return 2;
    case LSC_DTYPE_F64:
    case LSC_DTYPE_I64: return 8;
    case LSC_DTYPE_I8:
    case LSC_DTYPE_U8:
    case LSC_DTYPE_QINT8:
    case LSC_DTYPE_QUINT8: return 1;
    default: return 0;
  }
}

bool is_int8(int32_t dt) { return dt == LSC_DTYPE_I8 || dt == LSC_DTYPE_QINT8; }

int64_t numel(const lsc_tensor& t) {
  if (t.ndim < 0 || t.ndim > LSC_MAX_DIMS) return -1;
  int64_t n = 1;
  for (int i = 0; i < t.ndim; ++i) {
    if (t.shape[i] < 0) return -1;
    n *= t.shape[i];
  }
  return n;
}

DeviceGuard::DeviceGuard(int dev) {
  if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
  if (prev_ != dev) ok_ = cudaSetDevice(dev) == cudaSuccess;
}
DeviceGuard::~DeviceGuard() {
  int cur = -1;
  if (prev_ >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev_) cudaSetDevice(prev_);
}

// ------------------------------------------------------------------------- staging
lsc_status Staging::input(const lsc_tensor& t, int64_t bytes, const void** dptr) {
  if (bytes < 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "input '%s': bad shape", t.name ? t.name : "");
  if (bytes > 0 && !t.data) return set_error(LSC_ERROR_INVALID_ARGUMENT, "input '%s' has no data", t.name ? t.name : "");
  if (t.nbytes && t.nbytes < static_cast<uint64_t>(bytes))
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "input '%s': %llu bytes given, %lld needed",
                     t.name ? t.name : "", (unsigned long long)t.nbytes, (long long)bytes);
  if (t.location == LSC_MEM_DEVICE) {
    *dptr = t.data;
    return LSC_SUCCESS;
  }
  void* d = be->arena.alloc(static_cast<size_t>(bytes), 256);
  if (!d) return set_error(LSC_ERROR_OUT_OF_MEMORY, "arena: no room for %lld bytes", (long long)bytes);
  temps.push_back(d);
  touched_host = true;
  LSC_CUDA_TRY(cudaMemcpyAsync(d, t.data, static_cast<size_t>(bytes), cudaMemcpyHostToDevice, st));
  *dptr = d;
  return LSC_SUCCESS;
}

lsc_status Staging::output(lsc_tensor& t, int64_t bytes, void** dptr) {
  if (bytes > 0 && !t.data)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "output '%s' has no buffer", t.name ? t.name : "");
  if (t.nbytes && t.nbytes < static_cast<uint64_t>(bytes))
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "output '%s': %llu bytes given, %lld needed",
                     t.name ? t.name : "", (unsigned long long)t.nbytes, (long long)bytes);
  if (t.location == LSC_MEM_DEVICE) {
    *dptr = t.data;
    return LSC_SUCCESS;
  }
  void* d = be->arena.alloc(static_cast<size_t>(bytes), 256);
  if (!d) return set_error(LSC_ERROR_OUT_OF_MEMORY, "arena: no room for %lld bytes", (long long)bytes);
  temps.push_back(d);
  downs.push_back({t.data, d, bytes});
  touched_host = true;
  *dptr = d;
  return LSC_SUCCESS;
}

void* Staging::scratch(int64_t bytes) {
  void* d = be->arena.alloc(static_cast<size_t>(bytes), 256);
  if (d) temps.push_back(d);
  else set_error(LSC_ERROR_OUT_OF_MEMORY, "arena: no room for %lld bytes of scratch", (long long)bytes);
  return d;
}

lsc_status Staging::finish(lsc_status st_in) {
  lsc_status result = st_in;
  if (result == LSC_SUCCESS) {
    for (auto& d : downs) {
      cudaError_t e = cudaMemcpyAsync(d.host, d.dev, static_cast<size_t>(d.bytes), cudaMemcpyDeviceToHost, st);
      if (e != cudaSuccess) {
        result = cuda_error(e, "cudaMemcpyAsync(D2H)");
        break;
      }
    }
  }
  if (touched_host || result != LSC_SUCCESS) {
    // Host buffers are borrowed only for the call: finish before returning.
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess && result == LSC_SUCCESS) result = cuda_error(e, "cudaStreamSynchronize");
    for (void* p : temps) be->arena.free(p);
  } else {
    for (void* p : temps) be->arena.free_after(p, st);
  }
  temps.clear();
  downs.clear();
  return result;
}

void set_shape(lsc_tensor& t, std::initializer_list<int64_t> dims) {
  t.ndim = static_cast<int32_t>(dims.size());
  int i = 0;
  for (int64_t d : dims) t.shape[i++] = d;
}

// Copies a compile-time tensor's bytes to host memory (it may live on either side).
lsc_status read_tensor_bytes(const lsc_tensor& t, int64_t bytes, std::vector<uint8_t>& out) {
  if (bytes < 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "tensor '%s': bad shape", t.name ? t.name : "");
  out.resize(static_cast<size_t>(bytes));
  if (bytes == 0) return LSC_SUCCESS;
  if (!t.data) return set_error(LSC_ERROR_INVALID_ARGUMENT, "tensor '%s' has no data", t.name ? t.name : "");
  if (t.nbytes && t.nbytes < static_cast<uint64_t>(bytes))
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "tensor '%s': %llu bytes given, %lld needed",
                     t.name ? t.name : "", (unsigned long long)t.nbytes, (long long)bytes);
  if (t.location == LSC_MEM_DEVICE) {
    LSC_CUDA_TRY(cudaMemcpy(out.data(), t.data, static_cast<size_t>(bytes), cudaMemcpyDeviceToHost));
  } else {
    memcpy(out.data(), t.data, static_cast<size_t>(bytes));
  }
  return LSC_SUCCESS;
}

lsc_status upload(lsc_backend* be, const void* host, int64_t bytes, void** dptr) {
  void* d = be->arena.alloc(static_cast<size_t>(bytes), 256);
  if (!d) return set_error(LSC_ERROR_OUT_OF_MEMORY, "arena: no room for %lld bytes of weights", (long long)bytes);
  cudaError_t e = cudaMemcpy(d, host, static_cast<size_t>(bytes), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    be->arena.free(d);
    return cuda_error(e, "weight upload");
  }
  *dptr = d;
  return LSC_SUCCESS;
}

}  // namespace lsc

void lsc_backend::release() {
  if (refs.fetch_sub(1) == 1) {
    DeviceGuard g(device);
    cudaDeviceSynchronize();
    delete this;
  }
}

lsc_op::~lsc_op() {
  if (be) {
    {
      DeviceGuard g(be->device);
      for (void* p : owned) be->arena.free(p);
    }
    be->release();
  }
}

// --------------------------------------------------------------------------- C ABI
extern "C" {

lsc_status lsc_backend_create(const lsc_config* config, lsc_backend** out) {
  if (!out) return set_error(LSC_ERROR_INVALID_ARGUMENT, "backend_create: null out");
  *out = nullptr;
  lsc_config cfg{};
  cfg.device_id = 0;
  cfg.rounding = LSC_ROUND_HALF_AWAY;
  cfg.fp32_mode = LSC_FP32_3XTF32;
  if (config) cfg = *config;
  if (cfg.rounding != LSC_ROUND_HALF_AWAY && cfg.rounding != LSC_ROUND_HALF_EVEN)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "backend_create: bad rounding %d", cfg.rounding);
  if (cfg.fp32_mode != LSC_FP32_3XTF32 && cfg.fp32_mode != LSC_FP32_TF32 && cfg.fp32_mode != LSC_FP32_WINOGRAD)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "backend_create: bad fp32_mode %d", cfg.fp32_mode);
  const int ndev = lsc_device_count();
  if (cfg.device_id < 0 || cfg.device_id >= ndev)
    return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "no CUDA device %d (%d present)", cfg.device_id, ndev);
  DeviceState* ds = device_state(cfg.device_id);
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (ds->cc_major != 10)
    return set_error(LSC_ERROR_BACKEND_NOT_AVAILABLE, "device %d is sm_%d%d; this backend needs sm_100",
                     cfg.device_id, ds->cc_major, ds->cc_minor);
  std::unique_ptr<lsc_backend> be(new (std::nothrow) lsc_backend());
  if (!be) return set_error(LSC_ERROR_OUT_OF_MEMORY, "backend_create: host allocation");
  be->device = cfg.device_id;
  be->cfg = cfg;
  be->ds = ds;
  DeviceGuard g(be->device);
  const size_t bytes = cfg.arena_bytes ? cfg.arena_bytes : (size_t(1) << 30);
  cudaError_t e = be->arena.init(bytes);
  if (e != cudaSuccess) return cuda_error(e, "arena cudaMalloc");
  *out = be.release();
  return LSC_SUCCESS;
}

void lsc_backend_destroy(lsc_backend* be) {
  if (!be) return;
  be->release();  // freed now, or when its last compiled operator is destroyed
}

int32_t lsc_backend_is_available(const lsc_backend* be) {
  return be && be->ds && be->ds->cc_major == 10 ? 1 : 0;
}

lsc_status lsc_backend_capabilities(const lsc_backend* be, lsc_caps* caps) {
  if (!be || !caps) return set_error(LSC_ERROR_INVALID_ARGUMENT, "capabilities: null argument");
  memset(caps, 0, sizeof(*caps));
  caps->backend_type = 1;
  caps->device_id = be->device;
  caps->sm_count = be->ds->sm_count;
  caps->cc_major = be->ds->cc_major;
  caps->cc_minor = be->ds->cc_minor;
  caps->total_memory = be->ds->total_memory;
  caps->memory_alignment = 256;
  caps->supported_ops_mask = supported_ops_mask();
  return LSC_SUCCESS;
}

lsc_status lsc_compile_operator(lsc_backend* be, const lsc_op_desc* def, const lsc_tensor* inputs,
                                int32_t n_inputs, const lsc_tensor* outputs, int32_t n_outputs,
                                lsc_op** out) {
  if (!be || !def || !out || n_inputs < 0 || n_outputs < 0 || (n_inputs && !inputs) ||
      (n_outputs && !outputs))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "compile_operator: bad arguments");
  *out = nullptr;
  DeviceGuard g(be->device);
  std::unique_ptr<lsc_op> op(new (std::nothrow) lsc_op());
  if (!op) return set_error(LSC_ERROR_OUT_OF_MEMORY, "compile_operator: host allocation");
  be->retain();
  op->be = be;
  op->desc = *def;
  op->rounding = def->rounding >= 0 ? def->rounding : be->cfg.rounding;
  op->fp32_mode = def->fp32_mode >= 0 ? def->fp32_mode : be->cfg.fp32_mode;
  if (op->rounding != LSC_ROUND_HALF_AWAY && op->rounding != LSC_ROUND_HALF_EVEN)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "compile_operator: bad rounding %d", op->rounding);
  if (op->fp32_mode != LSC_FP32_3XTF32 && op->fp32_mode != LSC_FP32_TF32 && op->fp32_mode != LSC_FP32_WINOGRAD)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "compile_operator: bad fp32_mode %d", op->fp32_mode);
  lsc_status st = compile_op(be, op.get(), inputs, n_inputs, outputs, n_outputs);
  if (st != LSC_SUCCESS) return st == LSC_ERROR_UNSUPPORTED_OPERATOR ? st : st;
  *out = op.release();
  return LSC_SUCCESS;
}

lsc_status lsc_execute(lsc_backend* be, const lsc_op* op, const lsc_tensor* inputs,
                       int32_t n_inputs, lsc_tensor* outputs, int32_t n_outputs,
                       lsc_stream stream) {
  if (!be || !op || op->be != be || n_inputs < 0 || n_outputs < 0 || (n_inputs && !inputs) ||
      (n_outputs && !outputs))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "execute: bad arguments");
  DeviceGuard g(be->device);
  Staging s;
  s.be = be;
  s.st = static_cast<cudaStream_t>(stream);
  lsc_status st = execute_op(be, op, inputs, n_inputs, outputs, n_outputs, s);
  return s.finish(st);
}

void lsc_op_destroy(lsc_op* op) { delete op; }

lsc_status lsc_allocate(lsc_backend* be, uint64_t size, uint64_t alignment, lsc_memory_block* block) {
  if (!be || !block) return set_error(LSC_ERROR_INVALID_ARGUMENT, "allocate: null argument");
  // Backend::allocate rejects non-power-of-two alignments (cpu.rs:216-221)
  if (alignment == 0 || (alignment & (alignment - 1)))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "Invalid alignment: %llu", (unsigned long long)alignment);
  void* p = be->arena.alloc(size, alignment);
  if (!p) return set_error(LSC_ERROR_OUT_OF_MEMORY, "Out of memory (arena of %llu bytes)",
                           (unsigned long long)be->arena.capacity());
  block->id = be->next_id.fetch_add(1);
  block->ptr = p;
  block->size = size;
  block->alignment = alignment < 256 ? 256 : alignment;
  block->location = LSC_MEM_DEVICE;
  return LSC_SUCCESS;
}

void lsc_deallocate(lsc_backend* be, lsc_memory_block* block) {
  if (!be || !block || !block->ptr) return;
  be->arena.free(block->ptr);
  block->ptr = nullptr;
}

lsc_status lsc_synchronize(lsc_backend* be) {
  if (!be) return set_error(LSC_ERROR_INVALID_ARGUMENT, "synchronize: null backend");
  DeviceGuard g(be->device);
  return lsc_check_device(nullptr);
}

lsc_status lsc_memory_stats(const lsc_backend* be, uint64_t* current, uint64_t* peak,
                            uint64_t* capacity) {
  if (!be) return set_error(LSC_ERROR_INVALID_ARGUMENT, "memory_stats: null backend");
  if (current) *current = be->arena.current();
  if (peak) *peak = be->arena.peak();
  if (capacity) *capacity = be->arena.capacity();
  return LSC_SUCCESS;
}

}  // extern "C"
