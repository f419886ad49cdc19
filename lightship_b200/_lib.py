"""ctypes binding of ``liblightship_cuda.so`` (declared in ``include/lightship_cuda.h``).

The library is built in-tree by ``lightship_b200.build``.  Loading fails loudly when it
is missing: there is no CPU fallback for any operator of this package.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "liblightship_cuda.so")

# status codes (lightship_cuda.h)
SUCCESS = 0
ERROR_INVALID_ARGUMENT = 2
ERROR_OUT_OF_MEMORY = 3
ERROR_BACKEND_NOT_AVAILABLE = 6
ERROR_SHAPE_MISMATCH = 7
ERROR_UNSUPPORTED_DATATYPE = 8
ERROR_DEVICE_ERROR = 9
ERROR_NOT_IMPLEMENTED = 10
ERROR_UNSUPPORTED_OPERATOR = 11
ERROR_COMPILATION_FAILED = 12
ERROR_EXECUTION_FAILED = 13
ERROR_UNSUPPORTED_LAYOUT = 14
ERROR_TIMEOUT = 15

ACT_NONE, ACT_RELU, ACT_RELU6, ACT_SILU, ACT_GELU = 0, 1, 2, 3, 4
DTYPE_F32, DTYPE_F16 = 0, 1  # lsc_dtype
ROUND_HALF_AWAY, ROUND_HALF_EVEN = 0, 1
FP32_3XTF32, FP32_TF32, FP32_WINOGRAD = 0, 1, 2
MEM_HOST, MEM_DEVICE = 0, 1
PRECISION_F32, PRECISION_INT8 = 0, 1
MAX_DIMS = 8


class LightShipError(RuntimeError):
    """A non-zero lsc_status, with the library's message (mirrors LightShipError)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


class lsc_config(C.Structure):
    _fields_ = [("device_id", C.c_int32), ("enable_fp16", C.c_int32), ("rounding", C.c_int32),
                ("fp32_mode", C.c_int32), ("arena_bytes", C.c_uint64)]


class lsc_caps(C.Structure):
    _fields_ = [("backend_type", C.c_int32), ("device_id", C.c_int32), ("sm_count", C.c_int32),
                ("cc_major", C.c_int32), ("cc_minor", C.c_int32), ("total_memory", C.c_uint64),
                ("memory_alignment", C.c_uint32), ("supported_ops_mask", C.c_uint32)]


class lsc_quant(C.Structure):
    _fields_ = [("scale", C.POINTER(C.c_float)), ("zero_point", C.POINTER(C.c_int32)),
                ("count", C.c_int32), ("bit_width", C.c_int32)]


class lsc_tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("ndim", C.c_int32), ("shape", C.c_int64 * MAX_DIMS),
                ("dtype", C.c_int32), ("layout", C.c_int32), ("location", C.c_int32),
                ("device", C.c_int32), ("data", C.c_void_p), ("nbytes", C.c_uint64),
                ("quant", lsc_quant)]


class lsc_op_desc(C.Structure):
    _fields_ = [("op_type", C.c_int32), ("fusion", C.c_int32), ("stride_h", C.c_int32),
                ("stride_w", C.c_int32), ("pad_h", C.c_int32), ("pad_w", C.c_int32),
                ("dilation_h", C.c_int32), ("dilation_w", C.c_int32), ("groups", C.c_int32),
                ("activation", C.c_int32), ("rounding", C.c_int32), ("fp32_mode", C.c_int32),
                ("bn_epsilon", C.c_float), ("output_scale", C.c_float), ("output_dtype", C.c_int32),
                ("kernel_h", C.c_int32), ("kernel_w", C.c_int32),
                ("pad_h_end_delta", C.c_int32), ("pad_w_end_delta", C.c_int32)]


class lsc_session_options(C.Structure):
    _fields_ = [("precision", C.c_int32), ("rounding", C.c_int32), ("concurrent", C.c_int32),
                ("plan_memory", C.c_int32), ("calibration", C.POINTER(lsc_tensor))]


class lsc_memory_block(C.Structure):
    _fields_ = [("id", C.c_uint64), ("ptr", C.c_void_p), ("size", C.c_uint64),
                ("alignment", C.c_uint64), ("location", C.c_int32)]


P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
F32 = C.c_float
ST = C.c_int32

# name -> (restype, argtypes); every function of include/lightship_cuda.h
SIGNATURES = {
    "lsc_version": (C.c_char_p, []),
    "lsc_last_error": (C.c_char_p, []),
    "lsc_status_string": (C.c_char_p, [I32]),
    "lsc_device_count": (I32, []),
    "lsc_backend_create": (ST, [C.POINTER(lsc_config), C.POINTER(P)]),
    "lsc_backend_destroy": (None, [P]),
    "lsc_backend_is_available": (I32, [P]),
    "lsc_backend_capabilities": (ST, [P, C.POINTER(lsc_caps)]),
    "lsc_compile_operator": (ST, [P, C.POINTER(lsc_op_desc), C.POINTER(lsc_tensor), I32,
                                  C.POINTER(lsc_tensor), I32, C.POINTER(P)]),
    "lsc_execute": (ST, [P, P, C.POINTER(lsc_tensor), I32, C.POINTER(lsc_tensor), I32, P]),
    "lsc_op_destroy": (None, [P]),
    "lsc_allocate": (ST, [P, C.c_uint64, C.c_uint64, C.POINTER(lsc_memory_block)]),
    "lsc_deallocate": (None, [P, C.POINTER(lsc_memory_block)]),
    "lsc_synchronize": (ST, [P]),
    "lsc_memory_stats": (ST, [P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "lsc_memcpy_h2d": (ST, [P, P, C.c_uint64, P]),
    "lsc_memcpy_d2h": (ST, [P, P, C.c_uint64, P]),
    "lsc_check_device": (ST, [C.POINTER(C.c_uint32)]),
    "lsc_gemm_i8": (ST, [P, P, I64, I64, I64, P, P, F32, I32, I32, P, P, P, P]),
    "lsc_conv2d_i8_nhwc": (ST, [P, P] + [I64] * 13 + [P, P, F32, I32, I32, P, P, P, P, F32, P]),
    "lsc_quantize_f32": (ST, [P, P, I64, I32, F32, I32, I32, P]),
    "lsc_quantize_f32_per_channel": (ST, [P, P, I64, I32, P, P, I32, I64, I32, P]),
    "lsc_dequantize": (ST, [P, I32, P, I64, F32, I32, P]),
    "lsc_dequantize_per_channel": (ST, [P, I32, P, I64, P, P, I32, I64, P]),
    "lsc_find_scale_zp_workspace_size": (C.c_uint64, []),
    "lsc_find_scale_zp_f32": (ST, [P, I64, I32, I32, P, C.c_uint64, P, P, P]),
    "lsc_find_scale_zp_per_channel_workspace_size": (C.c_uint64, [I64]),
    "lsc_find_scale_zp_per_channel_f32": (ST, [P, I64, I64, I32, I32, P, C.c_uint64, P, P, P]),
    "lsc_find_scale_zp_per_channel_f32_noalloc": (ST, [P, I64, I64, I32, I32, P, P, P]),
    "lsc_debug_withhold_copy": (ST, [I32, C.c_uint64]),
    "lsc_probe_tensor_rate": (ST, [I32, I32, I32, I32, I32, I32, I32, I32, C.POINTER(C.c_double),
                                   C.POINTER(C.c_double)]),
    "lsc_probe_im2col_rate": (ST, [P, I64, I64, I64, I32, I32, I32, I32, C.POINTER(C.c_double),
                                   C.POINTER(C.c_double)]),
    "lsc_probe_tma_rate": (ST, [P, C.c_uint64, I64, I32, I32, I32, I32, I32, I32, I32, I32, C.POINTER(C.c_double),
                                C.POINTER(C.c_double)]),
    "lsc_gemm_f16_batched": (ST, [P, I64, I64, I64, I64, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, F32, P, I32,
                                  I64, I64, I64, P]),
    "lsc_transpose_heads_f16": (ST, [P, P, I64, I64, I64, I64, I64, I64, I64, I64, P]),
    "lsc_attention_f16": (ST, [P, I64, I64, I64, F32, P, P, F32, I32, P]),
    "lsc_model_load_onnx": (ST, [C.c_char_p, C.c_uint64, C.POINTER(P)]),
    "lsc_model_destroy": (None, [P]),
    "lsc_model_info": (ST, [P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "lsc_model_io": (ST, [P, I32, C.c_uint32, C.POINTER(C.c_char_p), C.POINTER(I32), C.POINTER(I64),
                          C.POINTER(C.c_uint32)]),
    "lsc_model_node": (ST, [P, C.c_uint32, C.POINTER(lsc_op_desc), C.POINTER(C.c_char_p), C.POINTER(C.c_char_p)]),
    "lsc_session_create": (ST, [P, P, C.POINTER(P)]),
    "lsc_session_destroy": (None, [P]),
    "lsc_session_run": (ST, [P, C.POINTER(lsc_tensor), C.c_uint32, C.POINTER(lsc_tensor), C.c_uint32, P]),
    "lsc_session_create_ex": (ST, [P, P, C.POINTER(lsc_session_options), C.POINTER(P)]),
    "lsc_session_run_async": (ST, [P, C.POINTER(lsc_tensor), C.c_uint32, C.POINTER(lsc_tensor), C.c_uint32, P]),
    "lsc_session_io_buffer": (ST, [P, I32, C.c_uint32, C.POINTER(P), C.POINTER(C.c_uint64)]),
    "lsc_session_memory_plan": (ST, [P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint32)]),
    "lsc_session_value": (ST, [P, C.c_char_p, C.POINTER(C.c_float), C.POINTER(P), C.POINTER(lsc_tensor)]),
}

_lib = None
_lock = threading.Lock()


def lib() -> C.CDLL:
    """Loads the CUDA backend library (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m lightship_b200.build` "
                    "(the CUDA backend has no CPU fallback)")
            l = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(l, name, None)
                if fn is None:
                    continue
                fn.restype = res
                fn.argtypes = args
            _lib = l
    return _lib


def last_error() -> str:
    msg = lib().lsc_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    """Raises LightShipError for a non-zero status."""
    if status != SUCCESS:
        raise LightShipError(status, last_error())
