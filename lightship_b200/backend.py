"""Python mirror of LightShip's Backend trait over the CUDA backend's C ABI.

Names and argument meaning follow the reference (lightship-core/src):

* ``DataType`` / ``StorageLayout``       common/types.rs
* ``OperatorType``, ``OperatorDef``      ir/operator.rs:9-226 (attributes -> fields)
* ``FusionType``, ``FusionInfo``         ir/fusion.rs:8-77
* ``Quantization``, ``Tensor``           ir/tensor.rs:9-54 (data: numpy array on the host,
                                          or a torch CUDA tensor for device-resident data)
* ``GpuBackendConfig``                   backend/backend.rs:81-96
* ``CudaBackend.compile_operator / execute / allocate / deallocate / synchronize``
                                          backend/backend.rs:128-163

Errors raise ``LightShipError`` carrying the C status code.  Every operator runs this
package's CUDA kernels; nothing falls back to the CPU.
"""
from __future__ import annotations

import ctypes as C
import enum
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import LightShipError, check, lib


class DataType(enum.IntEnum):
    F32 = 0
    F16 = 1
    F64 = 2
    I8 = 3
    I16 = 4
    I32 = 5
    I64 = 6
    U8 = 7
    QUInt8 = 8
    QInt8 = 9
    QInt32 = 10

    @property
    def numpy(self):
        return {DataType.F32: np.float32, DataType.F16: np.float16, DataType.F64: np.float64,
                DataType.I8: np.int8, DataType.I16: np.int16, DataType.I32: np.int32,
                DataType.I64: np.int64, DataType.U8: np.uint8, DataType.QUInt8: np.uint8,
                DataType.QInt8: np.int8, DataType.QInt32: np.int32}[self]


class StorageLayout(enum.IntEnum):
    NCHW = 0
    NHWC = 1
    OIHW = 2
    OHWI = 3
    Default = 4


class OperatorType(enum.IntEnum):
    Conv2d = 0
    FullyConnected = 1
    MatMul = 2
    BatchNorm = 3
    ReLU = 4
    ReLU6 = 5
    SiLU = 6
    Quantize = 7
    Dequantize = 8
    QGemm = 9
    MaxPool2d = 10
    GlobalAvgPool2d = 11
    GELU = 12
    LayerNorm = 13
    Softmax = 14
    Add = 15


class FusionType(enum.IntEnum):
    ConvReLU = 0
    ConvReLU6 = 1
    ConvSigmoid = 2
    ConvBatchNorm = 3
    BatchNormReLU = 4
    AddReLU = 5
    MulReLU = 6


class Activation(enum.IntEnum):
    NONE = 0
    ReLU = 1
    ReLU6 = 2
    SiLU = 3
    GELU = 4


class Rounding(enum.IntEnum):
    HalfAwayFromZero = 0
    HalfEven = 1


@dataclass
class FusionInfo:
    """ir/fusion.rs:41-77."""
    fusion_type: FusionType
    original_ops: list = field(default_factory=list)

    @property
    def eliminate_batch_norm(self) -> bool:
        return OperatorType.BatchNorm in self.original_ops

    @staticmethod
    def conv_relu():
        return FusionInfo(FusionType.ConvReLU, [OperatorType.Conv2d, OperatorType.ReLU])

    @staticmethod
    def conv_batch_norm():
        return FusionInfo(FusionType.ConvBatchNorm, [OperatorType.Conv2d, OperatorType.BatchNorm])


@dataclass
class OperatorDef:
    """ir/operator.rs:200-226; the attributes the dense path reads are plain fields."""
    name: str
    operator_type: OperatorType
    stride: tuple = (1, 1)
    padding: tuple = (0, 0)
    dilation: tuple = (1, 1)
    groups: int = 1
    activation: Activation = Activation.NONE
    rounding: Optional[Rounding] = None
    fp32_mode: Optional[int] = None
    epsilon: float = 1e-5
    output_scale: float = 0.0
    kernel: tuple = (1, 1)
    # Conv2d end (bottom, right) padding minus `padding`; no counterpart in the reference
    padding_end_delta: tuple = (0, 0)


@dataclass
class Quantization:
    """ir/tensor.rs:9-18."""
    scale: Sequence[float]
    zero_point: Sequence[int] = ()
    bit_width: int = 8


class Tensor:
    """ir/tensor.rs:39-54.  ``data`` is a numpy array (host, TensorData::Owned) or a torch
    CUDA tensor (device-resident); ``shape`` is set by the backend after execute."""

    def __init__(self, name: str, shape, data_type: DataType, data=None,
                 layout: StorageLayout = StorageLayout.Default,
                 quantization: Optional[Quantization] = None):
        self.name = name
        self.shape = list(shape)
        self.data_type = DataType(data_type)
        self.layout = StorageLayout(layout)
        self.data = data
        self.quantization = quantization

    @staticmethod
    def from_data(name, shape, data_type, values, **kw):
        arr = np.asarray(values, dtype=DataType(data_type).numpy).reshape(shape)
        return Tensor(name, shape, data_type, np.ascontiguousarray(arr), **kw)

    def numpy(self):
        d = self.data
        if d is None:
            return None
        if isinstance(d, np.ndarray):
            return d
        return d.detach().cpu().numpy()

    # -- C view ---------------------------------------------------------------------
    def _to_c(self, keep: list) -> _lib.lsc_tensor:
        t = _lib.lsc_tensor()
        name = self.name.encode()
        keep.append(name)
        t.name = name
        t.ndim = len(self.shape)
        for i, d in enumerate(self.shape):
            t.shape[i] = int(d)
        t.dtype = int(self.data_type)
        t.layout = int(self.layout)
        d = self.data
        if d is None:
            t.location = _lib.MEM_HOST
            t.data = None
            t.nbytes = 0
        elif isinstance(d, np.ndarray):
            if not d.flags.c_contiguous:
                raise ValueError(f"tensor {self.name}: host data must be C-contiguous")
            t.location = _lib.MEM_HOST
            t.data = d.ctypes.data
            t.nbytes = d.nbytes
        else:  # torch tensor
            if not d.is_contiguous():
                raise ValueError(f"tensor {self.name}: device data must be contiguous")
            t.location = _lib.MEM_DEVICE if d.is_cuda else _lib.MEM_HOST
            t.device = (d.device.index or 0) if d.is_cuda else 0
            t.data = d.data_ptr()
            t.nbytes = d.numel() * d.element_size()
        q = self.quantization
        if q is not None:
            sc = (C.c_float * len(q.scale))(*q.scale)
            keep.append(sc)
            t.quant.scale = sc
            t.quant.count = len(q.scale)
            t.quant.bit_width = q.bit_width
            if len(q.zero_point):
                zp = (C.c_int32 * len(q.zero_point))(*q.zero_point)
                keep.append(zp)
                t.quant.zero_point = zp
        return t


@dataclass
class GpuBackendConfig:
    """backend/backend.rs:81-96 plus the CUDA backend's extensions."""
    device_id: int = 0
    enable_fp16: bool = False
    rounding: Rounding = Rounding.HalfAwayFromZero
    fp32_mode: int = _lib.FP32_3XTF32
    arena_bytes: int = 0


@dataclass
class MemoryBlock:
    """backend/memory.rs:32-45."""
    id: int
    ptr: int
    size: int
    alignment: int
    location: str = "GPU"


class CompiledOperator:
    """backend/backend.rs:99-108: operator type, fusion and the C-side compiled handle."""

    def __init__(self, backend: "CudaBackend", handle, operator_type, fusion):
        self._backend = backend
        self._handle = handle
        self.operator_type = operator_type
        self.fusion = fusion

    def __del__(self):
        h, self._handle = getattr(self, "_handle", None), None
        if h:
            try:
                lib().lsc_op_destroy(h)
            except Exception:
                pass


class CudaBackend:
    """The CUDA backend: ``Backend`` trait methods over ``liblightship_cuda.so``."""

    def __init__(self, config: Optional[GpuBackendConfig] = None):
        config = config or GpuBackendConfig()
        cfg = _lib.lsc_config(config.device_id, int(config.enable_fp16), int(config.rounding),
                              int(config.fp32_mode), int(config.arena_bytes))
        h = C.c_void_p()
        check(lib().lsc_backend_create(C.byref(cfg), C.byref(h)))
        self._h = h
        self.config = config

    def close(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            lib().lsc_backend_destroy(h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- Backend trait ----------------------------------------------------------------
    def backend_type(self) -> str:
        return "GPU"

    def is_available(self) -> bool:
        return bool(lib().lsc_backend_is_available(self._h))

    def capabilities(self) -> dict:
        caps = _lib.lsc_caps()
        check(lib().lsc_backend_capabilities(self._h, C.byref(caps)))
        return {f: getattr(caps, f) for f, _ in caps._fields_}

    def compile_operator(self, op_def: OperatorDef, fusion: Optional[FusionInfo],
                         inputs: Sequence[Tensor], outputs: Sequence[Tensor]) -> CompiledOperator:
        d = _lib.lsc_op_desc()
        d.op_type = int(op_def.operator_type)
        d.fusion = int(fusion.fusion_type) if fusion is not None else -1
        d.stride_h, d.stride_w = op_def.stride
        d.pad_h, d.pad_w = op_def.padding
        d.dilation_h, d.dilation_w = op_def.dilation
        d.groups = op_def.groups
        d.activation = int(op_def.activation)
        d.rounding = -1 if op_def.rounding is None else int(op_def.rounding)
        d.fp32_mode = -1 if op_def.fp32_mode is None else int(op_def.fp32_mode)
        d.bn_epsilon = op_def.epsilon
        d.output_scale = op_def.output_scale
        d.output_dtype = int(outputs[0].data_type) if outputs else -1
        d.kernel_h, d.kernel_w = op_def.kernel
        d.pad_h_end_delta, d.pad_w_end_delta = op_def.padding_end_delta
        keep: list = []
        cin = (_lib.lsc_tensor * max(1, len(inputs)))(*[t._to_c(keep) for t in inputs])
        cout = (_lib.lsc_tensor * max(1, len(outputs)))(*[t._to_c(keep) for t in outputs])
        h = C.c_void_p()
        check(lib().lsc_compile_operator(self._h, C.byref(d), cin, len(inputs), cout, len(outputs),
                                         C.byref(h)))
        return CompiledOperator(self, h, op_def.operator_type, fusion)

    def execute(self, op: CompiledOperator, inputs: Sequence[Tensor], outputs: Sequence[Tensor],
                stream=None) -> None:
        keep: list = []
        cin = (_lib.lsc_tensor * max(1, len(inputs)))(*[t._to_c(keep) for t in inputs])
        cout = (_lib.lsc_tensor * max(1, len(outputs)))(*[t._to_c(keep) for t in outputs])
        st = C.c_void_p(stream) if isinstance(stream, int) else stream
        check(lib().lsc_execute(self._h, op._handle, cin, len(inputs), cout, len(outputs), st))
        for t, c in zip(outputs, cout):
            t.shape = [int(c.shape[i]) for i in range(c.ndim)]

    def allocate(self, size: int, alignment: int) -> MemoryBlock:
        blk = _lib.lsc_memory_block()
        check(lib().lsc_allocate(self._h, size, alignment, C.byref(blk)))
        return MemoryBlock(blk.id, blk.ptr, blk.size, blk.alignment)

    def deallocate(self, block: MemoryBlock) -> None:
        blk = _lib.lsc_memory_block(block.id, block.ptr, block.size, block.alignment, _lib.MEM_DEVICE)
        lib().lsc_deallocate(self._h, C.byref(blk))

    def synchronize(self) -> None:
        check(lib().lsc_synchronize(self._h))

    def memory_stats(self) -> dict:
        cur, peak, cap = C.c_uint64(), C.c_uint64(), C.c_uint64()
        check(lib().lsc_memory_stats(self._h, C.byref(cur), C.byref(peak), C.byref(cap)))
        return {"current": cur.value, "peak": peak.value, "capacity": cap.value}


class OnnxModel:
    """An ONNX model loaded from memory and fused (LightShipEngine_LoadModelFromMemory,
    c-api/include/lightship.h:186-198): attributes read, Conv->BN->Relu and Add->Relu fused."""

    def __init__(self, data: bytes):
        h = C.c_void_p()
        check(lib().lsc_model_load_onnx(data, len(data), C.byref(h)))
        self._h = h

    @staticmethod
    def from_file(path: str) -> "OnnxModel":
        with open(path, "rb") as f:
            return OnnxModel(f.read())

    def close(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            lib().lsc_model_destroy(h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _counts(self):
        ni, no, nn = C.c_uint32(), C.c_uint32(), C.c_uint32()
        check(lib().lsc_model_info(self._h, C.byref(ni), C.byref(no), C.byref(nn)))
        return ni.value, no.value, nn.value

    def _io(self, is_output: int, i: int):
        name, dt, nd = C.c_char_p(), C.c_int32(), C.c_uint32()
        shape = (C.c_int64 * _lib.MAX_DIMS)()
        check(lib().lsc_model_io(self._h, is_output, i, C.byref(name), C.byref(dt), shape, C.byref(nd)))
        return name.value.decode(), DataType(dt.value), [int(shape[k]) for k in range(nd.value)]

    @property
    def inputs(self):
        return [self._io(0, i) for i in range(self._counts()[0])]

    @property
    def outputs(self):
        return [self._io(1, i) for i in range(self._counts()[1])]

    def nodes(self):
        """(name, ONNX operator, lsc_op_desc) of every node of the fused graph."""
        out = []
        for i in range(self._counts()[2]):
            d, name, op = _lib.lsc_op_desc(), C.c_char_p(), C.c_char_p()
            check(lib().lsc_model_node(self._h, i, C.byref(d), C.byref(name), C.byref(op)))
            out.append((name.value.decode(), op.value.decode(), d))
        return out


class Session:
    """An inference session of an OnnxModel on a CudaBackend (LightShipEngine_CreateSession /
    LightShipSession_Run, lightship.h:283-331).

    ``precision="int8"`` compiles the model into the INT8 chain (``lsc_session_create_ex``):
    activation scales calibrated on ``calibration`` (an f32 Tensor of the input's shape), int8
    activations planned into one arena block by live range, the network captured by the
    library as a CUDA graph with sibling convolutions on a second stream."""

    def __init__(self, backend: CudaBackend, model: OnnxModel, precision: str = "f32",
                 calibration: Optional[Tensor] = None, rounding: Optional[Rounding] = None,
                 concurrent: bool = True, plan_memory: bool = True):
        h = C.c_void_p()
        if precision == "f32":
            check(lib().lsc_session_create(backend._h, model._h, C.byref(h)))
        elif precision == "int8":
            if calibration is None:
                raise ValueError("an INT8 session needs a calibration batch")
            keep: list = []
            cal = calibration._to_c(keep)
            opts = _lib.lsc_session_options(_lib.PRECISION_INT8, -1 if rounding is None else int(rounding),
                                            int(concurrent), int(plan_memory), C.pointer(cal))
            check(lib().lsc_session_create_ex(backend._h, model._h, C.byref(opts), C.byref(h)))
        else:
            raise ValueError(f"unknown precision {precision!r}")
        self._h = h
        self.precision = precision
        self._backend, self._model = backend, model  # both stay alive with the session

    def close(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            lib().lsc_session_destroy(h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def run(self, inputs: Sequence[Tensor], outputs: Sequence[Tensor], stream=None) -> None:
        self._run(lib().lsc_session_run, inputs, outputs, stream)

    def run_async(self, inputs: Sequence[Tensor], outputs: Sequence[Tensor], stream=None) -> None:
        """Enqueues one run on ``stream`` (INT8 sessions; see ``lsc_session_run_async``)."""
        self._run(lib().lsc_session_run_async, inputs, outputs, stream)

    def _run(self, fn, inputs, outputs, stream):
        keep: list = []
        cin = (_lib.lsc_tensor * max(1, len(inputs)))(*[t._to_c(keep) for t in inputs])
        cout = (_lib.lsc_tensor * max(1, len(outputs)))(*[t._to_c(keep) for t in outputs])
        st = C.c_void_p(stream) if isinstance(stream, int) else stream
        check(fn(self._h, cin, len(inputs), cout, len(outputs), st))
        for t, c in zip(outputs, cout):
            t.shape = [int(c.shape[i]) for i in range(c.ndim)]

    def io_buffer(self, is_output: bool):
        """(device pointer, bytes) of the INT8 session's input slot 0 or its output buffer."""
        p, n = C.c_void_p(), C.c_uint64()
        check(lib().lsc_session_io_buffer(self._h, int(is_output), 0, C.byref(p), C.byref(n)))
        return p.value, n.value

    def memory_plan(self) -> dict:
        a, b, v = C.c_uint64(), C.c_uint64(), C.c_uint32()
        check(lib().lsc_session_memory_plan(self._h, C.byref(a), C.byref(b), C.byref(v)))
        return {"planned_bytes": a.value, "unplanned_bytes": b.value, "values": v.value}

    def value(self, name: str) -> dict:
        """An INT8 activation: its calibrated scale, device pointer and NHWC shape."""
        sc, p, t = C.c_float(), C.c_void_p(), _lib.lsc_tensor()
        check(lib().lsc_session_value(self._h, name.encode(), C.byref(sc), C.byref(p), C.byref(t)))
        return {"scale": sc.value, "ptr": p.value, "shape": [int(t.shape[i]) for i in range(t.ndim)],
                "nbytes": int(t.nbytes)}


__all__ = ["DataType", "StorageLayout", "OperatorType", "FusionType", "FusionInfo", "Activation",
           "Rounding", "OperatorDef", "Quantization", "Tensor", "GpuBackendConfig", "MemoryBlock",
           "CompiledOperator", "CudaBackend", "LightShipError", "OnnxModel", "Session"]
