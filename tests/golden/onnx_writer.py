"""Writes ONNX models (ModelProto protobuf bytes) for the model-loader and session tests.

The `onnx` package is not available here, so this encodes the protobuf wire format directly
(the fields are those of onnx.proto: ModelProto.ir_version = 1, opset_import = 8, graph = 7;
GraphProto node = 1, name = 2, initializer = 5, input = 11, output = 12; NodeProto input = 1,
output = 2, name = 3, op_type = 4, attribute = 5; AttributeProto name = 1, f = 2, i = 3,
s = 4, ints = 8, type = 20; TensorProto dims = 1, data_type = 2, name = 8, raw_data = 9;
ValueInfoProto name = 1, type = 2).  Models are built from seeded numpy parameters, which the
tests reuse to compute the expected outputs with the oracle.
"""
from __future__ import annotations

import struct

import numpy as np

FLOAT, INT64 = 1, 7
A_FLOAT, A_INT, A_STRING, A_INTS = 1, 2, 3, 7


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _len(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _int(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(v)


def _str(field: int, s: str) -> bytes:
    return _len(field, s.encode())


def attr(name: str, value) -> bytes:
    """AttributeProto for an int, float, string or list of ints."""
    b = _str(1, name)
    if isinstance(value, float):
        b += _key(2, 5) + struct.pack("<f", value) + _int(20, A_FLOAT)
    elif isinstance(value, int):
        b += _int(3, value) + _int(20, A_INT)
    elif isinstance(value, str):
        b += _len(4, value.encode()) + _int(20, A_STRING)
    else:  # list of ints, packed
        b += _len(8, b"".join(_varint(int(v)) for v in value)) + _int(20, A_INTS)
    return b


def node(op: str, inputs, outputs, name: str = "", **attrs) -> bytes:
    b = b"".join(_str(1, i) for i in inputs) + b"".join(_str(2, o) for o in outputs)
    b += _str(3, name or outputs[0]) + _str(4, op)
    for k, v in attrs.items():
        b += _len(5, attr(k, v))
    return b


def tensor(name: str, arr: np.ndarray) -> bytes:
    arr = np.ascontiguousarray(arr)
    dt = FLOAT if arr.dtype == np.float32 else INT64
    b = b"".join(_int(1, int(d)) for d in arr.shape) + _int(2, dt) + _str(8, name)
    return b + _len(9, arr.astype("<f4" if dt == FLOAT else "<i8").tobytes())


def value_info(name: str, shape) -> bytes:
    dims = b"".join(_len(1, _int(1, int(d))) for d in shape)
    tensor_type = _int(1, FLOAT) + _len(2, dims)
    return _str(1, name) + _len(2, _len(1, tensor_type))


def model(nodes, inits: dict, inputs: dict, outputs: dict, name: str = "graph") -> bytes:
    g = b"".join(_len(1, n) for n in nodes) + _str(2, name)
    g += b"".join(_len(5, tensor(k, v)) for k, v in inits.items())
    g += b"".join(_len(11, value_info(k, s)) for k, s in inputs.items())
    g += b"".join(_len(12, value_info(k, s)) for k, s in outputs.items())
    opset = _str(1, "") + _int(2, 13)
    return _int(1, 8) + _len(8, opset) + _len(7, g)


# ---------------------------------------------------------------------------- test models
def conv_relu_model():
    """The shapes of the reference's ONNX fixture (tests/onnx_integration_test.rs:117-220):
    X [1, 3, 32, 32], Conv W [16, 3, 3, 3] + B [16] (no padding), Relu -> Y [1, 16, 30, 30]."""
    rng = np.random.default_rng(11)
    w = rng.normal(0, 0.2, (16, 3, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.1, 16).astype(np.float32)
    nodes = [node("Conv", ["X", "W", "B"], ["c"], kernel_shape=[3, 3]), node("Relu", ["c"], ["Y"])]
    return model(nodes, {"W": w, "B": b}, {"X": [1, 3, 32, 32]}, {"Y": [1, 16, 30, 30]}), {"W": w, "B": b}


def _bn(rng, c):
    return (rng.uniform(0.5, 1.5, c).astype(np.float32), rng.normal(0, 0.1, c).astype(np.float32),
            rng.normal(0, 0.1, c).astype(np.float32), rng.uniform(0.5, 1.5, c).astype(np.float32))


def small_resnet_model(batch: int = 2, seed: int = 5):
    """A residual CNN exercising every attribute and fusion the loader handles:
    Conv(3->16, 3x3, pad 1) BN Relu, MaxPool(3, s2, p1), a BasicBlock (Conv BN Relu, Conv BN,
    Add with the block input, Relu), a grouped strided Conv(16->32, 3x3, s2, p1, group 2) BN
    Clip(0, 6), a dilated Conv(32->32, 3x3, pad 2, dilation 2) + bias Relu,
    GlobalAveragePool, Flatten, Gemm(32->10, transB=1) and a MatMul(10->7) with a constant B."""
    rng = np.random.default_rng(seed)
    p = {}

    def conv(name, co, ci, k, bias=False):
        p[name + ".w"] = rng.normal(0, np.sqrt(2.0 / (ci * k * k)), (co, ci, k, k)).astype(np.float32)
        if bias:
            p[name + ".b"] = rng.normal(0, 0.1, co).astype(np.float32)

    def bn(name, c):
        p[name + ".g"], p[name + ".beta"], p[name + ".mu"], p[name + ".var"] = _bn(rng, c)

    conv("c1", 16, 3, 3); bn("bn1", 16)
    conv("c2", 16, 16, 3); bn("bn2", 16)
    conv("c3", 16, 16, 3); bn("bn3", 16)
    conv("c4", 32, 8, 3); bn("bn4", 32)
    conv("c5", 32, 32, 3, bias=True)
    p["fc.w"] = rng.normal(0, 0.2, (10, 32)).astype(np.float32)
    p["fc.b"] = rng.normal(0, 0.1, 10).astype(np.float32)
    p["mm.w"] = rng.normal(0, 0.3, (10, 7)).astype(np.float32)
    p["clip.lo"] = np.float32([0.0]).reshape(())
    p["clip.hi"] = np.float32([6.0]).reshape(())

    def bnn(name, x, y):
        return node("BatchNormalization", [x, name + ".g", name + ".beta", name + ".mu", name + ".var"], [y],
                    epsilon=1e-5)

    nodes = [
        node("Conv", ["X", "c1.w"], ["t1"], kernel_shape=[3, 3], pads=[1, 1, 1, 1], strides=[1, 1]),
        bnn("bn1", "t1", "t2"), node("Relu", ["t2"], ["t3"]),
        node("MaxPool", ["t3"], ["p"], kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1]),
        node("Conv", ["p", "c2.w"], ["u1"], kernel_shape=[3, 3], pads=[1, 1, 1, 1]),
        bnn("bn2", "u1", "u2"), node("Relu", ["u2"], ["u3"]),
        node("Conv", ["u3", "c3.w"], ["u4"], kernel_shape=[3, 3], pads=[1, 1, 1, 1]),
        bnn("bn3", "u4", "u5"),
        node("Add", ["u5", "p"], ["u6"]), node("Relu", ["u6"], ["u7"]),
        node("Conv", ["u7", "c4.w"], ["v1"], kernel_shape=[3, 3], pads=[1, 1, 1, 1], strides=[2, 2], group=2),
        bnn("bn4", "v1", "v2"), node("Clip", ["v2", "clip.lo", "clip.hi"], ["v3"]),
        node("Conv", ["v3", "c5.w", "c5.b"], ["w1"], kernel_shape=[3, 3], pads=[2, 2, 2, 2], dilations=[2, 2]),
        node("Relu", ["w1"], ["w2"]),
        node("GlobalAveragePool", ["w2"], ["g"]), node("Flatten", ["g"], ["f"], axis=1),
        node("Gemm", ["f", "fc.w", "fc.b"], ["logits"], transB=1),
        node("MatMul", ["logits", "mm.w"], ["Y"]),
    ]
    inits = {k: v for k, v in p.items()}
    return model(nodes, inits, {"X": [batch, 3, 16, 16]}, {"Y": [batch, 7]}, name="small_resnet"), p
