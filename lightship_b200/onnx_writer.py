"""ONNX model writer (ModelProto protobuf bytes), for models whose weights live in numpy.

The `onnx` package is not needed: the protobuf wire format is encoded directly, with the
fields of onnx.proto (ModelProto ir_version = 1, opset_import = 8, graph = 7; GraphProto
node = 1, name = 2, initializer = 5, input = 11, output = 12; NodeProto input = 1, output = 2,
name = 3, op_type = 4, attribute = 5; AttributeProto name = 1, f = 2, i = 3, s = 4, ints = 8,
type = 20; TensorProto dims = 1, data_type = 2, name = 8, raw_data = 9; ValueInfoProto
name = 1, type = 2).  ``resnet18_onnx`` exports the ResNet-18 of ``lightship_b200.resnet18``
(same seeded parameters, the tensors named after its layers) for ``lsc_model_load_onnx`` and
the INT8 session.
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


def resnet18_onnx(batch: int, seed: int = 0, image: int = 224, num_classes: int = 1000) -> bytes:
    """ResNet-18 (conv1 7x7/2 + BN + ReLU, MaxPool 3x3/2, four stages of two BasicBlocks,
    GlobalAveragePool, Flatten, Gemm) with the parameters of ``resnet18.build_params(seed)``.
    Tensor names: the input "X", each layer's output by its name in ``resnet18`` ("conv1",
    "pool", "layer1.0.conv1", ..., the block output "layerS.B.conv2" after the residual Add
    and ReLU), "pooled" (the average pool, [N, 512, 1, 1]), "logits" (the output)."""
    from .resnet18 import build_params
    convs, blocks, fc_w, fc_b = build_params(seed, num_classes)
    inits, nodes = {}, []

    def conv_bn(spec, x, out, relu):
        inits[spec.name + ".w"] = spec.w
        g, b, mu, var = spec.bn
        inits[spec.name + ".bn.g"], inits[spec.name + ".bn.b"] = g, b
        inits[spec.name + ".bn.mu"], inits[spec.name + ".bn.var"] = mu, var
        k, p, s = spec.k, spec.pad, spec.stride
        nodes.append(node("Conv", [x, spec.name + ".w"], [spec.name + ".c"], name=spec.name, kernel_shape=[k, k],
                          pads=[p, p, p, p], strides=[s, s]))
        bn_out = spec.name + ".bn" if relu else out
        nodes.append(node("BatchNormalization", [spec.name + ".c", spec.name + ".bn.g", spec.name + ".bn.b",
                                                 spec.name + ".bn.mu", spec.name + ".bn.var"], [bn_out],
                          name=spec.name + ".bn", epsilon=1e-5))
        if relu:
            nodes.append(node("Relu", [bn_out], [out], name=spec.name + ".relu"))

    conv_bn(convs[0], "X", "conv1", True)
    nodes.append(node("MaxPool", ["conv1"], ["pool"], kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1]))
    prev = "pool"
    for c1, c2, ds in blocks:
        conv_bn(c1, prev, c1.name, True)
        skip = prev
        if ds is not None:
            conv_bn(ds, prev, ds.name, False)
            skip = ds.name
        conv_bn(c2, c1.name, c2.name + ".pre", False)
        nodes.append(node("Add", [c2.name + ".pre", skip], [c2.name + ".sum"], name=c2.name + ".add"))
        nodes.append(node("Relu", [c2.name + ".sum"], [c2.name], name=c2.name + ".relu"))
        prev = c2.name
    nodes.append(node("GlobalAveragePool", [prev], ["pooled"]))
    nodes.append(node("Flatten", ["pooled"], ["flat"], axis=1))
    inits["fc.w"], inits["fc.b"] = fc_w, fc_b
    nodes.append(node("Gemm", ["flat", "fc.w", "fc.b"], ["logits"], name="fc", transB=1))
    return model(nodes, inits, {"X": [batch, 3, image, image]}, {"logits": [batch, num_classes]}, name="resnet18")
