"""Writes ONNX models (ModelProto protobuf bytes) for the model-loader and session tests.

The protobuf encoding is lightship_b200.onnx_writer's.  Models are built from seeded numpy
parameters, which the tests reuse to compute the expected outputs with the oracle.
"""
from __future__ import annotations

import numpy as np

from lightship_b200.onnx_writer import model, node  # noqa: F401  (the wire-format encoder)


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
