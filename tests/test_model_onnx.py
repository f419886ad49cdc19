"""ONNX models on the CUDA backend: the loader reads node attributes, the fusion pass makes the
graph optimizer's decisions (Conv->BN->Relu, Add->Relu, single-consumer rule), and a session
runs the fused graph.  Loader and fusion tests run on the CPU (no kernel launched); session
tests compare the device output with the oracle's composition of the reference operators.

Session tolerance (FP32, split-TF32 contractions, BN folded into the conv weights as the
reference's optimizer formula does): |y - y_ref| <= 1e-4 * max|y_ref| + 1e-4 * |y_ref|."""
import numpy as np
import pytest

from lightship_b200 import _lib
from oracle import oracle as orc
from tests.golden import onnx_writer as W

FUSION = {"none": -1, "conv_relu": 0, "conv_relu6": 1, "conv_bn": 3, "bn_relu": 4, "add_relu": 5}


def _B():
    from lightship_b200 import backend as B
    return B


# ------------------------------------------------------------------------------ loader (CPU)
def test_conv_relu_fixture_shapes_load_and_fuse():
    B = _B()
    data, _ = W.conv_relu_model()
    m = B.OnnxModel(data)
    assert m.inputs == [("X", B.DataType.F32, [1, 3, 32, 32])]
    assert m.outputs == [("Y", B.DataType.F32, [1, 16, 30, 30])]
    nodes = m.nodes()
    assert len(nodes) == 1  # Relu folded into the Conv
    name, op, d = nodes[0]
    assert op == "Conv" and d.op_type == B.OperatorType.Conv2d and d.fusion == FUSION["conv_relu"]
    assert (d.stride_h, d.pad_h, d.groups) == (1, 0, 1)


def test_small_resnet_attributes_and_fusions():
    B = _B()
    data, _ = W.small_resnet_model()
    nodes = B.OnnxModel(data).nodes()
    got = [(op, d.op_type, d.fusion, d.activation) for _, op, d in nodes]
    assert got == [
        ("Conv", 0, FUSION["conv_bn"], _lib.ACT_RELU),    # Conv -> BN -> Relu in one operator
        ("MaxPool", 10, -1, 0),
        ("Conv", 0, FUSION["conv_bn"], _lib.ACT_RELU),
        ("Conv", 0, FUSION["conv_bn"], 0),                # its output feeds the residual Add
        ("Add", 15, FUSION["add_relu"], 0),
        ("Conv", 0, FUSION["conv_bn"], _lib.ACT_RELU6),   # Clip(0, 6) as ReLU6
        ("Conv", 0, FUSION["conv_relu"], 0),
        ("GlobalAveragePool", 11, -1, 0),
        ("Flatten", -1, -1, 0),
        ("Gemm", 1, -1, 0),                               # constant B: FullyConnected
        ("MatMul", 1, -1, 0),
    ]
    conv_s2 = nodes[5][2]
    assert (conv_s2.stride_h, conv_s2.stride_w, conv_s2.pad_h, conv_s2.groups) == (2, 2, 1, 2)
    dil = nodes[6][2]
    assert (dil.dilation_h, dil.pad_h) == (2, 2)
    pool = nodes[1][2]
    assert (pool.kernel_h, pool.stride_h, pool.pad_h) == (3, 2, 1)
    assert abs(nodes[0][2].bn_epsilon - 1e-5) < 1e-12


def test_single_consumer_rule_keeps_a_shared_conv_output():
    """optimizer.rs:633-640: a Conv whose output also leaves the graph is not fused with its BN."""
    B = _B()
    rng = np.random.default_rng(1)
    w = rng.normal(size=(4, 3, 1, 1)).astype(np.float32)
    g, b, mu, var = (np.ones(4, np.float32), np.zeros(4, np.float32), np.zeros(4, np.float32), np.ones(4, np.float32))
    nodes = [W.node("Conv", ["X", "w"], ["c"]), W.node("BatchNormalization", ["c", "g", "b", "mu", "var"], ["Y"])]
    data = W.model(nodes, {"w": w, "g": g, "b": b, "mu": mu, "var": var}, {"X": [1, 3, 4, 4]},
                   {"Y": [1, 4, 4, 4], "c": [1, 4, 4, 4]})
    got = [(op, d.fusion) for _, op, d in B.OnnxModel(data).nodes()]
    assert got == [("Conv", -1), ("BatchNormalization", -1)]


def test_loader_errors():
    B = _B()
    with pytest.raises(B.LightShipError) as e:
        B.OnnxModel(b"\x3a\xff\xff\xff")  # graph field whose length runs past the end
    assert e.value.code == _lib.ERROR_INVALID_ARGUMENT
    data = W.model([W.node("Sigmoid", ["X"], ["Y"])], {}, {"X": [1, 4]}, {"Y": [1, 4]})
    with pytest.raises(B.LightShipError) as e:
        B.OnnxModel(data)
    assert e.value.code == _lib.ERROR_UNSUPPORTED_OPERATOR and "Sigmoid" in str(e.value)


# ------------------------------------------------------------------------------ session (GPU)
def _maxpool_nchw(x, k, s, p):
    n, c, h, w = x.shape
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    xp = np.full((n, c, h + 2 * p, w + 2 * p), -np.inf, np.float32)
    xp[:, :, p:p + h, p:p + w] = x
    y = np.full((n, c, oh, ow), -np.inf, np.float32)
    for r in range(k):
        for q in range(k):
            y = np.maximum(y, xp[:, :, r:r + s * oh:s, q:q + s * ow:s])
    return y


def small_resnet_reference(x, p):
    """The small residual CNN restated with the oracle's operators (conv, BatchNorm, activations)."""
    def cbn(x, c, bn, act, **kw):
        y = orc.conv2d_nchw(x, p[c + ".w"], p.get(c + ".b"), **kw)
        if bn:
            y = orc.batchnorm_inference(y, p[bn + ".g"], p[bn + ".beta"], p[bn + ".mu"], p[bn + ".var"])
        return orc.act(y, act)

    t = cbn(x, "c1", "bn1", orc.ACT_RELU, pad=(1, 1))
    pool = _maxpool_nchw(t, 3, 2, 1)
    u = cbn(pool, "c2", "bn2", orc.ACT_RELU, pad=(1, 1))
    u = cbn(u, "c3", "bn3", orc.ACT_NONE, pad=(1, 1))
    u = orc.act((u + pool).astype(np.float32), orc.ACT_RELU)
    v = cbn(u, "c4", "bn4", orc.ACT_RELU6, stride=(2, 2), pad=(1, 1), groups=2)
    w = cbn(v, "c5", None, orc.ACT_RELU, pad=(2, 2), dilation=(2, 2))
    g = w.mean(axis=(2, 3), dtype=np.float64).astype(np.float32)
    logits = orc.fully_connected(g, p["fc.w"]) + p["fc.b"]
    return orc.matmul(logits.astype(np.float32), p["mm.w"])


@pytest.fixture(scope="module")
def be(cuda):
    from lightship_b200.backend import CudaBackend, GpuBackendConfig
    b = CudaBackend(GpuBackendConfig(device_id=0, arena_bytes=256 << 20))
    yield b
    b.close()


@pytest.mark.gpu
def test_session_conv_relu_fixture_shapes(be):
    B = _B()
    data, p = W.conv_relu_model()
    sess = B.Session(be, B.OnnxModel(data))
    x = np.random.default_rng(3).normal(size=(1, 3, 32, 32)).astype(np.float32)
    y = B.Tensor("Y", [1], B.DataType.F32, np.zeros(16 * 30 * 30, np.float32))
    sess.run([B.Tensor("X", list(x.shape), B.DataType.F32, x)], [y])
    ref = orc.act(orc.conv2d_nchw(x, p["W"], p["B"]), orc.ACT_RELU)
    assert y.shape == [1, 16, 30, 30]
    out = y.numpy().reshape(ref.shape)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-4 * float(np.abs(ref).max()))


@pytest.mark.gpu
@pytest.mark.parametrize("device_io", [False, True])
def test_session_small_resnet_matches_oracle(be, cuda, device_io):
    import torch
    B = _B()
    data, p = W.small_resnet_model(batch=2)
    sess = B.Session(be, B.OnnxModel(data))
    rng = np.random.default_rng(8)
    for _ in range(2):  # two runs of one session: buffers and compiled operators are reused
        x = rng.normal(size=(2, 3, 16, 16)).astype(np.float32)
        ref = small_resnet_reference(x, p)
        if device_io:
            xt = B.Tensor("X", list(x.shape), B.DataType.F32, torch.from_numpy(x).to(cuda))
            yt = B.Tensor("Y", [2, 7], B.DataType.F32, torch.zeros(2, 7, device=cuda))
            sess.run([xt], [yt], stream=torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
        else:
            xt = B.Tensor("X", list(x.shape), B.DataType.F32, x)
            yt = B.Tensor("Y", [2, 7], B.DataType.F32, np.zeros((2, 7), np.float32))
            sess.run([xt], [yt])
        out = yt.numpy().reshape(ref.shape)
        assert yt.shape == [2, 7]
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-4 * float(np.abs(ref).max()))


@pytest.mark.gpu
def test_session_rejects_wrong_input_shape(be):
    B = _B()
    data, _ = W.conv_relu_model()
    sess = B.Session(be, B.OnnxModel(data))
    x = np.zeros((1, 3, 30, 32), np.float32)
    with pytest.raises(B.LightShipError) as e:
        sess.run([B.Tensor("X", list(x.shape), B.DataType.F32, x)],
                 [B.Tensor("Y", [1], B.DataType.F32, np.zeros(16 * 30 * 30, np.float32))])
    assert e.value.code == _lib.ERROR_SHAPE_MISMATCH
