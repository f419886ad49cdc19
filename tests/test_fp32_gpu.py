"""FP32 operators through the Backend (C ABI): MatMul, FullyConnected, Conv2d with folded
BatchNorm / bias / ReLU, standalone BatchNorm and activations, and INT8 Conv2d compiled from
f32 weights.  Compared with the reference KATs and the oracle.

Tolerances (contractions): every output element must satisfy
    |y - y_oracle| <= tol * (sum_k |a_k * b_k| + |bias|)
with tol = 2e-5 for split-TF32 (the default, three tensor-core products) and 2e-3 for
single-pass TF32.  Elementwise operators (BatchNorm, ReLU, ReLU6, SiLU, add) are bit-exact:
SiLU's exp restates the host libm's expf."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.golden import reference_kats as K

pytestmark = pytest.mark.gpu

TOL_3XTF32 = 2e-5
TOL_TF32 = 2e-3


@pytest.fixture(scope="module")
def be(cuda):
    from lightship_b200.backend import CudaBackend, GpuBackendConfig
    b = CudaBackend(GpuBackendConfig(device_id=0, arena_bytes=2 << 30))
    yield b
    b.close()


def _B():
    from lightship_b200 import backend as B
    return B


def _run(be, opdef, inputs, outputs, fusion=None, runtime_inputs=None):
    op = be.compile_operator(opdef, fusion, inputs, outputs)
    be.execute(op, runtime_inputs if runtime_inputs is not None else inputs, outputs)
    return outputs


def _rel_err(y, ref, mag):
    return float(np.max(np.abs(y.astype(np.float64) - ref.astype(np.float64)) / (mag + 1e-30)))


# ------------------------------------------------------------------------------ MatMul
def test_matmul_kat(be):
    B = _B()
    a = B.Tensor.from_data("a", [2, 3], B.DataType.F32, K.MATMUL_A)
    b = B.Tensor.from_data("b", [3, 2], B.DataType.F32, K.MATMUL_B)
    c = B.Tensor("c", [1], B.DataType.F32, np.zeros(4, np.float32))
    _run(be, B.OperatorDef("matmul", B.OperatorType.MatMul), [a, b], [c])
    assert c.shape == [2, 2]
    assert np.allclose(c.numpy(), K.MATMUL_C, atol=1e-3)


def test_matmul_ones_kat(be):
    B = _B()
    r = K.MATMUL_ONES
    a = B.Tensor("a", [r["m"], r["k"]], B.DataType.F32, np.ones((r["m"], r["k"]), np.float32))
    b = B.Tensor("b", [r["k"], r["n"]], B.DataType.F32, np.ones((r["k"], r["n"]), np.float32))
    c = B.Tensor("c", [1], B.DataType.F32, np.zeros(r["m"] * r["n"], np.float32))
    _run(be, B.OperatorDef("matmul", B.OperatorType.MatMul), [a, b], [c])
    assert c.shape == [r["m"], r["n"]] and np.allclose(c.numpy(), r["value"], atol=1e-3)


@pytest.mark.parametrize("m,k,n", [(512, 512, 512), (65, 67, 63), (3, 7, 5), (300, 1000, 129)])
@pytest.mark.parametrize("mode", [0, 1])
def test_matmul_random(be, m, k, n, mode):
    """The 512^3 case is the FP32 GEMM workload (A, B ~ U[-1, 1])."""
    B = _B()
    rng = np.random.default_rng(m + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c = B.Tensor("c", [1], B.DataType.F32, np.zeros(m * n, np.float32))
    _run(be, B.OperatorDef("matmul", B.OperatorType.MatMul, fp32_mode=mode),
         [B.Tensor("a", [m, k], B.DataType.F32, a), B.Tensor("b", [k, n], B.DataType.F32, b)], [c])
    ref = orc.matmul(a, b)
    mag = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)
    assert _rel_err(c.numpy().reshape(m, n), ref, mag) <= (TOL_3XTF32 if mode == 0 else TOL_TF32)


def test_matmul_dimension_mismatch(be):
    B = _B()
    a = B.Tensor("a", [2, 3], B.DataType.F32, np.zeros((2, 3), np.float32))
    b = B.Tensor("b", [4, 2], B.DataType.F32, np.zeros((4, 2), np.float32))
    op = be.compile_operator(B.OperatorDef("matmul", B.OperatorType.MatMul), None, [a, b],
                             [B.Tensor("c", [1], B.DataType.F32)])
    with pytest.raises(B.LightShipError) as e:
        be.execute(op, [a, b], [B.Tensor("c", [1], B.DataType.F32, np.zeros(4, np.float32))])
    assert e.value.code == 7 and "mismatch" in str(e.value)


# ------------------------------------------------------------------------------ FullyConnected
def test_fc_kat(be):
    B = _B()
    x = B.Tensor.from_data("x", [1, 4], B.DataType.F32, K.FC_X)
    w = B.Tensor.from_data("w", [3, 4], B.DataType.F32, K.FC_W)
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(3, np.float32))
    _run(be, B.OperatorDef("fc", B.OperatorType.FullyConnected), [x, w], [y], runtime_inputs=[x])
    assert y.shape == [1, 3] and np.allclose(y.numpy(), K.FC_Y, atol=1e-3)


@pytest.mark.parametrize("mode", [0, 1])
def test_fc_random_with_bias(be, mode):
    B = _B()
    rng = np.random.default_rng(10 + mode)
    bsz, fin, fout = 256, 512, 1000  # ResNet-18's FC at batch 256
    x = rng.normal(size=(bsz, fin)).astype(np.float32)
    w = rng.normal(0, 0.05, size=(fout, fin)).astype(np.float32)
    bias = rng.normal(size=fout).astype(np.float32)
    xt = B.Tensor("x", [bsz, fin], B.DataType.F32, x)
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(bsz * fout, np.float32))
    _run(be, B.OperatorDef("fc", B.OperatorType.FullyConnected, fp32_mode=mode),
         [xt, B.Tensor("w", [fout, fin], B.DataType.F32, w), B.Tensor("b", [fout], B.DataType.F32, bias)],
         [y], runtime_inputs=[xt])
    ref = orc.fully_connected(x, w) + bias
    mag = np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T + np.abs(bias)
    assert _rel_err(y.numpy().reshape(bsz, fout), ref, mag) <= (TOL_3XTF32 if mode == 0 else TOL_TF32)


# ------------------------------------------------------------------------------ Conv2d FP32
def test_conv_kats(be):
    B = _B()
    r = K.CONV_ONES
    x = B.Tensor("x", list(r["x_shape"]), B.DataType.F32, np.ones(r["x_shape"], np.float32))
    w = B.Tensor("w", list(r["w_shape"]), B.DataType.F32, np.ones(r["w_shape"], np.float32))
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(4, np.float32))
    _run(be, B.OperatorDef("conv", B.OperatorType.Conv2d), [x, w], [y])
    assert y.shape == list(r["y_shape"]) and np.allclose(y.numpy(), r["value"], atol=1e-5)
    r = K.CONV_BATCHED
    xb = np.concatenate([np.full((1,) + r["x_shape"][1:], b + 1, np.float32) for b in range(4)])
    x = B.Tensor("x", list(r["x_shape"]), B.DataType.F32, xb)
    w = B.Tensor("w", list(r["w_shape"]), B.DataType.F32, np.ones(r["w_shape"], np.float32))
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(16, np.float32))
    _run(be, B.OperatorDef("conv", B.OperatorType.Conv2d), [x, w], [y])
    out = y.numpy().reshape(r["y_shape"])
    for b in range(4):
        assert np.allclose(out[b], 9.0 * (b + 1), atol=1e-3)
    r = K.CONV_STRIDE2
    x = B.Tensor("x", list(r["x_shape"]), B.DataType.F32, np.ones(r["x_shape"], np.float32))
    w = B.Tensor("w", list(r["w_shape"]), B.DataType.F32, np.ones(r["w_shape"], np.float32))
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(4, np.float32))
    _run(be, B.OperatorDef("conv", B.OperatorType.Conv2d, stride=(2, 2)), [x, w], [y])
    assert y.shape == list(r["y_shape"]) and np.allclose(y.numpy(), 4.0)
    r = K.ONNX_CONV_RELU
    x = B.Tensor("x", list(r["x_shape"]), B.DataType.F32, np.ones(r["x_shape"], np.float32))
    w = B.Tensor("w", list(r["w_shape"]), B.DataType.F32, np.ones(r["w_shape"], np.float32))
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(int(np.prod(r["y_shape"])), np.float32))
    _run(be, B.OperatorDef("conv", B.OperatorType.Conv2d), [x, w], [y], fusion=B.FusionInfo.conv_relu())
    assert y.shape == list(r["y_shape"]) and np.allclose(y.numpy(), 27.0)


def _bn_params(rng, co):
    g = rng.uniform(0.5, 1.5, co).astype(np.float32)
    be_ = rng.normal(0, 0.1, co).astype(np.float32)
    mu = rng.normal(0, 0.1, co).astype(np.float32)
    var = rng.uniform(0.5, 1.5, co).astype(np.float32)
    return g, be_, mu, var


@pytest.mark.parametrize("mode", [0, 1])
def test_conv_bn_relu_config(be, mode):
    """The FP32 Conv2d workload: 1x64x56x56, 3x3 s1 p1, 64 out, He-normal weights, bias,
    BatchNorm folded (gamma~U[0.5,1.5], beta~N(0,0.1), mean~N(0,0.1), var~U[0.5,1.5]) + ReLU.
    Oracle: unfused conv -> BatchNorm -> ReLU."""
    B = _B()
    rng = np.random.default_rng(56)
    x = rng.normal(size=(1, 64, 56, 56)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / 576), size=(64, 64, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, 64).astype(np.float32)
    g, beta, mu, var = _bn_params(rng, 64)
    T = lambda n, a: B.Tensor(n, list(a.shape), B.DataType.F32, a)
    xt = T("x", x)
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(64 * 56 * 56, np.float32))
    opdef = B.OperatorDef("conv", B.OperatorType.Conv2d, padding=(1, 1), activation=B.Activation.ReLU,
                          fp32_mode=mode)
    _run(be, opdef, [xt, T("w", w), T("b", bias), T("g", g), T("beta", beta), T("mu", mu), T("var", var)],
         [y], fusion=B.FusionInfo.conv_batch_norm(), runtime_inputs=[xt])
    ref = orc.act(orc.batchnorm_inference(orc.conv2d_nchw(x, w, bias, pad=(1, 1)), g, beta, mu, var),
                  orc.ACT_RELU)
    f = (g / np.sqrt(var + np.float32(1e-5))).astype(np.float64)
    mag = orc.conv2d_nchw(np.abs(x), np.abs(w), pad=(1, 1)).astype(np.float64) * f[None, :, None, None] \
        + np.abs(f * (bias - mu) + beta)[None, :, None, None]
    assert y.shape == [1, 64, 56, 56]
    assert _rel_err(y.numpy().reshape(ref.shape), ref, mag) <= (TOL_3XTF32 if mode == 0 else TOL_TF32)


@pytest.mark.parametrize("n,ci,co,h,wd,k,s,p,d", [(2, 3, 16, 32, 32, 3, 1, 0, 1),
                                                  (2, 8, 12, 13, 11, 5, 2, 2, 1),
                                                  (1, 64, 128, 28, 28, 3, 2, 1, 1),
                                                  (3, 6, 4, 13, 11, 7, 2, 3, 1),
                                                  (2, 16, 24, 15, 15, 3, 1, 2, 2)])
def test_conv_f32_geometry(be, n, ci, co, h, wd, k, s, p, d):
    B = _B()
    rng = np.random.default_rng(n * 100 + ci + co)
    x = rng.normal(size=(n, ci, h, wd)).astype(np.float32)
    w = rng.normal(0, 0.2, size=(co, ci, k, k)).astype(np.float32)
    bias = rng.normal(size=co).astype(np.float32)
    xt = B.Tensor("x", list(x.shape), B.DataType.F32, x)
    oh = (h + 2 * p - d * (k - 1) - 1) // s + 1
    ow = (wd + 2 * p - d * (k - 1) - 1) // s + 1
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(n * co * oh * ow, np.float32))
    _run(be, B.OperatorDef("conv", B.OperatorType.Conv2d, stride=(s, s), padding=(p, p), dilation=(d, d)),
         [xt, B.Tensor("w", list(w.shape), B.DataType.F32, w), B.Tensor("b", [co], B.DataType.F32, bias)], [y],
         runtime_inputs=[xt])
    ref = orc.conv2d_nchw(x, w, bias, (s, s), (p, p), (d, d))
    mag = orc.conv2d_nchw(np.abs(x), np.abs(w), None, (s, s), (p, p), (d, d)).astype(np.float64) + np.abs(bias)[None, :, None, None]
    assert y.shape == list(ref.shape)
    assert _rel_err(y.numpy().reshape(ref.shape), ref, mag) <= TOL_3XTF32


def test_conv_groups_kat(be):
    """convolution.rs:411-447: groups=2, input channels filled 1, 2, 3, 4, a 1x1 ones filter of
    shape [4, 2, 1, 1]: output channels 0-1 sum channels 0-1 (3), channels 2-3 sum 2-3 (7)."""
    B = _B()
    r = K.CONV_GROUPS
    x = np.stack([np.full((2, 2), v, np.float32) for v in r["channel_values"]])[None]
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(16, np.float32))
    _run(be, B.OperatorDef("conv", B.OperatorType.Conv2d, groups=r["groups"]),
         [B.Tensor("x", list(x.shape), B.DataType.F32, x),
          B.Tensor("w", list(r["w_shape"]), B.DataType.F32, np.ones(r["w_shape"], np.float32))], [y])
    assert y.shape == list(r["y_shape"])
    out = y.numpy().reshape(r["y_shape"])
    assert np.all(out[0, :2] == 3.0) and np.all(out[0, 2:] == 7.0)


@pytest.mark.parametrize("n,ci,co,h,k,s,p,g", [(2, 8, 12, 13, 3, 1, 1, 2), (1, 32, 32, 14, 3, 2, 1, 32),
                                               (2, 12, 6, 9, 5, 1, 2, 3)])
def test_conv_f32_groups(be, n, ci, co, h, k, s, p, g):
    B = _B()
    rng = np.random.default_rng(n * 1000 + ci * 10 + g)
    x = rng.normal(size=(n, ci, h, h)).astype(np.float32)
    w = rng.normal(0, 0.2, size=(co, ci // g, k, k)).astype(np.float32)
    bias = rng.normal(size=co).astype(np.float32)
    xt = B.Tensor("x", list(x.shape), B.DataType.F32, x)
    oh = (h + 2 * p - k) // s + 1
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(n * co * oh * oh, np.float32))
    _run(be, B.OperatorDef("conv", B.OperatorType.Conv2d, stride=(s, s), padding=(p, p), groups=g),
         [xt, B.Tensor("w", list(w.shape), B.DataType.F32, w), B.Tensor("b", [co], B.DataType.F32, bias)], [y],
         runtime_inputs=[xt])
    ref = orc.conv2d_nchw(x, w, bias, (s, s), (p, p), groups=g)
    mag = orc.conv2d_nchw(np.abs(x), np.abs(w), None, (s, s), (p, p), groups=g).astype(np.float64) \
        + np.abs(bias)[None, :, None, None]
    assert y.shape == list(ref.shape)
    assert _rel_err(y.numpy().reshape(ref.shape), ref, mag) <= TOL_3XTF32


def test_conv_groups_must_divide_output_channels(be):
    B = _B()
    x = B.Tensor("x", [1, 4, 2, 2], B.DataType.F32, np.ones((1, 4, 2, 2), np.float32))
    w = B.Tensor("w", [3, 2, 1, 1], B.DataType.F32, np.ones((3, 2, 1, 1), np.float32))
    with pytest.raises(B.LightShipError) as e:
        be.compile_operator(B.OperatorDef("conv", B.OperatorType.Conv2d, groups=2), None, [x, w],
                            [B.Tensor("y", [1], B.DataType.F32)])
    assert e.value.code == 2  # LSC_ERROR_INVALID_ARGUMENT


# ------------------------------------------------------------------------------ BatchNorm / activations
def test_batchnorm_kats(be):
    B = _B()
    r = K.BN_DEFAULTS
    x = B.Tensor("x", list(r["shape"]), B.DataType.F32, np.full(r["shape"], r["value"], np.float32))
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(int(np.prod(r["shape"])), np.float32))
    _run(be, B.OperatorDef("bn", B.OperatorType.BatchNorm), [x], [y])
    assert y.shape == list(r["shape"]) and np.allclose(y.numpy(), r["value"], atol=r["tol"])
    for r, shape in ((K.BN_NONZERO_MEAN, (1, 1, 4)), (K.BN_GAMMA_BETA, (1, 1, 4)), (K.BN_MULTI, K.BN_MULTI["shape"])):
        x = B.Tensor.from_data("x", list(shape), B.DataType.F32, r["x"])
        params = [B.Tensor.from_data(n, [len(r[n])], B.DataType.F32, r[n]) for n in ("gamma", "beta", "mean", "var")]
        y = B.Tensor("y", [1], B.DataType.F32, np.zeros(len(r["x"]), np.float32))
        _run(be, B.OperatorDef("bn", B.OperatorType.BatchNorm), [x] + params, [y], runtime_inputs=[x])
        assert np.allclose(y.numpy().ravel(), r["y"], atol=1e-3)


@pytest.mark.parametrize("fused_relu", [False, True])
def test_batchnorm_bit_exact_batch_gt_one(be, fused_relu):
    B = _B()
    rng = np.random.default_rng(33)
    x = rng.normal(size=(4, 24, 9, 7)).astype(np.float32)
    g, beta, mu, var = _bn_params(rng, 24)
    xt = B.Tensor("x", list(x.shape), B.DataType.F32, x)
    params = [B.Tensor(n, [24], B.DataType.F32, a) for n, a in (("g", g), ("b", beta), ("m", mu), ("v", var))]
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(x.size, np.float32))
    fusion = B.FusionInfo(B.FusionType.BatchNormReLU, [B.OperatorType.BatchNorm, B.OperatorType.ReLU]) if fused_relu else None
    _run(be, B.OperatorDef("bn", B.OperatorType.BatchNorm), [xt] + params, [y], fusion=fusion, runtime_inputs=[xt])
    ref = orc.batchnorm_inference(x, g, beta, mu, var)
    if fused_relu:
        ref = orc.act(ref, orc.ACT_RELU)
    np.testing.assert_array_equal(y.numpy().reshape(x.shape).view(np.uint32), ref.view(np.uint32))


def test_activation_kats_and_bits(be):
    B = _B()
    rng = np.random.default_rng(5)
    big = np.concatenate([np.array(K.ACT_IN, np.float32), np.array([-0.0, np.nan, 20.5, -20.5, 19.9], np.float32),
                          rng.normal(0, 8, 100_001).astype(np.float32)])
    for optype, kind, kat in ((B.OperatorType.ReLU, orc.ACT_RELU, K.RELU_OUT),
                              (B.OperatorType.ReLU6, orc.ACT_RELU6, K.RELU6_OUT),
                              (B.OperatorType.SiLU, orc.ACT_SILU, None)):
        x = B.Tensor("x", [big.size], B.DataType.F32, big)
        y = B.Tensor("y", [1], B.DataType.F32, np.zeros(big.size, np.float32))
        _run(be, B.OperatorDef("act", optype), [x], [y])
        got, ref = y.numpy(), orc.act(big, kind)
        if kat is not None:
            assert got[:len(kat)].tolist() == kat
        else:
            for xv, want, tol in K.SILU_POINTS:
                assert abs(orc.act(np.float32([xv]), kind)[0] - want) < tol
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_silu_bit_exact_over_its_exp_range(cuda):
    """SiLU on every 7th float of [-20.5, 20.5] (the range where it evaluates exp, and past the
    cut-offs), on the device, against the oracle's x / (1 + expf(-x)) bit for bit."""
    import torch
    B = _B()
    be = B.CudaBackend(B.GpuBackendConfig(device_id=0, arena_bytes=64 << 20))
    try:
        op = None
        for lo, hi in ((0x00000000, 0x41A40000), (0x80000000, 0xC1A40000)):
            bits = np.arange(lo, hi, 7, dtype=np.uint64).astype(np.uint32)
            x = bits.view(np.float32)
            xt = B.Tensor("x", [x.size], B.DataType.F32, torch.from_numpy(x).to(cuda))
            yd = torch.empty(x.size, dtype=torch.float32, device=cuda)
            yt = B.Tensor("y", [x.size], B.DataType.F32, yd)
            if op is None:
                op = be.compile_operator(B.OperatorDef("silu", B.OperatorType.SiLU), None, [xt], [yt])
            be.execute(op, [xt], [yt])
            got = yd.cpu().numpy()
            ref = orc.act(x, orc.ACT_SILU)
            np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
        del op
    finally:
        be.close()


# ------------------------------------------------------------------------------ INT8 Conv2d via the Backend
@pytest.mark.parametrize("fold_bn", [False, True])
def test_conv_int8_compiled_from_f32_weights(be, fold_bn):
    """Conv2d on int8 NHWC activations: the backend folds BN into the f32 weights, quantizes
    them per output channel, quantizes the bias to int32 and runs the INT8 chain; the oracle
    takes the same steps with its own code."""
    B = _B()
    rng = np.random.default_rng(7 + fold_bn)
    n, h, wd, ci, co = 2, 14, 14, 64, 96
    x = rng.integers(-127, 128, size=(n, h, wd, ci), dtype=np.int8)
    w = rng.normal(0, np.sqrt(2 / (9 * ci)), size=(co, ci, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, co).astype(np.float32)
    s_a, s_out = 0.02, 0.05
    g, beta, mu, var = _bn_params(rng, co)
    if fold_bn:
        wf, bf = orc.bn_fold(w, bias, g, beta, mu, var)
    else:
        wf, bf = w, bias
    w_ohwi = np.ascontiguousarray(wf.transpose(0, 2, 3, 1))
    wq, sw = orc.quantize_weights_per_channel(w_ohwi)
    scale = (np.float32(s_a) * sw).astype(np.float32)
    bq = np.array([orc.quantize_value(float(bf[o]), float(scale[o]), 0, orc.QINT32) for o in range(co)], np.int32)
    want = orc.conv2d_i8_nhwc_chain(x, wq, bq, scale, (1, 1), (1, 1), (1, 1), 1, orc.ACT_RELU, s_out,
                                    orc.ROUND_HALF_EVEN)
    xt = B.Tensor("x", list(x.shape), B.DataType.QInt8, x, layout=B.StorageLayout.NHWC,
                  quantization=B.Quantization([s_a]))
    T = lambda nm, a: B.Tensor(nm, list(a.shape), B.DataType.F32, a)
    ins = [xt, T("w", w), T("b", bias)] + ([T("g", g), T("beta", beta), T("mu", mu), T("var", var)] if fold_bn else [])
    q = B.Tensor("q", [1], B.DataType.QInt8, np.zeros(want[0].size, np.int8))
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(want[0].size, np.float32))
    acc = B.Tensor("acc", [1], B.DataType.I32, np.zeros(want[0].size, np.int32))
    fusion = B.FusionInfo.conv_batch_norm() if fold_bn else B.FusionInfo.conv_relu()
    opdef = B.OperatorDef("conv", B.OperatorType.Conv2d, padding=(1, 1), activation=B.Activation.ReLU,
                          rounding=B.Rounding.HalfEven, output_scale=s_out)
    _run(be, opdef, ins, [q, y, acc], fusion=fusion, runtime_inputs=[xt])
    assert q.shape == [n, h, wd, co]
    np.testing.assert_array_equal(acc.numpy().reshape(want[2].shape), want[2])
    np.testing.assert_array_equal(y.numpy().reshape(want[1].shape).view(np.uint32), want[1].view(np.uint32))
    np.testing.assert_array_equal(q.numpy().reshape(want[0].shape), want[0])


@pytest.mark.parametrize("ci,co,groups,stride", [(64, 64, 2, 1), (32, 64, 4, 2), (48, 48, 48, 1)])
def test_conv_int8_groups(be, ci, co, groups, stride):
    """Grouped INT8 Conv2d (the last case depthwise): the backend quantizes the grouped f32
    filter per output channel and runs it densely with zeros outside each group; the oracle runs
    its grouped int8 convolution on the same quantized weights.  Bit-exact."""
    B = _B()
    rng = np.random.default_rng(ci + co + groups)
    n, h = 2, 11
    cig = ci // groups
    x = rng.integers(-127, 128, size=(n, h, h, ci), dtype=np.int8)
    w = rng.normal(0, np.sqrt(2 / (9 * cig)), size=(co, cig, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, co).astype(np.float32)
    s_a, s_out = 0.02, 0.05
    wq, sw = orc.quantize_weights_per_channel(np.ascontiguousarray(w.transpose(0, 2, 3, 1)))
    scale = (np.float32(s_a) * sw).astype(np.float32)
    bq = np.array([orc.quantize_value(float(bias[o]), float(scale[o]), 0, orc.QINT32) for o in range(co)], np.int32)
    want = orc.conv2d_i8_nhwc_chain(x, wq, bq, scale, (stride, stride), (1, 1), (1, 1), groups, orc.ACT_RELU,
                                    s_out, orc.ROUND_HALF_AWAY)
    xt = B.Tensor("x", list(x.shape), B.DataType.QInt8, x, layout=B.StorageLayout.NHWC,
                  quantization=B.Quantization([s_a]))
    q = B.Tensor("q", [1], B.DataType.QInt8, np.zeros(want[0].size, np.int8))
    acc = B.Tensor("acc", [1], B.DataType.I32, np.zeros(want[0].size, np.int32))
    opdef = B.OperatorDef("conv", B.OperatorType.Conv2d, stride=(stride, stride), padding=(1, 1), groups=groups,
                          activation=B.Activation.ReLU, output_scale=s_out)
    _run(be, opdef, [xt, B.Tensor("w", list(w.shape), B.DataType.F32, w), B.Tensor("b", [co], B.DataType.F32, bias)],
         [q, acc], fusion=B.FusionInfo.conv_relu(), runtime_inputs=[xt])
    assert q.shape == list(want[0].shape)
    np.testing.assert_array_equal(acc.numpy().reshape(want[2].shape), want[2])
    np.testing.assert_array_equal(q.numpy().reshape(want[0].shape), want[0])


# ------------------------------------------------------------------------------ Winograd
TOL_WINOGRAD = 1e-4  # |y - y_oracle| <= tol * (sum |x * w| + |bias|): transforms + split-TF32


@pytest.mark.parametrize("n,ci,co,h,wd,p", [(1, 64, 64, 56, 56, 1), (2, 5, 7, 9, 11, 1), (1, 16, 8, 10, 10, 0),
                                            (1, 8, 70, 7, 7, 2), (3, 3, 4, 6, 5, 1), (2, 130, 96, 15, 13, 1)])
def test_conv_winograd_matches_oracle(be, n, ci, co, h, wd, p):
    """fp32_mode LSC_FP32_WINOGRAD: the 3x3 stride-1 convolution as Winograd F(2x2, 3x3)
    (input transform, 16-batch split-TF32 GEMM, output transform) against the oracle's direct
    convolution; odd output sizes, channel counts off the 4 / 32 / 64 grids, padding 0-2."""
    B = _B()
    rng = np.random.default_rng(n * 1000 + ci * 7 + co + p)
    x = rng.normal(size=(n, ci, h, wd)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / (9 * ci)), size=(co, ci, 3, 3)).astype(np.float32)
    bias = rng.normal(size=co).astype(np.float32)
    xt = B.Tensor("x", list(x.shape), B.DataType.F32, x)
    oh, ow = h + 2 * p - 2, wd + 2 * p - 2
    y = B.Tensor("y", [1], B.DataType.F32, np.full(n * co * oh * ow, np.nan, np.float32))
    _run(be, B.OperatorDef("conv", B.OperatorType.Conv2d, padding=(p, p), fp32_mode=_lib().FP32_WINOGRAD),
         [xt, B.Tensor("w", list(w.shape), B.DataType.F32, w), B.Tensor("b", [co], B.DataType.F32, bias)], [y],
         runtime_inputs=[xt])
    ref = orc.conv2d_nchw(x, w, bias, (1, 1), (p, p))
    mag = orc.conv2d_nchw(np.abs(x), np.abs(w), None, (1, 1), (p, p)).astype(np.float64) + np.abs(bias)[None, :, None, None]
    assert y.shape == list(ref.shape)
    assert _rel_err(y.numpy().reshape(ref.shape), ref, mag) <= TOL_WINOGRAD


def test_conv_winograd_bn_relu_config(be):
    """The FP32 Conv2d workload (1x64x56x56, 3x3 s1 p1, bias, folded BatchNorm, ReLU) on the
    Winograd path."""
    B = _B()
    rng = np.random.default_rng(56)
    x = rng.normal(size=(1, 64, 56, 56)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / 576), size=(64, 64, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, 64).astype(np.float32)
    g, beta, mu, var = _bn_params(rng, 64)
    T = lambda n, a: B.Tensor(n, list(a.shape), B.DataType.F32, a)
    xt = T("x", x)
    y = B.Tensor("y", [1], B.DataType.F32, np.zeros(64 * 56 * 56, np.float32))
    opdef = B.OperatorDef("conv", B.OperatorType.Conv2d, padding=(1, 1), activation=B.Activation.ReLU,
                          fp32_mode=_lib().FP32_WINOGRAD)
    _run(be, opdef, [xt, T("w", w), T("b", bias), T("g", g), T("beta", beta), T("mu", mu), T("var", var)],
         [y], fusion=B.FusionInfo.conv_batch_norm(), runtime_inputs=[xt])
    ref = orc.act(orc.batchnorm_inference(orc.conv2d_nchw(x, w, bias, pad=(1, 1)), g, beta, mu, var),
                  orc.ACT_RELU)
    f = (g / np.sqrt(var + np.float32(1e-5))).astype(np.float64)
    mag = orc.conv2d_nchw(np.abs(x), np.abs(w), pad=(1, 1)).astype(np.float64) * f[None, :, None, None] \
        + np.abs(f * (bias - mu) + beta)[None, :, None, None]
    assert _rel_err(y.numpy().reshape(ref.shape), ref, mag) <= TOL_WINOGRAD


def test_conv_winograd_mode_leaves_other_convolutions_direct(be):
    """Under fp32_mode LSC_FP32_WINOGRAD a 5x5 or strided convolution runs the direct kernel."""
    B = _B()
    rng = np.random.default_rng(9)
    x = rng.normal(size=(1, 8, 12, 12)).astype(np.float32)
    for k, s in ((5, 1), (3, 2)):
        w = rng.normal(0, 0.2, size=(8, 8, k, k)).astype(np.float32)
        xt = B.Tensor("x", list(x.shape), B.DataType.F32, x)
        oh = (12 + 2 - k) // s + 1
        y = B.Tensor("y", [1], B.DataType.F32, np.zeros(8 * oh * oh, np.float32))
        _run(be, B.OperatorDef("conv", B.OperatorType.Conv2d, stride=(s, s), padding=(1, 1),
                               fp32_mode=_lib().FP32_WINOGRAD),
             [xt, B.Tensor("w", list(w.shape), B.DataType.F32, w)], [y], runtime_inputs=[xt])
        ref = orc.conv2d_nchw(x, w, None, (s, s), (1, 1))
        mag = orc.conv2d_nchw(np.abs(x), np.abs(w), None, (s, s), (1, 1)).astype(np.float64)
        assert _rel_err(y.numpy().reshape(ref.shape), ref, mag) <= TOL_3XTF32


def _lib():
    from lightship_b200 import _lib as L
    return L
