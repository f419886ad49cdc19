"""Pins the CPU oracle to LightShip's own known-answer tests (tests/golden/reference_kats.py)
and to math-level checks for what those tests leave unpinned (ties, per-channel, N>1 BN,
C_in>1 convolutions).  CPU only."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.golden import reference_kats as K


def f32(x):
    return np.asarray(x, np.float32)


# ---------------------------------------------------------------- INT8 primitives
def test_qgemm_kat():
    m, n, k = K.QGEMM_MNK
    a = np.array(K.QGEMM_A, np.int8).reshape(m, k)
    b = np.array(K.QGEMM_B, np.int8).reshape(k, n)
    assert orc.gemm_i8_nn(a, b).ravel().tolist() == K.QGEMM_C
    # the [N,K] weight layout gives the same sums
    assert orc.gemm_i8_tn(a, b.T.copy()).ravel().tolist() == K.QGEMM_C


def test_dequantize_kat():
    acc = np.array(K.DEQUANT_IN, np.int32).reshape(1, -1)
    scale = np.full(acc.shape[1], K.DEQUANT_SCALE, np.float32)
    _, y, _ = orc.requant(acc, None, scale)
    assert y.ravel().tolist() == K.DEQUANT_OUT


def test_quantize_sym_kat():
    q = orc.quantize_sym(f32(K.QSYM_IN), K.QSYM_SCALE, orc.ROUND_HALF_AWAY)
    assert q.tolist() == K.QSYM_OUT


def test_find_scale_zp_kats():
    s, z = orc.find_scale_zp(f32(K.FSZ_DATA), orc.QINT8, True)
    assert z == 0 and s == np.float32(1.0) / np.float32(127.0)
    s, z = orc.find_scale_zp(f32(K.FSZ_DATA), orc.QUINT8, False)
    assert z != 0  # asymmetric parameters are not symmetric (quantization_test.rs:93-99)
    assert s == np.float32(2.0) / np.float32(255.0)
    # zp = round(qmin - min/s) in f32: s = 2/255 rounds up, so -(-1)/s = 127.49999 -> 127
    zf = np.float32(0.0) - np.float32(-1.0) / np.float32(s)
    assert z == int(np.trunc(zf + np.copysign(np.float32(0.5), zf))) == 127
    # empty input -> QuantizationParameters::default() (scale 1, zp 0)
    assert orc.find_scale_zp(np.zeros(0, np.float32)) == (1.0, 0)


def test_quantize_roundtrip_kat():
    r = K.ROUNDTRIP
    q = orc.quantize_value(r["value"], r["scale"], r["zp"], orc.QINT8)
    assert abs(orc.dequantize_value(q, r["scale"], r["zp"]) - r["value"]) < r["tol"]


def test_quantize_value_semantics():
    # round half away from zero, then clamp
    assert orc.quantize_value(2.5, 1.0, 0, orc.QINT8) == 3
    assert orc.quantize_value(-2.5, 1.0, 0, orc.QINT8) == -3
    assert orc.quantize_value(1000.0, 1.0, 0, orc.QINT8) == 127
    assert orc.quantize_value(-1000.0, 1.0, 0, orc.QINT8) == -128
    assert orc.quantize_value(-1.0, 1.0, 0, orc.QUINT8) == 0
    assert orc.quantize_value(300.0, 1.0, 0, orc.QUINT8) == 255
    assert orc.quantize_value(float("nan"), 1.0, 5, orc.QINT8) == 5
    # the i32 add wraps as in a Rust release build: saturated 2^31-1 + 128 -> negative
    assert orc.quantize_value(1e30, 1.0, 128, orc.QUINT8) == 0


def test_non_quantized_dtypes_take_the_default_arm():
    """quantize_value and find_scale_zp send every dtype other than QUInt8 / QInt8 / QInt32
    (plain I8, I32, ...) to the `_` arm, (qmin, qmax) = (0, 255) (helpers.rs:109-114,
    :140-151)."""
    assert orc.quantize_value(-3.0, 1.0, 0, orc.OTHER) == 0
    assert orc.quantize_value(200.0, 1.0, 0, orc.OTHER) == 200
    assert orc.quantize_value(1000.0, 1.0, 0, orc.OTHER) == 255
    s, z = orc.find_scale_zp(f32([-2.0, 1.0]), orc.OTHER, True)
    assert z == 0 and s == np.float32(2.0) / np.float32(255.0)
    s, z = orc.find_scale_zp(f32([-2.0, 1.0]), orc.OTHER, False)
    assert s == np.float32(3.0) / np.float32(255.0)


def test_rounding_modes_on_ties():
    ties = f32([0.5, 1.5, 2.5, -0.5, -1.5, -2.5])
    away = [orc.lib().orc_round(float(t), orc.ROUND_HALF_AWAY) for t in ties]
    even = [orc.lib().orc_round(float(t), orc.ROUND_HALF_EVEN) for t in ties]
    assert away == [1.0, 2.0, 3.0, -1.0, -2.0, -3.0]
    assert even == [0.0, 2.0, 2.0, -0.0, -2.0, -2.0]


def test_requant_chain_matches_formula():
    rng = np.random.default_rng(11)
    acc = rng.integers(-2**20, 2**20, size=(8, 64), dtype=np.int32)
    bias = rng.integers(-1000, 1000, size=64, dtype=np.int32)
    scale = rng.uniform(1e-4, 1e-3, 64).astype(np.float32)
    q, y, a2 = orc.requant(acc, bias, scale, orc.ACT_RELU, 0.5, orc.ROUND_HALF_EVEN)
    ref_acc = acc + bias
    ref_y = (ref_acc.astype(np.float32) * scale).astype(np.float32)
    ref_y = np.where(ref_y > 0, ref_y, np.float32(0))
    ref_q = np.clip(np.rint(ref_y / np.float32(0.5)), -128, 127).astype(np.int8)
    assert (a2 == ref_acc).all()
    assert (y == ref_y).all()
    assert (q == ref_q).all()


def test_gemm_i8_chain_matches_int64():
    rng = np.random.default_rng(5)
    a = rng.integers(-128, 128, size=(33, 80), dtype=np.int8)
    w = rng.integers(-128, 128, size=(17, 80), dtype=np.int8)
    _, _, acc = orc.gemm_i8_chain(a, w, None, np.ones(17, np.float32))
    assert (acc == a.astype(np.int64) @ w.astype(np.int64).T).all()


def test_quantize_weights_per_channel():
    rng = np.random.default_rng(2)
    w = rng.normal(0, 0.02, size=(16, 3, 3, 8)).astype(np.float32)
    q, s = orc.quantize_weights_per_channel(w)
    absmax = np.abs(w.reshape(16, -1)).max(1)
    assert np.array_equal(s, (absmax / np.float32(127)).astype(np.float32))
    assert np.abs(q.reshape(16, -1)).max(1).tolist() == [127] * 16


# ---------------------------------------------------------------- FP32 GEMM / FC
def test_gemm_kats():
    m, n, k = K.GEMM_MNK
    a, b = f32(K.GEMM_A).reshape(m, k), f32(K.GEMM_B).reshape(k, n)
    assert orc.gemm_blocked(a, b).ravel().tolist() == K.GEMM_C
    c0 = f32(K.GEMM_C0).reshape(m, n)
    assert orc.gemm_blocked(a, b, c0).ravel().tolist() == K.GEMM_C_ACC
    assert orc.gemm_scalar(a, b, c0).ravel().tolist() == K.GEMM_C_ACC


def _ramp(n, step):
    return (np.arange(n, dtype=np.float32) * np.float32(step)).astype(np.float32)


def _seq_dot(a_row, b_col):
    s = np.float32(0)
    for x, y in zip(a_row, b_col):
        s = np.float32(s + np.float32(x * y))
    return s


def test_gemm_ramp_large_kat():
    r = K.GEMM_RAMP_LARGE
    m, n, k = r["m"], r["n"], r["k"]
    a = _ramp(m * k, r["a_step"]).reshape(m, k)
    b = _ramp(k * n, r["b_step"]).reshape(k, n)
    c = orc.gemm_blocked(a, b)
    for i, j in r["points"]:
        assert abs(c[i, j] - _seq_dot(a[i], b[:, j])) < r["abs_tol"]


def test_gemm_block_alignment_kat():
    r = K.GEMM_BLOCK_ALIGNMENT
    for m, n, k in r["cases"]:
        a = _ramp(m * k, r["step"]).reshape(m, k)
        b = _ramp(k * n, r["step"]).reshape(k, n)
        cb, cs = orc.gemm_blocked(a, b), orc.gemm_scalar(a, b)
        denom = np.where(np.abs(cs) > 1e-3, np.abs(cs), 1.0)
        assert (np.abs(cb - cs) / denom).max() < r["rel_tol"]


def test_gemm_ramp_256_kat():
    r = K.GEMM_RAMP_256
    a = _ramp(r["m"] * r["k"], r["a_step"]).reshape(r["m"], r["k"])
    b = _ramp(r["k"] * r["n"], r["b_step"]).reshape(r["k"], r["n"])
    c = orc.gemm_blocked(a, b)
    i, j = r["point"]
    e = _seq_dot(a[i], b[:, j])
    assert abs(c[i, j] - e) < abs(e) * 1e-3 + 1.0


def test_matmul_kats():
    a, b = f32(K.MATMUL_A).reshape(2, 3), f32(K.MATMUL_B).reshape(3, 2)
    assert np.allclose(orc.matmul(a, b).ravel(), K.MATMUL_C, atol=1e-3)
    r = K.MATMUL_ONES
    c = orc.matmul(np.ones((r["m"], r["k"]), np.float32), np.ones((r["k"], r["n"]), np.float32), threads=4)
    assert np.allclose(c, r["value"], atol=1e-3)


def test_matmul_threads_do_not_change_bits():
    rng = np.random.default_rng(9)
    a = rng.uniform(-1, 1, (257, 300)).astype(np.float32)
    b = rng.uniform(-1, 1, (300, 129)).astype(np.float32)
    assert np.array_equal(orc.matmul(a, b, 1), orc.matmul(a, b, 7))


def test_fc_kat():
    y = orc.fully_connected(f32(K.FC_X).reshape(1, 4), f32(K.FC_W).reshape(3, 4))
    assert np.allclose(y.ravel(), K.FC_Y, atol=1e-3)


# ---------------------------------------------------------------- Conv2d
def _conv_ref64(x, w, bias, stride, pad, dil, groups):
    """float64 direct convolution used to check the oracle's im2col path."""
    n, ci, h, wd = x.shape
    co, cpg, kh, kw = w.shape
    oh = (h + 2 * pad[0] - dil[0] * (kh - 1) - 1) // stride[0] + 1
    ow = (wd + 2 * pad[1] - dil[1] * (kw - 1) - 1) // stride[1] + 1
    xp = np.zeros((n, ci, h + 2 * pad[0], wd + 2 * pad[1]))
    xp[:, :, pad[0]:pad[0] + h, pad[1]:pad[1] + wd] = x
    y = np.zeros((n, co, oh, ow))
    opg = co // groups
    for o in range(co):
        g = o // opg
        for r in range(kh):
            for s in range(kw):
                patch = xp[:, g * cpg:(g + 1) * cpg,
                           r * dil[0]:r * dil[0] + stride[0] * (oh - 1) + 1:stride[0],
                           s * dil[1]:s * dil[1] + stride[1] * (ow - 1) + 1:stride[1]]
                y[:, o] += np.einsum("ncij,c->nij", patch, w[o, :, r, s].astype(np.float64))
    if bias is not None:
        y += bias[None, :, None, None]
    return y


def test_conv_kats():
    r = K.CONV_ONES
    y = orc.conv2d_nchw(np.ones(r["x_shape"], np.float32), np.ones(r["w_shape"], np.float32))
    assert y.shape == r["y_shape"] and np.allclose(y, r["value"], atol=1e-5)
    r = K.CONV_BATCHED
    x = np.concatenate([np.full((1,) + r["x_shape"][1:], b + 1, np.float32) for b in range(4)])
    y = orc.conv2d_nchw(x, np.ones(r["w_shape"], np.float32))
    assert y.shape == r["y_shape"]
    for b in range(4):
        assert np.allclose(y[b], 9.0 * (b + 1), atol=1e-3)
    r = K.CONV_STRIDE2
    y = orc.conv2d_nchw(np.ones(r["x_shape"], np.float32), np.ones(r["w_shape"], np.float32),
                        stride=(2, 2))
    assert y.shape == r["y_shape"] and np.allclose(y, 4.0)
    r = K.CONV_GROUPS
    x = np.stack([np.full((2, 2), v, np.float32) for v in r["channel_values"]])[None]
    y = orc.conv2d_nchw(x, np.ones(r["w_shape"], np.float32), groups=r["groups"])
    assert y.shape == r["y_shape"]
    assert np.allclose(y[0, :2], 3.0) and np.allclose(y[0, 2:], 7.0)
    r = K.CONV_OUT_SHAPE
    assert orc.conv_out_dim(r["in_hw"], r["k"], r["stride"], r["pad"], r["dil"]) == r["out"]
    r = K.ONNX_CONV_RELU
    y = orc.conv2d_nchw(np.ones(r["x_shape"], np.float32), np.ones(r["w_shape"], np.float32))
    assert y.shape == r["y_shape"]


@pytest.mark.parametrize("ci,co,k,s,p,d,g", [(3, 16, 3, 1, 1, 1, 1), (64, 64, 3, 1, 1, 1, 1),
                                             (8, 12, 5, 2, 2, 1, 1), (8, 8, 3, 1, 2, 2, 2),
                                             (6, 4, 7, 2, 3, 1, 1)])
def test_conv_against_float64(ci, co, k, s, p, d, g):
    rng = np.random.default_rng(ci * 100 + co)
    x = rng.normal(size=(2, ci, 13, 11)).astype(np.float32)
    w = rng.normal(0, 0.2, size=(co, ci // g, k, k)).astype(np.float32)
    b = rng.normal(size=co).astype(np.float32)
    y = orc.conv2d_nchw(x, w, b, (s, s), (p, p), (d, d), g)
    ref = _conv_ref64(x, w, b, (s, s), (p, p), (d, d), g)
    assert np.abs(y - ref).max() <= 1e-4 * (1 + np.abs(ref).max())


def test_reference_korder_defect_is_visible():
    """The reference pairs (kh,kw,c) columns with (c,kh,kw) filter rows; for C_in>1 and a
    kernel larger than 1x1 that is not a convolution.  The oracle follows the intended
    semantics and keeps the faithful variant only as this diagnostic."""
    rng = np.random.default_rng(1)
    x = rng.normal(size=(1, 4, 6, 6)).astype(np.float32)
    w = rng.normal(size=(2, 4, 3, 3)).astype(np.float32)
    good = orc.conv2d_nchw(x, w)
    bad = orc.conv2d_nchw(x, w, reference_korder=True)
    assert np.abs(good - _conv_ref64(x, w, None, (1, 1), (0, 0), (1, 1), 1)).max() < 1e-4
    assert np.abs(good - bad).max() > 1e-2
    # with C_in = 1 both orders agree (every reference conv test uses C_in = 1 or 1x1)
    x1 = x[:, :1].copy()
    w1 = w[:, :1].copy()
    assert np.array_equal(orc.conv2d_nchw(x1, w1), orc.conv2d_nchw(x1, w1, reference_korder=True))


# ---------------------------------------------------------------- BatchNorm / fold / act
def test_bn_kats():
    r = K.BN_DEFAULTS
    y = orc.batchnorm_inference(np.full(r["shape"], r["value"], np.float32))
    assert np.allclose(y, r["value"], atol=r["tol"])
    for r in (K.BN_NONZERO_MEAN, K.BN_GAMMA_BETA):
        y = orc.batchnorm_inference(f32(r["x"]).reshape(1, 1, 4), r["gamma"], r["beta"], r["mean"], r["var"])
        assert np.allclose(y.ravel(), r["y"], atol=1e-3)
    r = K.BN_MULTI
    y = orc.batchnorm_inference(f32(r["x"]).reshape(r["shape"]), r["gamma"], r["beta"], r["mean"], r["var"])
    assert np.allclose(y.ravel(), r["y"], atol=1e-3)


def test_bn_batch_gt_one_uses_each_images_channel():
    rng = np.random.default_rng(4)
    x = rng.normal(size=(3, 5, 7)).astype(np.float32)
    g, b = rng.uniform(0.5, 1.5, 5), rng.normal(0, 0.1, 5)
    mu, v = rng.normal(0, 0.1, 5), rng.uniform(0.5, 1.5, 5)
    y = orc.batchnorm_inference(x, g, b, mu, v)
    ref = (x - mu[None, :, None]) / np.sqrt(v[None, :, None] + 1e-5) * g[None, :, None] + b[None, :, None]
    assert np.abs(y - ref).max() < 1e-5


def test_bn_fold_equals_conv_then_bn():
    rng = np.random.default_rng(8)
    x = rng.normal(size=(2, 8, 9, 9)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / 72), size=(6, 8, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, 6).astype(np.float32)
    g, be = rng.uniform(0.5, 1.5, 6).astype(np.float32), rng.normal(0, 0.1, 6).astype(np.float32)
    mu, v = rng.normal(0, 0.1, 6).astype(np.float32), rng.uniform(0.5, 1.5, 6).astype(np.float32)
    unfused = orc.batchnorm_inference(orc.conv2d_nchw(x, w, bias, pad=(1, 1)), g, be, mu, v)
    wf, bf = orc.bn_fold(w, bias, g, be, mu, v)
    fused = orc.conv2d_nchw(x, wf, bf, pad=(1, 1))
    assert np.abs(fused - unfused).max() < 1e-4 * (1 + np.abs(unfused).max())


def test_activation_kats():
    assert orc.act(f32(K.ACT_IN), orc.ACT_RELU).tolist() == K.RELU_OUT
    assert orc.act(f32(K.ACT_IN), orc.ACT_RELU6).tolist() == K.RELU6_OUT
    for x, want, tol in K.SILU_POINTS:
        assert abs(orc.act(f32([x]), orc.ACT_SILU)[0] - want) < tol


def test_activation_signed_zero_and_nan():
    x = f32([-0.0, np.nan])
    r = orc.act(x, orc.ACT_RELU)
    assert r[0] == 0 and not np.signbit(r[0]) and r[1] == 0  # x > 0 ? x : 0
    r6 = orc.act(x, orc.ACT_RELU6)
    assert np.signbit(r6[0]) and np.isnan(r6[1])  # f32::clamp passes -0 and NaN through
    s = orc.act(f32([20.5, -20.5, 20.0]), orc.ACT_SILU)
    assert s[0] == np.float32(20.5) and s[1] == 0 and s[2] == np.float32(20.0)
    assert orc.act(f32([-19.5]), orc.ACT_SILU)[0] < 0  # inside the cut-offs: x / (1 + exp(-x))
