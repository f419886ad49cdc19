"""Oracle restatements of the transformer-block operators pinned to the reference's own tests:
GELU (core/operator/gelu.rs tests), LayerNorm (layernorm.rs:250-300), Softmax
(softmax.rs:224-270).  Also records the reference GELU's polynomial-tanh behaviour, which the
CUDA path reproduces for parity."""
import numpy as np

from oracle import oracle as orc


def gelu(x):
    return orc.act(np.asarray(x, np.float32), orc.ACT_GELU)


def test_gelu_reference_kats():
    # gelu.rs tests: GELU(0) ~ 0, 0 < GELU(1) < 1, GELU(-1) < 0, small inputs keep their sign
    g = gelu([0.0, 1.0, -1.0, -0.1, 0.1])
    assert abs(g[0]) < 1e-4
    assert 0.0 < g[1] < 1.0
    assert g[2] < 0.0
    assert g[3] < 0.0 and g[4] > 0.0
    # test_gelu_slice: [-1, 0, 1]
    s = gelu([-1.0, 0.0, 1.0])
    assert s[0] < 0.0 and abs(s[1]) < 1e-4 and s[2] > 0.0


def test_gelu_polynomial_tanh_and_saturation():
    """The reference's tanh_approx is x - x^3/3 + x^5/5 - x^7/7 for |t| <= 5 (gelu.rs:91-103),
    which leaves tanh for |t| > ~1: GELU(3) comes out large and negative, while past the +-5
    cut-off (|x| > ~3.5) the tanh saturates and GELU(x) is x or -0."""
    x = np.array([3.0, 4.0, -4.0, 10.0, -10.0], np.float32)
    g = gelu(x)
    assert g[0] < -100.0
    assert g[1] == np.float32(4.0) and g[3] == np.float32(10.0)
    assert g[2] == 0.0 and g[4] == 0.0
    # the f32 expression in the reference's order
    t = np.float32(0.7978845608) * (np.float32(1.5) + np.float32(0.044715) * (np.float32(1.5) ** 3))
    t2 = t * t
    th = t - (t2 * t) / np.float32(3) + (t2 * t * t2) / np.float32(5) - (t2 * t * t2 * t2) / np.float32(7)
    assert gelu([1.5])[0] == np.float32(0.5) * np.float32(1.5) * (np.float32(1) + th)


def test_layernorm_reference_kats():
    y = orc.layernorm(np.array([[1.0, 2.0, 3.0, 4.0]], np.float32), eps=1e-5)
    # test_normalize: mean 2.5, normalised variance ~ 1
    assert abs(float(np.var(y)) - 1.0) < 0.01
    assert abs(float(np.mean(y))) < 1e-6
    # affine weight / bias as in test_layernorm_affine
    g = np.array([1, 2, 3, 4], np.float32)
    b = np.array([0.1, 0.2, 0.3, 0.4], np.float32)
    ya = orc.layernorm(np.array([[1.0, 2.0, 3.0, 4.0]], np.float32), g, b)
    np.testing.assert_allclose(ya, g * y + b, rtol=1e-6)


def test_softmax_reference_kats():
    y = orc.softmax(np.array([[1.0, 2.0, 3.0]], np.float32))
    assert abs(float(y.sum()) - 1.0) < 1e-4 and (y > 0).all() and np.argmax(y) == 2
    s = np.exp(-2.0) + np.exp(-1.0) + 1.0
    np.testing.assert_allclose(y[0], np.exp(np.array([-2.0, -1.0, 0.0])) / s, rtol=1e-6)
    big = orc.softmax(np.array([[1000.0, 1001.0, 1002.0]], np.float32))
    assert abs(float(big.sum()) - 1.0) < 1e-4


def test_layernorm_and_softmax_match_float64():
    rng = np.random.default_rng(0)
    x = rng.normal(size=(64, 768)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, 768).astype(np.float32)
    b = rng.normal(scale=0.1, size=768).astype(np.float32)
    xd = x.astype(np.float64)
    ref = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + 1e-5) * g + b
    np.testing.assert_allclose(orc.layernorm(x, g, b), ref, atol=2e-5, rtol=1e-5)
    e = np.exp(xd - xd.max(1, keepdims=True))
    np.testing.assert_allclose(orc.softmax(x), e / e.sum(1, keepdims=True), atol=1e-7, rtol=1e-5)


def _ln64(v, g, b):
    m = v.mean(-1, keepdims=True)
    return (v - m) / np.sqrt(((v - m) ** 2).mean(-1, keepdims=True) + 1e-5) * g + b


def test_attention_helpers_match_float64():
    """Q/K/V head slicing of the [tokens, 3*heads*dim] projection, Q K^T / 8, and P V."""
    rng = np.random.default_rng(0)
    b, s, h, d = 2, 32, 3, 64
    qkv = rng.standard_normal((b * s, 3 * h * d)).astype(np.float16)
    sc = orc.attention_scores_f16(qkv, b, s, h, d)
    q = qkv.astype(np.float64).reshape(b, s, 3, h, d)
    ref = np.einsum("bihd,bjhd->bhij", q[:, :, 0], q[:, :, 1]) / 8.0
    np.testing.assert_allclose(sc.astype(np.float64), ref, rtol=2e-3, atol=2e-3)
    p = orc.softmax(sc.astype(np.float32)).astype(np.float16)
    o = orc.attention_context(p, qkv, b, s, h, d)
    ref_o = np.einsum("bhij,bjhd->bihd", p.astype(np.float64), q[:, :, 2]).reshape(b * s, h * d)
    np.testing.assert_allclose(o, ref_o, rtol=1e-5, atol=1e-5)


def test_encoder_block_oracle_tracks_float_model():
    """The quantized block's attention half against a float64 restatement: the residual
    stream after the output projection agrees to the INT8 quantization error."""
    from lightship_b200.bert import build_params
    b, s = 1, 64
    p = build_params(3)
    x = np.random.default_rng(4).standard_normal((b * s, 768)).astype(np.float32)
    ln1 = orc.layernorm(x, p["ln1_g"], p["ln1_b"], 1e-5)
    scales = {"q1": orc.find_scale_zp(ln1)[0], "q2": 1.0, "q3": 1.0, "u": 1.0}
    scales["q2"] = orc.find_scale_zp(orc.encoder_block_int8(x, p, scales, b, s)["o"])[0]
    r = orc.encoder_block_int8(x, p, scales, b, s)
    a = _ln64(x.astype(np.float64), p["ln1_g"], p["ln1_b"])
    qkv = (a @ p["wqkv"].T.astype(np.float64) + p["bqkv"]).reshape(b, s, 3, 12, 64)
    sc = np.einsum("bihd,bjhd->bhij", qkv[:, :, 0], qkv[:, :, 1]) / 8.0
    e = np.exp(sc - sc.max(-1, keepdims=True))
    o = np.einsum("bhij,bjhd->bihd", e / e.sum(-1, keepdims=True), qkv[:, :, 2]).reshape(b * s, 768)
    h = o @ p["wo"].T.astype(np.float64) + p["bo"] + x
    assert np.linalg.norm(r["h"] - h) <= 0.05 * np.linalg.norm(h - x)
    # the int8 stages are the oracle's own quantize of its f32 stages
    assert np.array_equal(r["q1"], orc.quantize_tensor(r["ln1"], scales["q1"], 0))
    assert r["u"].dtype == np.int8 and r["out"].shape == (b * s, 768)
