"""Transformer-block operators on the GPU against the oracle:
- GELU fused into the INT8 chain's epilogue (single CTAs and CTA pairs) and as a standalone
  FP32 operator: bit-exact (the GELU has no transcendental function, every operation rounds
  as the reference's f32 code does);
- LayerNorm and Softmax over the last axis, f32 and f16 storage: within the tolerances stated
  in each test (tree-ordered device sums against the reference's sequential f32 sums; f16
  storage adds its own rounding)."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be(cuda):
    from lightship_b200.backend import CudaBackend, GpuBackendConfig
    b = CudaBackend(GpuBackendConfig(device_id=0, arena_bytes=256 << 20))
    yield b
    b.close()


@pytest.mark.parametrize("m,n,k", [(512, 3072, 768), (300, 200, 96), (4096, 768, 3072)])
def test_gemm_i8_gelu_epilogue(cuda, m, n, k):
    """The BERT FFN up-projection shape (INT8 GEMM + GELU), a ragged one and the
    down-projection shape on CTA pairs; scales chosen so y spans the polynomial's range."""
    import torch
    from lightship_b200 import ops
    rng = np.random.default_rng(m + n + k)
    a = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    b = rng.integers(-20000, 20000, size=n, dtype=np.int32)
    scale = rng.uniform(1e-5, 8e-5, size=n).astype(np.float32)
    for rounding in (orc.ROUND_HALF_AWAY, orc.ROUND_HALF_EVEN):
        want = orc.gemm_i8_chain(a, w, b, scale, orc.ACT_GELU, 0.02, rounding)
        q, y, acc = ops.gemm_i8(torch.from_numpy(a).to(cuda), torch.from_numpy(w).to(cuda),
                                torch.from_numpy(scale).to(cuda), torch.from_numpy(b).to(cuda), s_out=0.02,
                                act=orc.ACT_GELU, rounding=rounding, out_i8=True, out_f32=True, out_i32=True)
        ops.check_device()
        np.testing.assert_array_equal(acc.cpu().numpy(), want[2])
        np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), want[1].view(np.uint32))
        np.testing.assert_array_equal(q.cpu().numpy(), want[0])
    yv = want[1]
    assert (yv < 0).any() and (yv > 1).any()


def test_gelu_operator_f32(be):
    from lightship_b200.backend import DataType, OperatorDef, OperatorType, Tensor
    rng = np.random.default_rng(17)
    tiny = np.float32(2.0) ** rng.integers(-149, -100, 20000).astype(np.float32)
    x = np.concatenate([np.linspace(-12, 12, 40001, dtype=np.float32),
                        rng.uniform(-4, 4, 1 << 21).astype(np.float32), tiny, -tiny,
                        np.array([0.0, -0.0, np.inf, -np.inf, np.nan], np.float32)])
    xt = Tensor("x", [x.size], DataType.F32, x)
    yt = Tensor("y", [x.size], DataType.F32, np.zeros_like(x))
    op = be.compile_operator(OperatorDef("gelu", OperatorType.GELU), None, [xt], [yt])
    be.execute(op, [xt], [yt])
    got, want = yt.numpy(), orc.act(x, orc.ACT_GELU)
    # NaN results (from NaN and -inf inputs) carry the platform's default NaN bits (x86 and the
    # GPU differ, as the reference's own results would between platforms); all else bit for bit
    nan = np.isnan(want)
    assert nan.sum() == 2 and np.isnan(got[nan]).all()
    np.testing.assert_array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def _rownorm(be, kind, x, dtype, gamma=None, beta=None, eps=0.0):
    import torch
    from lightship_b200.backend import DataType, OperatorDef, OperatorType, Tensor
    dt = DataType.F32 if dtype == np.float32 else DataType.F16
    xs = x.astype(dtype)
    xd = torch.from_numpy(xs).cuda()
    yd = torch.empty_like(xd)
    xt = Tensor("x", list(x.shape), dt, xd)
    yt = Tensor("y", list(x.shape), dt, yd)
    ins = [xt]
    if gamma is not None:
        ins += [Tensor("g", [x.shape[-1]], DataType.F32, gamma), Tensor("b", [x.shape[-1]], DataType.F32, beta)]
    otype = OperatorType.LayerNorm if kind == "ln" else OperatorType.Softmax
    op = be.compile_operator(OperatorDef(kind, otype, epsilon=eps), None, ins, [yt])
    be.execute(op, [xt], [yt])
    torch.cuda.synchronize()
    return xs, yd.cpu().numpy()


@pytest.mark.parametrize("rows,d", [(384 * 4, 768), (33, 1000), (7, 4096), (5, 1), (9, 100), (3, 6)])
def test_layernorm_f32(be, rows, d):
    """f32: |Δ| <= 2e-5 + 2e-5 |y| against the oracle (different summation order).  Rows of
    up to 1024 (d % 4 == 0) take the warp-per-row kernel, the rest the CTA-per-row one."""
    rng = np.random.default_rng(rows + d)
    x = (rng.normal(size=(rows, d)) * 3 + 1).astype(np.float32)
    g = rng.uniform(0.5, 1.5, d).astype(np.float32)
    b = rng.normal(scale=0.1, size=d).astype(np.float32)
    _, y = _rownorm(be, "ln", x, np.float32, g, b, eps=1e-5)
    np.testing.assert_allclose(y, orc.layernorm(x, g, b, 1e-5), atol=2e-5, rtol=2e-5)


def test_layernorm_f16_and_default_eps(be):
    """f16 storage: the oracle on the same f16 inputs, its f32 result rounded to f16;
    |Δ| <= 1 f16 ulp (rtol 1e-3, atol 2e-3).  eps 0 selects the reference's 1e-5."""
    rng = np.random.default_rng(3)
    x = rng.normal(size=(1536, 768)).astype(np.float32)
    xs, y = _rownorm(be, "ln", x, np.float16, eps=0.0)
    want = orc.layernorm(xs.astype(np.float32), eps=1e-5).astype(np.float16)
    np.testing.assert_allclose(y.astype(np.float32), want.astype(np.float32), atol=2e-3, rtol=1e-3)


@pytest.mark.parametrize("rows,d", [(32 * 12 * 384 // 8, 384), (50, 1000), (3, 1), (17, 12), (4, 1028)])
def test_softmax_f32(be, rows, d):
    """f32: |Δ| <= 1e-7 + 1e-5 |y| against the oracle (device exp is CUDA's expf, within 2 ulp;
    the oracle's is glibc's; tree-ordered sum)."""
    rng = np.random.default_rng(rows + d)
    x = (rng.normal(size=(rows, d)) * 4).astype(np.float32)
    _, y = _rownorm(be, "sm", x, np.float32)
    want = orc.softmax(x)
    np.testing.assert_allclose(y, want, atol=1e-7, rtol=1e-5)
    np.testing.assert_allclose(y.sum(1), 1.0, rtol=1e-5)


def test_softmax_f16_attention_rows(be):
    """f16 attention scores (32 x 12 heads x 384 rows of 384, a slice): f16 ulp tolerance."""
    rng = np.random.default_rng(9)
    x = (rng.normal(size=(4608, 384)) * 3).astype(np.float32)
    xs, y = _rownorm(be, "sm", x, np.float16)
    want = orc.softmax(xs.astype(np.float32)).astype(np.float16)
    np.testing.assert_allclose(y.astype(np.float32), want.astype(np.float32), atol=2e-4, rtol=1e-3)


@pytest.mark.parametrize("pad", [0, 1])
def test_softmax_large_values_and_in_place(be, pad):
    """Rows of 3 (CTA kernel) and of 4 (warp kernel), updated in place; -inf entries give 0."""
    import torch
    from lightship_b200.backend import DataType, OperatorDef, OperatorType, Tensor
    x = np.array([[1000.0, 1001.0, 1002.0], [-1e30, 0.0, 1e30]], np.float32)
    if pad:
        x = np.concatenate([x, np.full((2, 1), -np.inf, np.float32)], axis=1)
    xd = torch.from_numpy(x).cuda()
    t = Tensor("x", list(x.shape), DataType.F32, xd)
    op = be.compile_operator(OperatorDef("sm", OperatorType.Softmax), None, [t], [t])
    be.execute(op, [t], [t])
    np.testing.assert_allclose(xd.cpu().numpy(), orc.softmax(x), atol=1e-7, rtol=1e-5)


def _assert_quantized_close(q, ref, scale, slack):
    """q equals quantize_tensor(ref, scale) except where ref / scale lies within `slack` of a
    rounding boundary (a tolerance-level difference in ref may move it across), and there by one."""
    want = orc.quantize_tensor(ref, scale, 0).astype(np.int32)
    diff = q.astype(np.int32) - want
    t = np.abs(ref.astype(np.float64) / scale)
    near = np.abs(t - np.floor(t) - 0.5) <= slack
    assert np.abs(diff).max() <= 1
    assert (diff[~near] == 0).all(), int((diff[~near] != 0).sum())


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
@pytest.mark.parametrize("rounding", [0, 1])
def test_layernorm_int8_output(be, dtype, rounding):
    """LayerNorm writing int8 (the following Quantize folded in): against the oracle's
    quantize_tensor of its LayerNorm, equal except within the LayerNorm tolerance of a rounding
    boundary; and equal to the device's own f32 LayerNorm quantized by the Quantize operator."""
    import torch
    from lightship_b200.backend import DataType, OperatorDef, OperatorType, Quantization, Rounding, Tensor
    rng = np.random.default_rng(11 + rounding)
    rows, d, s_q = 2048, 768, 0.04
    x = rng.normal(size=(rows, d)).astype(dtype)
    g = rng.uniform(0.8, 1.2, d).astype(np.float32)
    b = rng.normal(scale=0.02, size=d).astype(np.float32)
    dt = DataType.F32 if dtype == np.float32 else DataType.F16
    xt = Tensor("x", [rows, d], dt, torch.from_numpy(x).cuda())
    qd = torch.empty((rows, d), dtype=torch.int8, device="cuda")
    qt = Tensor("q", [rows, d], DataType.QInt8, qd, quantization=Quantization([s_q]))
    ins = [xt, Tensor("g", [d], DataType.F32, g), Tensor("b", [d], DataType.F32, b)]
    op = be.compile_operator(OperatorDef("lnq", OperatorType.LayerNorm, rounding=Rounding(rounding)), None, ins, [qt])
    be.execute(op, [xt], [qt])
    # the same LayerNorm to f32 (same kernel arithmetic), then the Quantize operator
    yd = torch.empty((rows, d), dtype=torch.float32 if dtype == np.float32 else torch.float16, device="cuda")
    yt = Tensor("y", [rows, d], dt, yd)
    op2 = be.compile_operator(OperatorDef("ln", OperatorType.LayerNorm), None, ins, [yt])
    be.execute(op2, [xt], [yt])
    torch.cuda.synchronize()
    if dtype == np.float32:
        q2 = torch.empty((rows, d), dtype=torch.int8, device="cuda")
        q2t = Tensor("q2", [rows, d], DataType.QInt8, q2, quantization=Quantization([s_q]))
        opq = be.compile_operator(OperatorDef("q", OperatorType.Quantize, rounding=Rounding(rounding)), None,
                                  [yt], [q2t])
        be.execute(opq, [yt], [q2t])
        torch.cuda.synchronize()
        assert torch.equal(q2, qd)
    ref = orc.layernorm(x.astype(np.float32), g, b, 1e-5)
    _assert_quantized_close(qd.cpu().numpy(), ref, s_q, 2e-3)  # LayerNorm |dy| <= 2e-5 ~ 5e-4 steps
    assert (qd.cpu().numpy() != 0).mean() > 0.9


@pytest.mark.parametrize("m,n,k,act", [(384, 2304, 768, 0), (300, 200, 96, 4), (1024, 768, 3072, 0), (129, 40, 64, 1),
                                       (2048, 1024, 256, 1), (12288, 2304, 768, 0), (12288, 768, 3072, 0),
                                       (12288, 768, 768, 0)])
def test_fully_connected_f16_output_and_f32_residual(be, cuda, m, n, k, act):
    """The INT8 FullyConnected writing f16 (the QKV projection feeding FP16 attention) and
    adding an f32 residual before the activation (output projection, FFN down): vector
    stores on full chunks, scalar stores on ragged N.  The shapes with N > 256 and at least 32
    tiles of 256 x 256 run on CTA pairs: 2048 x 1024 (exactly 32 pair tiles) and the BERT
    block's own projections at batch 32 x seq 384 = 12288 tokens (QKV 432 pair tiles, FFN down
    and output projection 144); the others on single CTAs."""
    import torch
    from lightship_b200.backend import Activation, DataType, OperatorDef, OperatorType, Quantization, Tensor
    rng = np.random.default_rng(m * 7 + n)
    s_a = 0.04
    a = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    bias = rng.normal(0, 0.02, size=n).astype(np.float32)
    res = rng.standard_normal((m, n)).astype(np.float32)
    xa = Tensor("a", [m, k], DataType.QInt8, torch.from_numpy(a).to(cuda), quantization=Quantization([s_a]))
    y16 = torch.empty((m, n), dtype=torch.float16, device=cuda)
    y32 = torch.empty((m, n), dtype=torch.float32, device=cuda)
    outs = [Tensor("y16", [m, n], DataType.F16, y16), Tensor("y32", [m, n], DataType.F32, y32)]
    op = be.compile_operator(OperatorDef("fc", OperatorType.FullyConnected, activation=Activation(act)), None,
                             [xa, Tensor("w", [n, k], DataType.F32, w), Tensor("b", [n], DataType.F32, bias)], outs)
    rt = Tensor("r", [m, n], DataType.F32, torch.from_numpy(res).to(cuda))
    be.execute(op, [xa, rt], outs)
    chain = orc.fc_i8_f32_weights(a, s_a, w, bias)[1]
    want = orc.act(chain + res, act)
    np.testing.assert_array_equal(y32.cpu().numpy().view(np.uint32), want.view(np.uint32))
    np.testing.assert_array_equal(y16.cpu().numpy().view(np.uint16), want.astype(np.float16).view(np.uint16))
    # without the residual the same operator reproduces the plain chain
    be.execute(op, [xa], outs)
    plain = orc.act(chain, act)
    np.testing.assert_array_equal(y32.cpu().numpy().view(np.uint32), plain.view(np.uint32))
