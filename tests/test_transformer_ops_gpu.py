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
    x = np.concatenate([np.linspace(-12, 12, 40001, dtype=np.float32),
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


@pytest.mark.parametrize("rows,d", [(384 * 4, 768), (33, 1000), (7, 4096), (5, 1)])
def test_layernorm_f32(be, rows, d):
    """f32: |Δ| <= 2e-5 + 2e-5 |y| against the oracle (different summation order)."""
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


@pytest.mark.parametrize("rows,d", [(32 * 12 * 384 // 8, 384), (50, 1000), (3, 1)])
def test_softmax_f32(be, rows, d):
    """f32: |Δ| <= 1e-7 + 1e-5 |y| against the oracle (device exp is the correctly rounded
    one, the oracle's glibc expf; tree-ordered sum)."""
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


def test_softmax_large_values_and_in_place(be):
    import torch
    from lightship_b200.backend import DataType, OperatorDef, OperatorType, Tensor
    x = np.array([[1000.0, 1001.0, 1002.0], [-1e30, 0.0, 1e30]], np.float32)
    xd = torch.from_numpy(x).cuda()
    t = Tensor("x", list(x.shape), DataType.F32, xd)
    op = be.compile_operator(OperatorDef("sm", OperatorType.Softmax), None, [t], [t])
    be.execute(op, [t], [t])
    np.testing.assert_allclose(xd.cpu().numpy(), orc.softmax(x), atol=1e-7, rtol=1e-5)
