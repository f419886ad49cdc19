"""INT8 chain on the tensor cores vs the oracle: bit-exact int32 accumulators, f32
dequantized outputs and requantized int8 outputs, for every activation and both rounding
modes (quantized_ops.rs:13-48, helpers.rs:139-160)."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _run(cuda, a, w, bias, scale, act, s_out, rounding):
    import torch
    from lightship_b200 import ops
    ta = torch.from_numpy(a).to(cuda)
    tw = torch.from_numpy(w).to(cuda)
    ts = torch.from_numpy(scale).to(cuda)
    tb = None if bias is None else torch.from_numpy(bias).to(cuda)
    q, y, acc = ops.gemm_i8(ta, tw, ts, tb, s_out=s_out, act=act, rounding=rounding,
                            out_i8=True, out_f32=True, out_i32=True)
    ops.check_device()
    return q.cpu().numpy(), y.cpu().numpy(), acc.cpu().numpy()


def _case(rng, m, n, k, bias=True):
    a = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    b = rng.integers(-50000, 50000, size=n, dtype=np.int32) if bias else None
    scale = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    return a, w, b, scale


def _compare(got, want, f32_ulps=0):
    """Bit-exact comparison (f32_ulps = 0), SiLU included: the kernel's exp restates the
    host libm's expf that the oracle calls."""
    q, y, acc = got
    wq, wy, wacc = want
    np.testing.assert_array_equal(acc, wacc)
    if f32_ulps == 0:
        np.testing.assert_array_equal(y.view(np.uint32), wy.view(np.uint32))
        np.testing.assert_array_equal(q, wq)
        return
    ulps = np.abs(y.view(np.int32).astype(np.int64) - wy.view(np.int32).astype(np.int64))
    assert ulps.max() <= f32_ulps
    same = ulps == 0
    np.testing.assert_array_equal(q[same], wq[same])
    assert np.abs(q.astype(np.int32) - wq.astype(np.int32)).max() <= 1


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (256, 512, 1024), (1, 64, 16),
                                   (300, 200, 48), (129, 257, 144), (77, 1000, 512),
                                   (512, 64, 576), (1024, 128, 2304)])
@pytest.mark.parametrize("rounding", [orc.ROUND_HALF_AWAY, orc.ROUND_HALF_EVEN])
def test_gemm_i8_shapes(cuda, m, n, k, rounding):
    rng = np.random.default_rng(1000 + m + n + k)
    a, w, b, scale = _case(rng, m, n, k)
    want = orc.gemm_i8_chain(a, w, b, scale, orc.ACT_NONE, 2.0, rounding)
    got = _run(cuda, a, w, b, scale, orc.ACT_NONE, 2.0, rounding)
    _compare(got, want)


@pytest.mark.parametrize("act", [orc.ACT_RELU, orc.ACT_RELU6, orc.ACT_SILU])
def test_gemm_i8_activations(cuda, act):
    rng = np.random.default_rng(7 + act)
    a, w, b, _ = _case(rng, 256, 384, 256)
    # small scales keep y in the range where ReLU6 clamps and SiLU is non-trivial
    scale = rng.uniform(1e-5, 2e-4, size=384).astype(np.float32)
    for rounding in (orc.ROUND_HALF_AWAY, orc.ROUND_HALF_EVEN):
        want = orc.gemm_i8_chain(a, w, b, scale, act, 0.05, rounding)
        got = _run(cuda, a, w, b, scale, act, 0.05, rounding)
        _compare(got, want)


def test_gemm_i8_rounding_ties(cuda):
    """scale = 0.5 and s_out = 1 make every odd accumulator an exact .5 tie."""
    rng = np.random.default_rng(3)
    a, w, _, _ = _case(rng, 256, 256, 64, bias=False)
    a //= 16
    w //= 16
    scale = np.full(256, 0.5, np.float32)
    for rounding in (orc.ROUND_HALF_AWAY, orc.ROUND_HALF_EVEN):
        want = orc.gemm_i8_chain(a, w, None, scale, orc.ACT_NONE, 1.0, rounding)
        got = _run(cuda, a, w, None, scale, orc.ACT_NONE, 1.0, rounding)
        ties = (want[2] % 2 != 0) & (np.abs(want[2]) < 255)
        assert ties.sum() > 1000
        _compare(got, want)
    # the two modes must actually differ on ties
    ha = orc.gemm_i8_chain(a, w, None, scale, orc.ACT_NONE, 1.0, orc.ROUND_HALF_AWAY)[0]
    he = orc.gemm_i8_chain(a, w, None, scale, orc.ACT_NONE, 1.0, orc.ROUND_HALF_EVEN)[0]
    assert (ha != he).any()


def test_gemm_i8_extreme_values(cuda):
    """Full-range int8 (-128 included) at K=4096: |acc| up to 4096*128^2 = 2^26."""
    m, n, k = 256, 256, 4096
    a = np.full((m, k), -128, np.int8)
    w = np.full((n, k), -128, np.int8)
    w[1::2] = 127
    scale = np.full(n, 1e-3, np.float32)
    want = orc.gemm_i8_chain(a, w, None, scale, orc.ACT_NONE, 1.0, orc.ROUND_HALF_EVEN)
    got = _run(cuda, a, w, None, scale, orc.ACT_NONE, 1.0, orc.ROUND_HALF_EVEN)
    _compare(got, want)
    assert want[2][0, 0] == 4096 * 128 * 128


def test_gemm_i8_full_size_4096(cuda):
    """The 4096^3 per-channel workload, checked element by element against the oracle."""
    rng = np.random.default_rng(4096)
    a, w, b, scale = _case(rng, 4096, 4096, 4096)
    s_out = 40.0
    want = orc.gemm_i8_chain(a, w, b, scale, orc.ACT_NONE, s_out, orc.ROUND_HALF_EVEN)
    got = _run(cuda, a, w, b, scale, orc.ACT_NONE, s_out, orc.ROUND_HALF_EVEN)
    _compare(got, want)


@pytest.mark.parametrize("s_out", [0.1, 0.3, 0.7, 1.1e-38, 3.0e38])
def test_gemm_i8_requant_near_ties(cuda, s_out):
    """s_out values with inexact reciprocals and per-channel scales s_out * {1/2, 3/2, 5/2,
    1/3}: y / s_out lands within a few ulps of a half-integer for most odd accumulators, so
    the reciprocal-multiply requantization must fall back to the division there.  The last
    two s_out values (denormal reciprocal, denormal-adjacent scale) take the division for
    every element."""
    rng = np.random.default_rng(11)
    a, w, b, _ = _case(rng, 256, 256, 64, bias=False)
    a //= 16
    w //= 16
    mult = np.array([0.5, 1.5, 2.5, 1.0 / 3.0], np.float64)
    scale = (np.float64(np.float32(s_out)) * mult[np.arange(256) % 4]).astype(np.float32)
    for rounding in (orc.ROUND_HALF_AWAY, orc.ROUND_HALF_EVEN):
        want = orc.gemm_i8_chain(a, w, None, scale, orc.ACT_RELU, s_out, rounding)
        got = _run(cuda, a, w, None, scale, orc.ACT_RELU, s_out, rounding)
        _compare(got, want)


@pytest.mark.parametrize("n,k", [(64, 576), (128, 1152), (256, 512), (96, 64), (200, 320)])
def test_gemm_i8_weights_resident(cuda, n, k):
    """M large enough that every CTA runs several M tiles of the single N tile: the weight
    tile stays in shared memory and only A streams (K = 64 ... 1152, ragged N)."""
    rng = np.random.default_rng(n + k)
    a, w, b, scale = _case(rng, 40000, n, k)
    for act, rounding in ((orc.ACT_RELU, orc.ROUND_HALF_AWAY), (orc.ACT_NONE, orc.ROUND_HALF_EVEN)):
        want = orc.gemm_i8_chain(a, w, b, scale, act, 3.0, rounding)
        got = _run(cuda, a, w, b, scale, act, 3.0, rounding)
        _compare(got, want)


@pytest.mark.parametrize("m,n,k", [(9000, 600, 1040), (4352, 768, 256), (2100, 1100, 4096), (19000, 256, 96)])
def test_gemm_i8_cta_pairs(cuda, m, n, k):
    """Shapes that run on CTA pairs (cta_group::2, 256 x 256 tiles; fewer tiles than SM
    pairs included) and a single-N-tile shape that stays on single CTAs: ragged M, N and K,
    all three outputs, every activation / rounding combination of the chain."""
    rng = np.random.default_rng(m + n + k)
    a, w, b, scale = _case(rng, m, n, k)
    for act, rounding in ((orc.ACT_NONE, orc.ROUND_HALF_EVEN), (orc.ACT_RELU, orc.ROUND_HALF_AWAY),
                          (orc.ACT_RELU6, orc.ROUND_HALF_EVEN)):
        want = orc.gemm_i8_chain(a, w, b, scale, act, 5.0, rounding)
        got = _run(cuda, a, w, b, scale, act, 5.0, rounding)
        _compare(got, want)
