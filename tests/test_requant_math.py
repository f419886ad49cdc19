"""The INT8 epilogue requantizes with a reciprocal multiply, t = RN(y * RN(1/s)), clamps t
below, rounds it to an integer with the 1.5 * 2^23 magic-number addition, saturates, and
falls back to the IEEE division RN(y / s) only when t is within |t| * 2^-22 of a
half-integer.
This restates that rule in numpy float32 (IEEE round-to-nearest, like the kernel's
__fmul_rn / __fdiv_rn) and checks it against the reference's division-based requantization
(lightship-core/src/cpu/quantized_ops.rs:43-48), with and without a ReLU folded into the
clamp, on random values, on values placed within a few ulps of every half-integer tie, and
on saturating and special values."""
import numpy as np
import pytest

F = np.float32


def _requant_div(y, s, even):
    t = (y / s).astype(F)
    r = _round_exact(t, even)
    r = np.where(np.isnan(r), F(0), r)
    return np.clip(r, -128, 127).astype(np.int32)


def _round_exact(t, even):
    """rintf / roundf on float32 arrays: half-even or half-away-from-zero."""
    if even:
        return np.rint(t).astype(F)
    fl = np.floor(np.abs(t))
    frac = np.abs(t) - fl
    mag = np.where(frac >= F(0.5), fl + F(1), fl)
    return np.copysign(mag, t).astype(F)


def _requant_fast(y, s, even, relu_folded=False):
    """The kernel's rule: t = y * RN(1/s), clamped below at -256 (at 0 with a folded ReLU)
    keeping NaN; t + 1.5*2^23 stays positive and its bit pattern minus that of 1.5*2^23 is
    rint(t) (ordered like t beyond 2^22), saturated to int8; the division is redone unless
    RN(|tc - rint(tc)| + |tc| * 2^-22) < 0.5."""
    magic = F(12582912.0)
    inv = F(1) / F(s)
    lo = F(0) if relu_folded else F(-256)
    with np.errstate(over="ignore", invalid="ignore"):
        t = (y * inv).astype(F)
        tc = np.maximum(t, lo)  # numpy's maximum propagates NaN
        tm = (tc + magic).astype(F)
        d = (tc - (tm - magic).astype(F)).astype(F)
        # the kernel's fused multiply-add, rounded once: exact in float64 wherever the sum is
        # near 0.5, then rounded to float32
        near = (np.abs(tc).astype(np.float64) * 2.0 ** -22 + np.abs(d).astype(np.float64)).astype(F)
    bits = tm.view(np.int32)
    assert (bits[~np.isnan(tm)] > 0).all()  # tm stays positive: no int32 wrap below
    out = np.clip(bits - np.int32(0x4B400000), -128, 127).astype(np.int32)
    slow = ~(near < F(0.5))
    ys = y[slow]
    if relu_folded:
        ys = np.where(ys > 0, ys, F(0)).astype(F)
    out[slow] = _requant_div(ys, F(s), even)
    return out


SCALES = [0.1, 0.3, 0.7, 0.017, 1.0 / 3.0, 2.5e-3, 7.3e-5, 0.0421, 13.7, 1.0]


@pytest.mark.parametrize("even", [True, False])
@pytest.mark.parametrize("s", SCALES)
def test_fast_requant_matches_division(s, even):
    s = F(s)
    rng = np.random.default_rng(int(s * 1e6) + even)
    ys = [rng.uniform(-140, 140, 200_000).astype(F) * s]
    # values within +-8 ulps of every half-integer tie of y / s, and of integer multiples
    k = np.arange(-131, 131, dtype=np.float64)
    for base in (k + 0.5, k):
        centre = (base * np.float64(s)).astype(F)
        up, down = centre, centre
        ys.append(centre)
        for _ in range(8):
            up = np.nextafter(up, F(np.inf)).astype(F)
            down = np.nextafter(down, F(-np.inf)).astype(F)
            ys += [up, down]
    ys.append(np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 3e38, -3e38], F))
    ys.append((np.array([-2e7, -1.3e7, -1e6, -300, -129, -128.5, 127.5, 128, 300, 1e6, 2e7], F) * s).astype(F))
    y = np.concatenate(ys).astype(F)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        want = _requant_div(y, s, even)
        got = _requant_fast(y, s, even)
        relu = np.where(y > 0, y, F(0)).astype(F)  # the reference's ReLU: NaN -> 0
        want_relu = _requant_div(relu, s, even)
        got_relu = _requant_fast(y, s, even, relu_folded=True)
    bad = np.nonzero(want != got)[0]
    assert bad.size == 0, (s, y[bad[:5]], want[bad[:5]], got[bad[:5]])
    bad = np.nonzero(want_relu != got_relu)[0]
    assert bad.size == 0, (s, y[bad[:5]], want_relu[bad[:5]], got_relu[bad[:5]])


def test_fast_requant_fallback_is_rare():
    """On random data the division runs for a few elements in 10^5."""
    rng = np.random.default_rng(5)
    s = F(0.0421)
    y = (rng.uniform(-120, 120, 1_000_000) * s).astype(F)
    t = (y * (F(1) / s)).astype(F)
    near = ~((np.abs(t - np.rint(t)) + np.abs(t) * F(2.0 ** -22)) < F(0.5))
    assert 0 < near.mean() < 1e-4
