"""Failure detection on the device, in the form that faults nothing: a wait that runs out.

Every mbarrier wait of the INT8 contraction kernels is bounded.  The test hook
``lsc_debug_withhold_copy`` makes one launch leave an operand copy unissued -- a barrier that
nothing completes -- with a 10 ms wait limit.  The kernel must give up, drain what it issued,
free its tensor memory and return; the host then reads LSC_ERROR_TIMEOUT (the reference's
LightShipError::Timeout, lightship-core/src/common/error.rs:32-34) from lsc_check_device, and
the next launch on the same device is bit-exact against the oracle."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _gemm(lib, _lib, torch, cuda, a, w, bias, scale):
    m, k = a.shape
    n = w.shape[0]
    ta, tw = torch.from_numpy(a).to(cuda), torch.from_numpy(w).to(cuda)
    tb, ts = torch.from_numpy(bias).to(cuda), torch.from_numpy(scale).to(cuda)
    q = torch.full((m, n), 77, dtype=torch.int8, device=cuda)
    st = lib.lsc_gemm_i8(ta.data_ptr(), tw.data_ptr(), m, n, k, tb.data_ptr(), ts.data_ptr(), 0.5, 1, 0,
                         q.data_ptr(), None, None, torch.cuda.current_stream().cuda_stream)
    _lib.check(st)
    return q, (ta, tw, tb, ts)


def test_withheld_copy_times_out_and_device_recovers(cuda):
    import ctypes as C

    import torch
    from lightship_b200 import _lib
    lib = _lib.lib()
    rng = np.random.default_rng(5)
    m, n, k = 512, 128, 512  # single CTAs (N <= 256), 8 tiles, 4 k-blocks each
    a = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    bias = rng.integers(-5000, 5000, size=n, dtype=np.int32)
    scale = rng.uniform(1e-4, 1e-3, size=n).astype(np.float32)
    want = orc.gemm_i8_chain(a, w, bias, scale, orc.ACT_RELU, 0.5, orc.ROUND_HALF_AWAY)[0]

    word = C.c_uint32(0)
    _lib.check(lib.lsc_check_device(C.byref(word)))  # start from a clean error word
    _lib.check(lib.lsc_debug_withhold_copy(1, 10_000_000))
    q, keep = _gemm(lib, _lib, torch, cuda, a, w, bias, scale)
    st = lib.lsc_check_device(C.byref(word))
    assert st == _lib.ERROR_TIMEOUT, (st, _lib.last_error())
    assert word.value & 1
    assert "bounded device wait" in _lib.last_error()
    # the first tile of CTA 0 never received its operands: its outputs were not written
    assert not np.array_equal(q.cpu().numpy(), want)

    # the error word was cleared by the read; the device and the library still work
    q2, keep2 = _gemm(lib, _lib, torch, cuda, a, w, bias, scale)
    _lib.check(lib.lsc_check_device(C.byref(word)))
    assert word.value == 0
    np.testing.assert_array_equal(q2.cpu().numpy(), want)
