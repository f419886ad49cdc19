"""The allocation-free per-channel find_scale_zp entry point, for callers that cannot call
cudaMalloc (code embedded in a host runtime that owns the GPU's memory, where an allocation
would synchronise the device and fail once that memory is reserved).

It is checked through the C ABI against the workspace-taking entry point and against the
oracle's find_scale_zp applied to every channel, on consecutive calls: the shared static
scratch must not carry state from one call into the next.  This file is collected last so a
failure here cannot hide the other tests' results."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _reference_call(lib, _lib, tx, rows, cols, qdtype, symmetric, cuda, stream):
    import torch
    ws_bytes = lib.lsc_find_scale_zp_per_channel_workspace_size(rows)
    ws = torch.zeros(max(1, ws_bytes // 4), dtype=torch.int32, device=cuda)
    s = torch.full((rows,), -1.0, dtype=torch.float32, device=cuda)
    z = torch.full((rows,), -7, dtype=torch.int32, device=cuda)
    _lib.check(lib.lsc_find_scale_zp_per_channel_f32(tx.data_ptr(), rows, cols, qdtype, symmetric,
                                                     ws.data_ptr(), ws_bytes, s.data_ptr(),
                                                     z.data_ptr(), stream))
    return s, z


def _noalloc_call(lib, _lib, tx, rows, cols, qdtype, symmetric, cuda, stream):
    import torch
    s = torch.full((rows,), -1.0, dtype=torch.float32, device=cuda)
    z = torch.full((rows,), -7, dtype=torch.int32, device=cuda)
    _lib.check(lib.lsc_find_scale_zp_per_channel_f32_noalloc(tx.data_ptr(), rows, cols, qdtype,
                                                             symmetric, s.data_ptr(), z.data_ptr(),
                                                             stream))
    return s, z


def _oracle_per_channel(x, qdtype, symmetric):
    """find_scale_zp (quantization/helpers.rs:101-136) of the oracle on each row of x."""
    from oracle import oracle as orc
    od = {9: orc.QINT8, 8: orc.QUINT8, 10: orc.QINT32}.get(qdtype, orc.OTHER)
    s = np.empty(x.shape[0], np.float32)
    z = np.empty(x.shape[0], np.int32)
    for r in range(x.shape[0]):
        s[r], z[r] = orc.find_scale_zp(np.ascontiguousarray(x[r]), od, bool(symmetric))
    return s, z


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(cuda):
    import torch
    from lightship_b200 import _lib
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(2024)
    # call 1: wide-range data with long channels (several blocks per channel)
    x1 = rng.normal(0.0, 8.0, size=(512, 70_000)).astype(np.float32)
    # call 2: small, positive-only data on more channels -- stale minima/maxima from call 1
    # would change every scale and zero point here
    x2 = rng.uniform(0.01, 0.02, size=(1000, 300)).astype(np.float32)
    for x, qdtype, symmetric in ((x1, 9, 1), (x2, 8, 0)):
        rows, cols = x.shape
        tx = torch.from_numpy(x).to(cuda)
        want_s, want_z = _reference_call(lib, _lib, tx, rows, cols, qdtype, symmetric, cuda, stream)
        got_s, got_z = _noalloc_call(lib, _lib, tx, rows, cols, qdtype, symmetric, cuda, stream)
        torch.cuda.synchronize()
        assert torch.equal(got_s, want_s)
        assert torch.equal(got_z, want_z)
        orc_s, orc_z = _oracle_per_channel(x, qdtype, symmetric)
        assert np.array_equal(got_s.cpu().numpy().view(np.uint32), orc_s.view(np.uint32))
        assert np.array_equal(got_z.cpu().numpy(), orc_z)
    # and once more on the first input after the second
    tx1 = torch.from_numpy(x1).to(cuda)
    want_s, want_z = _reference_call(lib, _lib, tx1, 512, 70_000, 9, 1, cuda, stream)
    got_s, got_z = _noalloc_call(lib, _lib, tx1, 512, 70_000, 9, 1, cuda, stream)
    assert torch.equal(got_s, want_s) and torch.equal(got_z, want_z)


def test_noalloc_rejects_more_channels_than_its_scratch(cuda):
    import torch
    from lightship_b200 import _lib
    lib = _lib.lib()
    x = torch.zeros(16385, dtype=torch.float32, device=cuda)
    s = torch.zeros(16385, dtype=torch.float32, device=cuda)
    z = torch.zeros(16385, dtype=torch.int32, device=cuda)
    st = lib.lsc_find_scale_zp_per_channel_f32_noalloc(x.data_ptr(), 16385, 1, 9, 1, s.data_ptr(),
                                                       z.data_ptr(), None)
    assert st == _lib.ERROR_INVALID_ARGUMENT
    assert "16384" in _lib.last_error()
