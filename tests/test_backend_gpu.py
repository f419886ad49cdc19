"""The Backend-trait path (compile_operator / execute over the C ABI) and the quantization
kernels, checked against the reference KATs and the oracle.  Written like the reference's
tests/cpu_backend_test.rs: build an OperatorDef, compile, execute, read the output."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as orc
from tests.golden import reference_kats as K

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def backend(cuda):
    from lightship_b200.backend import CudaBackend, GpuBackendConfig
    be = CudaBackend(GpuBackendConfig(device_id=0, arena_bytes=1 << 30))
    yield be
    be.close()


def test_backend_identity(backend):
    caps = backend.capabilities()
    assert backend.is_available()
    assert caps["cc_major"] == 10 and caps["sm_count"] >= 100
    assert backend.backend_type() == "GPU"


def test_qgemm_kat_host_tensors(backend):
    """quantized_ops.rs:121-133 through the backend (K=3 exercises the K-padding path)."""
    from lightship_b200.backend import DataType, OperatorDef, OperatorType, Tensor
    m, n, k = K.QGEMM_MNK
    a = Tensor.from_data("a", [m, k], DataType.QInt8, K.QGEMM_A)
    b = Tensor.from_data("b", [k, n], DataType.QInt8, K.QGEMM_B)
    c = Tensor("c", [1], DataType.I32, np.zeros(m * n, np.int32))
    op = backend.compile_operator(OperatorDef("qgemm", OperatorType.QGemm), None, [a, b], [c])
    backend.execute(op, [a], [c])
    assert c.shape == [m, n]
    assert c.numpy().tolist() == K.QGEMM_C


def test_qgemm_dequant_and_requant_kats(backend):
    """dequantize (quantized_ops.rs:135-146) and quantize_sym (:148-159) as the epilogue."""
    from lightship_b200.backend import (DataType, OperatorDef, OperatorType, Quantization,
                                        Rounding, Tensor)
    # acc = [1, 2, 4] via A = [[1],[2],[4]] (padded to K=16) times W = [[1]]
    a = Tensor.from_data("a", [3, 1], DataType.QInt8, [1, 2, 4], quantization=Quantization([0.5]))
    w = Tensor.from_data("w", [1, 1], DataType.QInt8, [1], quantization=Quantization([1.0]))
    y = Tensor("y", [1], DataType.F32, np.zeros(3, np.float32))
    q = Tensor("q", [1], DataType.QInt8, np.zeros(3, np.int8))
    op = backend.compile_operator(OperatorDef("qgemm", OperatorType.QGemm, output_scale=K.QSYM_SCALE,
                                              rounding=Rounding.HalfAwayFromZero), None, [a, w], [y, q])
    backend.execute(op, [a], [y, q])
    assert y.numpy().ravel().tolist() == K.DEQUANT_OUT
    assert q.numpy().ravel().tolist() == K.QSYM_OUT


@pytest.mark.parametrize("device_resident", [False, True])
def test_fc_int8_per_channel(backend, cuda, device_resident):
    import torch
    from lightship_b200.backend import (DataType, OperatorDef, OperatorType, Quantization,
                                        Rounding, Tensor)
    rng = np.random.default_rng(21)
    m, n, k = 333, 1000, 512  # ResNet FC-like, odd batch
    x = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    sw = rng.uniform(0.001, 0.02, n).astype(np.float32)
    bias = rng.integers(-3000, 3000, n, dtype=np.int32)
    s_a, s_out = 0.05, 0.8
    scale = (np.float32(s_a) * sw).astype(np.float32)
    want = orc.gemm_i8_chain(x, w, bias, scale, orc.ACT_NONE, s_out, orc.ROUND_HALF_EVEN)
    xd = torch.from_numpy(x).to(cuda) if device_resident else x
    outs = [torch.zeros(m * n, dtype=dt, device=cuda) if device_resident else np.zeros(m * n, npdt)
            for dt, npdt in ((torch.int8, np.int8), (torch.float32, np.float32), (torch.int32, np.int32))]
    xt = Tensor("x", [m, k], DataType.QInt8, xd, quantization=Quantization([s_a]))
    wt = Tensor("w", [n, k], DataType.QInt8, w, quantization=Quantization(list(map(float, sw))))
    bt = Tensor("b", [n], DataType.QInt32, bias)
    q = Tensor("q", [1], DataType.QInt8, outs[0])
    y = Tensor("y", [1], DataType.F32, outs[1])
    acc = Tensor("acc", [1], DataType.I32, outs[2])
    op = backend.compile_operator(OperatorDef("fc", OperatorType.FullyConnected, output_scale=s_out,
                                              rounding=Rounding.HalfEven), None, [xt, wt, bt], [q, y, acc])
    backend.execute(op, [xt], [q, y, acc])
    if device_resident:
        torch.cuda.synchronize()
    assert q.shape == [m, n]
    np.testing.assert_array_equal(acc.numpy().reshape(m, n), want[2])
    np.testing.assert_array_equal(y.numpy().reshape(m, n).view(np.uint32), want[1].view(np.uint32))
    np.testing.assert_array_equal(q.numpy().reshape(m, n), want[0])


def test_fc_int8_from_f32_weights_quantizes_per_channel(backend):
    """f32 weights are quantized per output channel at compile (find_scale_zp symmetric +
    quantize_value, helpers.rs:101-155) -- the same integers the oracle produces."""
    from lightship_b200.backend import DataType, OperatorDef, OperatorType, Tensor
    rng = np.random.default_rng(4)
    m, n, k = 64, 48, 96
    x = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    wf = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    wq, sw = orc.quantize_weights_per_channel(wf)
    want = orc.gemm_i8_chain(x, wq, None, sw, orc.ACT_NONE, 1.0)
    xt = Tensor("x", [m, k], DataType.QInt8, x)
    wt = Tensor("w", [n, k], DataType.F32, wf)
    y = Tensor("y", [1], DataType.F32, np.zeros(m * n, np.float32))
    op = backend.compile_operator(OperatorDef("fc", OperatorType.FullyConnected), None, [xt, wt], [y])
    backend.execute(op, [xt], [y])
    np.testing.assert_array_equal(y.numpy().reshape(m, n).view(np.uint32), want[1].view(np.uint32))


@pytest.mark.parametrize("qdtype,zp", [(9, 0), (8, 128), (10, 3), (3, 5), (5, -7)])
@pytest.mark.parametrize("rounding", [0, 1])
def test_quantize_dequantize_ops(backend, qdtype, zp, rounding):
    """Quantize / Dequantize operators against quantize_value / dequantize_value
    (helpers.rs:139-160).  Plain I8 (3) and I32 (5) take the reference's `_` arm: the clamp
    range is (0, 255) whatever the storage, and an I8 code above 127 wraps as `as i8`."""
    from lightship_b200.backend import (DataType, OperatorDef, OperatorType, Quantization,
                                        Rounding, Tensor)
    rng = np.random.default_rng(qdtype * 10 + rounding)
    x = rng.normal(0, 3, size=(2, 3, 17, 19)).astype(np.float32)
    x.ravel()[:6] = [0.25, -0.25, 0.75, 1e30, -1e30, np.nan]  # ties at scale 0.5, saturation, NaN
    scale = 0.5
    npdt = {9: np.int8, 8: np.uint8, 10: np.int32, 3: np.int8, 5: np.int32}[qdtype]
    xt = Tensor("x", list(x.shape), DataType.F32, x)
    qt = Tensor("q", [1], DataType(qdtype), np.zeros(x.size, npdt), quantization=Quantization([scale], [zp]))
    op = backend.compile_operator(OperatorDef("q", OperatorType.Quantize, rounding=Rounding(rounding)),
                                  None, [xt], [qt])
    backend.execute(op, [xt], [qt])
    oq = {9: orc.QINT8, 8: orc.QUINT8, 10: orc.QINT32}.get(qdtype, orc.OTHER)
    if rounding == 0 and oq != orc.OTHER:
        want = orc.quantize_tensor(x, scale, zp, oq)
    elif rounding == 0:
        want = np.array([orc.quantize_value(float(v), scale, zp, oq) for v in x.ravel()],
                        np.int64).astype(npdt).reshape(x.shape)
    else:  # half-even variant of quantize_value
        t = (x / np.float32(scale)).astype(np.float32)
        r = np.rint(t)
        lo, hi = {9: (-128, 127), 10: (-2**31, 2**31 - 1)}.get(qdtype, (0, 255))
        ri = np.where(np.isnan(r), 0, np.clip(r, -2**31, 2**31 - 1)).astype(np.int64)
        ri = np.where(r >= 2**31, 2**31 - 1, ri)
        s = (ri + zp + 2**31) % 2**32 - 2**31  # wrapping i32 add
        want = np.clip(s, lo, hi).astype(npdt)
    assert qt.shape == list(x.shape)
    np.testing.assert_array_equal(qt.numpy().reshape(x.shape), want)
    # dequantize back
    qin = Tensor("qin", list(x.shape), DataType(qdtype), np.ascontiguousarray(want),
                 quantization=Quantization([scale], [zp]))
    yt = Tensor("y", [1], DataType.F32, np.zeros(x.size, np.float32))
    dop = backend.compile_operator(OperatorDef("dq", OperatorType.Dequantize), None, [qin], [yt])
    backend.execute(dop, [qin], [yt])
    if oq != orc.OTHER:
        want_y = orc.dequantize_tensor(want, scale, zp, oq)
    else:  # dequantize_value on the stored integers: (q as f32 - zp as f32) * scale
        want_y = (want.astype(np.float32) - np.float32(zp)) * np.float32(scale)
    np.testing.assert_array_equal(yt.numpy().reshape(x.shape), want_y)


def test_quantize_per_channel_nchw(backend):
    from lightship_b200.backend import (DataType, OperatorDef, OperatorType, Quantization,
                                        StorageLayout, Tensor)
    rng = np.random.default_rng(12)
    x = rng.normal(0, 1, size=(3, 8, 5, 7)).astype(np.float32)
    scales = rng.uniform(0.01, 0.05, 8).astype(np.float32)
    xt = Tensor("x", list(x.shape), DataType.F32, x, layout=StorageLayout.NCHW)
    qt = Tensor("q", list(x.shape), DataType.QInt8, np.zeros(x.size, np.int8),
                layout=StorageLayout.NCHW, quantization=Quantization(list(map(float, scales))))
    op = backend.compile_operator(OperatorDef("q", OperatorType.Quantize), None, [xt], [qt])
    backend.execute(op, [xt], [qt])
    want = np.stack([orc.quantize_tensor(x[:, c], float(scales[c]), 0, orc.QINT8) for c in range(8)], 1)
    np.testing.assert_array_equal(qt.numpy().reshape(x.shape), want)


@pytest.mark.parametrize("symmetric,qdtype", [(1, 9), (0, 8), (1, 8), (0, 10), (1, 3), (0, 3), (1, 5), (0, 5)])
def test_find_scale_zp_device(cuda, symmetric, qdtype):
    import torch
    from lightship_b200 import _lib
    lib = _lib.lib()
    rng = np.random.default_rng(symmetric * 7 + qdtype)
    for x in (rng.normal(0.3, 2.0, size=1_000_003).astype(np.float32),
              np.array(K.FSZ_DATA, np.float32),
              np.array([np.nan, 1.5, -0.25, np.nan], np.float32),
              np.zeros(0, np.float32)):
        tx = torch.from_numpy(x).to(cuda) if x.size else torch.zeros(1, device=cuda)
        ws = torch.zeros(4, dtype=torch.int32, device=cuda)
        s = torch.zeros(1, dtype=torch.float32, device=cuda)
        z = torch.zeros(1, dtype=torch.int32, device=cuda)
        _lib.check(lib.lsc_find_scale_zp_f32(tx.data_ptr(), x.size, qdtype, symmetric, ws.data_ptr(), 16,
                                             s.data_ptr(), z.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream))
        oq = {9: orc.QINT8, 8: orc.QUINT8, 10: orc.QINT32}.get(qdtype, orc.OTHER)
        ws_, wz = orc.find_scale_zp(x, oq, bool(symmetric))
        assert s.item() == np.float32(ws_) and z.item() == wz, (x[:4], s.item(), ws_, z.item(), wz)


def test_allocate_deallocate_and_stats(backend):
    blk = backend.allocate(1 << 20, 4096)
    assert blk.ptr % 4096 == 0 and blk.size == 1 << 20
    st = backend.memory_stats()
    assert st["current"] >= 1 << 20 and st["peak"] >= st["current"]
    backend.deallocate(blk)
    assert backend.memory_stats()["current"] <= st["current"] - (1 << 20)
    from lightship_b200.backend import LightShipError
    with pytest.raises(LightShipError) as e:
        backend.allocate(1024, 3)  # not a power of two (cpu.rs:216-221)
    assert e.value.code == 2
    with pytest.raises(LightShipError) as e:
        backend.allocate(1 << 40, 256)
    assert e.value.code == 3  # OutOfMemory


def test_unsupported_operator_is_an_error(backend):
    """CpuBackend returns Ok(()) for unimplemented operators (cpu.rs:205-211); this backend
    reports UnsupportedOperator instead."""
    from lightship_b200.backend import DataType, LightShipError, OperatorDef, OperatorType, Tensor
    x = Tensor("x", [2, 3], DataType.F16)
    with pytest.raises(LightShipError) as e:
        backend.compile_operator(OperatorDef("fc16", OperatorType.FullyConnected), None,
                                 [x, Tensor("w", [4, 3], DataType.F16)], [Tensor("y", [1], DataType.F16)])
    assert e.value.code in (8, 11)


def test_shape_mismatch_is_reported(backend):
    from lightship_b200.backend import DataType, LightShipError, OperatorDef, OperatorType, Tensor
    a = Tensor.from_data("a", [2, 3], DataType.QInt8, [1] * 6)
    b = Tensor.from_data("b", [4, 2], DataType.QInt8, [1] * 8)
    with pytest.raises(LightShipError) as e:
        backend.compile_operator(OperatorDef("qgemm", OperatorType.QGemm), None, [a, b],
                                 [Tensor("c", [1], DataType.I32)])
    assert e.value.code == 7


def test_backend_destroyed_before_its_operators(cuda):
    """Compiled operators keep the backend alive; destroy order does not matter."""
    from lightship_b200.backend import (CudaBackend, DataType, GpuBackendConfig, OperatorDef,
                                        OperatorType, Tensor)
    be = CudaBackend(GpuBackendConfig(device_id=0, arena_bytes=64 << 20))
    a = Tensor.from_data("a", [2, 3], DataType.QInt8, K.QGEMM_A)
    b = Tensor.from_data("b", [3, 2], DataType.QInt8, K.QGEMM_B)
    c = Tensor("c", [1], DataType.I32, np.zeros(4, np.int32))
    op = be.compile_operator(OperatorDef("qgemm", OperatorType.QGemm), None, [a, b], [c])
    be.close()
    del be
    import gc
    gc.collect()
    del op
    gc.collect()


@pytest.mark.parametrize("rows,cols,symmetric,qdtype", [(64, 576, 1, 9), (1000, 512, 1, 9),
                                                        (3, 200_003, 0, 8), (7, 1, 0, 10),
                                                        (5, 0, 1, 9), (9, 333, 0, 3), (4, 100, 1, 5)])
def test_find_scale_zp_per_channel(cuda, rows, cols, symmetric, qdtype):
    """find_scale_zp per output channel (weights [Cout, K]), including rows split over
    several blocks, NaN entries, an all-zero row and empty rows."""
    import torch
    from lightship_b200 import _lib
    lib = _lib.lib()
    rng = np.random.default_rng(rows + cols)
    x = rng.normal(0.1, 0.05, size=(rows, cols)).astype(np.float32)
    if cols > 2:
        x[0, 1] = np.nan
        x[rows - 1] = 0.0
    tx = torch.from_numpy(x).to(cuda) if x.size else torch.zeros(1, device=cuda)
    ws_bytes = lib.lsc_find_scale_zp_per_channel_workspace_size(rows)
    ws = torch.zeros(max(1, ws_bytes // 4), dtype=torch.int32, device=cuda)
    s = torch.zeros(rows, dtype=torch.float32, device=cuda)
    z = torch.zeros(rows, dtype=torch.int32, device=cuda)
    _lib.check(lib.lsc_find_scale_zp_per_channel_f32(tx.data_ptr(), rows, cols, qdtype, symmetric,
                                                     ws.data_ptr(), ws_bytes, s.data_ptr(), z.data_ptr(),
                                                     torch.cuda.current_stream().cuda_stream))
    oq = {9: orc.QINT8, 8: orc.QUINT8, 10: orc.QINT32}.get(qdtype, orc.OTHER)
    want = [orc.find_scale_zp(x[r], oq, bool(symmetric)) for r in range(rows)]
    assert s.cpu().numpy().tolist() == [np.float32(w[0]) for w in want]
    assert z.cpu().numpy().tolist() == [w[1] for w in want]
