"""The INT8 session through the C ABI: an ONNX ResNet-18 loaded with lsc_model_load_onnx,
compiled by lsc_session_create_ex into the INT8 chain (calibrated on the device, activations
planned by live range, the network captured as a CUDA graph with the downsample convolutions
on a second stream) and run by lsc_session_run / lsc_session_run_async with host or device
buffers.  Checked bit for bit against the oracle's quantized ResNet-18 run with the session's
own calibrated scales, and against the Backend-operator composition of the same network."""
import ctypes as C

import numpy as np
import pytest

from tests.golden.resnet_oracle import oracle_resnet18

pytestmark = pytest.mark.gpu

SEED = 11


@pytest.fixture(scope="module")
def be(cuda):
    from lightship_b200.backend import CudaBackend, GpuBackendConfig
    b = CudaBackend(GpuBackendConfig(device_id=0, arena_bytes=3 << 30))
    yield b
    b.close()


class _Net:
    """What oracle_resnet18 reads: the parameters and the calibrated scales by layer name."""

    def __init__(self, sess, num_classes=1000):
        from lightship_b200.resnet18 import build_params
        self.convs, self.blocks, self.fc_w, self.fc_b = build_params(SEED, num_classes)
        self.num_classes = num_classes
        self.scales = {"input": sess.value("X:q")["scale"], "pooled": sess.value("pooled")["scale"]}
        for spec in self.convs:
            self.scales[spec.name] = sess.value(spec.name)["scale"]
        self.scales["pool"] = sess.value("pool")["scale"]


def _session(be, batch, x, plan_memory=True, concurrent=True, rounding=0):
    from lightship_b200.backend import DataType, OnnxModel, Rounding, Session, StorageLayout, Tensor
    from lightship_b200.onnx_writer import resnet18_onnx
    model = OnnxModel(resnet18_onnx(batch, SEED))
    cal = Tensor("X", list(x.shape), DataType.F32, x, layout=StorageLayout.NCHW)
    return Session(be, model, precision="int8", calibration=cal, rounding=Rounding(rounding),
                   concurrent=concurrent, plan_memory=plan_memory)


def _run(sess, x):
    from lightship_b200.backend import DataType, StorageLayout, Tensor
    logits = np.zeros((x.shape[0], 1000), np.float32)
    out = Tensor("logits", [1], DataType.F32, logits)
    sess.run([Tensor("X", list(x.shape), DataType.F32, x, layout=StorageLayout.NCHW)], [out])
    assert out.shape == [x.shape[0], 1000]
    return logits


def _device_bytes(ptr, nbytes, dtype):
    import torch
    buf = (C.c_byte * nbytes)()
    assert torch.cuda.is_available()
    from lightship_b200 import _lib
    _lib.check(_lib.lib().lsc_memcpy_d2h(C.addressof(buf), C.c_void_p(ptr), nbytes, None))
    torch.cuda.synchronize()
    return np.frombuffer(bytes(buf), dtype=dtype)


@pytest.mark.parametrize("rounding", [0, 1])
def test_int8_session_matches_oracle_with_intermediates(be, cuda, rounding):
    """Batch 4, one buffer per activation (so every layer's output survives the run): the
    logits and each layer's int8 output equal the oracle's on the session's scales."""
    batch = 4
    x = np.random.default_rng(5).normal(size=(batch, 3, 224, 224)).astype(np.float32)
    sess = _session(be, batch, x, plan_memory=False, rounding=rounding)
    logits = _run(sess, x)
    net = _Net(sess)
    want, acts = oracle_resnet18(x, net, rounding)
    # the stem's convolution and max pool run as one launch: the conv output is not written
    for name in ["pool"] + [s.name for s in net.convs[1:]]:
        v = sess.value(name)
        got = _device_bytes(v["ptr"], v["nbytes"], np.int8).reshape(v["shape"])
        np.testing.assert_array_equal(got, acts[name], err_msg=name)
    np.testing.assert_array_equal(logits.view(np.uint32), want.view(np.uint32))
    assert not np.array_equal(logits[0], logits[1])


@pytest.mark.parametrize("batch", [32, 128, 256])
def test_int8_session_at_benchmark_batches(be, cuda, batch):
    """The benchmark's per-GPU batches with the memory plan and the captured graph: the first
    and last four images against the oracle; the session against the Backend-operator
    composition (resnet18.ResNet18Int8, same parameters and calibration batch, the stem's
    convolution and max pool as separate launches) on all images; the planned activation
    block smaller than one buffer per activation.  From batch 128 the session runs the stem's
    convolution and max pool as one launch (enough 4-row bands per CTA)."""
    import torch
    from lightship_b200.resnet18 import ResNet18Int8
    x = np.random.default_rng(batch).normal(size=(batch, 3, 224, 224)).astype(np.float32)
    sess = _session(be, batch, x)
    logits = _run(sess, x)
    plan = sess.memory_plan()
    assert plan["planned_bytes"] < 0.6 * plan["unplanned_bytes"], plan
    pick = np.r_[0:4, batch - 4:batch]
    net = _Net(sess)
    want, _ = oracle_resnet18(np.ascontiguousarray(x[pick]), net, 0)
    np.testing.assert_array_equal(logits[pick].view(np.uint32), want.view(np.uint32))
    ref = ResNet18Int8(be, batch, cuda, image=224, seed=SEED)
    xd = torch.from_numpy(x).to(cuda)
    ref.calibrate(xd)
    assert ref.scales["input"] == net.scales["input"] and ref.scales["layer4.1.conv2"] == net.scales["layer4.1.conv2"]
    ref_logits = ref.forward(xd).cpu().numpy()
    np.testing.assert_array_equal(logits.view(np.uint32), ref_logits.view(np.uint32))


def test_int8_session_async_pipeline_and_device_io(be, cuda):
    """run_async over several inputs (two input slots, uploads on the session's copy stream)
    gives each input's logits; the device-resident path (input written into the session's own
    input buffer, output read from its output buffer) copies nothing and agrees."""
    import torch
    from lightship_b200.backend import DataType, StorageLayout, Tensor
    batch = 8
    rng = np.random.default_rng(3)
    xs = [rng.normal(size=(batch, 3, 224, 224)).astype(np.float32) for _ in range(4)]
    sess = _session(be, batch, xs[0])
    want = [_run(sess, x) for x in xs]
    stream = torch.cuda.Stream(cuda)
    pinned_in = [torch.from_numpy(x).pin_memory() for x in xs]
    pinned_out = [torch.zeros((batch, 1000), dtype=torch.float32).pin_memory() for _ in xs]
    for _ in range(2):
        for xin, yout in zip(pinned_in, pinned_out):
            sess.run_async([Tensor("X", list(xin.shape), DataType.F32, xin, layout=StorageLayout.NCHW)],
                           [Tensor("logits", [1], DataType.F32, yout)], stream=stream.cuda_stream)
        stream.synchronize()
        for yout, w in zip(pinned_out, want):
            np.testing.assert_array_equal(yout.numpy().view(np.uint32), w.view(np.uint32))
    # device-resident input and output buffers of the session itself
    in_ptr, in_bytes = sess.io_buffer(False)
    out_ptr, out_bytes = sess.io_buffer(True)
    assert in_bytes == xs[2].nbytes and out_bytes == batch * 1000 * 4
    from lightship_b200 import _lib
    _lib.check(_lib.lib().lsc_memcpy_h2d(C.c_void_p(in_ptr), C.c_void_p(xs[2].ctypes.data), in_bytes, None))
    dev_in = _lib.lsc_tensor()
    dev_in.ndim = 4
    for i, d in enumerate(xs[2].shape):
        dev_in.shape[i] = d
    dev_in.dtype, dev_in.location, dev_in.data, dev_in.nbytes = 0, _lib.MEM_DEVICE, in_ptr, in_bytes
    dev_out = _lib.lsc_tensor()
    dev_out.dtype, dev_out.location, dev_out.data, dev_out.nbytes = 0, _lib.MEM_DEVICE, out_ptr, out_bytes
    _lib.check(_lib.lib().lsc_session_run(sess._h, C.byref(dev_in), 1, C.byref(dev_out), 1, None))
    got = _device_bytes(out_ptr, out_bytes, np.float32).reshape(batch, 1000)
    np.testing.assert_array_equal(got.view(np.uint32), want[2].view(np.uint32))


def test_int8_session_rejects_unsupported_graphs(be, cuda):
    """A graph the INT8 lowering cannot express fails at create with a clear status."""
    from lightship_b200 import _lib
    from lightship_b200.backend import DataType, LightShipError, OnnxModel, Session, StorageLayout, Tensor
    from tests.golden import onnx_writer as W
    blob, _ = W.small_resnet_model(batch=2)  # a grouped convolution and a MatMul after the Gemm
    x = np.zeros((2, 3, 16, 16), np.float32)
    with pytest.raises(LightShipError) as e:
        Session(be, OnnxModel(blob), precision="int8",
                calibration=Tensor("X", [2, 3, 16, 16], DataType.F32, x, layout=StorageLayout.NCHW))
    assert e.value.code == _lib.ERROR_UNSUPPORTED_OPERATOR


def _fill_device(ptr, nbytes, byte):
    from lightship_b200 import _lib
    buf = (C.c_byte * nbytes)(*([byte] * nbytes))
    _lib.check(_lib.lib().lsc_memcpy_h2d(C.c_void_p(ptr), C.addressof(buf), nbytes, None))


@pytest.mark.parametrize("batch,rounding", [(1, 0), (3, 1), (5, 0), (37, 1)])
def test_int8_session_fused_stem_matches_separate_launches(be, cuda, batch, rounding, monkeypatch):
    """The stem (input quantize, 7x7 / 2 convolution, 3x3 / 2 max pool) as one launch against
    the same session built with LSC_FUSED_STEM=0 (three launches): the pooled activation and
    the logits bit for bit, at batches whose pooled rows split unevenly over the CTAs (CTAs
    that start inside an image, ranges that cross images).  The fused run never writes the
    space-to-depth input, which the separate launches do."""
    x = np.random.default_rng(100 + batch).normal(size=(batch, 3, 224, 224)).astype(np.float32)
    x[0, :, :5, :] = 40.0  # saturating input codes along the top edge
    monkeypatch.setenv("LSC_FUSED_STEM", "0")
    sep = _session(be, batch, x, plan_memory=False, rounding=rounding)
    monkeypatch.delenv("LSC_FUSED_STEM")
    fused = _session(be, batch, x, plan_memory=False, rounding=rounding)
    for sess in (sep, fused):
        v = sess.value("X:q")
        _fill_device(v["ptr"], v["nbytes"], 0)
    want = _run(sep, x)
    got = _run(fused, x)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    a, b = sep.value("pool"), fused.value("pool")
    assert a["shape"] == b["shape"] == [batch, 56, 56, 64]
    np.testing.assert_array_equal(_device_bytes(b["ptr"], b["nbytes"], np.int8),
                                  _device_bytes(a["ptr"], a["nbytes"], np.int8))
    xq_sep = sep.value("X:q")
    xq_fused = fused.value("X:q")
    assert np.any(_device_bytes(xq_sep["ptr"], xq_sep["nbytes"], np.int8) != 0)
    assert not np.any(_device_bytes(xq_fused["ptr"], xq_fused["nbytes"], np.int8) != 0)
