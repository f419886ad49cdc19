"""ResNet-18-shaped INT8 network through the Backend API vs the oracle running the same
quantized network (same f32 parameters, the GPU's calibrated activation scales), bit for bit;
plus the INT8 glue operators (input quantize to NHWC, MaxPool2d, GlobalAvgPool2d, residual
Add+ReLU fused into a conv) on their own."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.golden.resnet_oracle import oracle_resnet18

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be(cuda):
    from lightship_b200.backend import CudaBackend, GpuBackendConfig
    b = CudaBackend(GpuBackendConfig(device_id=0, arena_bytes=1 << 30))
    yield b
    b.close()


@pytest.mark.parametrize("rounding", [0, 1])
def test_resnet18_int8_bit_exact(be, cuda, rounding):
    import torch
    from lightship_b200.backend import Rounding
    from lightship_b200.resnet18 import ResNet18Int8
    batch = 2
    model = ResNet18Int8(be, batch, cuda, image=224, seed=3, rounding=Rounding(rounding))
    rng = np.random.default_rng(99)
    x = rng.normal(size=(batch, 3, 224, 224)).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda)
    model.calibrate(xd)
    logits = model.forward(xd).cpu().numpy()
    torch.cuda.synchronize()
    want, acts = oracle_resnet18(x, model, rounding)
    for name in ("conv1", "pool", "layer1.0.conv2", "layer2.0.downsample", "layer4.1.conv2"):
        np.testing.assert_array_equal(model.buf[name].cpu().numpy(), acts[name], err_msg=name)
    np.testing.assert_array_equal(logits.view(np.uint32), want.view(np.uint32))
    # the oracle calibrating on its own reaches the same scales and logits
    own_logits, own_scales, _ = orc.resnet18_int8(x, model.convs, model.blocks, model.fc_w, model.fc_b,
                                                  None, rounding)
    assert own_scales == model.scales
    np.testing.assert_array_equal(own_logits.view(np.uint32), want.view(np.uint32))
    # the network is not degenerate: activations use the int8 range, logits differ per image
    assert np.abs(acts["layer4.1.conv2"]).max() >= 64
    assert not np.array_equal(logits[0], logits[1])


@pytest.mark.parametrize("branches,ds_side", [(1, False), (2, False), (4, True), (1, True)])
def test_resnet18_graph_replay_matches_eager(be, cuda, branches, ds_side):
    """The captured graph (one chain, or the batch cut into concurrent image groups, with or
    without the downsample convs on a side stream) gives the eager forward pass's logits bit
    for bit, on an input other than the captured one."""
    import torch
    from lightship_b200.resnet18 import ResNet18Int8
    batch = 4
    model = ResNet18Int8(be, batch, cuda, image=224, seed=5)
    rng = np.random.default_rng(7)
    x = torch.from_numpy(rng.normal(size=(batch, 3, 224, 224)).astype(np.float32)).to(cuda)
    model.calibrate(x)
    eager = model.forward(x).clone()
    static = x.clone()
    g = model.capture(static, branches=branches, concurrent_downsample=ds_side)
    x2 = torch.from_numpy(rng.normal(size=(batch, 3, 224, 224)).astype(np.float32)).to(cuda)
    static.copy_(x2)
    g.replay()
    torch.cuda.synchronize()
    replay = model.logits.clone()
    eager2 = model.forward(x2).clone()
    torch.cuda.synchronize()
    assert torch.equal(replay, eager2)
    assert not torch.equal(eager, eager2)


def test_maxpool_and_avgpool_ops(be):
    from lightship_b200.backend import (DataType, OperatorDef, OperatorType, Quantization, StorageLayout,
                                        Tensor)
    rng = np.random.default_rng(1)
    x = rng.integers(-128, 128, size=(3, 15, 13, 48), dtype=np.int8)
    xt = Tensor("x", list(x.shape), DataType.QInt8, x, layout=StorageLayout.NHWC, quantization=Quantization([0.03]))
    y = Tensor("y", [1], DataType.QInt8, np.zeros(3 * 8 * 7 * 48, np.int8))
    op = be.compile_operator(OperatorDef("mp", OperatorType.MaxPool2d, stride=(2, 2), padding=(1, 1), kernel=(3, 3)),
                             None, [xt], [y])
    be.execute(op, [xt], [y])
    assert y.shape == [3, 8, 7, 48]
    np.testing.assert_array_equal(y.numpy().reshape(3, 8, 7, 48), orc.maxpool_i8_nhwc(x, 3, 2, 1))
    for rounding in (0, 1):
        from lightship_b200.backend import Rounding
        yq = Tensor("yq", [1], DataType.QInt8, np.zeros(3 * 48, np.int8), quantization=Quantization([0.01]))
        yf = Tensor("yf", [1], DataType.F32, np.zeros(3 * 48, np.float32))
        op = be.compile_operator(OperatorDef("gap", OperatorType.GlobalAvgPool2d, rounding=Rounding(rounding)),
                                 None, [xt], [yq, yf])
        be.execute(op, [xt], [yq, yf])
        wq, wf = orc.avgpool_i8_nhwc(x, 0.03, 0.01, rounding)
        np.testing.assert_array_equal(yf.numpy().reshape(3, 48).view(np.uint32), wf.view(np.uint32))
        np.testing.assert_array_equal(yq.numpy().reshape(3, 48), wq)


def test_quantize_input_to_nhwc(be):
    from lightship_b200.backend import (DataType, OperatorDef, OperatorType, Quantization, StorageLayout,
                                        Tensor)
    rng = np.random.default_rng(2)
    x = rng.normal(size=(2, 3, 17, 19)).astype(np.float32)
    xt = Tensor("x", list(x.shape), DataType.F32, x, layout=StorageLayout.NCHW)
    q = Tensor("q", [2, 17, 19, 16], DataType.QInt8, np.zeros(2 * 17 * 19 * 16, np.int8),
               layout=StorageLayout.NHWC, quantization=Quantization([0.02]))
    op = be.compile_operator(OperatorDef("q", OperatorType.Quantize), None, [xt], [q])
    be.execute(op, [xt], [q])
    assert q.shape == [2, 17, 19, 16]
    np.testing.assert_array_equal(q.numpy().reshape(2, 17, 19, 16), orc.quantize_nchw_to_nhwc(x, 0.02, 16))


@pytest.mark.parametrize("c,cp,extra", [(3, 16, 0), (3, 16, 1), (5, 32, 0)])
def test_quantize_input_space_to_depth(be, c, cp, extra):
    """Quantize with stride 2: pad by 3 (and 2*extra more on the right), fold 2x2 pixel blocks
    into channels.  C=3 into 16 channels is the stem's specialised kernel; C=5 into 32 the
    general one."""
    from lightship_b200.backend import (DataType, OperatorDef, OperatorType, Quantization, StorageLayout,
                                        Tensor)
    rng = np.random.default_rng(6 + c + extra)
    x = rng.normal(size=(2, c, 26, 30)).astype(np.float32)
    hs, ws = (26 + 6) // 2, (30 + 6) // 2 + extra
    xt = Tensor("x", list(x.shape), DataType.F32, x, layout=StorageLayout.NCHW)
    q = Tensor("q", [2, hs, ws, cp], DataType.QInt8, np.zeros(2 * hs * ws * cp, np.int8),
               layout=StorageLayout.NHWC, quantization=Quantization([0.03]))
    op = be.compile_operator(OperatorDef("q", OperatorType.Quantize, stride=(2, 2), padding=(3, 3),
                                         padding_end_delta=(0, 2 * extra)), None, [xt], [q])
    be.execute(op, [xt], [q])
    assert q.shape == [2, hs, ws, cp]
    xp = np.zeros((2, c, 32, 36 + 2 * extra), np.float32)
    xp[:, :, 3:29, 3:33] = x
    qq = orc.quantize_nchw_to_nhwc(xp, 0.03, c)  # [2, 32, 36 + 2*extra, c]
    want = np.zeros((2, hs, ws, cp), np.int8)
    for dy in range(2):
        for dx in range(2):
            want[..., (dy * 2 + dx) * c:(dy * 2 + dx + 1) * c] = qq[:, dy::2, dx::2, :]
    np.testing.assert_array_equal(q.numpy().reshape(want.shape), want)


@pytest.mark.parametrize("n,h,c,co", [(3, 9, 64, 96), (24, 57, 128, 128)])
def test_conv_residual_kernel_level(cuda, n, h, c, co):
    """lsc_conv2d_i8_nhwc with a residual, including a ragged output tile; the second shape
    runs on the operand-swapped kernel (128 output channels, many pixels)."""
    import torch
    from lightship_b200 import ops
    rng = np.random.default_rng(4 + n)
    x = rng.integers(-127, 128, size=(n, h, h, c), dtype=np.int8)
    w = rng.integers(-127, 128, size=(co, 3, 3, c), dtype=np.int8)
    r = rng.integers(-128, 128, size=(n, h, h, co), dtype=np.int8)
    scale = rng.uniform(1e-5, 1e-4, co).astype(np.float32)
    want = orc.conv2d_i8_nhwc_chain(x, w, None, scale, (1, 1), (1, 1), (1, 1), 1, orc.ACT_RELU, 0.02,
                                    orc.ROUND_HALF_AWAY, residual=r, residual_scale=0.015)
    q, y, _ = ops.conv2d_i8_nhwc(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda),
                                 torch.from_numpy(scale).to(cuda), None, pad=(1, 1), s_out=0.02,
                                 act=1, out_i8=True, out_f32=True, residual=torch.from_numpy(r).to(cuda),
                                 residual_scale=0.015)
    ops.check_device()
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), want[1].view(np.uint32))
    np.testing.assert_array_equal(q.cpu().numpy(), want[0])


@pytest.mark.parametrize("batch", [32, 256])
def test_resnet18_int8_bit_exact_at_benchmark_batches(be, cuda, batch):
    """The network at the per-GPU batches the benchmark times (256 on one GPU, 32 per GPU on
    eight): tile widths, the operand-swapped kernel and weight residency are chosen from the
    batch, so these are different kernels from the batch-2 test.  Run as the benchmark runs it
    (one captured graph, downsample convs on a side stream); images are independent once the
    activation scales are fixed, so the first and last four images of the batch are checked
    against the oracle, logits and every block output."""
    import torch
    from lightship_b200.resnet18 import ResNet18Int8
    model = ResNet18Int8(be, batch, cuda, image=224, seed=11)
    rng = np.random.default_rng(batch)
    x = rng.normal(size=(batch, 3, 224, 224)).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda)
    model.calibrate(xd)
    g = model.capture(xd, branches=1, concurrent_downsample=True)
    model.logits.zero_()
    g.replay()
    torch.cuda.synchronize()
    logits = model.logits.cpu().numpy()
    pick = np.r_[0:4, batch - 4:batch]
    want, acts = oracle_resnet18(np.ascontiguousarray(x[pick]), model, 0)
    np.testing.assert_array_equal(logits[pick].view(np.uint32), want.view(np.uint32))
    for name in [f"layer{s}.{b}.conv2" for s in (1, 2, 3, 4) for b in (0, 1)] + ["conv1", "pool"]:
        np.testing.assert_array_equal(model.buf[name].cpu().numpy()[pick], acts[name], err_msg=name)
    del g
