"""INT8 NHWC implicit-GEMM convolution vs the oracle's direct convolution, bit-exact, over
ResNet-18's layer shapes and the geometry edge cases (stride, padding, dilation, channel
blocks of 16/32/64/128 bytes, ragged M tiles, the C_in=3 stem padded to 16 channels)."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _conv_case(cuda, n, h, w, c, co, k, s, p, d=1, act=orc.ACT_NONE, rounding=orc.ROUND_HALF_EVEN,
               c_store=None, kw=None, seed=0):
    import torch
    from lightship_b200 import ops
    kw = kw or k
    rng = np.random.default_rng(seed + n * 7 + h + c + co + k)
    x = rng.integers(-127, 128, size=(n, h, w, c), dtype=np.int8)
    wt = rng.integers(-127, 128, size=(co, k, kw, c), dtype=np.int8)
    bias = rng.integers(-20000, 20000, size=co, dtype=np.int32)
    scale = rng.uniform(1e-4, 1e-3, size=co).astype(np.float32)
    s_out = 0.5
    want = orc.conv2d_i8_nhwc_chain(x, wt, bias, scale, (s, s), (p, p), (d, d), 1, act, s_out, rounding)
    cs = c_store or c
    xs = np.zeros((n, h, w, cs), np.int8)
    xs[..., :c] = x
    ws = np.zeros((co, k, kw, cs), np.int8)
    ws[..., :c] = wt
    q, y, acc = ops.conv2d_i8_nhwc(torch.from_numpy(xs).to(cuda), torch.from_numpy(ws).to(cuda),
                                   torch.from_numpy(scale).to(cuda), torch.from_numpy(bias).to(cuda),
                                   stride=(s, s), pad=(p, p), dilation=(d, d), s_out=s_out, act=act,
                                   rounding=rounding, out_i8=True, out_f32=True, out_i32=True)
    ops.check_device()
    np.testing.assert_array_equal(acc.cpu().numpy(), want[2])
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), want[1].view(np.uint32))
    np.testing.assert_array_equal(q.cpu().numpy(), want[0])


# ResNet-18 (224x224) layer shapes at batch 2
@pytest.mark.parametrize("h,c,co,k,s,p", [
    (56, 64, 64, 3, 1, 1),     # layer1 3x3
    (56, 64, 128, 3, 2, 1),    # layer2 first conv
    (56, 64, 128, 1, 2, 0),    # layer2 downsample
    (28, 128, 128, 3, 1, 1),   # layer2 3x3
    (28, 128, 256, 3, 2, 1),   # layer3 first conv
    (14, 256, 256, 3, 1, 1),   # layer3 3x3
    (14, 256, 512, 1, 2, 0),   # layer4 downsample
    (7, 512, 512, 3, 1, 1),    # layer4 3x3
])
def test_conv_i8_resnet_layers(cuda, h, c, co, k, s, p):
    _conv_case(cuda, 2, h, h, c, co, k, s, p, act=orc.ACT_RELU)


def test_conv_i8_stem_padded_channels(cuda):
    """7x7 stride-2 pad-3 stem with C_in = 3 stored as 16 zero-padded channels."""
    _conv_case(cuda, 2, 64, 64, 3, 64, 7, 2, 3, act=orc.ACT_RELU, c_store=16)


@pytest.mark.parametrize("c", [16, 32, 48, 96, 192])
def test_conv_i8_channel_blocks(cuda, c):
    _conv_case(cuda, 3, 11, 13, c, 40, 3, 1, 1)


@pytest.mark.parametrize("k,s,p,d", [(3, 2, 0, 1), (5, 1, 2, 1), (3, 1, 2, 2), (3, 3, 1, 1),
                                     (1, 1, 0, 1), (2, 2, 0, 1)])
def test_conv_i8_geometry(cuda, k, s, p, d):
    _conv_case(cuda, 2, 17, 15, 64, 72, k, s, p, d)


def test_conv_i8_non_square_filter_and_rounding(cuda):
    _conv_case(cuda, 1, 9, 20, 64, 16, 1, 1, 0, kw=3, rounding=orc.ROUND_HALF_AWAY)
    _conv_case(cuda, 1, 9, 20, 32, 16, 3, 1, 1, kw=1, rounding=orc.ROUND_HALF_AWAY, act=orc.ACT_RELU6)


@pytest.mark.parametrize("n,h,w,c,co,k,p,d", [(5, 12, 10, 64, 40, 3, 1, 1), (2, 9, 14, 32, 24, 5, 2, 1),
                                              (3, 16, 16, 16, 64, 3, 2, 2), (2, 32, 32, 128, 72, 1, 0, 1),
                                              (1, 115, 115, 16, 64, 4, 0, 1)])
def test_conv_i8_stride1_tiles(cuda, n, h, w, c, co, k, p, d):
    """Stride-1 shapes whose 128-row tiles straddle output rows and images, including
    dilation, padding and the space-to-depth stem geometry (115x115x16, 4x4)."""
    _conv_case(cuda, n, h, w, c, co, k, 1, p, d, act=orc.ACT_RELU)


def test_conv_i8_large_batch_ragged_tiles(cuda):
    """M = 5*13*13 = 845 output pixels: tiles straddle images and the last tile is ragged."""
    _conv_case(cuda, 5, 13, 13, 128, 256, 3, 1, 1, act=orc.ACT_RELU)


@pytest.mark.parametrize("n,h,c,s,k,p,act,rounding", [
    (25, 56, 128, 1, 3, 1, orc.ACT_RELU, orc.ROUND_HALF_EVEN),   # layer2 3x3 / grouped layer1
    (25, 57, 128, 1, 3, 1, orc.ACT_NONE, orc.ROUND_HALF_AWAY),   # ragged last tile
    (25, 112, 64, 2, 3, 1, orc.ACT_RELU, orc.ROUND_HALF_AWAY),   # layer2.0.conv1 (64-byte blocks)
    (25, 56, 256, 1, 1, 0, orc.ACT_NONE, orc.ROUND_HALF_EVEN),   # 1x1, two k-blocks
    (22, 60, 128, 1, 3, 1, orc.ACT_RELU6, orc.ROUND_HALF_EVEN),
])
def test_conv_i8_operand_swap(cuda, n, h, c, s, k, p, act, rounding):
    """128 output channels, two or more k-blocks and at least two waves of 256-pixel tiles: the
    convolution runs with the filter as the MMA's A operand and 256 output pixels as its B
    operand; bit-exact int32, f32 and int8 outputs."""
    _conv_case(cuda, n, h, h, c, 128, k, s, p, act=act, rounding=rounding, seed=11)
