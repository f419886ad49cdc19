"""INT8 Conv2d through the Backend API on shapes that run pixel-grouped (G pixels of C
channels per im2col request, filter expanded to G*Cout columns), against the oracle's direct
convolution of the same quantized weights: bit-exact int8 outputs.  Covers the ResNet
layer1 shape (G=2), C=32 and C=16 inputs, a 5x5 filter, the space-to-depth stem geometry with
a padded row pitch cropped by a negative end padding (G=4), a fused residual, a batch other
than the compiled one, and a width that does not divide (plain path)."""
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


def _oracle(x, w, b, s_in, s_out, pad, crop, act, rounding, residual=None, r_scale=1.0):
    """The backend's compile-time quantization restated, then the oracle's int8 conv."""
    co, ci, k, _ = w.shape
    wq, sw = orc.quantize_weights_per_channel(np.ascontiguousarray(w.transpose(0, 2, 3, 1)))
    cs = x.shape[3]
    wp = np.zeros((co, k, k, cs), np.int8)
    wp[..., :ci] = wq
    scale = (np.float32(s_in) * sw).astype(np.float32)
    bq = np.array([orc.quantize_value(float(b[o]), float(scale[o]), 0, orc.QINT32) for o in range(co)], np.int32)
    xin = x[:, :, : x.shape[2] - crop, :] if crop else x
    q, _, _ = orc.conv2d_i8_nhwc_chain(np.ascontiguousarray(xin), wp, bq, scale, (1, 1), (pad, pad), (1, 1), 1,
                                       act, s_out, rounding, residual=residual, residual_scale=r_scale)
    return q


def _run(be, n, h, w_in, cs, ci, co, k, pad, crop=0, act=orc.ACT_RELU, rounding=orc.ROUND_HALF_AWAY,
         residual=False, seed=0, exec_n=None):
    import torch
    from lightship_b200.backend import (Activation, DataType, OperatorDef, OperatorType, Quantization,
                                        StorageLayout, Tensor)
    rng = np.random.default_rng(seed)
    s_in, s_out, r_scale = 0.02, 0.05, 0.03
    wt = (rng.normal(size=(co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
    bias = rng.normal(scale=0.1, size=co).astype(np.float32)

    def xdata(nb):
        x = np.zeros((nb, h, w_in, cs), np.int8)
        x[..., :ci] = rng.integers(-127, 128, size=(nb, h, w_in, ci), dtype=np.int8)
        return x

    x0 = xdata(n)
    oh = h + 2 * pad - k + 1
    ow = w_in - crop + 2 * pad - k + 1
    dev = torch.device("cuda:0")

    def t_in(x):
        return Tensor("x", list(x.shape), DataType.QInt8, torch.from_numpy(x).to(dev), layout=StorageLayout.NHWC,
                      quantization=Quantization([s_in]))

    def t_out(nb):
        return Tensor("y", [nb, oh, ow, co], DataType.QInt8, torch.zeros((nb, oh, ow, co), dtype=torch.int8,
                                                                         device=dev),
                      layout=StorageLayout.NHWC, quantization=Quantization([s_out]))

    op = be.compile_operator(
        OperatorDef("conv", OperatorType.Conv2d, padding=(pad, pad), padding_end_delta=(0, -crop),
                    activation=Activation(act), rounding=rounding_enum(rounding), output_scale=s_out),
        None, [t_in(x0), Tensor("w", list(wt.shape), DataType.F32, wt), Tensor("b", [co], DataType.F32, bias)],
        [t_out(n)])
    nb = exec_n or n
    x = xdata(nb) if exec_n else x0
    ins = [t_in(x)]
    r = None
    if residual:
        r = rng.integers(-128, 128, size=(nb, oh, ow, co), dtype=np.int8)
        ins.append(Tensor("r", list(r.shape), DataType.QInt8, torch.from_numpy(r).to(dev),
                          layout=StorageLayout.NHWC, quantization=Quantization([r_scale])))
    y = t_out(nb)
    be.execute(op, ins, [y])
    torch.cuda.synchronize()
    got = y.data.cpu().numpy()
    want = _oracle(x, wt, bias, s_in, s_out, pad, crop, act, rounding, r, r_scale)
    np.testing.assert_array_equal(got, want)
    assert np.abs(want.astype(np.int32)).max() > 20  # not a saturated or all-zero output


def rounding_enum(r):
    from lightship_b200.backend import Rounding
    return Rounding(r)


def test_grouped_layer1_shape(be):
    _run(be, 2, 56, 56, 64, 64, 64, 3, 1)


def test_grouped_layer1_residual_half_even(be):
    _run(be, 2, 56, 56, 64, 64, 64, 3, 1, residual=True, rounding=orc.ROUND_HALF_EVEN, seed=1)


@pytest.mark.parametrize("cs,ci,w_in,k,pad", [(32, 32, 20, 3, 1), (16, 9, 16, 5, 2), (16, 16, 12, 3, 1),
                                             (64, 40, 14, 3, 0)])
def test_grouped_channel_widths(be, cs, ci, w_in, k, pad):
    _run(be, 3, 11, w_in, cs, ci, 48, k, pad, seed=cs + k)


def test_grouped_stem_pitch_and_crop(be):
    """Space-to-depth stem geometry: 16 stored channels, 4x4 taps, input width 24 of which
    the last column is pitch padding cropped by a -1 end padding: 20 output columns, G=4."""
    _run(be, 2, 23, 24, 16, 12, 64, 4, 0, crop=1, seed=7)


def test_grouped_other_batch_and_act_none(be):
    _run(be, 2, 14, 14, 64, 64, 96, 3, 1, act=orc.ACT_NONE, seed=3, exec_n=5)


def test_grouped_weights_resident_layer1_batch32(be):
    """Batch 32 of the layer1 shape: 392 grouped M tiles, so the grouped filter stays
    resident in shared memory while the pixel tiles stream."""
    _run(be, 32, 56, 56, 64, 64, 64, 3, 1, residual=True, seed=11)


def test_grouped_weights_resident_stem_batch16(be):
    """Batch 16 of the space-to-depth stem (115 x 116 x 16, 4x4, cropped to 112 columns):
    G=4, the 256-column grouped filter resident."""
    _run(be, 16, 115, 116, 16, 12, 64, 4, 0, crop=1, seed=12)


def test_width_not_divisible_runs_plain(be):
    _run(be, 2, 15, 15, 64, 64, 64, 3, 1, seed=4)
