"""Winograd F(2x2, 3x3) as the FP32 convolution kernels compute it (winograd_f32.cu), restated
in numpy: 4x4 input patches at (2*ty - pad, 2*tx - pad) with zeros outside the image,
V = B^T d B, U = G g G^T (double, rounded once to f32), M = sum over channels of U (.) V,
Y = A^T M A, cropped to the output size.  Checked against a float64 direct convolution
(the reference's WinogradConv2d, lightship-core/src/cpu/winograd_conv2d.rs:50-397, computes
the same convolution; its own transform is not used as the check)."""
import numpy as np
import pytest

BT = np.array([[1, 0, -1, 0], [0, 1, 1, 0], [0, -1, 1, 0], [0, 1, 0, -1]], np.float64)
G = np.array([[1, 0, 0], [.5, .5, .5], [.5, -.5, .5], [0, 0, 1]], np.float64)
AT = np.array([[1, 1, 1, 0], [0, 1, -1, -1]], np.float64)


def direct64(x, w, pad):
    n, c, h, wd = x.shape
    oh, ow = h + 2 * pad - 2, wd + 2 * pad - 2
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    y = np.zeros((n, w.shape[0], oh, ow))
    for i in range(3):
        for j in range(3):
            y += np.einsum("nchw,oc->nohw", xp[:, :, i:i + oh, j:j + ow], w[:, :, i, j].astype(np.float64))
    return y


def winograd_f32(x, w, pad):
    """The kernels' arithmetic in f32, except the channel sum (the tensor-core GEMM), done in
    float64 and rounded once."""
    f = np.float32
    n, c, h, wd = x.shape
    oh, ow = h + 2 * pad - 2, wd + 2 * pad - 2
    th, tw = (oh + 1) // 2, (ow + 1) // 2
    xp = np.zeros((n, c, 2 * th + 2, 2 * tw + 2), f)
    hh, ww = min(h, 2 * th + 2 - pad), min(wd, 2 * tw + 2 - pad)
    xp[:, :, pad:pad + hh, pad:pad + ww] = x[:, :, :hh, :ww]
    d = np.stack([np.stack([xp[:, :, i:i + 2 * th:2, j:j + 2 * tw:2] for j in range(4)]) for i in range(4)])
    b = np.stack([d[0] - d[2], d[1] + d[2], d[2] - d[1], d[1] - d[3]])                 # B^T d (rows)
    v = np.stack([b[:, 0] - b[:, 2], b[:, 1] + b[:, 2], b[:, 2] - b[:, 1], b[:, 1] - b[:, 3]], axis=1)  # (B^T d) B
    u = np.einsum("ai,ocij,bj->aboc", G, w.astype(np.float64), G).astype(f)
    m = np.einsum("abncst,aboc->abnost", v.astype(np.float64), u.astype(np.float64)).astype(f)
    a = np.stack([m[0] + m[1] + m[2], m[1] - m[2] - m[3]])                              # A^T m
    y = np.stack([a[:, 0] + a[:, 1] + a[:, 2], a[:, 1] - a[:, 2] - a[:, 3]], axis=1)     # (A^T m) A
    y = y.transpose(2, 3, 4, 0, 5, 1).reshape(n, w.shape[0], 2 * th, 2 * tw)
    return y[:, :, :oh, :ow]


@pytest.mark.parametrize("n,c,co,h,wd,pad", [(1, 64, 64, 56, 56, 1), (2, 5, 7, 9, 11, 1), (1, 16, 8, 10, 10, 0),
                                             (1, 8, 8, 7, 7, 2), (3, 3, 4, 6, 5, 1)])
def test_winograd_restatement_matches_direct_convolution(n, c, co, h, wd, pad):
    rng = np.random.default_rng(n * 1000 + c * 10 + pad)
    x = rng.normal(size=(n, c, h, wd)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / (9 * c)), (co, c, 3, 3)).astype(np.float32)
    ref = direct64(x, w, pad)
    mag = direct64(np.abs(x), np.abs(w), pad)
    y = winograd_f32(x, w, pad)
    assert y.shape == ref.shape
    assert float(np.max(np.abs(y - ref) / mag)) < 1e-6
