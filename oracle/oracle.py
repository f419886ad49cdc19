"""ctypes wrapper of the CPU oracle ``oracle/liblsc_oracle.so``.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py``, as the checker (or the timed CPU baseline).  The product
(``lightship_b200``) never imports this module.  The algorithms and their reference
citations are in ``lsc_oracle.cpp``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblsc_oracle.so")

ROUND_HALF_AWAY = 0
ROUND_HALF_EVEN = 1
ACT_NONE, ACT_RELU, ACT_RELU6, ACT_SILU, ACT_GELU = 0, 1, 2, 3, 4
QUINT8, QINT8, QINT32 = 0, 1, 2
OTHER = 3  # any non-quantized DataType: the `_` arm of helpers.rs:109-114 / :140-151, (0, 255)


def build() -> str:
    """Runs the oracle's Makefile (g++ only, no GPU)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int32
F32 = C.c_float


def _declare(l):
    sig = {
        "orc_gemm_scalar": [P, P, P, I64, I64, I64],
        "orc_gemm_blocked": [P, P, P, I64, I64, I64],
        "orc_matmul": [P, P, P, I64, I64, I64, C.c_int],
        "orc_fully_connected": [P, P, P, I64, I64, I64, C.c_int],
        "orc_conv2d_nchw": [P, P, P, P] + [I64] * 14 + [C.c_int],
        "orc_conv2d_nchw_reference_korder": [P, P, P] + [I64] * 14,
        "orc_batchnorm_inference": [P, P, I64, I64, I64, P, P, P, P, F32],
        "orc_bn_fold": [P, P, P, P, P, P, F32, I64, I64, P, P],
        "orc_act_inplace": [P, I64, C.c_int],
        "orc_layernorm": [P, P, I64, I64, P, P, F32],
        "orc_softmax": [P, P, I64, I64],
        "orc_quantize_tensor": [P, I64, F32, I32, C.c_int, P],
        "orc_dequantize_tensor": [P, I64, F32, I32, C.c_int, P],
        "orc_quantize_sym": [P, P, I64, F32, C.c_int],
        "orc_quantize_weights_per_channel": [P, I64, I64, P, P],
        "orc_gemm_i8_nn": [P, P, P, I64, I64, I64, C.c_int],
        "orc_gemm_i8_tn": [P, P, P, I64, I64, I64, C.c_int],
        "orc_requant": [P, I64, I64, P, P, C.c_int, F32, C.c_int, P, P, P],
        "orc_gemm_i8_chain": [P, P, I64, I64, I64, P, P, C.c_int, F32, C.c_int, P, P, P, C.c_int],
        "orc_conv2d_i8_nhwc_chain": [P, P] + [I64] * 14 + [P, P, C.c_int, F32, C.c_int, P, P, P, C.c_int],
        "orc_conv2d_i8_nhwc_chain_res": [P, P] + [I64] * 13 + [P, P, C.c_int, F32, C.c_int, P, F32, P, P, P,
                                                                C.c_int],
        "orc_quantize_nchw_to_nhwc": [P, P, I64, I64, I64, I64, F32, C.c_int],
        "orc_maxpool_i8_nhwc": [P, P] + [I64] * 10,
        "orc_avgpool_i8_nhwc": [P, I64, I64, I64, F32, F32, C.c_int, P, P],
    }
    for name, args in sig.items():
        f = getattr(l, name)
        f.argtypes = args
        f.restype = None
    l.orc_act.argtypes = [F32, C.c_int]
    l.orc_act.restype = F32
    l.orc_round.argtypes = [F32, C.c_int]
    l.orc_round.restype = F32
    l.orc_quantize_value.argtypes = [F32, F32, I32, C.c_int]
    l.orc_quantize_value.restype = I32
    l.orc_dequantize_value.argtypes = [I32, F32, I32]
    l.orc_dequantize_value.restype = F32
    l.orc_find_scale_zp.argtypes = [P, I64, C.c_int, C.c_int, C.POINTER(F32), C.POINTER(I32)]
    l.orc_find_scale_zp.restype = C.c_int
    l.orc_conv_out_dim.argtypes = [I64] * 5
    l.orc_conv_out_dim.restype = I64
    l.orc_version.restype = C.c_char_p


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------- FP32 path
def gemm_scalar(a, b, c=None):
    a, b = _c(a, np.float32), _c(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), np.float32) if c is None else _c(c, np.float32).copy()
    lib().orc_gemm_scalar(_p(a), _p(b), _p(c), m, n, k)
    return c


def gemm_blocked(a, b, c=None):
    a, b = _c(a, np.float32), _c(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), np.float32) if c is None else _c(c, np.float32).copy()
    lib().orc_gemm_blocked(_p(a), _p(b), _p(c), m, n, k)
    return c


def matmul(a, b, threads=0):
    a, b = _c(a, np.float32), _c(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().orc_matmul(_p(a), _p(b), _p(c), m, n, k, threads)
    return c


def fully_connected(x, w, threads=0):
    x, w = _c(x, np.float32), _c(w, np.float32)
    b, i = x.shape
    o = w.shape[0]
    y = np.empty((b, o), np.float32)
    lib().orc_fully_connected(_p(x), _p(w), _p(y), b, i, o, threads)
    return y


def conv_out_dim(n, k, s, p, d):
    return lib().orc_conv_out_dim(n, k, s, p, d)


def conv2d_nchw(x, w, bias=None, stride=(1, 1), pad=(0, 0), dilation=(1, 1), groups=1,
                threads=0, reference_korder=False):
    x, w, bias = _c(x, np.float32), _c(w, np.float32), _c(bias, np.float32)
    n, ci, h, wd = x.shape
    co, _, kh, kw = w.shape
    oh = conv_out_dim(h, kh, stride[0], pad[0], dilation[0])
    ow = conv_out_dim(wd, kw, stride[1], pad[1], dilation[1])
    y = np.zeros((n, co, oh, ow), np.float32)
    args = [n, ci, h, wd, co, kh, kw, stride[0], stride[1], pad[0], pad[1], dilation[0], dilation[1], groups]
    if reference_korder:
        lib().orc_conv2d_nchw_reference_korder(_p(x), _p(w), _p(y), *args)
    else:
        lib().orc_conv2d_nchw(_p(x), _p(w), _p(bias), _p(y), *args, threads)
    return y


def batchnorm_inference(x, gamma=None, beta=None, mean=None, var=None, eps=1e-5):
    x = _c(x, np.float32)
    n, c = x.shape[0], x.shape[1]
    spatial = int(np.prod(x.shape[2:])) if x.ndim > 2 else 1
    y = np.empty_like(x)
    lib().orc_batchnorm_inference(_p(x), _p(y), n, c, spatial, _p(_c(gamma, np.float32)),
                                  _p(_c(beta, np.float32)), _p(_c(mean, np.float32)),
                                  _p(_c(var, np.float32)), eps)
    return y


def bn_fold(w, bias, gamma, beta, mean, var, eps=1e-5):
    w = _c(w, np.float32)
    co = w.shape[0]
    per = int(np.prod(w.shape[1:]))
    wo = np.empty_like(w)
    bo = np.empty(co, np.float32)
    lib().orc_bn_fold(_p(w), _p(_c(bias, np.float32)), _p(_c(gamma, np.float32)), _p(_c(beta, np.float32)),
                      _p(_c(mean, np.float32)), _p(_c(var, np.float32)), eps, co, per, _p(wo), _p(bo))
    return wo, bo


def act(x, kind):
    y = _c(x, np.float32).copy()
    lib().orc_act_inplace(_p(y), y.size, kind)
    return y


def layernorm(x, gamma=None, beta=None, eps=1e-5):
    """LayerNorm over the last axis (layernorm.rs:153-205)."""
    x = _c(x, np.float32)
    d = x.shape[-1]
    y = np.empty_like(x)
    g = None if gamma is None else _c(gamma, np.float32)
    b = None if beta is None else _c(beta, np.float32)
    lib().orc_layernorm(_p(x), _p(y), x.size // max(d, 1), d, _p(g) if g is not None else None,
                        _p(b) if b is not None else None, eps)
    return y


def softmax(x):
    """Softmax over the last axis (softmax.rs:106-146)."""
    x = _c(x, np.float32)
    d = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_softmax(_p(x), _p(y), x.size // max(d, 1), d)
    return y


# ---------------------------------------------------------------- quantization
def quantize_value(v, scale, zp, qdtype):
    return lib().orc_quantize_value(v, scale, zp, qdtype)


def dequantize_value(q, scale, zp):
    return lib().orc_dequantize_value(q, scale, zp)


def find_scale_zp(data, qdtype=QINT8, symmetric=True):
    d = _c(data, np.float32).ravel()
    s, z = F32(), I32()
    lib().orc_find_scale_zp(_p(d), d.size, qdtype, int(symmetric), C.byref(s), C.byref(z))
    return s.value, z.value


def quantize_tensor(x, scale, zp, qdtype=QINT8):
    x = _c(x, np.float32)
    dt = {QINT8: np.int8, QUINT8: np.uint8, QINT32: np.int32}[qdtype]
    out = np.empty(x.shape, dt)
    lib().orc_quantize_tensor(_p(x), x.size, scale, zp, qdtype, _p(out))
    return out


def dequantize_tensor(q, scale, zp, qdtype=QINT8):
    dt = {QINT8: np.int8, QUINT8: np.uint8, QINT32: np.int32}[qdtype]
    q = _c(q, dt)
    out = np.empty(q.shape, np.float32)
    lib().orc_dequantize_tensor(_p(q), q.size, scale, zp, qdtype, _p(out))
    return out


def quantize_sym(x, scale, rounding=ROUND_HALF_AWAY):
    x = _c(x, np.float32)
    q = np.empty(x.shape, np.int8)
    lib().orc_quantize_sym(_p(x), _p(q), x.size, scale, rounding)
    return q


def quantize_weights_per_channel(w):
    w = _c(w, np.float32)
    rows = w.shape[0]
    cols = w.size // rows
    q = np.empty(w.shape, np.int8)
    s = np.empty(rows, np.float32)
    lib().orc_quantize_weights_per_channel(_p(w), rows, cols, _p(q), _p(s))
    return q, s


# ---------------------------------------------------------------- INT8 chain
def gemm_i8_nn(a, b, threads=0):
    a, b = _c(a, np.int8), _c(b, np.int8)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.int32)
    lib().orc_gemm_i8_nn(_p(a), _p(b), _p(c), m, n, k, threads)
    return c


def gemm_i8_tn(a, w, threads=0):
    a, w = _c(a, np.int8), _c(w, np.int8)
    m, k = a.shape
    n = w.shape[0]
    c = np.empty((m, n), np.int32)
    lib().orc_gemm_i8_tn(_p(a), _p(w), _p(c), m, n, k, threads)
    return c


def requant(acc, bias, scale, act=ACT_NONE, s_out=1.0, rounding=ROUND_HALF_AWAY):
    acc = _c(acc, np.int32)
    m, n = acc.shape
    oi8 = np.empty((m, n), np.int8)
    of32 = np.empty((m, n), np.float32)
    oacc = np.empty((m, n), np.int32)
    lib().orc_requant(_p(acc), m, n, _p(_c(bias, np.int32)), _p(_c(scale, np.float32)), act, s_out,
                      rounding, _p(oi8), _p(of32), _p(oacc))
    return oi8, of32, oacc


def gemm_i8_chain(a, w, bias, scale, act=ACT_NONE, s_out=1.0, rounding=ROUND_HALF_AWAY,
                  threads=0, want=("i8", "f32", "i32")):
    a, w = _c(a, np.int8), _c(w, np.int8)
    m, k = a.shape
    n = w.shape[0]
    oi8 = np.empty((m, n), np.int8) if "i8" in want else None
    of32 = np.empty((m, n), np.float32) if "f32" in want else None
    oacc = np.empty((m, n), np.int32) if "i32" in want else None
    lib().orc_gemm_i8_chain(_p(a), _p(w), m, n, k, _p(_c(bias, np.int32)), _p(_c(scale, np.float32)), act,
                            s_out, rounding, _p(oi8), _p(of32), _p(oacc), threads)
    return oi8, of32, oacc


def conv2d_i8_nhwc_chain(x, w, bias, scale, stride=(1, 1), pad=(0, 0), dilation=(1, 1), groups=1,
                         act=ACT_NONE, s_out=1.0, rounding=ROUND_HALF_AWAY, threads=0,
                         residual=None, residual_scale=1.0):
    """x: [N,H,W,Cin] int8; w: [Cout,KH,KW,Cin/groups] int8; returns NHWC outputs.
    `residual` (int8, output-shaped) is added before the activation (groups must be 1)."""
    x, w = _c(x, np.int8), _c(w, np.int8)
    n, h, wd, ci = x.shape
    co, kh, kw, _ = w.shape
    oh = conv_out_dim(h, kh, stride[0], pad[0], dilation[0])
    ow = conv_out_dim(wd, kw, stride[1], pad[1], dilation[1])
    oi8 = np.empty((n, oh, ow, co), np.int8)
    of32 = np.empty((n, oh, ow, co), np.float32)
    oacc = np.empty((n, oh, ow, co), np.int32)
    if residual is None:
        lib().orc_conv2d_i8_nhwc_chain(_p(x), _p(w), n, h, wd, ci, co, kh, kw, stride[0], stride[1], pad[0],
                                       pad[1], dilation[0], dilation[1], groups, _p(_c(bias, np.int32)),
                                       _p(_c(scale, np.float32)), act, s_out, rounding, _p(oi8), _p(of32),
                                       _p(oacc), threads)
    else:
        r = _c(residual, np.int8)
        assert r.shape == oi8.shape and groups == 1
        lib().orc_conv2d_i8_nhwc_chain_res(_p(x), _p(w), n, h, wd, ci, co, kh, kw, stride[0], stride[1],
                                           pad[0], pad[1], dilation[0], dilation[1], _p(_c(bias, np.int32)),
                                           _p(_c(scale, np.float32)), act, s_out, rounding, _p(r),
                                           residual_scale, _p(oi8), _p(of32), _p(oacc), threads)
    return oi8, of32, oacc


def resnet18_int8(x, convs, blocks, fc_w, fc_b, scales=None, rounding=ROUND_HALF_AWAY, threads=0):
    """The quantized ResNet-18 restated with this module's functions.

    x: f32 NCHW batch.  convs/blocks: the network's conv specs (name, cin, cout, k, stride,
    pad, relu, w OIHW f32, bias, bn=(gamma, beta, mean, var)) with blocks = [(conv1, conv2,
    downsample or None)].  With scales=None the activation scales are calibrated on this
    batch the way a deployment calibrates them: each layer's dequantized f32 output goes
    through find_scale_zp (symmetric, QInt8).  Returns (logits f32, scales, activations).
    """
    calibrate = scales is None
    sc = {} if calibrate else dict(scales)
    if calibrate:
        sc["input"], _ = find_scale_zp(x, QINT8, True)
    acts = {"x_q": quantize_nchw_to_nhwc(x, sc["input"], 16, rounding)}

    def conv(spec, in_name, residual=None):
        xin = acts[in_name]
        s_in = sc["input"] if in_name == "x_q" else sc[in_name]
        wf, bf = bn_fold(spec.w, spec.bias, *spec.bn)
        wq, sw = quantize_weights_per_channel(np.ascontiguousarray(wf.transpose(0, 2, 3, 1)))
        cs = xin.shape[3]
        wp = np.zeros((spec.cout, spec.k, spec.k, cs), np.int8)
        wp[..., :spec.cin] = wq
        scale = (np.float32(s_in) * sw).astype(np.float32)
        bq = np.array([quantize_value(float(bf[o]), float(scale[o]), 0, QINT32) for o in range(spec.cout)],
                      np.int32)
        res = None if residual is None else acts[residual]
        rs = 1.0 if residual is None else sc[residual]
        act_kind = ACT_RELU if spec.relu else ACT_NONE
        args = (xin, wp, bq, scale, (spec.stride,) * 2, (spec.pad,) * 2, (1, 1), 1, act_kind)
        if calibrate:
            _, y, _ = conv2d_i8_nhwc_chain(*args, 1.0, rounding, threads, residual=res, residual_scale=rs)
            sc[spec.name], _ = find_scale_zp(y, QINT8, True)
        q, _, _ = conv2d_i8_nhwc_chain(*args, sc[spec.name], rounding, threads, residual=res, residual_scale=rs)
        acts[spec.name] = q

    conv(convs[0], "x_q")
    acts["pool"] = maxpool_i8_nhwc(acts[convs[0].name], 3, 2, 1)
    sc["pool"] = sc[convs[0].name]
    prev = "pool"
    for c1, c2, ds in blocks:
        conv(c1, prev)
        if ds is not None:
            conv(ds, prev)
            res = ds.name
        else:
            res = prev
        conv(c2, c1.name, residual=res)
        prev = c2.name
    if calibrate:
        _, pf = avgpool_i8_nhwc(acts[prev], sc[prev], 1.0, rounding)
        sc["pooled"], _ = find_scale_zp(pf, QINT8, True)
    pooled, _ = avgpool_i8_nhwc(acts[prev], sc[prev], sc["pooled"], rounding)
    wq, sw = quantize_weights_per_channel(fc_w)
    scale = (np.float32(sc["pooled"]) * sw).astype(np.float32)
    bq = np.array([quantize_value(float(fc_b[o]), float(scale[o]), 0, QINT32) for o in range(fc_w.shape[0])],
                  np.int32)
    _, logits, _ = gemm_i8_chain(pooled, wq, bq, scale, ACT_NONE, 1.0, rounding, threads, want=("f32",))
    return logits, sc, acts


def quantize_nchw_to_nhwc(x, scale, cp, rounding=ROUND_HALF_AWAY):
    x = _c(x, np.float32)
    n, c, h, w = x.shape
    y = np.empty((n, h, w, cp), np.int8)
    lib().orc_quantize_nchw_to_nhwc(_p(x), _p(y), n, c, h * w, cp, scale, rounding)
    return y


def maxpool_i8_nhwc(x, k=3, s=2, p=1):
    x = _c(x, np.int8)
    n, h, w, c = x.shape
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    y = np.empty((n, oh, ow, c), np.int8)
    lib().orc_maxpool_i8_nhwc(_p(x), _p(y), n, h, w, c, k, k, s, s, p, p)
    return y


def avgpool_i8_nhwc(x, s_in, s_out=1.0, rounding=ROUND_HALF_AWAY):
    x = _c(x, np.int8)
    n, h, w, c = x.shape
    yq = np.empty((n, c), np.int8)
    yf = np.empty((n, c), np.float32)
    lib().orc_avgpool_i8_nhwc(_p(x), n, h * w, c, s_in, s_out, rounding, _p(yq), _p(yf))
    return yq, yf


# ---------------------------------------------------------------- transformer encoder block
def fc_i8_f32_weights(a_q, s_a, w, b, act=ACT_NONE, s_out=1.0, rounding=ROUND_HALF_AWAY, threads=0):
    """FullyConnected on int8 activations (scale s_a) with f32 weights [N, K] quantized per
    output channel and an f32 bias quantized to int32 in accumulator units
    (quantized_ops.rs:13-48 with helpers.rs:101-160): returns (int8, f32) outputs of the chain."""
    wq, sw = quantize_weights_per_channel(w)
    scale = (np.float32(s_a) * sw).astype(np.float32)
    bq = np.array([quantize_value(float(b[o]), float(scale[o]), 0, QINT32) for o in range(w.shape[0])], np.int32)
    oi8, of32, _ = gemm_i8_chain(a_q, wq, bq, scale, act, s_out, rounding, threads, want=("i8", "f32"))
    return oi8, of32


def attention_scores_f16(qkv, batch, seq, heads, head_dim, threads=0):
    """Q K^T / sqrt(head_dim) per head from a [batch*seq, 3*heads*head_dim] f16 projection
    (Q, K, V head-major), products accumulated in f32 (the reference GEMM) and stored as f16."""
    x = np.asarray(qkv, np.float16).astype(np.float32).reshape(batch, seq, 3, heads, head_dim)
    out = np.empty((batch, heads, seq, seq), np.float16)
    alpha = np.float32(1.0 / np.sqrt(head_dim))
    for bi in range(batch):
        for h in range(heads):
            q = np.ascontiguousarray(x[bi, :, 0, h, :])
            kt = np.ascontiguousarray(x[bi, :, 1, h, :].T)
            out[bi, h] = (matmul(q, kt, threads) * alpha).astype(np.float16)
    return out


def attention_context(p, qkv, batch, seq, heads, head_dim, threads=0):
    """P V per head: f16 probabilities [batch, heads, seq, seq] times the f16 V heads,
    accumulated in f32, written token-major [batch*seq, heads*head_dim] f32."""
    x = np.asarray(qkv, np.float16).astype(np.float32).reshape(batch, seq, 3, heads, head_dim)
    pf = np.asarray(p, np.float16).astype(np.float32)
    out = np.empty((batch, seq, heads, head_dim), np.float32)
    for bi in range(batch):
        for h in range(heads):
            out[bi, :, h, :] = matmul(np.ascontiguousarray(pf[bi, h]), np.ascontiguousarray(x[bi, :, 2, h, :]),
                                      threads)
    return out.reshape(batch * seq, heads * head_dim)


def encoder_block_int8(x, params, scales, batch, seq, heads=12, head_dim=64, rounding=ROUND_HALF_AWAY,
                       threads=0):
    """A pre-LayerNorm encoder block with INT8 projections and f16 attention, composed of the
    reference operators: LayerNorm (layernorm.rs:153-205), per-tensor quantize
    (helpers.rs:138-156), the INT8 chain, Softmax (softmax.rs:106-146), GELU (gelu.rs:77-103).
    ``scales`` holds the per-tensor activation scales q1 (LN1 out), q2 (attention context),
    q3 (LN2 out) and u (GELU out).  Returns every intermediate by name."""
    p = params
    r = {}
    r["ln1"] = layernorm(x, p["ln1_g"], p["ln1_b"], 1e-5)
    r["q1"] = quantize_tensor(r["ln1"], scales["q1"], 0)
    r["qkv"] = fc_i8_f32_weights(r["q1"], scales["q1"], p["wqkv"], p["bqkv"], rounding=rounding,
                                 threads=threads)[1].astype(np.float16)
    r["scores"] = attention_scores_f16(r["qkv"], batch, seq, heads, head_dim, threads)
    r["p"] = softmax(r["scores"].astype(np.float32)).astype(np.float16)
    r["o"] = attention_context(r["p"], r["qkv"], batch, seq, heads, head_dim, threads)
    r["q2"] = quantize_tensor(r["o"], scales["q2"], 0)
    r["h"] = fc_i8_f32_weights(r["q2"], scales["q2"], p["wo"], p["bo"], rounding=rounding,
                               threads=threads)[1] + np.asarray(x, np.float32)
    r["ln2"] = layernorm(r["h"], p["ln2_g"], p["ln2_b"], 1e-5)
    r["q3"] = quantize_tensor(r["ln2"], scales["q3"], 0)
    r["u"] = fc_i8_f32_weights(r["q3"], scales["q3"], p["w1"], p["b1"], ACT_GELU, scales["u"], rounding,
                               threads)[0]
    r["out"] = fc_i8_f32_weights(r["u"], scales["u"], p["w2"], p["b2"], rounding=rounding,
                                 threads=threads)[1] + r["h"]
    return r
