"""Kernel-level operators on torch device tensors, calling the C ABI directly.

torch is only the device-memory and stream plumbing here: every operator below launches
this package's own sm_100a kernels through ``liblightship_cuda.so``.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import check, lib


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(device=None):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need(t, dtype, name):
    if t is None:
        return
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous CUDA {dtype} tensor, got {t.dtype} "
                         f"on {t.device} (contiguous={t.is_contiguous()})")


def gemm_i8(a, w, scale, bias=None, s_out=1.0, act=_lib.ACT_NONE,
            rounding=_lib.ROUND_HALF_AWAY, out_i8=True, out_f32=False, out_i32=False):
    """INT8 chain on the tensor cores: returns (q_i8, y_f32, acc_i32), each None unless asked.

    a: [M,K] int8, w: [N,K] int8, scale: [N] f32 (= s_a * s_w[n]), bias: [N] int32 or None.
    """
    _need(a, torch.int8, "a")
    _need(w, torch.int8, "w")
    _need(scale, torch.float32, "scale")
    _need(bias, torch.int32, "bias")
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"gemm_i8: K mismatch {a.shape} vs {w.shape}")
    dev = a.device
    q = torch.empty((m, n), dtype=torch.int8, device=dev) if out_i8 else None
    y = torch.empty((m, n), dtype=torch.float32, device=dev) if out_f32 else None
    acc = torch.empty((m, n), dtype=torch.int32, device=dev) if out_i32 else None
    check(lib().lsc_gemm_i8(_ptr(a), _ptr(w), m, n, k, _ptr(bias), _ptr(scale), float(s_out),
                            act, rounding, _ptr(q), _ptr(y), _ptr(acc), _stream(dev)))
    return q, y, acc


def conv2d_i8_nhwc(x, w, scale, bias=None, stride=(1, 1), pad=(0, 0), dilation=(1, 1),
                   s_out=1.0, act=_lib.ACT_NONE, rounding=_lib.ROUND_HALF_AWAY,
                   out_i8=True, out_f32=False, out_i32=False, residual=None, residual_scale=1.0):
    """INT8 NHWC convolution (implicit GEMM on the tensor cores, im2col by the TMA unit).

    x: [N,H,W,C] int8 (C a multiple of 16), w: [Cout,KH,KW,C] int8, scale: [Cout] f32,
    bias: [Cout] int32 or None.  Returns (q_i8, y_f32, acc_i32) as NHWC, None unless asked.
    """
    _need(x, torch.int8, "x")
    _need(w, torch.int8, "w")
    _need(scale, torch.float32, "scale")
    _need(bias, torch.int32, "bias")
    _need(residual, torch.int8, "residual")
    n, h, wd, c = x.shape
    co, kh, kw, cw = w.shape
    if cw != c:
        raise ValueError(f"conv2d_i8_nhwc: channel mismatch {x.shape} vs {w.shape}")
    oh = (h + 2 * pad[0] - dilation[0] * (kh - 1) - 1) // stride[0] + 1
    ow = (wd + 2 * pad[1] - dilation[1] * (kw - 1) - 1) // stride[1] + 1
    dev = x.device
    shape = (n, oh, ow, co)
    q = torch.empty(shape, dtype=torch.int8, device=dev) if out_i8 else None
    y = torch.empty(shape, dtype=torch.float32, device=dev) if out_f32 else None
    acc = torch.empty(shape, dtype=torch.int32, device=dev) if out_i32 else None
    check(lib().lsc_conv2d_i8_nhwc(_ptr(x), _ptr(w), n, h, wd, c, co, kh, kw, stride[0], stride[1],
                                   pad[0], pad[1], dilation[0], dilation[1], _ptr(bias), _ptr(scale),
                                   float(s_out), act, rounding, _ptr(q), _ptr(y), _ptr(acc),
                                   _ptr(residual), float(residual_scale), _stream(dev)))
    return q, y, acc


def check_device() -> int:
    """Synchronizes and returns the device error word (raises on a device-side error)."""
    w = C.c_uint32(0)
    check(lib().lsc_check_device(C.byref(w)))
    return w.value


def gemm_f16_batched(a, b, out, batch, heads, m, n, k, alpha=1.0, a_strides=None, b_strides=None,
                     out_strides=None, a_head0=0, b_head0=0):
    """Batched FP16 tensor-core GEMM with f32 accumulation (see ``lsc_gemm_f16_batched``):
    out[bb][m][n] = alpha * sum_k a[bb][m][k] * b[bb][n][k], bb = batch_index * heads + head.

    a, b: CUDA f16 tensors; ``*_strides`` = (row, head, batch) element strides, defaulting to a
    contiguous [batch, heads, rows, k] layout; out: CUDA f16 or f32 tensor with
    ``out_strides`` (row, head, batch), default contiguous [batch, heads, m, n].
    """
    _need(a, torch.float16, "a")
    _need(b, torch.float16, "b")
    if out.dtype not in (torch.float16, torch.float32) or not out.is_cuda:
        raise ValueError("out: expected a CUDA f16 or f32 tensor")
    a_strides = a_strides or (k, m * k, heads * m * k)
    b_strides = b_strides or (k, n * k, heads * n * k)
    out_strides = out_strides or (n, m * n, heads * m * n)
    dt = _lib.DTYPE_F16 if out.dtype == torch.float16 else _lib.DTYPE_F32
    check(lib().lsc_gemm_f16_batched(_ptr(a), *a_strides, a_head0, _ptr(b), *b_strides, b_head0, batch, heads,
                                     m, n, k, float(alpha), _ptr(out), dt, *out_strides, _stream(a.device)))
    return out


def transpose_heads_f16(x, y, batch, heads, rows, cols, x_strides, head0=0):
    """y[b][h][c][r] = x[b][h + head0][r][c]; x_strides = (batch, head, row) element strides."""
    _need(x, torch.float16, "x")
    _need(y, torch.float16, "y")
    check(lib().lsc_transpose_heads_f16(_ptr(x), _ptr(y), *x_strides, head0, batch, heads, rows, cols,
                                        _stream(x.device)))
    return y


def attention_f16(qkv, batch, seq, heads, alpha=0.125, out_f32=None, out_i8=None, s_out=1.0, rounding=0):
    """Fused attention (see ``lsc_attention_f16``) over the f16 QKV projection ``qkv``
    ([batch, seq, 3, heads, 64] elements, contiguous); outputs [batch * seq, heads * 64] f32
    and/or int8 (quantized with ``s_out``)."""
    _need(qkv, torch.float16, "qkv")
    if out_f32 is None and out_i8 is None:
        raise ValueError("attention_f16: no output")
    _need(out_f32, torch.float32, "out_f32")
    _need(out_i8, torch.int8, "out_i8")
    need = batch * seq * heads * 64
    for name, t in (("qkv", qkv), ("out_f32", out_f32), ("out_i8", out_i8)):
        if t is not None and t.numel() < (3 * need if name == "qkv" else need):
            raise ValueError(f"attention_f16: {name} too small")
    check(lib().lsc_attention_f16(_ptr(qkv), batch, seq, heads, float(alpha), _ptr(out_f32), _ptr(out_i8),
                                  float(s_out), int(rounding), _stream(qkv.device)))
