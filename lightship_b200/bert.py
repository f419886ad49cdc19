"""A BERT-base-shaped transformer encoder block (pre-LayerNorm) on the CUDA backend:

    h   = x + Wo . Attention(LN1(x))          Attention: softmax(Q K^T / 8) V per head (FP16)
    out = h + W2 . GELU(W1 . LN2(h))

hidden 768, 12 heads x 64, FFN 3072.  The four projections are INT8 FullyConnected operators
(per-channel weights quantized at compile from f32 N(0, 0.02); activations quantized per
tensor with scales calibrated on the first batch), their epilogues adding the bias, the GELU
(FFN up, requantized straight to int8 for FFN down), the f32 residual (output projection and
FFN down) or writing f16 (the fused QKV projection, read in place by the attention).  The
attention is one fused kernel (scores, f16 softmax and P V without the scores leaving the
chip) writing its output already quantized for the output projection, and LayerNorm writes
the int8 input of the projection after it, so the forward pass is one CUDA graph of 7 kernel
launches: LayerNorm, QKV, attention, output projection, LayerNorm, FFN up, FFN down.

Reference operators: LayerNorm (core/operator/layernorm.rs:153-205), GELU (gelu.rs:77-103),
Softmax (softmax.rs:106-146), the INT8 chain (core/cpu/quantized_ops.rs:13-48,
quantization/helpers.rs:101-160); the block shape is the BERT-base encoder-block benchmark
configuration (seq 384, batch 32).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib, ops
from .backend import (Activation, CudaBackend, DataType, OperatorDef, OperatorType, Quantization, Rounding,
                      Tensor)

HIDDEN, HEADS, HEAD_DIM, FFN = 768, 12, 64, 3072
# INT8 multiply-adds x 2 per token: QKV 768x2304, out 768x768, FFN 768x3072 twice
INT8_OPS_PER_TOKEN = 2 * (HIDDEN * 3 * HIDDEN + HIDDEN * HIDDEN + 2 * HIDDEN * FFN)


def attention_flops(batch, seq):
    """FP16 flops of Q K^T and P V."""
    return 2 * 2 * batch * HEADS * seq * seq * HEAD_DIM


def build_params(seed):
    rng = np.random.default_rng(seed)
    f = np.float32
    return {
        "ln1_g": rng.uniform(0.8, 1.2, HIDDEN).astype(f), "ln1_b": rng.normal(0, 0.02, HIDDEN).astype(f),
        "wqkv": rng.normal(0, 0.02, (3 * HIDDEN, HIDDEN)).astype(f), "bqkv": rng.normal(0, 0.02, 3 * HIDDEN).astype(f),
        "wo": rng.normal(0, 0.02, (HIDDEN, HIDDEN)).astype(f), "bo": rng.normal(0, 0.02, HIDDEN).astype(f),
        "ln2_g": rng.uniform(0.8, 1.2, HIDDEN).astype(f), "ln2_b": rng.normal(0, 0.02, HIDDEN).astype(f),
        "w1": rng.normal(0, 0.02, (FFN, HIDDEN)).astype(f), "b1": rng.normal(0, 0.02, FFN).astype(f),
        "w2": rng.normal(0, 0.02, (HIDDEN, FFN)).astype(f), "b2": rng.normal(0, 0.02, HIDDEN).astype(f),
    }


class BertBlockInt8:
    """The block compiled on one device for a fixed [batch, seq] shape."""

    def __init__(self, backend: CudaBackend, batch: int, seq: int, device, seed: int = 0,
                 rounding: Rounding = Rounding.HalfAwayFromZero):
        import torch
        self.torch = torch
        self.be = backend
        self.batch, self.seq, self.device, self.rounding = batch, seq, device, rounding
        self.params = build_params(seed)
        self.scales: dict = {}
        self.ops: dict = {}
        self.graph = None
        t = batch * seq
        e = dict(device=device)
        self.buf = {
            "x": torch.empty(t, HIDDEN, dtype=torch.float32, **e),
            "ln1": torch.empty(t, HIDDEN, dtype=torch.float32, **e),
            "q1": torch.empty(t, HIDDEN, dtype=torch.int8, **e),
            "qkv": torch.empty(batch, seq, 3 * HEADS, HEAD_DIM, dtype=torch.float16, **e),
            "o": torch.empty(t, HIDDEN, dtype=torch.float32, **e),
            "q2": torch.empty(t, HIDDEN, dtype=torch.int8, **e),
            "h": torch.empty(t, HIDDEN, dtype=torch.float32, **e),
            "ln2": torch.empty(t, HIDDEN, dtype=torch.float32, **e),
            "q3": torch.empty(t, HIDDEN, dtype=torch.int8, **e),
            "u": torch.empty(t, FFN, dtype=torch.int8, **e),
            "u_f32": torch.empty(t, FFN, dtype=torch.float32, **e),
            "out": torch.empty(t, HIDDEN, dtype=torch.float32, **e),
        }
        self.ws = torch.zeros(4, dtype=torch.int32, **e)

    # ------------------------------------------------------------------ helpers
    def _stream(self):
        return self.torch.cuda.current_stream(self.device).cuda_stream

    def _f32(self, name, t=None):
        t = self.buf[name] if t is None else t
        return Tensor(name, list(t.shape), DataType.F32, t)

    def _i8(self, name, scale):
        t = self.buf[name]
        return Tensor(name, list(t.shape), DataType.QInt8, t, quantization=Quantization([float(scale)]))

    def _scale_of(self, t) -> float:
        torch = self.torch
        s = torch.empty(1, dtype=torch.float32, device=self.device)
        z = torch.empty(1, dtype=torch.int32, device=self.device)
        flat = t.reshape(-1)
        _lib.check(_lib.lib().lsc_find_scale_zp_f32(C.c_void_p(flat.data_ptr()), flat.numel(), 9, 1,
                                                    C.c_void_p(self.ws.data_ptr()), 16, C.c_void_p(s.data_ptr()),
                                                    C.c_void_p(z.data_ptr()), C.c_void_p(self._stream())))
        return float(s.item())

    def _calibrated(self, q, src, fixed):
        return float(fixed[q]) if fixed else self._scale_of(self.buf[src])

    def _run(self, name, ins, outs):
        self.be.execute(self.ops[name], ins, outs, stream=self._stream())

    def _fc(self, name, in_name, s_in, w, b, outs, act=Activation.NONE):
        xin = self._i8(in_name, s_in)
        self.ops[name] = self.be.compile_operator(
            OperatorDef(name, OperatorType.FullyConnected, activation=act, rounding=self.rounding),
            None, [xin, Tensor("w", list(w.shape), DataType.F32, w), Tensor("b", [w.shape[0]], DataType.F32, b)],
            outs)

    # ------------------------------------------------------------------ stages
    def _attention(self, out_f32=None, out_i8=None):
        """softmax(Q K^T / 8) V per head, fused (one kernel), from the f16 QKV projection."""
        ops.attention_f16(self.buf["qkv"], self.batch, self.seq, HEADS, alpha=1.0 / 8.0, out_f32=out_f32,
                          out_i8=out_i8, s_out=self.scales.get("q2", 1.0), rounding=int(self.rounding))

    def _qkv_out(self):
        qkv = self.buf["qkv"].view(self.batch * self.seq, 3 * HIDDEN)
        return Tensor("qkv", list(qkv.shape), DataType.F16, qkv)

    # ------------------------------------------------------------------ calibration / forward
    def calibrate(self, x, scales=None):
        """Compiles every operator and fixes the activation scales (q1, q2, q3, u) from this
        batch ([batch*seq, 768] f32 on the device), or takes them from ``scales``.  Each
        scale comes from the f32 tensor it quantizes, computed here once in f32; the forward
        pass then writes the int8 tensors directly (LayerNorm with an int8 output, the FFN
        up-projection requantizing its GELU)."""
        torch = self.torch
        p = self.params
        self.buf["x"].copy_(x)
        # LN1 (f32) -> scale of q1 -> LN1 to int8 -> QKV -> attention -> scale of q2 -> out proj (+x) ...
        self._ln_calibrate("ln1", "x", "q1", p["ln1_g"], p["ln1_b"], scales)
        self._run("ln1", [self._f32("x")], [self._i8("q1", self.scales["q1"])])
        self._fc("qkv", "q1", self.scales["q1"], p["wqkv"], p["bqkv"], [self._qkv_out()])
        self._run("qkv", [self._i8("q1", self.scales["q1"])], [self._qkv_out()])
        self._attention(out_f32=self.buf["o"])
        self.scales["q2"] = self._calibrated("q2", "o", scales)
        self._attention(out_i8=self.buf["q2"])
        self._fc("out", "q2", self.scales["q2"], p["wo"], p["bo"], [self._f32("h")])
        self._run("out", [self._i8("q2", self.scales["q2"]), self._f32("x")], [self._f32("h")])
        self._ln_calibrate("ln2", "h", "q3", p["ln2_g"], p["ln2_b"], scales)
        self._run("ln2", [self._f32("h")], [self._i8("q3", self.scales["q3"])])
        # FFN up: calibrate its int8 output scale from the f32 GELU output, then run it requantized
        self._fc("ffn_up", "q3", self.scales["q3"], p["w1"], p["b1"], [self._f32("u_f32")], act=Activation.GELU)
        self._run("ffn_up", [self._i8("q3", self.scales["q3"])], [self._f32("u_f32")])
        self.scales["u"] = self._calibrated("u", "u_f32", scales)
        self._fc("ffn_up_i8", "q3", self.scales["q3"], p["w1"], p["b1"], [self._i8("u", self.scales["u"])],
                 act=Activation.GELU)
        self._fc("ffn_down", "u", self.scales["u"], p["w2"], p["b2"], [self._f32("out")])
        torch.cuda.synchronize(self.device)
        self.forward_device()
        torch.cuda.synchronize(self.device)

    def _ln_calibrate(self, name, src, q, g, b, fixed):
        """LayerNorm `name` of `src`: runs it once to f32 (into buf[name]) for the scale of
        `q`, then compiles it with the int8 output `q` the forward pass uses."""
        ins = [self._f32(src), Tensor("g", [HIDDEN], DataType.F32, g), Tensor("b", [HIDDEN], DataType.F32, b)]
        f32_op = self.be.compile_operator(OperatorDef(name, OperatorType.LayerNorm, epsilon=1e-5), None, ins,
                                          [self._f32(name)])
        self.be.execute(f32_op, [self._f32(src)], [self._f32(name)], stream=self._stream())
        self.scales[q] = self._calibrated(q, name, fixed)
        self.ops[name] = self.be.compile_operator(
            OperatorDef(name, OperatorType.LayerNorm, epsilon=1e-5, rounding=self.rounding), None, ins,
            [self._i8(q, self.scales[q])])

    def forward_device(self):
        """One block forward on the device-resident input buffer ``buf['x']`` (7 launches)."""
        sc = self.scales
        self._run("ln1", [self._f32("x")], [self._i8("q1", sc["q1"])])
        self._run("qkv", [self._i8("q1", sc["q1"])], [self._qkv_out()])
        self._attention(out_i8=self.buf["q2"])
        self._run("out", [self._i8("q2", sc["q2"]), self._f32("x")], [self._f32("h")])
        self._run("ln2", [self._f32("h")], [self._i8("q3", sc["q3"])])
        self._run("ffn_up_i8", [self._i8("q3", sc["q3"])], [self._i8("u", sc["u"])])
        self._run("ffn_down", [self._i8("u", sc["u"]), self._f32("h")], [self._f32("out")])
        return self.buf["out"]

    def capture(self):
        """The forward pass as one CUDA graph (replay after writing buf['x'])."""
        torch = self.torch
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.forward_device()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.forward_device()
        torch.cuda.synchronize(self.device)
        self.graph = g
        return g

    @staticmethod
    def kernel_launches():
        return 7

