"""ResNet-18-shaped INT8 CNN on the CUDA backend.

Network: conv1 7x7/2 (3 -> 64) + BN + ReLU, MaxPool 3x3/2, four stages of two BasicBlocks
(64, 128, 256, 512 channels; the first block of stages 2-4 has stride 2 and a 1x1/2
downsample conv + BN), global average pool, FC-1000.  Weights are He-initialised f32 with
random BatchNorm statistics (gamma ~ U[0.5, 1.5], beta ~ N(0, 0.1), mean ~ N(0, 0.1),
var ~ U[0.5, 1.5]); every conv is compiled through ``CudaBackend.compile_operator`` with its
BN folded and its weights quantized per output channel (INT8 Conv2d with
FusionType::ConvBatchNorm), ReLU fused, and each block's residual Add + ReLU fused into its
second conv's epilogue.  Activations stay int8 NHWC on the device between layers.

Activation scales are calibrated once (``calibrate``): each layer runs with a dequantized f32
output, ``find_scale_zp`` (symmetric) on the device gives its output scale, and the layer runs
again with the requantized int8 output that feeds the next layer.  ``forward`` then runs the
whole network with fixed scales; ``capture`` records it as one CUDA graph.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import _lib
from .backend import (Activation, CudaBackend, DataType, FusionInfo, OperatorDef, OperatorType,
                      Quantization, Rounding, StorageLayout, Tensor)

STEM_CHANNELS = 16  # the 3 input channels stored zero-padded to one 16-byte granule
GOPS_PER_IMAGE = 3.628  # 2 * MACs of ResNet-18 at 224x224 incl. FC (standard stem maxpool)


@dataclass
class ConvSpec:
    name: str
    cin: int
    cout: int
    k: int
    stride: int
    pad: int
    relu: bool
    w: np.ndarray = field(repr=False, default=None)
    bias: np.ndarray = field(repr=False, default=None)
    bn: tuple = field(repr=False, default=None)


def build_params(seed: int = 0, num_classes: int = 1000):
    """Seeded f32 parameters of the network (numpy)."""
    rng = np.random.default_rng(seed)

    def conv(name, cin, cout, k, s, p, relu):
        w = rng.normal(0, np.sqrt(2.0 / (cin * k * k)), size=(cout, cin, k, k)).astype(np.float32)
        bias = np.zeros(cout, np.float32)
        bn = (rng.uniform(0.5, 1.5, cout).astype(np.float32), rng.normal(0, 0.1, cout).astype(np.float32),
              rng.normal(0, 0.1, cout).astype(np.float32), rng.uniform(0.5, 1.5, cout).astype(np.float32))
        return ConvSpec(name, cin, cout, k, s, p, relu, w, bias, bn)

    convs = [conv("conv1", 3, 64, 7, 2, 3, True)]
    blocks = []
    cin = 64
    for stage, cout in enumerate((64, 128, 256, 512), start=1):
        for b in range(2):
            stride = 2 if (stage > 1 and b == 0) else 1
            pre = f"layer{stage}.{b}"
            c1 = conv(pre + ".conv1", cin, cout, 3, stride, 1, True)
            c2 = conv(pre + ".conv2", cout, cout, 3, 1, 1, True)  # ReLU after the residual add
            ds = conv(pre + ".downsample", cin, cout, 1, stride, 0, False) if (stride != 1 or cin != cout) else None
            convs += [c1, c2] + ([ds] if ds else [])
            blocks.append((c1, c2, ds))
            cin = cout
    fc_w = rng.normal(0, np.sqrt(1.0 / 512), size=(num_classes, 512)).astype(np.float32)
    fc_b = rng.normal(0, 0.01, num_classes).astype(np.float32)
    return convs, blocks, fc_w, fc_b


def _out_hw(h, k, s, p):
    return (h + 2 * p - k) // s + 1


def stem_space_to_depth(spec: ConvSpec) -> ConvSpec:
    """The stride-2 stem as a stride-1 conv over the space-to-depth input.

    With the input zero-padded by `pad` and every 2x2 pixel block folded into channels
    (channel (dy*2 + dx)*C + c), tap (r, s) = (2a + dy, 2b + dx) of the original filter moves
    to tap (a, b), channel (dy*2 + dx)*C + c of a ceil(k/2) x ceil(k/2) filter; taps past the
    original k are zero.  The integer sums are unchanged, and BN folding and per-channel
    quantization see the same non-zero weights, so the result is bit-identical."""
    co, c, k, _ = spec.w.shape
    kk = (k + 1) // 2
    w2 = np.zeros((co, 4 * c, kk, kk), np.float32)
    for dy in range(2):
        for dx in range(2):
            for a in range(kk):
                for b in range(kk):
                    r, s = 2 * a + dy, 2 * b + dx
                    if r < k and s < k:
                        w2[:, (dy * 2 + dx) * c:(dy * 2 + dx + 1) * c, a, b] = spec.w[:, :, r, s]
    return ConvSpec(spec.name, 4 * c, spec.cout, kk, 1, 0, spec.relu, w2, spec.bias, spec.bn)


class ResNet18Int8:
    """The network compiled on one device; ``forward`` takes an f32 NCHW batch on that device."""

    def __init__(self, backend: CudaBackend, batch: int, device, image: int = 224, seed: int = 0,
                 rounding: Rounding = Rounding.HalfAwayFromZero, num_classes: int = 1000):
        import torch
        self.torch = torch
        self.be = backend
        self.batch = batch
        self.device = device
        self.image = image
        self.rounding = rounding
        self.convs, self.blocks, self.fc_w, self.fc_b = build_params(seed, num_classes)
        self.num_classes = num_classes
        self.scales: dict = {}
        self.ops: dict = {}
        self.graph = None
        # static activation buffers (int8 NHWC)
        b = batch
        h = _out_hw(image, 7, 2, 3)
        # the stem runs as a stride-1 conv over the space-to-depth input (see stem_space_to_depth)
        self.stem = stem_space_to_depth(self.convs[0])
        hs = (image + 2 * self.convs[0].pad) // 2
        # the space-to-depth input is stored with its width rounded up to a multiple of 4 (a
        # zero column) so the stem conv can run pixel-grouped; the stem crops it again
        ws = (hs + 3) // 4 * 4
        self.stem_extra_cols = ws - hs
        self.buf = {"x_q": torch.empty((b, hs, ws, STEM_CHANNELS), dtype=torch.int8, device=device),
                    "conv1": torch.empty((b, h, h, 64), dtype=torch.int8, device=device)}
        hp = _out_hw(h, 3, 2, 1)
        self.buf["pool"] = torch.empty((b, hp, hp, 64), dtype=torch.int8, device=device)
        self.shapes = {"conv1": (b, h, h, 64), "pool": (b, hp, hp, 64)}
        hh = hp
        for c1, c2, ds in self.blocks:
            ho = _out_hw(hh, 3, c1.stride, 1)
            for spec in (c1, c2) + ((ds,) if ds else ()):
                self.buf[spec.name] = torch.empty((b, ho, ho, spec.cout), dtype=torch.int8, device=device)
                self.shapes[spec.name] = (b, ho, ho, spec.cout)
            hh = ho
        self.final_hw = hh
        self.buf["pooled"] = torch.empty((b, 512), dtype=torch.int8, device=device)
        self.logits = torch.empty((b, num_classes), dtype=torch.float32, device=device)
        self.f32_scratch = torch.empty(max(int(np.prod(s)) for s in self.shapes.values()),
                                       dtype=torch.float32, device=device)
        self.ws = torch.zeros(4, dtype=torch.int32, device=device)
        self._sl = slice(None)  # images of the batch the run methods act on
        self._ds_stream = None  # side stream for the downsample convs while a graph is captured

    # ------------------------------------------------------------------ helpers
    def _buf(self, name):
        """The activation buffer `name`, restricted to the images the current pass runs."""
        return self.buf[name][self._sl]

    def _stream(self):
        return self.torch.cuda.current_stream(self.device).cuda_stream

    def _t(self, name, tensor, dtype, scale=None, layout=StorageLayout.NHWC):
        q = Quantization([float(scale)]) if scale is not None else None
        return Tensor(name, list(tensor.shape), dtype, tensor, layout=layout, quantization=q)

    def _scale_of(self, f32_flat) -> float:
        torch = self.torch
        s = torch.empty(1, dtype=torch.float32, device=self.device)
        z = torch.empty(1, dtype=torch.int32, device=self.device)
        _lib.check(_lib.lib().lsc_find_scale_zp_f32(C.c_void_p(f32_flat.data_ptr()), f32_flat.numel(), 9, 1,
                                                    C.c_void_p(self.ws.data_ptr()), 16, C.c_void_p(s.data_ptr()),
                                                    C.c_void_p(z.data_ptr()), C.c_void_p(self._stream())))
        return float(s.item())

    def _compile_conv(self, spec: ConvSpec, in_name: str, in_scale: float):
        x = self.buf[in_name]
        xt = self._t("x", x, DataType.QInt8, in_scale)
        ins = [xt, Tensor("w", list(spec.w.shape), DataType.F32, spec.w),
               Tensor("b", [spec.cout], DataType.F32, spec.bias)]
        ins += [Tensor(n, [spec.cout], DataType.F32, a) for n, a in zip(("gamma", "beta", "mean", "var"), spec.bn)]
        out = self._t("y", self.buf[spec.name], DataType.QInt8, 1.0)
        crop = self.stem_extra_cols if in_name == "x_q" else 0
        opdef = OperatorDef(spec.name, OperatorType.Conv2d, stride=(spec.stride, spec.stride),
                            padding=(spec.pad, spec.pad), padding_end_delta=(0, -crop),
                            activation=Activation.ReLU if spec.relu else Activation.NONE,
                            rounding=self.rounding, output_scale=1.0)
        return self.be.compile_operator(opdef, FusionInfo.conv_batch_norm(), ins, [out])

    def _run_conv(self, spec, in_name, in_scale, out_scale, residual=None, f32_out=None):
        ins = [self._t("x", self._buf(in_name), DataType.QInt8, in_scale)]
        if residual is not None:
            rname, rscale = residual
            ins.append(self._t("r", self._buf(rname), DataType.QInt8, rscale))
        if f32_out is not None:
            outs = [self._t("y", f32_out, DataType.F32)]
        else:
            outs = [self._t("y", self._buf(spec.name), DataType.QInt8, out_scale)]
        self.be.execute(self.ops[spec.name], ins, outs, stream=self._stream())

    # ------------------------------------------------------------------ calibration
    def calibrate(self, x_f32):
        """Compiles every layer and fixes its output scale from this batch (f32 NCHW, device)."""
        torch = self.torch
        assert tuple(x_f32.shape) == (self.batch, 3, self.image, self.image)
        s_in = self._scale_of(x_f32.reshape(-1))
        self.scales["input"] = s_in
        qin = Tensor("xq", list(self.buf["x_q"].shape), DataType.QInt8, self.buf["x_q"],
                     layout=StorageLayout.NHWC, quantization=Quantization([s_in]))
        xt = Tensor("x", list(x_f32.shape), DataType.F32, x_f32, layout=StorageLayout.NCHW)
        pad = self.convs[0].pad
        self.ops["quant_in"] = self.be.compile_operator(
            OperatorDef("quantize_input", OperatorType.Quantize, rounding=self.rounding, stride=(2, 2),
                        padding=(pad, pad), padding_end_delta=(0, 2 * self.stem_extra_cols)), None, [xt], [qin])
        self.be.execute(self.ops["quant_in"], [xt], [qin], stream=self._stream())

        def layer(spec, in_name, residual=None):
            in_scale = self.scales[in_name] if in_name != "x_q" else s_in
            self.ops[spec.name] = self._compile_conv(spec, in_name, in_scale)
            shape = self.shapes[spec.name]
            f32 = self.f32_scratch[: int(np.prod(shape))].view(shape)
            self._run_conv(spec, in_name, in_scale, None, residual, f32_out=f32)
            self.scales[spec.name] = self._scale_of(f32.reshape(-1))
            self._run_conv(spec, in_name, in_scale, self.scales[spec.name], residual)

        layer(self.stem, "x_q")
        self._compile_pool()
        self._run_pool()
        self.scales["pool"] = self.scales["conv1"]
        prev = "pool"
        for c1, c2, ds in self.blocks:
            layer(c1, prev)
            if ds is not None:
                layer(ds, prev)
                res = (ds.name, self.scales[ds.name])
            else:
                res = (prev, self.scales[prev])
            layer(c2, c1.name, residual=res)
            prev = c2.name
        self.last = prev
        # global average pool: calibrate its int8 output from the f32 means
        gap = OperatorDef("gap", OperatorType.GlobalAvgPool2d, rounding=self.rounding, output_scale=1.0)
        xin = self._t("x", self.buf[prev], DataType.QInt8, self.scales[prev])
        pooled_f32 = self.f32_scratch[: self.batch * 512].view(self.batch, 512)
        self.ops["gap"] = self.be.compile_operator(gap, None, [xin], [self._t("y", pooled_f32, DataType.F32)])
        self.be.execute(self.ops["gap"], [xin], [self._t("y", pooled_f32, DataType.F32)], stream=self._stream())
        self.scales["pooled"] = self._scale_of(pooled_f32.reshape(-1))
        self._run_gap()
        # FC-1000: INT8 FullyConnected, per-channel weights, f32 logits
        pin = Tensor("p", [self.batch, 512], DataType.QInt8, self.buf["pooled"],
                     quantization=Quantization([self.scales["pooled"]]))
        self.ops["fc"] = self.be.compile_operator(
            OperatorDef("fc", OperatorType.FullyConnected, rounding=self.rounding), None,
            [pin, Tensor("w", list(self.fc_w.shape), DataType.F32, self.fc_w),
             Tensor("b", [self.num_classes], DataType.F32, self.fc_b)],
            [Tensor("logits", list(self.logits.shape), DataType.F32, self.logits)])
        self._run_fc()
        torch.cuda.synchronize(self.device)

    def _compile_pool(self):
        xin = self._t("x", self.buf["conv1"], DataType.QInt8, self.scales["conv1"])
        opdef = OperatorDef("maxpool", OperatorType.MaxPool2d, stride=(2, 2), padding=(1, 1), kernel=(3, 3))
        self.ops["maxpool"] = self.be.compile_operator(opdef, None, [xin], [self._t("y", self.buf["pool"], DataType.QInt8)])

    def _run_pool(self):
        self.be.execute(self.ops["maxpool"], [self._t("x", self._buf("conv1"), DataType.QInt8)],
                        [self._t("y", self._buf("pool"), DataType.QInt8)], stream=self._stream())

    def _run_gap(self):
        self.be.execute(self.ops["gap"], [self._t("x", self._buf(self.last), DataType.QInt8, self.scales[self.last])],
                        [self._t("y", self._buf("pooled"), DataType.QInt8, self.scales["pooled"])],
                        stream=self._stream())

    def _run_fc(self):
        pooled, logits = self._buf("pooled"), self.logits[self._sl]
        pin = Tensor("p", list(pooled.shape), DataType.QInt8, pooled, quantization=Quantization([self.scales["pooled"]]))
        self.be.execute(self.ops["fc"], [pin], [Tensor("logits", list(logits.shape), DataType.F32, logits)],
                        stream=self._stream())

    # ------------------------------------------------------------------ inference
    def forward(self, x_f32):
        """Runs the calibrated network on an f32 NCHW device batch; returns the logits buffer."""
        x_f32 = x_f32[self._sl]
        xt = Tensor("x", list(x_f32.shape), DataType.F32, x_f32, layout=StorageLayout.NCHW)
        x_q = self._buf("x_q")
        qin = Tensor("xq", list(x_q.shape), DataType.QInt8, x_q,
                     layout=StorageLayout.NHWC, quantization=Quantization([self.scales["input"]]))
        self.be.execute(self.ops["quant_in"], [xt], [qin], stream=self._stream())
        sc = self.scales
        self._run_conv(self.stem, "x_q", sc["input"], sc["conv1"])
        self._run_pool()
        prev = "pool"
        torch = self.torch
        for c1, c2, ds in self.blocks:
            side = self._ds_stream if ds is not None else None
            if side is not None:
                # the downsample reads the block input as conv1 does: run it beside conv1
                cur = torch.cuda.current_stream(self.device)
                side.wait_stream(cur)
                with torch.cuda.stream(side):
                    self._run_conv(ds, prev, sc[prev], sc[ds.name])
            self._run_conv(c1, prev, sc[prev], sc[c1.name])
            if ds is not None:
                if side is not None:
                    cur.wait_stream(side)
                else:
                    self._run_conv(ds, prev, sc[prev], sc[ds.name])
                res = (ds.name, sc[ds.name])
            else:
                res = (prev, sc[prev])
            self._run_conv(c2, c1.name, sc[c1.name], sc[c2.name], residual=res)
            prev = c2.name
        self._run_gap()
        self._run_fc()
        return self.logits

    def kernel_launches(self) -> int:
        """Kernels per forward: input quantize + 20 convs + maxpool + avgpool + FC."""
        return 1 + len(self.convs) + 1 + 1 + 1

    def capture(self, x_static, branches: int = 1, concurrent_downsample: bool = False):
        """Records ``forward(x_static)`` as a CUDA graph (call after ``calibrate``).

        With ``branches`` > 1 the batch is cut into that many equal groups of images, each run
        through the whole network on its own stream inside the graph (forked from and joined
        back to the capturing stream).  Every image's computation is independent of the others
        once the activation scales are fixed, so the logits are the same; the groups' kernels
        overlap, which fills the SMs that one small batch's kernels leave idle.  With
        ``concurrent_downsample`` each stage's 1x1 downsample conv runs on a side stream beside
        the block's first conv (both read the block input; the second conv joins them)."""
        torch = self.torch
        if branches < 1 or self.batch % branches:
            raise ValueError(f"batch {self.batch} does not split into {branches} branches")
        per = self.batch // branches
        slices = [slice(k * per, (k + 1) * per) for k in range(branches)]
        g = torch.cuda.CUDAGraph()
        ds_streams = [torch.cuda.Stream(self.device) if concurrent_downsample else None for _ in slices]
        try:
            # warm: every kernel variant (tile widths follow the group size) initialised first
            for sl in slices:
                self._sl = sl
                self.forward(x_static)
            self._sl = slice(None)
            torch.cuda.synchronize(self.device)
            if branches == 1:
                with torch.cuda.graph(g):
                    self._ds_stream = ds_streams[0]
                    self.forward(x_static)
            else:
                side = [torch.cuda.Stream(self.device) for _ in slices]
                with torch.cuda.graph(g):
                    main = torch.cuda.current_stream(self.device)
                    for sl, st, dst in zip(slices, side, ds_streams):
                        st.wait_stream(main)
                        with torch.cuda.stream(st):
                            self._sl, self._ds_stream = sl, dst
                            self.forward(x_static)
                    for st in side:
                        main.wait_stream(st)
        finally:
            self._sl, self._ds_stream = slice(None), None
        self.graph = g
        return g
