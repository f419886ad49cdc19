"""Benchmark of the CUDA backend on the headline workloads.

Default workload -- ResNet-18-shaped INT8 CNN, batch 256 split evenly over the GPUs:
conv1 7x7/2, four stages of BasicBlocks (64/128/256/512), global average pool, FC-1000;
He-initialised weights with random BatchNorm statistics, BN folded, weights INT8 per output
channel, ReLU and each block's residual Add+ReLU fused, activations int8 NHWC; input
224x224x3 ~ N(0, 1) (seeded synthetic data; no dataset).  Activation scales are calibrated
once on the first per-rank batch; the network then runs as one captured CUDA graph.

* ``value``: whole-job images per second: 256 / (max over ranks of the per-step device time).
  Each step is one graph replay of the rank's shard, timed with CUDA events on the launching
  stream; the L2 is flushed (256 MiB write) before every timed step.
* ``e2e``: the same through the host boundary: each step copies the rank's f32 input shard
  from pinned host memory (``lsc_memcpy_h2d``), runs the network and copies the logits back
  (``lsc_memcpy_d2h``).
* ``roofline``: tensor-bound; the dominant kernel is the INT8 implicit-GEMM convolution
  (``contraction_i8_kernel``).  achieved = algorithmic conv ops per image x images / summed
  conv-kernel time (events around every conv launch of one eager pass); peak = 2 x the
  measured bf16 burst peak (dense INT8 issues at twice the bf16 rate).
* ``int8_gemm_4096`` (rank 0): the INT8 per-channel GEMM M=N=K=4096 with int32 bias, in TOPS
  with its own roofline fraction: the requantized int8 output (half-even) is the value; the
  dequantized f32 output and both outputs from one launch are listed under ``variants``.
* ``cpu_baseline`` (rank 0, one GPU): the oracle's restatement of the same quantized network
  on the host cores (direct convolutions, OpenMP) on a bounded sample of images.

Multi-GPU: one rank per GPU (torchrun), each holding its own weights; no collective touches
the data path (NCCL is used only for barriers and the max-over-ranks timing reduction).

``--impl reference`` times the reference's CPU path (the oracle port; the Rust reference
cannot be built here) on the host cores, rank 0 only, and prints the same metric.
``--workload gemm`` makes the 4096^3 INT8 GEMM (TOPS) the headline instead; ``--workload bert``
the BERT-base encoder block (sequences/s, batch 32 x seq 384 split over the GPUs), which the
default line also carries on rank 0 as ``bert_block``.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "INT8 conv/GEMM TOPS (% peak); ResNet-18 INT8 img/s at 1/2/4/8 B200"
GLOBAL_BATCH = 256
IMAGE = 224
NET_SEED = 20260415
DATA_SEED = 1234
GEMM_M = GEMM_N = GEMM_K = 4096
GEMM_OPS = 2 * GEMM_M * GEMM_N * GEMM_K
GEMM_WORKLOAD = ("int8 per-channel GEMM M=N=K=4096, int32 bias, requant int8 (half-even); dequant f32 "
                 "variant alongside")
BERT_BATCH, BERT_SEQ, BERT_SEED = 32, 384, 20260501
BERT_WORKLOAD = ("BERT-base encoder block (pre-LN, hidden 768, 12 heads x 64, FFN 3072 GELU), seq 384, batch 32 "
                 "split over the GPUs; INT8 per-channel projections, FP16 attention")
RESNET_WORKLOAD = ("ResNet-18 INT8 (conv1 7x7/2, 4 BasicBlock stages 64/128/256/512, maxpool 3x3/2, "
                   "global avgpool, FC-1000), 224x224x3 input, batch 256 split over the GPUs")


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def load_traffic(profile):
    """dram bytes per launch of the profiled kernel from a committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", profile)
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    return int(line.split(":", 1)[1].strip())
                except ValueError:
                    return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_uuid):
        self.path = tempfile.mktemp(prefix="lsc_clocks_", suffix=".csv")
        self.proc = None
        self.uuid = device_uuid

    def start(self):
        try:
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(cmd, stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 8:
                    continue
                try:
                    rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        loaded = [r for r in rows if r[2] > 300.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3][1:5]) if v == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(loaded)}


def network_conv_ops(model):
    """{conv name: ops per image} from the model's activation shapes."""
    ops = {}
    for spec in model.convs:
        _, oh, ow, _ = model.shapes[spec.name]
        ops[spec.name] = 2 * spec.cout * oh * ow * spec.k * spec.k * spec.cin
    return ops


# --------------------------------------------------------------------------- CPU side
def host_threads():
    """Every host core this process may run on.  Passed explicitly to the CPU legs so that a
    launcher's OMP_NUM_THREADS (torchrun sets 1 per rank) cannot shrink the CPU baseline."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_resnet_sample(images, scales=None, threads=None):
    """The reference CPU path (oracle port) on `images` images; returns (seconds, logits)."""
    from lightship_b200.resnet18 import build_params
    from oracle import oracle as orc
    convs, blocks, fw, fb = build_params(NET_SEED)
    rng = np.random.default_rng(DATA_SEED)
    x = rng.normal(size=(images, 3, IMAGE, IMAGE)).astype(np.float32)
    t0 = time.perf_counter()
    logits, sc, _ = orc.resnet18_int8(x, convs, blocks, fw, fb, scales, 0, threads or host_threads())
    return time.perf_counter() - t0, logits, sc


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.workload == "gemm":
        return run_reference_gemm(args)
    if args.workload == "bert":
        return run_reference_bert(args)
    # calibrate once on two images, then size each step to about two minutes in total
    _, _, scales = cpu_resnet_sample(2)
    t1, _, _ = cpu_resnet_sample(1, scales)
    budget = 120.0 / max(1, args.steps + args.warmup)
    images = int(max(1, min(GLOBAL_BATCH, budget / max(t1, 1e-6))))
    for _ in range(args.warmup):
        cpu_resnet_sample(images, scales)
    times = [cpu_resnet_sample(images, scales)[0] for _ in range(args.steps)]
    t = sum(times) / len(times)
    value = images / t
    line = {"metric": METRIC, "value": value, "unit": "img/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": RESNET_WORKLOAD, "images_per_step": images},
            "cpu_baseline": {"value": value, "unit": "img/s", "cores": host_threads(), "kind": "port",
                             "sample": f"{images} images per step through the oracle's quantized ResNet-18 "
                                       "(direct int8 convolutions, OpenMP)"},
            "e2e": {"value": value, "unit": "img/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def gemm_inputs():
    rng = np.random.default_rng(NET_SEED)
    a = rng.integers(-127, 128, size=(GEMM_M, GEMM_K), dtype=np.int8)
    w = rng.integers(-127, 128, size=(GEMM_N, GEMM_K), dtype=np.int8)
    scale = rng.uniform(0.001, 0.02, size=GEMM_N).astype(np.float32)
    bias = rng.integers(-100000, 100000, size=GEMM_N, dtype=np.int32)
    return a, w, scale, bias


def cpu_gemm_rows(rows, a, w_kn, bias, scale, s_out):
    """The reference CPU chain on rows [0, rows) of A: NN triple loop then the epilogue."""
    from oracle import oracle as orc
    t0 = time.perf_counter()
    acc = orc.gemm_i8_nn(a[:rows], w_kn, host_threads())
    orc.requant(acc, bias, scale, orc.ACT_NONE, s_out, orc.ROUND_HALF_EVEN)
    return time.perf_counter() - t0


def run_reference_gemm(args):
    a, w, scale, bias = gemm_inputs()
    w_kn = np.ascontiguousarray(w.T)
    per_row = cpu_gemm_rows(16, a, w_kn, bias, scale, 40.0) / 16
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = int(max(8, min(GEMM_M, budget / max(per_row, 1e-9))))
    for _ in range(args.warmup):
        cpu_gemm_rows(rows, a, w_kn, bias, scale, 40.0)
    t = sum(cpu_gemm_rows(rows, a, w_kn, bias, scale, 40.0) for _ in range(args.steps)) / args.steps
    value = 2 * rows * GEMM_N * GEMM_K / t / 1e12
    line = {"metric": METRIC, "value": value, "unit": "TOPS", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": GEMM_WORKLOAD, "sample_rows_per_step": rows},
            "cpu_baseline": {"value": value, "unit": "TOPS", "cores": host_threads(), "kind": "port",
                             "sample": f"rows 0..{rows - 1} of A per step, reference loop order, OpenMP over M"},
            "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def cpu_bert_sample(seqs, scales=None, threads=None):
    """The oracle's quantized encoder block on `seqs` sequences of 384 tokens; returns seconds
    and the scales (calibrated from this sample when none are given)."""
    from lightship_b200.bert import HIDDEN, build_params
    from oracle import oracle as orc
    p = build_params(BERT_SEED)
    threads = threads or host_threads()
    x = np.random.default_rng(DATA_SEED).standard_normal((seqs * BERT_SEQ, HIDDEN)).astype(np.float32)
    if scales is None:
        scales = {"q1": 1.0, "q2": 1.0, "q3": 1.0, "u": 1.0}
        for q, src in (("q1", "ln1"), ("q2", "o"), ("q3", "ln2")):
            scales[q] = orc.find_scale_zp(orc.encoder_block_int8(x, p, scales, seqs, BERT_SEQ, threads=threads)[src])[0]
        q3 = orc.encoder_block_int8(x, p, scales, seqs, BERT_SEQ, threads=threads)["q3"]
        uf = orc.fc_i8_f32_weights(q3, scales["q3"], p["w1"], p["b1"], orc.ACT_GELU, 1.0, threads=threads)[1]
        scales["u"] = orc.find_scale_zp(uf)[0]
    t0 = time.perf_counter()
    orc.encoder_block_int8(x, p, scales, seqs, BERT_SEQ, threads=threads)
    return time.perf_counter() - t0, scales


def run_reference_bert(args):
    _, scales = cpu_bert_sample(1)
    t1, _ = cpu_bert_sample(1, scales)
    budget = 120.0 / max(1, args.steps + args.warmup)
    seqs = int(max(1, min(BERT_BATCH, budget / max(t1, 1e-6))))
    for _ in range(args.warmup):
        cpu_bert_sample(seqs, scales)
    times = [cpu_bert_sample(seqs, scales)[0] for _ in range(args.steps)]
    t = sum(times) / len(times)
    value = seqs / t
    line = {"metric": METRIC, "value": value, "unit": "sequences/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8+f16", "data": "synthetic",
            "config": {"workload": BERT_WORKLOAD, "sequences_per_step": seqs},
            "cpu_baseline": {"value": value, "unit": "sequences/s", "cores": host_threads(), "kind": "port",
                             "sample": f"{seqs} sequences of 384 tokens per step through the oracle's quantized "
                                       "encoder block (INT8 projections, f32 attention with f16 rounding points)"},
            "e2e": {"value": value, "unit": "sequences/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- GPU side
def bert_measure(torch, dev, batch, steps, warmup, be):
    """The encoder block for `batch` sequences of 384 on this device.

    Returns a dict: the graph-replayed block time (L2 flushed before every step), the per-stage
    breakdown of one eager pass (events around each launch, queued behind a device sleep),
    the INT8 projection kernels' TOPS, and the end-to-end time with the f32 input copied from
    pinned host memory and the f32 output copied back every step."""
    from lightship_b200 import _lib
    from lightship_b200.bert import HIDDEN, INT8_OPS_PER_TOKEN, BertBlockInt8, attention_flops
    blk = BertBlockInt8(be, batch, BERT_SEQ, dev, seed=BERT_SEED)
    x = np.random.default_rng(DATA_SEED).standard_normal((batch * BERT_SEQ, HIDDEN)).astype(np.float32)
    x_host = torch.from_numpy(x).pin_memory()
    blk.calibrate(x_host.to(dev))
    stream = torch.cuda.current_stream(dev)
    evs = {}

    def wrap(fn, name_of):
        def run(*a, **k):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn(*a, **k)
            e.record(stream)
            evs.setdefault(name_of(a), []).append((s, e))
        return run

    orig_run, orig_att = blk._run, blk._attention
    blk._run = wrap(orig_run, lambda a: a[0])
    blk._attention = wrap(orig_att, lambda a: "attention")
    for _ in range(3):
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(20_000_000)
        blk.forward_device()
    torch.cuda.synchronize(dev)
    blk._run, blk._attention = orig_run, orig_att
    stage = {k: float(np.mean([s.elapsed_time(e) for s, e in v])) for k, v in evs.items()}
    tokens = batch * BERT_SEQ
    gemm_ms = sum(stage[k] for k in ("qkv", "out", "ffn_up_i8", "ffn_down"))
    gemm_tops = INT8_OPS_PER_TOKEN * tokens / (gemm_ms * 1e-3) / 1e12

    graph = blk.capture()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(warmup):
        flush.zero_()
        graph.replay()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize(dev)
    for s, e in ev:
        flush.zero_()
        s.record(stream)
        graph.replay()
        e.record(stream)
    torch.cuda.synchronize(dev)
    ms = float(np.mean([s.elapsed_time(e) for s, e in ev]))

    lib = _lib.lib()
    out_host = torch.empty((tokens, HIDDEN), dtype=torch.float32).pin_memory()
    nbytes = tokens * HIDDEN * 4
    sptr = C.c_void_p(stream.cuda_stream)

    def e2e_step():
        _lib.check(lib.lsc_memcpy_h2d(C.c_void_p(blk.buf["x"].data_ptr()), C.c_void_p(x_host.data_ptr()), nbytes,
                                      sptr))
        graph.replay()
        _lib.check(lib.lsc_memcpy_d2h(C.c_void_p(out_host.data_ptr()), C.c_void_p(blk.buf["out"].data_ptr()),
                                      nbytes, sptr))

    e2e_steps = max(3, min(steps, 20))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    ee.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = es.elapsed_time(ee) / e2e_steps
    e2e_ok = bool(torch.equal(out_host, blk.buf["out"].cpu()))
    del graph
    blk.graph = None
    return {"ms": ms, "stage_ms": stage, "gemm_ms": gemm_ms, "gemm_tops": gemm_tops,
            "attention_tflops": attention_flops(batch, BERT_SEQ) / (stage["attention"] * 1e-3) / 1e12,
            "e2e_ms": e2e_ms, "bytes": nbytes, "e2e_ok": e2e_ok, "scales": dict(blk.scales),
            "launches": blk.kernel_launches()}


def gemm_measure(torch, dev, steps, warmup):
    """The 4096^3 INT8 chain on this device, timed per output variant.

    Returns {variant: (TOPS, ms per launch)} for "i8" (bias + requantized int8, half-even:
    the headline), "f32" (bias + dequantized f32) and "i8+f32" (both from one launch), plus
    the calibrated s_out.  Every timed launch follows an L2 flush (256 MiB write); the launches
    are queued behind a short device sleep so host-side launch latency is not timed."""
    from lightship_b200 import _lib
    lib = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)
    a, w, scale, bias = gemm_inputs()
    ta, tw = torch.from_numpy(a).to(dev), torch.from_numpy(w).to(dev)
    ts, tb = torch.from_numpy(scale).to(dev), torch.from_numpy(bias).to(dev)
    q = torch.empty((GEMM_M, GEMM_N), dtype=torch.int8, device=dev)
    y = torch.empty((GEMM_M, GEMM_N), dtype=torch.float32, device=dev)
    ws = torch.zeros(4, dtype=torch.int32, device=dev)
    s_dev = torch.empty(1, dtype=torch.float32, device=dev)
    z_dev = torch.empty(1, dtype=torch.int32, device=dev)
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    _lib.check(lib.lsc_gemm_i8(P(ta), P(tw), GEMM_M, GEMM_N, GEMM_K, P(tb), P(ts), 1.0, 0, 1, None, P(y), None, sptr))
    _lib.check(lib.lsc_find_scale_zp_f32(P(y), GEMM_M * GEMM_N, 9, 1, P(ws), 16, P(s_dev), P(z_dev), sptr))
    s_out = float(s_dev.item())
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    res = {}
    for name, oq, oy in (("i8", q, None), ("f32", None, y), ("i8+f32", q, y)):
        def launch():
            _lib.check(lib.lsc_gemm_i8(P(ta), P(tw), GEMM_M, GEMM_N, GEMM_K, P(tb), P(ts), s_out, 0, 1, P(oq), P(oy),
                                       None, sptr))
        for _ in range(warmup):
            flush.zero_()
            launch()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(20_000_000)
        for s, e in ev:
            flush.zero_()
            s.record(stream)
            launch()
            e.record(stream)
        torch.cuda.synchronize(dev)
        ms = float(np.mean([s.elapsed_time(e) for s, e in ev]))
        res[name] = (GEMM_OPS / (ms * 1e-3) / 1e12, ms)
    return res, s_out


def vendor_gemm_measure(torch, dev, steps, warmup):
    """Library yardsticks on the same box, same L2 flush: cuBLASLt's INT8 GEMM through
    torch._int_mm at 4096^3 (int32 output, no epilogue: it writes 64 MB where the INT8 chain
    writes 16 MB of int8) and cuBLAS bf16 at 4096^3.  Returns {name: (TOPS, ms)}."""
    g = torch.Generator(device=dev).manual_seed(NET_SEED)
    a = torch.randint(-127, 128, (GEMM_M, GEMM_K), dtype=torch.int8, device=dev, generator=g)
    w = torch.randint(-127, 128, (GEMM_N, GEMM_K), dtype=torch.int8, device=dev, generator=g)
    ab, wb = a.to(torch.bfloat16), w.to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    res = {}
    for name, fn in (("cublaslt_int8_int_mm", lambda: torch._int_mm(a, w.t())),
                     ("cublas_bf16_matmul", lambda: torch.matmul(ab, wb.t()))):
        try:
            for _ in range(warmup):
                flush.zero_()
                fn()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            torch.cuda.synchronize(dev)
            torch.cuda._sleep(20_000_000)
            for s_, e_ in ev:
                flush.zero_()
                s_.record(stream)
                fn()
                e_.record(stream)
            torch.cuda.synchronize(dev)
            ms = float(np.mean([s_.elapsed_time(e_) for s_, e_ in ev]))
            res[name] = (GEMM_OPS / (ms * 1e-3) / 1e12, ms)
        except Exception as exc:  # a library without the kernel on this build
            res[name] = (None, repr(exc)[:120])
    return res


def tensor_rate_probe():
    """tcgen05.mma issue rate on resident shared-memory operands (lsc_probe_tensor_rate), on
    every SM at once: {shape: {cycles, ns, TOPS (whole GPU)}}."""
    from lightship_b200 import _lib
    lib = _lib.lib()
    out = {}
    for kind, kname in ((0, "i8"), (1, "f16")):
        for pair in (0, 1):
            for n in (64, 128, 256):
                cyc, ns = C.c_double(), C.c_double()
                st = lib.lsc_probe_tensor_rate(kind, n, pair, 8192, 148, 0, 0, 0, C.byref(cyc), C.byref(ns))
                if st:
                    out[f"{kname}_m{256 if pair else 128}_n{n}"] = {"error": _lib.last_error()}
                    continue
                m = 256 if pair else 128
                k = 32 if kind == 0 else 16
                units = 74 if pair else 148
                ops = 2.0 * m * n * k * units / (ns.value * 1e-9) / 1e12
                out[f"{kname}_m{m}_n{n}"] = {"cycles_per_mma": round(cyc.value, 1), "ns_per_mma": round(ns.value, 2),
                                            "tops_all_sms": round(ops, 1)}
    return out


def pipeline_probes(torch, dev):
    """What bounds a pipelined contraction kernel, one factor at a time (lsc_probe_tensor_rate
    with a stage-release cadence, lsc_probe_tma_rate for operand delivery)."""
    from lightship_b200 import _lib
    lib = _lib.lib()
    out = {"mma_issue_loop": {}, "tma": {}}
    cases = [(0, 0, 0), (1, 0, 0), (1, 4, 0), (1, 4, 6), (2, 4, 0), (2, 4, 2), (2, 4, 6), (3, 4, 0), (3, 4, 6),
             (4, 4, 6)]
    for pair, n in ((0, 64), (0, 128), (0, 256), (1, 256)):
        for mode, ce, lag in cases:
            cyc, ns = C.c_double(), C.c_double()
            st = lib.lsc_probe_tensor_rate(0, n, pair, 8192, 148, mode, ce, lag, C.byref(cyc), C.byref(ns))
            key = f"i8_m{256 if pair else 128}_n{n}_mode{mode}_commit{ce}_lag{lag}"
            out["mma_issue_loop"][key] = (round(cyc.value, 1) if st == 0 else _lib.last_error())
    if os.environ.get("LSC_PROBE_MMA_ONLY"):
        return out
    for n, h in ((256, 14), (256, 56), (32, 7)):
        buf = torch.ones(n * h * h * 128, dtype=torch.uint8, device=dev)
        for depth, prods in ((2, 1), (3, 1), (2, 2), (2, 4), (3, 4)):
            bpc, gbs = C.c_double(), C.c_double()
            st = lib.lsc_probe_im2col_rate(C.c_void_p(buf.data_ptr()), n, h, h, depth, prods, 4096, 148,
                                           C.byref(bpc), C.byref(gbs))
            out["tma"][f"im2col_n{n}_h{h}_producers{prods}_depth{depth}"] = (
                {"B_per_clk_per_sm": round(bpc.value, 1), "GB_s": round(gbs.value)} if st == 0 else _lib.last_error())
        del buf
    return out


# ResNet-18 convolution shapes (name, batch-256 input H, C_in, C_out, k, stride, residual)
CONV_SHAPES = [("layer1.conv", 56, 64, 64, 3, 1, True), ("layer2.0.conv1", 56, 64, 128, 3, 2, False),
               ("layer2.conv", 28, 128, 128, 3, 1, True), ("layer3.conv", 14, 256, 256, 3, 1, True),
               ("layer4.conv", 7, 512, 512, 3, 1, True), ("layer4.0.downsample", 14, 256, 512, 1, 2, False)]


def conv_measure(torch, dev, batch, steps, warmup, only=()):
    """Each ResNet-18 convolution shape alone through lsc_conv2d_i8_nhwc (ReLU, requantized int8
    output, the block's int8 residual where it has one), L2 flushed before every launch:
    {name: (us per launch, TOPS)}."""
    from lightship_b200 import ops
    g = torch.Generator(device=dev).manual_seed(7)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    out = {}
    for name, h, ci, co, k, st, res in CONV_SHAPES:
        if only and name not in only:
            continue
        x = torch.randint(-127, 128, (batch, h, h, ci), dtype=torch.int8, device=dev, generator=g)
        w = torch.randint(-127, 128, (co, k, k, ci), dtype=torch.int8, device=dev, generator=g)
        scale = torch.full((co,), 1e-4, dtype=torch.float32, device=dev)
        pad = k // 2
        ho = (h + 2 * pad - k) // st + 1
        r = torch.randint(-127, 128, (batch, ho, ho, co), dtype=torch.int8, device=dev, generator=g) if res else None

        def launch():
            ops.conv2d_i8_nhwc(x, w, scale, None, stride=(st, st), pad=(pad, pad), s_out=0.05, act=1,
                               residual=r, residual_scale=0.02)
        for _ in range(warmup):
            flush.zero_()
            launch()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(20_000_000)
        for s_, e_ in ev:
            flush.zero_()
            s_.record(stream)
            launch()
            e_.record(stream)
        torch.cuda.synchronize(dev)
        us = 1e3 * float(np.mean([s_.elapsed_time(e_) for s_, e_ in ev]))
        ops_n = 2.0 * batch * ho * ho * co * k * k * ci
        out[name] = (round(us, 2), round(ops_n / (us * 1e-6) / 1e12, 1))
    return out


def auto_branches(per_gpu_batch):
    """Concurrent image groups for a per-GPU ResNet batch.  Measured on B200 (graph step time,
    batch 32 / 64 / 128 / 256): two groups 322 / 450 / 676 / 1132 us against one chain's
    299 / 411 / 666 / 1151 us, four groups at batch 32 362 us; one chain is kept."""
    return 1


def shard_bounds(batch, world, rank):
    """The contiguous slice [lo, hi) of the global batch that rank owns (batch % world == 0)."""
    if batch % world:
        raise ValueError(f"batch {batch} does not split over {world} ranks")
    per = batch // world
    return rank * per, (rank + 1) * per


def reduce_max(v, world, device=None):
    """Max of a per-rank float over the process group (the step time every rank reports)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_gpu(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def max_over_ranks(v):
        return reduce_max(v, world, dev)

    def barrier():
        if world > 1:
            dist.barrier()

    from lightship_b200 import _lib, ops
    bf16_peak, peak_src = load_peaks()
    int8_peak = 2.0 * bf16_peak
    peak_source = f"2 x {peak_src} bf16 burst ({bf16_peak} TFLOP/s); nominal dense INT8 4500 TOPS"
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass

    if args.workload == "gemm":
        sampler = ClockSampler(uuid)
        sampler.start()
        barrier()
        variants, s_out = gemm_measure(torch, dev, args.steps, args.warmup)
        tops, ms = variants["i8"]
        barrier()
        clocks = sampler.stop()
        ms_max = max_over_ranks(ms)
        line = {"metric": METRIC, "value": world * GEMM_OPS / (ms_max * 1e-3) / 1e12, "unit": "TOPS",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic",
                "config": {"workload": GEMM_WORKLOAD, "parallelism": f"replicas x{world}",
                           "l2": "flushed (256 MiB write) before every timed launch"},
                "roofline": {"bound": "tensor", "achieved": tops, "peak": int8_peak, "unit": "TOPS",
                             "frac": tops / int8_peak, "traffic": load_traffic("contraction_i8_gemm_4096.md"),
                             "peak_source": peak_source},
                "variants": {k: {"TOPS": v[0], "ms_per_launch": v[1], "roofline_frac": v[0] / int8_peak}
                             for k, v in variants.items()},
                "gpu_launches": 3 * args.steps, "clocks": clocks}
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(line), flush=True)
        return 0

    if args.workload == "conv":
        if rank == 0:
            only = tuple(args.only.split(",")) if args.only else ()
            res = {"batch": args.batch, "conv": conv_measure(torch, dev, args.batch, args.steps, args.warmup, only)}
            if not only:
                res["gemm_4096"] = {k: (round(v[1] * 1e3, 2), round(v[0], 1))
                                    for k, v in gemm_measure(torch, dev, args.steps, args.warmup)[0].items()}
            print(json.dumps(res), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0

    if args.workload == "probe":
        if rank == 0:
            print(json.dumps({"tensor_rate_probe": tensor_rate_probe(), "pipeline": pipeline_probes(torch, dev)}),
                  flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0

    if args.workload == "bert":
        from lightship_b200.backend import CudaBackend, GpuBackendConfig
        if BERT_BATCH % world:
            raise SystemExit(f"batch {BERT_BATCH} does not split over {world} GPUs")
        per = BERT_BATCH // world
        be = CudaBackend(GpuBackendConfig(device_id=local, arena_bytes=64 << 20))
        sampler = ClockSampler(uuid)
        sampler.start()
        barrier()
        r = bert_measure(torch, dev, per, args.steps, args.warmup, be)
        barrier()
        clocks = sampler.stop()
        ms_max = max_over_ranks(r["ms"])
        e2e_max = max_over_ranks(r["e2e_ms"])
        line = {"metric": METRIC, "value": BERT_BATCH / (ms_max * 1e-3), "unit": "sequences/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8+f16", "data": "synthetic",
                "config": {"workload": BERT_WORKLOAD, "global_batch": BERT_BATCH, "per_gpu_batch": per,
                           "seq_len": BERT_SEQ, "parallelism": f"batch split x{world} (no collective)",
                           "l2": "flushed (256 MiB write) before every timed step"},
                "roofline": {"bound": "tensor", "kernel": "contraction_i8_kernel (QKV/out/FFN projections)",
                             "achieved": r["gemm_tops"], "peak": int8_peak, "unit": "TOPS",
                             "frac": r["gemm_tops"] / int8_peak, "traffic": None, "peak_source": peak_source,
                             "projection_share_of_step": r["gemm_ms"] / r["ms"]},
                "stage_ms": r["stage_ms"], "attention_tflops": r["attention_tflops"],
                "e2e": {"value": BERT_BATCH / (e2e_max * 1e-3), "unit": "sequences/s",
                        "h2d_bytes_per_step": r["bytes"] * world, "d2h_bytes_per_step": r["bytes"] * world,
                        "api": "lsc_memcpy_h2d + block graph + lsc_memcpy_d2h", "matches_device_run": r["e2e_ok"]},
                "gpu_launches": r["launches"] * args.steps, "clocks": clocks}
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            seqs = 16
            dt, _ = cpu_bert_sample(seqs, r["scales"])
            line["cpu_baseline"] = {"value": seqs / dt, "unit": "sequences/s", "cores": host_threads(),
                                    "kind": "port", "sample": f"{seqs} sequences of 384 tokens through the "
                                                              f"oracle's quantized encoder block, {dt:.2f} s"}
        be.close()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(line), flush=True)
        return 0

    # ------------------------------------------------------------------ ResNet-18 INT8
    from lightship_b200.backend import CudaBackend, GpuBackendConfig
    from lightship_b200.resnet18 import ResNet18Int8
    batch = args.batch
    if batch % world:
        raise SystemExit(f"batch {batch} does not split over {world} GPUs")
    lo, hi = shard_bounds(batch, world, rank)
    per = hi - lo
    # the global batch is seeded; each rank takes its contiguous shard
    rng = np.random.default_rng(DATA_SEED)
    x_all = rng.normal(size=(batch, 3, IMAGE, IMAGE)).astype(np.float32)
    x_host = torch.from_numpy(x_all[lo:hi]).pin_memory()
    del x_all
    be = CudaBackend(GpuBackendConfig(device_id=local, arena_bytes=256 << 20))
    model = ResNet18Int8(be, per, dev, image=IMAGE, seed=NET_SEED)
    x_dev = x_host.to(dev, non_blocking=False)
    model.calibrate(x_dev)
    stream = torch.cuda.current_stream(dev)

    # eager pass with events around every conv launch: the conv kernel's share and TOPS
    conv_ops = network_conv_ops(model)
    fc_ops = 2 * 512 * model.num_classes
    img_ops = sum(conv_ops.values()) + fc_ops
    evs = {}
    orig_run_conv = model._run_conv

    def timed_conv(spec, *a, **k):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        orig_run_conv(spec, *a, **k)
        e.record(stream)
        evs.setdefault(spec.name, []).append((s, e))

    model._run_conv = timed_conv
    for _ in range(3):
        # queue the pass behind a device sleep so the events time the kernels, not host launches
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(20_000_000)
        model.forward(x_dev)
    torch.cuda.synchronize(dev)
    model._run_conv = orig_run_conv
    conv_ms = sum(np.mean([s.elapsed_time(e) for s, e in v]) for v in evs.values())
    conv_tops = sum(conv_ops.values()) * per / (conv_ms * 1e-3) / 1e12

    branches = args.branches if args.branches > 0 else auto_branches(per)
    graph = model.capture(x_dev, branches=branches, concurrent_downsample=bool(args.ds_side))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        flush.zero_()
        graph.replay()
    torch.cuda.synchronize(dev)
    ops.check_device()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(uuid)
    sampler.start()
    barrier()
    torch.cuda.synchronize(dev)
    for s, e in ev:
        flush.zero_()
        s.record(stream)
        graph.replay()
        e.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    ops.check_device()
    ms = float(np.mean([s.elapsed_time(e) for s, e in ev]))
    ms_max = max_over_ranks(ms)
    value = batch / (ms_max * 1e-3)

    # end to end: pinned host input -> device, the network, logits -> host
    lib = _lib.lib()
    logits_host = torch.empty((per, model.num_classes), dtype=torch.float32).pin_memory()
    in_bytes = x_host.numel() * 4
    out_bytes = logits_host.numel() * 4
    sptr = C.c_void_p(stream.cuda_stream)
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        _lib.check(lib.lsc_memcpy_h2d(C.c_void_p(x_dev.data_ptr()), C.c_void_p(x_host.data_ptr()), in_bytes, sptr))
        graph.replay()
        _lib.check(lib.lsc_memcpy_d2h(C.c_void_p(logits_host.data_ptr()), C.c_void_p(model.logits.data_ptr()),
                                      out_bytes, sptr))

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    ee.record(stream)
    torch.cuda.synchronize(dev)
    e2e_seq_ms = max_over_ranks(es.elapsed_time(ee) / e2e_steps)
    e2e_ok = bool(torch.equal(logits_host, model.logits.cpu()))

    # the same, pipelined as a server runs it: step i+1's input upload (copy stream) overlaps
    # step i's network (compute stream); two input buffers, one graph captured on each; the
    # logits download follows each graph on the compute stream
    x_dev2 = torch.empty_like(x_dev)
    graph2 = model.capture(x_dev2, branches=branches, concurrent_downsample=bool(args.ds_side))
    copy_stream = torch.cuda.Stream(dev)
    cptr = C.c_void_p(copy_stream.cuda_stream)
    bufs, graphs = (x_dev, x_dev2), (graph, graph2)
    loaded = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    for ev_ in freed:
        ev_.record(stream)

    def e2e_pipelined(n_steps):
        for i in range(n_steps):
            b = i & 1
            copy_stream.wait_event(freed[b])
            _lib.check(lib.lsc_memcpy_h2d(C.c_void_p(bufs[b].data_ptr()), C.c_void_p(x_host.data_ptr()), in_bytes,
                                          cptr))
            loaded[b].record(copy_stream)
            stream.wait_event(loaded[b])
            graphs[b].replay()
            _lib.check(lib.lsc_memcpy_d2h(C.c_void_p(logits_host.data_ptr()), C.c_void_p(model.logits.data_ptr()),
                                          out_bytes, sptr))
            freed[b].record(stream)

    e2e_pipelined(4)
    torch.cuda.synchronize(dev)
    barrier()
    ps, pe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ps.record(stream)
    copy_stream.wait_event(ps)
    e2e_pipelined(e2e_steps)
    pe.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(ps.elapsed_time(pe) / e2e_steps)
    e2e_value = batch / (e2e_ms * 1e-3)
    e2e_ok = e2e_ok and bool(torch.equal(logits_host, model.logits.cpu()))
    del graph2

    line = {
        "metric": METRIC, "value": value, "unit": "img/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": RESNET_WORKLOAD, "global_batch": batch, "per_gpu_batch": per,
                   "image": IMAGE, "parallelism": f"batch split x{world} (no collective)",
                   "graph_branches": branches, "downsample_side_stream": bool(args.ds_side),
                   "l2": "flushed (256 MiB write) before every timed step", "seed": NET_SEED},
        "network_tops": img_ops * batch / (ms_max * 1e-3) / 1e12,
        "roofline": {"bound": "tensor", "kernel": "contraction_i8_kernel + contraction_i8_swap_kernel (INT8 implicit-GEMM conv)",
                     "achieved": conv_tops, "peak": int8_peak, "unit": "TOPS", "frac": conv_tops / int8_peak,
                     "traffic": load_traffic("contraction_i8_conv_layer1_b256.md"), "peak_source": peak_source,
                     "conv_share_of_step": conv_ms / ms if ms > 0 else None},
        "conv_us": {k: round(1e3 * float(np.mean([s.elapsed_time(e) for s, e in v])), 2) for k, v in evs.items()},
        "e2e": {"value": e2e_value, "unit": "img/s", "h2d_bytes_per_step": in_bytes * world,
                "d2h_bytes_per_step": out_bytes * world, "api": "lsc_memcpy_h2d + network + lsc_memcpy_d2h",
                "pipelined": "step i+1's upload (copy stream) overlaps step i's network; every step's "
                             "upload and logits download are inside the timed region",
                "sequential_value": batch / (e2e_seq_ms * 1e-3), "matches_device_run": e2e_ok},
        "gpu_launches": model.kernel_launches() * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and not args.no_gemm:
        variants, _ = gemm_measure(torch, dev, max(50, min(args.steps, 200)), 10)
        tops, gms = variants["i8"]
        vendor = vendor_gemm_measure(torch, dev, max(50, min(args.steps, 200)), 10)
        line["tensor_rate_probe"] = tensor_rate_probe()
        line["int8_gemm_4096"] = {"value": tops, "unit": "TOPS", "ms_per_launch": gms, "workload": GEMM_WORKLOAD,
                                  "vendor": {k: {"TOPS": v[0], "ms_per_launch": v[1]} for k, v in vendor.items()},
                                  "roofline_frac": tops / int8_peak,
                                  "traffic": load_traffic("contraction_i8_gemm_4096.md"),
                                  "variants": {k: {"TOPS": v[0], "ms_per_launch": v[1],
                                                   "roofline_frac": v[0] / int8_peak} for k, v in variants.items()}}
    if rank == 0 and not args.no_bert:
        r = bert_measure(torch, dev, BERT_BATCH, max(20, min(args.steps, 100)), 5, be)
        line["bert_block"] = {"value": BERT_BATCH / (r["ms"] * 1e-3), "unit": "sequences/s", "ms_per_block": r["ms"],
                              "workload": BERT_WORKLOAD, "projection_tops": r["gemm_tops"],
                              "projection_roofline_frac": r["gemm_tops"] / int8_peak,
                              "attention_tflops": r["attention_tflops"], "stage_ms": r["stage_ms"],
                              "e2e_sequences_per_s": BERT_BATCH / (r["e2e_ms"] * 1e-3)}
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            imgs = 24
            dt, _, _ = cpu_resnet_sample(imgs, dict(model.scales))
            line["cpu_baseline"] = {"value": imgs / dt, "unit": "img/s", "cores": host_threads(), "kind": "port",
                                    "sample": f"{imgs} images through the oracle's quantized ResNet-18 "
                                              f"(direct int8 convolutions, OpenMP), {dt:.2f} s"}
    del graph
    model.graph = None
    be.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["lightship", "reference"], default="lightship")
    ap.add_argument("--workload", choices=["resnet18", "gemm", "bert", "probe", "conv"], default="resnet18")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--branches", type=int, default=0,
                    help="image groups run concurrently inside the ResNet graph (0 = chosen by the per-GPU batch)")
    ap.add_argument("--ds-side", type=int, default=1,
                    help="1 = run each stage's downsample conv on a side stream beside its first conv")
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH,
                    help="global ResNet batch (default 256, the benchmark's; smaller only for profiling)")
    ap.add_argument("--no-gemm", action="store_true", help="skip the 4096^3 GEMM sub-measurement")
    ap.add_argument("--no-bert", action="store_true", help="skip the encoder-block sub-measurement")
    ap.add_argument("--only", default="", help="--workload conv: comma-separated shape names to run")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
