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


def load_profile_value(profile, key):
    """A `key: value` number from a committed ncu summary under profiles/ (None if absent)."""
    p = os.path.join(ROOT, "profiles", profile)
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith(key + ":"):
                try:
                    return float(line.split(":", 1)[1].strip())
                except ValueError:
                    return None
    return None


def resnet_conv_ops_per_image():
    """Algorithmic ops (2 per MAC) of ResNet-18's 20 convolutions for one 224x224 image
    (outputs 112 for conv1, then 56 / 28 / 14 / 7 for the four stages)."""
    from lightship_b200.resnet18 import build_params
    convs, _, _, _ = build_params(NET_SEED)
    total = 0
    for spec in convs:
        o = 112 if spec.name == "conv1" else 56 >> (int(spec.name[5]) - 1)
        total += 2 * spec.cout * o * o * spec.k * spec.k * spec.cin
    return total


RESNET_GOPS_PER_IMAGE = 3.628  # 2 x MACs incl. the classifier, standard stem max pool
RESNET_KERNELS = 22  # the stem (input quantize, conv1, max pool), 19 convolutions, average pool, classifier


def resnet_kernels(per_gpu_batch, sm_count):
    """Kernel launches of one INT8-session pass: the session runs the stem (input quantize, 7x7/2
    convolution, 3x3/2 max pool) as one launch at every batch."""
    del per_gpu_batch, sm_count
    return RESNET_KERNELS


def session_scales(sess):
    """The INT8 session's calibrated scales under the layer names of lightship_b200.resnet18."""
    from lightship_b200.resnet18 import build_params
    convs, _, _, _ = build_params(NET_SEED)
    sc = {"input": sess.value("X:q")["scale"], "pool": sess.value("pool")["scale"],
          "pooled": sess.value("pooled")["scale"]}
    for spec in convs:
        sc[spec.name] = sess.value(spec.name)["scale"]
    return sc


def gemm_line(torch, dev, int8_peak, steps, cpu_leg):
    """The 4096^3 INT8 per-channel GEMM: device TOPS per output variant with the library
    yardsticks, the e2e figure (host A and W uploaded, the GEMM, the int8 output downloaded,
    through lsc_memcpy_h2d / lsc_gemm_i8 / lsc_memcpy_d2h) and, on the CPU leg, the reference
    chain on a row sample."""
    from lightship_b200 import _lib
    variants, s_out = gemm_measure(torch, dev, steps, 10)
    tops, gms = variants["i8"]
    vendor = vendor_gemm_measure(torch, dev, steps, 10)
    lib = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)
    a, w, scale, bias = gemm_inputs()
    ha, hw = torch.from_numpy(a).pin_memory(), torch.from_numpy(w).pin_memory()
    hq = torch.empty((GEMM_M, GEMM_N), dtype=torch.int8).pin_memory()
    ta, tw = torch.empty_like(ha, device=dev), torch.empty_like(hw, device=dev)
    ts, tb = torch.from_numpy(scale).to(dev), torch.from_numpy(bias).to(dev)
    tq = torch.empty((GEMM_M, GEMM_N), dtype=torch.int8, device=dev)
    P = lambda t: C.c_void_p(t.data_ptr())

    def e2e_step():
        _lib.check(lib.lsc_memcpy_h2d(P(ta), P(ha), a.nbytes, sptr))
        _lib.check(lib.lsc_memcpy_h2d(P(tw), P(hw), w.nbytes, sptr))
        _lib.check(lib.lsc_gemm_i8(P(ta), P(tw), GEMM_M, GEMM_N, GEMM_K, P(tb), P(ts), s_out, 0, 1, P(tq), None, None,
                                   sptr))
        _lib.check(lib.lsc_memcpy_d2h(P(hq), P(tq), hq.numel(), sptr))

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(dev)
    n_e2e = 20
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    for _ in range(n_e2e):
        e2e_step()
    ee.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = es.elapsed_time(ee) / n_e2e
    leg = {"value": tops, "unit": "TOPS", "ms_per_launch": gms, "workload": GEMM_WORKLOAD,
           "roofline_frac": tops / int8_peak, "traffic": load_traffic("contraction_i8_gemm_4096.md"),
           "variants": {k: {"TOPS": v[0], "ms_per_launch": v[1], "roofline_frac": v[0] / int8_peak}
                        for k, v in variants.items()},
           "vendor": {k: {"TOPS": v[0], "ms_per_launch": v[1]} for k, v in vendor.items()},
           "e2e": {"value": GEMM_OPS / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS",
                   "h2d_bytes_per_step": a.nbytes + w.nbytes, "d2h_bytes_per_step": hq.numel(),
                   "api": "lsc_memcpy_h2d (A, W) + lsc_gemm_i8 + lsc_memcpy_d2h (int8 C)"}}
    if cpu_leg:
        w_kn = np.ascontiguousarray(w.T)
        rows = 64
        dt = cpu_gemm_rows(rows, a, w_kn, bias, scale, s_out)
        leg["cpu_baseline"] = {"value": 2 * rows * GEMM_N * GEMM_K / dt / 1e12, "unit": "TOPS",
                               "cores": host_threads(), "kind": "port",
                               "sample": f"rows 0..{rows - 1} of A through the reference chain (NN triple loop, "
                                         f"OpenMP over M, half-even requantize), {dt:.2f} s"}
    return leg


def bert_line(torch, dev, be, world, rank, int8_peak, steps, max_over_ranks, barrier, cpu_leg):
    """The BERT-base encoder block, batch 32 x seq 384 split over the ranks (each rank its
    32/N sequences, the step time the max over ranks)."""
    if BERT_BATCH % world:
        return {"skipped": f"batch {BERT_BATCH} does not split over {world} GPUs"}
    per = BERT_BATCH // world
    barrier()
    r = bert_measure(torch, dev, per, steps, 5, be)
    ms = max_over_ranks(r["ms"])
    e2e_ms = max_over_ranks(r["e2e_ms"])
    leg = {"value": BERT_BATCH / (ms * 1e-3), "unit": "sequences/s", "ms_per_block": ms, "per_gpu_batch": per,
           "workload": BERT_WORKLOAD, "projection_tops": r["gemm_tops"],
           "projection_roofline_frac": r["gemm_tops"] / int8_peak, "attention_tflops": r["attention_tflops"],
           "stage_ms": r["stage_ms"], "e2e_sequences_per_s": BERT_BATCH / (e2e_ms * 1e-3),
           "e2e_matches_device_run": r["e2e_ok"]}
    if cpu_leg:
        seqs = 4
        dt, _ = cpu_bert_sample(seqs, r["scales"])
        leg["cpu_baseline"] = {"value": seqs / dt, "unit": "sequences/s", "cores": host_threads(), "kind": "port",
                               "sample": f"{seqs} sequences of 384 tokens through the oracle's quantized encoder "
                                         f"block, {dt:.2f} s"}
    return leg


def fp32_legs(torch, dev, be, bf16_peak, steps, cpu_leg):
    """The two FP32 configurations through FP32 ONNX sessions (lsc_session_run on device
    buffers, split-TF32 tensor-core kernels): the 512^3 MatMul of two runtime inputs, and the
    1x64x56x56 3x3 convolution with bias, folded BatchNorm and ReLU.  Both are latency-bound at
    their size; the peak is the three-product split-TF32 rate (bf16 burst / 2 for TF32, / 3)."""
    from lightship_b200 import _lib
    from lightship_b200.backend import DataType, OnnxModel, Session, StorageLayout, Tensor
    from lightship_b200.onnx_writer import model as onnx_model, node as onnx_node
    peak = bf16_peak / 2 / 3
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    rng = np.random.default_rng(DATA_SEED)
    out = {}

    def timed(run):
        for _ in range(5):
            flush.zero_()
            run()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        torch.cuda.synchronize(dev)
        for s_, e_ in ev:
            flush.zero_()
            s_.record(stream)
            run()
            e_.record(stream)
        torch.cuda.synchronize(dev)
        return float(np.mean([s_.elapsed_time(e_) for s_, e_ in ev]))

    # config 1: C = A B, 512^3, entries U[-1, 1]
    a = rng.uniform(-1, 1, (512, 512)).astype(np.float32)
    b = rng.uniform(-1, 1, (512, 512)).astype(np.float32)
    m1 = OnnxModel(onnx_model([onnx_node("MatMul", ["A", "B"], ["C"])], {}, {"A": [512, 512], "B": [512, 512]},
                              {"C": [512, 512]}, name="gemm512"))
    s1 = Session(be, m1)
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    tc = torch.empty((512, 512), dtype=torch.float32, device=dev)
    ins = [Tensor("A", [512, 512], DataType.F32, ta), Tensor("B", [512, 512], DataType.F32, tb)]
    outs = [Tensor("C", [512, 512], DataType.F32, tc)]
    ms = timed(lambda: s1.run(ins, outs, stream=stream.cuda_stream))
    hc = np.zeros((512, 512), np.float32)
    h_ins = [Tensor("A", [512, 512], DataType.F32, a), Tensor("B", [512, 512], DataType.F32, b)]
    h_outs = [Tensor("C", [512, 512], DataType.F32, hc)]
    e2e = timed(lambda: s1.run(h_ins, h_outs, stream=stream.cuda_stream))
    flops = 2 * 512 ** 3
    leg = {"workload": "FP32 GEMM via Session: A[512x512] B[512x512] (ONNX MatMul of two inputs), U[-1,1]",
           "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
           "roofline": {"bound": "latency (tensor split-TF32)", "achieved": flops / (ms * 1e-3) / 1e12,
                        "peak": peak, "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / peak},
           "e2e": {"value": flops / (e2e * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": a.nbytes + b.nbytes,
                   "d2h_bytes_per_step": hc.nbytes, "api": "lsc_session_run (host A, B, C)"}}
    if cpu_leg:
        from oracle import oracle as orc
        t0 = time.perf_counter()
        reps = 5
        for _ in range(reps):
            want = orc.matmul(a, b, host_threads())
        dt = (time.perf_counter() - t0) / reps
        leg["cpu_baseline"] = {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": host_threads(), "kind": "port",
                               "sample": "the whole 512^3 product, NEON-order blocked GEMM restated, row blocks over "
                                         "all host threads"}
        got = tc.cpu().numpy()
        leg["max_rel_err_vs_oracle"] = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
    out["gemm_512"] = leg
    del s1, m1

    # config 2: Conv2d 3x3 s1 p1, 1x64x56x56 -> 64, bias, BN folded, ReLU
    x = rng.normal(size=(1, 64, 56, 56)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / 576), (64, 64, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, 64).astype(np.float32)
    g, beta = rng.uniform(0.5, 1.5, 64).astype(np.float32), rng.normal(0, 0.1, 64).astype(np.float32)
    mu, var = rng.normal(0, 0.1, 64).astype(np.float32), rng.uniform(0.5, 1.5, 64).astype(np.float32)
    nodes = [onnx_node("Conv", ["X", "W", "Bc"], ["t"], kernel_shape=[3, 3], pads=[1, 1, 1, 1]),
             onnx_node("BatchNormalization", ["t", "g", "beta", "mu", "var"], ["u"], epsilon=1e-5),
             onnx_node("Relu", ["u"], ["Y"])]
    m2 = OnnxModel(onnx_model(nodes, {"W": w, "Bc": bias, "g": g, "beta": beta, "mu": mu, "var": var},
                              {"X": [1, 64, 56, 56]}, {"Y": [1, 64, 56, 56]}, name="conv_bn_relu"))
    s2 = Session(be, m2)
    tx = torch.from_numpy(x).to(dev)
    ty = torch.empty((1, 64, 56, 56), dtype=torch.float32, device=dev)
    ins = [Tensor("X", [1, 64, 56, 56], DataType.F32, tx, layout=StorageLayout.NCHW)]
    outs = [Tensor("Y", [1, 64, 56, 56], DataType.F32, ty, layout=StorageLayout.NCHW)]
    ms = timed(lambda: s2.run(ins, outs, stream=stream.cuda_stream))
    hy = np.zeros((1, 64, 56, 56), np.float32)
    h_ins = [Tensor("X", [1, 64, 56, 56], DataType.F32, x, layout=StorageLayout.NCHW)]
    h_outs = [Tensor("Y", [1, 64, 56, 56], DataType.F32, hy, layout=StorageLayout.NCHW)]
    e2e = timed(lambda: s2.run(h_ins, h_outs, stream=stream.cuda_stream))
    flops = 2 * 3136 * 64 * 576
    leg = {"workload": "FP32 Conv2d 3x3 s1 p1, 1x64x56x56 -> 64, bias, BatchNorm folded, ReLU (ONNX Conv+BN+Relu)",
           "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
           "roofline": {"bound": "latency (tensor split-TF32)", "achieved": flops / (ms * 1e-3) / 1e12,
                        "peak": peak, "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / peak},
           "e2e": {"value": flops / (e2e * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": x.nbytes,
                   "d2h_bytes_per_step": hy.nbytes, "api": "lsc_session_run (host X, Y)"}}
    if cpu_leg:
        from oracle import oracle as orc
        reps = 5
        for threads, key in ((1, "cpu_baseline"), (host_threads(), "cpu_baseline_all_cores")):
            t0 = time.perf_counter()
            for _ in range(reps):
                want = orc.act(orc.batchnorm_inference(orc.conv2d_nchw(x, w, bias, pad=(1, 1), threads=threads),
                                                       g, beta, mu, var), orc.ACT_RELU)
            dt = (time.perf_counter() - t0) / reps
            leg[key] = {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                        "sample": "the whole convolution (im2col + GEMM, BatchNorm, ReLU)" +
                                  (", one thread per image as the reference runs it" if threads == 1 else "")}
        got = ty.cpu().numpy()
        leg["max_rel_err_vs_oracle"] = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
    out["conv_bn_relu_64x56x56"] = leg
    del s2, m2
    out["conv3x3_algorithms"] = fp32_conv_algorithms(torch, dev, be, timed)
    return out


def fp32_conv_algorithms(torch, dev, be, timed):
    """The FP32 3x3 stride-1 convolution by the direct split-TF32 kernel and by Winograd
    F(2x2, 3x3) (fp32_mode LSC_FP32_WINOGRAD), Backend operator on device tensors, at the
    config-2 shape and at a layer1-sized batch of 32: device time per launch sequence and the
    direct convolution's algorithmic TFLOP/s."""
    from lightship_b200 import _lib
    from lightship_b200.backend import DataType, OperatorDef, OperatorType, Tensor
    stream = torch.cuda.current_stream(dev)
    res = {}
    for n in (1, 32):
        rng = np.random.default_rng(DATA_SEED + n)
        x = torch.from_numpy(rng.normal(size=(n, 64, 56, 56)).astype(np.float32)).to(dev)
        w = rng.normal(0, np.sqrt(2.0 / 576), (64, 64, 3, 3)).astype(np.float32)
        bias = rng.normal(0, 0.1, 64).astype(np.float32)
        y = torch.empty((n, 64, 56, 56), dtype=torch.float32, device=dev)
        xt = Tensor("x", [n, 64, 56, 56], DataType.F32, x)
        yt = Tensor("y", [n, 64, 56, 56], DataType.F32, y)
        flops = 2.0 * n * 3136 * 64 * 576
        row = {}
        outs = {}
        for name, mode in (("direct_3xtf32", _lib.FP32_3XTF32), ("winograd_f2x2_3x3", _lib.FP32_WINOGRAD)):
            op = be.compile_operator(OperatorDef("conv", OperatorType.Conv2d, padding=(1, 1), fp32_mode=mode), None,
                                     [xt, Tensor("w", list(w.shape), DataType.F32, w),
                                      Tensor("b", [64], DataType.F32, bias)], [yt])
            ms = timed(lambda: be.execute(op, [xt], [yt], stream=stream.cuda_stream))
            row[name] = {"us": round(ms * 1e3, 2), "TFLOP_s_algorithmic": round(flops / (ms * 1e-3) / 1e12, 1)}
            outs[name] = y.clone()
            del op
        d = outs["direct_3xtf32"].double()
        row["max_abs_diff_winograd_vs_direct"] = float((outs["winograd_f2x2_3x3"].double() - d).abs().max())
        row["winograd_speedup"] = round(row["direct_3xtf32"]["us"] / row["winograd_f2x2_3x3"]["us"], 3)
        res[f"n{n}_64x56x56_to_64"] = row
    return res


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
    # through the C ABI: the ONNX model compiled by lsc_session_create_ex into an INT8 session
    from lightship_b200.backend import CudaBackend, GpuBackendConfig, DataType, OnnxModel, Session, StorageLayout, Tensor
    from lightship_b200.onnx_writer import resnet18_onnx
    batch = args.batch
    if batch % world:
        raise SystemExit(f"batch {batch} does not split over {world} GPUs")
    lo, hi = shard_bounds(batch, world, rank)
    per = hi - lo
    # the global batch is seeded; each rank takes its contiguous shard
    rng = np.random.default_rng(DATA_SEED)
    x_all = rng.normal(size=(batch, 3, IMAGE, IMAGE)).astype(np.float32)
    x_np = np.ascontiguousarray(x_all[lo:hi])
    del x_all
    x_host = torch.from_numpy(x_np).pin_memory()
    arena = max(1 << 30, per * (12 << 20))  # calibration scratch + two input slots + the activation block
    be = CudaBackend(GpuBackendConfig(device_id=local, arena_bytes=arena))
    model = OnnxModel(resnet18_onnx(per, NET_SEED, IMAGE))
    cal = Tensor("X", list(x_np.shape), DataType.F32, x_np, layout=StorageLayout.NCHW)
    sess = Session(be, model, precision="int8", calibration=cal, concurrent=bool(args.ds_side))
    lib = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)
    in_ptr, in_bytes = sess.io_buffer(False)
    out_ptr, out_bytes = sess.io_buffer(True)
    _lib.check(lib.lsc_memcpy_h2d(C.c_void_p(in_ptr), C.c_void_p(x_host.data_ptr()), in_bytes, sptr))
    dev_in, dev_out = _lib.lsc_tensor(), _lib.lsc_tensor()
    dev_in.ndim = 4
    for i, d in enumerate(x_np.shape):
        dev_in.shape[i] = d
    dev_in.dtype, dev_in.location, dev_in.data, dev_in.nbytes = 0, _lib.MEM_DEVICE, in_ptr, in_bytes
    dev_out.dtype, dev_out.location, dev_out.data, dev_out.nbytes = 0, _lib.MEM_DEVICE, out_ptr, out_bytes

    def step():  # one forward pass on the session's own device buffers (nothing copied)
        _lib.check(lib.lsc_session_run(sess._h, C.byref(dev_in), 1, C.byref(dev_out), 1, sptr))

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize(dev)
    ops.check_device()
    # parity: the logits of the timed configuration against the oracle's quantized network on
    # the same images with the session's calibrated scales (first and last two of the shard)
    logits_dev = np.empty((per, 1000), np.float32)
    _lib.check(lib.lsc_memcpy_d2h(C.c_void_p(logits_dev.ctypes.data), C.c_void_p(out_ptr), out_bytes, sptr))
    torch.cuda.synchronize(dev)
    scales = session_scales(sess)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(uuid)
    sampler.start()
    barrier()
    torch.cuda.synchronize(dev)
    for s, e in ev:
        flush.zero_()
        s.record(stream)
        step()
        e.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    ops.check_device()
    ms = float(np.mean([s.elapsed_time(e) for s, e in ev]))
    ms_max = max_over_ranks(ms)
    value = batch / (ms_max * 1e-3)

    # end to end through the session's public API: pinned host input in, host logits out,
    # sequential (lsc_session_run, complete on return) and pipelined (lsc_session_run_async:
    # step i+1's upload on the session's copy stream overlaps step i's network)
    logits_host = torch.empty((per, 1000), dtype=torch.float32).pin_memory()
    host_in = Tensor("X", list(x_np.shape), DataType.F32, x_host, layout=StorageLayout.NCHW)
    host_out = Tensor("logits", [1], DataType.F32, logits_host)
    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        sess.run([host_in], [host_out], stream=stream.cuda_stream)
    barrier()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    for _ in range(e2e_steps):
        sess.run([host_in], [host_out], stream=stream.cuda_stream)
    ee.record(stream)
    torch.cuda.synchronize(dev)
    e2e_seq_ms = max_over_ranks(es.elapsed_time(ee) / e2e_steps)
    e2e_ok = bool(np.array_equal(logits_host.numpy().view(np.uint32), logits_dev.view(np.uint32)))
    for _ in range(4):
        sess.run_async([host_in], [host_out], stream=stream.cuda_stream)
    torch.cuda.synchronize(dev)
    barrier()
    ps, pe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ps.record(stream)
    for _ in range(e2e_steps):
        sess.run_async([host_in], [host_out], stream=stream.cuda_stream)
    pe.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(ps.elapsed_time(pe) / e2e_steps)
    e2e_value = batch / (e2e_ms * 1e-3)
    e2e_ok = e2e_ok and bool(np.array_equal(logits_host.numpy().view(np.uint32), logits_dev.view(np.uint32)))

    plan = sess.memory_plan()
    conv_ops_img = resnet_conv_ops_per_image()
    share = load_profile_value("resnet18_int8_b256_launches.md", "conv_kernel_share")
    conv_tops = conv_ops_img * batch / (ms_max * 1e-3 * share) / 1e12 if share else None
    line = {
        "metric": METRIC, "value": value, "unit": "img/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": RESNET_WORKLOAD, "global_batch": batch, "per_gpu_batch": per,
                   "image": IMAGE, "parallelism": f"batch split x{world} (no collective)",
                   "api": "ONNX model -> lsc_session_create_ex (INT8) -> lsc_session_run",
                   "l2": "flushed (256 MiB write) before every timed step", "seed": NET_SEED},
        "parity": None,
        "network_tops": RESNET_GOPS_PER_IMAGE * batch / (ms_max * 1e-3) / 1e3,
        "roofline": {"bound": "tensor", "kernel": "contraction_i8_kernel + contraction_i8_swap_kernel + stem_conv_pool_kernel (INT8 convolutions)",
                     "achieved": conv_tops, "peak": int8_peak, "unit": "TOPS",
                     "frac": conv_tops / int8_peak if conv_tops else None,
                     "traffic": load_profile_value("contraction_i8_swap_conv_layer1.md", "traffic_bytes_per_launch"),
                     "peak_source": peak_source,
                     "conv_share_of_step": share,
                     "method": "achieved = algorithmic conv ops / (graph step time x the conv kernels' share of the "
                               "step's device time in the committed launch list)"},
        "memory_plan": plan,
        "e2e": {"value": e2e_value, "unit": "img/s", "h2d_bytes_per_step": in_bytes * world,
                "d2h_bytes_per_step": out_bytes * world,
                "api": "lsc_session_run_async (pinned host input and logits, two input slots)",
                "pipelined": "step i+1's upload (the session's copy stream) overlaps step i's network; every step's "
                             "upload and logits download are inside the timed region",
                "sequential_value": batch / (e2e_seq_ms * 1e-3), "matches_device_run": e2e_ok},
        "gpu_launches": resnet_kernels(per, torch.cuda.get_device_properties(local).multi_processor_count) * args.steps,
        "clocks": clocks,
    }
    del sess, model
    if not args.no_gemm:
        gemm_leg = gemm_line(torch, dev, int8_peak, max(50, min(args.steps, 200)), rank == 0 and world == 1 and
                             not args.no_cpu_baseline)
        if rank == 0:
            line["int8_gemm_4096"] = gemm_leg
    if not args.no_bert:
        bert_leg = bert_line(torch, dev, be, world, rank, int8_peak, max(20, min(args.steps, 100)), max_over_ranks,
                             barrier, rank == 0 and world == 1 and not args.no_cpu_baseline)
        if rank == 0:
            line["bert_block"] = bert_leg
    if not args.no_fp32 and rank == 0:
        line["fp32_configs"] = fp32_legs(torch, dev, be, bf16_peak, max(20, min(args.steps, 100)),
                                         world == 1 and not args.no_cpu_baseline)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the CPU leg: the oracle's quantized ResNet-18 on the first images of the batch with the
        # session's calibrated scales -- timed as the baseline, and its logits compared with the
        # timed configuration's (parity)
        imgs = 24
        dt, cpu_logits, _ = cpu_resnet_sample(imgs, scales)
        line["cpu_baseline"] = {"value": imgs / dt, "unit": "img/s", "cores": host_threads(), "kind": "port",
                                "sample": f"{imgs} images through the oracle's quantized ResNet-18 "
                                          f"(direct int8 convolutions, OpenMP), {dt:.2f} s"}
        line["parity"] = {"images": imgs, "bit_exact_logits": bool(np.array_equal(
            cpu_logits.view(np.uint32), logits_dev[:imgs].view(np.uint32)))}
    elif rank == 0:
        # without the timed CPU leg (several GPUs, or --no-cpu-baseline): the oracle on the first
        # four images of this rank's shard (the first images of the batch) with its session's
        # calibrated scales, against the timed configuration's logits
        imgs = min(4, per)
        _, cpu_logits, _ = cpu_resnet_sample(imgs, scales)
        line["parity"] = {"images": imgs, "rank": 0, "bit_exact_logits": bool(np.array_equal(
            cpu_logits.view(np.uint32), logits_dev[:imgs].view(np.uint32)))}
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
    ap.add_argument("--ds-side", type=int, default=1,
                    help="1 = the session runs each stage's downsample conv on a second stream beside its first conv")
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH,
                    help="global ResNet batch (default 256, the benchmark's; smaller only for profiling)")
    ap.add_argument("--no-gemm", action="store_true", help="skip the 4096^3 GEMM sub-measurement")
    ap.add_argument("--no-bert", action="store_true", help="skip the encoder-block sub-measurement")
    ap.add_argument("--no-fp32", action="store_true", help="skip the FP32 configurations")
    ap.add_argument("--only", default="", help="--workload conv: comma-separated shape names to run")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
