"""Benchmark of the CUDA backend's headline workload.

Workload (one "step"): the INT8 per-channel symmetric GEMM M=N=K=4096 -- int8 A and W
uniform in [-127, 127], per-output-channel f32 scales U[0.001, 0.02], int32 bias, int32
accumulate, requantized int8 output (round-half-even, saturate) plus the dequantized f32
variant, both written by one fused launch of this package's tcgen05 kernel.

* ``value``: whole-job TOPS (2*M*N*K per GPU per step) with operands resident in HBM; the
  L2 is flushed before every timed launch (256 MiB write) and each launch is timed with CUDA
  events on the launching stream; the max over ranks is taken.
* ``e2e``: the same metric through the public Backend API (``CudaBackend.execute`` with host
  tensors): every step copies A from pinned host memory to the device and both outputs back.
* ``roofline``: tensor-bound; achieved INT8 TOPS of the kernel against the INT8 peak derived
  from the measured bf16 burst peak (B200 issues dense INT8 at twice the bf16 rate).
* ``cpu_baseline`` (rank 0, one GPU): the oracle's restatement of the reference CPU chain
  (quantized_gemm_int8 triple loop + dequantize/requantize, threaded over M) on a 512-row
  slice of the same workload, on all host threads.

Multi-GPU: replicas (the GEMM does not shard without a reduction; weak scaling), one rank
per GPU under torchrun; no collective touches the data path.

``--impl reference`` times the reference CPU implementation (the oracle port) on the host
cores, rank 0 only, and prints the same metric with ``"impl": "reference"``.
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

M = N = K = 4096
OPS_PER_STEP = 2 * M * N * K
METRIC = "INT8 conv/GEMM TOPS"
UNIT = "TOPS"
WORKLOAD = "int8 per-channel GEMM M=N=K=4096, int32 bias, requant int8 (half-even) + dequant f32"
SEED = 20260415
S_OUT_SAMPLE_SEED = 7


def make_inputs(rng):
    a = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    scale = rng.uniform(0.001, 0.02, size=N).astype(np.float32)
    bias = rng.integers(-100000, 100000, size=N, dtype=np.int32)
    return a, w, scale, bias


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def load_traffic():
    """dram bytes per launch of the GEMM kernel from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "contraction_i8_gemm_4096.md")
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
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                   "-lms", "50"]
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


# --------------------------------------------------------------------------- CPU baseline
def cpu_baseline_rows(rows, a, w_kn, bias, scale, s_out, threads=0):
    """The reference CPU chain on rows [0, rows) of A: NN triple loop then the epilogue."""
    from oracle import oracle as orc
    t0 = time.perf_counter()
    acc = orc.gemm_i8_nn(a[:rows], w_kn, threads)
    orc.requant(acc, bias, scale, orc.ACT_NONE, s_out, orc.ROUND_HALF_EVEN)
    return time.perf_counter() - t0


def run_cpu_baseline(a, w, bias, scale, s_out, rows=512):
    w_kn = np.ascontiguousarray(w.T)
    dt = cpu_baseline_rows(rows, a, w_kn, bias, scale, s_out)
    ops = 2 * rows * N * K
    return {"value": ops / dt / 1e12, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"rows 0..{rows - 1} of the 4096^3 chain (1/{M // rows} of M), reference "
                      f"loop order (i, j, p) over B[K,N], OpenMP over M, {dt:.2f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    rng = np.random.default_rng(SEED)
    a, w, scale, bias = make_inputs(rng)
    w_kn = np.ascontiguousarray(w.T)
    s_out = 40.0
    # size each step so that warmup + steps take about two minutes
    t_probe = cpu_baseline_rows(16, a, w_kn, bias, scale, s_out)
    per_row = t_probe / 16
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = int(max(8, min(M, budget / max(per_row, 1e-9))))
    for _ in range(args.warmup):
        cpu_baseline_rows(rows, a, w_kn, bias, scale, s_out)
    times = [cpu_baseline_rows(rows, a, w_kn, bias, scale, s_out) for _ in range(args.steps)]
    t = sum(times) / len(times)
    value = 2 * rows * N * K / t / 1e12
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sample_rows_per_step": rows},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "sample": f"rows 0..{rows - 1} of A per step (1/{M / rows:.1f} of M), "
                                       "reference loop order, OpenMP over M"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- GPU arm
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from lightship_b200 import _lib, ops
    from lightship_b200.backend import (CudaBackend, DataType, GpuBackendConfig, OperatorDef,
                                        OperatorType, Quantization, Rounding, Tensor)
    lib = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)

    rng = np.random.default_rng(SEED)
    a, w, scale, bias = make_inputs(rng)
    ta, tw = torch.from_numpy(a).to(dev), torch.from_numpy(w).to(dev)
    ts, tb = torch.from_numpy(scale).to(dev), torch.from_numpy(bias).to(dev)
    q = torch.empty((M, N), dtype=torch.int8, device=dev)
    y = torch.empty((M, N), dtype=torch.float32, device=dev)

    # output scale: find_scale_zp (symmetric) on the dequantized output, on the device
    ws = torch.zeros(4, dtype=torch.int32, device=dev)
    s_dev = torch.empty(1, dtype=torch.float32, device=dev)
    z_dev = torch.empty(1, dtype=torch.int32, device=dev)
    _lib.check(lib.lsc_gemm_i8(C.c_void_p(ta.data_ptr()), C.c_void_p(tw.data_ptr()), M, N, K,
                               C.c_void_p(tb.data_ptr()), C.c_void_p(ts.data_ptr()), 1.0, 0, 1,
                               None, C.c_void_p(y.data_ptr()), None, sptr))
    _lib.check(lib.lsc_find_scale_zp_f32(C.c_void_p(y.data_ptr()), M * N, 9, 1, C.c_void_p(ws.data_ptr()),
                                         16, C.c_void_p(s_dev.data_ptr()), C.c_void_p(z_dev.data_ptr()), sptr))
    s_out = float(s_dev.item())

    def launch():
        _lib.check(lib.lsc_gemm_i8(C.c_void_p(ta.data_ptr()), C.c_void_p(tw.data_ptr()), M, N, K,
                                   C.c_void_p(tb.data_ptr()), C.c_void_p(ts.data_ptr()), s_out, 0, 1,
                                   C.c_void_p(q.data_ptr()), C.c_void_p(y.data_ptr()), None, sptr))

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)

    for _ in range(args.warmup):
        flush.zero_()
        launch()
    torch.cuda.synchronize(dev)
    ops.check_device()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        launch()
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ops.check_device()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = float(np.mean(step_ms))
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * OPS_PER_STEP / (ms_max * 1e-3) / 1e12

    # ---- end to end through the Backend API with host tensors
    be = CudaBackend(GpuBackendConfig(device_id=local, rounding=Rounding.HalfEven))
    w_t = Tensor("W", [N, K], DataType.QInt8, w, quantization=Quantization(list(map(float, scale))))
    b_t = Tensor("bias", [N], DataType.QInt32, bias)
    a_host = torch.from_numpy(a).pin_memory()
    q_host = torch.empty((M, N), dtype=torch.int8).pin_memory()
    y_host = torch.empty((M, N), dtype=torch.float32).pin_memory()
    a_t = Tensor("A", [M, K], DataType.QInt8, a_host, quantization=Quantization([1.0]))
    q_t = Tensor("Q", [1], DataType.QInt8, q_host)
    y_t = Tensor("Y", [1], DataType.F32, y_host)
    opdef = OperatorDef("fc_int8", OperatorType.FullyConnected, rounding=Rounding.HalfEven,
                        output_scale=s_out)
    compiled = be.compile_operator(opdef, None, [a_t, w_t, b_t], [q_t, y_t])
    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        be.execute(compiled, [a_t], [q_t, y_t], stream=stream.cuda_stream)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(e2e_steps):
        be.execute(compiled, [a_t], [q_t, y_t], stream=stream.cuda_stream)
    e_end.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e_start.elapsed_time(e_end) / e2e_steps
    te = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * OPS_PER_STEP / (float(te.item()) * 1e-3) / 1e12
    # spot check of the e2e result against the device-resident run
    launch()
    torch.cuda.synchronize(dev)
    e2e_ok = bool(torch.equal(q_host, q.cpu())) and bool(torch.equal(y_host.view(torch.int32), y.cpu().view(torch.int32)))

    bf16_peak, peak_src = load_peaks()
    int8_peak = 2.0 * bf16_peak
    achieved = OPS_PER_STEP / (ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K, "parallelism": f"replicas x{world}",
                   "l2": "flushed (256 MiB write) before every timed launch", "seed": SEED},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOPS",
                     "frac": achieved / int8_peak, "traffic": load_traffic(),
                     "peak_source": f"2 x {peak_src} bf16 burst ({bf16_peak} TFLOP/s); nominal dense INT8 4500 TOPS",
                     "frac_of_nominal": achieved / 4500.0},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": M * K,
                "d2h_bytes_per_step": M * N * 5, "api": "CudaBackend.execute(FullyConnected int8) host tensors",
                "matches_device_run": e2e_ok},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "s_out": s_out,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = run_cpu_baseline(a, w, bias, scale, s_out)
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
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["lightship", "reference"], default="lightship")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
