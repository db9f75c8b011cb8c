"""Benchmark of the wide forward path on B200 (one JSON line on rank 0).

Workload (the headline config that fits one GPU):
WideLinear, N=64 models per GPU, in=1024, out=4096, B=256 rows per model,
bf16 weights/activations (W ~ N(0, 1/1024), bias zeros, x ~ N(0, 1)), fp32
accumulation. A step is one wide forward over the whole batch: one launch of
the tcgen05 grouped-GEMM kernel (bias fused in its epilogue).

  value   samples/s = N*B*world / t_step, t_step from CUDA events over K
          back-to-back steps with inputs resident in HBM (705 MB touched per
          step, far above the 126 MB L2, so no flush is needed); max over ranks.
  e2e     same metric through the public API (``WideLinear.__call__``) with
          the step's input copied host->device from pinned memory and the
          output copied device->host inside the timed region.
  roofline  HBM-bound (arithmetic intensity 195 FLOP/B < ridge): algorithmic
          bytes per launch / mean launch time vs the measured HBM copy peak.
  cpu_baseline  the reference's arithmetic (einsum + bias, bf16) on the host
          cores, on a bounded sample (a few models per timed step).

Multi-GPU (torchrun, one process per GPU, NCCL): each rank runs its own 64
models (weak scaling; the N models are independent, no collective is on the
data path). ``--gather`` adds the optional output all-gather to every step.

``--impl reference`` times the reference's CPU implementation of the path
(the oracle port of its torch arithmetic) on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "pytorch-parallel-compiler_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "wide-forward samples/s (N·B/s) at 1/2/4/8 B200; % of TC/HBM roofline"
N_MODELS, B_ROWS, IN_F, OUT_F = 64, 256, 1024, 4096
DTYPE = torch.bfloat16
ELEM = 2


def alg_bytes(n):
    """Compulsory HBM bytes per launch: W + x + y + bias, each touched once."""
    return ELEM * (n * OUT_F * IN_F + n * B_ROWS * IN_F + n * B_ROWS * OUT_F + n * OUT_F)


def alg_flops(n):
    return 2 * n * B_ROWS * IN_F * OUT_F


ALG_BYTES = alg_bytes(N_MODELS)
# DRAM traffic (read + write bytes) per launch of linear_tc_kernel measured by
# ncu on a 16-model capture scaled to 64 models; see profiles/linear_tc_cfg2.md.
NCU_TRAFFIC_BYTES = 593_080_000  # 148.27 MB for 16 models x 64/16


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the GPU is busy."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_workload(dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    import wide_compiler as wc
    lin = wc.WideLinear(N_MODELS, IN_F, OUT_F, bias=True)
    with torch.no_grad():
        w = (torch.randn(N_MODELS, OUT_F, IN_F, device=dev, generator=g) / (IN_F ** 0.5)).to(DTYPE)
        lin = lin.to(dev, DTYPE)
        lin.weight.copy_(w)
        lin.bias.zero_()
    x = torch.randn(N_MODELS, B_ROWS, IN_F, device=dev, generator=g).to(DTYPE)
    return lin, x


def cpu_baseline_sample(seconds: float = 10.0):
    """The reference's arithmetic for this path (wide_linear.py:165-168: einsum
    'noi,nbi->nbo' then + bias, in the config dtype) on the host cores, on a
    bounded sample of models; returns samples/s and what was sampled."""
    from oracle import wide_oracle as O
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    n_s = 2
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(n_s, OUT_F, IN_F, generator=g) / 32).to(DTYPE)
    b = torch.zeros(n_s, OUT_F, dtype=DTYPE)
    x = torch.randn(n_s, B_ROWS, IN_F, generator=g).to(DTYPE)
    O.linear_ref_dtype(x, w, b)  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while True:
        O.linear_ref_dtype(x, w, b)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    value = reps * n_s * B_ROWS / el
    return {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{reps} reps x {n_s} of the {N_MODELS} models (B={B_ROWS}, {IN_F}->{OUT_F}, bf16) "
                      f"in {el:.1f} s, torch CPU einsum+bias"}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import wide_oracle as O
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    n_s = 1
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(N_MODELS, OUT_F, IN_F, generator=g) / 32).to(DTYPE)
    b = torch.zeros(N_MODELS, OUT_F, dtype=DTYPE)
    x = torch.randn(N_MODELS, B_ROWS, IN_F, generator=g).to(DTYPE)
    for s in range(args.warmup):
        i = s % N_MODELS
        O.linear_ref_dtype(x[i:i + n_s], w[i:i + n_s], b[i:i + n_s])
    t0 = time.perf_counter()
    for s in range(args.steps):
        i = s % N_MODELS
        O.linear_ref_dtype(x[i:i + n_s], w[i:i + n_s], b[i:i + n_s])
    el = time.perf_counter() - t0
    value = args.steps * n_s * B_ROWS / el
    line = {
        "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * el / max(args.steps, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"WideLinear cfg2 sample: {n_s} of {N_MODELS} models per step, B={B_ROWS}, "
                               f"{IN_F}->{OUT_F}, bf16 (reference arithmetic on host CPU)"},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                         "sample": f"{n_s} model x {B_ROWS} rows per step, {args.steps} steps"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_b200(args):
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = False
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
        pg = True
    from wide_compiler import _native, ops
    _native.load()
    lin, x = make_workload(dev, seed=1234 + rank)
    out_gather = None
    if args.gather and world > 1:
        out_gather = torch.empty(world * N_MODELS, B_ROWS, OUT_F, device=dev, dtype=DTYPE)

    def step():
        y = ops.linear(x, lin.weight, lin.bias)
        if out_gather is not None:
            torch.distributed.all_gather_into_tensor(out_gather, y)
        return y

    def barrier():
        if pg:
            torch.distributed.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    clocks = ClockSampler(local)
    clocks.start()
    # Warm-up (untimed); also spins clocks up before the timed region.
    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if pg:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms_max = float(t.item())

    # End to end through the public API: pinned host input -> device ->
    # WideLinear forward -> host output, every step.
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    x_host = x.cpu().pin_memory()
    y_host = torch.empty(N_MODELS, B_ROWS, OUT_F, dtype=DTYPE).pin_memory()
    x_dev = torch.empty_like(x)
    for _ in range(2):
        x_dev.copy_(x_host, non_blocking=True)
        y_host.copy_(lin(x_dev), non_blocking=True)
    barrier()
    e0.record(stream)
    for _ in range(e2e_steps):
        x_dev.copy_(x_host, non_blocking=True)
        y = lin(x_dev)
        if out_gather is not None:
            torch.distributed.all_gather_into_tensor(out_gather, y)
        y_host.copy_(y, non_blocking=True)
    e1.record(stream)
    barrier()
    ms_e2e = e0.elapsed_time(e1) / e2e_steps
    t2 = torch.tensor([ms_e2e], device=dev, dtype=torch.float64)
    if pg:
        torch.distributed.all_reduce(t2, op=torch.distributed.ReduceOp.MAX)
    ms_e2e = float(t2.item())
    clk = clocks.stop()
    dev_err = _native.device_error()

    if rank == 0:
        samples = N_MODELS * B_ROWS * world
        peak, peak_kind = peaks()
        achieved = alg_bytes(N_MODELS) / (ms * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": samples / (ms_max * 1e-3),
            "unit": "samples/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": f"WideLinear cfg2: N={N_MODELS} models/GPU, in={IN_F}, out={OUT_F}, B={B_ROWS}, "
                            f"bf16, fp32 accumulate, bias fused",
                "models_per_gpu": N_MODELS, "rows_per_model": B_ROWS, "in_features": IN_F,
                "out_features": OUT_F, "l2": "inputs larger than L2 (705 MB touched per step), no flush",
                "gather": bool(out_gather is not None),
            },
            "e2e": {"value": samples / (ms_e2e * 1e-3), "unit": "samples/s",
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                    "d2h_bytes_per_step": y_host.numel() * y_host.element_size(),
                    "steps": e2e_steps, "ms_per_step": ms_e2e},
            "gpu_launches": args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": NCU_TRAFFIC_BYTES,
                         "algorithmic_bytes": alg_bytes(N_MODELS),
                         "tflops": alg_flops(N_MODELS) / (ms * 1e-3) / 1e12},
            "clocks": clk,
            "device_error": dev_err,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample(args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if pg:
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()
    return 0


def main():
    global N_MODELS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=100)
    ap.add_argument("--gather", action="store_true", help="include the optional output all-gather")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--models", type=int, default=N_MODELS,
                    help="models per GPU (default: the cfg2 value 64; smaller only for profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    N_MODELS = args.models
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
