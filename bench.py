"""Benchmark of the wide forward path on B200 (one JSON line on rank 0).

Default workload (the headline config that fits one
GPU): WideLinear, N=64 models per GPU, in=1024, out=4096, B=256 rows per
model, bf16 weights/activations (W ~ N(0, 1/1024), bias zeros, x ~ N(0, 1)),
fp32 accumulation. A step is one wide forward over the whole batch: one
launch of the tcgen05 grouped-GEMM kernel (bias fused in its epilogue).

  value   samples/s = N*B*world / t_step, t_step from CUDA events over K
          back-to-back steps with inputs resident in HBM (705 MB touched per
          step, far above the 126 MB L2, so no flush is needed); max over ranks.
  e2e     same metric through the public API (the module's __call__) with the
          step's input copied host->device from pinned memory and the output
          copied device->host inside the timed region.
  roofline  dominant kernel's algorithmic bytes (or FLOPs) per launch / mean
          launch time (CUDA events on the launching stream) vs the measured
          peak in MEASURED_PEAKS.json.
  cpu_baseline  the reference's arithmetic (its torch op sequence in the
          config dtype) on the host cores, on a bounded sample.

Other BASELINE configs (``--workload cfg1|cfg3|cfg4gru|cfg4lstm|cfg5``) print
the same line for that config; ``--graph`` replays the step from a CUDA graph.

Multi-GPU (torchrun, one process per GPU, NCCL): each rank runs its own set of
models (weak scaling; the N models are independent, no collective is on the
data path). ``--gather`` adds the optional output all-gather to every step.

``--impl reference`` times the reference's CPU implementation of the path
(the oracle's restatement of its torch op sequence) on rank 0 only.
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
import torch.nn as nn  # noqa: E402
import torch.nn.functional as F  # noqa: E402

METRIC = "wide-forward samples/s (N·B/s) at 1/2/4/8 B200; % of TC/HBM roofline"

# DRAM traffic (read + write bytes) per launch of linear_tc_kernel measured by
# ncu on a 16-model capture scaled to 64 models; see profiles/linear_tc_cfg2.md.
NCU_TRAFFIC_BYTES_CFG2 = 593_080_000


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm": float(p["hbm_gbs"]), "tensor_burst": float(p["bf16_tflops"]),
                "tensor_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "kind": "measured"}
    except Exception:
        return {"hbm": 6650.0, "tensor_burst": 1590.0, "tensor_sustained": 1400.0, "kind": "fallback"}


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


def _timed_cpu(fn, seconds):
    fn()
    t0 = time.perf_counter()
    reps = 0
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            return reps, el


# ---------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------

class Workload:
    """One BASELINE config: builds the wide module and resident inputs on a
    device, knows its per-step samples, algorithmic work and roofline."""
    name = ""
    dtype = "bf16"
    bound = "hbm"            # roofline of the dominant kernel(s)
    peak_key = "hbm"

    def forward(self, x):
        return self.module(x)

    def traffic(self):
        return None


class LinearCfg2(Workload):
    name = "cfg2"

    def torch_reference_step(self):
        """The reference's own GPU op sequence (wide_linear.py:162-171:
        einsum 'noi,nbi->nbo' + bias, cuBLAS through torch) on the same inputs."""
        w, b, x = self.module.weight, self.module.bias, self.x
        return lambda: torch.einsum('noi,nbi->nbo', w, x) + b.unsqueeze(1)

    def __init__(self, n=64, b=256, i=1024, o=4096):
        self.n, self.b, self.i, self.o = n, b, i, o

    def samples(self):
        return self.n * self.b

    def alg_bytes(self):
        return 2 * (self.n * self.o * self.i + self.n * self.b * self.i + self.n * self.b * self.o + self.n * self.o)

    def alg_flops(self):
        return 2 * self.n * self.b * self.i * self.o

    def traffic(self):
        return int(NCU_TRAFFIC_BYTES_CFG2 * self.n / 64)

    def config(self):
        return {"workload": f"WideLinear cfg2: N={self.n} models/GPU, in={self.i}, out={self.o}, B={self.b}, "
                            f"bf16, fp32 accumulate, bias fused",
                "models_per_gpu": self.n, "rows_per_model": self.b, "in_features": self.i,
                "out_features": self.o, "l2": "inputs larger than L2 (705 MB touched per step), no flush"}

    def setup(self, dev, seed):
        import wide_compiler as wc
        g = torch.Generator(device=dev).manual_seed(seed)
        lin = wc.WideLinear(self.n, self.i, self.o, bias=True).to(dev, torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(self.n, self.o, self.i, device=dev, generator=g) / self.i ** 0.5)
            lin.bias.zero_()
        self.module = lin
        self.x = torch.randn(self.n, self.b, self.i, device=dev, generator=g).to(torch.bfloat16)

    def cpu_sample(self, seconds):
        from oracle import wide_oracle as O
        n_s = 2
        g = torch.Generator().manual_seed(0)
        w = (torch.randn(n_s, self.o, self.i, generator=g) / 32).to(torch.bfloat16)
        b = torch.zeros(n_s, self.o, dtype=torch.bfloat16)
        x = torch.randn(n_s, self.b, self.i, generator=g).to(torch.bfloat16)
        reps, el = _timed_cpu(lambda: O.linear_ref_dtype(x, w, b), seconds)
        return reps * n_s * self.b / el, (f"{reps} reps x {n_s} of the {self.n} models (B={self.b}, "
                                          f"{self.i}->{self.o}, bf16) in {el:.1f} s, torch CPU einsum+bias")


class _MLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(64, 128)
        self.fc2 = nn.Linear(128, 64)

    def forward(self, x):
        return self.fc2(F.relu(self.fc1(x)))


class MlpCfg1(Workload):
    name = "cfg1"
    dtype = "fp32"
    bound = "fp32"           # one fused chain launch of CUDA-core fp32 FMAs

    def __init__(self, n=100, b=32):
        self.n, self.b = n, b

    def samples(self):
        return self.n * self.b

    def alg_flops(self):
        return 2 * self.n * self.b * (64 * 128 + 128 * 64)

    def alg_bytes(self):
        # whole-model compulsory bytes: x, W1, b1, W2, b2, y (fp32)
        return 4 * self.n * (self.b * 64 + 128 * 64 + 128 + 64 * 128 + 64 + self.b * 64)

    def config(self):
        return {"workload": f"cfg1 TracedWideModel of N={self.n} MLPs (Linear 64->128, ReLU, Linear 128->64), "
                            f"fp32, B={self.b}, packed input [{self.b}, {self.n * 64}]",
                "l2": "small working set (8 MB) stays in L2 between steps"}

    def setup(self, dev, seed):
        import wide_compiler as wc
        torch.manual_seed(seed)
        models = [_MLP().to(dev) for _ in range(self.n)]
        self.module = wc.compile(models, torch.randn(self.b, 64, device=dev))
        self.x = torch.randn(self.b, self.n * 64, device=dev)

    def cpu_sample(self, seconds):
        from oracle import wide_oracle as O
        g = torch.Generator().manual_seed(0)
        w1 = torch.randn(self.n, 128, 64, generator=g) / 8
        b1 = torch.zeros(self.n, 128)
        w2 = torch.randn(self.n, 64, 128, generator=g) / 11
        b2 = torch.zeros(self.n, 64)
        x = torch.randn(self.b, self.n * 64, generator=g)

        def run():
            xn = x.view(self.b, self.n, 64).movedim(1, 0).contiguous()
            y = O.mlp2_ref_dtype(xn, w1, b1, w2, b2)
            return y.movedim(0, 1).reshape(self.b, -1)
        reps, el = _timed_cpu(run, seconds)
        return reps * self.samples() / el, f"{reps} full cfg1 forwards in {el:.1f} s (fp32, torch CPU)"


class _ResBlock(nn.Module):
    def __init__(self, c=64):
        super().__init__()
        self.conv1 = nn.Conv2d(c, c, 3, padding=1)
        self.bn1 = nn.BatchNorm2d(c)
        self.conv2 = nn.Conv2d(c, c, 3, padding=1)
        self.bn2 = nn.BatchNorm2d(c)

    def forward(self, x):
        h = F.relu(self.bn1(self.conv1(x)))
        return self.bn2(self.conv2(h)) + x


class ResBlockCfg3(Workload):
    name = "cfg3"
    bound = "tensor"
    peak_key = "tensor_sustained"

    def torch_reference_step(self):
        """The reference's GPU op sequence for this graph (wide_conv2d.py:169-194
        permute + grouped conv, wide_batchnorm_2d.py:53-72 permute + BN,
        F.relu, + identity) with the same parameters, through torch (cuDNN)."""
        n, c, hw = self.n, self.c, self.hw
        st = self.module.stages
        conv1, bn1, conv2, bn2 = st['conv1'].grouped_conv, st['bn1'].op, st['conv2'].grouped_conv, st['bn2'].op
        x = self.x                                    # packed [B, N*C, H, W]

        def run():
            b = x.shape[0]
            h = F.batch_norm(F.conv2d(x, conv1.weight, conv1.bias, padding=1, groups=n), bn1.running_mean,
                             bn1.running_var, bn1.weight, bn1.bias, False, 0.0, bn1.eps)
            h = F.relu(h)
            y = F.batch_norm(F.conv2d(h, conv2.weight, conv2.bias, padding=1, groups=n), bn2.running_mean,
                             bn2.running_var, bn2.weight, bn2.bias, False, 0.0, bn2.eps)
            return y + x
        return run

    def __init__(self, n=100, b=32, c=64, hw=32):
        self.n, self.b, self.c, self.hw = n, b, c, hw

    def samples(self):
        return self.n * self.b

    def alg_flops(self):
        return 2 * 2 * self.n * self.b * self.hw * self.hw * self.c * self.c * 9

    def alg_bytes(self):
        return 2 * 2 * self.n * self.b * self.c * self.hw * self.hw   # fused block: x in, y out (bf16)

    def config(self):
        return {"workload": f"cfg3 TracedWideModel of N={self.n} ResBlocks (Conv3x3 {self.c}->{self.c} pad 1, BN "
                            f"eval, ReLU, Conv3x3, BN, + identity), B={self.b}, {self.hw}x{self.hw}, bf16",
                "l2": f"inputs larger than L2 ({self.n * self.b * self.c * self.hw * self.hw * 2 / 1e6:.0f} MB "
                      f"activation per step), no flush"}

    def setup(self, dev, seed):
        import wide_compiler as wc
        torch.manual_seed(seed)
        models = []
        for _ in range(self.n):
            m = _ResBlock(self.c)
            with torch.no_grad():
                for bn in (m.bn1, m.bn2):
                    bn.running_mean.normal_(0, 1)
                    bn.running_var.uniform_(0.5, 2.0)
                    bn.weight.uniform_(0.5, 1.5)
                    bn.bias.normal_(0, 0.1)
            models.append(m.to(dev, torch.bfloat16).eval())
        self.module = wc.compile(models, torch.randn(2, self.c, self.hw, self.hw, device=dev,
                                                     dtype=torch.bfloat16)).eval()
        self.x = torch.randn(self.b, self.n * self.c, self.hw, self.hw, device=dev).to(torch.bfloat16)

    def cpu_sample(self, seconds):
        from oracle import wide_oracle as O
        n_s, c = 1, self.c
        g = torch.Generator().manual_seed(0)
        bf = torch.bfloat16

        def mk(*s, sc=1.0):
            return (torch.randn(*s, generator=g) * sc).to(bf)

        def bn():
            return {'running_mean': mk(n_s * c), 'running_var': (torch.rand(n_s * c, generator=g) + 0.5).to(bf),
                    'weight': (torch.rand(n_s * c, generator=g) + 0.5).to(bf), 'bias': mk(n_s * c, sc=0.1)}
        c1w, c2w = mk(n_s * c, c, 3, 3, sc=1 / 24), mk(n_s * c, c, 3, 3, sc=1 / 24)
        c1b, c2b = mk(n_s * c, sc=0.1), mk(n_s * c, sc=0.1)
        bn1, bn2 = bn(), bn()
        x = mk(n_s, self.b, c, self.hw, self.hw)
        reps, el = _timed_cpu(lambda: O.resblock_ref_dtype(x, c1w, c1b, bn1, c2w, c2b, bn2), seconds)
        return reps * n_s * self.b / el, (f"{reps} reps x {n_s} of the {self.n} ResBlocks (B={self.b}, bf16) in "
                                          f"{el:.1f} s, torch CPU grouped conv + BN")


class RnnCfg4(Workload):
    dtype = "fp32"

    def __init__(self, kind, n=32, b=4, t=32, i=64, h=128):
        self.kind, self.n, self.b, self.t, self.i, self.h = kind, n, b, t, i, h
        self.name = f"cfg4{kind}"
        self.g = 3 if kind == "gru" else 4

    def samples(self):
        return self.n * self.b

    def alg_flops(self):
        return 2 * self.n * self.b * self.t * self.g * self.h * (self.i + self.h)

    def alg_bytes(self):
        return 4 * self.n * (self.b * self.t * (self.i + self.h) + self.g * self.h * (self.i + self.h)
                             + 2 * self.g * self.h)

    def config(self):
        return {"workload": f"cfg4 Wide{self.kind.upper()} N={self.n}, input {self.i}, hidden {self.h}, B={self.b}, "
                            f"T={self.t}, fp32 (TF32 off)",
                "l2": "small working set stays in L2 between steps"}

    def setup(self, dev, seed):
        import wide_compiler as wc
        torch.manual_seed(seed)
        cls = nn.GRU if self.kind == "gru" else nn.LSTM
        mods = [cls(self.i, self.h, batch_first=True) for _ in range(self.n)]
        wcls = wc.WideGRU if self.kind == "gru" else wc.WideLSTM
        self.module = wcls.from_modules(mods).to(dev)
        self.x = torch.randn(self.n, self.b, self.t, self.i, device=dev)

    def forward(self, x):
        return self.module(x)[0]

    def cpu_sample(self, seconds):
        from oracle import wide_oracle as O
        g = torch.Generator().manual_seed(0)
        s = 1 / self.h ** 0.5

        def u(*shape):
            return (torch.rand(*shape, generator=g) * 2 - 1) * s
        wih, whh = u(self.n, self.g * self.h, self.i), u(self.n, self.g * self.h, self.h)
        bih, bhh = u(self.n, self.g * self.h), u(self.n, self.g * self.h)
        x = torch.randn(self.n, self.b, self.t, self.i, generator=g)
        fn = O.gru_ref_dtype if self.kind == "gru" else O.lstm_ref_dtype
        reps, el = _timed_cpu(lambda: fn(x, wih, whh, bih, bhh), seconds)
        return reps * self.samples() / el, f"{reps} full cfg4 {self.kind} forwards in {el:.1f} s (fp32, torch CPU)"


class AttnCfg5(Workload):
    name = "cfg5"
    bound = "tensor"
    peak_key = "tensor_sustained"

    def torch_reference_step(self):
        """The reference's GPU op sequence (wide_attention.py:178-238 einsum
        projections, head split, SDPA causal, merge, out projection;
        wide_layernorm.py:41-67) with the same parameters, through torch."""
        a, ln, x = self.attn, self.ln, self.x
        n, d, hd = self.n, self.d, self.heads

        def run():
            _, b, t, _ = x.shape
            q = torch.einsum('nbtd,nod->nbto', x, a.q_weight) + a.q_bias.view(n, 1, 1, d)
            k = torch.einsum('nbtd,nod->nbto', x, a.kv_weight[:, :d]) + a.kv_bias[:, :d].view(n, 1, 1, d)
            v = torch.einsum('nbtd,nod->nbto', x, a.kv_weight[:, d:]) + a.kv_bias[:, d:].view(n, 1, 1, d)
            sp = lambda u: u.view(n, b, t, hd, d // hd).permute(0, 1, 3, 2, 4).reshape(n * b, hd, t, d // hd)
            o = F.scaled_dot_product_attention(sp(q), sp(k), sp(v), is_causal=True)
            o = o.view(n, b, hd, t, d // hd).permute(0, 1, 3, 2, 4).reshape(n, b, t, d)
            y = torch.einsum('nbtd,nod->nbto', o, a.out_weight) + a.out_bias.view(n, 1, 1, d)
            mean = y.mean(dim=-1, keepdim=True)
            var = y.var(dim=-1, unbiased=False, keepdim=True)
            return (y - mean) / torch.sqrt(var + ln.eps) * ln.weight.view(n, 1, 1, d) + ln.bias.view(n, 1, 1, d)
        return run

    def __init__(self, n=16, b=8, t=1024, d=512, heads=8):
        self.n, self.b, self.t, self.d, self.heads = n, b, t, d, heads

    def samples(self):
        return self.n * self.b

    def alg_flops(self):
        proj = 2 * self.n * self.b * self.t * self.d * self.d * 4
        core = 2 * 2 * self.n * self.b * self.heads * (self.t * self.t // 2) * (self.d // self.heads)
        return proj + core

    def alg_bytes(self):
        act = self.n * self.b * self.t * self.d * 2
        return act * 2 + 4 * self.n * self.d * self.d * 2 + act * 2     # x, y, weights, LN read + write

    def config(self):
        return {"workload": f"cfg5 WideAttention N={self.n}, d_model={self.d}, {self.heads} heads, causal, "
                            f"B={self.b}, T={self.t}, bf16, followed by WideLayerNorm({self.d})",
                "l2": "inputs larger than L2 (134 MB activation, ~0.5 GB of intermediates per step), no flush"}

    def setup(self, dev, seed):
        import wide_compiler as wc
        torch.manual_seed(seed)
        a = wc.WideAttention(self.n, self.d, self.heads)
        with torch.no_grad():
            for p in (a.q_weight, a.kv_weight, a.out_weight):
                p.normal_(0, 0.02)
            a.q_bias.zero_()
            a.kv_bias.zero_()
            a.out_bias.zero_()
        self.attn = a.to(dev, torch.bfloat16).eval()
        self.ln = wc.WideLayerNorm(self.n, self.d).to(dev, torch.bfloat16)
        self.module = self.attn
        self.x = torch.randn(self.n, self.b, self.t, self.d, device=dev).to(torch.bfloat16)

    def forward(self, x):
        return self.ln(self.attn(x, is_causal=True))

    def cpu_sample(self, seconds):
        from oracle import wide_oracle as O
        n_s = 1
        g = torch.Generator().manual_seed(0)
        bf = torch.bfloat16
        wq = (torch.randn(n_s, self.d, self.d, generator=g) * 0.02).to(bf)
        wkv = (torch.randn(n_s, 2 * self.d, self.d, generator=g) * 0.02).to(bf)
        wo = (torch.randn(n_s, self.d, self.d, generator=g) * 0.02).to(bf)
        lw, lb = torch.ones(n_s * self.d, dtype=bf), torch.zeros(n_s * self.d, dtype=bf)
        x = torch.randn(n_s, self.b, self.t, self.d, generator=g).to(bf)
        reps, el = _timed_cpu(lambda: O.attention_ln_ref_dtype(x, wq, wkv, wo, self.heads, lw, lb), seconds)
        return reps * n_s * self.b / el, (f"{reps} reps x {n_s} of the {self.n} models (B={self.b}, T={self.t}, "
                                          f"bf16) in {el:.1f} s, torch CPU einsum + SDPA + LN")


def make_workload(name, models=None):
    if name == "cfg2":
        return LinearCfg2(n=models or 64)
    if name == "cfg1":
        return MlpCfg1()
    if name == "cfg3":
        return ResBlockCfg3(n=models or 100)
    if name == "cfg4gru":
        return RnnCfg4("gru")
    if name == "cfg4lstm":
        return RnnCfg4("lstm")
    if name == "cfg5":
        return AttnCfg5()
    raise ValueError(name)


# ---------------------------------------------------------------------------
# Arms
# ---------------------------------------------------------------------------

def run_reference(args):
    """The reference's CPU path for the chosen workload, rank 0 only; each
    step is one bounded sample of the workload."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    wl = make_workload(args.workload, args.models)
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    per_step_s = max(0.0, args.ref_step_seconds)
    for _ in range(args.warmup):
        wl.cpu_sample(per_step_s)
    vals, desc = [], ""
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, desc = wl.cpu_sample(per_step_s)
        vals.append(v)
    el = time.perf_counter() - t0
    value = statistics.median(vals)
    line = {
        "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * el / max(args.steps, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
        "config": wl.config(), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                         "sample": f"median over steps; last step: {desc}"},
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
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = True
    from wide_compiler import _native
    _native.load()
    _native.check(_native.lib().widek_linear_set_variant(args.linear_variant), "widek_linear_set_variant")
    _native.check(_native.lib().widek_attention_set_variant(args.attn_variant), "widek_attention_set_variant")
    _native.check(_native.lib().widek_conv_set_variant(args.conv_variant), "widek_conv_set_variant")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    wl = make_workload(args.workload, args.models)
    wl.setup(dev, seed=1234 + rank)
    x = wl.x
    gather = args.gather and world > 1

    def step():
        y = wl.forward(x)
        if gather:
            from wide_compiler import parallel
            parallel.gather_outputs(y, y.shape[0] * world)
        return y

    def barrier():
        if pg:
            torch.distributed.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    run = step
    graph = None
    graph_launches = 0
    # TracedWideModel workloads run --graph through the library's own CUDA-graph
    # executor (what compile=True gives a user), for the timed loop and e2e;
    # the others capture the step here.
    from wide_compiler.core.traced_wide import TracedWideModel
    executor = bool(args.graph) and isinstance(getattr(wl, "module", None), TracedWideModel)
    if executor:
        from wide_compiler.core.graphed import GraphedWideModel
        n0 = _native.lib().widek_launch_count()
        wl.module(x)                          # one eager forward: the kernels a replay runs
        torch.cuda.synchronize(dev)
        graph_launches = _native.lib().widek_launch_count() - n0
        wl.module = GraphedWideModel(wl.module)
    elif args.graph:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                step()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        n0 = _native.lib().widek_launch_count()
        with torch.cuda.graph(graph):
            step()
        graph_launches = _native.lib().widek_launch_count() - n0   # kernels in one replay
        run = graph.replay

    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(max(args.warmup, 3)):
        run()
    barrier()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    launches0 = _native.lib().widek_launch_count()
    e0.record(stream)
    for _ in range(args.steps):
        run()
    e1.record(stream)
    # Our kernels launched in the timed region: counted by the library at
    # every launch (a graph replay runs the kernels counted at capture).
    gpu_launches = (graph_launches * args.steps if (graph is not None or executor)
                    else _native.lib().widek_launch_count() - launches0)
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if pg:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms_max = float(t.item())

    # End to end through the public API: every step copies its input from
    # pinned host memory to the device, runs the forward and copies the result
    # back to pinned host memory. The three run on separate streams with
    # double-buffered device inputs, so step i's upload, step i-1's forward
    # and step i-2's download overlap as in a serving pipeline.
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    x_host = x.cpu().pin_memory()
    y0 = wl.forward(x)
    y_host = [torch.empty(y0.shape, dtype=y0.dtype).pin_memory() for _ in range(2)]
    x_dev = [torch.empty_like(x) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        k = i % 2
        if i >= 2:
            s_in.wait_event(ev_comp[k])          # step i-2's forward has read x_dev[k]
            if executor:
                stream.wait_event(ev_out[k])     # and its result has been downloaded (a graph
                                                 # replay writes the same output tensor again)
        with torch.cuda.stream(s_in):
            x_dev[k].copy_(x_host, non_blocking=True)
            ev_in[k].record(s_in)
        stream.wait_event(ev_in[k])
        y = wl.forward(x_dev[k])
        if gather:
            from wide_compiler import parallel
            parallel.gather_outputs(y, y.shape[0] * world)
        ev_comp[k].record(stream)
        s_out.wait_event(ev_comp[k])
        with torch.cuda.stream(s_out):
            y_host[k].copy_(y, non_blocking=True)
            y.record_stream(s_out)
            ev_out[k].record(s_out)

    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    barrier()
    e0.record(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    stream.wait_stream(s_in)
    e1.record(stream)
    barrier()
    ms_e2e = e0.elapsed_time(e1) / e2e_steps
    t2 = torch.tensor([ms_e2e], device=dev, dtype=torch.float64)
    if pg:
        torch.distributed.all_reduce(t2, op=torch.distributed.ReduceOp.MAX)
    ms_e2e = float(t2.item())
    clk = clocks.stop()
    dev_err = _native.device_error()
    del graph

    if rank == 0:
        samples = wl.samples() * world
        pk = peaks()
        if wl.bound == "hbm":
            achieved = wl.alg_bytes() / (ms * 1e-3) / 1e9
            roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm"], "unit": "GB/s",
                    "frac": achieved / pk["hbm"], "peak_kind": f"{pk['kind']} HBM copy",
                    "traffic": wl.traffic(), "algorithmic_bytes": wl.alg_bytes(),
                    "tflops": wl.alg_flops() / (ms * 1e-3) / 1e12}
        elif wl.bound == "fp32":
            # CUDA-core fp32 FMA pipe: no measured figure exists for it, so the
            # nominal rate at the maximum SM clock is the denominator.
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            peak = sms * 128 * 2 * 1965e6 / 1e12
            achieved = wl.alg_flops() / (ms * 1e-3) / 1e12
            roof = {"bound": "fp32", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak,
                    "peak_kind": f"nominal fp32 FFMA ({sms} SMs x 128 lanes x 2 x 1965 MHz)",
                    "traffic": wl.traffic(), "algorithmic_flops": wl.alg_flops(),
                    "gbs": wl.alg_bytes() / (ms * 1e-3) / 1e9}
        else:
            achieved = wl.alg_flops() / (ms * 1e-3) / 1e12
            peak = pk[wl.peak_key]
            roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "peak_kind": f"{pk['kind']} bf16 dense ({wl.peak_key})",
                    "traffic": wl.traffic(), "algorithmic_flops": wl.alg_flops(),
                    "gbs": wl.alg_bytes() / (ms * 1e-3) / 1e9}
        cfg = wl.config()
        cfg["gather"] = bool(gather)
        cfg["cuda_graph"] = ("library CUDA-graph executor (compile=True)" if executor
                             else "step captured by the bench" if args.graph else False)
        cfg["linear_variant"] = "CTA-pair tiles" if args.linear_variant == 2 else "single-CTA tiles"
        if args.workload == "cfg3":
            cfg["conv_variant"] = "per-tap A tiles" if args.conv_variant == 1 else "halo-reuse A tiles"
        if args.workload == "cfg5":
            cfg["attention_variant"] = ("warp-level MMA" if args.attn_variant == 1 else
                                        "tcgen05/TMEM" + (f", {args.attn_variant - 10}/4 exp2 pairs on FMA"
                                                          if args.attn_variant >= 10 else ""))
        line = {
            "metric": METRIC, "value": samples / (ms_max * 1e-3), "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic", "config": cfg,
            "e2e": {"value": samples / (ms_e2e * 1e-3), "unit": "samples/s",
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                    "d2h_bytes_per_step": y_host[0].numel() * y_host[0].element_size(),
                    "steps": e2e_steps, "ms_per_step": ms_e2e,
                    "pipelined": "upload, forward and download on separate streams, double-buffered"},
            "gpu_launches": gpu_launches,
            "roofline": roof,
            "clocks": clk,
            "device_error": dev_err,
        }
        if world == 1 and hasattr(wl, "torch_reference_step"):
            # Extra column: the reference's torch GPU path (library kernels), same device, same inputs.
            fn = wl.torch_reference_step()
            with torch.no_grad():
                for _ in range(5):
                    fn()
                torch.cuda.synchronize(dev)
                e0.record(stream)
                for _ in range(args.steps):
                    fn()
                e1.record(stream)
                torch.cuda.synchronize(dev)
            tms = e0.elapsed_time(e1) / args.steps
            line["torch_gpu_reference"] = {"ms_per_step": tms, "value": wl.samples() / (tms * 1e-3),
                                           "unit": "samples/s",
                                           "note": "reference op sequence on this GPU via torch (cuBLAS/cuDNN/SDPA)"}
        if world == 1 and not args.no_cpu_baseline:
            torch.set_num_threads(len(os.sched_getaffinity(0)))
            v, desc = wl.cpu_sample(args.cpu_seconds)
            line["cpu_baseline"] = {"value": v, "unit": "samples/s", "cores": torch.get_num_threads(),
                                    "kind": "port", "sample": desc}
        print(json.dumps(line), flush=True)
    if pg:
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "cfg1", "cfg3", "cfg4gru", "cfg4lstm", "cfg5"])
    ap.add_argument("--models", type=int, default=None,
                    help="cfg2 models per GPU (default 64; smaller only for profiling captures)")
    ap.add_argument("--e2e-steps", type=int, default=100)
    ap.add_argument("--graph", action="store_true", help="replay each step from a CUDA graph")
    ap.add_argument("--gather", action="store_true", help="include the optional output all-gather")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-step-seconds", type=float, default=0.02,
                    help="reference arm: minimum CPU time of one step's bounded sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--linear-variant", type=int, default=0,
                    help="tensor-core GEMM tiling: 0 auto (single-CTA), 1 single-CTA tiles, 2 CTA-pair tiles")
    ap.add_argument("--attn-variant", type=int, default=0,
                    help="attention core: 0 tcgen05/TMEM kernel (default exponential split), 1 warp-level MMA "
                         "kernel, 10/11/12 tcgen05 with 0/1/2 of every 4 exponential pairs on the FMA pipe")
    ap.add_argument("--conv-variant", type=int, default=0,
                    help="tensor-core conv: 0 halo-reuse kernel where it applies, 1 per-tap kernel only")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    # An inference benchmark: autograd is off, so the fused kernels and the
    # CUDA-graph executor serve every forward (as they do under no_grad for a user).
    with torch.no_grad():
        return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
