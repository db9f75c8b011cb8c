"""Benchmark of the wide forward path on B200 (one JSON line on rank 0).

Headline workload: cfg3, the largest of the reference's configurations that
fits one GPU: a TracedWideModel of N=100 ResBlocks (Conv3x3 64->64, BatchNorm
eval, ReLU, Conv3x3, BatchNorm, + identity), B=32, 32x32, bf16, packed input
[32, 6400, 32, 32]. A step is one wide forward over the whole batch. Every
other configuration (cfg1 MLP and cfg5 attention -> LayerNorm as
TracedWideModels, cfg2 WideLinear, cfg4 GRU/LSTM) and four memory-bound norm
workloads are measured in the same run and reported under "configs" with
the same keys. Two training-step workloads (forward + backward: cfg2train,
lntrain) run only when named with --workload.

  value   samples/s = N*B / t_step; t_step from CUDA events over K
          back-to-back steps with inputs resident in HBM; max over ranks.
  e2e     the same metric through the public API call with the step's input
          copied host->device from pinned memory and the output copied back
          inside the timed region (upload, forward and download pipelined on
          three streams, double-buffered).
  roofline  the dominant kernel (the library entry point with the most device
          time per step): its algorithmic FLOPs or bytes per launch over its
          mean launch time, both from CUDA events around each launch inside
          the timed region (a CUDA-graph replay counts as one launch), against
          the measured peak in MEASURED_PEAKS.json.
  cpu_baseline  the reference's op sequence (its torch arithmetic in the
          configuration's dtype) for the whole workload, all N models, on the
          host cores; rank 0, one GPU only.

Multi-GPU (torchrun, one process per GPU, NCCL): the N models of each
configuration are split into contiguous slices, one per rank (strong scaling:
the total work is fixed; ``--weak`` gives every rank all N). No collective is
on the data path; ``--gather`` adds the optional output all-gather to every
step.

``--impl reference`` times the reference's CPU implementation of the path
(the oracle's restatement of its torch op sequence) on rank 0 only, for the
same configurations, each step one full forward of the whole workload.
"""
from __future__ import annotations

import argparse
import json
import math
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
HEADLINE = "cfg3"
ORDER = ["cfg3", "cfg1", "cfg2", "cfg4gru", "cfg4lstm", "cfg5", "bn2d_eval", "bn2d_train", "gn", "ln"]
TRAINING = ["cfg2train", "lntrain"]      # forward + backward steps, run only when named

# DRAM traffic (read + write bytes) per launch of the dominant kernel, from
# one ncu capture of a reduced case scaled to the full launch by the units it
# processes (traffic grows in proportion): None where no capture exists.
NCU_TRAFFIC_PER_LAUNCH = {
    # linear_tc_kernel: 148.27 MB over a 16-model cfg2 launch, x4 for 64 models
    "cfg2": 593_080_000,
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm": float(p["hbm_gbs"]), "tensor_burst": float(p["bf16_tflops"]),
                "tensor_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "kind": "measured"}
    except Exception:
        return {"hbm": 6650.0, "tensor_burst": 1590.0, "tensor_sustained": 1400.0, "kind": "fallback"}


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the GPU is busy.
    nvidia-smi writes to a pseudo-terminal, so that it line-buffers and each
    sample arrives (and is time-stamped) when it is taken."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []                  # (arrival time, line)
        self._t = None
        self._fd = None
        self.t_start = 0.0

    def start(self):
        try:
            import pty
            master, slave = pty.openpty()
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdin=subprocess.DEVNULL, stdout=slave, stderr=subprocess.DEVNULL, close_fds=True)
            os.close(slave)
            self._fd = master
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
            return
        # wait (bounded) for the first sample, so that a short run still has
        # samples in its window
        t0 = self.t_start = time.perf_counter()
        while not self.lines and self.proc.poll() is None and time.perf_counter() - t0 < 30.0:
            time.sleep(0.02)

    def _read(self):
        buf = b""
        while True:
            try:
                chunk = os.read(self._fd, 4096)
            except OSError:              # the terminal closes when nvidia-smi exits
                break
            if not chunk:
                break
            buf += chunk
            while b"\n" in buf:
                line, buf = buf.split(b"\n", 1)
                self.lines.append((time.perf_counter(), line.decode(errors="replace").strip()))

    def mark(self):
        return time.perf_counter()

    def stop(self):
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        try:
            os.close(self._fd)
        except OSError:
            pass

    def summary(self, start=0.0, end=None):
        """Samples that arrived between the marks start and end."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for t, ln in list(self.lines):
            if t < start or (end is not None and t > end):
                continue
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
    """Runs fn once untimed, then repeatedly until `seconds` have passed
    (at least once); returns (reps, elapsed)."""
    fn()
    t0 = time.perf_counter()
    reps = 0
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            return reps, el


def shard_range(n, world, rank):
    from wide_compiler.parallel import shard_range as sr
    return sr(n, world, rank)


# ---------------------------------------------------------------------------
# Workloads. Each builds models [lo, hi) of its deterministic set of N models
# (model j is initialised from seed + j, so any split of N across ranks runs
# the same models) and that slice's resident input.
# ---------------------------------------------------------------------------

class Workload:
    name = ""
    dtype = "bf16"
    bound = "hbm"            # roofline of the dominant kernel: hbm | tensor | fp32
    peak_key = "hbm"
    graph = False            # capture the step in a CUDA graph in the bench
    n_total = 1
    b = 1

    def setup(self, dev, lo, hi, seed):
        raise NotImplementedError

    def step(self, x):
        return self.module(x)

    def samples(self, n_models):
        return n_models * self.b

    def work(self, n_models):
        """{entry point: algorithmic FLOPs (tensor / fp32 bound) or bytes (hbm
        bound) per step} for n_models models."""
        raise NotImplementedError

    def traffic(self, n_models):
        t = NCU_TRAFFIC_PER_LAUNCH.get(self.name)
        return None if t is None else int(t * n_models / self.n_total)

    def config(self):
        raise NotImplementedError

    def cpu_workload(self):
        """(fn, samples per call, description): one full forward of the whole
        workload (all N models) with the reference's op sequence on the host."""
        raise NotImplementedError


def _gen(seed):
    return torch.Generator().manual_seed(seed)


class LinearCfg2(Workload):
    name = "cfg2"

    def __init__(self, n=64, b=256, i=1024, o=4096):
        self.n_total, self.b, self.i, self.o = n, b, i, o

    def _bytes(self, n):
        return 2 * (n * self.o * self.i + n * self.b * self.i + n * self.b * self.o + n * self.o)

    def work(self, n):
        return {"widek_linear_fwd": self._bytes(n)}

    def flops(self, n):
        return 2 * n * self.b * self.i * self.o

    def config(self):
        return {"workload": f"cfg2 WideLinear N={self.n_total}, in={self.i}, out={self.o}, B={self.b} rows per "
                            f"model, bf16, fp32 accumulate, bias fused; W ~ N(0, 1/in), bias 0, x ~ N(0, 1)",
                "models": self.n_total, "rows_per_model": self.b,
                "l2": "inputs larger than L2 (705 MB touched per step), no flush"}

    def setup(self, dev, lo, hi, seed):
        import wide_compiler as wc
        n = hi - lo
        lin = wc.WideLinear(n, self.i, self.o, bias=True).to(dev, torch.bfloat16)
        with torch.no_grad():
            for k, j in enumerate(range(lo, hi)):
                g = torch.Generator(device=dev).manual_seed(seed + j)
                lin.weight[k].copy_(torch.randn(self.o, self.i, device=dev, generator=g) / self.i ** 0.5)
            lin.bias.zero_()
        self.module = lin
        self.x = torch.empty(n, self.b, self.i, device=dev, dtype=torch.bfloat16)
        for k, j in enumerate(range(lo, hi)):
            g = torch.Generator(device=dev).manual_seed(seed + 100_000 + j)
            self.x[k].copy_(torch.randn(self.b, self.i, device=dev, generator=g))

    def torch_reference_step(self):
        """The reference's GPU op sequence (wide_linear.py:162-171: einsum
        'noi,nbi->nbo' + bias, cuBLAS through torch) on the same inputs."""
        w, b, x = self.module.weight, self.module.bias, self.x
        return lambda: torch.einsum('noi,nbi->nbo', w, x) + b.unsqueeze(1)

    def cpu_workload(self):
        from oracle import wide_oracle as O
        g = _gen(0)
        n = self.n_total
        w = (torch.randn(n, self.o, self.i, generator=g) / 32).to(torch.bfloat16)
        b = torch.zeros(n, self.o, dtype=torch.bfloat16)
        x = torch.randn(n, self.b, self.i, generator=g).to(torch.bfloat16)
        return (lambda: O.linear_ref_dtype(x, w, b)), n * self.b, \
            f"one full cfg2 forward per rep (all {n} models, B={self.b}), torch CPU einsum + bias in bf16"


class _MLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(64, 128)
        self.fc2 = nn.Linear(128, 64)

    def forward(self, x):
        return self.fc2(F.relu(self.fc1(x)))


class _Traced(Workload):
    """A TracedWideModel workload through the multi-GPU wrapper (this rank's
    slice of the models; packed input [B, n_local*C, ...])."""
    compile_model = False

    def build(self, dev, dtype, models, sample, per_model_inputs):
        """models: all N (host); this rank's slice is fused and moved to dev."""
        import wide_compiler as wc
        from wide_compiler import parallel
        world, rank = self._world_rank
        self.module = parallel.ShardedWideModel(models, sample, rank=rank, world=world,
                                                gather=self._gather, compile_model=self.compile_model,
                                                gather_chunks=getattr(self, '_gather_chunks', 1))
        self.module.to(dev, dtype).eval()
        self.x = wc.pack([t.to(dev, dtype) for t in per_model_inputs])


class MlpCfg1(_Traced):
    name = "cfg1"
    dtype = "fp32"
    bound = "fp32"
    compile_model = True      # the library's CUDA-graph executor (compile=True)

    def __init__(self, n=100, b=32):
        self.n_total, self.b = n, b

    def flops(self, n):
        return 2 * n * self.b * (64 * 128 + 128 * 64)

    def work(self, n):
        return {"graph replay": self.flops(n)}

    def config(self):
        return {"workload": f"cfg1 TracedWideModel of N={self.n_total} MLPs (Linear 64->128, ReLU, Linear "
                            f"128->64), fp32 (TF32 off), B={self.b}, packed input [{self.b}, {self.n_total * 64}], "
                            f"compile=True (CUDA-graph executor)",
                "models": self.n_total, "rows_per_model": self.b,
                "l2": "small working set (8 MB) stays in L2 between steps"}

    def setup(self, dev, lo, hi, seed):
        models, xs = [], []
        for j in range(self.n_total):
            torch.manual_seed(seed + j)
            models.append(_MLP())
        for j in range(lo, hi):
            xs.append(torch.randn(self.b, 64, generator=_gen(seed + 100_000 + j)))
        self.build(dev, torch.float32, models, torch.randn(self.b, 64), xs)

    def cpu_workload(self):
        from oracle import wide_oracle as O
        g = _gen(0)
        n = self.n_total
        w1 = torch.randn(n, 128, 64, generator=g) / 8
        b1 = torch.zeros(n, 128)
        w2 = torch.randn(n, 64, 128, generator=g) / 11
        b2 = torch.zeros(n, 64)
        x = torch.randn(self.b, n * 64, generator=g)

        def run():
            xn = x.view(self.b, n, 64).movedim(1, 0).contiguous()
            y = O.mlp2_ref_dtype(xn, w1, b1, w2, b2)
            return y.movedim(0, 1).reshape(self.b, -1)
        return run, n * self.b, f"one full cfg1 forward per rep (all {n} MLPs, B={self.b}), fp32, torch CPU"


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


def resblock_model(c, seed):
    """One cfg3 ResBlock: default conv init from `seed`, BatchNorm in eval with
    running_mean ~ N(0, 1), running_var ~ U(0.5, 2), weight ~ U(0.5, 1.5),
    bias ~ N(0, 0.1)."""
    torch.manual_seed(seed)
    m = _ResBlock(c)
    with torch.no_grad():
        for bn in (m.bn1, m.bn2):
            bn.running_mean.normal_(0, 1)
            bn.running_var.uniform_(0.5, 2.0)
            bn.weight.uniform_(0.5, 1.5)
            bn.bias.normal_(0, 0.1)
    return m.eval()


class ResBlockCfg3(_Traced):
    name = "cfg3"
    bound = "tensor"
    peak_key = "tensor_sustained"

    def __init__(self, n=100, b=32, c=64, hw=32):
        self.n_total, self.b, self.c, self.hw = n, b, c, hw

    def flops(self, n):
        return 2 * 2 * n * self.b * self.hw * self.hw * self.c * self.c * 9

    def work(self, n):
        return {"widek_conv_fwd_ex": self.flops(n)}

    def config(self):
        return {"workload": f"cfg3 TracedWideModel of N={self.n_total} ResBlocks (Conv3x3 {self.c}->{self.c} pad 1, "
                            f"BatchNorm eval, ReLU, Conv3x3, BatchNorm, + identity), B={self.b}, {self.hw}x{self.hw}, "
                            f"bf16, packed input [{self.b}, {self.n_total * self.c}, {self.hw}, {self.hw}]",
                "models": self.n_total, "rows_per_model": self.b,
                "l2": f"inputs larger than L2 ({self.n_total * self.b * self.c * self.hw * self.hw * 2 / 1e6:.0f} MB "
                      f"activation per step), no flush"}

    def setup(self, dev, lo, hi, seed):
        models = [resblock_model(self.c, seed + j) for j in range(self.n_total)]
        xs = [torch.randn(self.b, self.c, self.hw, self.hw, generator=_gen(seed + 100_000 + j))
              for j in range(lo, hi)]
        self.build(dev, torch.bfloat16, models, torch.randn(2, self.c, self.hw, self.hw), xs)

    def torch_reference_step(self):
        """The reference's GPU op sequence for this graph (wide_conv2d.py:169-194
        grouped conv, wide_batchnorm_2d.py:53-72 BN, F.relu, + identity) with
        the same parameters on the packed input, through torch (cuDNN)."""
        st = self.module.local.stages
        n = self.module.n_local
        conv1, bn1, conv2, bn2 = st['conv1'].grouped_conv, st['bn1'].op, st['conv2'].grouped_conv, st['bn2'].op
        x = self.x

        def run():
            h = F.batch_norm(F.conv2d(x, conv1.weight, conv1.bias, padding=1, groups=n), bn1.running_mean,
                             bn1.running_var, bn1.weight, bn1.bias, False, 0.0, bn1.eps)
            h = F.relu(h)
            y = F.batch_norm(F.conv2d(h, conv2.weight, conv2.bias, padding=1, groups=n), bn2.running_mean,
                             bn2.running_var, bn2.weight, bn2.bias, False, 0.0, bn2.eps)
            return y + x
        return run

    def cpu_workload(self):
        from oracle import wide_oracle as O
        n, c = self.n_total, self.c
        g = _gen(0)
        bf = torch.bfloat16

        def mk(*s, sc=1.0):
            return (torch.randn(*s, generator=g) * sc).to(bf)

        def bn():
            return {'running_mean': mk(n * c), 'running_var': (torch.rand(n * c, generator=g) * 1.5 + 0.5).to(bf),
                    'weight': (torch.rand(n * c, generator=g) + 0.5).to(bf), 'bias': mk(n * c, sc=0.1)}
        c1w, c2w = mk(n * c, c, 3, 3, sc=1 / 24), mk(n * c, c, 3, 3, sc=1 / 24)
        c1b, c2b = mk(n * c, sc=0.1), mk(n * c, sc=0.1)
        bn1, bn2 = bn(), bn()
        x = mk(n, self.b, c, self.hw, self.hw)
        return (lambda: O.resblock_ref_dtype(x, c1w, c1b, bn1, c2w, c2b, bn2)), n * self.b, \
            (f"one full cfg3 forward per rep (all {n} ResBlocks, B={self.b}), bf16, torch CPU grouped conv + BN "
             f"(groups=N, as the reference)")


class RnnCfg4(Workload):
    dtype = "fp32"
    bound = "fp32"
    graph = True

    def __init__(self, kind, n=32, b=4, t=32, i=64, h=128):
        self.kind, self.n_total, self.b, self.t, self.i, self.h = kind, n, b, t, i, h
        self.name = f"cfg4{kind}"
        self.g = 3 if kind == "gru" else 4

    def flops(self, n):
        return 2 * n * self.b * self.t * self.g * self.h * (self.i + self.h)

    def work(self, n):
        return {"graph replay": self.flops(n)}

    def config(self):
        return {"workload": f"cfg4 Wide{self.kind.upper()} N={self.n_total}, input {self.i}, hidden {self.h}, "
                            f"B={self.b}, T={self.t}, fp32 (TF32 off), U(+-1/sqrt(H)) init, step replayed from a "
                            f"CUDA graph",
                "models": self.n_total, "rows_per_model": self.b,
                "l2": "small working set stays in L2 between steps"}

    def setup(self, dev, lo, hi, seed):
        import wide_compiler as wc
        cls = nn.GRU if self.kind == "gru" else nn.LSTM
        mods = []
        for j in range(lo, hi):
            torch.manual_seed(seed + j)
            mods.append(cls(self.i, self.h, batch_first=True))
        wcls = wc.WideGRU if self.kind == "gru" else wc.WideLSTM
        self.module = wcls.from_modules(mods).to(dev)
        self.x = torch.stack([torch.randn(self.b, self.t, self.i, generator=_gen(seed + 100_000 + j))
                              for j in range(lo, hi)]).to(dev)

    def step(self, x):
        return self.module(x)[0]

    def cpu_workload(self):
        from oracle import wide_oracle as O
        g = _gen(0)
        n = self.n_total
        s = 1 / self.h ** 0.5

        def u(*shape):
            return (torch.rand(*shape, generator=g) * 2 - 1) * s
        wih, whh = u(n, self.g * self.h, self.i), u(n, self.g * self.h, self.h)
        bih, bhh = u(n, self.g * self.h), u(n, self.g * self.h)
        x = torch.randn(n, self.b, self.t, self.i, generator=g)
        fn = O.gru_ref_dtype if self.kind == "gru" else O.lstm_ref_dtype
        return (lambda: fn(x, wih, whh, bih, bhh)), n * self.b, \
            f"one full cfg4 {self.kind} forward per rep (all {n} models), fp32, torch CPU"


class _AttnLN(nn.Module):
    """One cfg5 model: causal self-attention (nn.MultiheadAttention, batch
    first) followed by LayerNorm."""

    def __init__(self, d, heads):
        super().__init__()
        self.attn = nn.MultiheadAttention(d, heads, batch_first=True)
        self.ln = nn.LayerNorm(d)

    def forward(self, x):
        a, _ = self.attn(x, x, x, need_weights=False, is_causal=True)
        return self.ln(a)


class AttnCfg5(_Traced):
    """cfg5 through wide_compiler.compile: a TracedWideModel of N (attention
    -> LayerNorm) models on the packed input [B, N*T, D]. The QKV projection
    reads the packed rows in place, the output projection runs with the
    LayerNorm in its epilogue and writes the packed output."""
    name = "cfg5"
    bound = "tensor"
    peak_key = "tensor_sustained"

    def __init__(self, n=16, b=8, t=1024, d=512, heads=8):
        self.n_total, self.b, self.t, self.d, self.heads = n, b, t, d, heads

    def work(self, n):
        core = 2 * 2 * n * self.b * self.heads * (self.t * (self.t + 1) // 2) * (self.d // self.heads)
        proj = 2 * n * self.b * self.t * self.d * self.d * 4
        return {"widek_attention_fwd": core, "widek_linear_fwd_ex": proj * 3 // 4,
                "widek_linear_ln_fwd_ex": proj // 4}

    def flops(self, n):
        return sum(self.work(n).values())

    def config(self):
        return {"workload": f"cfg5 TracedWideModel of N={self.n_total} (MultiheadAttention d_model={self.d}, "
                            f"{self.heads} heads, causal self-attention -> LayerNorm({self.d})), B={self.b}, "
                            f"T={self.t}, bf16, weights ~ N(0, 0.02), biases 0, packed input "
                            f"[{self.b}, {self.n_total * self.t}, {self.d}]",
                "models": self.n_total, "rows_per_model": self.b,
                "l2": "inputs larger than L2 (134 MB activation, ~0.5 GB of intermediates per step), no flush"}

    def setup(self, dev, lo, hi, seed):
        models = []
        for j in range(self.n_total):
            m = _AttnLN(self.d, self.heads)
            g = _gen(seed + j)
            with torch.no_grad():
                m.attn.in_proj_weight.copy_(torch.randn(m.attn.in_proj_weight.shape, generator=g) * 0.02)
                m.attn.out_proj.weight.copy_(torch.randn(m.attn.out_proj.weight.shape, generator=g) * 0.02)
                m.attn.in_proj_bias.zero_()
                m.attn.out_proj.bias.zero_()
            models.append(m.eval())
        xs = [torch.randn(self.b, self.t, self.d, generator=_gen(seed + 100_000 + j)) for j in range(lo, hi)]
        self.build(dev, torch.bfloat16, models, torch.randn(2, self.t, self.d), xs)

    def torch_reference_step(self):
        """The reference's GPU op sequence (wide_attention.py:178-238 einsum
        projections, head split, SDPA causal, merge, out projection;
        wide_layernorm.py:41-67) with the same parameters, through torch."""
        st = self.module.local.stages
        a, ln = st['attn'], st['ln']
        n, d, hd = a.n, self.d, self.heads
        b, t = self.b, self.t
        x = self.x.view(b, n, t, d).transpose(0, 1)

        def run():
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

    def cpu_workload(self):
        from oracle import wide_oracle as O
        n = self.n_total
        g = _gen(0)
        bf = torch.bfloat16
        wq = (torch.randn(n, self.d, self.d, generator=g) * 0.02).to(bf)
        wkv = (torch.randn(n, 2 * self.d, self.d, generator=g) * 0.02).to(bf)
        wo = (torch.randn(n, self.d, self.d, generator=g) * 0.02).to(bf)
        lw, lb = torch.ones(n * self.d, dtype=bf), torch.zeros(n * self.d, dtype=bf)
        x = torch.randn(n, self.b, self.t, self.d, generator=g).to(bf)
        return (lambda: O.attention_ln_ref_dtype(x, wq, wkv, wo, self.heads, lw, lb)), n * self.b, \
            f"one full cfg5 forward per rep (all {n} models, B={self.b}, T={self.t}), bf16, torch CPU einsum + " \
            f"SDPA + LN"


class _Norm(Workload):
    """A wide norm over a working set far above L2."""

    def _act_bytes(self, n):
        return n * self.rows * self.elem * 2

    def samples(self, n):
        return n * self.b


class BatchNormWl(_Norm):
    def __init__(self, training, n=100, b=32, c=64, hw=32):
        self.training = training
        self.name = "bn2d_train" if training else "bn2d_eval"
        self.n_total, self.b, self.c, self.hw = n, b, c, hw

    def work(self, n):
        act = n * self.b * self.c * self.hw * self.hw * 2
        entry = "widek_batchnorm_train_fwd" if self.training else "widek_batchnorm_fwd"
        return {entry: 2 * act}        # compulsory: read x once, write y once (bf16)

    def config(self):
        mode = ("training mode (batch statistics, running-stat update)" if self.training
                else "eval mode (running statistics)")
        return {"workload": f"WideBatchNorm2d N={self.n_total}, C={self.c}, B={self.b}, {self.hw}x{self.hw}, bf16, "
                            f"{mode}; the cfg3 BatchNorm shape, 419 MB in + 419 MB out",
                "models": self.n_total, "rows_per_model": self.b,
                "l2": "input larger than L2 (419 MB), no flush"}

    def setup(self, dev, lo, hi, seed):
        import wide_compiler as wc
        n = hi - lo
        m = wc.WideBatchNorm2d(n, self.c).to(dev, torch.bfloat16)
        g = _gen(seed + lo)
        with torch.no_grad():
            m.op.running_mean.copy_(torch.randn(n * self.c, generator=g))
            m.op.running_var.copy_(torch.rand(n * self.c, generator=g) * 1.5 + 0.5)
            m.op.weight.copy_(torch.rand(n * self.c, generator=g) + 0.5)
            m.op.bias.copy_(torch.randn(n * self.c, generator=g) * 0.1)
        self.module = m.train(self.training)
        self.x = torch.randn(n, self.b, self.c, self.hw, self.hw, device=dev,
                             generator=torch.Generator(device=dev).manual_seed(seed + lo)).to(torch.bfloat16)

    def cpu_workload(self):
        from oracle import wide_oracle as O
        n, c = self.n_total, self.c
        g = _gen(0)
        bf = torch.bfloat16
        x = torch.randn(n, self.b, c, self.hw, self.hw, generator=g).to(bf)
        rm, rv = torch.zeros(n * c, dtype=bf), torch.ones(n * c, dtype=bf)
        w, bb = torch.ones(n * c, dtype=bf), torch.zeros(n * c, dtype=bf)
        return (lambda: O.batchnorm2d_ref_dtype(x, rm, rv, w, bb, self.training)), n * self.b, \
            f"one full pass per rep (all {n} models), bf16, torch CPU permute + batch_norm + permute"


class GroupNormWl(_Norm):
    name = "gn"

    def __init__(self, n=100, b=32, c=64, groups=8, hw=32):
        self.n_total, self.b, self.c, self.groups, self.hw = n, b, c, groups, hw

    def work(self, n):
        return {"widek_groupnorm_fwd": 2 * n * self.b * self.c * self.hw * self.hw * 2}

    def config(self):
        return {"workload": f"WideGroupNorm N={self.n_total}, {self.groups} groups of C={self.c}, B={self.b}, "
                            f"{self.hw}x{self.hw}, bf16, affine; 419 MB in + 419 MB out",
                "models": self.n_total, "rows_per_model": self.b, "l2": "input larger than L2 (419 MB), no flush"}

    def setup(self, dev, lo, hi, seed):
        import wide_compiler as wc
        n = hi - lo
        m = wc.WideGroupNorm(n, self.groups, self.c).to(dev, torch.bfloat16)
        g = _gen(seed + lo)
        with torch.no_grad():
            m.norm.weight.copy_(torch.rand(n * self.c, generator=g) + 0.5)
            m.norm.bias.copy_(torch.randn(n * self.c, generator=g) * 0.1)
        self.module = m
        self.x = torch.randn(n, self.b, self.c, self.hw, self.hw, device=dev,
                             generator=torch.Generator(device=dev).manual_seed(seed + lo)).to(torch.bfloat16)

    def cpu_workload(self):
        from oracle import wide_oracle as O
        n, c = self.n_total, self.c
        g = _gen(0)
        bf = torch.bfloat16
        x = torch.randn(n, self.b, c, self.hw, self.hw, generator=g).to(bf)
        w, bb = torch.ones(n * c, dtype=bf), torch.zeros(n * c, dtype=bf)
        return (lambda: O.groupnorm_ref_dtype(x, self.groups, w, bb)), n * self.b, \
            f"one full pass per rep (all {n} models), bf16, torch CPU permute + group_norm + permute"


class LayerNormWl(_Norm):
    name = "ln"

    def __init__(self, n=16, b=32, t=1024, d=512):
        self.n_total, self.b, self.t, self.d = n, b, t, d

    def work(self, n):
        return {"widek_layernorm_fwd": 2 * n * self.b * self.t * self.d * 2}

    def config(self):
        return {"workload": f"WideLayerNorm N={self.n_total}, d={self.d}, B={self.b}, T={self.t}, bf16 (the cfg5 "
                            f"LayerNorm at 4x its batch: 537 MB in + 537 MB out)",
                "models": self.n_total, "rows_per_model": self.b, "l2": "input larger than L2 (537 MB), no flush"}

    def setup(self, dev, lo, hi, seed):
        import wide_compiler as wc
        n = hi - lo
        m = wc.WideLayerNorm(n, self.d).to(dev, torch.bfloat16)
        g = _gen(seed + lo)
        with torch.no_grad():
            m.weight.copy_(torch.rand(n * self.d, generator=g) + 0.5)
            m.bias.copy_(torch.randn(n * self.d, generator=g) * 0.1)
        self.module = m
        self.x = torch.randn(n, self.b, self.t, self.d, device=dev,
                             generator=torch.Generator(device=dev).manual_seed(seed + lo)).to(torch.bfloat16)

    def cpu_workload(self):
        from oracle import wide_oracle as O
        n = self.n_total
        g = _gen(0)
        bf = torch.bfloat16
        x = torch.randn(n, self.b, self.t, self.d, generator=g).to(bf)
        w, bb = torch.ones(n * self.d, dtype=bf), torch.zeros(n * self.d, dtype=bf)
        return (lambda: O.layernorm_ref_dtype(x, w, bb, n, self.d)), n * self.b, \
            f"one full pass per rep (all {n} models), bf16, torch CPU mean/var/normalize/affine"


class LinearCfg2Train(LinearCfg2):
    """cfg2's WideLinear trained one step: forward, then the backward kernels
    (dX, dW, db) for a fixed upstream gradient. Not in the default set; run
    with --workload cfg2train. The dominant entry is widek_linear_bwd, bound
    by the tensor pipe (two GEMMs of the forward's size) plus the transposes
    that give them K-major operands."""
    name = "cfg2train"
    bound = "tensor"
    peak_key = "tensor_sustained"

    def work(self, n):
        return {"widek_linear_bwd": 2 * 2 * n * self.b * self.i * self.o,
                "widek_linear_fwd": 2 * n * self.b * self.i * self.o}

    def config(self):
        c = super().config()
        c["workload"] = c["workload"].replace("cfg2 WideLinear", "cfg2 WideLinear training step (forward + "
                                              "backward: dX, dW, db for a fixed upstream gradient)")
        return c

    def setup(self, dev, lo, hi, seed):
        super().setup(dev, lo, hi, seed)
        g = torch.Generator(device=dev).manual_seed(seed + 7)
        self.dy = torch.randn(hi - lo, self.b, self.o, device=dev, generator=g).to(torch.bfloat16)

    def step(self, x):
        m = self.module
        m.weight.grad = None
        m.bias.grad = None
        xg = x.detach().requires_grad_(True)
        with torch.enable_grad():
            m(xg).backward(self.dy)
        return xg.grad

    def torch_reference_step(self):
        """The reference's training step on this GPU: its einsum + bias
        forward differentiated by torch autograd (cuBLAS)."""
        w = self.module.weight.detach().requires_grad_(True)
        b = self.module.bias.detach().requires_grad_(True)

        def fn():
            w.grad = None
            b.grad = None
            xg = self.x.detach().requires_grad_(True)
            with torch.enable_grad():
                (torch.einsum('noi,nbi->nbo', w, xg) + b.unsqueeze(1)).backward(self.dy)
            return xg.grad
        return fn

    def cpu_workload(self):
        n = max(1, self.n_total // 32)
        g = _gen(0)
        w = (torch.randn(n, self.o, self.i, generator=g) / 32).to(torch.bfloat16).requires_grad_(True)
        b = torch.zeros(n, self.o, dtype=torch.bfloat16, requires_grad=True)
        x = torch.randn(n, self.b, self.i, generator=g).to(torch.bfloat16).requires_grad_(True)
        dy = torch.randn(n, self.b, self.o, generator=g).to(torch.bfloat16)

        def fn():
            for t in (w, b, x):
                t.grad = None
            (torch.einsum('noi,nbi->nbo', w, x) + b.unsqueeze(1)).backward(dy)
        return fn, n * self.b, f"{n} of the {self.n_total} models per rep: torch CPU einsum + bias, autograd backward"


class LayerNormTrain(LayerNormWl):
    """The cfg5 LayerNorm (at 4x its batch) trained one step: forward, then
    widek_layernorm_bwd (dX, dgamma, dbeta). Not in the default set; run with
    --workload lntrain."""
    name = "lntrain"

    def work(self, n):
        elems = n * self.b * self.t * self.d
        return {"widek_layernorm_bwd": 3 * elems * 2, "widek_layernorm_fwd": 2 * elems * 2}

    def config(self):
        c = super().config()
        c["workload"] = c["workload"].replace("WideLayerNorm", "WideLayerNorm training step (forward + backward: "
                                              "dX, dgamma, dbeta for a fixed upstream gradient)", 1)
        return c

    def setup(self, dev, lo, hi, seed):
        super().setup(dev, lo, hi, seed)
        self.dy = torch.randn(self.x.shape, device=dev,
                              generator=torch.Generator(device=dev).manual_seed(seed + 7)).to(torch.bfloat16)

    def step(self, x):
        m = self.module
        m.weight.grad = None
        m.bias.grad = None
        xg = x.detach().requires_grad_(True)
        with torch.enable_grad():
            m(xg).backward(self.dy)
        return xg.grad

    def cpu_workload(self):
        n = max(1, self.n_total // 16)
        g = _gen(0)
        bf = torch.bfloat16
        x = torch.randn(n, self.b, self.t, self.d, generator=g).to(bf).requires_grad_(True)
        w = torch.ones(n * self.d, dtype=bf, requires_grad=True)
        bb = torch.zeros(n * self.d, dtype=bf, requires_grad=True)
        dy = torch.randn(x.shape, generator=g).to(bf)

        def fn():
            for t in (x, w, bb):
                t.grad = None
            shape = (n, 1, 1, self.d)
            (torch.nn.functional.layer_norm(x, (self.d,), eps=1e-5) * w.view(shape) + bb.view(shape)).backward(dy)
        return fn, n * self.b, f"{n} of the {self.n_total} models per rep: torch CPU layer_norm + affine, autograd"


def make_workload(name, models=None):
    wl = _make_workload(name)
    if models:
        wl.n_total = models
    return wl


def _make_workload(name):
    return {
        "cfg1": lambda: MlpCfg1(), "cfg2": lambda: LinearCfg2(), "cfg3": lambda: ResBlockCfg3(),
        "cfg4gru": lambda: RnnCfg4("gru"), "cfg4lstm": lambda: RnnCfg4("lstm"), "cfg5": lambda: AttnCfg5(),
        "bn2d_eval": lambda: BatchNormWl(False), "bn2d_train": lambda: BatchNormWl(True),
        "gn": lambda: GroupNormWl(), "ln": lambda: LayerNormWl(),
        "cfg2train": lambda: LinearCfg2Train(), "lntrain": lambda: LayerNormTrain(),
    }[name]()


# ---------------------------------------------------------------------------
# Reference arm
# ---------------------------------------------------------------------------

def _cpu_line(wl, steps, warmup, step_seconds):
    """Median samples/s over `steps` steps, each as many whole-workload
    forwards as fill `step_seconds` (at least one), after `warmup` forwards."""
    fn, samples, desc = wl.cpu_workload()
    for _ in range(warmup):
        fn()
    vals = []
    t0 = time.perf_counter()
    for _ in range(steps):
        ts = time.perf_counter()
        reps = 0
        while True:
            fn()
            reps += 1
            el = time.perf_counter() - ts
            if el >= step_seconds:
                break
        vals.append(reps * samples / el)
    wall = time.perf_counter() - t0
    return statistics.median(vals), wall, desc


def run_reference(args):
    """The reference's CPU path for the same configurations, rank 0 only;
    each step is at least `--ref-step-seconds` of full forwards of the whole
    workload (all N models)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    names = _workload_names(args)
    head = make_workload(names[0], args.models)
    value, wall, desc = _cpu_line(head, args.steps, args.warmup, args.ref_step_seconds)
    line = {
        "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * wall / max(args.steps, 1), "higher_is_better": True,
        "scaling": "weak" if args.weak else "strong", "vs_baseline": None, "dtype": head.dtype,
        "data": "synthetic", "config": head.config(), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                         "sample": f"median over steps of >= {args.ref_step_seconds} s each; {desc}"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    subs = {}
    for name in names[1:]:
        wl = make_workload(name)
        v, w2, d2 = _cpu_line(wl, args.ref_sub_steps, 1, args.ref_step_seconds)
        subs[name] = {"value": v, "unit": "samples/s", "ms_per_step": 1e3 * w2 / max(args.ref_sub_steps, 1),
                      "dtype": wl.dtype, "config": wl.config(),
                      "cpu_baseline": {"value": v, "unit": "samples/s", "cores": threads, "kind": "port",
                                       "sample": d2}}
    if subs:
        line["configs"] = subs
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------

def _workload_names(args):
    if args.workload == "all":
        return list(ORDER)
    return [args.workload]


class _Ctx:
    def __init__(self, args, world, rank, local, dev, pg):
        self.args, self.world, self.rank, self.local, self.dev, self.pg = args, world, rank, local, dev, pg

    def barrier(self):
        if self.pg:
            torch.distributed.barrier(device_ids=[self.local])
        torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, v):
        t = torch.tensor([v], device=self.dev, dtype=torch.float64)
        if self.pg:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())


def _runner(wl, x, dev):
    """Callable running one step on input buffer x (a CUDA-graph replay for
    workloads captured in the bench) and the number of our kernels one call
    launches when it is a replay."""
    from wide_compiler import _native as N
    if not wl.graph:
        return (lambda: wl.step(x)), None
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            wl.step(x)
    torch.cuda.current_stream(dev).wait_stream(side)
    g = torch.cuda.CUDAGraph()
    n0 = N.launch_count()
    with torch.cuda.graph(g):
        out = wl.step(x)
    launches = N.launch_count() - n0

    def replay():
        g.replay()
        return out
    replay.graph = g
    return replay, launches


def _gather_fn(wl, ctx):
    if not (ctx.args.gather and ctx.world > 1):
        return None
    from wide_compiler import parallel
    if isinstance(wl, _Traced):
        return None                          # ShardedWideModel gathers inside its forward
    return lambda y: parallel.gather_outputs(y, wl.n_total)


def measure(name, ctx, clocks):
    from wide_compiler import _native as N
    args = ctx.args
    mark_setup = clocks.mark()
    wl = make_workload(name, args.models)
    if args.weak:
        lo, hi = 0, wl.n_total
        wl._world_rank = (1, 0)
    else:
        lo, hi = shard_range(wl.n_total, ctx.world, ctx.rank)
        wl._world_rank = (ctx.world, ctx.rank)
    wl._gather = bool(args.gather and ctx.world > 1 and not args.weak)
    wl._gather_chunks = args.gather_chunks
    n_local = hi - lo
    wl.setup(ctx.dev, lo, hi, seed=args.seed)
    x = wl.x
    gather = _gather_fn(wl, ctx) if not args.weak else None
    run0, replay_launches = _runner(wl, x, ctx.dev)

    def step():
        y = run0()
        if gather is not None:
            y = gather(y)
        return y

    steps = args.steps if name == HEADLINE or args.workload != "all" else args.sub_steps
    warm = max(args.warmup, 3)
    torch.cuda.synchronize(ctx.dev)
    t_w = time.perf_counter()
    for _ in range(warm):
        step()
    torch.cuda.synchronize(ctx.dev)
    t_step = (time.perf_counter() - t_w) / warm
    ctx.barrier()
    # Clock window: untimed steps for about --clock-window seconds right
    # before the timed region, so that the 100 ms nvidia-smi samples see the
    # GPU under this workload's load even when the timed region itself is a
    # few ms. The step count is agreed over the ranks (max), since a step may
    # hold a collective and every rank must issue the same ones.
    mark0 = clocks.mark()
    n_cw = int(ctx.max_over_ranks(min(100000, math.ceil(args.clock_window / max(t_step, 1e-6)))))
    for i in range(n_cw):
        step()
        if i % 8 == 7:
            torch.cuda.synchronize(ctx.dev)
    ctx.barrier()
    stream = torch.cuda.current_stream(ctx.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = N.launch_count()
    with N.LaunchTimer() as timer:
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
    ctx.barrier()
    launches = N.launch_count() - launches0
    gpu_launches = launches + (replay_launches or 0) * steps
    ms_local = e0.elapsed_time(e1) / steps
    ms = ctx.max_over_ranks(ms_local)
    kern = timer.summary()

    # End to end through the public call: pinned host input uploaded, forward,
    # output downloaded, on three streams with double-buffered device inputs.
    e2e_steps = max(1, min(steps, args.e2e_steps))
    x_host = x.cpu().pin_memory()
    x_dev = [torch.empty_like(x) for _ in range(2)]
    runners = [_runner(wl, x_dev[k], ctx.dev)[0] for k in range(2)]
    y0 = runners[0]()
    if gather is not None:
        y0 = gather(y0)
    y_host = [torch.empty(y0.shape, dtype=y0.dtype).pin_memory() for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(ctx.dev), torch.cuda.Stream(ctx.dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        k = i % 2
        if i >= 2:
            s_in.wait_event(ev_comp[k])          # step i-2's forward has read x_dev[k]
            stream.wait_event(ev_out[k])         # and its output has been downloaded
        with torch.cuda.stream(s_in):
            x_dev[k].copy_(x_host, non_blocking=True)
            ev_in[k].record(s_in)
        stream.wait_event(ev_in[k])
        y = runners[k]()
        if gather is not None:
            y = gather(y)
        ev_comp[k].record(stream)
        s_out.wait_event(ev_comp[k])
        with torch.cuda.stream(s_out):
            y_host[k].copy_(y, non_blocking=True)
            y.record_stream(s_out)
            ev_out[k].record(s_out)

    for i in range(4):
        e2e_step(i)
    ctx.barrier()
    e0.record(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    stream.wait_stream(s_in)
    e1.record(stream)
    ctx.barrier()
    ms_e2e = ctx.max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    clk = clocks.summary(mark0, clocks.mark())
    clk["window"] = (f"nvidia-smi samples every 100 ms over {args.clock_window:.1f} s of untimed steps just "
                     f"before the timed region, the timed region and the e2e loop")
    if not clk.get("samples"):
        # no sample arrived in that window: widen it to this workload's whole
        # measurement (set-up, warm-up and the steps above), and say so
        wide = clocks.summary(mark_setup, clocks.mark())
        if wide.get("samples"):
            clk = wide
            clk["window"] = ("no nvidia-smi sample arrived during the timed steps; samples over this workload's "
                             "whole measurement (set-up, warm-up, timed and e2e steps)")
    clk["samples_total"] = len(clocks.lines)
    if clocks.lines:
        clk["first_sample_s"] = round(clocks.lines[0][0] - clocks.t_start, 3)

    total_models = wl.n_total if not args.weak else wl.n_total * ctx.world
    samples = wl.samples(total_models)
    rec = {"value": samples / (ms * 1e-3), "unit": "samples/s", "ms_per_step": ms, "steps": steps,
           "dtype": wl.dtype, "config": wl.config(),
           "e2e": {"value": samples / (ms_e2e * 1e-3), "unit": "samples/s",
                   "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                   "d2h_bytes_per_step": y_host[0].numel() * y_host[0].element_size(),
                   "steps": e2e_steps, "ms_per_step": ms_e2e,
                   "pipelined": "upload, forward and download on separate streams, double-buffered"},
           "gpu_launches": gpu_launches, "clocks": clk,
           "models_this_rank": n_local}
    rec["roofline"] = _roofline(wl, n_local, ms_local, steps, kern, replay_launches)
    rec["kernels"] = {k: {"launches_per_step": v["calls"] / steps, "mean_ms": v["mean_ms"],
                          "ms_per_step": v["total_ms"] / steps} for k, v in kern.items()}

    if ctx.rank == 0 and ctx.world == 1:
        if hasattr(wl, "torch_reference_step") and not args.no_torch_gpu:
            fn = wl.torch_reference_step()
            for _ in range(3):
                fn()
            torch.cuda.synchronize(ctx.dev)
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize(ctx.dev)
            tms = e0.elapsed_time(e1) / steps
            rec["torch_gpu_reference"] = {"ms_per_step": tms, "value": samples / (tms * 1e-3), "unit": "samples/s",
                                          "note": "the reference's op sequence on this GPU via torch "
                                                  "(cuBLAS / cuDNN / SDPA)"}
        if not args.no_cpu_baseline:
            torch.set_num_threads(len(os.sched_getaffinity(0)))
            fn, cpu_samples, desc = wl.cpu_workload()
            secs = args.cpu_seconds if name == HEADLINE else args.sub_cpu_seconds
            reps, el = _timed_cpu(fn, secs)
            rec["cpu_baseline"] = {"value": reps * cpu_samples / el, "unit": "samples/s",
                                   "cores": torch.get_num_threads(), "kind": "port",
                                   "sample": f"{reps} reps in {el:.1f} s: {desc}"}
            del fn
    for r in runners:
        if hasattr(r, "graph"):
            del r.graph
    if hasattr(run0, "graph"):
        del run0.graph
    del wl, x, x_dev, runners, run0
    torch.cuda.synchronize(ctx.dev)
    torch.cuda.empty_cache()
    return rec


def _roofline(wl, n_local, ms_step, steps, kern, replay_launches):
    pk = peaks()
    work = wl.work(n_local)
    if replay_launches is not None or not kern or "graph replay" in work:
        entry = "graph replay"
        units = sum(work.values())
        kms = ms_step
        per_step = 1
    else:
        entry = max(kern, key=lambda k: kern[k]["total_ms"])
        if entry not in work:
            entry = max((k for k in kern if k in work), key=lambda k: kern[k]["total_ms"], default=entry)
        units = work.get(entry, 0)
        kms = kern[entry]["total_ms"] / steps        # that entry's device time per step
        per_step = kern[entry]["calls"] / steps
    if wl.bound == "hbm":
        achieved = units / (kms * 1e-3) / 1e9
        peak, unit, kind = pk["hbm"], "GB/s", f"{pk['kind']} HBM copy"
    elif wl.bound == "fp32":
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        achieved = units / (kms * 1e-3) / 1e12
        peak, unit = sms * 128 * 2 * 1965e6 / 1e12, "TFLOP/s"
        kind = f"nominal fp32 FFMA ({sms} SMs x 128 lanes x 2 x 1965 MHz; no measured figure exists)"
    else:
        achieved = units / (kms * 1e-3) / 1e12
        peak, unit, kind = pk[wl.peak_key], "TFLOP/s", f"{pk['kind']} bf16 dense ({wl.peak_key})"
    tr = wl.traffic(n_local)
    scale = 1e9 if wl.bound == "hbm" else 1e12
    step_rate = sum(work.values()) / (ms_step * 1e-3) / scale
    return {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "peak_kind": kind, "traffic": None if tr is None else int(tr),
            "kernel": entry, "launches_per_step": per_step, "kernel_ms_per_step": kms,
            "algorithmic_per_step": units, "step_achieved": step_rate, "step_frac": step_rate / peak}


def run_b200(args):
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = False
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = True
    from wide_compiler import _native as N
    N.load()
    N.check(N.lib().widek_linear_set_variant(args.linear_variant), "widek_linear_set_variant")
    N.check(N.lib().widek_attention_set_variant(args.attn_variant), "widek_attention_set_variant")
    N.check(N.lib().widek_conv_set_variant(args.conv_variant), "widek_conv_set_variant")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    ctx = _Ctx(args, world, rank, local, dev, pg)
    clocks = ClockSampler(local)
    clocks.start()
    names = _workload_names(args)
    recs = {}
    try:
        for name in names:
            recs[name] = measure(name, ctx, clocks)
    finally:
        clocks.stop()
    dev_err = N.device_error()
    if rank == 0:
        head = recs[names[0]]
        line = {
            "metric": METRIC, "value": head["value"], "unit": "samples/s", "n_gpus": world, "steps": head["steps"],
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "weak" if args.weak else "strong", "vs_baseline": None, "dtype": head["dtype"],
            "data": "synthetic", "config": head["config"], "e2e": head["e2e"],
            "gpu_launches": head["gpu_launches"], "roofline": head["roofline"], "clocks": head["clocks"],
        }
        for k in ("cpu_baseline", "torch_gpu_reference", "kernels", "models_this_rank"):
            if k in head:
                line[k] = head[k]
        line["parallel"] = {"ranks": world, "split": "weak: every rank runs all N models" if args.weak else
                            "contiguous N-slices, one per rank (N fixed)", "gather": bool(args.gather and world > 1),
                            "gather_chunks": args.gather_chunks if args.gather and world > 1 else None}
        line["variants"] = {"linear": args.linear_variant, "attention": args.attn_variant, "conv": args.conv_variant}
        if len(names) > 1:
            line["configs"] = {k: recs[k] for k in names[1:]}
        line["device_error"] = dev_err
        print(json.dumps(line), flush=True)
    if pg:
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="all", choices=["all"] + ORDER + TRAINING,
                    help="all: the cfg3 headline plus every other configuration under 'configs'; "
                         "cfg2train / lntrain: forward + backward steps (not part of 'all')")
    ap.add_argument("--sub-steps", type=int, default=20, help="timed steps of each non-headline configuration")
    ap.add_argument("--models", type=int, default=None,
                    help="override the number of models N (reduced cases for profiling captures only)")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--clock-window", type=float, default=2.0,
                    help="seconds of untimed steps before each timed region while clocks are sampled")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--weak", action="store_true", help="every rank runs all N models (weak scaling)")
    ap.add_argument("--gather", action="store_true", help="include the optional output all-gather in every step")
    ap.add_argument("--gather-chunks", type=int, default=1,
                    help="with --gather on TracedWideModel workloads: batch slices whose gathers overlap the "
                         "next slice's forward")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline time for the headline")
    ap.add_argument("--sub-cpu-seconds", type=float, default=3.0, help="CPU baseline time per other configuration")
    ap.add_argument("--ref-step-seconds", type=float, default=1.0,
                    help="reference arm: minimum CPU time of one step (whole-workload forwards)")
    ap.add_argument("--ref-sub-steps", type=int, default=3,
                    help="reference arm: steps of each non-headline configuration")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-torch-gpu", action="store_true", help="skip the torch GPU reference column")
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
