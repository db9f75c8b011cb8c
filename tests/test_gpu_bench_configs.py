"""GPU parity at the benchmark sizes, on the exact modules and inputs bench.py
times (its workload builders): the cfg3 ResBlock TracedWideModel (fused halo
conv chain with the folded BatchNorm and the residual, packed input and
output) and the cfg1 MLP TracedWideModel (one chain launch, eager and under
the CUDA-graph executor), each checked against the oracle on sampled models
at the north-star tolerance: bf16 rtol 2e-2 against an fp64 computation from
the same rounded inputs and weights; fp32 rtol 1e-3 / atol 1e-4.
Reference forward: wide_compiler/core/traced_wide.py:450-534."""
import pytest
import torch

import bench
from gpu_util import FP32_TOL, LOWP_RTOL, assert_lowp_close, no_device_error
from oracle import wide_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def _bn(bn, sl):
    return {'weight': bn.weight[sl].detach().cpu(), 'bias': bn.bias[sl].detach().cpu(),
            'running_mean': bn.running_mean[sl].detach().cpu(), 'running_var': bn.running_var[sl].detach().cpu(),
            'eps': bn.eps}


def _workload(name):
    wl = bench.make_workload(name)
    wl._world_rank = (1, 0)
    wl._gather = False
    wl.setup(DEV, 0, wl.n_total, seed=1234)
    return wl


def test_cfg3_bench_path_matches_oracle():
    wl = _workload('cfg3')
    model = wl.module.local
    y = wl.step(wl.x)                                   # [32, 6400, 32, 32] bf16, packed
    torch.cuda.synchronize()
    assert model._fusion['groups'], "the fused conv groups must serve cfg3"
    n, c = wl.n_total, wl.c
    st = model.stages
    worst = 0.0
    for i, rows in ((0, [0, 31]), (57, [5, 17]), (99, [2, 30])):
        ch = slice(i * c, (i + 1) * c)
        x = wl.x[rows][:, ch].cpu().unsqueeze(0)        # [1, r, C, H, W] (model i, sampled rows)
        ref = O.resblock(x, 1, st['conv1'].grouped_conv.weight[ch].detach().cpu(),
                         st['conv1'].grouped_conv.bias[ch].detach().cpu(), _bn(st['bn1'].op, ch),
                         st['conv2'].grouped_conv.weight[ch].detach().cpu(),
                         st['conv2'].grouped_conv.bias[ch].detach().cpu(), _bn(st['bn2'].op, ch))[0]
        got = y[rows][:, ch].double().cpu()
        scale = float(ref.abs().max())
        err = (got - ref).abs()
        bound = LOWP_RTOL * ref.abs() + 1e-2 * scale
        worst = max(worst, float((err / bound).max()))
        torch.testing.assert_close(got, ref, rtol=LOWP_RTOL, atol=1e-2 * scale,
                                   msg=lambda m: f"model {i}: {m}")
    print(f"cfg3 worst |err| / (rtol*|ref| + atol) = {worst:.3f}")
    no_device_error()


@pytest.mark.parametrize("graphed", [True, False])
def test_cfg1_bench_path_matches_oracle(graphed):
    wl = _workload('cfg1')
    mod = wl.module.local
    eager = mod._orig_mod if graphed else mod
    run = mod if graphed else eager
    y = run(wl.x).clone()
    if graphed:
        y = run(wl.x).clone()                           # a replay
    torch.cuda.synchronize()
    st = eager.stages
    ref = O.mlp2(wl.x.cpu(), wl.n_total, st['fc1'].weight.detach().cpu(), st['fc1'].bias.detach().cpu(),
                 st['fc2'].weight.detach().cpu(), st['fc2'].bias.detach().cpu())
    torch.testing.assert_close(y.double().cpu(), ref, **FP32_TOL)
    no_device_error()


@pytest.mark.parametrize("name", ["bn2d_train", "bn2d_eval", "gn", "ln"])
def test_norm_workloads_match_oracle(name):
    """The memory-bound norm workloads bench.py times, at full size (419 MB
    / 537 MB inputs), checked against the oracle on three sampled models
    (training-mode BatchNorm also through its running-statistics update)."""
    wl = _workload(name)
    m = wl.module
    before = None
    if name == "bn2d_train":
        before = (m.op.running_mean.detach().cpu().clone(), m.op.running_var.detach().cpu().clone())
    y = wl.step(wl.x)
    torch.cuda.synchronize()
    n = wl.n_total
    for i in (0, n // 2, n - 1):
        xi = wl.x[i:i + 1].cpu()
        if name.startswith("bn2d"):
            c = wl.c
            sl = slice(i * c, (i + 1) * c)
            rm0 = before[0][sl] if before else m.op.running_mean[sl].detach().cpu()
            rv0 = before[1][sl] if before else m.op.running_var[sl].detach().cpu()
            ref, new_rm, new_rv = O.batchnorm(xi, 1, c, m.op.weight[sl].detach().cpu(), m.op.bias[sl].detach().cpu(),
                                              rm0, rv0, name == "bn2d_train", momentum=0.1)
            if name == "bn2d_train":
                assert_lowp_close(m.op.running_mean[sl], new_rm)
                assert_lowp_close(m.op.running_var[sl], new_rv)
        elif name == "gn":
            c = wl.c
            sl = slice(i * c, (i + 1) * c)
            ref = O.groupnorm(xi, 1, wl.groups, m.norm.weight[sl].detach().cpu(), m.norm.bias[sl].detach().cpu(),
                              m.norm.eps)
        else:
            d = wl.d
            sl = slice(i * d, (i + 1) * d)
            ref = O.layernorm(xi, m.weight[sl].detach().cpu(), m.bias[sl].detach().cpu(), 1, d, m.eps)
        assert_lowp_close(y[i:i + 1], ref)
    no_device_error()
