"""Gradients through the wide primitives (forward on the sm_100a kernels,
backward from the torch formulation of the reference's arithmetic) against
N stand-alone torch modules, as the reference's own training use relies on
(its primitives are torch code; wide_lstm.py:744-762 checks gradient flow).
fp32 with TF32 off; tolerance rtol 1e-3 / atol 1e-4 on forward values and
gradients (gradients scaled by their magnitude)."""
import pytest
import torch
import torch.nn as nn

import wide_compiler as wc
from gpu_util import no_device_error

pytestmark = [pytest.mark.gpu, pytest.mark.grad]
DEV = 'cuda'


def _close(a, b, rtol=1e-3, atol_frac=1e-4):
    a, b = a.double().cpu(), b.double().cpu()
    scale = max(float(b.abs().max()), 1e-6)
    torch.testing.assert_close(a, b, rtol=rtol, atol=atol_frac * scale + 1e-6)


def _run_each(mods, xs, fwd=lambda m, x: m(x)):
    return [fwd(m, x) for m, x in zip(mods, xs)]


def test_linear_grads():
    torch.manual_seed(0)
    n, b, i, o = 4, 6, 24, 40
    mods = [nn.Linear(i, o).to(DEV) for _ in range(n)]
    wide = wc.WideLinear.from_modules(mods)
    x = torch.randn(n, b, i, device=DEV, requires_grad=True)
    g = torch.randn(n, b, o, device=DEV)
    y = wide(x)
    (y * g).sum().backward()
    xs = [x.detach()[k].clone().requires_grad_(True) for k in range(n)]
    ys = _run_each(mods, xs)
    sum((yk * g[k]).sum() for k, yk in enumerate(ys)).backward()
    _close(y.detach(), torch.stack([yk.detach() for yk in ys]))
    _close(x.grad, torch.stack([xk.grad for xk in xs]))
    _close(wide.weight.grad, torch.stack([m.weight.grad for m in mods]))
    _close(wide.bias.grad, torch.stack([m.bias.grad for m in mods]))
    no_device_error()


def test_conv2d_and_batchnorm_train_grads():
    torch.manual_seed(1)
    n, b, c, hw = 3, 4, 8, 10
    convs = [nn.Conv2d(c, c, 3, padding=1).to(DEV) for _ in range(n)]
    bns = [nn.BatchNorm2d(c).to(DEV).train() for _ in range(n)]
    wconv = wc.WideConv2d.from_modules(convs)
    wbn = wc.WideBatchNorm2d.from_modules(bns).train()
    x = torch.randn(n, b, c, hw, hw, device=DEV, requires_grad=True)
    g = torch.randn(n, b, c, hw, hw, device=DEV)
    y = wbn(wconv(x))
    (y * g).sum().backward()
    xs = [x.detach()[k].clone().requires_grad_(True) for k in range(n)]
    ys = [bn(cv(xk)) for cv, bn, xk in zip(convs, bns, xs)]
    sum((yk * g[k]).sum() for k, yk in enumerate(ys)).backward()
    _close(y.detach(), torch.stack([yk.detach() for yk in ys]))
    _close(x.grad, torch.stack([xk.grad for xk in xs]))
    _close(wconv.grouped_conv.weight.grad, torch.cat([m.weight.grad for m in convs]))
    # the conv bias feeds a batch-statistics BatchNorm, so its gradient is
    # zero up to rounding: compare on the scale of the weight gradient
    db = (wconv.grouped_conv.bias.grad - torch.cat([m.bias.grad for m in convs])).abs().max()
    assert float(db) <= 1e-3 * float(wconv.grouped_conv.weight.grad.abs().max())
    _close(wbn.op.weight.grad, torch.cat([m.weight.grad for m in bns]))
    _close(wbn.op.running_mean, torch.cat([m.running_mean for m in bns]))
    _close(wbn.op.running_var, torch.cat([m.running_var for m in bns]))
    no_device_error()


def test_layernorm_groupnorm_embedding_grads():
    torch.manual_seed(2)
    n, b, t, d, v = 3, 4, 5, 32, 50
    lns = [nn.LayerNorm(d).to(DEV) for _ in range(n)]
    for m in lns:
        nn.init.uniform_(m.weight, 0.5, 1.5)
        nn.init.normal_(m.bias, 0, 0.1)
    wln = wc.WideLayerNorm.from_modules(lns)
    x = torch.randn(n, b, t, d, device=DEV, requires_grad=True)
    g = torch.randn(n, b, t, d, device=DEV)
    (wln(x) * g).sum().backward()
    xs = [x.detach()[k].clone().requires_grad_(True) for k in range(n)]
    sum((m(xk) * g[k]).sum() for k, (m, xk) in enumerate(zip(lns, xs))).backward()
    _close(x.grad, torch.stack([xk.grad for xk in xs]))
    _close(wln.weight.grad, torch.cat([m.weight.grad for m in lns]))

    gns = [nn.GroupNorm(4, 16).to(DEV) for _ in range(n)]
    wgn = wc.WideGroupNorm.from_modules(gns)
    x2 = torch.randn(n, b, 16, 6, 6, device=DEV, requires_grad=True)
    g2 = torch.randn_like(x2)
    (wgn(x2) * g2).sum().backward()
    xs2 = [x2.detach()[k].clone().requires_grad_(True) for k in range(n)]
    sum((m(xk) * g2[k]).sum() for k, (m, xk) in enumerate(zip(gns, xs2))).backward()
    _close(x2.grad, torch.stack([xk.grad for xk in xs2]))
    wp = [p for p in wgn.parameters()][0]
    _close(wp.grad.reshape(-1), torch.cat([m.weight.grad for m in gns]))

    embs = [nn.Embedding(v, d).to(DEV) for _ in range(n)]
    wemb = wc.WideEmbedding.from_modules(embs)
    idx = torch.randint(0, v, (b, t), device=DEV)
    g3 = torch.randn(n, b, t, d, device=DEV)
    (wemb(idx) * g3).sum().backward()
    sum((m(idx) * g3[k]).sum() for k, m in enumerate(embs)).backward()
    _close(wemb.weight.grad, torch.stack([m.weight.grad for m in embs]))
    no_device_error()


def test_attention_grads():
    torch.manual_seed(3)
    n, b, t, d, h = 2, 3, 16, 32, 4
    mhas = [nn.MultiheadAttention(d, h, batch_first=True).to(DEV) for _ in range(n)]
    for m in mhas:
        nn.init.normal_(m.in_proj_bias, 0, 0.1)
    wide = wc.WideAttention.from_modules(mhas).eval()
    x = torch.randn(n, b, t, d, device=DEV, requires_grad=True)
    g = torch.randn(n, b, t, d, device=DEV)
    (wide(x, is_causal=True) * g).sum().backward()
    mask = torch.triu(torch.ones(t, t, dtype=torch.bool, device=DEV), 1)
    xs = [x.detach()[k].clone().requires_grad_(True) for k in range(n)]
    ys = [m(xk, xk, xk, attn_mask=mask, need_weights=False)[0] for m, xk in zip(mhas, xs)]
    sum((yk * g[k]).sum() for k, yk in enumerate(ys)).backward()
    _close(x.grad, torch.stack([xk.grad for xk in xs]))
    _close(wide.q_weight.grad, torch.stack([m.in_proj_weight.grad[:d] for m in mhas]))
    _close(wide.kv_weight.grad, torch.stack([m.in_proj_weight.grad[d:] for m in mhas]))
    _close(wide.out_weight.grad, torch.stack([m.out_proj.weight.grad for m in mhas]))
    no_device_error()


@pytest.mark.parametrize("kind", ["gru", "lstm"])
def test_recurrent_grads(kind):
    torch.manual_seed(4)
    n, b, t, i, hsz = 3, 2, 7, 8, 16
    cls = nn.GRU if kind == "gru" else nn.LSTM
    mods = [cls(i, hsz, batch_first=True).to(DEV) for _ in range(n)]
    wide = (wc.WideGRU if kind == "gru" else wc.WideLSTM).from_modules(mods)
    x = torch.randn(n, b, t, i, device=DEV, requires_grad=True)
    g = torch.randn(n, b, t, hsz, device=DEV)
    out = wide(x)[0]
    (out * g).sum().backward()
    xs = [x.detach()[k].clone().requires_grad_(True) for k in range(n)]
    outs = [m(xk)[0] for m, xk in zip(mods, xs)]
    sum((o * g[k]).sum() for k, o in enumerate(outs)).backward()
    _close(out.detach(), torch.stack([o.detach() for o in outs]))
    _close(x.grad, torch.stack([xk.grad for xk in xs]))
    if kind == "gru":
        _close(wide.weight_hh.grad, torch.stack([m.weight_hh_l0.grad for m in mods]))
    else:
        whh = wide.weight_hh.grad.view(n, 4 * hsz, n, hsz)
        blocks = torch.stack([whh[k, :, k, :] for k in range(n)])
        _close(blocks, torch.stack([m.weight_hh_l0.grad for m in mods]))
    no_device_error()


class _MLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(16, 32)
        self.fc2 = nn.Linear(32, 8)

    def forward(self, x):
        return self.fc2(torch.relu(self.fc1(x)))


def test_traced_model_training_step():
    """The packed TracedWideModel trains like the N models: same loss, same
    gradients, and an SGD step moves it the same way."""
    torch.manual_seed(5)
    n, b = 5, 12
    models = [_MLP().to(DEV) for _ in range(n)]
    wide = wc.compile(models, torch.randn(b, 16, device=DEV))
    xs = [torch.randn(b, 16, device=DEV) for _ in range(n)]
    tgt = torch.randn(b, n * 8, device=DEV)
    y = wide(wc.pack_inputs(xs))
    loss = ((y - tgt) ** 2).mean()
    loss.backward()
    outs = [m(x) for m, x in zip(models, xs)]
    ref = ((torch.cat(outs, dim=1) - tgt) ** 2).mean()
    ref.backward()
    _close(loss.detach(), ref.detach())
    wfc1 = wide.stages['fc1'].weight.grad
    _close(wfc1, torch.stack([m.fc1.weight.grad for m in models]))
    opt = torch.optim.SGD(wide.parameters(), lr=0.1)
    opt.step()
    with torch.no_grad():
        for m in models:
            for p in m.parameters():
                p -= 0.1 * p.grad
        y2 = wide(wc.pack_inputs(xs))
        ref2 = torch.cat([m(x) for m, x in zip(models, xs)], dim=1)
    _close(y2, ref2)
    no_device_error()
