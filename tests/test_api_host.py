"""Host-side logic that needs no GPU: package surface, registry, config,
parameter layouts (state_dict compatibility with the reference fixtures),
FX graph construction, and the loud failure on non-CUDA tensors."""
import dataclasses

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import wide_compiler as wc
from conftest import golden_names, load_golden
from wide_compiler.core import primitives as P


REFERENCE_ALL = ['compile', 'WideBuilder', 'pack', 'unpack', 'WideConfig', 'get_default_config',
                 'set_default_config', 'register', 'unregister', 'get_registry', 'list_registered',
                 'TracedWideModel', 'FunctionalOp', 'BinaryOp', 'print_trace', 'pack_inputs', 'unpack_outputs',
                 'WideLinear', 'WideConv1d', 'WideConv2d', 'WideConv3d', 'WideBatchNorm1d', 'WideBatchNorm2d',
                 'WideLayerNorm', 'WideGroupNorm', 'WideInstanceNorm1d', 'WideInstanceNorm2d', 'WideEmbedding',
                 'WideAttention', 'WideGRU', 'WideLSTM']


def test_public_surface_matches_reference():
    for name in REFERENCE_ALL:
        assert hasattr(wc, name), name
    assert wc.benchmark_primitive is None


def test_registry_has_all_builtins_and_api():
    assert set(wc.list_registered()) == set(P.BUILTIN_PRIMITIVES)
    reg = wc.get_registry()
    assert reg.get_class('Linear') is wc.WideLinear
    assert 'GRU' in reg

    class NoFrom(nn.Module):
        pass

    with pytest.raises(TypeError):
        wc.register('Bogus', NoFrom)

    @wc.register('MyThing')
    class WideThing(nn.Module):
        @classmethod
        def from_modules(cls, modules):
            return cls()

    assert reg.build([nn.Identity()]) is None
    assert 'MyThing' in wc.list_registered()
    wc.unregister('MyThing')
    assert 'MyThing' not in wc.list_registered()


def test_config_presets_and_debug_field():
    c = wc.WideConfig()
    assert c.debug is False
    d = wc.WideConfig.debug()
    assert d.debug is True and d.validate is True and d.compile is False
    assert dataclasses.replace(c, debug=True).debug is True
    with pytest.raises(ValueError):
        wc.WideConfig(compile_mode='bogus')
    assert wc.WideConfig.fast().compile is True


def _build_from_state(g):
    k, m, s = g['kind'], g['meta'], g['state']
    if k in ('linear', 'grad_linear'):
        mod = wc.WideLinear(m['n'], m['in'], m['out'], bias=m['bias'])
    elif k in ('layernorm', 'grad_layernorm'):
        mod = wc.WideLayerNorm(m['n'], m['d'], m['eps'])
    elif k == 'grad_batchnorm':
        mod = wc.WideBatchNorm2d(m['n'], m['c'])
    elif k == 'batchnorm':
        cls = wc.WideBatchNorm2d if m['dims'] == 5 else wc.WideBatchNorm1d
        mod = cls(m['n'], m['c'])
    elif k == 'grad_groupnorm':
        mod = wc.WideGroupNorm(m['n'], m['groups'], m['c'])
    elif k == 'groupnorm':
        mod = wc.WideGroupNorm(m['n'], m['groups'], m['c'], affine=m['affine'])
    elif k == 'instancenorm':
        cls = wc.WideInstanceNorm2d if m['dims'] == 5 else wc.WideInstanceNorm1d
        mod = cls(m['n'], m['c'], affine=m['affine'])
    elif k == 'embedding':
        mod = wc.WideEmbedding(m['n'], m['v'], m['d'])
    elif k == 'conv':
        if m['dims'] == 2:
            mod = wc.WideConv2d(m['n'], m['cin'], m['cout'], m['k'], m['s'], m['p'], m['d'], bias=m['bias'],
                                strategy='grouped')
        elif m['dims'] == 1:
            mod = wc.WideConv1d(m['n'], m['cin'], m['cout'], m['k'], m['s'], m['p'], m['d'], bias=m['bias'],
                                strategy=P.Conv1dStrategy.GROUPED)
        else:
            mod = wc.WideConv3d(m['n'], m['cin'], m['cout'], m['k'], m['s'], m['p'], m['d'], bias=m['bias'])
    elif k == 'attention':
        mod = wc.WideAttention(m['n'], m['d'], m['heads'])
    elif k == 'gru':
        mod = wc.WideGRU(m['n'], m['i'], m['h'])
    elif k == 'lstm':
        mod = wc.WideLSTM(m['n'], m['i'], m['h'])
    else:
        return None
    mod.load_state_dict(s, strict=True)
    return mod


@pytest.mark.parametrize("name", [n for n in golden_names() if not n.startswith('traced')])
def test_reference_state_dict_loads_strictly(name):
    """Parameter names/shapes match the reference: its state_dict loads with strict=True."""
    assert _build_from_state(load_golden(name)) is not None


def test_from_modules_layouts():
    lin = [nn.Linear(6, 10) for _ in range(3)]
    w = wc.WideLinear.from_modules(lin)
    assert w.weight.shape == (3, 10, 6)
    torch.testing.assert_close(w.weight[1], lin[1].weight)
    lstms = [nn.LSTM(4, 5, batch_first=True) for _ in range(3)]
    wl = wc.WideLSTM.from_modules(lstms)
    assert wl.weight_ih.shape == (60, 12)
    bih, bhh = wl._blocks()
    torch.testing.assert_close(bih[2], lstms[2].weight_ih_l0)
    torch.testing.assert_close(bhh[0], lstms[0].weight_hh_l0)
    assert float(wl.weight_hh[0:20, 5:15].abs().sum()) == 0.0
    mha = [nn.MultiheadAttention(8, 2, batch_first=True) for _ in range(2)]
    wa = wc.WideAttention.from_modules(mha)
    torch.testing.assert_close(wa.kv_weight[1], mha[1].in_proj_weight[8:])
    wqkv, bqkv = wa._fused_qkv()
    torch.testing.assert_close(wqkv[0], mha[0].in_proj_weight)


def test_lstm_block_cache_invalidates_on_update():
    wl = wc.WideLSTM(2, 3, 4)
    a, _ = wl._blocks()
    with torch.no_grad():
        wl.weight_ih[0, 0] += 1.0
    b, _ = wl._blocks()
    assert float(b[0, 0, 0] - a[0, 0, 0]) == pytest.approx(1.0)


class _MLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(8, 16)
        self.fc2 = nn.Linear(16, 8)

    def forward(self, x):
        return self.fc2(F.relu(self.fc1(x)))


def test_traced_model_structure_cpu():
    models = [_MLP() for _ in range(4)]
    wide = wc.TracedWideModel.from_models(models, torch.randn(2, 8))
    kinds = [type(wide.stages[k]).__name__ for k in wide.stages]
    assert kinds == ['WideLinear', 'FunctionalOp', 'WideLinear']
    assert wide.stages['relu'].unary == 'relu'
    assert 'Total:' in wide.summary()


def test_compile_argument_errors():
    with pytest.raises(ValueError):
        wc.compile(_MLP(), torch.randn(2, 8))          # n missing
    with pytest.raises(ValueError):
        wc.compile([], torch.randn(2, 8))
    with pytest.raises(ValueError):
        wc.compile([_MLP()], None)


def test_cpu_tensors_fail_loudly():
    w = wc.WideLinear(2, 4, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        w(torch.randn(2, 3, 4))
    ln = wc.WideLayerNorm(2, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        ln(torch.randn(2, 3, 4))


def test_unpack_outputs_views_and_errors():
    out = torch.arange(2 * 12).view(2, 12).float()
    parts = wc.unpack(out, 3)
    assert len(parts) == 3 and parts[1].shape == (2, 4)
    assert parts[1].data_ptr() == out.data_ptr() + 4 * 4
    with pytest.raises(ValueError):
        wc.unpack(out, 5)


class _ResBlockT(nn.Module):
    def __init__(self, c=4, post_relu=False):
        super().__init__()
        self.post_relu = post_relu
        self.conv1 = nn.Conv2d(c, c, 3, padding=1)
        self.bn1 = nn.BatchNorm2d(c)
        self.conv2 = nn.Conv2d(c, c, 3, padding=1)
        self.bn2 = nn.BatchNorm2d(c)

    def forward(self, x):
        h = F.relu(self.bn1(self.conv1(x)))
        y = self.bn2(self.conv2(h)) + x
        return F.relu(y) if self.post_relu else y


def test_fusion_plan_structure():
    mlp = wc.TracedWideModel.from_models([_MLP() for _ in range(3)], torch.randn(2, 8))
    plan = mlp._build_fusion_plan()
    # Linear -> ReLU -> Linear is one chain group (one launch, packed in/out)
    g = plan['groups']
    assert list(g) == ['fc2'] and g['fc2']['kind'] == 'chain'
    assert g['fc2']['layers'] == ['fc1', 'fc2'] and g['fc2']['acts'] == [1, 0]
    assert plan['folded'] == {'fc1', 'relu'}
    rb = wc.TracedWideModel.from_models([_ResBlockT() for _ in range(2)], torch.randn(1, 4, 6, 6))
    plan = rb._build_fusion_plan()
    kinds = {k: (g['kind'], g['act'], g['residual']) for k, g in plan['groups'].items()}
    assert kinds['relu'] == ('conv', 1, None)
    assert kinds['add'] == ('conv', 0, 'x')
    rb2 = wc.TracedWideModel.from_models([_ResBlockT(post_relu=True) for _ in range(2)], torch.randn(1, 4, 6, 6))
    g = rb2._build_fusion_plan()['groups']
    assert g['relu_1']['residual'] == 'x' and g['relu_1']['residual_first'] and g['relu_1']['act'] == 1


class _AttnLNT(nn.Module):
    def __init__(self, causal=False, reuse=False):
        super().__init__()
        self.attn = nn.MultiheadAttention(16, 2, batch_first=True)
        self.ln = nn.LayerNorm(16)
        self.causal, self.reuse = causal, reuse

    def forward(self, x):
        a, _ = self.attn(x, x, x, need_weights=False, is_causal=self.causal)
        return self.ln(a) + a if self.reuse else self.ln(a)


def test_fusion_plan_attention_layernorm():
    """Self-attention whose output (getitem 0) only feeds a LayerNorm of the
    same width becomes one 'attn_ln' group (the LayerNorm runs in the output
    projection's epilogue); the unused getitem of the weights folds in; when
    the attention output is read elsewhere too, the pair stays unfused."""
    m = wc.TracedWideModel.from_models([_AttnLNT(causal=True) for _ in range(2)], torch.randn(2, 8, 16))
    g = m._build_fusion_plan()['groups']
    assert list(g) == ['ln'] and g['ln']['kind'] == 'attn_ln' and g['ln']['is_causal']
    assert g['ln']['nodes'][0] == 'attn' and g['ln']['nodes'][-1] == 'ln' and len(g['ln']['nodes']) == 4
    m2 = wc.TracedWideModel.from_models([_AttnLNT(reuse=True) for _ in range(2)], torch.randn(2, 8, 16))
    assert not any(g['kind'] == 'attn_ln' for g in m2._build_fusion_plan()['groups'].values())


def test_compile_flag_gives_graph_executor():
    """compile=True (the reference's torch.compile switch, api.py:137-147)
    returns the CUDA-graph executor, which forwards attribute access to the
    TracedWideModel and keeps its parameters under '_orig_mod.' as
    torch.compile's wrapper does; CPU inputs take the eager path and fail
    loudly in the kernels."""
    from wide_compiler.core.graphed import GraphedWideModel
    models = [_MLP() for _ in range(3)]
    g = wc.compile(models, torch.randn(2, 8), compile_model=True)
    assert isinstance(g, GraphedWideModel)
    assert g.n == 3 and 'fc1' in g.stages
    assert all(k.startswith('_orig_mod.') for k in g.state_dict())
    b = wc.WideBuilder(models).with_sample(torch.randn(2, 8)).compile().build()
    assert isinstance(b, GraphedWideModel)
    with pytest.raises(RuntimeError, match="CUDA"):
        g(torch.randn(2, 24))


def _attention_dropout_reference(mod, query, key, value, attn_mask, is_causal):
    """The reference's fused WideAttention forward in training mode
    (wide_attention.py:178-238): einsum projections, head split by
    view/permute/reshape, SDPA with dropout_p = module dropout."""
    n, d, h = mod.n, mod.d_model, mod.n_heads
    dh = d // h
    _, b, tq, _ = query.shape
    tk = key.shape[2]
    q = torch.einsum('nbtd,nod->nbto', query, mod.q_weight) + mod.q_bias.view(n, 1, 1, d)
    k = torch.einsum('nbtd,nod->nbto', key, mod.kv_weight[:, :d]) + mod.kv_bias[:, :d].view(n, 1, 1, d)
    v = torch.einsum('nbtd,nod->nbto', value, mod.kv_weight[:, d:]) + mod.kv_bias[:, d:].view(n, 1, 1, d)
    split = lambda t, tt: t.view(n, b, tt, h, dh).permute(0, 1, 3, 2, 4).reshape(n * b, h, tt, dh)
    o = F.scaled_dot_product_attention(split(q, tq), split(k, tk), split(v, tk), attn_mask=attn_mask,
                                       dropout_p=mod.dropout, is_causal=is_causal)
    o = o.view(n, b, h, tq, dh).permute(0, 1, 3, 2, 4).reshape(n, b, tq, d)
    return torch.einsum('nbtd,nod->nbto', o, mod.out_weight) + mod.out_bias.view(n, 1, 1, d)


@pytest.mark.parametrize("case", ["self", "causal", "bool_mask", "cross"])
def test_attention_dropout_composition(monkeypatch, case):
    """Training-mode attention dropout: WideAttention.forward routes to
    ops.attention_dropout, whose projections, head split, SDPA call and merge
    reproduce the reference's forward, drawing the same dropout mask from a
    seeded generator. The projection kernels are replaced by their torch
    formulation here (no GPU); only the composition is under test."""
    from wide_compiler import _native, ops
    monkeypatch.setattr(_native, "require_cuda", lambda *t, what: torch.device("cpu"))
    monkeypatch.setattr(ops, "linear", lambda x, w, b, act=0: torch.einsum('n...k,nok->n...o', x, w)
                        + b.view(b.shape[0], *([1] * (x.dim() - 2)), b.shape[1]))
    torch.manual_seed(0)
    mod = wc.WideAttention(3, 32, 4, dropout=0.25).train()
    with torch.no_grad():
        for p in (mod.q_bias, mod.kv_bias, mod.out_bias):
            p.normal_(0, 0.1)
    query = torch.randn(3, 2, 6, 32)
    key = value = query
    kw = {}
    if case == "cross":
        key = torch.randn(3, 2, 5, 32)
        value = torch.randn(3, 2, 5, 32)
    if case == "causal":
        kw = {"is_causal": True}
    if case == "bool_mask":
        kw = {"attn_mask": torch.rand(6, 6) > 0.3}
    torch.manual_seed(11)
    got = mod(query, key if case == "cross" else None, value if case == "cross" else None, **kw)
    got = got[0] if case == "cross" else got
    torch.manual_seed(11)
    want = _attention_dropout_reference(mod, query, key, value, kw.get("attn_mask"), kw.get("is_causal", False))
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
    torch.manual_seed(12)
    other = mod(query, key if case == "cross" else None, value if case == "cross" else None, **kw)
    other = other[0] if case == "cross" else other
    assert not torch.allclose(got, other)                        # the mask is random
    got.sum().backward()
    for p in (mod.q_weight, mod.kv_weight, mod.out_weight, mod.q_bias, mod.kv_bias, mod.out_bias):
        assert p.grad is not None and torch.isfinite(p.grad).all()
    mod.eval()
    with pytest.raises(RuntimeError, match="CUDA"):              # eval mode: the kernels, which need a GPU
        monkeypatch.undo()
        mod(query)
