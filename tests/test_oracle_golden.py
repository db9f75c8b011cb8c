"""The oracle (oracle/wide_oracle.py) against the golden fixtures produced by
running the reference implementation itself (tests/golden/make_golden.py).
This pins the oracle that the GPU parity tests then use at larger sizes."""
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import wide_oracle as O

TOL = dict(rtol=1e-5, atol=1e-5)


def _close(a, b, **tol):
    torch.testing.assert_close(a.to(torch.float64), b.to(torch.float64), **(tol or TOL))


def oracle_eval(g):
    """Runs the oracle for one fixture; returns {output name: tensor}."""
    k, m, s, inp = g['kind'], g['meta'], g['state'], g['inputs']
    if k == 'linear':
        return {'y': O.linear(inp['x'], s['weight'], s.get('bias'))}
    if k == 'layernorm':
        return {'y': O.layernorm(inp['x'], s['weight'], s['bias'], m['n'], m['d'], m['eps'])}
    if k == 'batchnorm':
        y, rm, rv = O.batchnorm(inp['x'], m['n'], m['c'], s['op.weight'], s['op.bias'], s['op.running_mean'],
                                s['op.running_var'], use_batch_stats=m['train'])
        out = {'y': y}
        if m['train']:
            out.update(running_mean=rm, running_var=rv)
        return out
    if k == 'groupnorm':
        return {'y': O.groupnorm(inp['x'], m['n'], m['groups'], s.get('norm.weight'), s.get('norm.bias'), 1e-5)}
    if k == 'instancenorm':
        return {'y': O.groupnorm(inp['x'], m['n'], m['c'], s.get('norm.weight'), s.get('norm.bias'), 1e-5)}
    if k == 'embedding':
        return {'y': O.embedding(inp['idx'], s['weight'])}
    if k == 'conv':
        pre = {1: 'op', 2: 'grouped_conv', 3: 'conv'}[m['dims']]
        nd = m['dims']
        return {'y': O.conv_nd(inp['x'], s[f'{pre}.weight'], s.get(f'{pre}.bias'), m['n'], (m['s'],) * nd,
                               (m['p'],) * nd, (m['d'],) * nd)}
    if k == 'attention':
        q = inp['q']
        kk = inp['k'] if inp['k'] is not None else q
        v = inp['v'] if inp['v'] is not None else kk
        return {'y': O.attention(q, kk, v, s['q_weight'], s['kv_weight'], s.get('q_bias'), s.get('kv_bias'),
                                 s['out_weight'], s.get('out_bias'), m['heads'], inp['mask'], m['causal'])}
    if k == 'gru':
        y, hn = O.gru(inp['x'], inp['h0'], s['weight_ih'], s['weight_hh'], s.get('bias_ih'), s.get('bias_hh'))
        return {'y': y, 'h_n': hn}
    if k == 'lstm':
        n = m['n']
        wih, whh = O.lstm_blocks(s['weight_ih'], s['weight_hh'], n)
        bih = s['bias_ih'].view(n, -1) if 'bias_ih' in s else None
        bhh = s['bias_hh'].view(n, -1) if 'bias_hh' in s else None
        y, (hn, cn) = O.lstm(inp['x'], inp['h0'], inp['c0'], wih, whh, bih, bhh)
        return {'y': y, 'h_n': hn, 'c_n': cn}
    if k == 'traced':
        n = m['n']
        if m['model'] == 'MLP':
            st = lambda key: torch.stack([s[f'm{i}.{key}'] for i in range(n)])
            return {'y': O.mlp2(inp['packed'], n, st('fc1.weight'), st('fc1.bias'), st('fc2.weight'),
                                st('fc2.bias'))}
        if m['model'] == 'ResBlock':
            cat = lambda key: torch.cat([s[f'm{i}.{key}'] for i in range(n)])
            bn = lambda p: {f: cat(f'{p}.{f}') for f in ('weight', 'bias', 'running_mean', 'running_var')}
            x = O.packed_to_nfirst(inp['packed'], n)
            y = O.resblock(x, n, cat('conv1.weight'), cat('conv1.bias'), bn('bn1'), cat('conv2.weight'),
                           cat('conv2.bias'), bn('bn2'))
            return {'y': O.nfirst_to_packed(y)}
        st = lambda key: torch.stack([s[f'm{i}.{key}'] for i in range(n)])
        x = O.packed_to_nfirst(inp['packed'], n)
        if m['model'] == 'AttnLN':
            # MultiheadAttention's packed in_proj: q rows [0, D), then k and v
            d = x.shape[-1]
            w_in, b_in = st('attn.in_proj_weight'), st('attn.in_proj_bias')
            y = O.attention(x, x, x, w_in[:, :d], w_in[:, d:], b_in[:, :d], b_in[:, d:],
                            st('attn.out_proj.weight'), st('attn.out_proj.bias'), m['heads'], None, m['causal'])
            y = O.layernorm(y, st('ln.weight').reshape(-1), st('ln.bias').reshape(-1), n, d, 1e-5)
            return {'y': O.nfirst_to_packed(y)}
        if m['model'] == 'GRUOut':
            y, _ = O.gru(x, None, st('gru.weight_ih_l0'), st('gru.weight_hh_l0'), st('gru.bias_ih_l0'),
                         st('gru.bias_hh_l0'))
            return {'y': O.nfirst_to_packed(y)}
        if m['model'] == 'LSTMOut':
            y, _ = O.lstm(x, None, None, st('lstm.weight_ih_l0'), st('lstm.weight_hh_l0'), st('lstm.bias_ih_l0'),
                          st('lstm.bias_hh_l0'))
            return {'y': O.nfirst_to_packed(y)}
    if k == 'grad_linear':
        y = O.activation(O.linear(inp['x'], s['weight'], s.get('bias')), m['act'])
        dx, dw, db = O.linear_grads(inp['x'], s['weight'], s.get('bias'), inp['dy'], m['act'])
        out = {'y': y, 'grads.x': dx, 'grads.weight': dw}
        if db is not None:
            out['grads.bias'] = db
        return out
    if k == 'grad_layernorm':
        dx, dw, db = O.layernorm_grads(inp['x'], s['weight'], inp['dy'], m['n'], m['d'], m['eps'])
        return {'y': O.layernorm(inp['x'], s['weight'], s['bias'], m['n'], m['d'], m['eps']),
                'grads.x': dx, 'grads.weight': dw, 'grads.bias': db}
    if k == 'grad_batchnorm':
        dx, dw, db = O.batchnorm_grads(inp['x'], m['n'], m['c'], s['op.weight'], s['op.running_mean'],
                                       s['op.running_var'], inp['dy'], m['train'], m['eps'])
        return {'grads.x': dx, 'grads.op.weight': dw, 'grads.op.bias': db}
    if k == 'grad_groupnorm':
        dx, dw, db = O.groupnorm_grads(inp['x'], m['n'], m['groups'], s['norm.weight'], inp['dy'], m['eps'])
        return {'y': O.groupnorm(inp['x'], m['n'], m['groups'], s['norm.weight'], s['norm.bias'], m['eps']),
                'grads.x': dx, 'grads.norm.weight': dw, 'grads.norm.bias': db}
    raise KeyError(k)


def _expected(g, key):
    if key.startswith('grads.'):
        return g['outputs']['grads'][key[len('grads.'):]]
    return g['outputs'][key]


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_fixture(name):
    g = load_golden(name)
    got = oracle_eval(g)
    if g['kind'].startswith('grad_'):
        assert {k[len('grads.'):] for k in got if k.startswith('grads.')} == set(g['outputs']['grads'])
    for key, val in got.items():
        _close(val, _expected(g, key))


def test_fixture_set_covers_every_primitive():
    kinds = {load_golden(n)['kind'] for n in golden_names()}
    assert {'linear', 'layernorm', 'batchnorm', 'groupnorm', 'instancenorm', 'embedding', 'conv', 'attention',
            'gru', 'lstm', 'traced', 'grad_linear', 'grad_layernorm', 'grad_batchnorm', 'grad_groupnorm'} <= kinds


def test_pack_roundtrip_oracle():
    g = load_golden('traced_mlp')
    packed = O.pack_inputs(g['inputs']['inputs'])
    torch.testing.assert_close(packed, g['inputs']['packed'])
    nf = O.packed_to_nfirst(packed, g['meta']['n'])
    torch.testing.assert_close(O.nfirst_to_packed(nf), packed)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_oracle_gradient_formulas_match_autograd(seed):
    """The oracle's explicit gradient formulas against torch autograd of the
    primitives' torch forms (float64) on random shapes, beyond the reference
    fixtures: WideLinear (+ ReLU / GELU), LayerNorm, BatchNorm with batch and
    with running statistics, GroupNorm."""
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)
    tol = dict(rtol=1e-9, atol=1e-10)
    n, b, k, o = 2 + seed, 3 + seed, 5 + 2 * seed, 4 + seed
    acts = {'none': lambda t: t, 'relu': torch.relu, 'gelu': F.gelu}
    for act, fn in acts.items():
        x, w, bb, dy = r(n, b, k).requires_grad_(), r(n, o, k).requires_grad_(), r(n, o).requires_grad_(), r(n, b, o)
        fn(torch.einsum('noi,nbi->nbo', w, x) + bb[:, None, :]).backward(dy)
        for got, want in zip(O.linear_grads(x.detach(), w.detach(), bb.detach(), dy, act), (x.grad, w.grad, bb.grad)):
            torch.testing.assert_close(got, want, **tol)
    d = 6 + seed
    x, w, bb, dy = r(n, b, 2, d).requires_grad_(), r(n * d).requires_grad_(), r(n * d).requires_grad_(), r(n, b, 2, d)
    (F.layer_norm(x, (d,), eps=1e-5) * w.view(n, 1, 1, d) + bb.view(n, 1, 1, d)).backward(dy)
    for got, want in zip(O.layernorm_grads(x.detach(), w.detach(), dy, n, d, 1e-5), (x.grad, w.grad, bb.grad)):
        torch.testing.assert_close(got, want, **tol)
    c = 3
    for stats in (True, False):
        x, w, bb = r(n, b, c, 4, 5).requires_grad_(), r(n * c).requires_grad_(), r(n * c).requires_grad_()
        rm, rv, dy = r(n * c), torch.rand(n * c, generator=g, dtype=torch.float64) + 0.5, r(n, b, c, 4, 5)
        # the reference's inner nn.BatchNorm over N*C channels on [B, N*C, H, W]
        xt = x.transpose(0, 1).reshape(b, n * c, 4, 5)
        y = F.batch_norm(xt, rm.clone(), rv.clone(), w, bb, training=stats, momentum=0.0, eps=1e-5)
        y.reshape(b, n, c, 4, 5).transpose(0, 1).backward(dy)
        got = O.batchnorm_grads(x.detach(), n, c, w.detach(), rm, rv, dy, stats, 1e-5)
        for gt, want in zip(got, (x.grad, w.grad, bb.grad)):
            torch.testing.assert_close(gt, want, **tol)
    groups, c = 2, 4
    x, w, bb, dy = r(n, b, c, 3, 3).requires_grad_(), r(n * c).requires_grad_(), r(n * c).requires_grad_(), r(n, b, c, 3, 3)
    # the reference's nn.GroupNorm(N*G, N*C) on [B, N*C, H, W]
    xt = x.transpose(0, 1).reshape(b, n * c, 3, 3)
    F.group_norm(xt, n * groups, w, bb, eps=1e-5).reshape(b, n, c, 3, 3).transpose(0, 1).backward(dy)
    for got, want in zip(O.groupnorm_grads(x.detach(), n, groups, w.detach(), dy, 1e-5), (x.grad, w.grad, bb.grad)):
        torch.testing.assert_close(got, want, **tol)
