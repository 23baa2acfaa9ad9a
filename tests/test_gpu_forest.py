"""Block forest (attn='block') on the GPU: the content sort (ta_lane_order on blocks), the level sums and soft gate
(ta_forest_levels, ta_soft_gate), the descent (ta_forest_select) and TreeAttention, against the numpy oracle and
the reference's golden vectors, plus the reference's own block-attention tests (test_core.py) on this
implementation. Queries or blocks whose oracle decisions come within TIE of an fp32 tie are counted, not compared."""
import math

import numpy as np
import pytest
import torch

import oracle
from tests._compare import record
from tests._golden import load

pytestmark = pytest.mark.gpu
DEV = 'cuda'
TIE = 1e-5


def _no_device_error():
    from treeattn_b200 import _ops
    assert _ops.device_error()[0] == 0


def to_dev(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a)).to(DEV, dtype)


def _cfg(**kw):
    from treeattn_b200.config import Config
    return Config(**kw)


@pytest.mark.parametrize('P,G,S,D', [(16, 2, 32, 64), (4, 1, 256, 32), (3, 4, 512, 16), (64, 8, 4, 128)])
def test_two_means_order_vs_oracle(P, G, S, D):
    """forest.two_means_order: the same order in every group whose 2-means decisions are clear of fp32 ties."""
    from treeattn_b200.forest import two_means_order
    rng = np.random.default_rng(S + D)
    X = rng.standard_normal((P, G, S, D)).astype(np.float32)
    got = two_means_order(to_dev(X), 3).cpu().numpy()
    ref, margin = oracle.two_means_order(X, 3, with_margin=True)
    ok = margin > TIE
    record(int(ok.sum()), int((~ok).sum()), 0, 'groups')
    assert ok.mean() >= 0.5, ok.mean()
    assert np.array_equal(got[ok], ref[ok])
    _no_device_error()


def test_build_forest_golden():
    """forest.build_forest against the reference: the same rank order in every block, level sums within fp32
    rounding, with and without the soft gate."""
    from treeattn_b200.forest import build_forest
    g = load('forest_build')
    k = to_dev(g['k'])
    perm, sums = build_forest(k, 32, 4, _cfg(kmeans_iters=3, gate=False))
    assert np.array_equal(perm.cpu().numpy(), g['perm'])
    for l in range(5):
        np.testing.assert_allclose(sums[l].cpu().numpy(), g['S%d' % l], atol=2e-5)
    _, sums_g = build_forest(k, 32, 4, _cfg(kmeans_iters=3, gate=True, gate_q=0.25, gate_temp=0.3))
    for l in range(5):
        np.testing.assert_allclose(sums_g[l].cpu().numpy(), g['G%d' % l], atol=2e-5)
    _no_device_error()


@pytest.mark.parametrize('dtype,dh', [(torch.float32, 64), (torch.bfloat16, 64), (torch.bfloat16, 128)])
def test_build_forest_vs_oracle(dtype, dh):
    """Larger forests (64-key blocks), fp32 and bf16 keys, gate on: rank order on tie-free blocks, sums in the keys'
    precision."""
    from treeattn_b200.forest import build_forest
    rng = np.random.default_rng(dh)
    k = torch.as_tensor(rng.standard_normal((2, 3, 1024, dh)).astype(np.float32)).to(dtype)
    kn = k.float().numpy()
    cfg = _cfg(kmeans_iters=3, gate=True, gate_q=0.25, gate_temp=0.3)
    perm, sums = build_forest(k.to(DEV), 64, 5, cfg)
    rperm, rsums, margin = oracle.build_forest(kn, 64, 5, 3, gate=(0.25, 0.3), bf16=dtype == torch.bfloat16)
    ok = np.repeat(margin > TIE, 64, axis=-1)
    record(int((margin > TIE).sum()), int((margin <= TIE).sum()), 0, 'blocks')
    assert ok.mean() >= 0.5
    assert np.array_equal(perm.cpu().numpy()[ok], rperm[ok])
    okb = margin > TIE
    tol = 2e-5 if dtype == torch.float32 else 2e-2
    for l in range(6):
        a = sums[l].float().cpu().numpy().reshape(2, 3, 16, 1 << l, dh)[okb]
        b = rsums[l].reshape(2, 3, 16, 1 << l, dh)[okb]
        np.testing.assert_allclose(a, b, atol=tol * (1 + np.abs(b).max()), rtol=0)
    _no_device_error()


def test_soft_gate_vs_oracle():
    from treeattn_b200.forest import soft_gate
    rng = np.random.default_rng(5)
    grp = rng.standard_normal((3, 8, 16, 64)).astype(np.float32)
    sm = grp.sum(2)
    out = soft_gate(to_dev(sm), to_dev(grp), _cfg(gate_q=0.25, gate_temp=0.3)).cpu().numpy()
    np.testing.assert_allclose(out, oracle.soft_gate(sm, grp, 0.25, 0.3), rtol=1e-5, atol=1e-5)
    _no_device_error()


def _tree_attn_module(H, dh, T, B, wmax, beam, **kw):
    from treeattn_b200.attention import TreeAttention
    cfg = _cfg(n_embd=H * dh, n_head=H, seq_len=T, tree_block=B, wmax=wmax, beam=beam, **kw)
    return TreeAttention(cfg).to(DEV).eval()


@pytest.mark.parametrize('name', ['tree_attn_a', 'tree_attn_b'])
def test_tree_attention_golden(name):
    """TreeAttention.sparse_attend against the reference's outputs (fp32, 1e-4) on every query whose selection is
    clear of fp32 ties; statistics within the tied queries' share."""
    g = load(name)
    B_, H, T, dh = g['q'].shape
    m = _tree_attn_module(H, dh, T, int(g['tree_block']), int(g['wmax']), int(g['beam']))
    with torch.no_grad():
        out = m.sparse_attend(to_dev(g['q']), to_dev(g['k']), to_dev(g['v'])).cpu().numpy()
    _, _, margin = oracle.tree_attention(g['q'], g['k'], g['v'], int(g['tree_block']), int(g['wmax']),
                                         int(g['beam']))
    ok = margin > TIE
    record(int(ok.sum()), int((~ok).sum()), 0, 'queries')
    assert ok.mean() > 0.9
    np.testing.assert_allclose(out[ok], g['o'][ok], atol=1e-4)
    for key in ('keys_tree', 'keys_total'):
        assert abs(float(m.aux[key]) - float(g['stat_' + key])) < 0.05, key
    _no_device_error()


@pytest.mark.parametrize('T,B,dh,wmax,beam', [(1024, 64, 64, 8, 4), (8192, 32, 16, 8, 8), (2048, 32, 128, 16, 6)])
def test_forest_select_vs_oracle(T, B, dh, wmax, beam):
    """The descent kernel against the oracle's descent on the oracle's own forest (uploaded): the same valid leaves
    on every query whose cuts are clear of ties (with 256 blocks the roots are ranked in chunks)."""
    from treeattn_b200 import _lib, _ops
    from treeattn_b200.forest import _ptr_array
    rng = np.random.default_rng(T + dh)
    q = rng.standard_normal((1, 2, T, dh)).astype(np.float32)
    k = rng.standard_normal((1, 2, T, dh)).astype(np.float32)
    depth = int(round(math.log2(B // 2)))
    perm, sums, _ = oracle.build_forest(k, B, depth, 3)
    bq = np.full((1, 2, T), beam, np.int64)
    _, leaf, leafv, margin = oracle.forest_descent(q, sums, B, depth, wmax, bq)
    wl = leaf.shape[-1]
    qd = to_dev(q)
    sd = [to_dev(s) for s in sums]
    pd = to_dev(perm.reshape(-1, B), torch.int32)
    out = [torch.empty(1, 2, T, wl, device=DEV, dtype=torch.int64), torch.empty(1, 2, T, wl, device=DEV, dtype=torch.bool),
           torch.empty(1, 2, T, 2 * wl, device=DEV, dtype=torch.int64),
           torch.empty(1, 2, T, 2 * wl, device=DEV, dtype=torch.bool)]
    lv = _ptr_array([s.data_ptr() for s in sd])
    st = qd.stride()
    _lib.call('ta_forest_select', _ops._p(qd), 0, 1, 2, T, dh, st[0], st[1], st[2], lv[0], _ops._p(pd), B, depth,
              None, beam, wmax, *[_ops._p(o) for o in out], None, None, _ops._stream(qd))
    gl, gv = out[0].cpu().numpy(), out[1].cpu().numpy()
    ok = margin > TIE
    record(int(ok.sum()), int((~ok).sum()), 0, 'queries')
    assert ok.mean() > 0.9
    big = np.iinfo(np.int64).max
    sa = np.sort(np.where(gv, gl, big), -1)
    sb = np.sort(np.where(leafv, leaf, big), -1)
    assert np.array_equal(sa[ok], sb[ok])
    _no_device_error()


def tiny(**kw):
    base = dict(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=32, tree_block=32, wmax=4, beam=2,
                beam_classes=(2, 3, 4))
    base.update(kw)
    return _cfg(**base)


@pytest.mark.parametrize('name,kw', [('tiny_gpt_block', dict()),
                                     ('tiny_gpt_block_pred', dict(beam_mode='pred', global_pool=True, gate=True))])
def test_tiny_gpt_block_golden(name, kw):
    """A tiny GPT with TreeAttention: logits within 1e-4 of the reference's (fp32), the same statistics."""
    from treeattn_b200.model import GPT
    torch.manual_seed(43)
    m = GPT(tiny(**kw)).to(DEV).eval()
    g = load(name)
    with torch.no_grad():
        logits, _, stats = m(to_dev(g['idx'], torch.int64))
    err = (logits.cpu() - torch.as_tensor(g['logits'])).abs().max().item()
    assert err < 1e-4, err
    for key in ('keys_tree', 'keys_total'):
        assert abs(stats[key] - float(g['stat_' + key])) < 1e-4, key
    _no_device_error()


def test_all_keys_matches_dense():
    """Reference test_core.py:20-36: with every key selected the block attention equals causal attention."""
    from treeattn_b200.attention import TreeAttention
    torch.manual_seed(0)
    cfg = tiny(n_layer=1, wmax=64, beam=64)
    attn = TreeAttention(cfg).to(DEV).eval()
    x = torch.randn(2, 128, 32, device=DEV)
    with torch.no_grad():
        out = attn(x)
        C, H, dh = 32, 2, 16
        q, k, v = attn.c_attn(x).split(C, 2)
        q, k, v = [t.view(2, 128, H, dh).transpose(1, 2) for t in (q, k, v)]
        s = (q @ k.transpose(-1, -2)) / dh ** 0.5
        s = s.masked_fill(~torch.tril(torch.ones(128, 128, dtype=torch.bool, device=DEV)), float('-inf'))
        ref = attn.c_proj((torch.softmax(s, -1) @ v).transpose(1, 2).reshape(2, 128, C))
    assert (out - ref).abs().max().item() < 1e-4


@pytest.mark.parametrize('kw', [dict(), dict(gate=True), dict(beam_mode='pred', global_pool=True, gate=True)])
def test_causality(kw):
    """Reference test_core.py:39-56: changing a token changes no output at an earlier position."""
    from treeattn_b200.model import GPT
    torch.manual_seed(1)
    model = GPT(tiny(**kw)).to(DEV).eval()
    idx = torch.randint(0, 64, (2, 128), device=DEV)
    idx2 = idx.clone()
    pos = 70
    idx2[:, pos] = (idx[:, pos] + 1) % 64
    with torch.no_grad():
        l1, _, _ = model(idx)
        l2, _, _ = model(idx2)
    assert (l1[:, :pos] - l2[:, :pos]).abs().max().item() < 1e-4
    assert (l1[:, pos:] - l2[:, pos:]).abs().max().item() > 1e-6


def test_backward_and_losses():
    """Reference test_core.py:59-73 with the routing loss switched on (route_weight 1; the reference's default 0
    leaves it at 0): finite loss and gradients, routing and budget-head losses positive."""
    from treeattn_b200.model import GPT
    torch.manual_seed(2)
    model = GPT(tiny(beam_mode='pred', global_pool=True, gate=True, route_weight=1.0)).to(DEV).train()
    idx = torch.randint(0, 64, (2, 128), device=DEV)
    tgt = torch.randint(0, 64, (2, 128), device=DEV)
    _, loss, st = model(idx, tgt)
    loss.backward()
    assert torch.isfinite(loss)
    for n, p in model.named_parameters():
        if p.grad is not None:
            assert torch.isfinite(p.grad).all(), n
    assert model.blocks[0].attn.c_attn.weight.grad.abs().sum() > 0
    assert st['route'] > 0 and st['pred'] > 0


def test_bf16_block_model_runs():
    """A bf16 block-attention GPT at the reference's train.py size (512 tokens, 64-key blocks): finite logits."""
    from treeattn_b200.model import GPT
    cfg = _cfg(vocab_size=8192, seq_len=512, n_layer=2, n_head=6, n_embd=384, tree_block=64, wmax=8, beam=4)
    torch.manual_seed(3)
    m = GPT(cfg).to(DEV, torch.bfloat16).eval()
    with torch.no_grad():
        logits, _, st = m(torch.randint(0, 8192, (2, 512), device=DEV))
    assert torch.isfinite(logits.float()).all()
    assert st['keys_tree'] > 0
    _no_device_error()
