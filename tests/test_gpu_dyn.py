"""Dynamic content tree (attn='dyn') on the GPU: the 2-means build (ta_lane_order / ta_lane_sums), insertion
(ta_lane_insert) and select_keys (ta_lane_select) against the numpy oracle and the reference's golden vectors, and
the reference's own dynamic-tree tests (test_dyn.py) on this implementation.

Trees are compared in canonical child order (oracle.canonical_tree: a two-key split's orientation is an exact fp32
tie that only mirrors a subtree). A lane whose oracle decisions (argmax, nearer centre, median side, insertion side,
top-k cut, neighbour threshold) come within TIE of an fp32 tie is counted, not compared: the kernel sums in a
different order and may take the other side."""
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


def _canon(tree):
    sums, cnt = tree.packed
    return oracle.canonical_tree(tree.slot.cpu().numpy(), sums.cpu().numpy(), cnt.cpu().numpy())


def _compare_trees(tree, ref, min_frac):
    """Canonical slots, counts and sums of every node whose key set depends on no near-tie decision of the oracle
    (LaneTreeNP.excluded): equal, equal, within fp32 reduction error. Returns the compared fraction of groups."""
    a = _canon(tree)
    b = oracle.canonical_tree(ref.slot, ref.sums, ref.cnt, with_order=True)
    ar = np.arange(ref.P)[:, None]
    ex = ref.excluded(TIE)[ar, b[3]]  # in canonical rows
    offD = (1 << ref.D) - 1
    okg = ~ex[:, offD:]
    record(int(okg.sum()), int((~okg).sum()), 0, 'tree groups')
    assert okg.mean() >= min_frac, okg.mean()
    assert np.array_equal(a[0][okg], b[0][okg])
    assert np.array_equal(a[2][~ex], b[2][~ex])
    scale = np.abs(b[1]).max() + 1.0
    np.testing.assert_allclose(a[1][~ex], b[1][~ex], atol=2e-6 * scale * np.sqrt(ref.C))
    return float(okg.mean())


@pytest.mark.parametrize('P,C,dh,seed', [(6, 64, 16, 0), (5, 1024, 64, 1), (3, 4096, 32, 2), (4, 512, 128, 3),
                                         (2, 16384, 16, 4)])
def test_lane_build_and_insert_vs_oracle(P, C, dh, seed):
    """The 2-means build over lanes with different prefixes (warp teams for groups <= 256 slots, CTA teams above),
    then 32 insertions: the same keys in the same groups, counts equal, sums within fp32 reduction error."""
    from treeattn_b200.dyntree import LaneTree
    rng = np.random.default_rng(seed)
    kfull = rng.standard_normal((P, C, dh)).astype(np.float32)
    n = rng.integers(0, C - 40, P)
    n[0] = 0
    n[-1] = C - 40
    tree = LaneTree(to_dev(kfull), torch.as_tensor(n))
    ref = oracle.LaneTreeNP(kfull, n, 3)
    _compare_trees(tree, ref, 0.3)
    ar = np.arange(P)
    for i in range(32):
        kpos = n + i
        act = kpos >= 1
        tree.insert(to_dev(kfull[ar, kpos]), torch.as_tensor(kpos), torch.as_tensor(act))
        ref.insert(kfull[ar, kpos], kpos, act)
    _compare_trees(tree, ref, 0.3)
    _no_device_error()


def test_tree_insertion_consistent():
    """Reference test_dyn.py:20-38 on this implementation: after 16 insertions every node sum / count equals a
    recomputation from the slots, and the slots hold exactly the keys [1, n + 16)."""
    from treeattn_b200.dyntree import LaneTree
    torch.manual_seed(0)
    P, C, dh = 4, 64, 16
    kfull = torch.randn(P, C, dh, device=DEV)
    n = torch.tensor([0, 8, 20, 33])
    tree = LaneTree(kfull, n, iters=3)
    assert tree.check() < 1e-4
    ar = torch.arange(P)
    for i in range(16):
        kpos = n + i
        tree.insert(kfull[ar, kpos.to(DEV)], kpos, kpos >= 1)
    assert tree.check() < 1e-4
    pos = tree.slot.reshape(P, C).cpu()
    for p in range(P):
        assert sorted(pos[p][pos[p] >= 0].tolist()) == list(range(1, int(n[p]) + 16))
    _no_device_error()


def _cfg_from(g):
    from treeattn_b200.config import Config
    return Config(attn='dyn', seq_len=g['q'].shape[2], chunk=int(g['chunk']), wmax=int(g['wmax']),
                  nb_window=int(g['nb_window']), nb_store=int(g['nb_store']), nb_rho=float(g['nb_rho']),
                  nb_probe=int(g['nb_probe']), nb_cap_min=int(g['nb_cap_min']))


def _compare_select(sel, ref, Y, min_frac, build=True):
    """Every query whose results depend on no oracle decision within TIE of an fp32 tie (its lane's build, when
    `build`, its own step and the earlier steps of its lane): tree / neighbour position sets, leaf validity, tree
    budget and neighbour-leaf count equal the reference's."""
    ok = ref['query_margin'] > TIE
    if build:
        ok &= np.repeat(ref['build_margin'] > TIE, Y, axis=-1)
    record(int(ok.sum()), int((~ok).sum()), 0, 'select_keys')
    assert ok.mean() >= min_frac, ok.mean()
    srt = lambda a: np.sort(np.asarray(a), -1)
    got = {k: v.cpu().numpy() for k, v in sel.items()}
    assert np.array_equal(srt(got['tree_pos'])[ok], srt(ref['tree_pos'])[ok])
    assert np.array_equal(srt(got['nb_pos'])[ok], srt(ref['nb_pos'])[ok])
    assert np.array_equal(got['leaf_ok'].sum(-1)[ok], ref['leaf_ok'].sum(-1)[ok])
    assert np.array_equal(got['n_tree'][ok], ref['n_tree'][ok])
    assert np.array_equal(got['nb_leaves'][ok], ref['nb_leaves'][ok])
    return int(ok.sum())


@pytest.mark.parametrize('name', ['dyn_sel_a', 'dyn_sel_b'])
def test_select_keys_golden(name):
    """dyntree.select_keys against the reference's own outputs (neighbours on, random leaf budgets)."""
    from treeattn_b200.dyntree import select_keys
    g = load(name)
    cfg = _cfg_from(g)
    sel = select_keys(to_dev(g['q']), to_dev(g['k']), to_dev(g['lhat'], torch.int64), cfg)
    r = oracle.select_keys(g['q'], g['k'], g['lhat'], cfg.chunk, cfg.wmax, cfg.nb_window, cfg.nb_store, cfg.nb_rho,
                           cfg.nb_probe, cfg.nb_cap_min)
    ref = dict(g, query_margin=r['query_margin'], build_margin=r['build_margin'])
    n = _compare_select(sel, ref, cfg.chunk, 0.75)
    assert n >= 0.75 * g['q'].shape[0] * g['q'].shape[1] * g['q'].shape[2]
    _no_device_error()


@pytest.mark.parametrize('B,H,T,dh,chunk,wmax,neighbors', [(1, 4, 512, 64, 64, 8, True),
                                                           (2, 2, 1024, 32, 128, 16, True),
                                                           (1, 2, 2048, 128, 256, 8, False)])
def test_select_loop_vs_oracle(B, H, T, dh, chunk, wmax, neighbors):
    """The token loop (ta_lane_select) on the oracle's own trees (uploaded), against the oracle's loop: every lane
    whose loop decisions (searches, neighbour tests, insertions) are clear of fp32 ties matches on every query."""
    from treeattn_b200 import _lib, _ops
    from treeattn_b200.config import Config
    rng = np.random.default_rng(T + dh)
    q = rng.standard_normal((B, H, T, dh)).astype(np.float32)
    k = rng.standard_normal((B, H, T, dh)).astype(np.float32)
    cfg = Config(attn='dyn', seq_len=T, chunk=chunk, wmax=wmax, neighbors=neighbors)
    lhat = rng.integers(2, wmax + 1, (B, H, T))
    nl = T // chunk
    P = B * H * nl
    kfull = np.broadcast_to(k[:, :, None], (B, H, nl, T, dh)).reshape(P, T, dh)
    tree = oracle.LaneTreeNP(kfull, np.broadcast_to(np.arange(nl) * chunk, (B, H, nl)).reshape(P), 3)
    sums, cnt, slot = to_dev(tree.sums), to_dev(tree.cnt, torch.int32), to_dev(tree.slot, torch.int32)
    ref = oracle.select_loop(tree, q, k, lhat, chunk, wmax, cfg.nb_window, cfg.nb_store, cfg.nb_rho, cfg.nb_probe,
                             cfg.nb_cap_min, neighbors=neighbors)
    wl = min(wmax, T // 2)
    W = cfg.nb_window * cfg.nb_store
    out = dict(tree_pos=torch.empty(B, H, T, 2 * wl, device=DEV, dtype=torch.int64),
               leaf_ok=torch.empty(B, H, T, wl, device=DEV, dtype=torch.bool),
               nb_pos=torch.empty(B, H, T, 2 * W, device=DEV, dtype=torch.int64),
               n_tree=torch.empty(B, H, T, device=DEV, dtype=torch.int64),
               nb_leaves=torch.empty(B, H, T, device=DEV, dtype=torch.int64))
    qd, kd, ld = to_dev(q), to_dev(k), to_dev(lhat, torch.int64)
    _lib.call('ta_lane_select', _ops._p(qd), _ops._p(kd), _ops._p(ld), B, H, T, dh, chunk, wmax, cfg.nb_window,
              cfg.nb_store, cfg.nb_probe, cfg.nb_cap_min, cfg.nb_rho, int(neighbors), _ops._p(sums), _ops._p(cnt),
              _ops._p(slot), *[_ops._p(out[key]) for key in ('tree_pos', 'leaf_ok', 'nb_pos', 'n_tree',
                                                              'nb_leaves')], _ops._stream(qd))
    _compare_select(out, ref, chunk, 0.3, build=False)
    _no_device_error()


@pytest.mark.parametrize('B,H,T,dh,chunk,wmax', [(1, 4, 512, 64, 64, 8), (1, 2, 2048, 128, 256, 8)])
def test_select_keys_end_to_end_vs_oracle(B, H, T, dh, chunk, wmax):
    """Build + loop through the public select_keys at sizes where most lanes see some near-tie 2-means decision:
    the selected key positions overlap the oracle's (mean recall >= 0.95), and exactly on tie-free lanes."""
    from treeattn_b200.config import Config
    from treeattn_b200.dyntree import select_keys
    rng = np.random.default_rng(T + dh + 1)
    q = rng.standard_normal((B, H, T, dh)).astype(np.float32)
    k = rng.standard_normal((B, H, T, dh)).astype(np.float32)
    cfg = Config(attn='dyn', seq_len=T, chunk=chunk, wmax=wmax)
    lhat = rng.integers(2, wmax + 1, (B, H, T))
    sel = select_keys(to_dev(q), to_dev(k), to_dev(lhat, torch.int64), cfg)
    ref = oracle.select_keys(q, k, lhat, chunk, wmax, cfg.nb_window, cfg.nb_store, cfg.nb_rho, cfg.nb_probe,
                             cfg.nb_cap_min)
    _compare_select(sel, ref, chunk, 0.0)
    got = sel['tree_pos'].cpu().numpy()
    hit = [len(set(a[a >= 0]) & set(b[b >= 0])) / max(1, len(set(b[b >= 0])))
           for a, b in zip(got.reshape(-1, got.shape[-1]), ref['tree_pos'].reshape(-1, got.shape[-1]))]
    assert np.mean(hit) >= 0.95, np.mean(hit)
    _no_device_error()


def tiny(**kw):
    from treeattn_b200.config import Config
    base = dict(vocab_size=64, seq_len=64, n_layer=2, n_head=2, n_embd=32, attn='dyn', chunk=16, wmax=4, beam=2,
                beam_classes=(2, 3, 4), nb_window=4, nb_store=2, nb_probe=2, nb_cap_min=1)
    base.update(kw)
    return Config(**base)


@pytest.mark.parametrize('name,kw', [('tiny_gpt_dyn', dict(beam_mode='fixed')),
                                     ('tiny_gpt_dyn_pred', dict(beam_mode='pred', global_pool=True, local=8))])
def test_tiny_gpt_dyn_golden(name, kw):
    """A tiny GPT with DynAttention (attn='dyn'): logits within 1e-4 of the reference's (fp32), same statistics."""
    from treeattn_b200.model import GPT
    torch.manual_seed(33)
    m = GPT(tiny(**kw)).to(DEV).eval()
    g = load(name)
    with torch.no_grad():
        logits, _, stats = m(to_dev(g['idx'], torch.int64))
    err = (logits.cpu() - torch.as_tensor(g['logits'])).abs().max().item()
    assert err < 1e-4, err
    for key in ('keys_total', 'keys_tree', 'keys_nb', 'nb_leaves', 'leaves_used'):
        assert abs(stats[key] - float(g['stat_' + key])) < 1e-5, key
    _no_device_error()


def test_all_keys_matches_dense():
    """Reference test_dyn.py:57-73: with every key selected the sparse attention equals causal attention."""
    from treeattn_b200.attention_dyn import DynAttention
    torch.manual_seed(2)
    cfg = tiny(n_layer=1, wmax=32, beam=32, neighbors=False, local=3, beam_mode='fixed')
    attn = DynAttention(cfg).to(DEV).eval()
    x = torch.randn(2, 64, 32, device=DEV)
    with torch.no_grad():
        out = attn(x)
        C, H, dh = 32, 2, 16
        q, k, v = attn.c_attn(x).split(C, 2)
        q, k, v = [t.view(2, 64, H, dh).transpose(1, 2) for t in (q, k, v)]
        s = (q @ k.transpose(-1, -2)) / dh ** 0.5
        s = s.masked_fill(~torch.tril(torch.ones(64, 64, dtype=torch.bool, device=DEV)), float('-inf'))
        ref = attn.c_proj((torch.softmax(s, -1) @ v).transpose(1, 2).reshape(2, 64, C))
    assert (out - ref).abs().max().item() < 1e-4


@pytest.mark.parametrize('kw', [dict(beam_mode='fixed'), dict(beam_mode='pred', global_pool=True),
                                dict(beam_mode='pred', local=8)])
def test_causality(kw):
    """Reference test_dyn.py:76-91: changing a token changes no output at an earlier position."""
    from treeattn_b200.model import GPT
    torch.manual_seed(3)
    model = GPT(tiny(**kw)).to(DEV).eval()
    idx = torch.randint(0, 64, (2, 64), device=DEV)
    idx2 = idx.clone()
    pos = 37
    idx2[:, pos] = (idx[:, pos] + 1) % 64
    with torch.no_grad():
        l1, _, _ = model(idx)
        l2, _, _ = model(idx2)
    assert (l1[:, :pos] - l2[:, :pos]).abs().max().item() < 1e-4
    assert (l1[:, pos:] - l2[:, pos:]).abs().max().item() > 1e-6


def test_backward_and_losses():
    """Reference test_dyn.py:94-108: training with the learned budget head - finite loss and gradients."""
    from treeattn_b200.model import GPT
    torch.manual_seed(4)
    model = GPT(tiny(beam_mode='pred', global_pool=True)).to(DEV).train()
    idx = torch.randint(0, 64, (2, 64), device=DEV)
    tgt = torch.randint(0, 64, (2, 64), device=DEV)
    _, loss, st = model(idx, tgt)
    loss.backward()
    assert torch.isfinite(loss)
    for n, p in model.named_parameters():
        if p.grad is not None:
            assert torch.isfinite(p.grad).all(), n
    assert model.blocks[0].attn.c_attn.weight.grad.abs().sum() > 0
    assert st['pred'] > 0


def test_fullsize_causality():
    """Reference test_dyn.py:111-127 at the default model size (512 tokens, 6 layers)."""
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    cfg = Config(attn='dyn', beam_mode='pred', global_pool=True)
    torch.manual_seed(5)
    model = GPT(cfg).to(DEV).eval()
    idx = torch.randint(0, cfg.vocab_size, (1, cfg.seq_len), device=DEV)
    with torch.no_grad():
        l1, _, _ = model(idx)
        for pos in (70, 200, 333, 500):
            idx2 = idx.clone()
            idx2[:, pos] = (idx[:, pos] + 1) % cfg.vocab_size
            l2, _, _ = model(idx2)
            assert (l1[:, :pos] - l2[:, :pos]).abs().max().item() < 1e-3, pos
    _no_device_error()
