"""Pins the numpy oracle (oracle/) to golden vectors produced by the reference itself
(tests/golden/make_golden.py). CPU only."""
import math

import numpy as np
import pytest
import torch

import oracle
from tests._compare import compare_sets, tied
from tests._golden import load


def _close_scores(a, b, ok):
    """Scores agree to fp32 reduction error: |a - b| <= 5e-5 * (largest |score| of the query) + 1e-6."""
    scale = np.where(ok, np.abs(b), 0).max(-1, keepdims=True)
    err = np.where(ok, np.abs(a - b) - (5e-5 * scale + 1e-6), 0)
    assert (err <= 0).all(), err.max()


def test_level_sums_bit_exact():
    g = load('levels')
    S = oracle.level_sums(g['k'], 1, 5, zero_sink=False)
    for l in range(1, 6):
        assert np.array_equal(S[l], g['S%d' % l]), l


@pytest.mark.parametrize('name', ['sel_w4', 'sel_w8'])
def test_select_seg_leaf2(name):
    g = load(name)
    wmax, beam = int(g['wmax']), int(g['beam'])
    q, k = g['q'], g['k']
    B, H, T, dh = q.shape
    lhat = np.full((B, H, T), beam)
    sel = oracle.select_seg(q, k, lhat, wmax, L0=1, nb_width=16, with_margin=True)
    excl = tied(sel['margin'])
    bad, n, nx = compare_sets(sel['ids'], sel['leaf_ok'], g['ids'], g['vld'], excl)
    assert bad == 0 and n > 0.99 * B * H * T, (bad, n, nx)
    assert np.array_equal(sel['n_tree'], g['n_tree'])
    assert np.array_equal(sel['nb_pos'], g['nb_pos'])
    # same positions as the reference (as sets) and the same best-first scores where not tied
    bad, n, _ = compare_sets(sel['tree_pos'], sel['tree_pos'] >= 0, g['tree_pos'], g['tree_pos'] >= 0, excl)
    assert bad == 0
    _close_scores(sel['sct'], g['sct'], ~excl[..., None] & g['vld'])


@pytest.mark.parametrize('name', ['tp_l3', 'tp_l5', 'tp_l6'])
def test_tree_pass_leaf_blocks(name):
    g = load(name)
    L0, wmax = int(g['L0']), int(g['wmax'])
    q, k = g['q'], g['k']
    B, H, T, dh = q.shape
    Lm = int(round(math.log2(T))) - 1
    S = oracle.level_sums(k, L0, Lm, zero_sink=True)
    ids, vld, sct, margin = oracle.tree_pass(q, S, np.arange(T), L0, Lm, wmax, with_margin=True)
    excl = tied(margin)
    bad, n, nx = compare_sets(ids, vld, g['ids'], g['vld'], excl)
    assert bad == 0 and n > 0.99 * B * H * T, (bad, n, nx)
    # the adapter scores q.S / 2^(l-L0+1); the natural scale is q.S / 2^l
    _close_scores(sct * 2.0 ** (L0 - 1), g['sct_adapter'], ~excl[..., None] & vld)


def test_dedupe_exact():
    g = load('dedupe')
    assert np.array_equal(oracle.dedupe(g['cand'], g['valid']), g['keep'])


def test_sparse_attn_and_gather_dot():
    g = load('attn')
    o = oracle.sparse_attn(g['q'], g['k'], g['v'], g['cand'], 0.125)
    np.testing.assert_allclose(o, g['o'], atol=2e-6, rtol=1e-5)
    d = oracle.gather_dot(g['q'], g['S'], g['cd'], 0.5)
    np.testing.assert_allclose(d, g['dot'], atol=2e-6, rtol=1e-5)


def test_seg_attend_filled_state():
    g = load('seg_attend')
    K, V, q = g['K'][0], g['V'][0], g['q'][0, :, 0]
    H, T, dh = K.shape
    st = oracle.SegStateNP(H, dh, T, 1, int(round(math.log2(T))) - 1)
    st.fill(K, V)
    out, keys = oracle.seg_attend(st, q, None, None, T - 1, int(g['wmax']), int(g['beam']), int(g['local']),
                                  update=False)
    np.testing.assert_allclose(out, g['out'][0, :, 0], atol=2e-6, rtol=1e-5)
    assert keys == float(g['keys'])


def _tiny_cfg():
    from treeattn_b200.config import Config
    return Config(vocab_size=64, seq_len=64, n_layer=2, n_head=2, n_embd=32, attn='seg', wmax=4, beam=2,
                  neighbors=False, beam_mode='fixed')


def test_tiny_gpt_forward_and_engine():
    from treeattn_b200.model import GPT
    g = load('tiny_gpt')
    torch.manual_seed(4)
    cfg = _tiny_cfg()
    m = GPT(cfg)
    # the same seeded construction gives the reference's weights
    wsum = np.array([float(p.double().sum()) for p in m.state_dict().values()])
    np.testing.assert_allclose(wsum, g['wsum'], rtol=0, atol=0)
    W = oracle.weights_from_state_dict(m.state_dict(), cfg.n_layer)
    logits, stats = oracle.gpt_forward(W, g['idx'], cfg.n_head, cfg.wmax, cfg.beam, cfg.local)
    np.testing.assert_allclose(logits, g['logits'], atol=1e-5)
    for k in ('keys_total', 'keys_tree', 'leaves_used'):
        assert abs(stats[k] - float(g['stat_' + k])) < 1e-5, k
    dec = oracle.DecoderNP(W, cfg.n_head, 64, cfg.wmax, cfg.beam, cfg.local)
    dec.reset(1)
    steps = [dec.step(g['idx'][:, t], t) for t in range(64)]
    np.testing.assert_allclose(np.stack([s[0][0] for s in steps]), g['dec_logits'], atol=1e-5)
    np.testing.assert_allclose([s[1] for s in steps], g['dec_keys'], atol=1e-6)


def test_config1_forward():
    """Configuration 1 (GPT 4x256, vocab 4096, T 512, leaf 32, top-4, window 64) against the reference run
    through the leaf-block adapter."""
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    g = load('config1')
    L0 = int(g['L0'])
    cfg = Config(vocab_size=4096, seq_len=512, n_layer=4, n_head=4, n_embd=256, attn='seg', wmax=4, beam=4,
                 local=64, neighbors=False, beam_mode='fixed', leaf=1 << L0)
    torch.manual_seed(0)
    m = GPT(cfg)
    wsum = np.array([float(p.double().sum()) for p in m.state_dict().values()])
    np.testing.assert_allclose(wsum, g['wsum'], rtol=0, atol=0)
    W = oracle.weights_from_state_dict(m.state_dict(), cfg.n_layer)
    logits, stats = oracle.gpt_forward(W, g['idx'], cfg.n_head, cfg.wmax, cfg.beam, cfg.local, L0=L0)
    np.testing.assert_allclose(logits[:, ::32], g['logits_sub'], atol=1e-4)
    lse = np.log(np.exp(logits.astype(np.float64) - logits.max(-1, keepdims=True)).sum(-1)) + logits.max(-1)
    np.testing.assert_allclose(lse, g['lse'], atol=1e-4)
    assert (logits.argmax(-1) == g['argmax']).mean() > 0.999
    # the adapter hands SegAttention each block as 2^(L0-1) level-1 leaves, so its leaves_used counts those
    unit = dict(keys_total=1, keys_tree=1, leaves_used=2 ** (L0 - 1))
    for k, u in unit.items():
        assert abs(stats[k] * u - float(g['stat_' + k])) < 1e-3, (k, stats[k], float(g['stat_' + k]))


def test_engine_matches_forward_leaf_blocks():
    """Oracle decode with leaf blocks (L0=3) gives the logits of the oracle's whole-sequence forward
    (the property reference test_seg.test_engine_matches_forward checks at leaf 2)."""
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=64, attn='seg', wmax=4, beam=3, local=16,
                 neighbors=False, beam_mode='fixed', leaf=8)
    torch.manual_seed(9)
    m = GPT(cfg)
    W = oracle.weights_from_state_dict(m.state_dict(), cfg.n_layer)
    idx = np.random.default_rng(0).integers(0, 64, (2, 128))
    ref, _ = oracle.gpt_forward(W, idx, cfg.n_head, cfg.wmax, cfg.beam, cfg.local, L0=3)
    dec = oracle.DecoderNP(W, cfg.n_head, 128, cfg.wmax, cfg.beam, cfg.local, L0=3)
    dec.reset(2)
    got = np.stack([dec.step(idx[:, t], t)[0] for t in range(128)], 1)
    np.testing.assert_allclose(got, ref, atol=1e-5)


@pytest.mark.parametrize('wmax', [4, 8, 3])
def test_lane_search_golden(wmax):
    """LaneTree.search (dyntree.py:108-127) on a tree the reference built and grew: the oracle's descent keeps
    the same valid leaves (no query is near a tie here) with scores within 1e-6."""
    g = load('lanetree')
    ids, vld, sct, margin = oracle.lane_search(g['q'], g['sums'], g['cnt'], int(g['D']), wmax, with_margin=True)
    bad, n, _ = compare_sets(ids, vld, g['ids_%d' % wmax], g['vld_%d' % wmax], tied(margin))
    assert bad == 0 and n == g['q'].shape[0]
    np.testing.assert_allclose(np.where(vld, sct, 0), np.where(g['vld_%d' % wmax], g['sct_%d' % wmax], 0), atol=1e-6)


def _nb_cfg(g):
    return dict(nb_window=int(g['nb_window']), nb_store=int(g['nb_store']), nb_rho=float(g['nb_rho']),
                nb_probe=int(g['nb_probe']), nb_cap_min=int(g['nb_cap_min']))


def test_select_seg_with_neighbours_golden():
    """seg.select_seg with neighbour borrowing on (cfg.neighbors=True, the reference's default), leaf 2: tree
    positions, neighbour positions (1232 matched), budgets and nb_leaves equal the reference's on every query."""
    g = load('sel_nb')
    sel = oracle.select_seg(g['q'], g['k'], g['lhat'], int(g['wmax']), L0=1, with_margin=True, nb=_nb_cfg(g))
    assert (sel['margin'] > 1e-6).all() and (sel['nb_margin'] > 1e-6).all()  # no near-tie in this fixture
    srt = lambda a: np.sort(a, -1)
    assert (srt(sel['tree_pos']) == srt(g['tree_pos'])).all()
    assert (srt(sel['nb_pos']) == srt(g['nb_pos'])).all() and (g['nb_pos'] >= 0).sum() > 1000
    assert (sel['leaf_ok'] == g['leaf_ok']).all()
    assert (sel['n_tree'] == g['n_tree']).all() and (sel['nb_leaves'] == g['nb_leaves']).all()


def test_select_seg_gate_golden():
    """fastseg.select_seg_fast on mean-log gated levels (gate_q 0.25, gate_min_level 2, neighbours on), leaf 2:
    the oracle's selection equals the reference's on every query."""
    g = load('sel_gate')
    nb = dict(nb_window=8, nb_store=2, nb_rho=0.35, nb_probe=3, nb_cap_min=2)
    sel = oracle.select_seg(g['q'], g['k'], g['lhat'], int(g['wmax']), L0=1, with_margin=True, nb=nb,
                            gate=(float(g['gate_q']), int(g['gate_min'])))
    srt = lambda a: np.sort(a, -1)
    assert (srt(sel['tree_pos']) == srt(g['tree_pos'])).all()
    assert (srt(sel['nb_pos']) == srt(g['nb_pos'])).all()
    assert (sel['n_tree'] == g['n_tree']).all() and (sel['nb_leaves'] == g['nb_leaves']).all()


def test_quantile_matches_torch():
    """The gate's threshold: torch.quantile's interpolation with its fused lerp, for several q."""
    gen = torch.Generator().manual_seed(0)
    for q in (0.25, 0.1, 0.33, 0.5, 0.9):
        x = torch.randn(2000, 64, generator=gen)
        np.testing.assert_array_equal(oracle.torch_quantile(x.numpy(), q), torch.quantile(x, q, dim=-1,
                                                                                            keepdim=True).numpy())


# ------------------------------------------------------------------------------------------------ dynamic tree
def test_dyn_tree_build_and_insert_golden():
    """dyntree.LaneTree (dyntree.py:46-106): the oracle's 2-means build, then 16 insertions, hold the same keys in the
    same groups as the reference's tree (children compared in canonical order: a two-key split's orientation is an
    exact fp32 tie), with the same counts and node sums within fp32 rounding; no decision is near a tie."""
    g = load('dyn_tree')
    t = oracle.LaneTreeNP(g['kfull'], g['n'], 3)
    assert (t.margin > 1e-5).all()
    a = oracle.canonical_tree(t.slot, t.sums, t.cnt)
    b = oracle.canonical_tree(g['slot0'], g['sums0'], g['cnt0'])
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[2], b[2])
    np.testing.assert_allclose(a[1], b[1], atol=1e-5)
    ar = np.arange(len(g['n']))
    for i in range(16):
        kpos = g['n'] + i
        t.insert(g['kfull'][ar, kpos], kpos, kpos >= 1)
    assert (t.margin > 1e-5).all()
    a = oracle.canonical_tree(t.slot, t.sums, t.cnt)
    b = oracle.canonical_tree(g['slot1'], g['sums1'], g['cnt1'])
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[2], b[2])
    np.testing.assert_allclose(a[1], b[1], atol=1e-5)
    assert t.check() < 1e-4


def _dyn_sel_args(g):
    return (int(g['chunk']), int(g['wmax']), int(g['nb_window']), int(g['nb_store']), float(g['nb_rho']),
            int(g['nb_probe']), int(g['nb_cap_min']))


@pytest.mark.parametrize('name', ['dyn_sel_a', 'dyn_sel_b'])
def test_dyn_select_keys_golden(name):
    """dyntree.select_keys (dyntree.py:150-243), neighbours on, random leaf budgets: every output equals the
    reference's on every query (no lane is near a tie)."""
    g = load(name)
    sel = oracle.select_keys(g['q'], g['k'], g['lhat'], *_dyn_sel_args(g))
    assert (sel['margin'] > 1e-6).all()
    for key in ('tree_pos', 'leaf_ok', 'nb_pos', 'n_tree', 'nb_leaves'):
        assert np.array_equal(sel[key], g[key]), key
    assert (g['nb_pos'] >= 0).sum() > 100


@pytest.mark.parametrize('name,kw', [('tiny_gpt_dyn', dict(beam_mode='fixed')),
                                     ('tiny_gpt_dyn_pred', dict(beam_mode='pred', global_pool=True, local=8))])
def test_tiny_gpt_dyn_golden(name, kw):
    """A tiny GPT with DynAttention (attn='dyn', attention_dyn.py): the oracle's logits within 1e-6 of the
    reference's and the same statistics (the model's weights come from the same seeded init)."""
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    cfg = Config(vocab_size=64, seq_len=64, n_layer=2, n_head=2, n_embd=32, attn='dyn', chunk=16, wmax=4, beam=2,
                 beam_classes=(2, 3, 4), nb_window=4, nb_store=2, nb_probe=2, nb_cap_min=1, **kw)
    torch.manual_seed(33)
    m = GPT(cfg)
    g = load(name)
    logits, st = oracle.gpt_forward_dyn(m.state_dict(), cfg.to_dict(), g['idx'])
    np.testing.assert_allclose(logits, g['logits'], atol=1e-6)
    for key in ('keys_total', 'keys_tree', 'keys_nb', 'nb_leaves', 'leaves_used'):
        assert abs(st[key] - float(g['stat_' + key])) < 1e-6, key


# ------------------------------------------------------------------------------------------------ block forest
def test_forest_build_golden():
    """forest.build_forest (forest.py:47-75): the oracle's rank order equals the reference's on every block (no
    decision near a tie), level sums within fp32 rounding, with and without the soft gate (forest.py:36-44)."""
    g = load('forest_build')
    perm, sums, margin = oracle.build_forest(g['k'], 32, 4, 3)
    assert (margin > 1e-6).all()
    assert np.array_equal(perm, g['perm'])
    for l in range(5):
        np.testing.assert_allclose(sums[l], g['S%d' % l], atol=2e-5)
    _, sums_g, _ = oracle.build_forest(g['k'], 32, 4, 3, gate=(0.25, 0.3))
    for l in range(5):
        np.testing.assert_allclose(sums_g[l], g['G%d' % l], atol=2e-5)


@pytest.mark.parametrize('name', ['tree_attn_a', 'tree_attn_b'])
def test_tree_attention_golden(name):
    """TreeAttention.sparse_attend (attention.py:47-143) on random q, k, v: outputs within 1e-5, same statistics."""
    g = load(name)
    out, st, margin = oracle.tree_attention(g['q'], g['k'], g['v'], int(g['tree_block']), int(g['wmax']),
                                            int(g['beam']))
    np.testing.assert_allclose(out, g['o'], atol=1e-5)
    for key in ('keys_tree', 'keys_total'):
        assert abs(st[key] - float(g['stat_' + key])) < 1e-4, key


@pytest.mark.parametrize('name,kw', [('tiny_gpt_block', dict()),
                                     ('tiny_gpt_block_pred', dict(beam_mode='pred', global_pool=True, gate=True))])
def test_tiny_gpt_block_golden(name, kw):
    """A tiny GPT with TreeAttention (attn='block'): the oracle's logits within 1e-5 of the reference's and the same
    statistics (the weights come from the same seeded init)."""
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=32, tree_block=32, wmax=4, beam=2,
                 beam_classes=(2, 3, 4), **kw)
    torch.manual_seed(43)
    m = GPT(cfg)
    g = load(name)
    logits, st = oracle.gpt_forward_block(m.state_dict(), cfg.to_dict(), g['idx'])
    np.testing.assert_allclose(logits, g['logits'], atol=1e-5)
    for key in ('keys_tree', 'keys_total'):
        assert abs(st[key] - float(g['stat_' + key])) < 1e-4, key
