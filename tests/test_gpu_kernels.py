"""Kernel-level parity on the GPU: every C-ABI entry point against the numpy oracle and the reference's golden
vectors. Node sums and selected index sets must match bit-exactly (selection: except queries whose reference
scores tie at a cut, see tests/_compare.py); attention outputs within 1e-4 (fp32) / 2e-2 (bf16)."""
import math

import numpy as np
import pytest
import torch

import oracle
from tests._compare import compare_sets, record, tied
from tests._golden import load

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def _ops():
    from treeattn_b200 import _ops
    return _ops


def _no_device_error():
    code = _ops().device_error()
    assert code[0] == 0, code


def to_dev(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a)).to(DEV, dtype)


def bf16_np(t):
    return t.float().cpu().numpy()


# ------------------------------------------------------------------------------------------------ levels
@pytest.mark.parametrize('L0,dtype,zero_sink', [(1, torch.float32, False), (1, torch.float32, True),
                                                (3, torch.bfloat16, True), (6, torch.bfloat16, True),
                                                (5, torch.float16, True), (2, torch.float32, True)])
def test_levels_bit_exact(L0, dtype, zero_sink):
    ops = _ops()
    g = torch.Generator().manual_seed(L0)
    B, H, T, dh = 2, 3, 512, 64
    k = torch.randn(B, T, H, dh, generator=g).to(DEV, dtype).transpose(1, 2)  # strided (b, T, H, dh) storage
    Lm = 8
    lv = ops.build_levels(k, T, L0, Lm, zero_sink=zero_sink)
    ref = oracle.level_sums(k.float().cpu().numpy(), L0, Lm, zero_sink=zero_sink)
    for l in range(L0, Lm + 1):
        assert np.array_equal(lv.level(l).cpu().numpy(), ref[l]), l
    _no_device_error()


def test_levels_golden():
    ops = _ops()
    g = load('levels')
    k = to_dev(g['k'])
    lv = ops.build_levels(k, 64, 1, 5, zero_sink=False)
    for l in range(1, 6):
        assert np.array_equal(lv.level(l).cpu().numpy(), g['S%d' % l]), l


def test_levels_partial_length():
    """T_len below capacity: only complete nodes are formed (SegState.fill of a shorter prompt)."""
    ops = _ops()
    g = torch.Generator().manual_seed(5)
    k = torch.randn(1, 2, 300, 32, generator=g).to(DEV)
    lv = ops.build_levels(k, 1024, 2, 9, zero_sink=True)
    ref = oracle.level_sums(k.cpu().numpy(), 2, 9, zero_sink=True)
    for l in range(2, 10):
        n = 300 >> l
        assert np.array_equal(lv.level(l)[:, :, :n].cpu().numpy(), ref[l][:, :, :n]), l


# ------------------------------------------------------------------------------------------------ selection
def _check_select(q, k, L0, wmax, qdtype=torch.float32, kdtype=torch.float32, T=None):
    ops = _ops()
    B, H, T_, dh = q.shape
    T = T or T_
    Lm = int(round(math.log2(T))) - 1
    kd = to_dev(k, kdtype)
    qd = to_dev(q, qdtype)
    lv = ops.build_levels(kd, T, L0, Lm, zero_sink=True)
    ids, vld, sct = ops.select(qd, lv, torch.arange(T, device=DEV), wmax)
    qn, kn = qd.float().cpu().numpy(), kd.float().cpu().numpy()
    S = oracle.level_sums(kn, L0, Lm, zero_sink=True)
    rids, rvld, rsct, margin = oracle.tree_pass(qn, S, np.arange(T), L0, Lm, wmax, with_margin=True)
    excl = tied(margin)
    bad, n, nx = compare_sets(ids.cpu().numpy(), vld.cpu().numpy(), rids, rvld, excl)
    assert bad == 0, (bad, n, nx)
    assert n >= 0.98 * B * H * T
    # same width, valid count and (where not tied) best-first scores
    assert ids.shape[-1] == rids.shape[-1]
    assert np.array_equal(vld.cpu().numpy().sum(-1), rvld.sum(-1))
    ok = ~excl[..., None] & rvld
    s_gpu, s_ref = sct.cpu().numpy(), rsct
    scale = np.where(ok, np.abs(s_ref), 0).max(-1, keepdims=True)
    assert (np.where(ok, np.abs(s_gpu - s_ref) - (5e-5 * scale + 1e-6), 0) <= 0).all()
    _no_device_error()
    return ids, vld


@pytest.mark.parametrize('name', ['sel_w4', 'sel_w8'])
def test_select_golden_leaf2(name):
    """GPU descent vs the reference's own select_seg output (leaf 2)."""
    g = load(name)
    ids, vld = _check_select(g['q'], g['k'], 1, int(g['wmax']))
    B, H, T, _ = g['q'].shape
    # against the reference directly (tie exclusion from the oracle's margins)
    Lm = int(round(math.log2(T))) - 1
    _, _, _, margin = oracle.tree_pass(g['q'], oracle.level_sums(g['k'], 1, Lm), np.arange(T), 1, Lm,
                                       int(g['wmax']), with_margin=True)
    bad, n, _ = compare_sets(ids.cpu().numpy(), vld.cpu().numpy(), g['ids'], g['vld'], tied(margin))
    assert bad == 0 and n > 0.98 * B * H * T


@pytest.mark.parametrize('name', ['tp_l3', 'tp_l5', 'tp_l6'])
def test_select_golden_leaf_blocks(name):
    g = load(name)
    L0, wmax = int(g['L0']), int(g['wmax'])
    ids, vld = _check_select(g['q'], g['k'], L0, wmax)
    B, H, T, _ = g['q'].shape
    Lm = int(round(math.log2(T))) - 1
    _, _, _, margin = oracle.tree_pass(g['q'], oracle.level_sums(g['k'], L0, Lm), np.arange(T), L0, Lm, wmax,
                                       with_margin=True)
    bad, n, _ = compare_sets(ids.cpu().numpy(), vld.cpu().numpy(), g['ids'], g['vld'], tied(margin))
    assert bad == 0 and n > 0.98 * B * H * T


@pytest.mark.parametrize('T,L0,wmax,dh,dt', [(1024, 1, 8, 16, torch.float32), (2048, 4, 32, 32, torch.bfloat16),
                                             (4096, 6, 16, 64, torch.bfloat16), (2048, 7, 32, 128, torch.bfloat16),
                                             (512, 2, 64, 64, torch.float16)])
def test_select_random(T, L0, wmax, dh, dt):
    g = np.random.default_rng(T + L0)
    q = g.standard_normal((1, 2, T, dh)).astype(np.float32)
    k = g.standard_normal((1, 2, T, dh)).astype(np.float32)
    _check_select(q, k, L0, wmax, qdtype=dt, kdtype=dt)


@pytest.mark.parametrize('T,L0,wmax,dh,dt,perm', [(8192, 6, 16, 64, torch.bfloat16, False),
                                                  (512, 5, 4, 64, torch.float32, False),
                                                  (1024, 3, 8, 128, torch.float16, True),
                                                  (4096, 5, 16, 32, torch.bfloat16, True),
                                                  (1000, 3, 16, 64, torch.float32, False),
                                                  (2048, 4, 12, 64, torch.bfloat16, False)])
def test_select_tile_matches_warp_kernel(T, L0, wmax, dh, dt, perm):
    """Whole sequences go through the tile kernel (dense per-level scores in shared memory, one thread per query);
    fewer than 32 queries per call through the warp-per-query kernel. Same scores in the same order, so ids,
    validity and scores are bit-identical (shuffled positions, a ragged last tile, a capacity that is not a power
    of two)."""
    ops = _ops()
    g = np.random.default_rng(T + L0 + dh)
    B, H = 2, 3
    q = torch.as_tensor(g.standard_normal((B, H, T, dh)).astype(np.float32)).to(DEV, dt)
    k = torch.as_tensor(g.standard_normal((B, H, T, dh)).astype(np.float32)).to(DEV, dt)
    Lm = int(math.ceil(math.log2(T))) - 1
    lv = ops.build_levels(k, T, L0, Lm)
    tq = torch.randperm(T, device=DEV) if perm else torch.arange(T, device=DEV)
    ids, vld, sct = ops.select(q, lv, tq, wmax)
    for s0 in range(0, T, 16):
        i2, v2, s2 = ops.select(q[:, :, s0:s0 + 16], lv, tq[s0:s0 + 16], wmax)
        assert torch.equal(i2, ids[:, :, s0:s0 + 16]), s0
        assert torch.equal(v2, vld[:, :, s0:s0 + 16]), s0
        assert torch.equal(s2, sct[:, :, s0:s0 + 16]), s0
    _no_device_error()


def test_select_per_batch_positions_and_small_lm():
    """Per-sequence positions (decode form) and a top level below the highest position bit (the reference then
    never injects the older subtrees: seg.py:54-57 with Lm < log2 t)."""
    ops = _ops()
    g = np.random.default_rng(3)
    B, H, T, dh, L0, wmax = 3, 2, 1024, 32, 3, 4
    k = g.standard_normal((B, H, T, dh)).astype(np.float32)
    q = g.standard_normal((B, H, 1, dh)).astype(np.float32)
    for Lm in (9, 6):
        lv = ops.build_levels(to_dev(k), T, L0, Lm)
        pos = torch.tensor([1000, 513, 77], device=DEV)
        ids, vld, sct = ops.select(to_dev(q), lv, pos, wmax)
        S = oracle.level_sums(k, L0, Lm)
        rids, rvld, _, margin = oracle.tree_pass(q, S, pos.cpu().numpy()[:, None], L0, Lm, wmax, with_margin=True)
        bad, n, _ = compare_sets(ids.cpu().numpy(), vld.cpu().numpy(), rids, rvld, tied(margin))
        assert bad == 0 and n >= B * H - 1, (Lm, bad, n)


def test_finish_matches_oracle():
    ops = _ops()
    g = np.random.default_rng(0)
    Q, wl, nbw, leaf, wmax = 300, 8, 6, 4, 8
    ids = g.integers(0, 50, (Q, wl))
    vld = g.random((Q, wl)) < 0.7
    nid = g.integers(0, 50, (Q, nbw))
    match = g.random((Q, nbw)) < 0.4
    nL = g.integers(0, 6, Q)
    lhat = g.integers(0, 9, Q)
    r = ops.finish(to_dev(ids, torch.int64), to_dev(vld, torch.bool), to_dev(lhat, torch.int64), wmax, leaf,
                   nid=to_dev(nid, torch.int64), match=to_dev(match, torch.bool), nL=to_dev(nL, torch.int64))
    ref = oracle.finish(ids, vld, nid, match, nL, lhat, wmax, leaf=leaf)
    for key in ('tree_pos', 'nb_pos', 'n_tree', 'nb_leaves'):
        assert np.array_equal(r[key].cpu().numpy(), ref[key]), key


# ------------------------------------------------------------------------------------------------ attention
def test_sparse_attn_golden():
    from treeattn_b200.fastseg import sparse_attn
    g = load('attn')
    q, k, v = to_dev(g['q']), to_dev(g['k']), to_dev(g['v'])
    with torch.no_grad():
        o = sparse_attn(q, k, v, to_dev(g['cand'], torch.int64), 0.125)
    np.testing.assert_allclose(o.cpu().numpy(), g['o'], atol=1e-4)
    o32 = sparse_attn(q, k, v, to_dev(g['cand'], torch.int32), 0.125)
    np.testing.assert_allclose(o32.cpu().numpy(), g['o'], atol=1e-4)
    ob = sparse_attn(q.bfloat16(), k.bfloat16(), v.bfloat16(), to_dev(g['cand'], torch.int32), 0.125)
    ref_b = oracle.sparse_attn(bf16_np(q.bfloat16()), bf16_np(k.bfloat16()), bf16_np(v.bfloat16()), g['cand'], 0.125)
    np.testing.assert_allclose(ob.float().cpu().numpy(), ref_b, atol=2e-2)
    _no_device_error()


def test_gather_dot_golden():
    from treeattn_b200.fastseg import gather_dot
    g = load('attn')
    d = gather_dot(to_dev(g['q']), to_dev(g['S']), to_dev(g['cd'], torch.int64), 0.5)
    np.testing.assert_allclose(d.cpu().numpy(), g['dot'], atol=1e-4, rtol=1e-5)


def test_gather_dot_blocks_config2_shape():
    """Configuration 2 shapes: B=8, H=12, dh=64, T=4096 bf16, 16 sorted unique blocks of 64 per (b, h)."""
    ops = _ops()
    torch.manual_seed(0)
    B, H, T, dh, blk, nblk = 8, 12, 4096, 64, 64, 16
    q = torch.randn(B, H, dh, device=DEV).bfloat16()
    K = torch.randn(B, H, T, dh, device=DEV).bfloat16()
    blocks = torch.stack([torch.randperm(T // blk, device=DEV)[:nblk].sort().values for _ in range(B * H)])
    blocks = blocks.view(B, H, nblk).int()
    for nb_cta in (1, 2, 4, 16):
        out = ops.gather_dot_blocks(q, K, blocks, blk, 0.125, nb_cta=nb_cta)
        cand = (blocks.long().unsqueeze(-1) * blk + torch.arange(blk, device=DEV)).view(B, H, 1, nblk * blk)
        ref = oracle.gather_dot(bf16_np(q)[:, :, None], bf16_np(K), cand.cpu().numpy(), 0.125)[:, :, 0]
        np.testing.assert_allclose(out.cpu().numpy(), ref, atol=1e-4, rtol=1e-5)
        gen = ops.gather_dot(q[:, :, None], K, cand, 0.125)[:, :, 0]
        np.testing.assert_allclose(gen.cpu().numpy(), ref, atol=1e-4, rtol=1e-5)
    _no_device_error()


def test_dedupe_golden():
    from treeattn_b200.attention_dyn import dedupe
    from treeattn_b200.fastseg import dedupe_fast
    g = load('dedupe')
    c, v = to_dev(g['cand'], torch.int64), to_dev(g['valid'], torch.bool)
    assert np.array_equal(dedupe(c, v).cpu().numpy(), g['keep'])
    assert np.array_equal(dedupe_fast(c, v).cpu().numpy(), g['keep'])


@pytest.mark.parametrize('T,L0,wmax,beam,local,dh,dt', [(256, 1, 4, 2, 3, 16, torch.float32),
                                                        (512, 5, 4, 4, 64, 64, torch.float32),
                                                        (1024, 6, 16, 16, 128, 64, torch.bfloat16),
                                                        (1024, 4, 8, 3, 20, 32, torch.float16),
                                                        (512, 7, 4, 4, 256, 128, torch.bfloat16)])
def test_seg_attn_vs_oracle(T, L0, wmax, beam, local, dh, dt):
    """Attention over the GPU's own selection vs the oracle's key assembly + dedupe + exact softmax."""
    ops = _ops()
    g = np.random.default_rng(T + dh)
    B, H = 2, 2
    q, k, v = [to_dev(g.standard_normal((B, H, T, dh)).astype(np.float32), dt) for _ in range(3)]
    Lm = int(round(math.log2(T))) - 1
    lv = ops.build_levels(k, T, L0, Lm)
    tq = torch.arange(T, device=DEV)
    ids, vld, _ = ops.select(q, lv, tq, wmax)
    ntree = oracle.n_tree_fixed(beam, wmax)
    Lw = max(local, 3)
    o, lse, nkeys = ops.seg_attn(q, k, v, tq, ids, vld, ntree, 1 << L0, Lw, 1 / math.sqrt(dh), want_lse=True)
    # oracle key set from the same selection
    idn, vdn = ids.cpu().numpy(), vld.cpu().numpy()
    wl = idn.shape[-1]
    used = vdn & (np.arange(wl) < ntree)
    tree_pos = oracle.leaves_to_pos(idn, vdn, 1 << L0)
    tv = np.concatenate([used] * (1 << L0), -1) & (tree_pos >= 0)
    st = np.broadcast_to(oracle.static_keys(np.arange(T), Lw), (B, H, T, 1 + Lw))
    cand = np.concatenate([tree_pos, st], -1)
    keep = oracle.dedupe(cand, np.concatenate([tv, st >= 0], -1))
    ref = oracle.sparse_attn(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                             np.where(keep, cand, -1), 1 / math.sqrt(dh))
    tol = 1e-4 if dt == torch.float32 else 2e-2
    np.testing.assert_allclose(o.float().cpu().numpy(), ref, atol=tol)
    assert np.array_equal(nkeys.cpu().numpy(), keep.sum(-1))
    _no_device_error()


# ------------------------------------------------------------------------------------------------ append
@pytest.mark.parametrize('L0,dt', [(1, torch.float32), (3, torch.bfloat16), (6, torch.bfloat16)])
def test_append_incremental_tree(L0, dt):
    """SegState.add token by token == bulk level build (reference engine.py:41-55 vs 57-71)."""
    ops = _ops()
    from treeattn_b200._ops import Levels
    g = torch.Generator().manual_seed(L0)
    B, H, dh, cap, Lm = 2, 3, 64, 300, 9
    K = torch.randn(B, H, cap, dh, generator=g).to(DEV, dt)
    V = torch.randn(B, H, cap, dh, generator=g).to(DEV, dt)
    kc = torch.zeros_like(K)
    vc = torch.zeros_like(V)
    lv = Levels.empty(B, H, dh, cap, L0, Lm, DEV)
    for t in range(cap):
        pos = torch.full((B,), t, device=DEV, dtype=torch.int32)
        ops.append(K[:, :, t], V[:, :, t], kc, vc, lv, pos)
    assert torch.equal(kc, K) and torch.equal(vc, V)
    ref = ops.build_levels(K, cap, L0, Lm, zero_sink=True)
    for l in range(L0, Lm + 1):
        n = cap >> l
        assert torch.equal(lv.level(l)[:, :, :n], ref.level(l)[:, :, :n]), l
    _no_device_error()


# ------------------------------------------------------------------------------------------------ fused decode
@pytest.mark.parametrize('dt,dh,L0,wmax,beam,local,splits', [
    (torch.bfloat16, 64, 6, 16, 16, 128, -1),
    (torch.bfloat16, 128, 7, 32, 32, 256, -1),
    (torch.float32, 32, 2, 8, 3, 8, -1),
    (torch.bfloat16, 64, 6, 16, 16, 128, 1),
    (torch.bfloat16, 64, 6, 16, 16, 128, 4),
    (torch.bfloat16, 64, 6, 16, 16, 128, 8),
    (torch.bfloat16, 128, 7, 8, 8, 256, 2),
    (torch.float32, 64, 1, 4, 2, 3, 1),
    (torch.float32, 32, 3, 8, 3, 16, 2),
    (torch.float16, 16, 2, 4, 4, 8, 1),
])
def test_decode_step_vs_oracle(dt, dh, L0, wmax, beam, local, splits):
    """Fused decode (descent + attention + append + tree update) over steps that cross leaf-block boundaries,
    with ragged per-sequence positions, against the oracle's seg_attend on the same cache contents."""
    ops = _ops()
    from treeattn_b200._ops import Levels
    rng = np.random.default_rng(dh + L0 + splits)
    B, H = 3, 2
    C = H * dh
    leaf = 1 << L0
    T0 = [5 * leaf + 3, 4 * leaf - 7, 7 * leaf + leaf // 2]
    steps = 2 * leaf + 5
    cap = max(T0) + steps + 1
    Tcap = 1 << int(math.ceil(math.log2(cap)))
    Lm = int(round(math.log2(Tcap))) - 1
    Lw = max(local, 3)
    rnd = (lambda a: a) if dt == torch.float32 else (lambda a: torch.as_tensor(a).to(dt).float().numpy())
    kc = torch.zeros(B, H, cap, dh, device=DEV, dtype=dt)
    vc = torch.zeros_like(kc)
    lv = Levels.empty(B, H, dh, cap, L0, Lm, DEV)
    states = []
    for b in range(B):
        K0 = rnd(rng.standard_normal((H, T0[b], dh)).astype(np.float32))
        V0 = rnd(rng.standard_normal((H, T0[b], dh)).astype(np.float32))
        kc[b, :, :T0[b]] = torch.as_tensor(K0).to(DEV, dt)
        vc[b, :, :T0[b]] = torch.as_tensor(V0).to(DEV, dt)
        lvb = Levels(lv.nodes[b:b + 1], cap, L0, Lm)
        ops.build_levels(kc[b:b + 1, :, :T0[b]], cap, L0, Lm, zero_sink=True, out=lvb)
        s = oracle.SegStateNP(H, dh, cap, L0, Lm)
        s.fill(K0, V0)
        states.append(s)
    out = torch.empty(B, C, device=DEV, dtype=dt)
    nkeys = torch.empty(B, H, device=DEV, dtype=torch.int32)
    sel = torch.empty(B, H, wmax + 1, device=DEV, dtype=torch.int32)
    lse = torch.empty(B, H, device=DEV, dtype=torch.float32)
    ntree = oracle.n_tree_fixed(beam, wmax)
    n_cmp = n_bad = n_tie = 0
    for s_i in range(steps):
        pos = torch.tensor([T0[b] + s_i for b in range(B)], device=DEV, dtype=torch.int32)
        qkv_np = rnd(rng.standard_normal((B, 3 * C)).astype(np.float32))
        qkv = torch.as_tensor(qkv_np).to(DEV, dt)
        ops.decode_step(qkv, kc, vc, lv, pos, H, wmax, ntree, Lw, 1 / math.sqrt(dh), out, lse=lse, nkeys=nkeys,
                        sel=sel, splits=splits)
        o_n, nk_n, sel_n = out.float().cpu().numpy(), nkeys.cpu().numpy(), sel.cpu().numpy()
        for b in range(B):
            q, k, v = [qkv_np[b, j * C:(j + 1) * C].reshape(H, dh) for j in range(3)]
            ro, rkeys, (rids, rused, margin) = oracle.seg_attend(states[b], q, k, v, T0[b] + s_i, wmax, beam, local,
                                                                 with_sel=True)
            for h in range(H):
                if margin[h] <= 1e-6:
                    n_tie += 1
                    continue
                n_cmp += 1
                got = sorted(sel_n[b, h, 1:1 + sel_n[b, h, 0]].tolist())
                want = sorted(rids[h][rused[h]].tolist())
                if got != want:
                    n_bad += 1
                    continue
                tol = 1e-4 if dt == torch.float32 else 2e-2
                np.testing.assert_allclose(o_n[b, h * dh:(h + 1) * dh], ro[h], atol=tol)
                assert nk_n[b, h] == len(set(
                    [p for p in oracle.leaves_to_pos(rids[h], rused[h], leaf).tolist() if p >= 0] +
                    [0] + list(range(max(0, T0[b] + s_i - Lw + 1), T0[b] + s_i + 1)))), (b, h, s_i)
    record(n_cmp, n_tie, n_bad)
    assert n_bad == 0 and n_cmp > 0.95 * steps * B * H, (n_bad, n_cmp)
    # caches and tree equal the oracle's after all appends (nodes bit-exact)
    for b in range(B):
        n = T0[b] + steps
        np.testing.assert_array_equal(kc[b, :, :n].float().cpu().numpy(), states[b].K[:, :n])
        np.testing.assert_array_equal(vc[b, :, :n].float().cpu().numpy(), states[b].V[:, :n])
        for l in range(L0, Lm + 1):
            m = n >> l
            np.testing.assert_array_equal(lv.level(l)[b, :, :m].cpu().numpy(), states[b].levels[l][0, :, :m])
    _no_device_error()


@pytest.mark.parametrize('dt,dh,L0', [(torch.bfloat16, 64, 4), (torch.float16, 128, 5)])
def test_decode_persistent_many_items(dt, dh, L0):
    """Persistent kernel with several (b, h) items per CTA (descriptor-slot reuse, partial-state hand-off), ragged
    positions, steps crossing leaf-block boundaries: outputs, key counts, caches and tree vs the oracle."""
    ops = _ops()
    from treeattn_b200._ops import Levels
    rng = np.random.default_rng(dh)
    B, H = 40, 16
    C = H * dh
    leaf = 1 << L0
    wmax, beam, local = 8, 8, 2 * leaf
    T0 = rng.integers(3 * leaf, 12 * leaf, B).tolist()
    steps = leaf + 3
    cap = max(T0) + steps + 1
    Tcap = 1 << int(math.ceil(math.log2(cap)))
    Lm = int(round(math.log2(Tcap))) - 1
    rnd = lambda a: torch.as_tensor(a).to(dt).float().numpy()
    kc = torch.zeros(B, H, cap, dh, device=DEV, dtype=dt)
    vc = torch.zeros_like(kc)
    lv = Levels.empty(B, H, dh, cap, L0, Lm, DEV)
    states = []
    for b in range(B):
        K0 = rnd(rng.standard_normal((H, T0[b], dh)).astype(np.float32))
        V0 = rnd(rng.standard_normal((H, T0[b], dh)).astype(np.float32))
        kc[b, :, :T0[b]] = torch.as_tensor(K0).to(DEV, dt)
        vc[b, :, :T0[b]] = torch.as_tensor(V0).to(DEV, dt)
        st = oracle.SegStateNP(H, dh, cap, L0, Lm)
        st.fill(K0, V0)
        states.append(st)
    ops.build_levels(kc, cap, L0, Lm, zero_sink=True, out=lv)  # complete nodes of each row's own prefix only
    for b in range(B):  # rows with shorter prompts: clear nodes beyond their own complete prefix
        for l in range(L0, Lm + 1):
            lv.level(l)[b, :, T0[b] >> l:] = 0
    out = torch.empty(B, C, device=DEV, dtype=dt)
    nkeys = torch.empty(B, H, device=DEV, dtype=torch.int32)
    ntree = oracle.n_tree_fixed(beam, wmax)
    worst = 0.0
    for s_i in range(steps):
        pos = torch.tensor([T0[b] + s_i for b in range(B)], device=DEV, dtype=torch.int32)
        qkv_np = rnd(rng.standard_normal((B, 3 * C)).astype(np.float32))
        ops.decode_step(torch.as_tensor(qkv_np).to(DEV, dt), kc, vc, lv, pos, H, wmax, ntree, local,
                        1 / math.sqrt(dh), out, nkeys=nkeys, splits=-1)
        o_n, nk_n = out.float().cpu().numpy(), nkeys.cpu().numpy()
        for b in range(B):
            q, k, v = [qkv_np[b, j * C:(j + 1) * C].reshape(H, dh) for j in range(3)]
            ro, _, (rids, rused, margin) = oracle.seg_attend(states[b], q, k, v, T0[b] + s_i, wmax, beam, local,
                                                             with_sel=True)
            ok = margin > 1e-6
            record(int(ok.sum()), int((~ok).sum()), 0, 'outputs')
            d = np.abs(o_n[b].reshape(H, dh) - ro).max(-1)
            worst = max(worst, float(d[ok].max(initial=0)))
    assert worst < 2e-2, worst
    for b in range(B):
        n = T0[b] + steps
        np.testing.assert_array_equal(kc[b, :, :n].float().cpu().numpy(), states[b].K[:, :n])
        for l in range(L0, Lm + 1):
            m = n >> l
            np.testing.assert_array_equal(lv.level(l)[b, :, :m].cpu().numpy(), states[b].levels[l][0, :, :m])
    _no_device_error()


@pytest.mark.parametrize('splits', [-1, 1])
def test_decode_long_context_wide_heads(splits):
    """dh=128 with 128-token leaf blocks and long prompts: the descent gathers several levels below the prefetched
    ones on demand, each item streams ~130 stages through the ring (every slot reused many times by both consumer
    groups), and the window alone spans 8 stages. Selected sets, outputs and key counts vs the oracle."""
    ops = _ops()
    from treeattn_b200._ops import Levels
    dt, dh, L0, wmax, beam, local = torch.bfloat16, 128, 7, 32, 32, 256
    rng = np.random.default_rng(5)
    B, H = 6, 4
    C = H * dh
    leaf = 1 << L0
    T0 = rng.integers(7000, 12000, B).tolist()
    steps = 3
    cap = max(T0) + steps + 1
    Tcap = 1 << int(math.ceil(math.log2(cap)))
    Lm = int(round(math.log2(Tcap))) - 1
    rnd = lambda a: torch.as_tensor(a).to(dt).float().numpy()
    kc = torch.zeros(B, H, cap, dh, device=DEV, dtype=dt)
    vc = torch.zeros_like(kc)
    lv = Levels.empty(B, H, dh, cap, L0, Lm, DEV)
    states = []
    for b in range(B):
        K0 = rnd(rng.standard_normal((H, T0[b], dh)).astype(np.float32))
        V0 = rnd(rng.standard_normal((H, T0[b], dh)).astype(np.float32))
        kc[b, :, :T0[b]] = torch.as_tensor(K0).to(DEV, dt)
        vc[b, :, :T0[b]] = torch.as_tensor(V0).to(DEV, dt)
        st = oracle.SegStateNP(H, dh, cap, L0, Lm)
        st.fill(K0, V0)
        states.append(st)
    ops.build_levels(kc, cap, L0, Lm, zero_sink=True, out=lv)
    for b in range(B):
        for l in range(L0, Lm + 1):
            lv.level(l)[b, :, T0[b] >> l:] = 0
    out = torch.empty(B, C, device=DEV, dtype=dt)
    nkeys = torch.empty(B, H, device=DEV, dtype=torch.int32)
    sel = torch.empty(B, H, wmax + 1, device=DEV, dtype=torch.int32)
    ntree = oracle.n_tree_fixed(beam, wmax)
    worst, n_cmp, n_tie = 0.0, 0, 0
    for s_i in range(steps):
        pos = torch.tensor([T0[b] + s_i for b in range(B)], device=DEV, dtype=torch.int32)
        qkv_np = rnd(rng.standard_normal((B, 3 * C)).astype(np.float32))
        ops.decode_step(torch.as_tensor(qkv_np).to(DEV, dt), kc, vc, lv, pos, H, wmax, ntree, local,
                        1 / math.sqrt(dh), out, nkeys=nkeys, sel=sel, splits=splits)
        o_n, nk_n, sel_n = out.float().cpu().numpy(), nkeys.cpu().numpy(), sel.cpu().numpy()
        for b in range(B):
            q, k, v = [qkv_np[b, j * C:(j + 1) * C].reshape(H, dh) for j in range(3)]
            ro, _, (rids, rused, margin) = oracle.seg_attend(states[b], q, k, v, T0[b] + s_i, wmax, beam, local,
                                                             with_sel=True)
            for h in range(H):
                if margin[h] <= 1e-6:
                    n_tie += 1
                    continue
                n_cmp += 1
                assert sorted(sel_n[b, h, 1:1 + sel_n[b, h, 0]].tolist()) == sorted(rids[h][rused[h]].tolist())
                worst = max(worst, float(np.abs(o_n[b, h * dh:(h + 1) * dh] - ro[h]).max()))
                assert nk_n[b, h] == len(set(
                    [p for p in oracle.leaves_to_pos(rids[h], rused[h], leaf).tolist() if p >= 0] +
                    [0] + list(range(T0[b] + s_i - local + 1, T0[b] + s_i + 1)))), (b, h, s_i)
    record(n_cmp, n_tie)
    assert worst < 2e-2 and n_cmp > 0.9 * steps * B * H, (worst, n_cmp)
    _no_device_error()


@pytest.mark.parametrize('B,H,steps,dh', [(10, 16, 6, 128), (20, 16, 3, 128), (8, 12, 4, 64), (3, 12, 3, 64)])
def test_decode_split_items_match_whole_items(B, H, steps, dh):
    """Persistent decode with the split scratch: items cut into parts (windows and leaf rows shared out, partial
    states merged by the last part) give the outputs of whole items up to the merge order, the same selections and
    key counts, and the same caches and tree (appended once), over steps that complete leaf blocks. 256-byte rows
    (dh 128 bf16, one CTA per SM) split the last round's items; 128-byte rows split every item when there are fewer
    items than CTA slots (small batches: 96 and 36 items)."""
    ops = _ops()
    from treeattn_b200._ops import Levels
    dt = torch.bfloat16
    L0, wmax, local = (7, 32, 256) if dh == 128 else (6, 16, 128)
    rng = np.random.default_rng(B)
    C = H * dh
    T0 = (rng.integers(3000, 6000, B) // (1 << L0) * (1 << L0) - 2).tolist()
    cap = max(T0) + steps + 1
    Lm = int(math.ceil(math.log2(cap)))
    kc = torch.randn(B, H, cap, dh, device=DEV).to(dt)
    vc = torch.randn(B, H, cap, dh, device=DEV).to(dt)
    lv = Levels.empty(B, H, dh, cap, L0, Lm, DEV)
    ops.build_levels(kc, cap, L0, Lm, zero_sink=True, out=lv)
    kc2, vc2 = kc.clone(), vc.clone()
    lv2 = Levels(lv.nodes.clone(), cap, L0, Lm)
    scratch = ops.split_scratch(B, H, dh, DEV)
    outs = [torch.empty(B, C, device=DEV, dtype=dt) for _ in range(2)]
    lses = [torch.empty(B, H, device=DEV) for _ in range(2)]
    nks = [torch.empty(B, H, device=DEV, dtype=torch.int32) for _ in range(2)]
    sels = [torch.empty(B, H, wmax + 1, device=DEV, dtype=torch.int32) for _ in range(2)]
    for s_i in range(steps):
        pos = torch.tensor([T0[b] + s_i for b in range(B)], device=DEV, dtype=torch.int32)
        qkv = torch.randn(B, 3 * C, device=DEV).to(dt)
        ops.decode_step(qkv, kc, vc, lv, pos, H, wmax, wmax, local, 1 / math.sqrt(dh), outs[0], lse=lses[0],
                        nkeys=nks[0], sel=sels[0], splits=-1)
        ops.decode_step(qkv, kc2, vc2, lv2, pos, H, wmax, wmax, local, 1 / math.sqrt(dh), outs[1], lse=lses[1],
                        nkeys=nks[1], sel=sels[1], splits=-1, scratch=scratch)
        assert (outs[0].float() - outs[1].float()).abs().max().item() < 2e-2
        # p is rounded to bf16 against the running maximum of the part that holds it: the sums differ at that
        # precision (2^-9 relative at most)
        assert (lses[0] - lses[1]).abs().max().item() < 2e-3
        assert torch.equal(nks[0], nks[1]) and torch.equal(sels[0], sels[1])
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(lv.nodes, lv2.nodes)
    assert int(scratch[1].abs().sum()) == 0  # every counter reset by its merging part
    _no_device_error()


def test_decode_bad_position_records_error():
    """A position outside the capacity is rejected inside the kernel (no memory access, error recorded)."""
    ops = _ops()
    from treeattn_b200._ops import Levels
    B, H, dh, cap = 2, 2, 64, 128
    kc = torch.zeros(B, H, cap, dh, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    lv = Levels.empty(B, H, dh, cap, 3, 6, DEV)
    qkv = torch.randn(B, 3 * H * dh, device=DEV).bfloat16()
    out = torch.empty(B, H * dh, device=DEV, dtype=torch.bfloat16)
    ops.device_error()
    pos = torch.tensor([5, cap + 10], device=DEV, dtype=torch.int32)
    for splits in (1, -1):
        kc.zero_()
        ops.decode_step(qkv, kc, vc, lv, pos, H, 4, 4, 8, 0.125, out, splits=splits)
        code = ops.device_error()
        assert code[0] == 2 and code[2] == cap + 10, (splits, code)
        assert kc[0, :, 5].abs().sum() > 0  # the valid sequence was still processed


def test_bounded_wait_gives_up_and_context_stays_usable():
    """A wait that nothing completes (ta_wait_probe: an mbarrier no thread arrives at) gives up after its limit,
    records code 1 (bounded wait gave up) for kernel 13 and ends; the next kernels run and give correct results."""
    import time
    from treeattn_b200 import _lib
    from treeattn_b200 import _ops as ops_mod
    _no_device_error()
    torch.cuda.synchronize()
    t0 = time.time()
    _lib.call('ta_wait_probe', 200 * 1000 * 1000, ops_mod._stream(torch.empty(1, device=DEV)))
    assert ops_mod.device_error() == (1, 13, 7, 0)
    assert 0.15 < time.time() - t0 < 30
    g = load('levels')  # the context still works: the golden level build afterwards
    lv = _ops().build_levels(to_dev(g['k']), 64, 1, 5, zero_sink=False)
    for l in range(1, 6):
        assert np.array_equal(lv.level(l).cpu().numpy(), g['S%d' % l]), l
    _no_device_error()


def test_bad_arguments_raise():
    ops = _ops()
    from treeattn_b200._lib import TreeAttnError
    q = torch.randn(1, 2, 16, 48, device=DEV)  # head dim 48 unsupported
    with pytest.raises(TreeAttnError):
        ops.build_levels(q, 16, 1, 3)
    q = torch.randn(1, 2, 16, 64, device=DEV)
    lv = ops.build_levels(q, 16, 1, 3)
    with pytest.raises(TreeAttnError):
        ops.select(q, lv, torch.arange(16, device=DEV), 0)  # wmax 0
    with pytest.raises(ValueError):
        ops.build_levels(q.cpu(), 16, 1, 3)  # CPU tensors: no CPU path


# ------------------------------------------------------------------------------------------------ lane tree
@pytest.mark.parametrize('wmax', [4, 8, 3])
def test_lane_search_golden(wmax):
    """LaneTree.search on the tree the reference built and grew (golden): same valid leaves, scores within 1e-6."""
    from treeattn_b200.dyntree import LaneTree
    g = load('lanetree')
    tree = LaneTree.from_levels(to_dev(g['sums']), torch.as_tensor(g['cnt']).to(DEV))
    assert tree.D == int(g['D'])
    ids, vld, sct = tree.search(to_dev(g['q']), wmax)
    _, _, _, margin = oracle.lane_search(g['q'], g['sums'], g['cnt'], int(g['D']), wmax, with_margin=True)
    bad, n, _ = compare_sets(ids.cpu().numpy(), vld.cpu().numpy(), g['ids_%d' % wmax], g['vld_%d' % wmax],
                             tied(margin))
    assert bad == 0 and n == g['q'].shape[0]
    v = vld.cpu().numpy()
    np.testing.assert_allclose(np.where(v, sct.cpu().numpy(), 0), np.where(g['vld_%d' % wmax], g['sct_%d' % wmax], 0),
                               atol=1e-6)
    _no_device_error()


@pytest.mark.parametrize('P,D,dh,wmax', [(300, 9, 64, 16), (64, 6, 128, 8), (100, 10, 16, 64), (7, 3, 32, 2)])
def test_lane_search_random(P, D, dh, wmax):
    """Random trees with empty subtrees (count 0 prunes a node and everything below it): kernel vs oracle."""
    from treeattn_b200.dyntree import LaneTree
    rng = np.random.default_rng(P + D)
    NN = (2 << D) - 1
    leaf_cnt = rng.integers(0, 3, (P, 1 << D))
    leaf_cnt[rng.random((P, 1 << D)) < 0.3] = 0
    leaf_sum = (rng.standard_normal((P, 1 << D, dh)) * leaf_cnt[..., None]).astype(np.float32)
    sums, cnt = [leaf_sum], [leaf_cnt]
    for _ in range(D):
        s_, c_ = sums[0], cnt[0]
        sums.insert(0, s_.reshape(P, -1, 2, dh).sum(2))
        cnt.insert(0, c_.reshape(P, -1, 2).sum(2))
    S = np.concatenate(sums, 1).astype(np.float32)
    Cn = np.concatenate(cnt, 1).astype(np.int32)
    assert S.shape[1] == NN
    q = rng.standard_normal((P, dh)).astype(np.float32)
    tree = LaneTree.from_levels(to_dev(S), torch.as_tensor(Cn).to(DEV))
    ids, vld, sct = tree.search(to_dev(q), wmax)
    rids, rvld, rsct, margin = oracle.lane_search(q, S, Cn, D, wmax, with_margin=True)
    bad, n, _ = compare_sets(ids.cpu().numpy(), vld.cpu().numpy(), rids, rvld, tied(margin))
    assert bad == 0 and n >= 0.98 * P, (bad, n)
    assert (vld.cpu().numpy().sum(-1) == rvld.sum(-1)).all()
    _no_device_error()
