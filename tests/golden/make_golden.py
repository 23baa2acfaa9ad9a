"""Generate the golden fixtures in tests/golden/ by running the reference implementation itself.

The reference (Dex8123/treeattn, pure Python/PyTorch) is importable only in the build container, where it is
mounted read-only; it is made importable as the package `treeattn` through a symlink in a temp directory.
The GPU box never runs this script: the tests read the committed .npz files.

    python tests/golden/make_golden.py /path/to/reference [--only=lanetree|tiny_gpt_nb|gate|dyn|forest|interop]

Leaf blocks of 2^L0 tokens (the benchmark configs use 32, 64 and 128) are produced with the reference's own
functions on the level-shifted tree ("adapter"): seg.level_sums, then seg.tree_pass with
getU(l, c) = gather_nodes(S[l + L0 - 1], c), query positions t >> (L0 - 1) and top level Lm - (L0 - 1).
For the whole-model golden of configuration 1 the adapter result is handed to the reference's SegAttention in
its own level-1 representation (each selected block = 2^(L0-1) level-1 leaves, n_tree scaled the same way).
"""
import math
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def import_reference(path):
    d = tempfile.mkdtemp(prefix='refpkg_')
    os.symlink(os.path.abspath(path), os.path.join(d, 'treeattn'))
    sys.path.insert(0, d)
    import treeattn  # noqa: F401
    from treeattn import config, engine, fastseg, forest, model, seg, attention_dyn, dyntree
    return dict(config=config, engine=engine, fastseg=fastseg, forest=forest, model=model, seg=seg,
                attention_dyn=attention_dyn, dyntree=dyntree)


def lanetree_golden(R):
    """dyntree.LaneTree.search (dyntree.py:108-127) on a tree the reference builds (2-means splits) and grows
    (insertions), lanes with different prefix lengths; the node sums / counts are stored packed level by level
    (level l at rows 2^l - 1 .. 2^(l+1) - 2), the way the B200 kernel reads them."""
    dyn = R['dyntree']
    torch.manual_seed(5)
    P, C, dh = 6, 256, 32
    kfull = torch.randn(P, C, dh)
    n = torch.tensor([0, 17, 64, 100, 150, 200])
    tree = dyn.LaneTree(kfull, n, iters=3)
    ar = torch.arange(P)
    for i in range(20):
        kpos = n + i
        tree.insert(kfull[ar, kpos], kpos, kpos >= 1)
    qt = torch.randn(P, dh)
    d = dict(q=np_(qt), sums=np_(torch.cat(tree.sums, 1)), cnt=np_(torch.cat(tree.cnt, 1)), D=tree.D)
    for wmax in (4, 8, 3):
        cur, cvld, sct = tree.search(qt, wmax)
        d['ids_%d' % wmax], d['vld_%d' % wmax], d['sct_%d' % wmax] = np_(cur), np_(cvld), np_(sct)
    return d


def np_(t):
    return t.detach().cpu().numpy()


def adapter_tree_pass(R, q, k, L0, wmax):
    """Reference tree_pass on the level-shifted tree (leaves = level-L0 nodes)."""
    seg, forest = R['seg'], R['forest']
    b, H, T, dh = q.shape
    Lm = int(round(math.log2(T))) - 1
    kidx = k.float().clone()
    kidx[:, :, 0, :] = 0
    S = seg.level_sums(kidx, Lm, False, 0.25)
    sh = L0 - 1

    def getU(l, c):
        return forest.gather_nodes(S[l + sh], c)

    tq = torch.arange(T) >> sh
    return seg.tree_pass(q.float(), getU, tq, Lm - sh, wmax)


def tiny_gpt_nb_golden(R):
    """A tiny GPT with neighbour borrowing on (the reference's default cfg.neighbors=True), leaf 2: the forward
    logits and statistics, and the reference engine's token-by-token logits on the same weights (its decode step
    stores every position's best leaves and borrows from the previous nb_window positions)."""
    Config, engine = R['config'].Config, R['engine']
    cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=32, attn='seg', wmax=4, beam=3,
                 neighbors=True, beam_mode='fixed')
    torch.manual_seed(6)
    m = R['model'].GPT(cfg).eval()
    idx = torch.randint(0, 64, (1, 128), generator=torch.Generator().manual_seed(7))
    with torch.no_grad():
        logits, _, stats = m(idx)
        dec = engine.Decoder(engine.weights_from_ours(m.state_dict(), cfg), cfg.n_layer, cfg.n_head, cfg.n_embd,
                             128, 'seg', cfg, 'cpu')
        steps = [dec.step(int(idx[0, t]), t) for t in range(128)]
    return dict(idx=np_(idx), logits=np_(logits), dec_logits=np.stack([np_(st[0]) for st in steps]),
                dec_keys=np.array([st[1] for st in steps]), **{'stat_' + kk: vv for kk, vv in stats.items()})


def gate_goldens(R):
    """The mean-log gate (seg.py:16-23, fastseg.py:238-251, engine.py:33-37): fastseg.select_seg_fast on gated
    levels (gate_min_level 2, neighbours on), and a tiny GPT with the gate - forward logits and the reference
    engine's token-by-token logits (its SegState keeps the log-magnitude tree and gates gathered nodes)."""
    Config, fastseg, engine = R['config'].Config, R['fastseg'], R['engine']
    g = torch.Generator().manual_seed(21)
    q, k = torch.randn(2, 2, 128, 32, generator=g), torch.randn(2, 2, 128, 32, generator=g)
    cfg = Config(attn='seg', seq_len=128, wmax=8, beam=4, beam_mode='fixed', gate=True, gate_q=0.25,
                 gate_min_level=2)
    lhat = torch.randint(2, 9, (2, 2, 128), generator=g)
    sel = fastseg.select_seg_fast(q, k, lhat, cfg)
    out = dict(sel_gate=dict(q=np_(q), k=np_(k), lhat=np_(lhat), wmax=8, gate_q=0.25, gate_min=2,
                             **{kk: np_(vv) for kk, vv in sel.items()}))
    cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=32, attn='seg', wmax=4, beam=3,
                 neighbors=True, beam_mode='fixed', gate=True, gate_q=0.25, gate_min_level=1)
    torch.manual_seed(8)
    m = R['model'].GPT(cfg).eval()
    idx = torch.randint(0, 64, (1, 128), generator=torch.Generator().manual_seed(9))
    with torch.no_grad():
        logits, _, stats = m(idx)
        dec = engine.Decoder(engine.weights_from_ours(m.state_dict(), cfg), cfg.n_layer, cfg.n_head, cfg.n_embd,
                             128, 'seg', cfg, 'cpu')
        steps = [dec.step(int(idx[0, t]), t) for t in range(128)]
    out['tiny_gpt_gate'] = dict(idx=np_(idx), logits=np_(logits), dec_logits=np.stack([np_(st[0]) for st in steps]),
                                dec_keys=np.array([st[1] for st in steps]),
                                **{'stat_' + kk: vv for kk, vv in stats.items()})
    return out


def dyn_goldens(R):
    """The dynamic content tree (attn='dyn'): a LaneTree the reference builds (2-means splits, dyntree.py:46-80) and
    grows (insertions, dyntree.py:83-106), stored as slots, packed node sums and counts after the build and after
    the insertions; dyntree.select_keys (dyntree.py:150-243) on two configurations (neighbours on, learned-budget
    style random leaf budgets); and tiny GPTs with DynAttention (attn='dyn', fixed and pred budgets): logits and
    statistics."""
    dyn, Config = R['dyntree'], R['config'].Config
    out = {}
    g = torch.Generator().manual_seed(31)
    P, C, dh = 5, 64, 8
    kfull = torch.randn(P, C, dh, generator=g)
    n = torch.tensor([0, 8, 20, 33, 40])
    tree = dyn.LaneTree(kfull, n, iters=3)
    d = dict(kfull=np_(kfull), n=np_(n), slot0=np_(tree.slot.clone()), sums0=np_(torch.cat(tree.sums, 1)),
             cnt0=np_(torch.cat(tree.cnt, 1)))
    ar = torch.arange(P)
    for i in range(16):
        kpos = n + i
        tree.insert(kfull[ar, kpos], kpos, kpos >= 1)
    d.update(slot1=np_(tree.slot), sums1=np_(torch.cat(tree.sums, 1)), cnt1=np_(torch.cat(tree.cnt, 1)))
    out['dyn_tree'] = d
    for name, (B, H, T, hd, kw) in dict(
            dyn_sel_a=(2, 2, 64, 16, dict(chunk=16, wmax=4, nb_window=4, nb_store=2, nb_probe=2, nb_cap_min=1)),
            dyn_sel_b=(1, 3, 128, 32, dict(chunk=32, wmax=8))).items():
        cfg = Config(attn='dyn', seq_len=T, **kw)
        q, k = torch.randn(B, H, T, hd, generator=g), torch.randn(B, H, T, hd, generator=g)
        lhat = torch.randint(2, cfg.wmax + 1, (B, H, T), generator=g)
        sel = dyn.select_keys(q, k, lhat, cfg)
        out[name] = dict(q=np_(q), k=np_(k), lhat=np_(lhat), chunk=cfg.chunk, wmax=cfg.wmax, nb_window=cfg.nb_window,
                         nb_store=cfg.nb_store, nb_rho=cfg.nb_rho, nb_probe=cfg.nb_probe, nb_cap_min=cfg.nb_cap_min,
                         **{kk: np_(vv) for kk, vv in sel.items()})
    for name, kw in dict(tiny_gpt_dyn=dict(beam_mode='fixed'),
                         tiny_gpt_dyn_pred=dict(beam_mode='pred', global_pool=True, local=8)).items():
        cfg = Config(vocab_size=64, seq_len=64, n_layer=2, n_head=2, n_embd=32, attn='dyn', chunk=16, wmax=4, beam=2,
                     beam_classes=(2, 3, 4), nb_window=4, nb_store=2, nb_probe=2, nb_cap_min=1, **kw)
        torch.manual_seed(33)
        m = R['model'].GPT(cfg).eval()
        idx = torch.randint(0, 64, (2, 64), generator=torch.Generator().manual_seed(34))
        with torch.no_grad():
            logits, _, stats = m(idx)
        out[name] = dict(idx=np_(idx), logits=np_(logits), **{'stat_' + kk: vv for kk, vv in stats.items()})
    return out


def forest_goldens(R):
    """The block forest (attn='block'): forest.build_forest (forest.py:47-75) with and without the soft gate,
    TreeAttention.sparse_attend (attention.py:47-143) on random q, k, v at two sizes, and tiny GPTs with
    TreeAttention (fixed budget; learned budget + global pool + gate): logits and statistics."""
    forest, Config = R['forest'], R['config'].Config
    from treeattn.attention import TreeAttention
    out = {}
    g = torch.Generator().manual_seed(41)
    k = torch.randn(2, 2, 128, 16, generator=g)
    cfg = Config(kmeans_iters=3, gate=False)
    perm, sums = forest.build_forest(k, 32, 4, cfg)
    cfg_g = Config(kmeans_iters=3, gate=True, gate_q=0.25, gate_temp=0.3)
    _, sums_g = forest.build_forest(k, 32, 4, cfg_g)
    out['forest_build'] = dict(k=np_(k), perm=np_(perm), **{'S%d' % l: np_(sums[l]) for l in range(5)},
                               **{'G%d' % l: np_(sums_g[l]) for l in range(5)})
    for name, (B, H, T, dh, blk, wmax, beam) in dict(tree_attn_a=(2, 2, 128, 16, 32, 4, 2),
                                                     tree_attn_b=(1, 3, 512, 32, 64, 8, 4)).items():
        cfg = Config(n_embd=H * dh, n_head=H, seq_len=T, tree_block=blk, wmax=wmax, beam=beam)
        m = TreeAttention(cfg).eval()
        q, kk, v = [torch.randn(B, H, T, dh, generator=g) for _ in range(3)]
        with torch.no_grad():
            o = m.sparse_attend(q, kk, v)
        out[name] = dict(q=np_(q), k=np_(kk), v=np_(v), o=np_(o), tree_block=blk, wmax=wmax, beam=beam,
                         **{'stat_' + kk_: float(vv) for kk_, vv in m.aux.items()})
    for name, kw in dict(tiny_gpt_block=dict(), tiny_gpt_block_pred=dict(beam_mode='pred', global_pool=True,
                                                                         gate=True)).items():
        cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=32, tree_block=32, wmax=4, beam=2,
                     beam_classes=(2, 3, 4), **kw)
        torch.manual_seed(43)
        m = R['model'].GPT(cfg).eval()
        idx = torch.randint(0, 64, (2, 128), generator=torch.Generator().manual_seed(44))
        with torch.no_grad():
            logits, _, stats = m(idx)
        out[name] = dict(idx=np_(idx), logits=np_(logits), **{'stat_' + kk: vv for kk, vv in stats.items()})
    return out


def interop_goldens(R):
    """Checkpoint interop (engine.py:123-146, train.py:144): a tiny seg GPT with the learned budget head saved the way
    the reference's training scripts save it (ckpt_tiny_seg.pt), its forward logits and the reference Decoder's
    token-by-token logits; the same weights renamed to a nanoGPT state dict (ckpt_tiny_nanogpt.pt, torch.compile's
    '_orig_mod.' prefix) and the reference's dense-mode Decoder logits over it."""
    Config, engine = R['config'].Config, R['engine']
    cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=32, attn='seg', wmax=4, beam=3,
                 beam_mode='pred', global_pool=True, beam_classes=(2, 3, 4), neighbors=True)
    torch.manual_seed(51)
    m = R['model'].GPT(cfg).eval()
    sd = {kk: vv.clone() for kk, vv in m.state_dict().items()}
    torch.save({'model': sd, 'cfg': cfg.to_dict()}, os.path.join(HERE, 'ckpt_tiny_seg.pt'))
    idx = torch.randint(0, 64, (1, 128), generator=torch.Generator().manual_seed(52))
    with torch.no_grad():
        logits, _, _ = m(idx)
        dec = engine.Decoder(engine.weights_from_ours(sd, cfg), 2, 2, 32, 128, 'seg', cfg, 'cpu')
        seg_steps = np.stack([np_(dec.step(int(idx[0, t]), t)[0]) for t in range(128)])
        names = dict(wte='transformer.wte.weight', wpe='transformer.wpe.weight', ln_f='transformer.ln_f.weight')
        nano = {'_orig_mod.' + names[kk]: sd[kk + '.weight'] for kk in ('wte', 'wpe', 'ln_f')}
        for i in range(2):
            p, o = 'blocks.%d.' % i, '_orig_mod.transformer.h.%d.' % i
            nano.update({o + 'ln_1.weight': sd[p + 'ln1.weight'], o + 'attn.c_attn.weight': sd[p + 'attn.c_attn.weight'],
                         o + 'attn.c_proj.weight': sd[p + 'attn.c_proj.weight'], o + 'ln_2.weight': sd[p + 'ln2.weight'],
                         o + 'mlp.c_fc.weight': sd[p + 'mlp.c_fc.weight'], o + 'mlp.c_proj.weight': sd[p + 'mlp.c_proj.weight']})
        torch.save(nano, os.path.join(HERE, 'ckpt_tiny_nanogpt.pt'))
        dd = engine.Decoder(engine.weights_from_nanogpt(nano, 2), 2, 2, 32, 128, 'dense', None, 'cpu')
        dense_steps = np.stack([np_(dd.step(int(idx[0, t]), t)[0]) for t in range(128)])
    return dict(interop=dict(idx=np_(idx), logits=np_(logits), seg_steps=seg_steps, dense_steps=dense_steps))


def main(ref_path, only=None):
    R = import_reference(ref_path)
    single = dict(lanetree=lanetree_golden, tiny_gpt_nb=tiny_gpt_nb_golden)
    if only in single:  # regenerate this fixture alone (the others are left untouched)
        d = single[only](R)
        np.savez_compressed(os.path.join(HERE, only + '.npz'), **{kk: np.asarray(vv) for kk, vv in d.items()})
        print('wrote', only)
        return
    if only in ('gate', 'dyn', 'forest', 'interop'):
        for name, d in dict(gate=gate_goldens, dyn=dyn_goldens, forest=forest_goldens,
                            interop=interop_goldens)[only](R).items():
            np.savez_compressed(os.path.join(HERE, name + '.npz'), **{kk: np.asarray(vv) for kk, vv in d.items()})
            print('wrote', name)
        return
    Config = R['config'].Config
    seg, fastseg, engine, ad = R['seg'], R['fastseg'], R['engine'], R['attention_dyn']
    out = {}

    # A. level sums (seg.level_sums), sink not zeroed (as test_seg.test_levels_additive calls it)
    g = torch.Generator().manual_seed(100)
    k = torch.randn(1, 2, 64, 16, generator=g)
    S = seg.level_sums(k, 5, False, 0.25)
    out['levels'] = dict(k=np_(k), **{'S%d' % l: np_(S[l]) for l in range(1, 6)})

    # B/C. select_seg at leaf 2 (L0 = 1), neighbours off, fixed budget
    for name, (shape, wmax, beam, seed) in dict(sel_w4=((2, 2, 128, 16), 4, 2, 11),
                                                sel_w8=((2, 2, 256, 64), 8, 8, 12)).items():
        g = torch.Generator().manual_seed(seed)
        q, k = torch.randn(*shape, generator=g), torch.randn(*shape, generator=g)
        cfg = Config(attn='seg', seq_len=shape[2], wmax=wmax, beam=beam, neighbors=False, beam_mode='fixed')
        lhat = torch.full(shape[:3], beam, dtype=torch.long)
        sel = seg.select_seg(q, k, lhat, cfg)
        Lm = int(round(math.log2(shape[2]))) - 1
        kidx = k.float().clone()
        kidx[:, :, 0] = 0
        SS = seg.level_sums(kidx, Lm, False, 0.25)
        ids, vld, sct = seg.tree_pass(q.float(), lambda l, c: R['forest'].gather_nodes(SS[l], c),
                                      torch.arange(shape[2]), Lm, wmax)
        out[name] = dict(q=np_(q), k=np_(k), wmax=wmax, beam=beam, tree_pos=np_(sel['tree_pos']),
                         leaf_ok=np_(sel['leaf_ok']), n_tree=np_(sel['n_tree']), nb_pos=np_(sel['nb_pos']),
                         ids=np_(ids), vld=np_(vld), sct=np_(sct))

    # D. select_seg with neighbour borrowing on (the reference default), for the neighbour-pass row
    g = torch.Generator().manual_seed(7)
    q, k = torch.randn(2, 2, 128, 32, generator=g), torch.randn(2, 2, 128, 32, generator=g)
    cfg = Config(attn='seg', seq_len=128, wmax=8, beam=4, beam_mode='fixed')
    lhat = torch.randint(2, 9, (2, 2, 128), generator=g)
    sel = seg.select_seg(q, k, lhat, cfg)
    out['sel_nb'] = dict(q=np_(q), k=np_(k), lhat=np_(lhat), wmax=8, nb_window=cfg.nb_window,
                         nb_store=cfg.nb_store, nb_rho=cfg.nb_rho, nb_probe=cfg.nb_probe, nb_cap_min=cfg.nb_cap_min,
                         **{kk: np_(vv) for kk, vv in sel.items()})

    # E. tree_pass on leaf blocks of 2^L0 tokens (adapter)
    for name, (shape, L0, wmax) in dict(tp_l3=((2, 2, 256, 32), 3, 4), tp_l5=((1, 2, 512, 64), 5, 4),
                                        tp_l6=((1, 2, 1024, 64), 6, 16)).items():
        g = torch.Generator().manual_seed(L0 * 11)
        q, k = torch.randn(*shape, generator=g), torch.randn(*shape, generator=g)
        ids, vld, sct = adapter_tree_pass(R, q, k, L0, wmax)
        out[name] = dict(q=np_(q), k=np_(k), L0=L0, wmax=wmax, ids=np_(ids), vld=np_(vld),
                         sct_adapter=np_(sct))

    # F. dedupe (attention_dyn.dedupe == fastseg.dedupe_fast)
    g = torch.Generator().manual_seed(0)
    cand = torch.randint(-1, 12, (3, 2, 50, 36), generator=g)
    valid = (torch.rand(3, 2, 50, 36, generator=g) < 0.8) & (cand >= 0)
    keep = ad.dedupe(cand, valid)
    assert (keep == fastseg.dedupe_fast(cand, valid)).all()
    out['dedupe'] = dict(cand=np_(cand), valid=np_(valid), keep=np_(keep))

    # G. sparse_attn_ref and gather_dot on the shapes of the reference's own kernel self-check
    g = torch.Generator().manual_seed(0)
    b, H, T, dh, K_ = 1, 2, 160, 64, 12
    q, k, v = [torch.randn(b, H, T, dh, generator=g) for _ in range(3)]
    cand = torch.randint(-1, T, (b, H, T, K_), generator=g)
    cand[..., 0] = torch.arange(T)
    o = fastseg.sparse_attn_ref(q, k, v, cand, 0.125)
    Sg = torch.randn(b, H, 100, dh, generator=g)
    cd = torch.randint(0, 100, (b, H, T, 9), generator=g)
    d = fastseg.gather_dot(q, Sg, cd, 0.5)
    out['attn'] = dict(q=np_(q), k=np_(k), v=np_(v), cand=np_(cand), o=np_(o), S=np_(Sg), cd=np_(cd), dot=np_(d))

    # H. tiny GPT with SegAttention (forward logits) and the token-by-token engine on the same weights
    tiny = dict(vocab_size=64, seq_len=64, n_layer=2, n_head=2, n_embd=32, attn='seg', wmax=4, beam=2,
                neighbors=False, beam_mode='fixed')
    torch.manual_seed(4)
    cfg = Config(**tiny)
    m = R['model'].GPT(cfg).eval()
    idx = torch.randint(0, 64, (1, 64))
    with torch.no_grad():
        logits, _, stats = m(idx)
        dec = engine.Decoder(engine.weights_from_ours(m.state_dict(), cfg), cfg.n_layer, cfg.n_head, cfg.n_embd, 64,
                             'seg', cfg, 'cpu')
        steps = [dec.step(int(idx[0, t]), t) for t in range(64)]
    out['tiny_gpt'] = dict(idx=np_(idx), logits=np_(logits), dec_logits=np.stack([np_(s[0]) for s in steps]),
                           dec_keys=np.array([s[1] for s in steps]),
                           wsum=np.array([float(p.double().sum()) for p in m.state_dict().values()]),
                           **{'stat_' + kk: vv for kk, vv in stats.items()})

    # I. one decode step of one layer on a filled state (bench_decode.py pattern), leaf 2
    g = torch.Generator().manual_seed(3)
    H, dh, T = 2, 64, 512
    cfg = Config(seq_len=T, n_head=H, n_embd=H * dh, attn='seg', beam=4, beam_mode='fixed', local=3,
                 neighbors=False)
    K, V = torch.randn(1, H, T, dh, generator=g), torch.randn(1, H, T, dh, generator=g)
    qd = torch.randn(1, H, 1, dh, generator=g)
    st = engine.SegState(cfg, T, H, dh, 'cpu')
    st.fill(K, V)
    od, kr = engine.seg_attend(st, None, qd, None, None, T - 1, update=False)
    out['seg_attend'] = dict(K=np_(K), V=np_(V), q=np_(qd), out=np_(od), keys=kr, wmax=cfg.wmax, beam=4, local=3)

    # J. configuration 1: GPT 4 x 256, 4 heads, vocab 4096, T 512, leaf 32, top-4, window 64 (adapter), fp32
    L0 = 5
    c1 = dict(vocab_size=4096, seq_len=512, n_layer=4, n_head=4, n_embd=256, attn='seg', wmax=4, beam=4, local=64,
              neighbors=False, beam_mode='fixed')
    cfg = Config(**c1)

    def select_adapter(q, k, lhat, cfg_):
        ids, vld, sct = adapter_tree_pass(R, q, k, L0, cfg_.wmax)
        sub = 1 << (L0 - 1)
        b_, H_, T_, wl = ids.shape
        ids1 = (ids.unsqueeze(-1) * sub + torch.arange(sub)).reshape(b_, H_, T_, wl * sub)
        vld1 = vld.unsqueeze(-1).expand(b_, H_, T_, wl, sub).reshape(b_, H_, T_, wl * sub)
        nbw = cfg_.nb_window * cfg_.nb_store
        n_tree = torch.full((b_, H_, T_), min(max(cfg_.beam, 2), cfg_.wmax) * sub, dtype=torch.long)
        return dict(tree_pos=seg.leaves_to_pos(ids1, vld1), leaf_ok=vld1,
                    nb_pos=torch.full((b_, H_, T_, 2 * nbw), -1, dtype=torch.long), n_tree=n_tree,
                    nb_leaves=torch.zeros(b_, H_, T_, dtype=torch.long))

    saved = fastseg.select_seg_fast
    fastseg.select_seg_fast = select_adapter
    try:
        torch.manual_seed(0)
        m = R['model'].GPT(cfg).eval()
        g = torch.Generator().manual_seed(1)
        idx = torch.randint(0, 4096, (2, 512), generator=g)
        with torch.no_grad():
            logits, _, stats = m(idx)
    finally:
        fastseg.select_seg_fast = saved
    lf = logits.double()
    out['config1'] = dict(idx=np_(idx), logits_sub=np_(logits[:, ::32, :]), lse=np_(torch.logsumexp(lf, -1)),
                          argmax=np_(logits.argmax(-1)), wsum=np.array([float(p.double().sum())
                                                                         for p in m.state_dict().values()]),
                          L0=L0, **{'stat_' + kk: vv for kk, vv in stats.items()})

    out['lanetree'] = lanetree_golden(R)
    out['tiny_gpt_nb'] = tiny_gpt_nb_golden(R)
    out.update(gate_goldens(R))
    out.update(dyn_goldens(R))
    out.update(forest_goldens(R))
    out.update(interop_goldens(R))

    for name, d in out.items():
        np.savez_compressed(os.path.join(HERE, name + '.npz'), **{kk: np.asarray(vv) for kk, vv in d.items()})
        print('wrote', name, sum(np.asarray(vv).nbytes for vv in d.values()) // 1024, 'KiB')


if __name__ == '__main__':
    args = [x for x in sys.argv[1:] if not x.startswith('--only=')]
    only = next((x.split('=', 1)[1] for x in sys.argv[1:] if x.startswith('--only=')), None)
    ref = args[0] if args else os.environ.get('TREEATTN_REFERENCE')
    if not ref:
        sys.exit('usage: python tests/golden/make_golden.py <path of the treeattn checkout> [--only=name]  '
                 '(or set TREEATTN_REFERENCE)')
    main(ref, only)
