"""numpy (fp32) restatement of treeattn's block-forest attention (attn='block': forest.py, attention.py).

TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline); never imported by the treeattn_b200 package.

Every function cites the reference code it restates. As in the dynamic tree's oracle, decisions that compare two
fp32 values (the 2-means steps, the descent's top-k cuts) can flip under another summation order, so the build and
the descent report MARGINS (smallest relative gaps) per block and per query; parity tests compare what no near-tie
decision can have changed.
"""
import math

import numpy as np

from .dyn_oracle import _rel_gap, masked_two_means_order
from .seg_oracle import F32, bf16_round, gelu, layer_norm, sparse_attn, torch_quantile

__all__ = ['two_means_order', 'soft_gate', 'build_forest', 'forest_descent', 'tree_attention', 'gpt_forward_block']


def two_means_order(X, iters, with_margin=False):
    """forest.py:13-33 two_means_order: every key of every group is valid, so this is masked_two_means_order
    (dyntree.py:6-31) with an all-true mask (the valid mean is X.mean, no key is ever masked)."""
    X = np.asarray(X, F32)
    return masked_two_means_order(X, np.ones(X.shape[:-1], bool), iters, with_margin=with_margin)


def _log_mag(x):
    """log(|x| + 1e-6) of fp32 values: the sum in fp32, the logarithm correctly rounded to fp32."""
    a = (np.abs(np.asarray(x, F32)) + F32(1e-6)).astype(F32)
    return np.log(a.astype(np.float64)).astype(F32)


def soft_gate(sm, grp, gate_q, gate_temp):
    """forest.py:36-44 soft_gate: per node, the mean log-magnitude ml of every dimension over the node's member keys,
    thr = its gate_q quantile over the dimensions (torch.quantile), g = sigmoid((ml - thr) / gate_temp),
    out = sm * g * (d / max(sum g, 1)) (fp32, then sm's precision)."""
    sm = np.asarray(sm, F32)
    S = grp.shape[-2]
    ml = (_log_mag(grp).sum(-2, dtype=F32) / F32(S)).astype(F32)
    thr = torch_quantile(ml, gate_q)
    z = ((ml - thr) / F32(gate_temp)).astype(F32)
    g = (1.0 / (1.0 + np.exp(-z.astype(np.float64)))).astype(F32)
    kept = np.maximum(g.sum(-1, keepdims=True, dtype=F32), F32(1))
    return ((sm * g).astype(F32) * (F32(sm.shape[-1]) / kept).astype(F32)).astype(F32)


def build_forest(k, B, depth, iters, gate=None, bf16=False):
    """forest.py:47-75 build_forest: one content-sorted binary tree per block of B keys. k (b, H, T, d).
    Returns perm_flat (b, H, nb B) (rank -> local position inside the block), sums[l] (b, H, nb 2^l, d) for
    l = 0..depth (level depth = groups of 2 keys; node id = block 2^l + m), and the build margin per block
    (b, H, nb). gate = (gate_q, gate_temp) applies soft_gate; bf16 rounds the sums as a bf16 tensor would."""
    k = np.asarray(k, F32)
    b, H, T, d = k.shape
    nb = T // B
    P = b * H * nb
    kb = k.reshape(P, B, d)
    ar = np.arange(P)[:, None]
    perm = np.broadcast_to(np.arange(B), (P, B)).copy()
    margin = np.full(P, np.inf)
    for lvl in range(depth):
        G = 1 << lvl
        S = B // G
        order, mg = two_means_order(kb[ar, perm].reshape(P, G, S, d), iters, with_margin=True)
        margin = np.minimum(margin, mg.min(-1))
        perm = np.take_along_axis(perm.reshape(P, G, S), order, 2).reshape(P, B)
    kp = kb[ar, perm]
    rnd = bf16_round if bf16 else (lambda a: a)
    sums = []
    for lvl in range(depth + 1):
        nn = 1 << lvl
        grp = kp.reshape(P, nn, B // nn, d)
        sm = rnd(grp.sum(2, dtype=F32))
        if gate is not None:
            sm = rnd(soft_gate(sm, grp, gate[0], gate[1]))
        sums.append(sm.reshape(b, H, nb * nn, d))
    return perm.reshape(b, H, nb * B), sums, margin.reshape(b, H, nb)


def forest_descent(q, sums, B, depth, wmax, bq):
    """attention.py:73-90: score the roots of every earlier block (q . sum, no normalisation), keep the best
    min(wmax, width) (only the first bq of them stay valid), expand to the children, down to level `depth`.
    q (b, H, T, d); sums as build_forest; bq (b, H, T). Returns levels [(sc, cur, cv)] per level, leaf ids and
    validity (b, H, T, wl), and the query margin (b, H, T): the smallest relative gap at a cut between a kept valid
    candidate and the best dropped valid one."""
    q = np.asarray(q, F32)
    b, H, T, d = q.shape
    nb = T // B
    blk = np.arange(T) // B
    cur = np.broadcast_to(np.arange(nb), (b, H, T, nb))
    cv = np.broadcast_to((np.arange(nb)[None, :] < blk[:, None])[None, None], (b, H, T, nb))
    bq = np.asarray(bq, np.int64)
    qn = np.linalg.norm(q.astype(np.float64), axis=-1)
    margin = np.full((b, H, T), np.inf)
    levels = []
    sel = selv = None
    for lvl in range(depth + 1):
        Wc = cur.shape[-1]
        S = np.asarray(sums[lvl], F32)
        U = S[np.arange(b)[:, None, None, None], np.arange(H)[None, :, None, None], cur]
        sc = np.einsum('bhtd,bhtwd->bhtw', q, U).astype(F32)
        sc = np.where(cv, sc, F32(-np.inf))
        w_keep = min(wmax, Wc)
        order = np.argsort(-sc, axis=-1, kind='stable')
        srt = np.take_along_axis(sc, order, -1).astype(np.float64)
        nv = cv.sum(-1)
        if w_keep < Wc:
            nrm = np.linalg.norm(U.astype(np.float64), axis=-1).max(-1) * qn
            gap = _rel_gap(srt[..., w_keep - 1], srt[..., w_keep], nrm)
            margin = np.minimum(margin, np.where(nv > w_keep, gap, np.inf))
        order = order[..., :w_keep]
        sel = np.take_along_axis(cur, order, -1)
        selv = np.take_along_axis(cv, order, -1) & (np.arange(w_keep) < bq[..., None])
        levels.append((sc, cur, cv))
        if lvl < depth:
            cur = np.concatenate([2 * sel, 2 * sel + 1], -1)
            cv = np.concatenate([selv, selv], -1)
    return levels, sel, selv, margin


def _pred_lhat(q, sums0, B, pw, classes, H, global_pool):
    """attention.py:95-108: the learned budget head's leaf budget per query."""
    q = np.asarray(q, F32)
    b, Hh, T, d = q.shape
    nb = T // B
    blk = np.arange(T) // B
    feats = [q, np.log(np.linalg.norm(q, axis=-1, keepdims=True).astype(F32) + F32(1e-6)).astype(F32),
             np.broadcast_to(np.eye(H, dtype=F32)[None, :, None, :], (b, H, T, H))]
    if global_pool:
        cum = np.cumsum(np.asarray(sums0, F32), axis=2, dtype=F32)
        prev = np.concatenate([np.zeros_like(cum[:, :, :1]), cum[:, :, :-1]], 2)
        denom = (np.maximum(np.arange(nb), 1) * B).astype(F32)[None, None, :, None]
        feats.append((prev / denom).astype(F32)[:, :, blk, :])
    x = np.concatenate(feats, -1).astype(F32)
    w0, b0, w2, b2 = [np.asarray(a, F32) for a in pw]
    h = np.maximum((x @ w0.T + b0).astype(F32), F32(0))
    plog = (h @ w2.T + b2).astype(F32)
    return np.asarray(classes, np.int64)[plog.argmax(-1)]


def tree_attention(q, k, v, B, wmax, beam, kmeans_iters=3, gate=None, pred=None, chunk=64):
    """attention.py:47-143 TreeAttention.sparse_attend (inference): exact causal attention inside the query's own
    block, the sink and the two previous tokens when they lie in earlier blocks, and the keys of the leaf groups
    found by the descent over the trees of the earlier blocks (duplicates of the static keys dropped).
    pred = (pw, classes, H, global_pool) for the learned budget. Returns (out, stats, margin) with the margin per
    query (b, H, T) over the build of the blocks it searches and its own descent."""
    q = np.asarray(q, F32)
    k = np.asarray(k, F32)
    b, H, T, dh = q.shape
    nb = T // B
    scale = 1.0 / math.sqrt(dh)
    t = np.arange(T)
    blk = t // B
    own = blk[:, None] * B + np.arange(B)[None, :]
    own = np.where(own <= t[:, None], own, -1)
    if nb == 1:
        cand = np.broadcast_to(own, (b, H, T, B))
        return sparse_attn(q, k, v, cand, scale, chunk=chunk), {}, np.full((b, H, T), np.inf)
    depth = int(round(math.log2(B // 2)))
    k_idx = k.copy()
    k_idx[:, :, 0] = 0
    perm_flat, sums, bmargin = build_forest(k_idx, B, depth, kmeans_iters, gate=gate)
    bq = np.full((b, H, T), wmax if pred is not None else beam, np.int64)
    levels, leaf, leafv, qmargin = forest_descent(q, sums, B, depth, wmax, bq)
    wl = leaf.shape[-1]
    leafv_use = leafv
    if pred is not None:
        bq_pred = _pred_lhat(q, sums[0], B, *pred)
        leafv_use = leafv & (np.arange(wl) < bq_pred[..., None])
    pf = np.concatenate([2 * leaf, 2 * leaf + 1], -1)
    loc = np.take_along_axis(perm_flat, pf.reshape(b, H, -1), 2).reshape(b, H, T, -1)
    tkey = (pf // B) * B + loc
    s_idx = np.stack([np.zeros_like(t), t - 1, t - 2], -1)
    s_valid = (s_idx >= 0) & (s_idx < (blk * B)[:, None])
    dup = ((tkey[..., None] == s_idx[None, None, :, None, :]) & s_valid[None, None, :, None, :]).any(-1)
    tvalid = np.concatenate([leafv_use, leafv_use], -1) & ~dup
    st = np.where(s_valid, s_idx, -1)
    cand = np.concatenate([np.broadcast_to(own, (b, H, T, B)), np.broadcast_to(st, (b, H, T, 3)),
                           np.where(tvalid, tkey, -1)], -1)
    out = sparse_attn(q, k, v, cand, scale, chunk=chunk)
    tcount = tvalid.sum(-1).astype(np.float64)
    stats = dict(keys_tree=float(tcount[:, :, B:].mean()),
                 keys_total=float((t % B + 1).mean() + s_valid.sum(-1).mean() + tcount.mean()))
    # a query depends on the builds of the blocks before its own
    bm = np.minimum.accumulate(bmargin, axis=-1)
    prior = np.concatenate([np.full((b, H, 1), np.inf), bm[..., :-1]], -1)[..., blk]
    return out, stats, np.minimum(qmargin, prior)


def gpt_forward_block(sd, cfg, idx):
    """model.py:75-93 GPT.forward with TreeAttention (attn='block') blocks, fp32 (inference). sd: the model's
    state dict; cfg: a dict with n_layer, n_head, tree_block, wmax, beam, beam_mode, beam_classes, global_pool, gate,
    gate_q, gate_temp, kmeans_iters. Returns (logits, stats)."""
    g = lambda name: np.asarray(sd[name].detach().float().cpu().numpy() if hasattr(sd[name], 'detach') else sd[name],
                                F32)
    idx = np.asarray(idx, np.int64)
    Bt, T = idx.shape
    wte = g('wte.weight')
    C = wte.shape[1]
    H = cfg['n_head']
    dh = C // H
    x = (wte[idx] + g('wpe.weight')[np.arange(T)]).astype(F32)
    acc = {}
    margin = np.inf
    gate = (cfg['gate_q'], cfg['gate_temp']) if cfg['gate'] else None
    for i in range(cfg['n_layer']):
        p = 'blocks.%d.' % i
        h = layer_norm(x, g(p + 'ln1.weight'))
        qkv = (h @ g(p + 'attn.c_attn.weight').T).astype(F32)
        q, k, v = [qkv[..., j * C:(j + 1) * C].reshape(Bt, T, H, dh).transpose(0, 2, 1, 3) for j in range(3)]
        pred = None
        if cfg['beam_mode'] == 'pred':
            pw = [g(p + 'attn.pred.%s' % n) for n in ('0.weight', '0.bias', '2.weight', '2.bias')]
            pred = (pw, cfg['beam_classes'], H, cfg['global_pool'])
        o, st, mg = tree_attention(q, k, v, cfg['tree_block'], cfg['wmax'], cfg['beam'], cfg['kmeans_iters'],
                                   gate=gate, pred=pred)
        margin = min(margin, float(mg.min()))
        for name, val in st.items():
            acc[name] = acc.get(name, 0.0) + val
        x = (x + (o.transpose(0, 2, 1, 3).reshape(Bt, T, C) @ g(p + 'attn.c_proj.weight').T)).astype(F32)
        f = gelu((layer_norm(x, g(p + 'ln2.weight')) @ g(p + 'mlp.c_fc.weight').T).astype(F32))
        x = (x + (f @ g(p + 'mlp.c_proj.weight').T)).astype(F32)
    logits = (layer_norm(x, g('ln_f.weight')) @ wte.T).astype(F32)
    n = cfg['n_layer']
    stats = {name: val / n for name, val in acc.items()}
    stats['margin'] = margin
    return logits, stats
