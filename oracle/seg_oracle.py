"""numpy (fp32) restatement of treeattn's segment-tree sparse-attention path.

TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline); never imported by the treeattn_b200 package.

Every function cites the reference code it restates (paths inside Dex8123/treeattn). Leaf blocks of 2^L0
tokens are handled by running the reference's descent on the level-shifted tree (leaf level L0 instead of 1);
at L0 = 1 this is exactly the reference. Scores are kept on the natural scale q . S_l / 2^l (the reference's
adapter scale differs by the exact power of two 2^(L0-1), which does not change any ordering).
"""
import math

import numpy as np

F32 = np.float32

__all__ = ['level_sums', 'tree_pass', 'lane_search', 'neighbor_pass', 'gate_apply', 'log_sums', 'gated_levels',
           'torch_quantile', 'leaves_to_pos', 'finish', 'n_tree_fixed', 'static_keys', 'dedupe',
           'sparse_attn', 'gather_dot', 'select_seg', 'seg_attention', 'layer_norm', 'gelu', 'gpt_forward',
           'weights_from_state_dict', 'SegStateNP', 'seg_attend', 'DecoderNP', 'bf16_round', 'Lw_of']


def bf16_round(x):
    """Round fp32 values to the nearest bfloat16 (ties to even) and return them as fp32."""
    a = np.ascontiguousarray(x, dtype=F32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(F32).reshape(a.shape)
    return np.where(np.isnan(a), a, out).astype(F32)


def Lw_of(local):
    """Window length of the static keys (fastseg.py:372: Lw = max(cfg.local, 3))."""
    return max(int(local), 3)


# ------------------------------------------------------------------------------------------------ tree
def level_sums(k, L0, Lm, zero_sink=True):
    """seg.py:26-41 level_sums (and engine.py:57-71 SegState.fill): node sums of levels L0..Lm.

    k (..., T, dh) -> {l: (..., T >> l, dh)} fp32, each parent the fp32 sum of its two children in adjacent-pair
    order (seg.py:35); the key at position 0 enters as 0 when zero_sink (seg.py:128-130, engine.py:62)."""
    x = np.array(k, dtype=F32, copy=True)
    if zero_sink and x.shape[-2] > 0:
        x[..., 0, :] = 0
    out = {}
    for l in range(1, Lm + 1):
        n = x.shape[-2] // 2
        x = x[..., 0:2 * n:2, :] + x[..., 1:2 * n:2, :]
        if l >= L0:
            out[l] = x
    return out


def torch_quantile(x, q):
    """torch.quantile(x, q, dim=-1, keepdim=True) for fp32 x (linear interpolation): ranks = q (n - 1) in fp32, the
    values a, b at floor and ceil of the rank, weight w = rank - floor, then torch's two-sided lerp with one
    rounding: w < 0.5 -> a + w (b - a), else b - (1 - w)(b - a) (a fused multiply-add on b - a; evaluated here in
    float64, where the product is exact)."""
    x = np.asarray(x, F32)
    n = x.shape[-1]
    v = np.sort(x, -1)
    rank = F32(q) * F32(n - 1)
    lo = int(np.floor(rank))
    hi = int(np.ceil(rank))
    w = F32(rank - F32(lo))
    a, b = v[..., lo:lo + 1], v[..., hi:hi + 1]
    d = (b - a).astype(np.float64)
    if w < 0.5:
        return (a.astype(np.float64) + np.float64(w) * d).astype(F32)
    return (b.astype(np.float64) - np.float64(F32(1) - w) * d).astype(F32)


def gate_apply(raw, lgsum, size, gate_q):
    """seg.py:16-23 mean-log dilution gate: keep the dimensions whose mean log-magnitude in the group is at least
    the gate_q quantile, zero the rest, rescale the kept ones by dh / kept."""
    raw = np.asarray(raw, F32)
    ml = (np.asarray(lgsum, F32) / F32(size)).astype(F32)
    thr = torch_quantile(ml, gate_q)
    g = (ml >= thr).astype(F32)
    kept = np.maximum(g.sum(-1, keepdims=True), F32(1)).astype(F32)
    return ((raw * g).astype(F32) * (F32(raw.shape[-1]) / kept).astype(F32)).astype(F32)


def log_sums(k, L0, Lm, zero_sink=True):
    """The mean-log statistic's tree (seg.py:31-37, fastseg.py:238-251): log(|k| + 1e-6) of the (sink-zeroed)
    keys summed in the same adjacent-pair order as level_sums."""
    x = np.array(k, dtype=F32, copy=True)
    if zero_sink and x.shape[-2] > 0:
        x[..., 0, :] = 0
    return level_sums(np.log(np.abs(x) + F32(1e-6)).astype(F32), L0, Lm, zero_sink=False)


def gated_levels(k, L0, Lm, gate_q, gate_min=0):
    """fastseg.py:238-251 level_sums_min with the gate: levels l >= gate_min gated, the others raw."""
    S = level_sums(k, L0, Lm, zero_sink=True)
    G = log_sums(k, L0, Lm)
    return {l: (gate_apply(S[l], G[l], 1 << l, gate_q) if l >= gate_min else S[l]) for l in S}


def _gather_rows(S, idx):
    """S (B, H, M, d), idx (B, H, N, C) -> (B, H, N, C, d) (forest.py:4-9 gather_nodes)."""
    B, H = S.shape[:2]
    bi = np.arange(B).reshape(B, 1, 1, 1)
    hi = np.arange(H).reshape(1, H, 1, 1)
    return S[bi, hi, idx]


def tree_pass(q, levels, tq, L0, Lm, wmax, with_margin=False):
    """seg.py:44-70 tree_pass on the tree whose leaves are the level-L0 nodes.

    q (B, H, Nq, dh); levels {l: (B, H, n_l, dh)} for L0 <= l <= Lm; tq (Nq,) or (B, Nq) positions.
    Per level from Lm down to L0 the candidates are [2*ids, 2*ids+1, injected (t>>l)-1] with validity
    [vld, vld, bit l of t] (seg.py:55-62); scores q . S_l[c] / 2^l, invalid -> -inf (seg.py:64-65); the best
    min(wmax, C) are kept, best first (seg.py:66-69; ties by position in the list).
    Returns ids, vld, sct (B, H, Nq, wl) and, with with_margin, the smallest gap between the last kept and the
    best dropped VALID candidate over all levels, relative to ||q|| * ||S_c|| / 2^l (inf if nothing valid was
    ever dropped): below ~1e-6 the order is within fp32 rounding, i.e. a tie."""
    q = np.asarray(q, F32)
    B, H, Nq, dh = q.shape
    tq = np.asarray(tq, np.int64)
    if tq.ndim == 1:
        tq = np.broadcast_to(tq[None], (B, Nq))
    tqb = np.broadcast_to(tq[:, None, :], (B, H, Nq))
    ids = vld = sct = None
    margin = np.full((B, H, Nq), np.inf)
    qn = np.linalg.norm(q.astype(np.float64), axis=-1)
    for l in range(Lm, L0 - 1, -1):
        bit = ((tqb >> l) & 1) == 1
        inj = np.maximum((tqb >> l) - 1, 0)
        if ids is None:
            cand, cv = inj[..., None].copy(), bit[..., None].copy()
        else:
            cand = np.concatenate([2 * ids, 2 * ids + 1, inj[..., None]], -1)
            cv = np.concatenate([vld, vld, bit[..., None]], -1)
        S = levels[l]
        n_l = S.shape[-2]
        U = _gather_rows(S, np.clip(cand, 0, max(n_l - 1, 0))) if n_l > 0 else np.zeros(cand.shape + (dh,), F32)
        sc = np.einsum('bhnd,bhncd->bhnc', q, U).astype(F32) * F32(2.0 ** -l)
        sc = np.where(cv, sc, F32(-np.inf)).astype(F32)
        w = min(wmax, cand.shape[-1])
        order = np.argsort(-sc, axis=-1, kind='stable')
        if with_margin:
            # gap between the last kept and the best dropped valid candidate, normalised by the bound
            # ||q|| * ||S_c|| / 2^l on the score magnitude (the scale of any fp32 reduction error)
            srt = np.take_along_axis(sc, order, -1)
            nrm = np.take_along_axis(np.linalg.norm(U, axis=-1), order, -1) * qn[..., None] * 2.0 ** -l
            nv = cv.sum(-1)
            cut = nv > w
            if cut.any() and w < sc.shape[-1]:
                with np.errstate(invalid='ignore', divide='ignore'):
                    a = srt[..., w - 1].astype(np.float64)
                    b_ = srt[..., w].astype(np.float64)
                    den = np.maximum(np.maximum(nrm[..., w - 1], nrm[..., w]), 1e-30)
                    gap = np.where(cut, (a - b_) / den, np.inf)
                margin = np.minimum(margin, gap)
        order = order[..., :w]
        ids = np.take_along_axis(cand, order, -1)
        vld = np.take_along_axis(cv, order, -1)
        sct = np.take_along_axis(sc, order, -1)
    if with_margin:
        return ids, vld, sct, margin
    return ids, vld, sct


def leaves_to_pos(ids, ok, leaf=2):
    """seg.py:106-108 leaves_to_pos for leaf blocks of `leaf` positions: slot j*wl + i holds ids[i]*leaf + j."""
    ids = np.asarray(ids, np.int64)
    pos = np.concatenate([ids * leaf + j for j in range(leaf)], -1)
    okr = np.concatenate([np.asarray(ok, bool)] * leaf, -1)
    return np.where(okr, pos, -1)


def finish(ids, vld, nid, match, nL, lhat, wmax, leaf=2):
    """seg.py:111-119 finish: leaf budget -> n_tree, and leaf ids -> positions."""
    L = np.asarray(lhat, np.int64)
    nL = np.asarray(nL, np.int64)
    lo = (L + 1) // 2
    need = np.maximum(L - nL, 0)
    floor_b = np.where(nL < lo, 2, 1)
    b_tree = np.minimum(np.where(nL >= L, 0, np.maximum(need, floor_b)), wmax)
    return dict(tree_pos=leaves_to_pos(ids, vld, leaf), leaf_ok=np.asarray(vld, bool),
                nb_pos=leaves_to_pos(nid, match, leaf), n_tree=b_tree, nb_leaves=nL)


def n_tree_fixed(beam, wmax):
    """finish() with no neighbour matches (nL = 0) and a fixed budget: min(max(beam, 2), wmax), 0 for beam 0."""
    if beam <= 0:
        return 0
    return min(max(beam, 2), wmax)


def static_keys(tq, Lw):
    """fastseg.py:372-375 / engine.py:109-110: [0, t, t-1, ..., t-Lw+1], negatives -> -1."""
    tq = np.asarray(tq, np.int64)
    st = np.concatenate([np.zeros(tq.shape + (1,), np.int64), tq[..., None] - np.arange(Lw)], -1)
    return np.where(st < 0, -1, st)


def dedupe(cand, valid):
    """attention_dyn.py:12-17 dedupe / fastseg.py:227-234 dedupe_fast: keep the first valid copy of each value."""
    cand = np.asarray(cand, np.int64)
    valid = np.asarray(valid, bool)
    key = np.where(valid, cand, np.iinfo(np.int64).min)
    order = np.argsort(key, axis=-1, kind='stable')
    sk = np.take_along_axis(key, order, -1)
    dup_sorted = np.zeros_like(valid)
    dup_sorted[..., 1:] = (sk[..., 1:] == sk[..., :-1]) & (sk[..., 1:] != np.iinfo(np.int64).min)
    dup = np.zeros_like(valid)
    np.put_along_axis(dup, order, dup_sorted, -1)
    return valid & ~dup


def sparse_attn(q, k, v, cand, scale, chunk=64):
    """fastseg.py:134-141 sparse_attn_ref: exact softmax attention over cand (-1 = unused), fp32."""
    q = np.asarray(q, F32)
    k = np.asarray(k, F32)
    v = np.asarray(v, F32)
    cand = np.asarray(cand, np.int64)
    B, H, T, dh = q.shape
    out = np.zeros((B, H, T, dh), F32)
    for s in range(0, T, chunk):
        c = cand[:, :, s:s + chunk]
        keep = c >= 0
        kg = _gather_rows(k, np.maximum(c, 0))
        vg = _gather_rows(v, np.maximum(c, 0))
        S = np.einsum('bhtd,bhtkd->bhtk', q[:, :, s:s + chunk], kg).astype(F32) * F32(scale)
        S = np.where(keep, S, F32(-np.inf))
        m = S.max(-1, keepdims=True)
        m = np.where(np.isfinite(m), m, 0)
        e = np.exp(S - m).astype(F32)
        w = e / e.sum(-1, keepdims=True)
        out[:, :, s:s + chunk] = np.einsum('bhtk,bhtkd->bhtd', w.astype(F32), vg)
    return out


def gather_dot(q, S, cand, scale):
    """fastseg.py:118-122 gather_dot (fallback form): scale * q . S[cand], ids clamped to [0, M-1]."""
    S = np.asarray(S, F32)
    U = _gather_rows(S, np.clip(np.asarray(cand, np.int64), 0, S.shape[2] - 1))
    return (np.einsum('bhnd,bhncd->bhnc', np.asarray(q, F32), U) * F32(scale)).astype(F32)


# ------------------------------------------------------------------------------------------------ selection
def neighbor_pass(q, S_leaf, st_leaf, st_score, st_ok, tq, L0, nb_window, nb_store, nb_rho, nb_probe, nb_cap_min,
                  neighbors=True, with_margin=False):
    """seg.py:73-103 neighbor_pass: every query looks at the nb_store best leaves stored by each of the
    nb_window previous positions (st_* (B, H, T_st, NS) indexed by position), scores them itself
    (q . S_L0[leaf] / 2^L0) and matches those it scores at least base - rho |base| (base = the stored score); the
    scan depth is capped by the match rate over the first nb_probe positions: cap = cap_min + round((Wn - cap_min)
    * rate) (round half to even). Returns ids (B, H, Nq, Wn*NS), match, nL = distinct matched leaves (and, with
    with_margin, the smallest |score - threshold| relative to |q| |S| / 2^L0: near 0 the match is an fp32 tie)."""
    q = np.asarray(q, F32)
    B, H, Nq, dh = q.shape
    Wn, NS = nb_window, nb_store
    tq = np.asarray(tq, np.int64)
    jpos = tq[:, None] - np.arange(1, Wn + 1)[None, :]
    jval = jpos >= 0
    jc = np.maximum(jpos, 0)
    ids = np.asarray(st_leaf)[:, :, jc].reshape(B, H, Nq, Wn * NS)
    base = np.asarray(st_score, F32)[:, :, jc].reshape(B, H, Nq, Wn * NS)
    ok0 = (np.asarray(st_ok, bool)[:, :, jc] & jval[None, None, :, :, None]).reshape(B, H, Nq, Wn * NS)
    U = _gather_rows(np.asarray(S_leaf, F32), np.clip(ids, 0, S_leaf.shape[2] - 1))
    sc_t = (np.einsum('bhnd,bhncd->bhnc', q, U).astype(F32) * F32(2.0 ** -L0)).astype(F32)
    thr = (base - (F32(nb_rho) * np.abs(base)).astype(F32)).astype(F32)
    match = ok0 & (sc_t >= thr)
    probe = nb_probe * NS
    rate = (match[..., :probe].sum(-1).astype(F32) / np.maximum(ok0[..., :probe].sum(-1), 1).astype(F32)).astype(F32)
    cap = nb_cap_min + np.rint(F32(Wn - nb_cap_min) * rate).astype(np.int64)
    didx = np.arange(Wn * NS) // NS + 1
    match = match & (didx <= cap[..., None])
    if not neighbors:
        match = np.zeros_like(match)
    idm = np.where(match, ids, -1)
    ss = np.sort(idm, -1)
    vs = ss >= 0
    nL = vs.sum(-1) - ((ss[..., 1:] == ss[..., :-1]) & vs[..., 1:]).sum(-1)
    if with_margin:
        nrm = np.linalg.norm(U.astype(np.float64), axis=-1) * np.linalg.norm(q.astype(np.float64), axis=-1)[..., None]
        gap = np.where(ok0, np.abs(sc_t.astype(np.float64) - thr) / np.maximum(nrm * 2.0 ** -L0, 1e-30), np.inf)
        return ids, match, nL, gap.min(-1)
    return ids, match, nL


def select_seg(q, k, lhat, wmax, L0=1, nb_width=0, with_margin=False, nb=None, gate=None):
    """seg.py:122-140 select_seg: fp32 copies, sink zeroed, levels, descent, neighbour pass, finish. nb = None
    stands for cfg.neighbors=False (neighbor_pass returns no matches, seg.py:97-98; nb_width slots of empty
    matches); otherwise nb = dict(nb_window, nb_store, nb_rho, nb_probe, nb_cap_min) runs the neighbour pass on
    the descent's own results (the nb_store best leaves and scores of every position). gate = (gate_q,
    gate_min_level) selects on the mean-log gated levels (fastseg.select_seg_fast)."""
    q = np.asarray(q, F32)
    B, H, T, dh = q.shape
    Lm = int(round(math.log2(T))) - 1
    if gate is None:
        S = level_sums(k, L0, Lm, zero_sink=True)
    else:  # gate = (gate_q, gate_min): fastseg.select_seg_fast's gated levels
        S = gated_levels(k, L0, Lm, gate[0], gate[1])
    tq = np.arange(T)
    r = tree_pass(q, S, tq, L0, Lm, wmax, with_margin=with_margin)
    ids, vld, sct = r[:3]
    nb_margin = None
    if nb is None:
        nid = np.zeros((B, H, T, nb_width), np.int64)
        match = np.zeros((B, H, T, nb_width), bool)
        nL = np.zeros((B, H, T), np.int64)
    else:
        NS = nb['nb_store']
        nid, match, nL, nb_margin = neighbor_pass(q, S[L0], ids[..., :NS], sct[..., :NS], vld[..., :NS], tq, L0,
                                                  nb['nb_window'], NS, nb['nb_rho'], nb['nb_probe'],
                                                  nb['nb_cap_min'], with_margin=True)
    sel = finish(ids, vld, nid, match, nL, lhat, wmax, leaf=1 << L0)
    if nb_margin is not None:
        sel['nb_margin'] = nb_margin
    sel['ids'], sel['sct'] = ids, sct
    if with_margin:
        sel['margin'] = r[3]
    return sel


def seg_attention(q, k, v, wmax, beam, local, L0=1, chunk=64):
    """fastseg.py:345-389 SegAttention.sparse_attend (fixed budget, no neighbours): selection, static keys,
    dedupe, exact attention. Returns (out, stats) with the aux statistics of fastseg.py:385-389."""
    q = np.asarray(q, F32)
    B, H, T, dh = q.shape
    scale = 1.0 / math.sqrt(dh)
    lhat = np.full((B, H, T), beam, np.int64)
    sel = select_seg(q, k, lhat, wmax, L0=L0)
    leaf = 1 << L0
    wl = sel['leaf_ok'].shape[-1]
    Lw = Lw_of(local)
    st = np.broadcast_to(static_keys(np.arange(T), Lw), (B, H, T, 1 + Lw))
    used = sel['leaf_ok'] & (np.arange(wl) < sel['n_tree'][..., None])
    tv = np.concatenate([used] * leaf, -1) & (sel['tree_pos'] >= 0)
    cand = np.concatenate([sel['tree_pos'], st], -1)
    keep = dedupe(cand, np.concatenate([tv, st >= 0], -1))
    out = sparse_attn(q, k, v, np.where(keep, cand, -1), scale, chunk=chunk)
    stats = dict(keys_total=float(keep.sum(-1).mean()), keys_tree=float(keep[..., :leaf * wl].sum(-1).mean()),
                 keys_nb=0.0, nb_leaves=0.0, leaves_used=float(used.sum(-1).mean()))
    return out, stats


# ------------------------------------------------------------------------------------------------ dynamic tree
def lane_search(q, sums, cnt, D, wmax, with_margin=False):
    """dyntree.py:108-127 LaneTree.search: beam descent from the root (level 0) to level D over a tree whose
    nodes hold key SUMS and counts, packed level by level (level l at rows 2^l - 1 .. 2^(l+1) - 2). A node is
    valid when its parent is and its count is positive; its score is q . sum / count. At each level the children
    [2*cur, 2*cur + 1] of the kept nodes are ranked and the best min(wmax, 2 * width) are kept, best first.
    q (P, dh); sums (P, 2^(D+1) - 1, dh); cnt (P, 2^(D+1) - 1). Returns ids, vld, sct (P, wl) (+ the tie margin:
    smallest gap between the last kept and the best dropped valid candidate, relative to |q| |mean|)."""
    q = np.asarray(q, F32)
    sums = np.asarray(sums, F32)
    cnt = np.asarray(cnt, np.int64)
    P, dh = q.shape
    cur = np.zeros((P, 1), np.int64)
    cvld = cnt[:, :1] > 0
    sct = None
    margin = np.full(P, np.inf)
    qn = np.linalg.norm(q.astype(np.float64), axis=-1)
    for l in range(1, D + 1):
        off = (1 << l) - 1
        ch = np.concatenate([2 * cur, 2 * cur + 1], -1)
        cv = np.concatenate([cvld, cvld], -1)
        cc = np.take_along_axis(cnt[:, off:off + (1 << l)], ch, 1)
        cv = cv & (cc > 0)
        sm = sums[np.arange(P)[:, None], off + ch]
        sc = (np.einsum('pd,pcd->pc', q, sm).astype(F32) / np.maximum(cc, 1).astype(F32)).astype(F32)
        sc = np.where(cv, sc, F32(-np.inf))
        w = min(wmax, ch.shape[-1])
        order = np.argsort(-sc, axis=-1, kind='stable')
        if with_margin:
            srt = np.take_along_axis(sc, order, -1).astype(np.float64)
            nrm = np.linalg.norm(sm.astype(np.float64), axis=-1) / np.maximum(cc, 1)
            nrm = np.take_along_axis(nrm, order, -1) * qn[:, None]
            cut = cv.sum(-1) > w
            if w < sc.shape[-1]:
                with np.errstate(invalid='ignore', divide='ignore'):
                    gap = (srt[:, w - 1] - srt[:, w]) / np.maximum(np.maximum(nrm[:, w - 1], nrm[:, w]), 1e-30)
                margin = np.minimum(margin, np.where(cut, gap, np.inf))
        order = order[:, :w]
        cur = np.take_along_axis(ch, order, -1)
        cvld = np.take_along_axis(cv, order, -1)
        sct = np.take_along_axis(sc, order, -1)
    if with_margin:
        return cur, cvld, sct, margin
    return cur, cvld, sct


# ------------------------------------------------------------------------------------------------ model
def layer_norm(x, w, eps=1e-5):
    """model.py:12-18 LayerNorm (no bias)."""
    x = np.asarray(x, F32)
    mu = x.mean(-1, keepdims=True, dtype=np.float64).astype(F32)
    d = x - mu
    var = (d * d).mean(-1, keepdims=True, dtype=np.float64).astype(F32)
    return (d / np.sqrt(var + F32(eps)) * np.asarray(w, F32)).astype(F32)


def gelu(x):
    """Exact (erf) GELU, F.gelu's default (model.py:31)."""
    from scipy.special import erf
    x = np.asarray(x, F32)
    return (F32(0.5) * x * (F32(1.0) + erf(x / F32(math.sqrt(2.0))).astype(F32))).astype(F32)


def weights_from_state_dict(sd, n_layer):
    """engine.py:123-134 weights_from_ours, as numpy fp32 arrays."""
    g = lambda name: np.asarray(sd[name].detach().float().cpu().numpy() if hasattr(sd[name], 'detach') else sd[name],
                                F32)
    W = dict(wte=g('wte.weight'), wpe=g('wpe.weight'), ln_f=g('ln_f.weight'), layers=[])
    for i in range(n_layer):
        p = 'blocks.%d.' % i
        W['layers'].append(dict(ln1=g(p + 'ln1.weight'), c_attn=g(p + 'attn.c_attn.weight'),
                                c_proj=g(p + 'attn.c_proj.weight'), ln2=g(p + 'ln2.weight'),
                                c_fc=g(p + 'mlp.c_fc.weight'), c_mlp=g(p + 'mlp.c_proj.weight')))
    return W


def gpt_forward(W, idx, n_head, wmax, beam, local, L0=1, chunk=64, bf16=False):
    """model.py:75-93 GPT.forward with SegAttention blocks (model.py:34-44, fastseg.py:338-343), fp32.

    bf16=True mirrors a bf16 nn.Module forward: every stored activation (embedding sum, residual stream, layer-norm
    and matmul outputs, attention output, GELU output, logits) is rounded to bfloat16; arithmetic stays fp32.
    Returns (logits (B, T, V), per-layer-averaged stats)."""
    r = bf16_round if bf16 else (lambda a: a)
    idx = np.asarray(idx, np.int64)
    B, T = idx.shape
    C = W['wte'].shape[1]
    dh = C // n_head
    x = r((W['wte'][idx] + W['wpe'][np.arange(T)]).astype(F32))
    acc = {}
    for L in W['layers']:
        h = r(layer_norm(x, L['ln1']))
        qkv = r((h @ L['c_attn'].T).astype(F32))
        q, k, v = [qkv[..., i * C:(i + 1) * C].reshape(B, T, n_head, dh).transpose(0, 2, 1, 3) for i in range(3)]
        o, st = seg_attention(q, k, v, wmax, beam, local, L0=L0, chunk=chunk)
        o = r(o)
        for name, val in st.items():
            acc[name] = acc.get(name, 0.0) + val
        x = r(x + r((o.transpose(0, 2, 1, 3).reshape(B, T, C) @ L['c_proj'].T).astype(F32)))
        f = r(gelu(r(r(layer_norm(x, L['ln2'])) @ L['c_fc'].T)))
        x = r(x + r((f @ L['c_mlp'].T).astype(F32)))
    logits = r((r(layer_norm(x, W['ln_f'])) @ W['wte'].T).astype(F32))
    n = len(W['layers'])
    return logits, {name: val / n for name, val in acc.items()}


# ------------------------------------------------------------------------------------------------ decode engine
class SegStateNP:
    """engine.py:18-71 SegState for one sequence (all heads): key/value cache and the tree levels >= L0.

    `kv_round` (e.g. bf16_round) is applied to keys/values entering the cache, to mirror a low-precision cache."""

    def __init__(self, H, dh, cap, L0, Lm, kv_round=None):
        self.H, self.dh, self.cap, self.L0, self.Lm = H, dh, cap, L0, Lm
        self.K = np.zeros((H, cap, dh), F32)
        self.V = np.zeros((H, cap, dh), F32)
        self.levels = {l: np.zeros((1, H, cap >> l, dh), F32) for l in range(L0, Lm + 1)}
        self.kv_round = kv_round

    def add(self, t, k, v):
        """engine.py:41-55: write k, v (H, dh) at t; form every node completed by t (leaf block first)."""
        if self.kv_round is not None:
            k, v = self.kv_round(k), self.kv_round(v)
        self.K[:, t], self.V[:, t] = k, v
        leaf = 1 << self.L0
        if (t + 1) % leaf != 0:
            return
        n = t >> self.L0
        blk = self.K[None, :, n * leaf:(n + 1) * leaf]
        node = level_sums(blk, self.L0, self.L0, zero_sink=(n == 0))[self.L0]
        self.levels[self.L0][:, :, n] = node[:, :, 0]
        for l in range(self.L0 + 1, self.Lm + 1):
            if (t + 1) % (1 << l) != 0:
                break
            m = t >> l
            lv = self.levels[l - 1]
            self.levels[l][:, :, m] = lv[:, :, 2 * m] + lv[:, :, 2 * m + 1]

    def fill(self, K, V):
        """engine.py:57-71 fill: load positions [0, T) at once and build the levels."""
        T = K.shape[1]
        if self.kv_round is not None:
            K, V = self.kv_round(K), self.kv_round(V)
        self.K[:, :T], self.V[:, :T] = K, V
        lv = level_sums(self.K[None, :, :T], self.L0, self.Lm, zero_sink=True)
        for l, a in lv.items():
            self.levels[l][:, :, :a.shape[2]] = a


def seg_attend(state, q, k, v, t, wmax, beam, local, update=True, with_sel=False):
    """engine.py:84-120 seg_attend (fixed budget, no neighbours) for one sequence: q, k, v (H, dh).
    Returns (out (H, dh), keys read per head) and, with with_sel, (leaf ids (H, wl), used (H, wl), margin (H,))."""
    H, dh = state.H, state.dh
    qf = np.asarray(q, F32)[None, :, None, :]
    ids, vld, sct, margin = tree_pass(qf, state.levels, np.array([t]), state.L0, state.Lm, wmax, with_margin=True)
    ntree = n_tree_fixed(beam, wmax)
    if update:
        state.add(t, np.asarray(k, F32), np.asarray(v, F32))
    leaf = 1 << state.L0
    wl = ids.shape[-1]
    Lw = Lw_of(local)
    used = vld[0, :, 0] & (np.arange(wl) < ntree)                       # (H, wl)
    tree_pos = leaves_to_pos(ids[0, :, 0], vld[0, :, 0], leaf)          # (H, leaf*wl)
    tv = np.concatenate([used] * leaf, -1) & (tree_pos >= 0)
    st = np.broadcast_to(static_keys(np.array(t), Lw), (H, 1 + Lw))
    cand = np.concatenate([tree_pos, st], -1)
    keep = dedupe(cand, np.concatenate([tv, st >= 0], -1))
    out = np.zeros((H, dh), F32)
    scale = F32(1.0 / math.sqrt(dh))
    for h in range(H):
        pos = cand[h][keep[h]]
        s = (state.K[h, pos] @ qf[0, h, 0]).astype(F32) * scale
        e = np.exp(s - s.max()).astype(F32)
        out[h] = (e / e.sum()) @ state.V[h, pos]
    res = (out, float(keep.sum(-1).mean()))
    if with_sel:
        return res + ((ids[0, :, 0], used, margin[0, :, 0]),)
    return res


class DecoderNP:
    """engine.py:149-177 Decoder ('seg' mode) for a batch of sequences, fp32, token by token.

    bf16=True mirrors a decoder with bf16 weights and cache and an fp32 residual stream: layer-norm outputs,
    matmul outputs, the attention output, the GELU output and the logits are rounded to bfloat16 (and so are the
    keys/values entering the cache)."""

    def __init__(self, W, n_head, Tcap, wmax, beam, local, L0=1, cap=None, kv_round=None, bf16=False):
        self.W, self.H = W, n_head
        self.C = W['wte'].shape[1]
        self.dh = self.C // n_head
        self.Lm = int(round(math.log2(Tcap))) - 1
        self.L0, self.wmax, self.beam, self.local = L0, wmax, beam, local
        self.cap = cap or Tcap
        self.kv_round = kv_round
        self.r = bf16_round if bf16 else (lambda a: a)
        self.states = None

    def reset(self, batch):
        self.states = [[SegStateNP(self.H, self.dh, self.cap, self.L0, self.Lm, self.kv_round)
                        for _ in self.W['layers']] for _ in range(batch)]

    def step(self, toks, t):
        """toks (B,) token ids at position t (an int or (B,) array). Returns (logits (B, V), keys read); the final
        hidden state (the layer-normed, rounded rows the lm_head multiplies) stays in self.last_h."""
        W, H, C, dh, r = self.W, self.H, self.C, self.dh, self.r
        toks = np.asarray(toks, np.int64)
        B = toks.shape[0]
        tt = np.broadcast_to(np.asarray(t, np.int64), (B,))
        x = (W['wte'][toks] + W['wpe'][tt]).astype(F32)
        keys = 0.0
        for i, L in enumerate(W['layers']):
            qkv = r((r(layer_norm(x, L['ln1'])) @ L['c_attn'].T).astype(F32))
            o = np.zeros((B, C), F32)
            for b in range(B):
                q, k, v = [qkv[b, j * C:(j + 1) * C].reshape(H, dh) for j in range(3)]
                ob, kr = seg_attend(self.states[b][i], q, k, v, int(tt[b]), self.wmax, self.beam, self.local)
                o[b] = ob.reshape(C)
                keys += kr / B
            x = (x + r((r(o) @ L['c_proj'].T).astype(F32))).astype(F32)
            f = r(gelu(r((r(layer_norm(x, L['ln2'])) @ L['c_fc'].T).astype(F32))))
            x = (x + r((f @ L['c_mlp'].T).astype(F32))).astype(F32)
        self.last_h = r(layer_norm(x, W['ln_f']))
        return r((self.last_h @ W['wte'].T).astype(F32)), keys / len(W['layers'])
