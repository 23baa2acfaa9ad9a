"""numpy (fp32) restatement of treeattn's dynamic content tree (attn='dyn': dyntree.py, attention_dyn.py).

TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline); never imported by the treeattn_b200 package.

The 2-means splits, insertion and lane-by-lane selection are restated step by step from the reference (cited per
function). Decisions that compare two fp32 values (argmax / argmin, the side of the median split, the child an
insertion takes, the top-k cut, the neighbour threshold) can flip under a different fp32 summation order, so every
function can also return a per-lane MARGIN: the smallest relative gap of any decision it took. Parity tests compare
lanes whose margin is clear of fp32 noise exactly and count the rest as ties.

The node sums of a built tree are formed bottom-up in adjacent pairs (level D from the two slots of each group,
every upper node from its two children); the reference sums each node's keys in one torch reduction, which
agrees to fp32 rounding.
"""
import math

import numpy as np

from .seg_oracle import F32, dedupe, lane_search, sparse_attn

__all__ = ['masked_two_means_order', 'LaneTreeNP', 'canonical_tree', 'select_keys', 'select_loop', 'dyn_attention',
           'prefix_mean', 'budget_head', 'gpt_forward_dyn']

INF = np.float32(np.inf)


def _rel_gap(a, b, scale):
    with np.errstate(invalid='ignore', divide='ignore'):
        return np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)) / np.maximum(scale, 1e-30)


def _argmax_margin(d2, valid, scale):
    """Relative gap between the largest and second-largest valid value of d2 (P, G, S); inf with < 2 valid."""
    v = np.where(valid, d2.astype(np.float64), -np.inf)
    top2 = -np.sort(-v, axis=-1)[..., :2] if v.shape[-1] >= 2 else np.concatenate([v, -np.inf * v], -1)
    gap = _rel_gap(top2[..., 0], top2[..., 1], scale)
    return np.where(np.isfinite(top2[..., 1]), gap, np.inf)


def masked_two_means_order(X, valid, iters, with_margin=False):
    """dyntree.py:6-31 masked_two_means_order. X (P, G, S, D) fp32, valid (P, G, S) bool -> order (P, G, S): the
    valid keys first, ascending by their projection on the difference of two 2-means centres (ties by index),
    empty slots last.

    Centres start at the valid key farthest from the valid mean (a) and the valid key farthest from a (b) (first
    index on ties, torch.argmax); each of `iters` rounds labels every key by the nearer centre
    (|x|^2 - 2 x.c + |c|^2, first centre on ties) and moves a centre to the mean of its valid members (kept when it
    has none). With with_margin also returns the smallest relative decision gap per (P, G)."""
    X = np.asarray(X, F32)
    valid = np.asarray(valid, bool)
    P, G, S, D = X.shape
    vm = valid[..., None].astype(F32)
    cnt = np.maximum(vm.sum(2, keepdims=True), F32(1))
    mean = ((X * vm).sum(2, keepdims=True) / cnt).astype(F32)
    xnorm2 = (X.astype(np.float64) ** 2).sum(-1)
    scale2 = np.maximum(np.where(valid, xnorm2, 0).max(-1), 1e-30)  # (P, G) largest |x|^2
    d2 = np.where(valid, ((X - mean) ** 2).sum(-1), F32(-1)).astype(F32)
    a_idx = d2.argmax(-1)
    # two valid keys are equally far from their mean: whichever is taken first, the two centres are the two keys
    # and the split puts one key on each side, so the choice only mirrors the subtree (no margin is needed)
    ng = valid.sum(-1)
    margin = np.where(ng == 2, np.inf, _argmax_margin(d2, valid, 4 * scale2))
    a = np.take_along_axis(X, a_idx[..., None, None], 2)
    d2b = np.where(valid, ((X - a) ** 2).sum(-1), F32(-1)).astype(F32)
    b_idx = d2b.argmax(-1)
    margin = np.minimum(margin, _argmax_margin(d2b, valid, 4 * scale2))
    b = np.take_along_axis(X, b_idx[..., None, None], 2)
    c = np.concatenate([a, b], 2).astype(F32)
    xx = (X ** 2).sum(-1, keepdims=True).astype(F32)
    for _ in range(iters):
        dot = np.einsum('pgsd,pgcd->pgsc', X, c).astype(F32)
        dist = (xx - F32(2) * dot + (c ** 2).sum(-1)[:, :, None, :]).astype(F32)
        lab = dist.argmin(-1)
        # equal centres (a group of one key) give bitwise-equal distances: the first centre, in any summation order
        same = (c[:, :, 0] == c[:, :, 1]).all(-1)[..., None]
        gap = np.where(valid & ~same, _rel_gap(dist[..., 0], dist[..., 1], 4 * scale2[..., None]), np.inf)
        margin = np.minimum(margin, gap.min(-1))
        newc = c.copy()
        for j in (0, 1):
            m = ((lab == j) & valid)[..., None].astype(F32)
            cj = m.sum(2, keepdims=True)
            nc = ((X * m).sum(2, keepdims=True) / np.maximum(cj, F32(1))).astype(F32)
            newc[:, :, j:j + 1] = np.where(cj > 0, nc, c[:, :, j:j + 1])
        c = newc
    diff = (c[:, :, 0] - c[:, :, 1]).astype(F32)
    proj = np.einsum('pgsd,pgd->pgs', X, diff).astype(F32)
    proj = np.where(valid, proj, INF)
    order = np.argsort(proj, axis=-1, kind='stable')
    if not with_margin:
        return order
    # the side of the median split: the gap between the ranks nl - 1 and nl of the sorted valid projections
    nl = (ng + 1) // 2
    srt = np.take_along_axis(proj, order, -1).astype(np.float64)
    lo = np.take_along_axis(srt, np.maximum(nl - 1, 0)[..., None], -1)[..., 0]
    hi = np.take_along_axis(srt, np.minimum(nl, S - 1)[..., None], -1)[..., 0]
    dn = np.sqrt(scale2) * np.linalg.norm(diff.astype(np.float64), axis=-1)
    split = np.where((nl >= 1) & (nl < ng), _rel_gap(lo, hi, dn), np.inf)
    return order, np.minimum(margin, split)


class LaneTreeNP:
    """dyntree.py:34-131 LaneTree: one balanced binary tree per lane over a prefix of its keys.

    kfull (P, C, dh) fp32 (C a power of two), n (P,): lane p indexes the keys [1, n[p]). Levels 0..D with
    D = log2(C) - 1; node sums (fp32) and counts are held packed level by level (level l at rows 2^l - 1 ..
    2^(l+1) - 2), slots (P, 2^D, 2) hold the key positions of every last-level group (-1 = empty).

    node_margin (P, 2^(D+1) - 1) is the smallest relative gap of the decisions taken AT each node (its 2-means
    split, and the child choices of insertions passing through it): a near-tie there can only change what lies
    below the node. `margin` (P,) is the lane's smallest gap overall (plus, in select_keys, its searches)."""

    def __init__(self, kfull, n, iters=3):
        kfull = np.asarray(kfull, F32)
        P, C, dh = kfull.shape
        self.P, self.C, self.dh = P, C, dh
        self.D = D = int(round(math.log2(C))) - 1
        self.kfull = kfull
        ar = np.arange(P)[:, None]
        n = np.asarray(n, np.int64)
        perm = np.broadcast_to(np.arange(C), (P, C)).copy()
        valid = (perm >= 1) & (perm < n[:, None])
        self.node_margin = np.full(P, np.inf)[:, None].repeat((2 << D) - 1, 1)
        self.loop_margin = np.full(P, np.inf)
        for lvl in range(D):  # dyntree.py:54-73
            G = 1 << lvl
            S = C // G
            Xg = kfull[ar, perm].reshape(P, G, S, dh)
            vg = valid.reshape(P, G, S)
            pg = perm.reshape(P, G, S)
            order, mg = masked_two_means_order(Xg, vg, iters, with_margin=True)
            self.node_margin[:, G - 1:2 * G - 1] = np.minimum(self.node_margin[:, G - 1:2 * G - 1], mg)
            pg = np.take_along_axis(pg, order, 2)
            vg = np.take_along_axis(vg, order, 2)
            ng = vg.sum(-1)
            nl = (ng + 1) // 2
            nr = ng - nl
            r = np.arange(S).reshape(1, 1, S)
            half = S // 2
            left = r < half
            src_real = np.where(left, r, nl[..., None] + (r - half))
            cond = np.where(left, r < nl[..., None], (r - half) < nr[..., None])
            src = np.where(cond, src_real, S - 1)
            perm = np.take_along_axis(pg, src, 2).reshape(P, C)
            valid = cond.reshape(P, C)
        self.slot = np.where(valid, perm, -1).reshape(P, 1 << D, 2)
        self._sums_from_slots()

    def _sums_from_slots(self):
        P, C, dh, D = self.P, self.C, self.dh, self.D
        pos = self.slot.reshape(P, C)
        ok = pos >= 0
        kp = np.where(ok[..., None], self.kfull[np.arange(P)[:, None], np.maximum(pos, 0)], F32(0))
        NN = (2 << D) - 1
        self.sums = np.zeros((P, NN, dh), F32)
        self.cnt = np.zeros((P, NN), np.int64)
        offD = (1 << D) - 1
        self.sums[:, offD:offD + (1 << D)] = (kp[:, 0::2] + kp[:, 1::2]).astype(F32)
        self.cnt[:, offD:offD + (1 << D)] = ok[:, 0::2].astype(np.int64) + ok[:, 1::2]
        for l in range(D - 1, -1, -1):
            o, oc = (1 << l) - 1, (2 << l) - 1
            ch = self.sums[:, oc:oc + (2 << l)]
            self.sums[:, o:o + (1 << l)] = (ch[:, 0::2] + ch[:, 1::2]).astype(F32)
            cc = self.cnt[:, oc:oc + (2 << l)]
            self.cnt[:, o:o + (1 << l)] = cc[:, 0::2] + cc[:, 1::2]

    @property
    def margin(self):
        return np.minimum(self.node_margin.min(-1), self.loop_margin)

    def excluded(self, tie):
        """(P, 2^(D+1) - 1) bool, packed like the sums: nodes whose key set depends on a decision within `tie` of an
        fp32 tie (a strict ancestor's split or insertion choice came that close)."""
        P, D = self.P, self.D
        ex = np.zeros((P, (2 << D) - 1), bool)
        for l in range(D):
            o, oc = (1 << l) - 1, (2 << l) - 1
            bad = ex[:, o:o + (1 << l)] | (self.node_margin[:, o:o + (1 << l)] <= tie)
            ex[:, oc:oc + (2 << l)] = np.repeat(bad, 2, axis=1)
        return ex

    def level(self, l):
        o = (1 << l) - 1
        return self.sums[:, o:o + (1 << l)], self.cnt[:, o:o + (1 << l)]

    def insert(self, kv, kpos, active):
        """dyntree.py:83-106 LaneTree.insert: the new key is added to the root, then walks down, at each level to
        the child whose MEAN key scores higher against it (kv . sum / count; an empty child scores -1e9, a full one
        -inf; ties go left), adding itself to every node on its path; it takes the first free slot of the group it
        ends in. Inactive lanes change nothing."""
        kv = np.asarray(kv, F32)
        active = np.asarray(active, bool)
        kpos = np.asarray(kpos, np.int64)
        P, D, C = self.P, self.D, self.C
        ar = np.arange(P)
        act = active.astype(np.int64)
        kva = (kv * act[:, None].astype(F32)).astype(F32)
        node = np.zeros(P, np.int64)
        self.sums[ar, 0] += kva
        self.cnt[ar, 0] += act
        kn = np.linalg.norm(kv.astype(np.float64), axis=-1)
        gap_min = np.full(P, np.inf)
        for lvl in range(D):
            o = (2 << lvl) - 1
            left, right = 2 * node, 2 * node + 1
            cap = C >> (lvl + 1)
            cL, cR = self.cnt[ar, o + left], self.cnt[ar, o + right]
            SL, SR = self.sums[ar, o + left], self.sums[ar, o + right]
            sL = ((kv * SL).sum(-1).astype(F32) / np.maximum(cL, 1).astype(F32)).astype(F32)
            sR = ((kv * SR).sum(-1).astype(F32) / np.maximum(cR, 1).astype(F32)).astype(F32)
            sL = np.where(cL == 0, F32(-1e9), sL)
            sL = np.where(cL >= cap, -INF, sL)
            sR = np.where(cR == 0, F32(-1e9), sR)
            sR = np.where(cR >= cap, -INF, sR)
            both = active & (cL > 0) & (cR > 0) & (cL < cap) & (cR < cap)
            nrm = kn * np.maximum(np.linalg.norm(SL.astype(np.float64), axis=-1) / np.maximum(cL, 1),
                                  np.linalg.norm(SR.astype(np.float64), axis=-1) / np.maximum(cR, 1))
            par = (1 << lvl) - 1 + node
            gap = np.where(both, _rel_gap(sL, sR, nrm), np.inf)
            self.node_margin[ar, par] = np.minimum(self.node_margin[ar, par], gap)
            gap_min = np.minimum(gap_min, gap)
            node = np.where(sR > sL, right, left)
            self.sums[ar, o + node] += kva
            self.cnt[ar, o + node] += act
        s = (self.slot[ar, node, 0] >= 0).astype(np.int64)
        old = self.slot[ar, node, s]
        self.slot[ar, node, s] = np.where(active, kpos, old)
        return gap_min

    def search(self, qt, wmax):
        """dyntree.py:108-127 LaneTree.search (seg_oracle.lane_search on the packed levels). Returns ids, vld,
        sct (P, wl) and the cut margin (P,)."""
        return lane_search(qt, self.sums, self.cnt, self.D, wmax, with_margin=True)

    def leaf_keys(self, ids):
        """dyntree.py:129-131: leaf group ids (P, W) -> key positions (P, W, 2), -1 where a slot is empty."""
        return np.take_along_axis(self.slot, np.asarray(ids, np.int64)[..., None].repeat(2, -1), 1)

    def check(self):
        """dyntree.py:133-147 check: the worst mismatch between the node sums / counts and a recomputation from
        the slots."""
        P, C, dh, D = self.P, self.C, self.dh, self.D
        pos = self.slot.reshape(P, C)
        ok = pos >= 0
        kp = np.where(ok[..., None], self.kfull[np.arange(P)[:, None], np.maximum(pos, 0)], F32(0))
        worst = 0.0
        for l in range(D + 1):
            nn = 1 << l
            s = kp.reshape(P, nn, C // nn, dh).sum(2)
            c = ok.reshape(P, nn, C // nn).sum(2)
            S, Cn = self.level(l)
            worst = max(worst, float(np.abs(s - S).max()), float((c != Cn).sum()))
        return worst


def select_keys(q, k, lhat, chunk, wmax, nb_window, nb_store, nb_rho, nb_probe, nb_cap_min, neighbors=True,
                kmeans_iters=3):
    """dyntree.py:150-243 select_keys: the sequence (T a power of two) is cut into lanes of `chunk` tokens; lane l
    starts from a tree built over the keys [1, l*chunk) and walks its tokens in order: (1) neighbour search over
    the best groups stored by the previous nb_window queries OF THE LANE (rescored on the current tree:
    q . sum / count, matched when >= base - rho |base|, scan depth capped by the probe rate), (2) beam descent for
    the tree budget, (3) insertion of the token's key (position 0, the sink, is never inserted).

    q, k (B, H, T, dh); lhat (B, H, T). Returns tree_pos (B, H, T, 2 wl), leaf_ok (B, H, T, wl),
    nb_pos (B, H, T, 2 Wn NS), n_tree, nb_leaves (B, H, T), and margin (B, H, T // chunk): the smallest relative
    decision gap of each lane over the build, its insertions, searches and neighbour tests."""
    q = np.asarray(q, F32)
    k = np.asarray(k, F32)
    B, H, T, dh = q.shape
    Y = chunk
    assert T % Y == 0 and (T & (T - 1)) == 0
    nl = T // Y
    P = B * H * nl
    Wn, NS = nb_window, nb_store
    D = int(round(math.log2(T))) - 1
    wl = min(wmax, 1 << D)
    starts = np.arange(nl) * Y
    kfull = np.broadcast_to(k[:, :, None], (B, H, nl, T, dh)).reshape(P, T, dh)
    n0 = np.broadcast_to(starts, (B, H, nl)).reshape(P)
    tree = LaneTreeNP(kfull, n0, kmeans_iters)
    return select_loop(tree, q, k, lhat, chunk, wmax, nb_window, nb_store, nb_rho, nb_probe, nb_cap_min,
                       neighbors=neighbors)


def select_loop(tree, q, k, lhat, chunk, wmax, nb_window, nb_store, nb_rho, nb_probe, nb_cap_min, neighbors=True):
    """dyntree.py:177-243, the token loop of select_keys on the lanes' trees as built (LaneTreeNP over the keys
    [1, l chunk) of lane l; the tree is updated in place). Outputs as select_keys; `margin` (B, H, T // chunk) is
    the lane's smallest gap over the build and the loop, `loop_margin` over the loop's decisions alone,
    `query_margin` (B, H, T) over the loop decisions a query's results depend on (its own step and the earlier
    steps of its lane), `build_margin` (B, H, T // chunk) over the build."""
    q = np.asarray(q, F32)
    k = np.asarray(k, F32)
    B, H, T, dh = q.shape
    Y = chunk
    nl = T // Y
    P = B * H * nl
    Wn, NS = nb_window, nb_store
    D = int(round(math.log2(T))) - 1
    wl = min(wmax, 1 << D)
    starts = np.arange(nl) * Y
    lhat = np.asarray(lhat, np.int64)
    build_margin = tree.margin.copy()
    tree.loop_margin = np.full(P, np.inf)
    step_margin = np.full((B, H, T), np.inf)

    tree_pos = np.full((B, H, T, 2 * wl), -1, np.int64)
    leaf_ok = np.zeros((B, H, T, wl), bool)
    nb_pos = np.full((B, H, T, Wn * NS * 2), -1, np.int64)
    n_tree = np.zeros((B, H, T), np.int64)
    nb_leaves = np.zeros((B, H, T), np.int64)
    st_leaf = np.zeros((B, H, T, NS), np.int64)
    st_score = np.zeros((B, H, T, NS), F32)
    st_ok = np.zeros((B, H, T, NS), bool)
    dist_idx = np.arange(Wn * NS) // NS + 1
    back = np.arange(1, Wn + 1)
    probe = nb_probe * NS
    rho = F32(nb_rho)
    offD = (1 << D) - 1
    for i in range(Y):
        tpos = starts + i
        qt = q[:, :, tpos].reshape(P, dh)
        kt = k[:, :, tpos].reshape(P, dh)
        tposP = np.broadcast_to(tpos, (B, H, nl)).reshape(P)
        L = lhat[:, :, tpos].reshape(P)

        # (1) neighbour search, dyntree.py:197-214
        jpos = tpos[:, None] - back[None, :]
        jval = jpos >= starts[:, None]
        jc = np.maximum(jpos, 0)
        ids = st_leaf[:, :, jc].reshape(P, Wn * NS)
        base = st_score[:, :, jc].reshape(P, Wn * NS)
        ok0 = (st_ok[:, :, jc] & jval[None, None, :, :, None]).reshape(P, Wn * NS)
        sm = tree.sums[np.arange(P)[:, None], offD + ids]
        cn = tree.cnt[np.arange(P)[:, None], offD + ids]
        sc_t = (np.einsum('pd,pcd->pc', qt, sm).astype(F32) / np.maximum(cn, 1).astype(F32)).astype(F32)
        thr = (base - (rho * np.abs(base)).astype(F32)).astype(F32)
        match = ok0 & (cn > 0) & (sc_t >= thr)
        nrm = (np.linalg.norm(qt.astype(np.float64), axis=-1)[:, None]
               * np.linalg.norm(sm.astype(np.float64), axis=-1) / np.maximum(cn, 1))
        gap = np.where(ok0 & (cn > 0), _rel_gap(sc_t, thr, nrm), np.inf)
        step_m = gap.min(-1)
        rate = (match[:, :probe].sum(1).astype(F32) / np.maximum(ok0[:, :probe].sum(1), 1).astype(F32)).astype(F32)
        cap = nb_cap_min + np.rint(F32(Wn - nb_cap_min) * rate).astype(np.int64)
        match = match & (dist_idx[None, :] <= cap[:, None])
        if not neighbors:
            match = np.zeros_like(match)
        idm = np.where(match, ids, -1)
        ss = np.sort(idm, -1)
        vs = ss >= 0
        nL = vs.sum(1) - ((ss[:, 1:] == ss[:, :-1]) & vs[:, 1:]).sum(1)

        # (2) tree search for the rest of the budget, dyntree.py:216-227
        lo = (L + 1) // 2
        need = np.maximum(L - nL, 0)
        floor_b = np.where(nL < lo, 2, 1)
        b_tree = np.minimum(np.where(nL >= L, 0, np.maximum(need, floor_b)), wmax)
        cur, cvld, sct, mg = tree.search(qt, wmax)
        step_m = np.minimum(step_m, mg)
        pos = tree.leaf_keys(cur)
        pos = np.where((pos >= 0) & cvld[..., None], pos, -1)
        tp = np.concatenate([pos[..., 0], pos[..., 1]], -1)
        npos = tree.leaf_keys(ids)
        npos = np.where((npos >= 0) & match[..., None], npos, -1)
        npos = np.concatenate([npos[..., 0], npos[..., 1]], -1)

        tree_pos[:, :, tpos] = tp.reshape(B, H, nl, 2 * wl)
        leaf_ok[:, :, tpos] = cvld.reshape(B, H, nl, wl)
        nb_pos[:, :, tpos] = npos.reshape(B, H, nl, Wn * NS * 2)
        n_tree[:, :, tpos] = b_tree.reshape(B, H, nl)
        nb_leaves[:, :, tpos] = nL.reshape(B, H, nl)
        st_leaf[:, :, tpos] = cur[:, :NS].reshape(B, H, nl, NS)
        st_score[:, :, tpos] = sct[:, :NS].reshape(B, H, nl, NS)
        st_ok[:, :, tpos] = cvld[:, :NS].reshape(B, H, nl, NS)

        # (3) insertion, dyntree.py:238-239
        step_m = np.minimum(step_m, tree.insert(kt, tposP, tposP >= 1))
        step_margin[:, :, tpos] = step_m.reshape(B, H, nl)
        tree.loop_margin = np.minimum(tree.loop_margin, step_m)

    # a query's results depend on the decisions of its own step and of every earlier step of its lane
    lane_steps = step_margin.reshape(B, H, nl, Y)
    upto = np.minimum.accumulate(lane_steps, axis=-1).reshape(B, H, T)
    loop = tree.loop_margin
    return dict(tree_pos=tree_pos, leaf_ok=leaf_ok, nb_pos=nb_pos, n_tree=n_tree, nb_leaves=nb_leaves,
                margin=np.minimum(build_margin, loop).reshape(B, H, nl), loop_margin=loop.reshape(B, H, nl),
                query_margin=upto, build_margin=build_margin.reshape(B, H, nl))


def canonical_tree(slot, sums=None, cnt=None, with_order=False):
    """The tree with the two children of every node put in a canonical order: the child whose subtree holds the
    smaller key position first (an empty subtree last), and the two positions of every last-level group sorted.

    The build decides a subtree's left/right orientation by comparisons that can be exact fp32 ties (a group of two
    keys: both are equally far from their mean); both orientations hold the same keys in mirrored places, and a
    search or insertion takes the same keys in either, so trees are compared in this form. slot (P, 2^D, 2);
    sums (P, 2^(D+1) - 1, dh) and cnt (P, 2^(D+1) - 1) packed by level are reordered along."""
    slot = np.asarray(slot, np.int64)
    P, NL, _ = slot.shape
    D = NL.bit_length() - 1
    big = np.iinfo(np.int64).max
    # subtree minimum position of every node, bottom-up
    mins = [None] * (D + 1)
    mins[D] = np.where(slot >= 0, slot, big).min(-1)
    for l in range(D - 1, -1, -1):
        mins[l] = np.minimum(mins[l + 1][:, 0::2], mins[l + 1][:, 1::2])
    # canonical node order per level: new index i at level l -> original node id
    ar = np.arange(P)[:, None]
    order = [np.zeros((P, 1), np.int64)]
    for l in range(1, D + 1):
        par = order[-1]
        c0, c1 = 2 * par, 2 * par + 1
        swap = mins[l][ar, c1] < mins[l][ar, c0]
        first = np.where(swap, c1, c0)
        second = np.where(swap, c0, c1)
        order.append(np.stack([first, second], -1).reshape(P, -1))
    slot_c = np.sort(np.where(slot >= 0, slot, big)[ar, order[D]], -1)
    slot_c = np.where(slot_c == big, -1, slot_c)
    idx = np.concatenate([(1 << l) - 1 + order[l] for l in range(D + 1)], 1)  # canonical row -> original row
    if sums is None:
        return (slot_c, idx) if with_order else slot_c
    out = (slot_c, np.asarray(sums)[ar, idx], np.asarray(cnt)[ar, idx])
    return out + (idx,) if with_order else out


def prefix_mean(k):
    """attention_dyn.py:66-69: the mean of the keys before each position, (cumsum - k) / max(t, 1)."""
    k = np.asarray(k, F32)
    T = k.shape[-2]
    cs = np.cumsum(k, axis=-2, dtype=F32)
    return ((cs - k) / np.maximum(np.arange(T), 1).astype(F32)[:, None]).astype(F32)


def dyn_attention(q, k, v, sel, local, chunk=64):
    """attention_dyn.py:80-98 DynAttention.sparse_attend after the selection: the candidates
    [tree positions, neighbour positions, sink + local window], the tree part limited to the first n_tree found
    groups, deduplicated, then exact softmax attention. Returns (out, stats)."""
    q = np.asarray(q, F32)
    B, H, T, dh = q.shape
    scale = 1.0 / math.sqrt(dh)
    tree_pos, nb_pos, leaf_ok = sel['tree_pos'], sel['nb_pos'], sel['leaf_ok']
    wl = leaf_ok.shape[-1]
    NBK = nb_pos.shape[-1]
    Lw = max(int(local), 3)
    t = np.arange(T)
    st = np.concatenate([np.zeros((T, 1), np.int64), t[:, None] - np.arange(Lw)[None, :]], 1)
    st = np.broadcast_to(np.where(st < 0, -1, st), (B, H, T, 1 + Lw))
    cand = np.concatenate([tree_pos, nb_pos, st], -1)
    used = leaf_ok & (np.arange(wl) < sel['n_tree'][..., None])
    tv_used = np.concatenate([used, used], -1) & (tree_pos >= 0)
    rest = np.concatenate([nb_pos >= 0, st >= 0], -1)
    keep = dedupe(cand, np.concatenate([tv_used, rest], -1))
    out = sparse_attn(q, k, v, np.where(keep, cand, -1), scale, chunk=chunk)
    stats = dict(keys_total=float(keep.sum(-1).mean()), keys_tree=float(keep[..., :2 * wl].sum(-1).mean()),
                 keys_nb=float(keep[..., 2 * wl:2 * wl + NBK].sum(-1).mean()),
                 nb_leaves=float(sel['nb_leaves'].mean()), leaves_used=float(used.sum(-1).mean()))
    return out, stats


def budget_head(q, k, pw, classes, H, global_pool):
    """attention_dyn.py:57-72: the learned leaf budget. Features [q, log(|q| + 1e-6), one-hot head, (prefix mean of
    the keys)] -> Linear -> ReLU -> Linear -> argmax over the budget classes. pw = (w0, b0, w2, b2)."""
    q = np.asarray(q, F32)
    B, Hq, T, dh = q.shape
    feats = [q, np.log(np.linalg.norm(q, axis=-1, keepdims=True).astype(F32) + F32(1e-6)).astype(F32),
             np.broadcast_to(np.eye(H, dtype=F32)[None, :, None, :], (B, H, T, H))]
    if global_pool:
        feats.append(prefix_mean(k))
    x = np.concatenate(feats, -1).astype(F32)
    w0, b0, w2, b2 = [np.asarray(a, F32) for a in pw]
    h = np.maximum((x @ w0.T + b0).astype(F32), F32(0))
    plog = (h @ w2.T + b2).astype(F32)
    return np.asarray(classes, np.int64)[plog.argmax(-1)]


def gpt_forward_dyn(sd, cfg, idx):
    """model.py:75-93 GPT.forward with DynAttention (attn='dyn') blocks, fp32. sd: the model's state dict (numpy
    or torch); cfg: a dict with n_layer, n_head, chunk, wmax, beam, beam_mode, beam_classes, global_pool, local,
    neighbors, nb_window, nb_store, nb_rho, nb_probe, nb_cap_min, kmeans_iters. Returns (logits, stats)."""
    from .seg_oracle import gelu, layer_norm
    g = lambda name: np.asarray(sd[name].detach().float().cpu().numpy() if hasattr(sd[name], 'detach') else sd[name],
                                F32)
    idx = np.asarray(idx, np.int64)
    B, T = idx.shape
    wte = g('wte.weight')
    C = wte.shape[1]
    H = cfg['n_head']
    dh = C // H
    x = (wte[idx] + g('wpe.weight')[np.arange(T)]).astype(F32)
    acc = {}
    for i in range(cfg['n_layer']):
        p = 'blocks.%d.' % i
        h = layer_norm(x, g(p + 'ln1.weight'))
        qkv = (h @ g(p + 'attn.c_attn.weight').T).astype(F32)
        q, k, v = [qkv[..., j * C:(j + 1) * C].reshape(B, T, H, dh).transpose(0, 2, 1, 3) for j in range(3)]
        if cfg['beam_mode'] == 'pred':
            pw = [g(p + 'attn.pred.%s' % n) for n in ('0.weight', '0.bias', '2.weight', '2.bias')]
            lhat = budget_head(q, k, pw, cfg['beam_classes'], H, cfg['global_pool'])
        else:
            lhat = np.full((B, H, T), cfg['beam'], np.int64)
        sel = select_keys(q, k, lhat, cfg['chunk'], cfg['wmax'], cfg['nb_window'], cfg['nb_store'], cfg['nb_rho'],
                          cfg['nb_probe'], cfg['nb_cap_min'], neighbors=cfg['neighbors'],
                          kmeans_iters=cfg['kmeans_iters'])
        o, st = dyn_attention(q, k, v, sel, cfg['local'])
        for name, val in st.items():
            acc[name] = acc.get(name, 0.0) + val
        acc['margin'] = min(acc.get('margin', np.inf), float(sel['margin'].min()))
        x = (x + (o.transpose(0, 2, 1, 3).reshape(B, T, C) @ g(p + 'attn.c_proj.weight').T)).astype(F32)
        f = gelu((layer_norm(x, g(p + 'ln2.weight')) @ g(p + 'mlp.c_fc.weight').T).astype(F32))
        x = (x + (f @ g(p + 'mlp.c_proj.weight').T)).astype(F32)
    logits = (layer_norm(x, g('ln_f.weight')) @ wte.T).astype(F32)
    n = cfg['n_layer']
    margin = acc.pop('margin')
    stats = {name: val / n for name, val in acc.items()}
    stats['margin'] = margin
    return logits, stats
