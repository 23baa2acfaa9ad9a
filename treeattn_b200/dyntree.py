"""Dynamic content tree (reference dyntree.py, attn='dyn') on the B200.

The reference's LaneTree keeps, per lane, a balanced binary tree over the keys seen so far: every node holds the
SUM of the keys below it and their count; a tree is built by 2-means splits (dyntree.py:6-73), grows by insertion
(dyntree.py:83-106) and is searched by the MEAN key of each node (dyntree.py:108-127). select_keys
(dyntree.py:150-243) walks the tokens of every lane in order: neighbour search, tree search, insertion.

Here a tree's levels live packed in one fp32 tensor (level l at rows 2^l - 1 .. 2^(l+1) - 2) with a parallel int32
count tensor and int32 group slots, and every step is a CUDA kernel of libtreeattn_b200: ta_lane_order (the 2-means
splits, level by level), ta_lane_sums (slots and node sums), ta_lane_insert, ta_lane_search and ta_lane_select (one
warp per lane runs the whole token loop of select_keys, updating its tree in place).

A build decides the left/right orientation of a subtree by fp32 comparisons, some of which are exact ties (a group
of two keys: both are equally far from their mean); either orientation holds the same keys in mirrored places and
every search and insertion takes the same keys from both, so two builds are compared in a canonical child order.
"""
import math

import torch

from . import _lib, _ops


def _pack(levels, dtype):
    return torch.cat(list(levels), 1).to(dtype)


def _order(keys, lane_div, n, first, P, C, dh, iters, levels):
    """ta_lane_order over fp32 keys (lane p reads the (C, dh) array p // lane_div) -> (perm (P, C) int32,
    valid (P, C) uint8)."""
    dev = keys.device
    perm = torch.empty(P, C, device=dev, dtype=torch.int32)
    valid = torch.empty(P, C, device=dev, dtype=torch.uint8)
    perm_t = torch.empty_like(perm)
    valid_t = torch.empty_like(valid)
    n = n.to(device=dev, dtype=torch.int64).contiguous()
    _lib.call('ta_lane_order', _ops._p(keys), int(lane_div), C * dh, _ops._p(n), int(first), P, C, dh,
              int(iters), int(levels), _ops._p(perm), _ops._p(valid), _ops._p(perm_t), _ops._p(valid_t),
              _ops._stream(keys))
    return perm, valid


class LaneTree:
    """dyntree.py:34-147 LaneTree: node sums (P, 2^(D+1) - 1, dh) fp32 and counts (P, 2^(D+1) - 1) int32, packed level
    by level (`sums[l]` / `cnt[l]` are per-level views, as the reference's lists), and the group slots
    (P, 2^D, 2) key positions (-1 = empty)."""

    def __init__(self, kfull, n, iters=3):
        """dyntree.py:46-80: kfull (P, C, dh) (C a power of two), n (P,): lane p starts from the keys [1, n[p])."""
        _ops._need_cuda('LaneTree', kfull)
        P, C, dh = kfull.shape
        if C < 4 or C & (C - 1):
            raise ValueError('LaneTree: capacity C=%d must be a power of two >= 4' % C)
        self.P, self.C, self.dh = P, C, dh
        self.D = int(round(math.log2(C))) - 1
        self.dev = kfull.device
        self.kfull = kfull
        kf = kfull.float().contiguous()
        perm, valid = _order(kf, 1, torch.as_tensor(n), 1, P, C, dh, iters, self.D)
        self._alloc()
        _lib.call('ta_lane_sums', _ops._p(kf), 1, C * dh, _ops._p(perm), _ops._p(valid), P, C, dh,
                  _ops._p(self._sums), _ops._p(self._cnt), _ops._p(self._slot), _ops._stream(kf))

    def _alloc(self):
        NN = (2 << self.D) - 1
        self._sums = torch.empty(self.P, NN, self.dh, device=self.dev, dtype=torch.float32)
        self._cnt = torch.empty(self.P, NN, device=self.dev, dtype=torch.int32)
        self._slot = torch.empty(self.P, 1 << self.D, 2, device=self.dev, dtype=torch.int32)

    @property
    def sums(self):
        return [self._sums[:, (1 << l) - 1:(2 << l) - 1] for l in range(self.D + 1)]

    @property
    def cnt(self):
        return [self._cnt[:, (1 << l) - 1:(2 << l) - 1] for l in range(self.D + 1)]

    @property
    def slot(self):
        return None if self._slot is None else self._slot.long()

    @property
    def packed(self):
        """(sums, counts) packed level by level, as the kernels read them."""
        return self._sums, self._cnt

    @classmethod
    def from_levels(cls, sums, cnt, slot=None):
        """sums: list of (P, 2^l, dh) per level l = 0..D (or the packed tensor); cnt likewise (P, 2^l);
        slot: (P, 2^D, 2) positions of the two keys of every last-level group (optional, for leaf_keys)."""
        t = cls.__new__(cls)
        if isinstance(sums, (list, tuple)):
            sums = _pack(sums, torch.float32)
            cnt = _pack(cnt, torch.int32)
        t._sums = sums.to(torch.float32).contiguous()
        t._cnt = cnt.to(torch.int32).contiguous()
        t.P, NN, t.dh = t._sums.shape
        t.D = (NN + 1).bit_length() - 2  # NN = 2^(D+1) - 1
        if (2 << t.D) - 1 != NN or tuple(t._cnt.shape) != (t.P, NN):
            raise ValueError('packed tree: %d rows is not 2^(D+1) - 1, or counts do not match' % NN)
        t.C = 2 << t.D
        t.dev = t._sums.device
        t.kfull = None
        t._slot = None if slot is None else slot.to(torch.int32).contiguous()
        return t

    def insert(self, kv, kpos, active):
        """dyntree.py:83-106: kv (P, dh) new keys, kpos (P,) their positions, active (P,) bool (False = no change)."""
        if self._slot is None:
            raise ValueError('this tree was wrapped without its slots')
        _ops._need_cuda('LaneTree.insert', kv, self._sums)
        kv = kv.to(torch.float32).contiguous()
        kpos = kpos.to(device=self.dev, dtype=torch.int64).contiguous()
        active = active.to(device=self.dev, dtype=torch.uint8).contiguous()
        _lib.call('ta_lane_insert', _ops._p(kv), _ops._p(kpos), _ops._p(active), self.P, self.C, self.dh,
                  _ops._p(self._sums), _ops._p(self._cnt), _ops._p(self._slot), _ops._stream(kv))

    def search(self, qt, wmax):
        """Beam descent for one query per lane (dyntree.py:108-127). qt (P, dh). Returns leaf ids (P, wl),
        validity (P, wl) and scores (P, wl), best first; wl = min(wmax, 2^D)."""
        _ops._need_cuda('LaneTree.search', qt, self._sums, self._cnt)
        q = qt.to(torch.float32).contiguous()
        wl = min(wmax, 1 << self.D)
        dev = q.device
        ids = torch.empty(self.P, wl, device=dev, dtype=torch.int64)
        vld = torch.empty(self.P, wl, device=dev, dtype=torch.bool)
        sct = torch.empty(self.P, wl, device=dev, dtype=torch.float32)
        _lib.call('ta_lane_search', _ops._p(q), _ops._p(self._sums), _ops._p(self._cnt), self.P, self.D, self.dh,
                  int(wmax), wl, _ops._p(ids), _ops._p(vld), _ops._p(sct), _ops._stream(q))
        return ids, vld, sct

    def leaf_keys(self, ids):
        """ids: (P, W) leaf group ids -> key positions (P, W, 2), -1 where a slot is empty."""
        if self._slot is None:
            raise ValueError('this tree was wrapped without its slots')
        return self._slot.long().gather(1, ids.unsqueeze(-1).expand(-1, -1, 2))

    def check(self):
        """dyntree.py:133-147: the worst mismatch between the node sums / counts and a recomputation from the
        slots (0 = consistent)."""
        if self._slot is None or self.kfull is None:
            raise ValueError('check needs a tree built here (keys and slots)')
        P, C, dh = self.P, self.C, self.dh
        pos = self.slot.reshape(P, C)
        valid = pos >= 0
        kp = self.kfull.float().gather(1, pos.clamp(min=0).unsqueeze(-1).expand(-1, -1, dh)) \
            * valid.unsqueeze(-1).float()
        worst = 0.0
        for lvl, (S, Cn) in enumerate(zip(self.sums, self.cnt)):
            nn = 2 ** lvl
            s = kp.reshape(P, nn, C // nn, dh).sum(2)
            c = valid.reshape(P, nn, C // nn).sum(2)
            worst = max(worst, (s - S).abs().max().item(), float((c != Cn).sum().item()))
            assert (Cn <= C // nn).all(), 'node over capacity at level %d' % lvl
        return worst


@torch.no_grad()
def select_keys(q, k, lhat, cfg):
    """dyntree.py:150-243 select_keys: lanes of cfg.chunk tokens, each starting from a tree over the keys before
    its first token; per token the neighbour search, the tree search for the rest of the budget lhat, and the
    insertion of its key (ta_lane_select, one warp per lane). q, k (b, H, T, dh); lhat (b, H, T).
    Returns tree_pos (b, H, T, 2 wl), leaf_ok (b, H, T, wl), nb_pos (b, H, T, 2 nb_window nb_store), n_tree,
    nb_leaves (b, H, T)."""
    _ops._need_cuda('select_keys', q, k)
    b, H, T, dh = q.shape
    Y = cfg.chunk
    if T % Y or T & (T - 1):
        raise ValueError('select_keys: T=%d must be a power of two and a multiple of chunk=%d' % (T, Y))
    nl = T // Y
    P = b * H * nl
    dev = q.device
    D = int(round(math.log2(T))) - 1
    wl = min(cfg.wmax, 1 << D)
    Wn, NS = cfg.nb_window, cfg.nb_store
    qf = q.float().contiguous()
    kf = k.float().contiguous()
    n0 = (torch.arange(nl, device=dev, dtype=torch.int64) * Y).repeat(b * H)
    perm, valid = _order(kf, nl, n0, 1, P, T, dh, cfg.kmeans_iters, D)
    tree = LaneTree.__new__(LaneTree)
    tree.P, tree.C, tree.dh, tree.D, tree.dev, tree.kfull = P, T, dh, D, dev, None
    tree._alloc()
    _lib.call('ta_lane_sums', _ops._p(kf), nl, T * dh, _ops._p(perm), _ops._p(valid), P, T, dh,
              _ops._p(tree._sums), _ops._p(tree._cnt), _ops._p(tree._slot), _ops._stream(kf))
    del perm, valid
    lh = lhat.to(device=dev, dtype=torch.int64).contiguous()
    tree_pos = torch.empty(b, H, T, 2 * wl, device=dev, dtype=torch.int64)
    leaf_ok = torch.empty(b, H, T, wl, device=dev, dtype=torch.bool)
    nb_pos = torch.empty(b, H, T, 2 * Wn * NS, device=dev, dtype=torch.int64)
    n_tree = torch.empty(b, H, T, device=dev, dtype=torch.int64)
    nb_leaves = torch.empty(b, H, T, device=dev, dtype=torch.int64)
    _lib.call('ta_lane_select', _ops._p(qf), _ops._p(kf), _ops._p(lh), b, H, T, dh, Y, int(cfg.wmax), Wn, NS,
              int(cfg.nb_probe), int(cfg.nb_cap_min), float(cfg.nb_rho), int(bool(cfg.neighbors)),
              _ops._p(tree._sums), _ops._p(tree._cnt), _ops._p(tree._slot), _ops._p(tree_pos), _ops._p(leaf_ok),
              _ops._p(nb_pos), _ops._p(n_tree), _ops._p(nb_leaves), _ops._stream(qf))
    return dict(tree_pos=tree_pos, leaf_ok=leaf_ok, nb_pos=nb_pos, n_tree=n_tree, nb_leaves=nb_leaves)
