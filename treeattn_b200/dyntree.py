"""Dynamic content tree (reference dyntree.py): the search side on the B200.

The reference's LaneTree keeps, per lane, a balanced binary tree over the keys seen so far: every node holds the
SUM of the keys below it and their count, and a query descends it by the MEAN key of each node
(LaneTree.search, dyntree.py:108-127). Here the tree's levels live packed in one fp32 tensor (level l at rows
2^l - 1 .. 2^(l+1) - 2) with a parallel int32 count tensor, and the descent is one CUDA kernel (ta_lane_search).

Building a tree (the 2-means splits, dyntree.py:6-73), inserting keys (dyntree.py:83-106) and the lane-by-lane
selection loop select_keys (dyntree.py:150-243) are not implemented in this package: they raise
NotImplementedError. A tree built elsewhere (for instance by the reference itself) is wrapped with
LaneTree.from_levels and searched here.
"""
import torch

from . import _lib, _ops


def _pack(levels, dtype):
    return torch.cat(list(levels), 1).to(dtype)


class LaneTree:
    """Node sums (P, 2^(D+1) - 1, dh) fp32 and counts (P, 2^(D+1) - 1) int32, packed level by level, and the
    leaf-group slots (P, 2^D, 2) key positions (-1 = empty), as the reference's LaneTree holds them."""

    def __init__(self, kfull, n, iters=3):
        raise NotImplementedError('building a LaneTree (2-means splits, dyntree.py:35-73) is not implemented in '
                                  'treeattn_b200; wrap a built tree with LaneTree.from_levels')

    @classmethod
    def from_levels(cls, sums, cnt, slot=None):
        """sums: list of (P, 2^l, dh) per level l = 0..D (or the packed tensor); cnt likewise (P, 2^l);
        slot: (P, 2^D, 2) positions of the two keys of every last-level group (optional, for leaf_keys)."""
        t = cls.__new__(cls)
        if isinstance(sums, (list, tuple)):
            sums = _pack(sums, torch.float32)
            cnt = _pack(cnt, torch.int32)
        t.sums = sums.to(torch.float32).contiguous()
        t.cnt = cnt.to(torch.int32).contiguous()
        t.P, NN, t.dh = t.sums.shape
        t.D = (NN + 1).bit_length() - 2  # NN = 2^(D+1) - 1
        if (2 << t.D) - 1 != NN or tuple(t.cnt.shape) != (t.P, NN):
            raise ValueError('packed tree: %d rows is not 2^(D+1) - 1, or counts do not match' % NN)
        t.slot = slot
        return t

    def search(self, qt, wmax):
        """Beam descent for one query per lane (dyntree.py:108-127). qt (P, dh). Returns leaf ids (P, wl),
        validity (P, wl) and scores (P, wl), best first; wl = min(wmax, 2^D)."""
        _ops._need_cuda('LaneTree.search', qt, self.sums, self.cnt)
        q = qt.to(torch.float32).contiguous()
        wl = min(wmax, 1 << self.D)
        dev = q.device
        ids = torch.empty(self.P, wl, device=dev, dtype=torch.int64)
        vld = torch.empty(self.P, wl, device=dev, dtype=torch.bool)
        sct = torch.empty(self.P, wl, device=dev, dtype=torch.float32)
        _lib.call('ta_lane_search', _ops._p(q), _ops._p(self.sums), _ops._p(self.cnt), self.P, self.D, self.dh,
                  int(wmax), wl, _ops._p(ids), _ops._p(vld), _ops._p(sct), _ops._stream(q))
        return ids, vld, sct

    def leaf_keys(self, ids):
        """ids: (P, W) leaf group ids -> key positions (P, W, 2), -1 where a slot is empty."""
        if self.slot is None:
            raise ValueError('this tree was wrapped without its slots')
        return self.slot.gather(1, ids.unsqueeze(-1).expand(-1, -1, 2))

    def insert(self, kv, kpos, active):
        raise NotImplementedError('LaneTree.insert (dyntree.py:83-106) is not implemented in treeattn_b200')


def select_keys(q, k, lhat, cfg):
    """dyntree.py:150-243 (attn='dyn' key selection). Not implemented in this package."""
    raise NotImplementedError("dyntree.select_keys (attn='dyn') is not implemented in treeattn_b200")
