"""Segment-tree key selection (reference seg.py), backed by the sm_100a kernels.

Same names, arguments and results as the reference module. Differences, all explicit:
  * tree_pass takes the tree itself (the dict returned by level_sums, a Levels object or a SegState /
    its bound getU) instead of an arbitrary getU callable: the descent runs inside one CUDA kernel.
  * Leaf blocks of cfg.leaf tokens (default 2 = the reference) are supported; positions of a leaf block m are
    [m*leaf, (m+1)*leaf), stored leaf-slot-major as the reference's cat([2*ids, 2*ids+1]) is at leaf 2.
"""
import torch

from . import _ops
from ._ops import Levels, LevelDict


def _leaf_level(cfg):
    return _ops.log2_exact(getattr(cfg, 'leaf', 2), 'cfg.leaf') if cfg is not None else 1


@torch.no_grad()
def gate_apply(raw, lgsum, size, gate_q):
    """Mean-log dilution gate (seg.py:16-23) on rows (..., dh) of node sums and their log-magnitude sums over
    groups of `size` (a power of two) keys (ta_gate_levels on the rows as one tree level)."""
    l = _ops.log2_exact(size, 'size')
    if l < 1:
        raise ValueError('gate_apply: group size must be at least 2')
    dh = raw.shape[-1]
    n = raw.numel() // dh
    rv = raw.float().reshape(1, 1, n, dh).contiguous()
    gv = lgsum.float().reshape(1, 1, n, dh).contiguous()
    out = torch.empty_like(rv)
    mk = lambda t: Levels(t, n << l, l, l)
    _ops.gate_levels(mk(rv), mk(gv), gate_q, 0, n << l, out=mk(out))
    return out.reshape(raw.shape)


def gated_tree(k, cap, L0, Lm, gate_q, gate_min, zero_sink=True, raw=None):
    """(raw levels, log-magnitude levels, gated levels) of keys k (B, H, T, dh): the gate of fastseg.level_sums_min
    (levels >= gate_min gated, the others copied)."""
    T = k.shape[2]
    if raw is None:
        raw = _ops.build_levels(k, cap, L0, Lm, zero_sink=zero_sink)
    lg = _ops.build_log_levels(k, cap, L0, Lm, zero_sink=zero_sink)
    return raw, lg, _ops.gate_levels(raw, lg, gate_q, gate_min, T)


@torch.no_grad()
def level_sums(kidx, Lm, gate, gate_q):
    """seg.py:26-41: {l: (b, H, T >> l, dh)} fp32 node sums for l = 1..Lm from kidx (b, H, T, dh) as given
    (select_seg zeroes the sink before calling it), mean-log gated at every level when `gate`. The returned dict
    carries the packed storage."""
    T = kidx.shape[2]
    if gate:
        return gated_tree(kidx, T, 1, Lm, gate_q, 0, zero_sink=False)[2].as_dict()
    lv = _ops.build_levels(kidx, T, 1, Lm, zero_sink=False)
    return lv.as_dict()


def _as_levels(getU):
    if isinstance(getU, Levels):
        return getU
    if isinstance(getU, LevelDict):
        return getU.packed
    owner = getattr(getU, '__self__', None)
    if owner is not None and hasattr(owner, 'levels') and isinstance(owner.levels, Levels):
        return owner.levels
    if hasattr(getU, 'levels') and isinstance(getU.levels, Levels):
        return getU.levels
    raise TypeError('tree_pass needs the tree itself (level_sums() result, Levels, or a SegState / its getU); '
                    'an arbitrary getU callable cannot run inside the CUDA descent')


@torch.no_grad()
def tree_pass(q, getU, tq, Lm, wmax):
    """seg.py:44-70: past-only beam descent. q (b, H, Nq, dh); tq (Nq,) positions (or (b,) / (b, Nq)).
    Returns leaf ids (b, H, Nq, wl), validity and scores (q . S_L0 / 2^L0), best first."""
    lv = _as_levels(getU)
    if Lm != lv.Lm:
        lv = Levels(lv.nodes, lv.cap, lv.L0, Lm) if Lm <= lv.Lm else None
        if lv is None:
            raise ValueError('tree_pass: Lm=%d above the stored levels' % Lm)
    return _ops.select(q, lv, tq.to(q.device), wmax)


@torch.no_grad()
def neighbor_pass(q, getU1, st_leaf, st_score, st_ok, tq, cfg):
    """seg.py:73-103: borrow the best leaves stored by the nb_window previous positions (st_* (b, H, T, NS)) that
    this query also scores well on (ta_neighbor_pass). getU1 is the tree (its leaf level scores the stored
    leaves). Returns ids (b, H, Nq, Wn*NS), match and nL; with cfg.neighbors=False no leaf matches."""
    lv = _as_levels(getU1)
    return _ops.neighbor_pass(q, lv, st_leaf, st_score, st_ok, tq.to(q.device), cfg.nb_window, cfg.nb_store,
                              cfg.nb_rho, cfg.nb_probe, cfg.nb_cap_min, neighbors=cfg.neighbors)


def leaves_to_pos(ids, ok, leaf=2):
    """seg.py:106-108 (leaf positions, -1 where not ok)."""
    lhat = torch.zeros(ids.shape[:-1], dtype=torch.long, device=ids.device)
    return _ops.finish(ids, ok, lhat, 1, leaf)['tree_pos']


def finish(ids, vld, nid, match, nL, lhat, cfg):
    """seg.py:111-119."""
    return _ops.finish(ids, vld, lhat, cfg.wmax, getattr(cfg, 'leaf', 2), nid=nid, match=match, nL=nL)


def select_tree(q, k, cfg, gate_min=None):
    """Levels + descent for a whole sequence: returns (ids, vld, sct, Levels). With cfg.gate the descent runs on the
    gated levels (levels >= gate_min, default cfg.gate_min_level as fastseg.select_seg_fast; seg.select_seg gates
    every level) and those are returned."""
    if gate_min is None:
        gate_min = getattr(cfg, 'gate_min_level', 0)
    b, H, T, dh = q.shape
    Lm = _ops.lm_of(T)
    L0 = _leaf_level(cfg)
    if Lm < L0:
        raise ValueError('sequence length %d too short for leaf blocks of %d' % (T, 1 << L0))
    if cfg.gate:
        lv = gated_tree(k, T, L0, Lm, cfg.gate_q, gate_min)[2]
    else:
        lv = _ops.build_levels(k, T, L0, Lm, zero_sink=True)
    tq = torch.arange(T, device=q.device)
    ids, vld, sct = _ops.select(q, lv, tq, cfg.wmax)
    return ids, vld, sct, lv


@torch.no_grad()
def select_seg(q, k, lhat, cfg):
    """seg.py:122-140: key selection for a whole sequence (levels - every level gated with cfg.gate -, descent,
    neighbour pass, finish)."""
    b, H, T, dh = q.shape
    ids, vld, sct, lv = select_tree(q, k, cfg, gate_min=0)
    NS = cfg.nb_store
    tq = torch.arange(T, device=q.device)
    nid, match, nL = neighbor_pass(q, lv, ids[..., :NS], sct[..., :NS], vld[..., :NS], tq, cfg)
    return _ops.finish(ids, vld, lhat, cfg.wmax, 1 << lv.L0, nid=nid, match=match, nL=nL)
