"""Segment-tree sparse attention on B200 (reference fastseg.py): the SegAttention module and the kernels it uses.

Names and signatures follow the reference module. Every function runs a hand-written sm_100a kernel through
the C ABI; there is no Triton and no PyTorch fallback (CPU tensors are rejected, a missing library raises).
"""
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, _ops
from .budget import budget_features, budget_label, mean_before
from .seg import finish, gate_apply, neighbor_pass, select_seg, select_tree, tree_pass  # noqa: F401

FAST = [True]  # kept for callers that toggle it; this package has only the CUDA path


def fast_available():
    """True when the CUDA library is built and a GPU is present (reference fastseg.py:180-223 ran a kernel
    self-check with a silent fallback; here a failure raises instead)."""
    if not torch.cuda.is_available():
        return False
    _lib.load()
    return True


# ------------------------------------------------------------------ scores of queries against gathered nodes
def gather_dot(q, S, cand, scale):
    """q (b,H,N,dh), S (b,H,M,dh), cand (b,H,N,C) node ids -> (b,H,N,C) float32 = scale * q . S[cand]."""
    return _ops.gather_dot(q, S, cand, scale)


# ------------------------------------------------------------------ attention over the selected keys
class _SparseAttnFn(torch.autograd.Function):
    """fastseg.py:143-170: forward saves q, k, v, cand, o and the log-sum-exp; backward recomputes the softmax
    weights from them (ta_sparse_attn_bwd)."""

    @staticmethod
    def forward(ctx, q, k, v, cand, scale):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        o, lse = _ops.sparse_attn_fwd(q, k, v, cand, scale)
        ctx.save_for_backward(q, k, v, cand, o, lse)
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, cand, o, lse = ctx.saved_tensors
        dq, dk, dv = _ops.sparse_attn_bwd(q, k, v, cand, o, lse, do, ctx.scale)
        return dq, dk, dv, None, None


def sparse_attn(q, k, v, cand, scale):
    """cand: (b,H,T,K) int, -1 = unused slot. Exact softmax attention over the used keys; differentiable in q, k
    and v (fastseg.py:173-177)."""
    return _SparseAttnFn.apply(q, k, v, cand, scale)


# ------------------------------------------------------------------ duplicate removal
def dedupe_fast(cand, valid):
    """Keep the first valid copy of every key position (same result as attention_dyn.dedupe)."""
    return _ops.dedupe(cand, valid)


# ------------------------------------------------------------------ key selection (same logic as seg.select_seg)
@torch.no_grad()
def level_sums_min(kidx, Lm, gate, gate_q, gate_min):
    """fastseg.py:238-251: level sums of kidx (sink already zeroed), mean-log gated at levels >= gate_min."""
    from .seg import gated_tree, level_sums
    if not gate:
        return level_sums(kidx, Lm, False, gate_q)
    T = kidx.shape[2]
    return gated_tree(kidx, T, 1, Lm, gate_q, gate_min, zero_sink=False)[2].as_dict()


@torch.no_grad()
def tree_pass_fast(q, S, tq, Lm, wmax):
    return tree_pass(q, S, tq, Lm, wmax)


@torch.no_grad()
def neighbor_pass_fast(q, S1, st_leaf, st_score, st_ok, tq, cfg):
    return neighbor_pass(q, S1, st_leaf, st_score, st_ok, tq, cfg)


@torch.no_grad()
def select_seg_fast(q, k, lhat, cfg):
    """fastseg.py:302-314: select_seg with the gate applied from cfg.gate_min_level up."""
    b, H, T, dh = q.shape
    ids, vld, sct, lv = select_tree(q, k, cfg)
    NS = cfg.nb_store
    tq = torch.arange(T, device=q.device)
    nid, match, nL = neighbor_pass(q, lv, ids[..., :NS], sct[..., :NS], vld[..., :NS], tq, cfg)
    return _ops.finish(ids, vld, lhat, cfg.wmax, 1 << lv.L0, nid=nid, match=match, nL=nL)


def n_tree_fixed(beam, wmax):
    """seg.finish with no neighbour matches and a fixed budget: min(max(beam, 2), wmax) (0 for beam <= 0)."""
    return 0 if beam <= 0 else min(max(beam, 2), wmax)


# ------------------------------------------------------------------ the module
class SegAttention(nn.Module):
    """Reference fastseg.py:318-405: same parameters (c_attn, c_proj, optional pred head), same math.

    Per layer: node sums of the keys (fp32, bit-exact), the past-only top-k descent, then exact attention over
    the used leaf blocks + the sink + the local window, each position once. The attention output is written
    straight into the (b, T, H, dh) layout that c_proj consumes."""

    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        C = cfg.n_embd
        self.H = cfg.n_head
        self.dh = C // cfg.n_head
        assert cfg.seq_len % cfg.chunk == 0 and (cfg.seq_len & (cfg.seq_len - 1)) == 0
        self.c_attn = nn.Linear(C, 3 * C, bias=False)
        self.c_proj = nn.Linear(C, C, bias=False)
        if cfg.beam_mode == 'pred':
            assert max(cfg.beam_classes) <= cfg.wmax
            fin = self.dh + 1 + self.H + (self.dh if cfg.global_pool else 0)
            self.pred = nn.Sequential(nn.Linear(fin, 64), nn.ReLU(), nn.Linear(64, len(cfg.beam_classes)))
            self.register_buffer('classes', torch.tensor(list(cfg.beam_classes)), persistent=False)
        self.aux = {}

    def forward(self, x):
        b, T, C = x.shape
        q, k, v = self.c_attn(x).split(C, dim=2)
        q, k, v = [t.view(b, T, self.H, self.dh).transpose(1, 2) for t in (q, k, v)]
        if self._needs_grad(q, k, v):
            out = self.sparse_attend(q, k, v)
            return self.c_proj(out.transpose(1, 2).reshape(b, T, C))
        out = torch.empty(b, T, self.H, self.dh, device=x.device, dtype=q.dtype)
        self.sparse_attend(q, k, v, out=out.transpose(1, 2))
        return self.c_proj(out.view(b, T, C))

    @staticmethod
    def _needs_grad(q, k, v):
        return torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v))

    def _lhat(self, q, k, with_logits=False):
        """Leaf budget per query from the budget head (beam_mode 'pred', fastseg.py:352-365), or None."""
        if self.cfg.beam_mode != 'pred':
            return (None, None) if with_logits else None
        qd = q.detach()
        kmean = mean_before(k.detach().float(), 2).to(qd.dtype) if self.cfg.global_pool else None
        plog = self.pred(budget_features(qd, kmean))
        lhat = self.classes[plog.argmax(-1).detach()]
        return (lhat, plog) if with_logits else lhat

    def sparse_attend(self, q, k, v, out=None):
        cfg = self.cfg
        if self._needs_grad(q, k, v):
            o = self._sparse_attend_autograd(q, k, v)
            if out is not None:
                out.copy_(o)
                return out
            return o
        b, H, T, dh = q.shape
        scale = 1.0 / math.sqrt(dh)
        self.aux = {}
        with torch.no_grad():
            lhat = self._lhat(q, k)
            ids, vld, sct, lv = select_tree(q.detach(), k.detach(), cfg)
            leaf = 1 << lv.L0
            wl = ids.shape[-1]
            Lw = max(cfg.local, 3)
            tq = torch.arange(T, device=q.device)
            keys_nb = torch.zeros((), device=q.device)
            nb_leaves = torch.zeros((), device=q.device)
            if cfg.neighbors:
                # neighbour borrowing (fastseg.py:359-366): matched leaves of earlier queries join the tree's
                # first n_tree leaves; a leaf held by both counts once (dedupe over leaf ids)
                NS = cfg.nb_store
                nid, match, nL = neighbor_pass(q.detach(), lv, ids[..., :NS], sct[..., :NS], vld[..., :NS], tq,
                                               cfg)
                if lhat is None:
                    lhat = torch.full((b, H, T), cfg.beam, dtype=torch.long, device=q.device)
                n_tree = _ops.finish(ids, vld, lhat, cfg.wmax, leaf, nid=nid, match=match, nL=nL,
                                     positions=False)['n_tree']
                used = vld & (torch.arange(wl, device=q.device) < n_tree.unsqueeze(-1))
                leaves = torch.cat([ids, nid], -1)
                keep = _ops.dedupe(leaves, torch.cat([used, match], -1))
                out, _, nkeys = _ops.attend_leaves(q, k, v, tq, leaves, keep, leaves.shape[-1], leaf, Lw, scale,
                                                   out=out)
                keys_nb = (keep[..., wl:].sum(-1).float() * leaf).mean()
                nb_leaves = nL.float().mean()
            else:
                if lhat is None:
                    n_tree = n_tree_fixed(cfg.beam, cfg.wmax)
                    used = vld & (torch.arange(wl, device=q.device) < n_tree)
                else:
                    n_tree = _ops.finish(ids, vld, lhat, cfg.wmax, leaf, positions=False)['n_tree']
                    used = vld & (torch.arange(wl, device=q.device) < n_tree.unsqueeze(-1))
                out, _, nkeys = _ops.attend_leaves(q, k, v, tq, ids, vld, n_tree, leaf, Lw, scale, out=out)
            n_used = used.sum(-1).float()
            self.aux['keys_total'] = nkeys.float().mean()
            self.aux['keys_tree'] = (n_used * leaf).mean()
            self.aux['keys_nb'] = keys_nb
            self.aux['nb_leaves'] = nb_leaves
            self.aux['leaves_used'] = n_used.mean()
        return out

    def _select(self, q, k, lhat):
        """The non-differentiable key selection of the training form (the segment tree's)."""
        return select_seg_fast(q, k, lhat, self.cfg)

    def _sparse_attend_autograd(self, q, k, v):
        """The training form (fastseg.py:345-405 as the reference runs it): selection without gradients, the
        explicit candidate list [tree positions, neighbour positions, static keys] deduplicated, then the
        differentiable sparse_attn (ta_sparse_attn / ta_sparse_attn_bwd); in training mode with the learned budget
        head also its classification loss in aux['pred']."""
        cfg = self.cfg
        b, H, T, dh = q.shape
        dev = q.device
        scale = 1.0 / math.sqrt(dh)
        t = torch.arange(T, device=dev)
        self.aux = {}
        lhat, plog = self._lhat(q, k, with_logits=True)
        if lhat is None:
            lhat = torch.full((b, H, T), cfg.beam, dtype=torch.long, device=dev)
        with torch.no_grad():
            sel = self._select(q.detach(), k.detach(), lhat)
            tree_pos, nb_pos, leaf_ok = sel['tree_pos'], sel['nb_pos'], sel['leaf_ok']
            wl = leaf_ok.shape[-1]
            leaf = tree_pos.shape[-1] // max(wl, 1)
            NBK = nb_pos.shape[-1]
            Lw = max(cfg.local, 3)
            st = torch.cat([torch.zeros(T, 1, dtype=torch.long, device=dev),
                            t.unsqueeze(1) - torch.arange(Lw, device=dev).unsqueeze(0)], 1)
            st = st.masked_fill(st < 0, -1).view(1, 1, T, 1 + Lw).expand(b, H, T, 1 + Lw)
            cand = torch.cat([tree_pos, nb_pos, st], -1)
            used = leaf_ok & (torch.arange(wl, device=dev) < sel['n_tree'].unsqueeze(-1))
            tv_used = torch.cat([used] * leaf, -1) & (tree_pos >= 0)
            rest = torch.cat([nb_pos >= 0, st >= 0], -1)
            keep = dedupe_fast(cand, torch.cat([tv_used, rest], -1))
            cand_k = torch.where(keep, cand, torch.full_like(cand, -1)).to(torch.int32)
        out = sparse_attn(q, k, v, cand_k, scale)
        self.aux['keys_total'] = keep.sum(-1).float().mean()
        self.aux['keys_tree'] = keep[..., :leaf * wl].sum(-1).float().mean()
        self.aux['keys_nb'] = keep[..., leaf * wl:leaf * wl + NBK].sum(-1).float().mean()
        self.aux['nb_leaves'] = sel['nb_leaves'].float().mean()
        self.aux['leaves_used'] = used.sum(-1).float().mean()
        if self.training and plog is not None:
            with torch.no_grad():
                label, rows = self._budget_target(q.detach(), k.detach(), cand, tree_pos, leaf_ok, rest, leaf, scale)
            if bool(rows.any()):
                self.aux['pred'] = F.cross_entropy(plog.float()[rows], label[rows])
        return out

    def _budget_target(self, qd, kd, cand, tree_pos, leaf_ok, rest, leaf, scale):
        """Budget-head target (fastseg.py:394-405): the attention weights a query would give ALL of its found leaves
        (every valid one, not only the budgeted), summed per leaf block, through budget.budget_label. Returns
        (label, rows): rows are the queries whose leaves take any weight."""
        wl = leaf_ok.shape[-1]
        every_leaf = torch.cat([leaf_ok] * leaf, -1) & (tree_pos >= 0)
        keep = dedupe_fast(cand, torch.cat([every_leaf, rest], -1))
        s = gather_dot(qd, kd, cand, scale).masked_fill(~keep, float('-inf'))
        w_leaf_keys = torch.softmax(s, -1)[..., :leaf * wl]  # slot j * wl + i: key j of leaf i
        per_leaf = w_leaf_keys[..., :wl]
        for j in range(1, leaf):
            per_leaf = per_leaf + w_leaf_keys[..., j * wl:(j + 1) * wl]
        return budget_label(per_leaf, self.classes)
