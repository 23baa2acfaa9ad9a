"""TreeAttention (reference attention.py, attn='block'): causal block-tree sparse attention on the B200.

Every query attends to (1) its own block exactly (causal), (2) three static keys - the sink (position 0) and the
two previous tokens - when they lie in earlier blocks, and (3) the keys found by descending the content-sorted trees
of all EARLIER, completed blocks (attention.py:10-16). Here the trees are built by ta_lane_order + ta_forest_levels
(forest.build_forest_raw), the descent and the leaf -> key-position step are one kernel (ta_forest_select, a warp per
query), and the attention is the exact sparse attention (ta_sparse_attn, differentiable through ta_sparse_attn_bwd)
over the candidate list [own block (causal) | static keys | tree keys], -1 marking unused slots - the same keys and
the same softmax as the reference's concatenated scores. Training adds the learned budget head's loss and, with
cfg.route_weight > 0, the routing loss (attention.py:145-174).
"""
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, _ops
from .budget import budget_features, budget_label
from .fastseg import gather_dot, sparse_attn
from .forest import _ptr_array, build_forest_raw, gather_nodes


def _static_cands(T, B, dev):
    """(T, B + 3) int32: the own block's positions up to t (-1 after t) and the static keys 0, t-1, t-2 when they lie
    before t's block (-1 otherwise), attention.py:57-62 and 118-121."""
    t = torch.arange(T, device=dev)
    blk = t // B
    own = blk[:, None] * B + torch.arange(B, device=dev)[None, :]
    own = torch.where(own <= t[:, None], own, torch.full_like(own, -1))
    s_idx = torch.stack([torch.zeros_like(t), t - 1, t - 2], -1)
    s_valid = (s_idx >= 0) & (s_idx < (blk * B)[:, None])
    st = torch.where(s_valid, s_idx, torch.full_like(s_idx, -1))
    return torch.cat([own, st], -1).to(torch.int32), s_valid


class TreeAttention(nn.Module):
    """attention.py:10-176: same parameters (c_attn, c_proj, optional budget head), same selection and attention."""

    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        C = cfg.n_embd
        self.H = cfg.n_head
        self.dh = C // cfg.n_head
        assert cfg.seq_len % cfg.tree_block == 0
        assert cfg.tree_block >= 4 and (cfg.tree_block & (cfg.tree_block - 1)) == 0
        self.c_attn = nn.Linear(C, 3 * C, bias=False)
        self.c_proj = nn.Linear(C, C, bias=False)
        mask = torch.ones(1, 1, cfg.seq_len, 1)
        mask[:, :, 0, :] = 0  # the sink is left out of the trees (it is still always attended)
        self.register_buffer('idx_mask', mask, persistent=False)
        if cfg.beam_mode == 'pred':
            assert max(cfg.beam_classes) <= cfg.wmax
            fin = self.dh + 1 + self.H + (self.dh if cfg.global_pool else 0)
            self.pred = nn.Sequential(nn.Linear(fin, 64), nn.ReLU(), nn.Linear(64, len(cfg.beam_classes)))
            self.register_buffer('classes', torch.tensor(list(cfg.beam_classes)), persistent=False)
        self.aux = {}
        self._cands = {}

    def forward(self, x):
        b, T, C = x.shape
        q, k, v = self.c_attn(x).split(C, dim=2)
        q, k, v = [t.view(b, T, self.H, self.dh).transpose(1, 2) for t in (q, k, v)]
        out = self.sparse_attend(q, k, v)
        return self.c_proj(out.transpose(1, 2).reshape(b, T, C))

    def _static(self, T, B, dev):
        key = (T, B, str(dev))
        if key not in self._cands:
            self._cands[key] = _static_cands(T, B, dev)
        return self._cands[key]

    def _select(self, q, sums, perm, B, depth, bq, with_levels):
        """ta_forest_select: leaf ids / validity, key positions and their validity (not a static key), and, for the
        routing loss, every level's kept lists."""
        b, H, T, dh = q.shape
        dev = q.device
        nb = T // B
        w = min(self.cfg.wmax, nb)
        ws = [w]
        for _ in range(depth):
            w = min(self.cfg.wmax, 2 * w)
            ws.append(w)
        wl = ws[-1]
        leaf = torch.empty(b, H, T, wl, device=dev, dtype=torch.int64)
        leafv = torch.empty(b, H, T, wl, device=dev, dtype=torch.bool)
        tkey = torch.empty(b, H, T, 2 * wl, device=dev, dtype=torch.int64)
        tok = torch.empty(b, H, T, 2 * wl, device=dev, dtype=torch.bool)
        lv = _ptr_array([s.data_ptr() for s in sums])
        lsel = lselv = None
        sel_lists = None
        if with_levels:
            sel_lists = [(torch.empty(b, H, T, wi, device=dev, dtype=torch.int32),
                          torch.empty(b, H, T, wi, device=dev, dtype=torch.bool)) for wi in ws]
            lsel = _ptr_array([a.data_ptr() for a, _ in sel_lists])
            lselv = _ptr_array([a.data_ptr() for _, a in sel_lists])
        qs = q.stride()
        _lib.call('ta_forest_select', _ops._p(q), _ops._code(q), b, H, T, dh, qs[0], qs[1], qs[2], lv[0],
                  _ops._p(perm), B, depth, None, int(bq), int(self.cfg.wmax), _ops._p(leaf), _ops._p(leafv),
                  _ops._p(tkey), _ops._p(tok), lsel[0] if lsel else None, lselv[0] if lselv else None,
                  _ops._stream(q))
        return leaf, leafv, tkey, tok, sel_lists

    def sparse_attend(self, q, k, v):
        cfg = self.cfg
        b, H, T, dh = q.shape
        B = cfg.tree_block
        assert T % B == 0 and T <= cfg.seq_len
        _ops._need_cuda('TreeAttention', q, k, v)
        nb = T // B
        dev = q.device
        scale = 1.0 / math.sqrt(dh)
        t = torch.arange(T, device=dev)
        blk = t // B
        self.aux = {}
        static, s_valid = self._static(T, B, dev)
        if nb == 1:  # attention.py:64-66: the own block only
            cand = static[:, :B].view(1, 1, T, B).expand(b, H, T, B).contiguous()
            return sparse_attn(q, k, v, cand, scale)

        # (2) one content-sorted tree per block (the sink left out of the node sums), (3) the descent
        depth = int(round(math.log2(B // 2)))
        qd, kd = q.detach(), k.detach()
        perm, sums = build_forest_raw(kd, B, depth, cfg, zero_sink=True)
        pred_mode = cfg.beam_mode == 'pred'
        route_on = self.training and cfg.route_weight > 0
        leaf, leafv, tkey, tok, sel_lists = self._select(qd, sums, perm, B, depth,
                                                         cfg.wmax if pred_mode else cfg.beam, route_on)
        wl = leaf.shape[-1]

        # (4) the learned budget head (attention.py:92-108): a query keeps only its first `budget` valid leaves
        plog = None
        leafv_use = leafv
        if pred_mode:
            kmean = self._earlier_blocks_mean(sums[0], B, blk, qd.dtype) if cfg.global_pool else None
            plog = self.pred(budget_features(qd, kmean))
            budget = self.classes[plog.argmax(-1).detach()]
            leafv_use = leafv & (torch.arange(wl, device=dev) < budget.unsqueeze(-1))

        # (5)-(6) key positions of the used leaves, then exact attention over own block + static + tree keys
        tvalid = tok & torch.cat([leafv_use, leafv_use], -1)
        st = static.view(1, 1, T, B + 3).expand(b, H, T, B + 3)
        cand = torch.cat([st, torch.where(tvalid, tkey, torch.full_like(tkey, -1)).to(torch.int32)], -1).contiguous()
        out = sparse_attn(q, k, v, cand, scale)

        tcount = tvalid.sum(-1).float()
        self.aux['keys_tree'] = tcount[:, :, B:].mean().detach()
        self.aux['keys_total'] = ((t % B + 1).float().mean() + s_valid.float().sum(-1).mean()
                                  + tcount.mean()).detach()

        # (7) training signals (attention.py:145-174), both read off this layer's own attention weights
        if self.training:
            with torch.no_grad():
                target = self._leaf_targets(qd, kd, st, cand, tkey, tok, tvalid, leaf, blk, scale, pred_mode)
            route = q.new_zeros(()).float()
            leafnode, ok = target['leafnode'], target['ok']
            if route_on and bool(ok.any()):
                route = self._route_loss(q, k, perm, B, depth, sel_lists, leafnode, ok, blk)
            self.aux['route'] = route
            if pred_mode:
                rows = (blk >= 1).view(1, 1, T).expand(b, H, T)  # the first block has no earlier leaves
                self.aux['pred'] = F.cross_entropy(plog.float()[rows], target['budget'][rows])
        return out

    @staticmethod
    def _earlier_blocks_mean(roots, B, blk, dtype):
        """Global pooling input of the budget head: per query, the mean of the keys in the blocks before its own
        (zero in the first block). roots (b, H, nb, dh): each block's key sum (the level-0 node)."""
        nb = roots.shape[2]
        before = F.pad(roots.cumsum(2), (0, 0, 1, 0))[:, :, :nb]  # key sums of blocks 0 .. j-1
        n_keys = (torch.arange(nb, device=roots.device).clamp(min=1) * B).to(dtype).view(1, 1, nb, 1)
        return (before / n_keys)[:, :, blk, :]

    def _leaf_targets(self, qd, kd, st, cand, tkey, tok, tvalid, leaf, blk, scale, pred_mode):
        """Targets of the two training losses from the softmax weights of each query over its keys: the leaf whose
        key took the largest weight (the routing loss steers the descent toward its ancestors; `ok` marks the
        queries where that key is a used tree key with weight, in blocks >= 1) and, with the budget head, the
        budget class that covers 90 % of the weight on the leaves (budget.budget_label). In 'pred' mode the weights
        come from attention over every found leaf, not only the budgeted ones, so the label does not depend on the
        head's own choice."""
        T = qd.shape[2]
        wl = leaf.shape[-1]
        nb_static = st.shape[-1]
        if pred_mode:
            tree = torch.where(tok, tkey, torch.full_like(tkey, -1)).to(torch.int32)
            cand, counted = torch.cat([st, tree], -1).contiguous(), tok
        else:
            counted = tvalid
        s = gather_dot(qd, kd, cand, scale).masked_fill(cand < 0, float('-inf'))
        w_tree = torch.softmax(s, -1)[..., nb_static:]  # weights of the tree keys: [first keys | second keys]
        top = w_tree.argmax(-1)
        ok = counted.gather(-1, top.unsqueeze(-1)).squeeze(-1) & (w_tree.amax(-1) > 0) & (blk >= 1).view(1, 1, T)
        target = dict(ok=ok, leafnode=leaf.gather(-1, (top % wl).unsqueeze(-1)).squeeze(-1))
        if pred_mode:
            per_leaf = w_tree.unflatten(-1, (2, wl)).sum(-2)  # a block-forest leaf holds two keys
            target['budget'] = budget_label(per_leaf, self.classes)[0]
        return target

    def _route_loss(self, q, k, perm, B, depth, sel_lists, leafnode, ok, blk):
        """attention.py:162-174: per level, cross entropy of the scaled node scores toward the ancestor of the leaf
        that took the most attention. The node sums are formed here with autograd (the routing loss trains the keys
        through them) on the kernel's rank order and kept lists."""
        cfg = self.cfg
        b, H, T, dh = q.shape
        nb = T // B
        dev = q.device
        k_idx = k * self.idx_mask[:, :, :T].to(k.dtype)
        kp = k_idx.reshape(b * H * nb, B, dh).gather(1, perm.long().unsqueeze(-1).expand(-1, -1, dh))
        ar_nb = torch.arange(nb, device=dev)
        cur = ar_nb.view(1, 1, 1, nb).expand(b, H, T, nb)
        cv = (ar_nb[None, :] < blk[:, None]).view(1, 1, T, nb).expand(b, H, T, nb)
        terms = []
        for lvl in range(depth + 1):
            n_nodes = 1 << lvl
            grp = kp.reshape(b * H * nb, n_nodes, B // n_nodes, dh)
            sm = grp.sum(2)
            if cfg.gate:
                ml = torch.log(grp.float().abs() + 1e-6).mean(2)
                g = torch.sigmoid((ml - torch.quantile(ml, cfg.gate_q, dim=-1, keepdim=True)) / cfg.gate_temp)
                sm = (sm.float() * g * (dh / g.sum(-1, keepdim=True).clamp(min=1.0))).to(sm.dtype)
            S = sm.reshape(b, H, nb * n_nodes, dh)
            sc = torch.einsum('bhtd,bhtwd->bhtw', q, gather_nodes(S, cur.long())).masked_fill(~cv, float('-inf'))
            anc = leafnode >> (depth - lvl)
            match = (cur == anc.unsqueeze(-1)) & cv
            rows = ok & match.any(-1)
            if bool(rows.any()):
                size = B // (2 ** lvl)
                lg = (sc / (size * math.sqrt(dh))).float()[rows]
                terms.append(F.cross_entropy(lg, match.float().argmax(-1)[rows]))
            if lvl < depth:
                sel, selv = sel_lists[lvl]
                cur = torch.cat([2 * sel.long(), 2 * sel.long() + 1], -1)
                cv = torch.cat([selv, selv], -1)
        return torch.stack(terms).mean() if terms else q.new_zeros(()).float()
