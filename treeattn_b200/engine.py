"""KV-cache decoding with the segment tree (reference engine.py), batched and on B200 kernels.

Reference engine.py is batch 1, fp32, one Python loop over layers and tree levels with a host sync per layer.
Here a SegState holds a whole batch (B, H, cap, dh) of keys/values (fp32 or bf16/fp16) plus the packed tree
levels >= the leaf level; one decode step of one layer is ONE fused kernel (ta_decode_step: descent, exact
attention over used leaves + sink + window + the new token, append, incremental tree update), and the whole
model step is captured in a CUDA graph. `keys` results are device tensors (no host sync per layer).
"""
import math

import torch
import torch.nn.functional as F

from . import _ops
from ._ops import Levels
from .budget import budget_features, mean_before
from .fastseg import n_tree_fixed
from .forest import gather_nodes


def _ln(x, w):
    return F.layer_norm(x, (x.shape[-1],), w, None, 1e-5)


def _positions(t, B, device):
    if torch.is_tensor(t):
        return t.to(device=device, dtype=torch.int32).expand(B).contiguous()
    return torch.full((B,), int(t), device=device, dtype=torch.int32)


FUSED_LINEAR_MAX_BATCH = 32  # Decoder's default: projections on ta_linear_rows up to this many sequences


def _pick_splits(N, K, target=36, min_k=128):
    """K splits of an (N, K) projection for ta_linear_rows: the fewest that give `target` CTAs (N / 128 feature
    tiles each) with slices of at least min_k, a whole number of 64-wide blocks each."""
    tiles, blocks = -(-N // _ops.LIN_TILE), K // 64
    best = 1
    for sp in range(1, blocks + 1):
        if blocks % sp or (K // sp) < min_k:
            continue
        best = sp
        if tiles * sp >= target:
            break
    return best


class SegState:
    """Per-layer cache for a batch of sequences: keys, values and the tree levels L0..Lm (reference
    engine.py:18-71; a node is formed the moment its last position is added).

    Tcap sets the tree height (Lm = round(log2 Tcap) - 1, as the reference); `cap` (default Tcap) is the number
    of positions actually allocated, so a 4352-token context with Tcap 8192 does not pay for 8192 rows."""

    def __init__(self, cfg, Tcap, H, dh, dev, batch=1, dtype=torch.float32, cap=None):
        self.cfg, self.Tcap, self.H, self.dh = cfg, Tcap, H, dh
        self.Lm = _ops.lm_of(Tcap)
        self.L0 = _ops.log2_exact(getattr(cfg, 'leaf', 2), 'cfg.leaf')
        self.cap = int(cap or Tcap)
        self.batch = batch
        dev = torch.device(dev)
        self.K = torch.zeros(batch, H, self.cap, dh, device=dev, dtype=dtype)
        self.V = torch.zeros(batch, H, self.cap, dh, device=dev, dtype=dtype)
        self.levels = Levels.empty(batch, H, dh, self.cap, self.L0, self.Lm, dev)
        if cfg.gate:  # the log-magnitude tree and the gated nodes the descent scores (engine.py:26-27, 33-37)
            self.lg = Levels.empty(batch, H, dh, self.cap, self.L0, self.Lm, dev)
            self.gated = Levels.empty(batch, H, dh, self.cap, self.L0, self.Lm, dev)
        if cfg.neighbors:  # the best leaves every position found, for neighbour borrowing (engine.py:28-31)
            NS = cfg.nb_store
            self.st_leaf = torch.zeros(batch, H, self.cap, NS, device=dev, dtype=torch.int64)
            self.st_score = torch.zeros(batch, H, self.cap, NS, device=dev, dtype=torch.float32)
            self.st_ok = torch.zeros(batch, H, self.cap, NS, device=dev, dtype=torch.bool)
        self.ksum = torch.zeros(batch, H, dh, device=dev, dtype=torch.float32)  # sum of the keys added so far

    @property
    def raw(self):
        """{level: (B, H, cap >> l, dh)} views of the stored levels (reference SegState.raw, levels >= L0)."""
        return self.levels.as_dict()

    @property
    def sel_levels(self):
        """The tree the descent scores: the gated nodes with cfg.gate, else the sums themselves."""
        return self.gated if self.cfg.gate else self.levels

    def getU(self, l, cand):
        return gather_nodes(self.sel_levels.level(l), cand)

    def add(self, t, k, v):
        """k, v: (B, H, dh) (or (B, H, 1, dh)) for position t (int or (B,) tensor)."""
        if k.dim() == 4:
            k, v = k[:, :, 0], v[:, :, 0]
        pos = _positions(t, self.batch, self.K.device)
        _ops.append(k.to(self.K.dtype), v.to(self.V.dtype), self.K, self.V, self.levels, pos)
        if self.cfg.gate:
            _ops.gate_append(self.K, self.levels, self.lg, self.gated, pos, self.cfg.gate_q,
                             getattr(self.cfg, 'gate_min_level', 0))
        self.ksum += k.float()

    def fill(self, K, V):
        """Load positions [0, T) at once (K, V: (B, H, T, dh)) and build the levels (reference fill)."""
        T = K.shape[2]
        if T > self.cap:
            raise ValueError('fill: %d positions above capacity %d' % (T, self.cap))
        self.K[:, :, :T].copy_(K)
        self.V[:, :, :T].copy_(V)
        _ops.build_levels(self.K[:, :, :T], self.cap, self.L0, self.Lm, zero_sink=True, out=self.levels)
        if self.cfg.gate:
            _ops.build_log_levels(self.K[:, :, :T], self.cap, self.L0, self.Lm, zero_sink=True, out=self.lg)
            _ops.gate_levels(self.levels, self.lg, self.cfg.gate_q, getattr(self.cfg, 'gate_min_level', 0), T,
                             out=self.gated)
        self.ksum.copy_(K.float().sum(2))


def pred_budget(pw, q, kmean, H):
    """The learned leaf budget (engine.py:89-94, fastseg.py:352-365): features [q, log |q|, one-hot head] (+ the
    mean of the earlier keys with cfg.global_pool) through the two-layer head, argmax over the budget classes.
    q (B, H, N, dh); kmean (B, H, N, dh) or None. Returns (B, H, N) int64 leaf budgets."""
    feats = budget_features(q.float(), None if kmean is None else kmean.float())
    h = F.relu(F.linear(feats, pw['w1'].float(), pw['b1'].float()))
    lg = F.linear(h, pw['w2'].float(), pw['b2'].float())
    return pw['classes'][lg.argmax(-1)]


def _general_step(state, pw, q, k, v, pos, out=None, update=True):
    """One decoding step with the general selection (engine.py:84-120): learned budget (beam_mode='pred') and
    neighbour borrowing (cfg.neighbors) - descent, neighbour pass and budget on the tree before position t,
    this position's best leaves stored for the following ones, then append and exact attention over the used tree
    leaves, the matched borrowed ones (deduplicated), the sink and the window. q, k, v (B, H, 1, dh) in the cache
    dtype, pos (B,) int32. update=False selects and attends without storing or appending (the cache must then
    already hold position t). Returns (out (B, H, 1, dh), keys (B, H, 1) int32)."""
    cfg = state.cfg
    B, H, _, dh = q.shape
    leaf = 1 << state.L0
    tq = pos.to(torch.int64)
    if cfg.beam_mode == 'pred':
        kmean = (state.ksum / tq.clamp(min=1).view(B, 1, 1).float()).unsqueeze(2) if cfg.global_pool else None
        lhat = pred_budget(pw, q, kmean, H)
    else:
        lhat = torch.full((B, H, 1), cfg.beam, device=q.device, dtype=torch.int64)
    ids, vld, sct = _ops.select(q, state.sel_levels, tq, cfg.wmax)
    wl = ids.shape[-1]
    if cfg.neighbors:
        NS = cfg.nb_store
        nid, match, nL = _ops.neighbor_pass(q, state.sel_levels, state.st_leaf, state.st_score, state.st_ok, tq,
                                            cfg.nb_window, NS, cfg.nb_rho, cfg.nb_probe, cfg.nb_cap_min)
        n_tree = _ops.finish(ids, vld, lhat, cfg.wmax, leaf, nid=nid, match=match, nL=nL, positions=False)['n_tree']
        if update:
            bi = torch.arange(B, device=q.device)
            state.st_leaf[bi, :, tq] = ids[:, :, 0, :NS]
            state.st_score[bi, :, tq] = sct[:, :, 0, :NS]
            state.st_ok[bi, :, tq] = vld[:, :, 0, :NS]
    else:
        n_tree = _ops.finish(ids, vld, lhat, cfg.wmax, leaf, positions=False)['n_tree']
    if update:
        state.add(pos, k, v)
    used = vld & (torch.arange(wl, device=q.device) < n_tree.unsqueeze(-1))
    if cfg.neighbors:
        leaves = torch.cat([ids, nid], -1)
        keep = _ops.dedupe(leaves, torch.cat([used, match], -1))
    else:
        leaves, keep = ids, used
    o, _, nkeys = _ops.seg_attn(q, state.K, state.V, tq, leaves, keep, leaves.shape[-1], leaf, max(cfg.local, 3),
                                1.0 / math.sqrt(dh), out=out)
    return o, nkeys


@torch.no_grad()
def seg_attend(state, pw, q, k, v, t, update=True):
    """One decoding step of segment-tree attention for a batch. q, k, v: (B, H, 1, dh). Returns (out (B, H, 1,
    dh), keys read per head as a 0-d device tensor)."""
    cfg = state.cfg
    B, H, _, dh = q.shape
    pos = _positions(t, B, q.device)
    qx = q.to(state.K.dtype)
    kx, vx = [None if t_ is None else t_.to(state.K.dtype) for t_ in (k, v)]  # k / v unused when update=False
    if cfg.neighbors or cfg.beam_mode == 'pred' or cfg.gate:
        out, nkeys = _general_step(state, pw, qx, kx, vx, pos, update=update)
        return out, nkeys.float().mean()
    if update:
        state.add(pos, k, v)
    ids, vld, _ = _ops.select(qx, state.levels, pos.to(torch.int64), cfg.wmax)
    n_tree = n_tree_fixed(cfg.beam, cfg.wmax)
    out, _, nkeys = _ops.seg_attn(qx, state.K, state.V, pos.to(torch.int64), ids, vld, n_tree,
                                  1 << state.L0, max(cfg.local, 3), 1.0 / math.sqrt(dh))
    return out, nkeys.float().mean()


def weights_from_ours(sd, cfg):
    """engine.py:123-134: a GPT state dict -> the decoder's weight dict."""
    W = dict(wte=sd['wte.weight'], wpe=sd['wpe.weight'], ln_f=sd['ln_f.weight'], layers=[])
    for i in range(cfg.n_layer):
        p = 'blocks.%d.' % i
        L = dict(ln1=sd[p + 'ln1.weight'], c_attn=sd[p + 'attn.c_attn.weight'], c_proj=sd[p + 'attn.c_proj.weight'],
                 ln2=sd[p + 'ln2.weight'], c_fc=sd[p + 'mlp.c_fc.weight'], c_mlp=sd[p + 'mlp.c_proj.weight'])
        if cfg.beam_mode == 'pred':
            L['pw'] = dict(w1=sd[p + 'attn.pred.0.weight'], b1=sd[p + 'attn.pred.0.bias'],
                           w2=sd[p + 'attn.pred.2.weight'], b2=sd[p + 'attn.pred.2.bias'],
                           classes=torch.tensor(list(cfg.beam_classes), device=sd['wte.weight'].device))
        W['layers'].append(L)
    return W


def weights_from_nanogpt(sd, n_layer):
    """engine.py:137-146: a nanoGPT state dict -> the decoder's weight dict."""
    sd = {k.replace('_orig_mod.', ''): v for k, v in sd.items()}
    W = dict(wte=sd['transformer.wte.weight'], wpe=sd['transformer.wpe.weight'],
             ln_f=sd['transformer.ln_f.weight'], layers=[])
    for i in range(n_layer):
        p = 'transformer.h.%d.' % i
        W['layers'].append(dict(ln1=sd[p + 'ln_1.weight'], c_attn=sd[p + 'attn.c_attn.weight'],
                                c_proj=sd[p + 'attn.c_proj.weight'], ln2=sd[p + 'ln_2.weight'],
                                c_fc=sd[p + 'mlp.c_fc.weight'], c_mlp=sd[p + 'mlp.c_proj.weight']))
    return W


class DenseCache:
    """engine.py:74-81 DenseState, batched: the key/value cache of one layer for the dense baseline decoder
    ('dense' mode, nanoGPT weights); a step writes k, v at every sequence's position and attends over its prefix
    (torch's scaled-dot-product attention over the whole cache, later positions masked)."""

    def __init__(self, B, H, cap, dh, dev, dtype):
        self.K = torch.zeros(B, H, cap, dh, device=dev, dtype=dtype)
        self.V = torch.zeros(B, H, cap, dh, device=dev, dtype=dtype)
        self.ar = torch.arange(cap, device=dev)
        self.ksum = torch.zeros(1, device=dev)

    def attend(self, qkv, pos, out, nkeys):
        B, H, cap, dh = self.K.shape
        C = H * dh
        q, k, v = [qkv[:, j * C:(j + 1) * C].view(B, H, 1, dh) for j in range(3)]
        idx = pos.long().view(B, 1, 1, 1).expand(B, H, 1, dh)
        self.K.scatter_(2, idx, k)
        self.V.scatter_(2, idx, v)
        mask = (self.ar.view(1, 1, 1, cap) <= pos.view(B, 1, 1, 1))
        o = F.scaled_dot_product_attention(q, self.K, self.V, attn_mask=mask)
        out.view(B, H, 1, dh).copy_(o)
        nkeys.copy_((pos + 1).view(B, 1).expand(B, H))


class Decoder:
    """Token-by-token decoding for a batch of sequences (reference engine.py:149-177): mode 'seg' (the segment-tree
    attention) or 'dense' (ordinary attention over the whole prefix, the nanoGPT baseline; weights_from_nanogpt).

    Decoder(W, n_layer, n_head, n_embd, Tcap, 'seg', cfg, dev) keeps the reference's arguments; `batch`, `dtype`
    (weights / cache precision, default: the weights' dtype), `cap` (allocated positions) and `graphs` are
    additions. The residual stream is kept in fp32; matmuls run in `dtype` on cuBLAS."""

    def __init__(self, W, n_layer, n_head, n_embd, Tcap, mode='seg', cfg=None, dev='cuda', batch=1, dtype=None,
                 cap=None, graphs=True, splits=0, fused_linear=None, block_tail=None):
        if mode not in ('seg', 'dense'):
            raise NotImplementedError("Decoder mode '%s' is not implemented in treeattn_b200 ('seg', 'dense')" % mode)
        if mode == 'seg' and cfg is None:
            raise ValueError("mode 'seg' needs cfg")
        self.dev = torch.device(dev)
        self.dtype = dtype or W['wte'].dtype
        cast = lambda t: t.to(device=self.dev, dtype=self.dtype).contiguous()
        self.W = dict(wte=cast(W['wte']), wpe=cast(W['wpe']), ln_f=W['ln_f'].to(self.dev, torch.float32),
                      layers=[dict(ln1=L['ln1'].to(self.dev, torch.float32), c_attn=cast(L['c_attn']),
                                   c_proj=cast(L['c_proj']), ln2=L['ln2'].to(self.dev, torch.float32),
                                   c_fc=cast(L['c_fc']), c_mlp=cast(L['c_mlp'])) for L in W['layers'][:n_layer]])
        # general selection (learned budget, neighbour borrowing): per layer the separate kernels of
        # _general_step instead of the single fused decode kernel
        seg = mode == 'seg'
        self.general = seg and (cfg.neighbors or cfg.beam_mode == 'pred' or cfg.gate)
        if seg and cfg.beam_mode == 'pred':
            for Ld, L in zip(self.W['layers'], W['layers'][:n_layer]):
                Ld['pw'] = {k_: (t.to(self.dev) if torch.is_tensor(t) else t) for k_, t in L['pw'].items()}
        self.nl, self.H, self.C, self.Tcap = n_layer, n_head, n_embd, Tcap
        self.dh, self.mode, self.cfg = n_embd // n_head, mode, cfg
        self.batch = batch
        self.cap = int(cap or Tcap)
        self.wmax = cfg.wmax if seg else 0
        self.n_tree = n_tree_fixed(cfg.beam, cfg.wmax) if seg else 0
        self.Lw = max(cfg.local, 3) if seg else 0
        self.scale = 1.0 / math.sqrt(self.dh)
        self.use_graphs = graphs
        self.splits = (splits or _ops.default_splits(batch, n_head, self.dh, self.dtype)) if seg else 0
        # fused_linear=True: the linear layers on the library's tensor-core kernel (ta_linear_rows: 16-bit weights,
        # K slices of 64) instead of torch matmuls; K splits of c_proj and c_mlp so that enough CTAs stream their
        # weights. Default (None): on for batches of at most FUSED_LINEAR_MAX_BATCH sequences, where cuBLAS's small-row
        # GEMMs are slowest (whole configuration-4 steps: 8 sequences 0.652 -> 0.590 ms, 16: 0.658 -> 0.567 ms, 32:
        # 0.789 -> 0.724 ms); off above (64 sequences: 0.948 ms with it against 0.937 on cuBLAS).
        V = self.W['wte'].shape[0]
        C = n_embd
        # per projection: K splits on ta_linear_rows, or 0 = torch's matmul (cuBLAS) where that measured faster
        # (configuration 4, whole steps: c_fc with its GELU, c_proj and c_mlp here, c_attn and the lm_head on cuBLAS)
        self.lin_splits = dict(qkv=0, proj=_pick_splits(C, C), fc=1, mlp=_pick_splits(C, 4 * C, target=96), lm=0)
        shapes = dict(qkv=(3 * C, C), proj=(C, C), fc=(4 * C, C), mlp=(C, 4 * C), lm=(V, C))
        ok = all(sp == 0 or _ops.linear_supported(self.dtype, batch, shapes[k][0], shapes[k][1], sp)
                 for k, sp in self.lin_splits.items())
        if fused_linear is None:
            self.fused_linear = ok and batch <= FUSED_LINEAR_MAX_BATCH and self.dev.type == 'cuda'
        else:
            self.fused_linear = bool(fused_linear)
        if self.fused_linear and not ok:
            raise ValueError('fused_linear: ta_linear_rows does not take this model (16-bit weights, width and '
                             'batch it supports)')
        # block_tail=True: per layer, everything after the attention and the next layer's c_attn in one launch
        # (ta_block_tail) instead of four matmuls and three row kernels
        plans = [_ops.block_tail_plan(self.dtype, batch, C, q) for q in (True, False)]
        tail_ok = self.dev.type == 'cuda' and all(pl is not None for pl in plans)
        self.block_tail = False if block_tail is None else bool(block_tail)
        if self.block_tail and not tail_ok:
            raise ValueError('block_tail: ta_block_tail does not take this model (16-bit weights, width a multiple '
                             'of 128, at most 128 sequences)')
        self._tail_plans = plans
        self.reset()

    @classmethod
    def from_checkpoint(cls, path, Tcap, dev='cuda', **kw):
        """A Decoder (mode 'seg') over a checkpoint written by the reference's training scripts
        ({'model': state_dict, 'cfg': Config.to_dict()}, train.py:144), through weights_from_ours (engine.py:123-134)."""
        from .config import Config
        ck = torch.load(path, map_location='cpu', weights_only=True)
        cfg = Config(**ck['cfg'])
        return cls(weights_from_ours(ck['model'], cfg), cfg.n_layer, cfg.n_head, cfg.n_embd, Tcap, 'seg', cfg, dev, **kw)

    # -------------------------------------------------------------- state
    def reset(self):
        B, C, dev = self.batch, self.C, self.dev
        if self.mode == 'seg':
            self.states = [SegState(self.cfg, self.Tcap, self.H, self.dh, dev, B, self.dtype, self.cap)
                           for _ in range(self.nl)]
        else:
            self.states = [DenseCache(B, self.H, self.cap, self.dh, dev, self.dtype) for _ in range(self.nl)]
        self._tok = torch.zeros(B, device=dev, dtype=torch.int64)
        self._pos = torch.zeros(B, device=dev, dtype=torch.int32)
        dt = self.dtype
        self._x = torch.empty(B, C, device=dev, dtype=torch.float32)   # residual stream (fp32)
        self._h = torch.empty(B, C, device=dev, dtype=dt)               # layer-norm output
        self._qkv = torch.empty(B, 3 * C, device=dev, dtype=dt)
        self._att = torch.empty(B, C, device=dev, dtype=dt)
        self._proj = torch.empty(B, C, device=dev, dtype=dt)
        self._fc = torch.empty(B, 4 * C, device=dev, dtype=dt)
        self._mlp = torch.empty(B, C, device=dev, dtype=dt)
        self._logits = torch.empty(B, self.W['wte'].shape[0], device=dev, dtype=dt)
        self._nkeys = torch.zeros(self.nl, B, self.H, device=dev, dtype=torch.int32)
        # partial-state scratch that lets the decode kernel cut items into parts when whole items would leave SMs
        # idle (shared by the layers: their launches run in order on one stream)
        self._split = _ops.split_scratch(B, self.H, self.dh, dev) if self.mode == 'seg' else None
        if self.fused_linear:  # K-split sums of c_proj / c_mlp, the lm_head's per-tile argmax keys, split workspace
            ls = self.lin_splits
            self._part = torch.empty(max(ls['proj'], ls['mlp'], 1), B, C, device=dev, dtype=torch.float32)
            V = self.W['wte'].shape[0]
            self._keys = torch.zeros(-(-V // _ops.LIN_TILE), B, device=dev, dtype=torch.int64)
            n_ws = max([ls[k] * -(-N // _ops.LIN_TILE) for k, N in (('qkv', 3 * C), ('fc', 4 * C), ('lm', V))
                        if ls[k] > 1] + [1])
            self._ws = (torch.empty(n_ws * B * _ops.LIN_TILE, device=dev, dtype=torch.float32),
                        torch.zeros(-(-V // _ops.LIN_TILE), device=dev, dtype=torch.int32))
        if self.block_tail:  # one workspace and one set of sync words, shared by the layers' launches (in order)
            self._tail_bufs = (torch.empty(max(pl[0] for pl in self._tail_plans), device=dev, dtype=torch.uint8),
                               torch.zeros(self._tail_plans[0][1], device=dev, dtype=torch.int32))
        self._graph = None
        self._graph_greedy = None

    # -------------------------------------------------------------- one model step on the static buffers
    def _attend(self, i, record):
        """Layer i's attention for the step: q/k/v rows in self._qkv -> self._att (and the cache / tree update)."""
        st = self.states[i]
        if self.mode == 'dense':
            st.attend(self._qkv, self._pos, self._att, self._nkeys[i])
        elif self.general:
            B, C, H, dh = self.batch, self.C, self.H, self.dh
            q, k, v = [self._qkv[:, j * C:(j + 1) * C].view(B, H, 1, dh) for j in range(3)]
            _, nk = _general_step(st, self.W['layers'][i].get('pw'), q, k, v, self._pos,
                                  out=self._att.view(B, H, 1, dh))
            self._nkeys[i].copy_(nk.view(B, H))
        else:
            sel = None
            if record is not None:  # the selected leaves as well: (B, H, 1 + wmax) count, then leaf ids
                sel = torch.empty(self.batch, self.H, self.wmax + 1, device=self.dev, dtype=torch.int32)
                record[-1]['sel'] = sel
            _ops.decode_step(self._qkv, st.K, st.V, st.levels, self._pos, self.H, self.wmax, self.n_tree, self.Lw,
                             self.scale, self._att, nkeys=self._nkeys[i], sel=sel, splits=self.splits,
                             scratch=self._split)

    def _linear(self, name, act, w, mode, out=None, part=None):
        """One projection of the step: ta_linear_rows with self.lin_splits[name] K splits, or torch's matmul (and
        the GELU kernel) when that is 0."""
        sp = self.lin_splits[name]
        if sp == 0:
            torch.mm(act, w.t(), out=out)
            if mode == _ops.LIN_GELU:
                _ops.gelu_(out)
            return
        _ops.linear_rows(act, w, mode, out=out, splits=sp, part=part, keys=self._keys, ws=self._ws)

    def _forward_step_fused(self, record=None, greedy=False):
        """_forward_step on the library's linear kernel: per layer [h] qkv = h Wa^T, attention, part = att Wp^T
        (K split), [x += sum(part); h = ln2(x)], fc = gelu(h Wf^T), part = fc Wm^T (K split), [x += sum(part);
        h = ln1'(x)]; then the lm_head, with the greedy argmax and the position advance when `greedy`. The library's
        launches are chained by programmatic dependent launch; projections marked 0 in lin_splits stay on cuBLAS."""
        W = self.W
        L = W['layers']
        sp, sm = self.lin_splits['proj'], self.lin_splits['mlp']
        _ops.embed_ln(W['wte'], W['wpe'], self._tok, self._pos, L[0]['ln1'], self._x, self._h)
        for i, Li in enumerate(L):
            if record is not None:
                record.append(dict(x_in=self._x.clone()))
            self._linear('qkv', self._h, Li['c_attn'], _ops.LIN_STORE, out=self._qkv)
            self._attend(i, record)
            if sp:
                _ops.linear_rows(self._att, Li['c_proj'], _ops.LIN_PARTIAL, splits=sp, part=self._part[:sp])
                _ops.add_splits_ln(self._x, self._part[:sp], Li['ln2'], self._h)
            else:
                torch.mm(self._att, Li['c_proj'].t(), out=self._proj)
                _ops.add_ln(self._x, self._proj, Li['ln2'], self._h)
            self._linear('fc', self._h, Li['c_fc'], _ops.LIN_GELU, out=self._fc)
            nxt = L[i + 1]['ln1'] if i + 1 < len(L) else W['ln_f']
            if sm:
                _ops.linear_rows(self._fc, Li['c_mlp'], _ops.LIN_PARTIAL, splits=sm, part=self._part[:sm])
                _ops.add_splits_ln(self._x, self._part[:sm], nxt, self._h)
            else:
                torch.mm(self._fc, Li['c_mlp'].t(), out=self._mlp)
                _ops.add_ln(self._x, self._mlp, nxt, self._h)
            if record is not None:
                record[-1].update(qkv=self._qkv.clone(), att=self._att.clone(), x_out=self._x.clone())
        if greedy and self.lin_splits['lm']:
            self._linear('lm', self._h, W['wte'], _ops.LIN_ARGMAX, out=self._logits)
            _ops.argmax_finish(self._keys, W['wte'].shape[0], self._tok, self._pos)
        else:
            self._linear('lm', self._h, W['wte'], _ops.LIN_STORE, out=self._logits)
            if greedy:
                _ops.argmax_advance(self._logits, self._tok, self._pos)
        return self._logits

    def _forward_step_tail(self, record=None, greedy=False):
        """_forward_step with the block tail: embedding + ln_1 and layer 0's c_attn, then per layer the attention
        and ONE ta_block_tail launch (c_proj, residual, ln_2, c_fc + GELU, c_mlp, residual, the next layer's ln_1 and
        c_attn - or ln_f after the last layer); then the lm_head (and the greedy argmax with the position advance)."""
        W = self.W
        L = W['layers']
        _ops.embed_ln(W['wte'], W['wpe'], self._tok, self._pos, L[0]['ln1'], self._x, self._h)
        self._linear('qkv', self._h, L[0]['c_attn'], _ops.LIN_STORE, out=self._qkv)
        for i, Li in enumerate(L):
            if record is not None:
                record.append(dict(x_in=self._x.clone()))
            self._attend(i, record)
            if record is not None:
                record[-1].update(qkv=self._qkv.clone(), att=self._att.clone())
            nxt = L[i + 1] if i + 1 < len(L) else None
            _ops.block_tail(self._att, self._x, Li['c_proj'], Li['ln2'], Li['c_fc'], Li['c_mlp'],
                            nxt['ln1'] if nxt is not None else W['ln_f'], self._h,
                            w_qkv=nxt['c_attn'] if nxt is not None else None,
                            qkv_out=self._qkv if nxt is not None else None, bufs=self._tail_bufs)
            if record is not None:
                record[-1].update(x_out=self._x.clone())
        if greedy and self.fused_linear and self.lin_splits['lm']:
            self._linear('lm', self._h, W['wte'], _ops.LIN_ARGMAX, out=self._logits)
            _ops.argmax_finish(self._keys, W['wte'].shape[0], self._tok, self._pos)
        else:
            self._linear('lm', self._h, W['wte'], _ops.LIN_STORE, out=self._logits)
            if greedy:
                _ops.argmax_advance(self._logits, self._tok, self._pos)
        return self._logits

    def _forward_step(self, record=None):
        """Logits (B, V) of the tokens in self._tok at positions self._pos; appends their K/V to every layer.
        Per layer: [x += mlp; h = ln1(x)] qkv-matmul, fused decode attention, c_proj-matmul, [x += proj;
        h = ln2(x)], c_fc-matmul, GELU, c_mlp-matmul (the bracketed steps are single launches).
        `record` (a list; eager steps only) receives per layer copies of the residual entering it (x_in), its
        q/k/v rows, its attention output, its selected leaves (fused decode only) and the residual leaving it
        (x_out), for layer-by-layer checks."""
        if self.block_tail:
            return self._forward_step_tail(record)
        if self.fused_linear:
            return self._forward_step_fused(record)
        W = self.W
        L = W['layers']
        _ops.embed_ln(W['wte'], W['wpe'], self._tok, self._pos, L[0]['ln1'], self._x, self._h)
        for i, Li in enumerate(L):
            if record is not None:
                record.append(dict(x_in=self._x.clone()))
            torch.mm(self._h, Li['c_attn'].t(), out=self._qkv)
            self._attend(i, record)
            torch.mm(self._att, Li['c_proj'].t(), out=self._proj)
            _ops.add_ln(self._x, self._proj, Li['ln2'], self._h)
            torch.mm(self._h, Li['c_fc'].t(), out=self._fc)
            torch.mm(_ops.gelu_(self._fc), Li['c_mlp'].t(), out=self._mlp)
            nxt = L[i + 1]['ln1'] if i + 1 < len(L) else W['ln_f']
            _ops.add_ln(self._x, self._mlp, nxt, self._h)
            if record is not None:
                record[-1].update(qkv=self._qkv.clone(), att=self._att.clone(), x_out=self._x.clone())
        torch.mm(self._h, W['wte'].t(), out=self._logits)
        return self._logits

    def _greedy_step(self):
        if self.block_tail:
            return self._forward_step_tail(greedy=True)
        if self.fused_linear:
            return self._forward_step_fused(greedy=True)
        logits = self._forward_step()
        _ops.argmax_advance(logits, self._tok, self._pos)
        return logits

    def _capture(self, fn):
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                out = fn()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        return g, out

    def _ensure_graphs(self):
        """Capture the step graphs once. Capturing records the launches without running them; the one eager
        warm-up step before it (library attribute set-up, cuBLAS handles) feeds the current tokens at the current
        positions, which the next real step repeats exactly: it writes the same k/v rows at the same positions, forms
        the same tree nodes and stores the same best leaves, and it advances no token or position, so the caches
        need no copy around it (a copy of every cache would double the memory of a long-context decoder); only the
        running key sums, which it would count twice, are saved and restored."""
        if self._graph is not None or not self.use_graphs:
            return
        ksums = [st.ksum.clone() for st in self.states]  # the running key sums are not idempotent: restored
        self._forward_step()
        torch.cuda.current_stream(self.dev).synchronize()
        for st, ks in zip(self.states, ksums):
            st.ksum.copy_(ks)
        self._graph, _ = self._capture(self._forward_step)
        self._graph_greedy, _ = self._capture(self._greedy_step)

    # -------------------------------------------------------------- public API
    @torch.no_grad()
    def step(self, tok, t):
        """Feed tokens `tok` at positions t. Returns (logits, average keys read per head and layer).

        tok: int (batch 1, as the reference) or (B,) tensor; t: int or (B,) tensor. Logits are (V,) for an int
        token and (B, V) otherwise; keys is a 0-d device tensor."""
        scalar = not torch.is_tensor(tok)
        self._tok.copy_(torch.as_tensor(tok, dtype=torch.int64).reshape(-1).expand(self.batch))
        self._pos.copy_(_positions(t, self.batch, self.dev))
        if self.use_graphs:
            self._ensure_graphs()
            self._graph.replay()
            logits = self._logits
        else:
            logits = self._forward_step()
        keys = self._nkeys.float().mean()
        return (logits[0] if scalar and self.batch == 1 else logits), keys

    @torch.no_grad()
    def greedy_steps(self, n):
        """n greedy decode steps entirely on the device, continuing from the current token/position buffers
        (set by prefill() or step()). The generated tokens end in the token buffer (self.tokens)."""
        if not self.use_graphs:
            for _ in range(n):
                self._greedy_step()
            return
        self._ensure_graphs()
        for _ in range(n):
            self._graph_greedy.replay()

    @torch.no_grad()
    def serve_step(self, tok_host, out=None):
        """One greedy step for a serving loop that keeps tokens on the host: copy the current tokens (B,) from
        host (pinned) memory, run the step, copy the next tokens back to `out` (host) and wait for them.
        Positions advance by one on the device."""
        self._ensure_graphs()
        self._tok.copy_(tok_host, non_blocking=True)
        if self.use_graphs:
            self._graph_greedy.replay()
        else:
            self._greedy_step()
        if out is None:
            out = torch.empty(self.batch, dtype=torch.int64, pin_memory=True)
        out.copy_(self._tok, non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return out

    @property
    def tokens(self):
        return self._tok

    @property
    def positions(self):
        return self._pos

    def _prefill_selection(self, st, L, q, k, lv, tq, ids, vld, sct, b0, b1):
        """General selection for a prompt (the whole-sequence form of _general_step): learned budgets, the
        neighbour pass over the prompt's own descents, whose best leaves are stored for the decode steps that
        follow. Returns the leaf list and the kept (used, deduplicated) mask."""
        cfg = self.cfg
        nb, H, T0, _ = q.shape
        leaf = 1 << st.L0
        wl = ids.shape[-1]
        if cfg.beam_mode == 'pred':
            km = None
            if cfg.global_pool:
                km = mean_before(k.float(), 2)
            lhat = pred_budget(L['pw'], q, km, H)
        else:
            lhat = torch.full((nb, H, T0), cfg.beam, device=q.device, dtype=torch.int64)
        if not cfg.neighbors:
            n_tree = _ops.finish(ids, vld, lhat, cfg.wmax, leaf, positions=False)['n_tree']
            return ids, vld & (torch.arange(wl, device=q.device) < n_tree.unsqueeze(-1))
        NS = cfg.nb_store
        nid, match, nL = _ops.neighbor_pass(q, lv, ids[..., :NS], sct[..., :NS], vld[..., :NS], tq, cfg.nb_window,
                                            NS, cfg.nb_rho, cfg.nb_probe, cfg.nb_cap_min)
        n_tree = _ops.finish(ids, vld, lhat, cfg.wmax, leaf, nid=nid, match=match, nL=nL, positions=False)['n_tree']
        st.st_leaf[b0:b1, :, :T0] = ids[..., :NS]
        st.st_score[b0:b1, :, :T0] = sct[..., :NS]
        st.st_ok[b0:b1, :, :T0] = vld[..., :NS]
        used = vld & (torch.arange(wl, device=q.device) < n_tree.unsqueeze(-1))
        leaves = torch.cat([ids, nid], -1)
        return leaves, _ops.dedupe(leaves, torch.cat([used, match], -1))

    @torch.no_grad()
    def prefill(self, idx, chunk=16):
        """Run a prompt idx (B, T0) through the model (the training-mode forward semantics, reference
        model.py:75 / fastseg.py:338), filling every layer's cache and tree. Sets the token buffer to the greedy
        next token and the positions to T0. Returns the logits of the last prompt position (B, V)."""
        B, T0 = idx.shape
        if B != self.batch:
            raise ValueError('prefill: batch %d != decoder batch %d' % (B, self.batch))
        if T0 > self.cap:
            raise ValueError('prefill: %d positions above capacity %d' % (T0, self.cap))
        W, dt, H, dh, C = self.W, self.dtype, self.H, self.dh, self.C
        tq = torch.arange(T0, device=self.dev)
        last = torch.empty(B, W['wte'].shape[0], device=self.dev, dtype=dt)
        for b0 in range(0, B, chunk):
            b1 = min(B, b0 + chunk)
            ib = idx[b0:b1].to(self.dev)
            nb = b1 - b0
            x = W['wte'][ib].float() + W['wpe'][:T0].float()
            for i, L in enumerate(W['layers']):
                st = self.states[i]
                qkv = F.linear(_ln(x, L['ln1']).to(dt), L['c_attn'])
                q = qkv[..., :C].view(nb, T0, H, dh).transpose(1, 2)
                k = qkv[..., C:2 * C].view(nb, T0, H, dh).transpose(1, 2)
                v = qkv[..., 2 * C:].view(nb, T0, H, dh).transpose(1, 2)
                Kc, Vc = st.K[b0:b1, :, :T0], st.V[b0:b1, :, :T0]
                Kc.copy_(k)
                Vc.copy_(v)
                if self.mode == 'dense':  # the nanoGPT baseline: causal dense attention over the prompt
                    o = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).contiguous()
                    x = x + F.linear(o.view(nb, T0, C), L['c_proj']).float()
                    x = x + F.linear(F.gelu(F.linear(_ln(x, L['ln2']).to(dt), L['c_fc'])), L['c_mlp']).float()
                    continue
                lv = Levels(st.levels.nodes[b0:b1], st.cap, st.L0, st.Lm)
                _ops.build_levels(Kc, st.cap, st.L0, st.Lm, zero_sink=True, out=lv)
                if self.cfg.gate:  # the descent scores the gated nodes (levels >= gate_min_level)
                    lg = Levels(st.lg.nodes[b0:b1], st.cap, st.L0, st.Lm)
                    _ops.build_log_levels(Kc, st.cap, st.L0, st.Lm, zero_sink=True, out=lg)
                    lv = _ops.gate_levels(lv, lg, self.cfg.gate_q, getattr(self.cfg, 'gate_min_level', 0), T0,
                                          out=Levels(st.gated.nodes[b0:b1], st.cap, st.L0, st.Lm))
                ids, vld, sct = _ops.select(q, lv, tq, self.wmax)
                o = torch.empty(nb, T0, H, dh, device=self.dev, dtype=dt)
                if self.general:
                    leaves, keep = self._prefill_selection(st, L, q, k, lv, tq, ids, vld, sct, b0, b1)
                    _ops.attend_leaves(q, Kc, Vc, tq, leaves, keep, leaves.shape[-1], 1 << st.L0, self.Lw,
                                       self.scale, out=o.transpose(1, 2), want_nkeys=False)
                    del leaves, keep
                else:
                    _ops.attend_leaves(q, Kc, Vc, tq, ids, vld, self.n_tree, 1 << st.L0, self.Lw, self.scale,
                                       out=o.transpose(1, 2), want_nkeys=False)
                if self.cfg.beam_mode == 'pred' and self.cfg.global_pool:  # running key sums for the budget head
                    st.ksum[b0:b1] = Kc.float().sum(2)
                del ids, vld, sct
                x = x + F.linear(o.view(nb, T0, C), L['c_proj']).float()
                x = x + F.linear(F.gelu(F.linear(_ln(x, L['ln2']).to(dt), L['c_fc'])), L['c_mlp']).float()
            last[b0:b1] = F.linear(_ln(x[:, -1], W['ln_f']).to(dt), W['wte'])
        self._tok.copy_(last.argmax(-1))
        self._pos.fill_(T0)
        return last
