"""Tensor-level wrappers over the C ABI (include/treeattn_b200.h).

Every function here takes CUDA tensors, checks shapes / dtypes / layouts, allocates its outputs with torch (the
library itself allocates nothing) and enqueues the kernel on the current torch stream of the tensors' device.
CPU tensors are rejected: there is no CPU, Triton or eager-PyTorch fallback.
"""
import ctypes
import math

import torch

from . import _lib

_DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _code(t):
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError('unsupported dtype %s (float32, bfloat16, float16)' % t.dtype) from None


def _need_cuda(name, *ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError('%s: tensors must be CUDA tensors (this package has no CPU path)' % name)


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _unit_inner(name, *ts):
    for t in ts:
        if t is not None and t.stride(-1) != 1:
            raise ValueError('%s: the innermost (head) dimension must be contiguous' % name)


def log2_exact(n, what='value'):
    n = int(n)
    if n < 1 or (n & (n - 1)):
        raise ValueError('%s must be a power of two (got %d)' % (what, n))
    return n.bit_length() - 1


def output_width(n_levels, wmax):
    """Slots the reference's tree_pass returns (seg.py:66: min(wmax, #candidates) at the last level)."""
    w = min(wmax, 1)
    for _ in range(n_levels - 1):
        w = min(wmax, 2 * w + 1)
    return w


def level_counts(cap, L0, Lm):
    """{l: (offset, count)} of the packed level layout."""
    out, o = {}, 0
    for l in range(L0, Lm + 1):
        out[l] = (o, cap >> l)
        o += cap >> l
    return out


class Levels:
    """Packed segment-tree levels L0..Lm for a batch of (b, h) trees.

    `nodes` is (B, H, n_nodes, dh) fp32; level l occupies nodes[:, :, off_l:off_l + (cap >> l)], node m covering
    positions [m*2^l, (m+1)*2^l)."""

    def __init__(self, nodes, cap, L0, Lm):
        self.nodes, self.cap, self.L0, self.Lm = nodes, int(cap), int(L0), int(Lm)
        self.counts = level_counts(self.cap, self.L0, self.Lm)

    @classmethod
    def empty(cls, B, H, dh, cap, L0, Lm, device):
        n = sum(c for _, c in level_counts(cap, L0, Lm).values())
        return cls(torch.zeros(B, H, max(n, 1), dh, device=device, dtype=torch.float32), cap, L0, Lm)

    def level(self, l):
        o, c = self.counts[l]
        return self.nodes[:, :, o:o + c]

    def as_dict(self):
        return LevelDict({l: self.level(l) for l in range(self.L0, self.Lm + 1)}, self)


class LevelDict(dict):
    """{level: tensor view} as the reference's level_sums returns, carrying the packed storage."""

    def __init__(self, d, packed):
        super().__init__(d)
        self.packed = packed


def build_levels(k, cap, L0, Lm, zero_sink=True, out=None):
    """Levels L0..Lm from keys k (B, H, T, dh) (any strides, contiguous head dim). Returns Levels."""
    _need_cuda('build_levels', k)
    _unit_inner('build_levels', k)
    B, H, T, dh = k.shape
    if out is None:
        out = Levels.empty(B, H, dh, cap, L0, Lm, k.device)
    nd = out.nodes
    _lib.call('ta_build_levels', _p(k), _code(k), B, H, T, dh, k.stride(0), k.stride(1), k.stride(2), out.cap,
              out.L0, out.Lm, 1 if zero_sink else 0, _p(nd), nd.stride(0), nd.stride(1), _stream(k))
    return out


def build_log_levels(k, cap, L0, Lm, zero_sink=True, out=None):
    """The gate's log-magnitude tree: levels L0..Lm of pairwise sums of log(|k| + 1e-6). Returns Levels."""
    _need_cuda('build_log_levels', k)
    _unit_inner('build_log_levels', k)
    B, H, T, dh = k.shape
    if out is None:
        out = Levels.empty(B, H, dh, cap, L0, Lm, k.device)
    nd = out.nodes
    _lib.call('ta_build_log_levels', _p(k), _code(k), B, H, T, dh, k.stride(0), k.stride(1), k.stride(2), out.cap,
              out.L0, out.Lm, 1 if zero_sink else 0, _p(nd), nd.stride(0), nd.stride(1), _stream(k))
    return out


def gate_levels(raw, lg, gate_q, gate_min, T_len, out=None):
    """Gated copy of a tree (seg.gate_apply on every complete node of levels >= gate_min). Returns Levels."""
    _need_cuda('gate_levels', raw.nodes, lg.nodes)
    B, H, _, dh = raw.nodes.shape
    if out is None:
        out = Levels.empty(B, H, dh, raw.cap, raw.L0, raw.Lm, raw.nodes.device)
    for t_ in (lg.nodes, out.nodes):
        if t_.stride() != raw.nodes.stride():
            raise ValueError('gate_levels: raw, lg and out must share one layout')
    nd = raw.nodes
    _lib.call('ta_gate_levels', _p(nd), _p(lg.nodes), _p(out.nodes), B, H, dh, int(T_len), nd.stride(0),
              nd.stride(1), raw.cap, raw.L0, raw.Lm, float(gate_q), int(gate_min), _stream(nd))
    return out


def gate_append(kc, raw, lg, gated, pos, gate_q, gate_min):
    """After appending position pos[b]: log-magnitude and gated nodes completed by it (decoding with the gate)."""
    B, H, cap, dh = kc.shape
    nd = raw.nodes
    _lib.call('ta_gate_append', _p(kc), _code(kc), B, H, dh, kc.stride(0), kc.stride(1), kc.stride(2), _p(nd),
              _p(lg.nodes), _p(gated.nodes), nd.stride(0), nd.stride(1), raw.cap, raw.L0, raw.Lm, _p(pos),
              float(gate_q), int(gate_min), _stream(kc))


def _tq_strides(tq, B, Nq):
    if tq.dim() == 1:
        if tq.shape[0] == Nq:
            return 0, tq.stride(0)
        if Nq == 1 and tq.shape[0] == B:
            return tq.stride(0), 0
    elif tq.dim() == 2 and tuple(tq.shape) == (B, Nq):
        return tq.stride(0), tq.stride(1)
    raise ValueError('query positions must have shape (Nq,), (B,) with Nq == 1, or (B, Nq)')


def select(q, levels, tq, wmax, wl=None):
    """Tree descent (seg.tree_pass) for queries q (B, H, Nq, dh) at positions tq.

    Returns ids (int64), vld (bool), sct (fp32), each (B, H, Nq, wl), best first."""
    _need_cuda('select', q, tq, levels.nodes)
    _unit_inner('select', q)
    B, H, Nq, dh = q.shape
    if wl is None:
        wl = output_width(levels.Lm - levels.L0 + 1, wmax)
    tq = tq.to(torch.int64)
    sb, st = _tq_strides(tq, B, Nq)
    ids = torch.empty(B, H, Nq, wl, device=q.device, dtype=torch.int64)
    vld = torch.empty(B, H, Nq, wl, device=q.device, dtype=torch.bool)
    sct = torch.empty(B, H, Nq, wl, device=q.device, dtype=torch.float32)
    nd = levels.nodes
    _lib.call('ta_select', _p(q), _code(q), B, H, Nq, dh, q.stride(0), q.stride(1), q.stride(2), _p(tq), sb, st,
              _p(nd), nd.stride(0), nd.stride(1), levels.cap, levels.L0, levels.Lm, wmax, wl, _p(ids), _p(vld),
              _p(sct), _stream(q))
    return ids, vld, sct


def neighbor_pass(q, levels, st_leaf, st_score, st_ok, tq, nb_window, nb_store, nb_rho, nb_probe, nb_cap_min,
                  neighbors=True):
    """seg.neighbor_pass on leaf blocks: q (B, H, Nq, dh), the tree (its leaf level is read), stored best leaves
    st_* (B, H, T_st, NS) indexed by position, tq positions. Returns nid (int64), match (bool) (B, H, Nq, Wn*NS)
    and nL (B, H, Nq) int64."""
    _need_cuda('neighbor_pass', q, tq, levels.nodes, st_leaf)
    _unit_inner('neighbor_pass', q)
    B, H, Nq, dh = q.shape
    st_leaf = st_leaf.to(torch.int64).contiguous()
    st_score = st_score.to(torch.float32).contiguous()
    st_ok = st_ok.to(torch.bool).contiguous()
    T_st = st_leaf.shape[2]
    tq = tq.to(torch.int64)
    sb, stq = _tq_strides(tq, B, Nq)
    leaf = levels.level(levels.L0)
    W = nb_window * nb_store
    nid = torch.empty(B, H, Nq, W, device=q.device, dtype=torch.int64)
    match = torch.empty(B, H, Nq, W, device=q.device, dtype=torch.bool)
    nL = torch.empty(B, H, Nq, device=q.device, dtype=torch.int64)
    _lib.call('ta_neighbor_pass', _p(q), _code(q), B, H, Nq, dh, q.stride(0), q.stride(1), q.stride(2), _p(tq), sb,
              stq, _p(leaf), leaf.stride(0), leaf.stride(1), leaf.shape[2], levels.L0, _p(st_leaf), _p(st_score),
              _p(st_ok), T_st, int(nb_window), int(nb_store), float(nb_rho), int(nb_probe), int(nb_cap_min),
              1 if neighbors else 0, _p(nid), _p(match), _p(nL), _stream(q))
    return nid, match, nL


def finish(ids, vld, lhat, wmax, leaf, nid=None, match=None, nL=None, positions=True):
    """seg.finish: returns dict(tree_pos, leaf_ok, nb_pos, n_tree, nb_leaves) (positions=False: n_tree only)."""
    _need_cuda('finish', ids, vld, lhat)
    shp = ids.shape[:-1]
    wl = ids.shape[-1]
    Q = int(torch.Size(shp).numel())
    ids = ids.contiguous()
    vld = vld.contiguous()
    lhat = lhat.to(torch.int64).expand(shp).contiguous()
    nbw = nid.shape[-1] if nid is not None else 0
    if nid is not None:
        nid = nid.to(torch.int64).contiguous()
        match = match.contiguous()
    if nL is not None:
        nL = nL.to(torch.int64).contiguous()
    dev = ids.device
    n_tree = torch.empty(shp, device=dev, dtype=torch.int64)
    nb_leaves = torch.empty(shp, device=dev, dtype=torch.int64)
    tree_pos = torch.empty(shp + (leaf * wl,), device=dev, dtype=torch.int64) if positions else None
    nb_pos = torch.empty(shp + (leaf * nbw,), device=dev, dtype=torch.int64) if positions else None
    _lib.call('ta_finish', _p(ids), _p(vld), _p(nid), _p(match), _p(nL), _p(lhat), Q, wl, nbw, leaf, wmax,
              _p(tree_pos), _p(nb_pos), _p(n_tree), _p(nb_leaves), _stream(ids))
    return dict(tree_pos=tree_pos, leaf_ok=vld, nb_pos=nb_pos, n_tree=n_tree, nb_leaves=nb_leaves)


def prefill_supported(dtype, dh, T_kv, leaf):
    """Whether ta_prefill_attn (tensor-core tiles) takes this shape: 16-bit, dh 64 / 128, <= 1024 leaves."""
    return dtype in (torch.bfloat16, torch.float16) and dh in (64, 128) and leaf >= 2 and -(-T_kv // leaf) <= 1024


def seg_attn(q, k, v, tq, ids, vld, n_tree, leaf, Lw, scale, out=None, want_lse=False, want_nkeys=True,
             entry='ta_seg_attn'):
    """Attention of each query over its used leaves (first n_tree valid of ids/vld), sink and window.

    q (B, H, Nq, dh), k / v (B, H, T_kv, dh): any strides with a contiguous head dim. n_tree: int or (B, H, Nq).
    `out` (B, H, Nq, dh) may be a strided view (e.g. of a (B, Nq, H, dh) buffer). Returns (out, lse, nkeys).
    entry: 'ta_seg_attn' (a warp per query) or 'ta_prefill_attn' (tensor-core tiles of 128 queries; 16-bit,
    dh 64 / 128)."""
    _need_cuda('seg_attn', q, k, v, tq, ids, vld)
    _unit_inner('seg_attn', q, k, v)
    B, H, Nq, dh = q.shape
    T_kv = k.shape[2]
    if q.dtype != k.dtype or k.dtype != v.dtype:
        raise TypeError('seg_attn: q, k and v must share a dtype')
    if out is None:
        out = torch.empty(B, H, Nq, dh, device=q.device, dtype=q.dtype)
    _unit_inner('seg_attn', out)
    tq = tq.to(torch.int64)
    sb, st = _tq_strides(tq, B, Nq)
    wl = ids.shape[-1]
    ids = ids.contiguous()
    vld = vld.contiguous()
    if torch.is_tensor(n_tree):
        ntp, ntc = n_tree.to(torch.int64).expand(B, H, Nq).contiguous(), 0
    else:
        ntp, ntc = None, int(n_tree)
    lse = torch.empty(B, H, Nq, device=q.device, dtype=torch.float32) if want_lse else None
    nkeys = torch.empty(B, H, Nq, device=q.device, dtype=torch.int32) if want_nkeys else None
    _lib.call(entry, _p(q), _p(k), _p(v), _code(q), B, H, Nq, dh, q.stride(0), q.stride(1), q.stride(2),
              k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1), v.stride(2), T_kv, _p(tq), sb, st,
              _p(ids), _p(vld), wl, _p(ntp), ntc, leaf, Lw, float(scale), _p(out), out.stride(0), out.stride(1),
              out.stride(2), _p(lse), _p(nkeys), _stream(q))
    return out, lse, nkeys


def prefill_attn(q, k, v, tq, ids, vld, n_tree, leaf, Lw, scale, out=None, want_lse=False, want_nkeys=True):
    """seg_attn on the tensor-core tile kernel (ta_prefill_attn)."""
    return seg_attn(q, k, v, tq, ids, vld, n_tree, leaf, Lw, scale, out, want_lse, want_nkeys, 'ta_prefill_attn')


def attend_leaves(q, k, v, tq, ids, vld, n_tree, leaf, Lw, scale, out=None, want_lse=False, want_nkeys=True):
    """seg_attn on the kernel that suits the call: tensor-core tiles (ta_prefill_attn) for runs of at least 64
    queries of a supported shape (prefill: consecutive positions), otherwise a warp per query (ta_seg_attn)."""
    Nq, dh = q.shape[2], q.shape[3]
    tiles = Nq >= 64 and prefill_supported(q.dtype, dh, k.shape[2], leaf)
    return seg_attn(q, k, v, tq, ids, vld, n_tree, leaf, Lw, scale, out, want_lse, want_nkeys,
                    'ta_prefill_attn' if tiles else 'ta_seg_attn')


def sparse_attn_fwd(q, k, v, cand, scale):
    """fastseg sparse_attn forward: cand (B, H, T, Kc) positions, -1 unused. Returns (o, lse)."""
    _need_cuda('sparse_attn', q, k, v, cand)
    _unit_inner('sparse_attn', q, k, v)
    B, H, T, dh = q.shape
    if q.dtype != k.dtype or k.dtype != v.dtype:
        raise TypeError('sparse_attn: q, k and v must share a dtype')
    if cand.dtype not in (torch.int32, torch.int64):
        cand = cand.to(torch.int64)
    cand = cand.contiguous()
    Kc = cand.shape[-1]
    o = torch.empty(B, H, T, dh, device=q.device, dtype=q.dtype)
    lse = torch.empty(B, H, T, device=q.device, dtype=torch.float32)
    _lib.call('ta_sparse_attn', _p(q), _p(k), _p(v), _code(q), B, H, T, dh, q.stride(0), q.stride(1), q.stride(2),
              k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1), v.stride(2), k.shape[2], _p(cand),
              1 if cand.dtype == torch.int64 else 0, Kc, float(scale), _p(o), o.stride(0), o.stride(1), o.stride(2),
              _p(lse), _stream(q))
    return o, lse


def sparse_attn_bwd(q, k, v, cand, o, lse, do, scale):
    """Gradients of sparse_attn (fastseg _attn_bwd): returns dq (q's dtype), dk, dv (k's / v's dtype; accumulated
    in fp32 by the kernel)."""
    _need_cuda('sparse_attn_bwd', q, k, v, cand, o, lse, do)
    q, k, v, o, do = [t.contiguous() for t in (q, k, v, o, do)]
    if cand.dtype not in (torch.int32, torch.int64):
        cand = cand.to(torch.int64)
    cand = cand.contiguous()
    B, H, T, dh = q.shape
    T_kv = k.shape[2]
    dq = torch.empty_like(q)
    dk = torch.zeros(B, H, T_kv, dh, device=q.device, dtype=torch.float32)
    dv = torch.zeros(B, H, T_kv, dh, device=q.device, dtype=torch.float32)
    _lib.call('ta_sparse_attn_bwd', _p(q), _p(k), _p(v), _p(o), _p(do), _p(lse.contiguous()), _code(q), B, H, T,
              T_kv, dh, _p(cand), 1 if cand.dtype == torch.int64 else 0, cand.shape[-1], float(scale), _p(dq),
              _p(dk), _p(dv), _stream(q))
    return dq, dk.to(k.dtype), dv.to(v.dtype)


def gather_dot(q, S, cand, scale):
    """fastseg.gather_dot: (B, H, N, C) fp32 = scale * q . S[cand] (ids clamped to [0, M-1])."""
    _need_cuda('gather_dot', q, S, cand)
    _unit_inner('gather_dot', q, S)
    if q.dtype != S.dtype:
        S = S.to(q.dtype)
    B, H, N, dh = q.shape
    M = S.shape[2]
    C = cand.shape[-1]
    if cand.dtype not in (torch.int32, torch.int64):
        cand = cand.to(torch.int64)
    cand = cand.contiguous()
    out = torch.empty(B, H, N, C, device=q.device, dtype=torch.float32)
    _lib.call('ta_gather_dot', _p(q), _p(S), _code(q), B, H, N, M, C, dh, q.stride(0), q.stride(1), q.stride(2),
              S.stride(0), S.stride(1), S.stride(2), _p(cand), 1 if cand.dtype == torch.int64 else 0, float(scale),
              _p(out), _stream(q))
    return out


def gather_dot_blocks(q, k, blocks, blk, scale, nb_cta=1, out=None):
    """Block form: q (B, H, dh), k (B, H, T, dh) with contiguous rows, blocks (B, H, nblk) int32 block ids.
    Returns (B, H, nblk*blk) fp32 scores."""
    _need_cuda('gather_dot_blocks', q, k, blocks)
    B, H, T, dh = k.shape
    nblk = blocks.shape[-1]
    blocks = blocks.to(torch.int32).contiguous()
    if out is None:
        out = torch.empty(B, H, nblk * blk, device=q.device, dtype=torch.float32)
    _lib.call('ta_gather_dot_blocks', _p(q), _p(k), _code(k), B, H, T, dh, q.stride(0), q.stride(1), k.stride(0),
              k.stride(1), k.stride(2), _p(blocks), nblk, blk, nb_cta, float(scale), _p(out), _stream(q))
    return out


def dedupe(cand, valid):
    """Keep the first valid copy of every value along the last dim (attention_dyn.dedupe)."""
    _need_cuda('dedupe', cand, valid)
    shp = cand.shape
    Kc = shp[-1]
    c = cand.to(torch.int64).contiguous()
    vv = valid.to(torch.bool).contiguous()
    keep = torch.empty(shp, device=cand.device, dtype=torch.bool)
    rows = c.numel() // max(Kc, 1)
    _lib.call('ta_dedupe', _p(c), _p(vv), _p(keep), rows, Kc, _stream(cand))
    return keep


def append(k, v, kc, vc, levels, pos):
    """SegState.add for a batch: k, v (B, H, dh) at positions pos (B,) int32."""
    _need_cuda('append', k, v, kc, vc, pos)
    B, H, dh = k.shape
    pos = pos.to(torch.int32)
    nd = levels.nodes
    _lib.call('ta_append', _p(k), _p(v), _code(kc), B, H, dh, k.stride(0), k.stride(1), v.stride(0), v.stride(1),
              _p(kc), _p(vc), kc.stride(0), kc.stride(1), kc.stride(2), _p(nd), nd.stride(0), nd.stride(1),
              levels.cap, levels.L0, levels.Lm, _p(pos), _stream(kc))


def split_scratch(B, H, dh, device):
    """Scratch for decode_step's split items: (B*H*4*(dh+4) fp32 partials, B*H int32 counters, zeroed)."""
    return (torch.empty(B * H * 4 * (dh + 4), device=device, dtype=torch.float32),
            torch.zeros(B * H, device=device, dtype=torch.int32))


def decode_step(qkv, kc, vc, levels, pos, H, wmax, n_tree, Lw, scale, out, lse=None, nkeys=None, sel=None,
                splits=0, scratch=None):
    """Fused decode step of one layer (seg_attend): qkv (B, 3*H*dh) rows, caches (B, H, cap, dh), pos (B,) int32.
    Writes out (B, H*dh) and appends k/v + updates the tree in place. scratch = split_scratch(...) lets the
    persistent kernel cut items into parts when whole items would leave SMs idle."""
    B = qkv.shape[0]
    dh = kc.shape[-1]
    C = H * dh
    nd = levels.nodes
    _lib.call('ta_decode_step', _p(qkv), _code(qkv), B, H, dh, qkv.stride(0), C, 2 * C, _p(kc), _p(vc),
              kc.stride(0), kc.stride(1), kc.stride(2), _p(nd), nd.stride(0), nd.stride(1), levels.cap, levels.L0,
              levels.Lm, _p(pos), wmax, n_tree, Lw, float(scale), _p(out), out.stride(0), _p(lse), _p(nkeys),
              _p(sel), int(splits), _p(scratch[0]) if scratch else None, _p(scratch[1]) if scratch else None,
              _stream(qkv))


def embed_ln(wte, wpe, tok, pos, w, x_out, h_out, eps=1e-5):
    """x_out = wte[tok] + wpe[pos] (fp32), h_out = LayerNorm(x_out) * w (h_out's dtype, same as the tables)."""
    B, C = x_out.shape
    _lib.call('ta_embed_ln', _p(wte), _p(wpe), _code(wte), _p(tok), _p(pos), B, wte.shape[0], wpe.shape[0], C, _p(w),
              float(eps), _p(x_out), _p(h_out), _stream(x_out))


def add_ln(x, y, w, h_out, eps=1e-5):
    """x += y (if y is not None), h_out = LayerNorm(x) * w in h_out's dtype. x: (B, C) fp32 contiguous."""
    B, C = x.shape
    _lib.call('ta_add_ln', _p(x), _p(y), _code(h_out), B, C, _p(w), float(eps), _p(h_out), _stream(x))


def gelu_(x):
    """In-place exact GELU (contiguous tensor, numel a multiple of 8)."""
    _lib.call('ta_gelu', _p(x), _code(x), x.numel(), _stream(x))
    return x


def argmax_advance(logits, tok, pos):
    """tok = logits.argmax(-1), pos += 1 (one fused launch)."""
    B, V = logits.shape
    _lib.call('ta_argmax_advance', _p(logits), _code(logits), B, V, _p(tok), _p(pos), _stream(logits))


LIN_STORE, LIN_GELU, LIN_PARTIAL, LIN_ARGMAX = 0, 1, 2, 3
LIN_TILE = 128  # output features per CTA of ta_linear_rows


def linear_supported(dtype, B, N, K, splits=1):
    """Whether ta_linear_rows takes these rows: 16-bit, 1..256 rows, K a multiple of 64 x splits that fits."""
    if dtype not in (torch.bfloat16, torch.float16):
        return False
    return bool(_lib.load().ta_linear_supported(_DT[dtype], B, N, K, splits))


def linear_workspace(B, N, splits, device):
    """(ws, counters) for ta_linear_rows' STORE / GELU / ARGMAX modes with K splits."""
    tiles = -(-N // LIN_TILE)
    return (torch.empty(tiles * splits * B * LIN_TILE, device=device, dtype=torch.float32),
            torch.zeros(tiles, device=device, dtype=torch.int32))


def linear_rows(act, w, mode=LIN_STORE, out=None, splits=1, part=None, keys=None, ws=None):
    """Rows times an nn.Linear weight on the tensor cores (ta_linear_rows): act (B, K) with a contiguous last dim,
    w (N, K) contiguous, same 16-bit dtype. mode STORE: out (B, N) = act w^T; GELU: exact GELU of it; PARTIAL: the
    fp32 sums of each of `splits` K slices into part (splits, B, N); ARGMAX: STORE plus each 128-feature tile's best
    (value, first index) per row in keys (ceil(N / 128), B) int64 for argmax_finish. STORE / GELU / ARGMAX with
    splits > 1 use ws = linear_workspace(...) (allocated here when not given). Returns out / part."""
    _need_cuda('linear_rows', act, w)
    B, K = act.shape
    N = w.shape[0]
    if act.stride(1) != 1 or not w.is_contiguous() or w.shape[1] != K or w.dtype != act.dtype:
        raise ValueError('linear_rows: act (B, K) with a unit inner stride and w (N, K) contiguous of its dtype')
    if mode == LIN_PARTIAL:
        if part is None:
            part = torch.empty(splits, B, N, device=act.device, dtype=torch.float32)
        res = part
    else:
        if out is None:
            out = torch.empty(B, N, device=act.device, dtype=act.dtype)
        res = out
    if mode != LIN_PARTIAL and splits > 1 and ws is None:
        ws = linear_workspace(B, N, splits, act.device)
    _lib.call('ta_linear_rows', _p(act), act.stride(0), _code(act), B, N, K, _p(w), int(splits), int(mode),
              _p(out) if mode != LIN_PARTIAL else None, out.stride(0) if mode != LIN_PARTIAL else 0,
              _p(part) if mode == LIN_PARTIAL else None, _p(keys) if mode == LIN_ARGMAX else None,
              _p(ws[0]) if ws is not None else None, _p(ws[1]) if ws is not None else None, _stream(act))
    return res


def add_splits_ln(x, part, w, h_out, eps=1e-5):
    """x += (sum of the splits of part (S, B, C), rounded to h_out's dtype); h_out = LayerNorm(x) * w."""
    B, C = x.shape
    _lib.call('ta_add_splits_ln', _p(x), _p(part), part.shape[0], _code(h_out), B, C, _p(w), float(eps), _p(h_out),
              _stream(x))


def argmax_finish(keys, V, tok, pos):
    """tok = the argmax packed in keys (tiles, B) by linear_rows' ARGMAX mode, pos += 1."""
    _lib.call('ta_argmax_finish', _p(keys), keys.shape[0], keys.shape[1], int(V), _p(tok), _p(pos), _stream(keys))


def block_tail_plan(dtype, B, C, with_qkv=True):
    """(workspace bytes, sync words) of ta_block_tail for B rows of width C on the current device, or None when it
    does not take the shape."""
    if dtype not in (torch.bfloat16, torch.float16):
        return None
    ws, ns = ctypes.c_int64(0), ctypes.c_int(0)
    if _lib.load().ta_block_tail_plan(_DT[dtype], int(B), int(C), int(bool(with_qkv)), ctypes.byref(ws),
                                      ctypes.byref(ns)) != 0:
        return None
    return int(ws.value), int(ns.value)


def block_tail_buffers(dtype, B, C, device, with_qkv=True):
    """(ws, sync) for block_tail: a byte workspace and zeroed int32 sync words (one pair per stream of calls)."""
    plan = block_tail_plan(dtype, B, C, with_qkv)
    if plan is None:
        raise ValueError('block_tail: %d rows of width %d are not taken' % (B, C))
    return (torch.empty(plan[0], device=device, dtype=torch.uint8),
            torch.zeros(plan[1], device=device, dtype=torch.int32))


def block_tail(att, x, w_proj, ln2, w_fc, w_mlp, ln_next, h_out, w_qkv=None, qkv_out=None, bufs=None, eps=1e-5):
    """The rest of a block after its attention and the next block's projection, one launch (ta_block_tail):
    x += c_proj(att); h2 = ln_2(x); x += c_mlp(gelu(c_fc(h2))); h_out = ln_next(x); qkv_out = c_attn'(h_out) when
    w_qkv is given. att, h_out, qkv_out (B, *) 16-bit contiguous, x (B, C) fp32 in place, weights (out, in)
    contiguous, ln weights fp32. bufs = block_tail_buffers(...) (allocated here when not given)."""
    _need_cuda('block_tail', att, x, w_proj, w_fc, w_mlp, h_out)
    B, C = x.shape
    with_qkv = w_qkv is not None
    if bufs is None:
        bufs = block_tail_buffers(att.dtype, B, C, att.device, with_qkv)
    for t in (att, x, w_proj, w_fc, w_mlp, h_out) + ((w_qkv, qkv_out) if with_qkv else ()):
        if not t.is_contiguous():
            raise ValueError('block_tail: contiguous tensors only')
    ws, sync = bufs
    _lib.call('ta_block_tail', _p(att), _p(x), _p(w_proj), _p(ln2), _p(w_fc), _p(w_mlp), _p(ln_next),
              _p(w_qkv) if with_qkv else None, float(eps), _code(att), B, C, _p(h_out),
              _p(qkv_out) if with_qkv else None, _p(ws), ws.numel(), _p(sync), _stream(x))
    return h_out


def default_splits(B, H, dh, dtype):
    """The decode mode ta_decode_step picks for B*H (b, h) pairs of head dim dh and element type dtype."""
    return _lib.load().ta_decode_default_splits(B, H, dh, _DT[dtype])


def device_error():
    return _lib.device_error()


def lm_of(T):
    """Top tree level for a sequence / capacity T (seg.py:127, engine.py:24): round(log2 T) - 1."""
    return int(round(math.log2(T))) - 1
