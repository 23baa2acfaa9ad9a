"""Block forest (reference forest.py) on the B200: one content-sorted binary tree per block of B keys.

The content sort (forest.py:13-33 two_means_order, repeated per level in build_forest) is the dynamic tree's 2-means
split with every slot valid: ta_lane_order, each block a lane of B slots. The node sums of every level, and the
optional soft mean-log gate (forest.py:36-44), are ta_forest_levels (one CTA per block, sums formed bottom-up in
adjacent pairs in fp32, written in the keys' dtype); soft_gate on explicit nodes is ta_soft_gate.
"""
import torch

from . import _lib, _ops


def gather_nodes(S, idx):
    """forest.py:4-9: S (b, H, M, d); idx (b, H, T, W) long -> (b, H, T, W, d)."""
    b, H, T, W = idx.shape
    d = S.shape[-1]
    out = S.gather(2, idx.reshape(b, H, T * W, 1).expand(-1, -1, -1, d))
    return out.reshape(b, H, T, W, d)


def _ptr_array(addrs):
    """A host array of device pointers for an entry point taking `void* const*`: (address, keep-alive)."""
    arr = (_lib.ctypes.c_void_p * len(addrs))(*addrs)
    return _lib.ctypes.cast(arr, _lib.c_void_p), arr


def _order_blocks(kf, P, B, dh, iters, levels):
    """ta_lane_order over P lanes of B fp32 key rows (all valid) -> perm (P, B) int32 (rank -> local position)."""
    dev = kf.device
    perm = torch.empty(P, B, device=dev, dtype=torch.int32)
    valid = torch.empty(P, B, device=dev, dtype=torch.uint8)
    perm_t = torch.empty_like(perm)
    valid_t = torch.empty_like(valid)
    n = torch.full((P,), B, device=dev, dtype=torch.int64)
    _lib.call('ta_lane_order', _ops._p(kf), 1, B * dh, _ops._p(n), 0, P, B, dh, int(iters), int(levels),
              _ops._p(perm), _ops._p(valid), _ops._p(perm_t), _ops._p(valid_t), _ops._stream(kf))
    return perm


@torch.no_grad()
def two_means_order(X, iters):
    """forest.py:13-33: X (P, G, S, D) -> order (P, G, S) long; inside every group the keys sorted by their projection
    on the difference of two 2-means centres, so that the halves are two balanced clusters."""
    _ops._need_cuda('two_means_order', X)
    P, G, S, D = X.shape
    if S < 4 or S & (S - 1):
        raise ValueError('two_means_order: group size %d must be a power of two >= 4' % S)
    kf = X.float().contiguous().view(P * G, S, D)
    return _order_blocks(kf, P * G, S, D, iters, 1).view(P, G, S).long()


def soft_gate(sm, grp, cfg):
    """forest.py:36-44 soft_gate: sm (P, n, d) summed keys of every node; grp (P, n, S, d) the member keys.
    Dimensions whose mean log-magnitude inside the group is low are faded out, the rest rescaled (ta_soft_gate)."""
    _ops._need_cuda('soft_gate', sm, grp)
    P, n, S, d = grp.shape
    smc = sm.contiguous()
    gc = grp.to(sm.dtype).contiguous()
    out = torch.empty_like(smc)
    _lib.call('ta_soft_gate', _ops._p(smc), _ops._p(gc), _ops._code(smc), P * n, S, d, float(cfg.gate_q),
              float(cfg.gate_temp), _ops._p(out), _ops._stream(smc))
    return out


@torch.no_grad()
def build_forest_raw(k, B, depth, cfg, zero_sink=False):
    """build_forest's work: the rank order (b H nb, B) int32 and the level sums [(b, H, nb 2^l, d)] in k's dtype.
    zero_sink counts the key at position 0 of every (b, h) as 0 (TreeAttention's idx_mask) without a copy of k."""
    _ops._need_cuda('build_forest', k)
    b, H, T, d = k.shape
    if B < 4 or B & (B - 1) or T % B:
        raise ValueError('build_forest: block %d must be a power of two >= 4 dividing T=%d' % (B, T))
    if (2 << depth) != B:
        raise ValueError('build_forest: depth %d must be log2(B / 2) for B=%d' % (depth, B))
    nb = T // B
    P = b * H * nb
    kc = k.contiguous()
    kf = kc.float()
    if zero_sink:
        if kf.data_ptr() == kc.data_ptr():
            kf = kf.clone()
        kf[:, :, 0] = 0
    perm = _order_blocks(kf, P, B, d, cfg.kmeans_iters, depth)
    sums = [torch.empty(b, H, nb << l, d, device=k.device, dtype=k.dtype) for l in range(depth + 1)]
    ptrs = _ptr_array([s.data_ptr() for s in sums])
    _lib.call('ta_forest_levels', _ops._p(kc), _ops._code(kc), P, B, d, depth, nb, int(bool(zero_sink)),
              _ops._p(perm), int(bool(cfg.gate)), float(cfg.gate_q), float(cfg.gate_temp), ptrs[0], _ops._stream(kc))
    return perm, sums


def build_forest(k, B, depth, cfg):
    """forest.py:47-75: one content-sorted tree per block of B keys. k (b, H, T, d).
    Returns perm_flat (b, H, nb B) long (rank -> local position inside the block) and sums[l] (b, H, nb 2^l, d)
    (level 0 = block root, level depth = groups of 2 keys; flat node id = block 2^l + m)."""
    b, H, T, d = k.shape
    perm, sums = build_forest_raw(k, B, depth, cfg)
    return perm.view(b, H, T).long(), sums
