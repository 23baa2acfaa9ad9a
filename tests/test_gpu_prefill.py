"""Tensor-core prefill tiles (ta_prefill_attn) against the warp-per-query kernel (ta_seg_attn) and against an
independent fp64 evaluation of each query's deduplicated key set (used leaves before the window, sink, window),
on random leaf selections with invalid slots, n_tree budgets, ragged query tiles and strided views."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def _ops():
    from treeattn_b200 import _ops
    return _ops


def _selection(rng, B, H, tq, wl, L0, Lw, p_invalid=0.15):
    """Random leaf ids per query (best-first order random), some slots invalid, some ids inside the window."""
    Nq = tq.shape[1]
    ids = np.full((B, H, Nq, wl), -1, np.int64)
    vld = np.zeros((B, H, Nq, wl), np.uint8)
    ntree = rng.integers(0, wl + 1, (B, H, Nq)).astype(np.int64)
    for b in range(B):
        for i in range(Nq):
            t = int(tq[b, i])
            nl = t >> L0  # complete leaves before the block of t
            for h in range(H):
                if nl == 0:
                    continue
                k = min(wl, nl)
                ids[b, h, i, :k] = rng.choice(nl, k, replace=False)
                vld[b, h, i, :k] = rng.random(k) > p_invalid
    return ids, vld, ntree


def _keys(t, ids, vld, ntree, L0, Lw):
    leaf = 1 << L0
    w0 = max(t - Lw + 1, 0)
    ks = set(range(w0, t + 1)) | {0}
    for i in range(min(len(ids), ntree)):
        m = int(ids[i])
        if vld[i] and m >= 0 and m * leaf < w0:
            ks |= set(range(m * leaf, min(m * leaf + leaf, w0)))
    return sorted(ks)


def _run(B, H, T, dh, leaf, Lw, wl, dt, seed, Nq=None, t_off=0, n_check=64, strided=True, k_growth=None):
    ops = _ops()
    rng = np.random.default_rng(seed)
    L0 = int(math.log2(leaf))
    Nq = T - t_off if Nq is None else Nq
    g = torch.Generator(device=DEV).manual_seed(seed)
    C = H * dh
    if strided:  # q as a view of a (B, Nq, 3, H, dh) projection, output into a (B, Nq, H, dh) buffer
        qkv = torch.randn(B, Nq, 3, H, dh, device=DEV, generator=g).to(dt)
        q = qkv[:, :, 0].permute(0, 2, 1, 3)
    else:
        q = torch.randn(B, H, Nq, dh, device=DEV, generator=g).to(dt)
    k = torch.randn(B, H, T, dh, device=DEV, generator=g) * 0.7
    if k_growth:  # key norms grow with position: a row's max rises tile after tile
        k = k * (1.0 + torch.arange(T, device=DEV, dtype=torch.float32) / k_growth).view(1, 1, T, 1)
    k = k.to(dt)
    v = torch.randn(B, H, T, dh, device=DEV, generator=g).to(dt)
    tq_np = np.tile(np.arange(t_off, t_off + Nq, dtype=np.int64), (B, 1))
    ids_np, vld_np, nt_np = _selection(rng, B, H, tq_np, wl, L0, Lw)
    tq = torch.as_tensor(tq_np, device=DEV)
    ids = torch.as_tensor(ids_np, device=DEV)
    vld = torch.as_tensor(vld_np, device=DEV)
    nt = torch.as_tensor(nt_np, device=DEV)
    scale = 1.0 / math.sqrt(dh)
    out_buf = torch.empty(B, Nq, H, dh, device=DEV, dtype=dt)
    out = out_buf.permute(0, 2, 1, 3) if strided else None
    o_t, lse_t, nk_t = ops.prefill_attn(q, k, v, tq, ids, vld, nt, leaf, Lw, scale, out=out, want_lse=True)
    o_w, lse_w, nk_w = ops.seg_attn(q, k, v, tq, ids, vld, nt, leaf, Lw, scale, want_lse=True)
    torch.cuda.synchronize()
    code = ops.device_error()
    assert code[0] == 0, code
    assert torch.equal(nk_t, nk_w)
    d = (o_t.float() - o_w.float()).abs().max().item()
    assert d < 2e-2, d
    dl = (lse_t - lse_w).abs().max().item()
    assert dl < 2e-2, dl
    # independent fp64 check of the key sets on sampled queries
    qf, kf, vf = q.double().cpu().numpy(), k.double().cpu().numpy(), v.double().cpu().numpy()
    of, nkn = o_t.double().cpu().numpy(), nk_t.cpu().numpy()
    worst = 0.0
    for _ in range(n_check):
        b, h, i = rng.integers(B), rng.integers(H), rng.integers(Nq)
        ks = _keys(int(tq_np[b, i]), ids_np[b, h, i], vld_np[b, h, i], int(nt_np[b, h, i]), L0, Lw)
        assert nkn[b, h, i] == len(ks)
        s = kf[b, h, ks] @ qf[b, h, i] * scale
        p = np.exp(s - s.max())
        ref = (p[:, None] * vf[b, h, ks]).sum(0) / p.sum()
        worst = max(worst, float(np.abs(of[b, h, i] - ref).max()))
    assert worst < 2e-2, worst


def test_prefill_config3_shape_strided():
    """Configuration-3 selection shape (leaf 64, top-16, window 128), ragged last tile, q / out as views."""
    _run(2, 3, 1000, 64, 64, 128, 16, torch.bfloat16, 1)


def test_prefill_dh128_leaf128():
    """Configuration-5 shape (dh 128, leaf 128, top-32, window 256): a leaf spans two key tiles."""
    _run(1, 2, 2100, 128, 128, 256, 32, torch.bfloat16, 2, strided=False)


def test_prefill_small_leaves_f16():
    """Leaves smaller than a key tile (leaf 16: four leaves per tile, masked per position), f16."""
    _run(2, 2, 700, 64, 16, 40, 8, torch.float16, 3)


def test_prefill_leaf2_min_window():
    """The reference's default leaf of 2 tokens and the minimum window of 3."""
    _run(1, 2, 300, 64, 2, 3, 8, torch.bfloat16, 4, strided=False)


def test_prefill_chunk_offset():
    """A chunk of 200 queries at positions 1300..1499 over a 1500-row cache (chunked prefill)."""
    _run(2, 2, 1500, 64, 32, 64, 8, torch.bfloat16, 5, Nq=200, t_off=1300, strided=False)


@pytest.mark.parametrize('dh,leaf,Lw,wl', [(64, 64, 128, 16), (128, 128, 256, 32)])
def test_prefill_rising_scores_rescale(dh, leaf, Lw, wl):
    """Key norms growing with position, so that a row's running max rises by more than 2^8 (log2 domain) again and
    again over its key tiles: the tile kernel's in-place rescale of the O accumulator (its reference max moves only
    then) must give the same rows as the warp kernel and the fp64 evaluation."""
    _run(2, 2, 1200, dh, leaf, Lw, wl, torch.bfloat16, 7, strided=False, k_growth=16.0)


def test_prefill_rejects_unsupported():
    ops = _ops()
    from treeattn_b200._lib import TreeAttnError
    q = torch.zeros(1, 1, 8, 64, device=DEV)
    tq = torch.arange(8, device=DEV).view(1, 8)
    ids = torch.zeros(1, 1, 8, 2, device=DEV, dtype=torch.int64)
    vld = torch.zeros(1, 1, 8, 2, device=DEV, dtype=torch.uint8)
    with pytest.raises(TreeAttnError, match='bf16 or f16'):
        ops.prefill_attn(q, q, q, tq, ids, vld, 2, 2, 3, 0.125)
    qb = q.bfloat16()
    with pytest.raises(TreeAttnError, match='leaf'):
        ops.prefill_attn(qb, qb, qb, tq, ids, vld, 2, 1, 3, 0.125)
