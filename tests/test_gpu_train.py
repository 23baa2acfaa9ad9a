"""Training path on the GPU: the backward of sparse_attn (ta_sparse_attn_bwd) against a plain PyTorch fp32
reference of the same op differentiated by autograd (the reference's own test_fast.py:47-64 compares the Triton
kernels with sparse_attn_ref the same way), and SegAttention / GPT trained through it.

Tolerances: fp32 1e-4 (absolute, on O(1) inputs), bf16 2e-2 relative to the gradient scale; dk / dv are summed
with atomics in an unspecified order, so only tolerances (not bits) are compared."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def sparse_attn_torch(q, k, v, cand, scale):
    """fastseg.py:134-141 sparse_attn_ref in plain fp32 PyTorch (differentiable)."""
    keep = cand >= 0
    idx = cand.clamp(min=0).long()
    B, H, T, K = cand.shape
    bi = torch.arange(B, device=idx.device)[:, None, None, None]
    hi = torch.arange(H, device=idx.device)[None, :, None, None]
    kg, vg = k[bi, hi, idx], v[bi, hi, idx]
    s = torch.einsum('bhtd,bhtkd->bhtk', q, kg) * scale
    w = torch.softmax(s.masked_fill(~keep, float('-inf')), -1)
    return torch.einsum('bhtk,bhtkd->bhtd', w, vg)


def _rand_cand(B, H, T, Tkv, K, g):
    cand = torch.randint(0, Tkv, (B, H, T, K), generator=g)
    cand[torch.rand(B, H, T, K, generator=g) < 0.2] = -1
    cand[..., 0] = torch.arange(T).clamp(max=Tkv - 1).view(1, 1, T)  # every query has a key
    cand[..., 1] = cand[..., 0]  # a duplicate counts twice, as in the reference kernel
    return cand


@pytest.mark.parametrize('dtype,dh,K', [(torch.float32, 64, 40), (torch.float32, 16, 9), (torch.float32, 128, 33),
                                        (torch.bfloat16, 64, 70), (torch.float16, 128, 17), (torch.bfloat16, 32, 5)])
def test_sparse_attn_grad_vs_torch(dtype, dh, K):
    from treeattn_b200.fastseg import sparse_attn
    g = torch.Generator().manual_seed(dh + K)
    B, H, T, Tkv = 2, 3, 50, 61
    q, k, v = [torch.randn(B, H, n, dh, generator=g) for n in (T, Tkv, Tkv)]
    do = torch.randn(B, H, T, dh, generator=g)
    cand = _rand_cand(B, H, T, Tkv, K, g)
    scale = 1.0 / math.sqrt(dh)
    qd, kd, vd = [t.to(DEV, dtype).requires_grad_(True) for t in (q, k, v)]
    o = sparse_attn(qd, kd, vd, cand.to(DEV).int(), scale)
    o.backward(do.to(DEV, dtype))
    # reference on the same (rounded) inputs, fp32
    qr, kr, vr = [t.to(dtype).float().requires_grad_(True) for t in (q, k, v)]
    orf = sparse_attn_torch(qr, kr, vr, cand, scale)
    orf.backward(do.to(dtype).float())
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    for name, a, r in (('o', o.detach(), orf.detach()), ('dq', qd.grad, qr.grad), ('dk', kd.grad, kr.grad),
                       ('dv', vd.grad, vr.grad)):
        scale_r = float(r.abs().max()) if dtype != torch.float32 else 1.0
        err = float((a.float().cpu() - r).abs().max())
        assert err <= tol * max(scale_r, 1.0), (name, err)
    from treeattn_b200 import _ops
    assert _ops.device_error()[0] == 0


def test_seg_attention_autograd_matches_fast_path_and_torch():
    """SegAttention with gradients: its forward equals the inference path (same key sets), and the gradients of
    q, k, v through sparse_attn equal those of the plain PyTorch formulation on the same candidates."""
    from treeattn_b200.config import Config
    from treeattn_b200.fastseg import SegAttention
    cfg = Config(vocab_size=64, seq_len=256, n_layer=1, n_head=2, n_embd=64, attn='seg', wmax=4, beam=3, local=16,
                 neighbors=False, beam_mode='fixed', leaf=8)
    torch.manual_seed(1)
    m = SegAttention(cfg).to(DEV)
    x = torch.randn(2, 256, 64, device=DEV)
    with torch.no_grad():
        y_fast = m(x)
    xg = x.clone().requires_grad_(True)
    y = m(xg)
    assert float((y.detach() - y_fast).abs().max()) < 1e-5
    y.square().sum().backward()
    # the same gradient through the plain PyTorch attention on the module's own candidate list
    import treeattn_b200.fastseg as fs
    orig = fs.sparse_attn
    fs.sparse_attn = lambda q, k, v, cand, scale: sparse_attn_torch(q, k, v, cand.long(), scale)
    try:
        xr = x.clone().requires_grad_(True)
        m.zero_grad()
        yr = m(xr)
        yr.square().sum().backward()
        gx_ref = xr.grad
    finally:
        fs.sparse_attn = orig
    assert float((xg.grad - gx_ref).abs().max()) < 1e-4 * max(1.0, float(gx_ref.abs().max()))
    for k_ in ('keys_total', 'keys_tree', 'leaves_used'):
        assert k_ in m.aux


def test_gpt_training_step_with_budget_head():
    """A few optimizer steps of the seg GPT in training mode with the learned budget head (beam_mode='pred'):
    the language-model loss goes down and the budget head gets a classification loss and gradients."""
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    cfg = Config(vocab_size=128, seq_len=128, n_layer=2, n_head=2, n_embd=64, attn='seg', wmax=8, beam=4, local=8,
                 neighbors=False, beam_mode='pred', beam_classes=(2, 4, 8), leaf=4)
    torch.manual_seed(2)
    m = GPT(cfg).to(DEV).train()
    idx = torch.randint(0, 128, (4, 128), device=DEV)
    opt = torch.optim.AdamW(m.parameters(), lr=3e-3)
    losses = []
    for _ in range(6):
        logits, loss, stats = m(idx, torch.roll(idx, -1, 1))
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(stats['lm']))
        assert math.isfinite(float(loss.detach()))
        assert stats['pred'] > 0
    assert losses[-1] < losses[0]
    pred_grad = m.blocks[0].attn.pred[0].weight.grad
    assert pred_grad is not None and float(pred_grad.abs().sum()) > 0


def test_sparse_attn_queries_without_keys():
    """A query whose candidates are all unused attends to nothing: output 0 (the reference kernel's l_safe rule),
    no gradient to q, none from it to any key; the other queries are unaffected."""
    from treeattn_b200.fastseg import sparse_attn
    g = torch.Generator().manual_seed(4)
    B, H, T, dh, K = 1, 2, 16, 64, 6
    q, k, v = [torch.randn(B, H, T, dh, generator=g) for _ in range(3)]
    cand = _rand_cand(B, H, T, T, K, g)
    cand[:, :, 5] = -1
    qd, kd, vd = [t.to(DEV).requires_grad_(True) for t in (q, k, v)]
    o = sparse_attn(qd, kd, vd, cand.to(DEV), 0.125)
    o.sum().backward()
    assert float(o[:, :, 5].abs().max()) == 0.0
    assert float(qd.grad[:, :, 5].abs().max()) == 0.0
    assert torch.isfinite(kd.grad).all() and torch.isfinite(vd.grad).all()
    qr, kr, vr = [t.clone().requires_grad_(True) for t in (q, k, v)]
    keep = torch.ones(T, dtype=torch.bool)
    keep[5] = False
    orf = sparse_attn_torch(qr[:, :, keep], kr, vr, cand[:, :, keep], 0.125)
    orf.sum().backward()
    assert float((o.detach().cpu()[:, :, keep] - orf.detach()).abs().max()) < 1e-4
    assert float((kd.grad.cpu() - kr.grad).abs().max()) < 1e-4
