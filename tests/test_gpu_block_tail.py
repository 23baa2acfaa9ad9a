"""The block tail in one launch (ta_block_tail: c_proj, residual, ln_2, c_fc + GELU, c_mlp, residual, the next
block's ln_1 and c_attn) against a plain PyTorch fp32 reference of the same chain with the same roundings to the
model dtype, and the Decoder on it against the Decoder on torch matmuls (reference model.py:21-44 Block.forward,
engine.py:161-177 Decoder.step)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def _ops():
    from treeattn_b200 import _ops
    return _ops


def _no_device_error():
    code = _ops().device_error()
    assert code[0] == 0, code


def _ln(x, w, eps=1e-5):
    m = x.mean(-1, keepdim=True)
    v = ((x - m) ** 2).mean(-1, keepdim=True)
    return (x - m) * torch.rsqrt(v + eps) * w


def _layer(B, C, dt, seed, with_qkv=True):
    g = torch.Generator(device=DEV).manual_seed(seed)
    r = lambda *s, sc=1.0: torch.randn(*s, device=DEV, generator=g) * sc
    Wt = dict(att=r(B, C).to(dt), x=r(B, C), w_proj=r(C, C, sc=0.03).to(dt), ln2=1 + 0.1 * r(C),
              w_fc=r(4 * C, C, sc=0.03).to(dt), w_mlp=r(C, 4 * C, sc=0.02).to(dt), ln_next=1 + 0.1 * r(C))
    Wt['w_qkv'] = r(3 * C, C, sc=0.03).to(dt) if with_qkv else None
    return Wt


def _reference(Wt, dt):
    """The chain in fp32 with the model-dtype roundings where the step has them (every projection's output, the
    layer norms' outputs, the GELU's output)."""
    mm = lambda a, w: (a.float() @ w.float().t()).to(dt).float()
    x = Wt['x'] + mm(Wt['att'], Wt['w_proj'])
    h2 = _ln(x, Wt['ln2']).to(dt)
    fc = F.gelu(mm(h2, Wt['w_fc'])).to(dt)
    x = x + mm(fc, Wt['w_mlp'])
    h = _ln(x, Wt['ln_next']).to(dt)
    qkv = mm(h, Wt['w_qkv']).to(dt) if Wt['w_qkv'] is not None else None
    return x, h, qkv


def _run(Wt, bufs=None):
    ops = _ops()
    B, C = Wt['x'].shape
    x = Wt['x'].clone()
    h = torch.empty(B, C, device=DEV, dtype=Wt['att'].dtype)
    qkv = torch.empty(B, 3 * C, device=DEV, dtype=Wt['att'].dtype) if Wt['w_qkv'] is not None else None
    ops.block_tail(Wt['att'], x, Wt['w_proj'], Wt['ln2'], Wt['w_fc'], Wt['w_mlp'], Wt['ln_next'], h,
                   w_qkv=Wt['w_qkv'], qkv_out=qkv, bufs=bufs)
    return x, h, qkv


def _close(got, want, what, rel=2e-2, mean_rel=2e-3):
    """Within a few steps of the 16-bit format: every fp32 sum runs in another order than torch's, so a rounding
    to the dtype can land one step away and carry into what follows."""
    d = (got.float() - want.float()).abs()
    scale = want.float().abs().max().clamp(min=1e-6)
    assert float(d.max() / scale) <= rel, (what, float(d.max()), float(scale))
    assert float(d.mean() / want.float().abs().mean().clamp(min=1e-6)) <= mean_rel, (what, float(d.mean()))


@pytest.mark.parametrize('B,C,dt,with_qkv', [(64, 768, torch.bfloat16, True), (64, 768, torch.bfloat16, False),
                                             (8, 768, torch.bfloat16, True), (3, 128, torch.bfloat16, True),
                                             (128, 768, torch.bfloat16, True), (17, 512, torch.float16, True),
                                             (1, 256, torch.bfloat16, False), (40, 512, torch.bfloat16, True),
                                             (20, 2048, torch.bfloat16, True)])
def test_block_tail_matches_fp32_reference(B, C, dt, with_qkv):
    Wt = _layer(B, C, dt, B * 7 + C, with_qkv)
    x, h, qkv = _run(Wt)
    rx, rh, rq = _reference(Wt, dt)
    _close(x, rx, 'x')
    _close(h, rh, 'h')
    if with_qkv:
        _close(qkv, rq, 'qkv')
    _no_device_error()


def test_block_tail_repeatable_and_sync_left_zero():
    """The same inputs give bit-identical outputs call after call (fixed summation orders), and every call leaves
    the sync words zero for the next."""
    ops = _ops()
    Wt = _layer(64, 768, torch.bfloat16, 11)
    bufs = ops.block_tail_buffers(torch.bfloat16, 64, 768, DEV)
    outs = [_run(Wt, bufs) for _ in range(3)]
    for o in outs[1:]:
        for a, b in zip(outs[0], o):
            assert torch.equal(a, b)
    torch.cuda.synchronize()
    assert int(bufs[1].abs().sum()) == 0
    _no_device_error()


def test_block_tail_rejects_untaken_shapes():
    ops = _ops()
    assert ops.block_tail_plan(torch.bfloat16, 64, 768) is not None
    assert ops.block_tail_plan(torch.float32, 64, 768) is None      # 16-bit weights only
    assert ops.block_tail_plan(torch.bfloat16, 64, 96) is None      # width not a multiple of 128
    assert ops.block_tail_plan(torch.bfloat16, 129, 768) is None    # more than 128 rows
    assert ops.block_tail_plan(torch.bfloat16, 20, 4096) is None    # wider than the layer-norm phases take
    Wt = _layer(4, 128, torch.bfloat16, 3)
    with pytest.raises(Exception):
        ops.block_tail(Wt['att'], Wt['x'].clone(), Wt['w_proj'], Wt['ln2'], Wt['w_fc'], Wt['w_mlp'], Wt['ln_next'],
                       torch.empty(4, 128, device=DEV, dtype=torch.bfloat16), w_qkv=Wt['w_qkv'], qkv_out=None)


def test_decoder_block_tail_matches_matmul_path():
    """A 4-layer, 768-wide bf16 Decoder on the block tail against the same Decoder on torch matmuls and the
    separate row kernels: teacher-forced logits within 2e-2 of their scale (bf16 drift between two bf16
    pipelines), the residual stream layer by layer within the same bound."""
    import bench
    from treeattn_b200.engine import Decoder
    M = bench.CFG4
    cfg = bench.make_cfg(M)
    W = bench.make_weights(torch.device(DEV), 1234, torch.bfloat16, M)
    B, T0, nl = 8, 512, 4
    decs = []
    for tail in (False, True):
        dec = Decoder(W, nl, M.H, M.C, M.tcap, 'seg', cfg, DEV, batch=B, dtype=torch.bfloat16, cap=T0 + 64,
                      block_tail=tail, graphs=False)
        assert dec.block_tail == tail
        g = torch.Generator(device=DEV).manual_seed(5)
        prompts = torch.randint(0, M.V, (B, T0), device=DEV, generator=g)
        dec.prefill(prompts)
        decs.append(dec)
    g = torch.Generator(device=DEV).manual_seed(9)
    for t in range(6):
        tok = torch.randint(0, M.V, (B,), device=DEV, generator=g)
        recs = [[], []]
        outs = []
        for dec, rec in zip(decs, recs):
            dec._tok.copy_(tok)
            dec._pos.fill_(T0 + t)
            outs.append(dec._forward_step(record=rec).float().clone())
        for la, lb in zip(*recs):
            _close(lb['x_out'], la['x_out'], 'x_out', rel=2e-2, mean_rel=5e-3)
        _close(outs[1], outs[0], 'logits', rel=2e-2, mean_rel=5e-3)
    _no_device_error()
