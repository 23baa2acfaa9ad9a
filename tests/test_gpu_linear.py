"""The decode step's linear layers on the library's tensor-core kernel (ta_linear_rows, ta_add_splits_ln,
ta_argmax_finish) against a plain PyTorch fp32 reference of the same op, and the Decoder on them against the
Decoder on torch matmuls (reference model.py:21-44, 90; engine.py:161-177; phase2.py:61-62)."""
import math

import numpy as np
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


def _step(x):
    """One step of the 16-bit format at |x| (bf16: 8 significant bits)."""
    return 2.0 ** (torch.floor(torch.log2(x.abs().clamp(min=1e-30))) - 7)


def _rows(B, N, K, dt, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    act = torch.randn(B, K, device=DEV, generator=g).to(dt)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(dt)
    return act, w


@pytest.mark.parametrize('B,N,K,dt', [(64, 2304, 768, torch.bfloat16), (2, 384, 128, torch.bfloat16),
                                      (20, 6144, 2048, torch.bfloat16), (256, 128, 64, torch.bfloat16),
                                      (37, 200, 320, torch.float16), (64, 50304, 768, torch.bfloat16)])
def test_linear_store_and_gelu(B, N, K, dt):
    """STORE = F.linear rounded to the dtype (one rounding step of the fp32 product, summation order aside); GELU =
    F.gelu of that rounded product."""
    ops = _ops()
    act, w = _rows(B, N, K, dt, B + N)
    ref = act.float() @ w.float().t()
    out = ops.linear_rows(act, w, ops.LIN_STORE)
    d = (out.float() - ref).abs()
    assert (d <= _step(ref) + 1e-3 * ref.abs().max()).all(), float(d.max())
    g = ops.linear_rows(act, w, ops.LIN_GELU)
    want = F.gelu(out.float()).to(dt).float()
    # the GELU input is this kernel's own rounded product; rounding the GELU output can differ by one step
    assert ((g.float() - want).abs() <= _step(want) + 1e-6).all()
    _no_device_error()


@pytest.mark.parametrize('mode,splits', [(0, 2), (1, 3), (3, 4)])
def test_linear_split_modes_match_unsplit(mode, splits):
    """STORE / GELU / ARGMAX with K splits (the last split of each tile adds the workspace sums in split order):
    the same rounded outputs as one split, up to one step of the dtype (fp32 sums in another order), and the same
    keys wherever the largest logit is not tied within that step."""
    ops = _ops()
    B, N, K = 64, 2304, 768
    act, w = _rows(B, N, K, torch.bfloat16, 7 + mode)
    keys = [torch.empty(-(-N // 128), B, device=DEV, dtype=torch.int64) for _ in range(2)]
    outs = [ops.linear_rows(act, w, mode, splits=sp, keys=keys[i]) for i, sp in enumerate((1, splits))]
    d = (outs[0].float() - outs[1].float()).abs()
    # one step of the rounded product; GELU rounds twice (its input, then its output): two steps
    assert (d <= (2 if mode == ops.LIN_GELU else 1) * _step(outs[0].float()) + 1e-6).all(), float(d.max())
    ws = ops.linear_workspace(B, N, splits, DEV)
    again = ops.linear_rows(act, w, mode, splits=splits, keys=keys[1], ws=ws)
    ops.linear_rows(act, w, mode, splits=splits, keys=keys[1], ws=ws)  # the counters were left at zero
    assert torch.equal(again, outs[1])
    assert int(ws[1].abs().sum()) == 0
    _no_device_error()


@pytest.mark.parametrize('B,N,K,splits', [(64, 768, 768, 6), (64, 768, 3072, 8), (5, 256, 1024, 16),
                                          (20, 2048, 8192, 4)])
def test_linear_partial_splits(B, N, K, splits):
    """PARTIAL: split s holds the fp32 product over K slice s (fp32 accumulation on the tensor cores)."""
    ops = _ops()
    act, w = _rows(B, N, K, torch.bfloat16, K + splits)
    part = ops.linear_rows(act, w, ops.LIN_PARTIAL, splits=splits)
    Ks = K // splits
    for s in range(splits):
        ref = act[:, s * Ks:(s + 1) * Ks].float() @ w[:, s * Ks:(s + 1) * Ks].float().t()
        torch.testing.assert_close(part[s], ref, atol=1e-4 * math.sqrt(Ks), rtol=1e-4)
    _no_device_error()


def test_add_splits_ln():
    """x += round_bf16(sum of the splits in order), h = LayerNorm(x) * w, against torch in fp32."""
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(2)
    S, B, C = 8, 64, 768
    part = torch.randn(S, B, C, device=DEV, generator=g) * 0.1
    x = torch.randn(B, C, device=DEV, generator=g)
    w = torch.rand(C, device=DEV, generator=g) + 0.5
    h = torch.empty(B, C, device=DEV, dtype=torch.bfloat16)
    s_ref = part[0].clone()
    for i in range(1, S):
        s_ref += part[i]
    x_ref = x + s_ref.to(torch.bfloat16).float()
    h_ref = F.layer_norm(x_ref, (C,), w, None, 1e-5)
    ops.add_splits_ln(x, part, w, h)
    torch.testing.assert_close(x, x_ref, atol=0, rtol=0)
    assert ((h.float() - h_ref).abs() <= _step(h_ref) + 1e-5).all()
    _no_device_error()


@pytest.mark.parametrize('B,V', [(64, 50304), (3, 304), (16, 128)])
def test_linear_argmax(B, V):
    """ARGMAX + argmax_finish: the token is torch.argmax of the kernel's own rounded logits (the first index among
    equal values) and the position advances; the logits are stored as in STORE mode."""
    ops = _ops()
    act, w = _rows(B, V, 768, torch.bfloat16, V)
    if V >= 300:  # planted ties: two vocabulary rows equal, so their logits tie in every row
        w[V - 1] = w[7]
    logits = torch.empty(B, V, device=DEV, dtype=torch.bfloat16)
    keys = torch.empty(-(-V // ops.LIN_TILE), B, device=DEV, dtype=torch.int64)
    tok = torch.zeros(B, device=DEV, dtype=torch.int64)
    pos = torch.arange(B, device=DEV, dtype=torch.int32)
    ops.linear_rows(act, w, ops.LIN_ARGMAX, out=logits, keys=keys)
    ops.argmax_finish(keys, V, tok, pos)
    assert torch.equal(logits, ops.linear_rows(act, w, ops.LIN_STORE))
    assert torch.equal(tok, logits.float().argmax(-1))
    assert torch.equal(pos, torch.arange(1, B + 1, device=DEV, dtype=torch.int32))
    _no_device_error()


def test_linear_rejects_bad_arguments():
    ops = _ops()
    from treeattn_b200._lib import TreeAttnError
    act, w = _rows(4, 128, 96, torch.bfloat16, 1)
    with pytest.raises(TreeAttnError, match='multiple'):
        ops.linear_rows(act, w)  # K = 96 is not a whole number of 64-wide blocks
    act, w = _rows(4, 128, 128, torch.bfloat16, 1)
    out = torch.empty(4, 128, device=DEV, dtype=torch.bfloat16)
    from treeattn_b200 import _lib
    with pytest.raises(TreeAttnError, match='workspace'):  # STORE with K splits and no workspace
        _lib.call('ta_linear_rows', ops._p(act), 128, 1, 4, 128, 128, ops._p(w), 2, ops.LIN_STORE, ops._p(out), 128,
                  None, None, None, None, ops._stream(act))
    big, _ = _rows(300, 128, 128, torch.bfloat16, 1)
    with pytest.raises(TreeAttnError, match='bad sizes'):
        ops.linear_rows(big, w)
    assert not ops.linear_supported(torch.float32, 4, 128, 128)


def _tiny_decoder(fused, dtype=torch.bfloat16, batch=3, seed=5):
    from treeattn_b200.config import Config
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    cfg = Config(vocab_size=512, seq_len=512, n_layer=3, n_head=2, n_embd=128, attn='seg', wmax=4, beam=4, local=16,
                 neighbors=False, beam_mode='fixed', leaf=8)
    torch.manual_seed(seed)
    m = GPT(cfg).eval()
    W = weights_from_ours({k: v.to(dtype) for k, v in m.state_dict().items()}, cfg)
    return Decoder(W, cfg.n_layer, cfg.n_head, cfg.n_embd, 512, 'seg', cfg, DEV, batch=batch, dtype=dtype,
                   fused_linear=fused)


def test_decoder_fused_linear_matches_torch_matmuls():
    """The Decoder on ta_linear_rows vs on torch matmuls, same weights and prompts: prefill, then 24 steps fed with
    the same tokens (logits within 2e-2 in bf16) and 16 greedy steps on the captured graphs, each giving the same
    token wherever the two largest logits are not near-tied (both decoders then continue from the same token)."""
    g = torch.Generator().manual_seed(1)
    idx = torch.randint(0, 512, (3, 200), generator=g).to(DEV)
    decs = [_tiny_decoder(f) for f in (True, False)]
    assert decs[0].fused_linear and not decs[1].fused_linear
    for d in decs:
        d.prefill(idx[:, :100])
    worst = 0.0
    for t in range(100, 124):
        lg = [d.step(idx[:, t], t)[0].float() for d in decs]
        worst = max(worst, float((lg[0] - lg[1]).abs().max()))
    assert worst < 2e-2, worst
    for d in decs:
        d.step(idx[:, 124], 124)
    n_clear = 0
    for _ in range(16):
        for d in decs:
            d.greedy_steps(1)
        top2 = decs[1]._logits.float().topk(2, -1).values
        clear = (top2[:, 0] - top2[:, 1]) > 4e-2
        n_clear += int(clear.sum())
        assert torch.equal(decs[0].tokens[clear], decs[1].tokens[clear])
        assert torch.equal(decs[0].positions, decs[1].positions)
        decs[0].tokens.copy_(decs[1].tokens)
    assert n_clear >= 24
    _no_device_error()
