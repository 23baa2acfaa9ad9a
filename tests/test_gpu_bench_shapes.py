"""Parity at the shapes bench.py times, against the numpy oracle.

* configuration 4, one decode layer: batch 64 x 12 heads (768 (b, h) items) of 64-wide bf16 rows, 64-token leaves,
  top-16, a 128-token window, 4094-token caches, the persistent kernel's grid (splits -1, 3 items per CTA, with the
  split scratch the Decoder passes), four steps across a leaf boundary (t = 4095 completes the 4096-token subtree);
  every item's selection, key count and output, and the caches and tree afterwards (reference engine.py:41-55,
  84-120);
* configuration 4, the whole model: the 12 x 768, vocab-50304 bf16 Decoder for 2 sequences after a 4096-token
  prefill, layer by layer and free running, against the oracle's decoder on the same caches (engine.py:149-177);
* configuration 3, one prefill layer: 4 x 12 x 8192 bf16 queries, the selection from ta_select and the attention
  from ta_prefill_attn, against the oracle's tree_pass and attention on 384 queries drawn from all 64 query tiles
  (fastseg.py:345-389, seg.py:44-70).

Selections compare exactly except queries the oracle marks as fp32 ties at a cut (tests/_compare.py); outputs and
logits within 2e-2 (bf16)."""
import math

import numpy as np
import pytest
import torch

import oracle
from tests._compare import compare_sets, record, tied

pytestmark = pytest.mark.gpu
DEV = 'cuda'
TOL = 2e-2


def _ops():
    from treeattn_b200 import _ops
    return _ops


def _no_device_error():
    code = _ops().device_error()
    assert code[0] == 0, code


def _keyset(ids, used, leaf, t, Lw):
    """Positions one decode query reads: the used leaves, the sink and the window (deduplicated)."""
    tree = [p for p in oracle.leaves_to_pos(ids, used, leaf).tolist() if p >= 0]
    return set(tree) | {0} | set(range(max(0, t - Lw + 1), t + 1))


# ------------------------------------------------------------------------------------------------ config 4 layer
def test_config4_decode_layer_every_item():
    ops = _ops()
    from treeattn_b200._ops import Levels
    B, H, dh, L0, wmax, local = 64, 12, 64, 6, 16, 128
    leaf, C, dt = 1 << L0, H * dh, torch.bfloat16
    T0, steps, cap = 4094, 4, 4352
    Lm = ops.lm_of(8192)
    splits = ops.default_splits(B, H, dh, dt)
    assert splits == -1, splits  # the persistent kernel the bench times
    g = torch.Generator(device=DEV).manual_seed(4)
    kc = torch.zeros(B, H, cap, dh, device=DEV, dtype=dt)
    vc = torch.zeros_like(kc)
    for b in range(B):  # bench.py fill_random: N(0, 0.25) keys, N(0, 1) values
        kc[b, :, :T0] = (torch.randn(H, T0, dh, device=DEV, generator=g) * 0.5).to(dt)
        vc[b, :, :T0] = torch.randn(H, T0, dh, device=DEV, generator=g).to(dt)
    lv = Levels.empty(B, H, dh, cap, L0, Lm, DEV)
    ops.build_levels(kc[:, :, :T0], cap, L0, Lm, zero_sink=True, out=lv)
    K0, V0 = kc[:, :, :T0].cpu(), vc[:, :, :T0].cpu()
    scratch = ops.split_scratch(B, H, dh, DEV)
    out = torch.empty(B, C, device=DEV, dtype=dt)
    nkeys = torch.empty(B, H, device=DEV, dtype=torch.int32)
    sel = torch.empty(B, H, wmax + 1, device=DEV, dtype=torch.int32)
    ntree = oracle.n_tree_fixed(wmax, wmax)
    rec = []
    for s_i in range(steps):
        qkv = torch.randn(B, 3 * C, device=DEV, generator=g).to(dt)
        pos = torch.full((B,), T0 + s_i, device=DEV, dtype=torch.int32)
        ops.decode_step(qkv, kc, vc, lv, pos, H, wmax, ntree, local, 1 / math.sqrt(dh), out, nkeys=nkeys, sel=sel,
                        splits=splits, scratch=scratch)
        rec.append((qkv.float().cpu().numpy(), out.float().cpu().numpy(), nkeys.cpu().numpy(), sel.cpu().numpy()))
    _no_device_error()
    n_cmp = n_tie = n_bad = 0
    worst = 0.0
    for b in range(B):
        st = oracle.SegStateNP(H, dh, cap, L0, Lm)
        st.fill(K0[b].float().numpy(), V0[b].float().numpy())
        for s_i, (qkv, o, nk, sl) in enumerate(rec):
            t = T0 + s_i
            q, k, v = [qkv[b, j * C:(j + 1) * C].reshape(H, dh) for j in range(3)]
            ro, _, (rids, rused, margin) = oracle.seg_attend(st, q, k, v, t, wmax, wmax, local, with_sel=True)
            for h in range(H):
                if margin[h] <= 1e-6:
                    n_tie += 1
                    continue
                n_cmp += 1
                if sorted(sl[b, h, 1:1 + sl[b, h, 0]].tolist()) != sorted(rids[h][rused[h]].tolist()):
                    n_bad += 1
                    continue
                assert nk[b, h] == len(_keyset(rids[h], rused[h], leaf, t, local)), (b, h, t)
                worst = max(worst, float(np.abs(o[b, h * dh:(h + 1) * dh] - ro[h]).max()))
        n = T0 + steps
        np.testing.assert_array_equal(kc[b, :, :n].float().cpu().numpy(), st.K[:, :n])
        np.testing.assert_array_equal(vc[b, :, :n].float().cpu().numpy(), st.V[:, :n])
        for l in range(L0, Lm + 1):
            m = n >> l
            np.testing.assert_array_equal(lv.level(l)[b, :, :m].cpu().numpy(), st.levels[l][0, :, :m])
    record(n_cmp, n_tie, n_bad, 'config-4 items x steps')
    assert n_bad == 0 and n_cmp >= 0.98 * B * H * steps, (n_bad, n_cmp, n_tie)
    assert worst < TOL, worst
    # the step at t = 4095 formed the 4096-token root (level 12, node 0) from the bulk-built halves
    assert torch.equal(lv.level(12)[:, :, 0], lv.level(11)[:, :, 0] + lv.level(11)[:, :, 1])


# ------------------------------------------------------------------------------------------------ config 4 model
def _bench_weights(seed, V, C, NL, tcap):
    """bench.py make_weights: N(0, 0.02), the residual projections 0.02 / sqrt(2 L), layer norms 1, bf16."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    n = lambda *s, std=0.02: (torch.randn(*s, generator=g, device=DEV) * std).to(torch.bfloat16)
    sp = 0.02 / math.sqrt(2 * NL)
    W = dict(wte=n(V, C), wpe=n(tcap, C), ln_f=torch.ones(C, device=DEV), layers=[])
    for _ in range(NL):
        W['layers'].append(dict(ln1=torch.ones(C, device=DEV), c_attn=n(3 * C, C), c_proj=n(C, C, std=sp),
                                ln2=torch.ones(C, device=DEV), c_fc=n(4 * C, C), c_mlp=n(C, 4 * C, std=sp)))
    return W


def test_config4_decoder_logits():
    """The 12 x 768 bf16 Decoder after a 4096-token prefill on the GPU; the oracle takes over the same caches (its
    own trees, built from them, equal the GPU's).

    Layer by layer (one eager step at t = 4096, each layer of the oracle started from the residual the GPU's layer
    received): q/k/v rows within 2e-2; from the GPU's own q/k/v the selected leaves equal the oracle's (fp32 ties
    excluded) and the attention output is within 2e-2; the residual leaving the layer within 2e-2; the logits of
    the final hidden state (fp32 products with the embedding) within 2e-2 and the bf16 logits within 2e-2 plus one
    bf16 step of the logit (|logit| >= 2 is stored in steps of 2^-6).

    Free running (8 teacher-forced tokens through Decoder.step's graph against the oracle's decoder): the two bf16
    decoders round each layer's outputs independently, so one-step differences of the rounded values reach later
    layers, move queries whose selection margin is below ~1e-4 and accumulate over the 12 layers; the logits of the
    final hidden states then agree within 5e-2 (about 0.02 measured). Layer 0's prompt keys / values equal the
    oracle's projection of the prompt up to one bf16 rounding."""
    from treeattn_b200.config import Config
    from treeattn_b200.engine import Decoder
    V, C, H, NL, leaf, topk, window, tcap = 50304, 768, 12, 12, 64, 16, 128, 8192
    B, T0, steps, cap = 2, 4096, 8, 4352
    dh, r = C // H, oracle.bf16_round
    cfg = Config(vocab_size=V, seq_len=tcap, n_layer=NL, n_head=H, n_embd=C, attn='seg', wmax=topk, beam=topk,
                 local=window, neighbors=False, beam_mode='fixed', leaf=leaf)
    W = _bench_weights(1234, V, C, NL, tcap)
    dec = Decoder(W, NL, H, C, tcap, 'seg', cfg, DEV, batch=B, dtype=torch.bfloat16, cap=cap)
    g = torch.Generator(device=DEV).manual_seed(8)
    idx = torch.randint(0, V, (B, T0 + steps), device=DEV, generator=g)
    dec.prefill(idx[:, :T0])
    torch.cuda.synchronize()
    Wn = dict(wte=W['wte'].float().cpu().numpy(), wpe=W['wpe'].float().cpu().numpy(),
              ln_f=W['ln_f'].cpu().numpy(),
              layers=[{k_: t_.float().cpu().numpy() for k_, t_ in L.items()} for L in W['layers']])
    wte = Wn['wte']
    free = oracle.DecoderNP(Wn, H, tcap, topk, topk, window, L0=6, cap=cap, kv_round=r, bf16=True)
    free.reset(B)
    forced = [[oracle.SegStateNP(H, dh, cap, 6, 12, r) for _ in range(NL)] for _ in range(B)]
    for i, st in enumerate(dec.states):
        for b in range(B):
            K_, V_ = st.K[b, :, :T0].float().cpu().numpy(), st.V[b, :, :T0].float().cpu().numpy()
            free.states[b][i].fill(K_, V_)
            forced[b][i].fill(K_, V_)
            for l in range(st.L0, st.Lm + 1):  # the GPU's bulk-built tree equals the oracle's
                m = T0 >> l
                np.testing.assert_array_equal(st.levels.level(l)[b, :, :m].cpu().numpy(),
                                              free.states[b][i].levels[l][0, :, :m])
    # layer 0's caches are the prompt's projections: one matmul in the oracle
    tok = idx[:, :T0].cpu().numpy()
    x0 = Wn['wte'][tok] + Wn['wpe'][:T0]
    L = Wn['layers'][0]
    qkv0 = r(r(oracle.layer_norm(x0, L['ln1'])) @ L['c_attn'].T)
    for j, cache in ((1, dec.states[0].K), (2, dec.states[0].V)):
        want = qkv0[..., j * C:(j + 1) * C].reshape(B, T0, H, dh).transpose(0, 2, 1, 3)
        got = cache[:, :, :T0].float().cpu().numpy()
        assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max()

    # ---- layer by layer at t = T0
    t = T0
    dec.tokens.copy_(idx[:, t])
    dec.positions.fill_(t)
    rec = []
    with torch.no_grad():
        lg = dec._forward_step(record=rec).float().cpu().numpy()
    n_cmp = n_tie = n_bad = 0
    worst = dict(qkv=0.0, att=0.0, x=0.0)
    for i, (Lw, R) in enumerate(zip(Wn['layers'], rec)):
        R = {k_: v_.float().cpu().numpy() if k_ != 'sel' else v_.cpu().numpy() for k_, v_ in R.items()}
        qkv = r(r(oracle.layer_norm(R['x_in'], Lw['ln1'])) @ Lw['c_attn'].T)
        worst['qkv'] = max(worst['qkv'], float(np.abs(R['qkv'] - qkv).max()))
        o = np.zeros((B, C), np.float32)
        for b in range(B):
            q, k, v = [R['qkv'][b, j * C:(j + 1) * C].reshape(H, dh) for j in range(3)]
            ob, _, (rids, rused, margin) = oracle.seg_attend(forced[b][i], q, k, v, t, topk, topk, window,
                                                             with_sel=True)
            o[b] = ob.reshape(C)
            for h in range(H):
                if margin[h] <= 1e-6:
                    n_tie += 1
                    continue
                n_cmp += 1
                sl = R['sel'][b, h]
                n_bad += sorted(sl[1:1 + sl[0]].tolist()) != sorted(rids[h][rused[h]].tolist())
        worst['att'] = max(worst['att'], float(np.abs(R['att'] - r(o)).max()))
        x = R['x_in'] + r(R['att'] @ Lw['c_proj'].T)
        f = r(oracle.gelu(r(r(oracle.layer_norm(x, Lw['ln2'])) @ Lw['c_fc'].T)))
        x = x + r(f @ Lw['c_mlp'].T)
        worst['x'] = max(worst['x'], float(np.abs(R['x_out'] - x).max()))
    record(n_cmp, n_tie, n_bad, 'config-4 model, layer by layer')
    h_ref = r(oracle.layer_norm(rec[-1]['x_out'].cpu().numpy(), Wn['ln_f']))
    l32 = float(np.abs(dec._h.float().cpu().numpy() @ wte.T - h_ref @ wte.T).max())
    rl = r(h_ref @ wte.T)
    step16 = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(rl), 2.0 ** -126))) - 7)  # one bf16 step at the logit
    l16 = float((np.abs(lg - rl) - step16).max())
    print('config-4 decoder layer by layer: qkv %.3g, attention %.3g, residual %.3g, logits fp32 %.3g / bf16 %.3g '
          'beyond one step; selections %d compared, %d ties, %d differ' % (
              worst['qkv'], worst['att'], worst['x'], l32, l16, n_cmp, n_tie, n_bad))
    assert n_bad == 0 and n_cmp >= 0.95 * NL * B * H
    assert max(worst.values()) < TOL and l32 < TOL and l16 < TOL, (worst, l32, l16)

    # ---- free running through the captured step
    drift = 0.0
    for s_i in range(steps):
        t = T0 + s_i
        dec.step(idx[:, t], t)
        free.step(idx[:, t].cpu().numpy(), t)
        drift = max(drift, float(np.abs(dec._h.float().cpu().numpy() @ wte.T - free.last_h @ wte.T).max()))
    print('config-4 decoder free running over %d steps: logits of the final hidden states within %.3g' % (
        steps, drift))
    assert drift < 5e-2, drift
    _no_device_error()


# ------------------------------------------------------------------------------------------------ config 3 layer
def test_config3_prefill_layer_with_real_selection():
    ops = _ops()
    B, H, T, dh, L0, wmax, local = 4, 12, 8192, 64, 6, 16, 128
    leaf, dt = 1 << L0, torch.bfloat16
    Lm = ops.lm_of(T)
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.randn(B, H, T, dh, device=DEV, generator=g).to(dt)
    k = torch.randn(B, H, T, dh, device=DEV, generator=g).to(dt)
    v = torch.randn(B, H, T, dh, device=DEV, generator=g).to(dt)
    tq = torch.arange(T, device=DEV)
    lv = ops.build_levels(k, T, L0, Lm, zero_sink=True)
    ids, vld, _ = ops.select(q, lv, tq, wmax)
    ntree = oracle.n_tree_fixed(wmax, wmax)
    scale = 1.0 / math.sqrt(dh)
    o, lse, nk = ops.prefill_attn(q, k, v, tq, ids, vld, ntree, leaf, local, scale, want_lse=True)
    torch.cuda.synchronize()
    _no_device_error()
    rng = np.random.default_rng(3)
    picks = {}  # (b, h) -> query positions: 6 per 128-query tile, spread over the (b, h)
    for tile in range(T // 128):
        for _ in range(6):
            bh = (int(rng.integers(B)), int(rng.integers(H)))
            picks.setdefault(bh, []).append(tile * 128 + int(rng.integers(128)))
    ids_n, vld_n, o_n, nk_n = ids.cpu().numpy(), vld.cpu().numpy(), o.float().cpu().numpy(), nk.cpu().numpy()
    worst, n_out = 0.0, 0
    for (b, h), tl in sorted(picks.items()):
        tl = np.array(sorted(tl))
        kf = k[b:b + 1, h:h + 1].float().cpu().numpy()
        vf = v[b, h].float().cpu().numpy()
        qf = q[b, h, tl].float().cpu().numpy()
        S = oracle.level_sums(kf, L0, Lm, zero_sink=True)
        rids, rvld, _, margin = oracle.tree_pass(qf[None, None], S, tl, L0, Lm, wmax, with_margin=True)
        excl = tied(margin)[0, 0]
        bad, _, _ = compare_sets(ids_n[b, h, tl], vld_n[b, h, tl], rids[0, 0], rvld[0, 0], excl)
        assert bad == 0, ((b, h), bad)
        for i, t in enumerate(tl.tolist()):
            if excl[i]:
                continue
            used = rvld[0, 0, i] & (np.arange(rids.shape[-1]) < ntree)
            ks = sorted(_keyset(rids[0, 0, i], used, leaf, t, local))
            assert nk_n[b, h, t] == len(ks), (b, h, t)
            s = (kf[0, 0, ks] @ qf[i]).astype(np.float32) * np.float32(scale)
            p = np.exp(s - s.max())
            ref = (p / p.sum()) @ vf[ks]
            worst = max(worst, float(np.abs(o_n[b, h, t] - ref).max()))
            n_out += 1
    assert n_out >= 0.98 * 6 * (T // 128), n_out
    assert worst < TOL, worst
