"""Module-level parity on the GPU: SegAttention / GPT / SegState / seg_attend / Decoder against the reference's
golden outputs and the oracle, plus the reference's own invariant tests (test_seg.py) on this implementation."""
import math

import numpy as np
import pytest
import torch

import oracle
from tests._compare import record
from tests._golden import load

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def tiny(**kw):
    from treeattn_b200.config import Config
    base = dict(vocab_size=64, seq_len=64, n_layer=2, n_head=2, n_embd=32, attn='seg', wmax=4, beam=2,
                beam_classes=(2, 3, 4), nb_window=4, nb_store=2, nb_probe=2, nb_cap_min=1, neighbors=False,
                beam_mode='fixed')
    base.update(kw)
    return Config(**base)


def _no_device_error():
    from treeattn_b200 import _ops
    assert _ops.device_error()[0] == 0


def test_tiny_gpt_forward_golden():
    from treeattn_b200.model import GPT
    g = load('tiny_gpt')
    torch.manual_seed(4)
    m = GPT(tiny()).eval()
    m.to(DEV)
    with torch.no_grad():
        logits, _, stats = m(torch.as_tensor(g['idx']).to(DEV))
    np.testing.assert_allclose(logits.cpu().numpy(), g['logits'], atol=1e-4)
    for k in ('keys_total', 'keys_tree', 'leaves_used'):
        assert abs(stats[k] - float(g['stat_' + k])) < 1e-4, k
    _no_device_error()


def test_config1_forward_golden():
    """Configuration 1: GPT 4x256, 4 heads, vocab 4096, T 512, leaf 32, top-4, window 64, fp32, batch 2."""
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    g = load('config1')
    L0 = int(g['L0'])
    cfg = Config(vocab_size=4096, seq_len=512, n_layer=4, n_head=4, n_embd=256, attn='seg', wmax=4, beam=4,
                 local=64, neighbors=False, beam_mode='fixed', leaf=1 << L0)
    torch.manual_seed(0)
    m = GPT(cfg).eval().to(DEV)
    with torch.no_grad():
        logits, _, stats = m(torch.as_tensor(g['idx']).to(DEV))
    lg = logits.cpu().numpy()
    np.testing.assert_allclose(lg[:, ::32], g['logits_sub'], atol=1e-3)
    assert (lg.argmax(-1) == g['argmax']).mean() > 0.999
    lse = torch.logsumexp(logits.double(), -1).cpu().numpy()
    np.testing.assert_allclose(lse, g['lse'], atol=1e-3)
    assert abs(stats['keys_total'] - float(g['stat_keys_total'])) < 1e-2
    _no_device_error()


def test_engine_golden_tiny():
    """Decoder.step token by token (fp32) vs the reference engine's logits and keys."""
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    g = load('tiny_gpt')
    torch.manual_seed(4)
    cfg = tiny()
    m = GPT(cfg).eval()
    for graphs in (False, True):
        dec = Decoder(weights_from_ours(m.state_dict(), cfg), cfg.n_layer, cfg.n_head, cfg.n_embd, 64, 'seg', cfg,
                      DEV, graphs=graphs)
        got, keys = [], []
        for t in range(64):
            lg, kr = dec.step(int(g['idx'][0, t]), t)
            got.append(lg.clone())
            keys.append(float(kr))
        np.testing.assert_allclose(torch.stack(got).cpu().numpy(), g['dec_logits'], atol=1e-4)
        np.testing.assert_allclose(keys, g['dec_keys'], atol=1e-5)
    _no_device_error()


def test_seg_attend_golden():
    from treeattn_b200.config import Config
    from treeattn_b200.engine import SegState, seg_attend
    g = load('seg_attend')
    K, V, q = [torch.as_tensor(g[n]).to(DEV) for n in ('K', 'V', 'q')]
    H, T, dh = K.shape[1:]
    cfg = Config(seq_len=T, n_head=H, n_embd=H * dh, attn='seg', beam=4, beam_mode='fixed', local=3, neighbors=False)
    st = SegState(cfg, T, H, dh, DEV)
    st.fill(K, V)
    out, keys = seg_attend(st, None, q, None, None, T - 1, update=False)
    np.testing.assert_allclose(out.cpu().numpy(), g['out'], atol=1e-5)
    assert abs(float(keys) - float(g['keys'])) < 1e-6


@pytest.mark.parametrize('dtype,leaf', [(torch.float32, 8), (torch.float32, 2)])
def test_engine_matches_forward(dtype, leaf):
    """Reference test_seg.test_engine_matches_forward with leaf blocks and a batch: prefill of the first half
    of the sequence, then token-by-token steps, equal the whole-sequence forward (fp32, 1e-4)."""
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    cfg = tiny(seq_len=128, n_embd=64, wmax=4, beam=3, local=16, leaf=leaf)
    torch.manual_seed(9)
    m = GPT(cfg).eval().to(DEV)
    idx = torch.randint(0, 64, (3, 128), device=DEV)
    with torch.no_grad():
        ref = m(idx)[0]
    W = weights_from_ours(m.state_dict(), cfg)
    dec = Decoder(W, cfg.n_layer, cfg.n_head, cfg.n_embd, 128, 'seg', cfg, DEV, batch=3, dtype=dtype)
    last = dec.prefill(idx[:, :64])
    np.testing.assert_allclose(last.float().cpu().numpy(), ref[:, 63].cpu().numpy(), atol=1e-4)
    for t in range(64, 128):
        lg, _ = dec.step(idx[:, t], t)
        np.testing.assert_allclose(lg.float().cpu().numpy(), ref[:, t].cpu().numpy(), atol=1e-4)
    _no_device_error()


def test_bf16_decoder_vs_oracle():
    """bf16 weights and cache: prefill + token-by-token steps vs the oracle decoder that rounds to bf16 at the
    same points (max-abs 2e-2 on the logits)."""
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    cfg = tiny(seq_len=256, n_embd=128, n_head=2, vocab_size=128, wmax=8, beam=8, local=32, leaf=16)
    torch.manual_seed(7)
    m = GPT(cfg).eval()
    sd = {k: v.to(torch.bfloat16) for k, v in m.state_dict().items()}
    W = weights_from_ours(sd, cfg)
    idx = torch.randint(0, 128, (2, 192))
    dec = Decoder(W, cfg.n_layer, cfg.n_head, cfg.n_embd, 256, 'seg', cfg, DEV, batch=2, dtype=torch.bfloat16)
    dec.prefill(idx[:, :128].to(DEV))
    Wn = oracle.weights_from_state_dict({k: v.float() for k, v in sd.items()}, cfg.n_layer)
    ref = oracle.DecoderNP(Wn, cfg.n_head, 256, cfg.wmax, cfg.beam, cfg.local, L0=4, kv_round=oracle.bf16_round,
                           bf16=True)
    ref.reset(2)
    worst = 0.0
    for t in range(192):
        rl, _ = ref.step(idx[:, t].numpy(), t)
        if t >= 128:
            lg, _ = dec.step(idx[:, t].to(DEV), t)
            worst = max(worst, float(np.abs(lg.float().cpu().numpy() - rl).max()))
    assert worst < 2e-2, worst
    _no_device_error()


def test_greedy_graph_matches_eager():
    """The captured greedy loop gives the same tokens as eager steps."""
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    cfg = tiny(seq_len=256, n_embd=64, wmax=4, beam=4, local=16, leaf=8)
    torch.manual_seed(11)
    m = GPT(cfg).eval()
    W = weights_from_ours(m.state_dict(), cfg)
    idx = torch.randint(0, 64, (4, 100), device=DEV)
    toks = []
    for graphs in (False, True):
        dec = Decoder(W, cfg.n_layer, cfg.n_head, cfg.n_embd, 256, 'seg', cfg, DEV, batch=4, graphs=graphs)
        dec.prefill(idx)
        seq = []
        for _ in range(40):
            dec.greedy_steps(1)
            seq.append(dec.tokens.clone())
        toks.append(torch.stack(seq, 1))
        assert int(dec.positions[0]) == 140
    assert torch.equal(toks[0], toks[1])


def test_serve_step_matches_greedy_steps():
    """serve_step (tokens host -> device, the step's graph, next tokens device -> host; and the eager form without
    graphs) returns the tokens the device greedy loop produces, step after step."""
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    cfg = tiny(seq_len=256, n_embd=64, wmax=4, beam=4, local=16, leaf=8)
    torch.manual_seed(12)
    m = GPT(cfg).eval()
    W = weights_from_ours(m.state_dict(), cfg)
    idx = torch.randint(0, 64, (4, 100), device=DEV)
    ref = Decoder(W, cfg.n_layer, cfg.n_head, cfg.n_embd, 256, 'seg', cfg, DEV, batch=4)
    ref.prefill(idx)
    want = []
    for _ in range(30):
        ref.greedy_steps(1)
        want.append(ref.tokens.cpu().clone())
    for graphs in (True, False):
        dec = Decoder(W, cfg.n_layer, cfg.n_head, cfg.n_embd, 256, 'seg', cfg, DEV, batch=4, graphs=graphs)
        dec.prefill(idx)
        host = torch.empty(4, dtype=torch.int64, pin_memory=True)
        host.copy_(dec.tokens.cpu())
        for i in range(30):
            dec.serve_step(host, out=host)
            assert torch.equal(host, want[i]), (graphs, i)
        assert int(dec.positions[0]) == 130


def test_past_is_covered_exactly():
    """Reference test_seg.test_past_is_covered_exactly: with a wide beam the tree keys plus the static keys
    cover [0, t] exactly and nothing later."""
    from treeattn_b200.seg import select_seg
    torch.manual_seed(1)
    cfg = tiny(wmax=32, beam=32)
    T = 64
    q, k = torch.randn(1, 1, T, 16, device=DEV), torch.randn(1, 1, T, 16, device=DEV)
    sel = select_seg(q, k, torch.full((1, 1, T), 32, dtype=torch.long, device=DEV), cfg)
    tp = sel['tree_pos'][0, 0].cpu()
    for t in range(T):
        pos = set(tp[t][tp[t] >= 0].tolist())
        assert all(p < t for p in pos), ('future key selected', t)
        got = {p for p in pos | {0, t, t - 1, t - 2} if p >= 0}
        assert got == set(range(t + 1)), t


def test_all_keys_matches_dense():
    """Reference test_seg.test_all_keys_matches_dense on DynAttention(attn='seg')."""
    from treeattn_b200.attention_dyn import DynAttention
    torch.manual_seed(2)
    cfg = tiny(n_layer=1, wmax=32, beam=32)
    attn = DynAttention(cfg).eval().to(DEV)
    x = torch.randn(2, 64, 32, device=DEV)
    with torch.no_grad():
        out = attn(x)
        C, H, dh = 32, 2, 16
        q, k, v = attn.c_attn(x).split(C, 2)
        q, k, v = [t.view(2, 64, H, dh).transpose(1, 2) for t in (q, k, v)]
        s = (q @ k.transpose(-1, -2)) / dh ** 0.5
        s = s.masked_fill(~torch.tril(torch.ones(64, 64, dtype=torch.bool, device=DEV)), float('-inf'))
        ref = attn.c_proj((torch.softmax(s, -1) @ v).transpose(1, 2).reshape(2, 64, C))
    assert (out - ref).abs().max().item() < 1e-4


def test_causality():
    """Reference test_seg.test_causality (fixed budget): changing token 37 changes nothing before it."""
    from treeattn_b200.model import GPT
    torch.manual_seed(3)
    model = GPT(tiny()).eval().to(DEV)
    idx = torch.randint(0, 64, (2, 64), device=DEV)
    idx2 = idx.clone()
    idx2[:, 37] = (idx[:, 37] + 1) % 64
    with torch.no_grad():
        l1, _, _ = model(idx)
        l2, _, _ = model(idx2)
    assert (l1[:, :37] - l2[:, :37]).abs().max().item() < 1e-4
    assert (l1[:, 37:] - l2[:, 37:]).abs().max().item() > 1e-6


def test_bf16_model_vs_oracle():
    """bf16 weights through SegAttention (bf16 nn.Module forward) vs the oracle forward that rounds to bf16 at the
    same points (max-abs 2e-2 on the logits)."""
    from treeattn_b200.model import GPT
    cfg = tiny(seq_len=256, n_embd=128, n_head=2, wmax=8, beam=8, local=32, leaf=16, vocab_size=128)
    torch.manual_seed(5)
    m = GPT(cfg).eval()
    m = m.to(DEV, torch.bfloat16)
    idx = torch.randint(0, 128, (2, 256))
    with torch.no_grad():
        logits, _, _ = m(idx.to(DEV))
    W = oracle.weights_from_state_dict({k: v.float() for k, v in m.state_dict().items()}, cfg.n_layer)
    ref, _ = oracle.gpt_forward(W, idx.numpy(), cfg.n_head, cfg.wmax, cfg.beam, cfg.local, L0=4, bf16=True)
    assert np.abs(logits.float().cpu().numpy() - ref).max() < 2e-2


# ------------------------------------------------------------------------------------------------ neighbours
def test_select_seg_neighbours_golden():
    """seg.select_seg with neighbour borrowing (ta_neighbor_pass + ta_finish) on the reference's fixture, leaf 2:
    tree positions, neighbour positions, budgets and nb_leaves equal the reference's on every query."""
    from treeattn_b200.config import Config
    from treeattn_b200.seg import select_seg
    g = load('sel_nb')
    cfg = Config(attn='seg', seq_len=128, wmax=int(g['wmax']), beam=4, beam_mode='fixed')
    assert cfg.neighbors and cfg.nb_window == int(g['nb_window']) and cfg.nb_store == int(g['nb_store'])
    sel = select_seg(torch.as_tensor(g['q']).to(DEV), torch.as_tensor(g['k']).to(DEV),
                     torch.as_tensor(g['lhat']).to(DEV), cfg)
    srt = lambda a: np.sort(a, -1)
    assert (srt(sel['tree_pos'].cpu().numpy()) == srt(g['tree_pos'])).all()
    assert (srt(sel['nb_pos'].cpu().numpy()) == srt(g['nb_pos'])).all()
    assert (sel['n_tree'].cpu().numpy() == g['n_tree']).all()
    assert (sel['nb_leaves'].cpu().numpy() == g['nb_leaves']).all()
    _no_device_error()


def test_gpt_neighbours_golden():
    """The reference's tiny GPT with neighbour borrowing on (leaf 2): logits within 1e-4 and the aux statistics
    (keys_total / keys_tree / keys_nb / nb_leaves / leaves_used) equal."""
    from treeattn_b200.config import Config
    from treeattn_b200.model import GPT
    g = load('tiny_gpt_nb')
    cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=32, attn='seg', wmax=4, beam=3,
                 neighbors=True, beam_mode='fixed')
    torch.manual_seed(6)
    m = GPT(cfg).eval().to(DEV)
    with torch.no_grad():
        logits, _, stats = m(torch.as_tensor(g['idx']).to(DEV))
    np.testing.assert_allclose(logits.cpu().numpy(), g['logits'], atol=1e-4)
    for k in ('keys_total', 'keys_tree', 'keys_nb', 'nb_leaves', 'leaves_used'):
        assert abs(stats[k] - float(g['stat_' + k])) < 1e-4, (k, stats[k], float(g['stat_' + k]))
    _no_device_error()


@pytest.mark.parametrize('dt', [torch.float32, torch.bfloat16])
def test_neighbours_leaf_blocks_vs_oracle(dt):
    """Neighbour borrowing on 8-token leaf blocks, longer sequences: kernel selection vs the oracle's, queries
    near an fp32 tie (their own descent, a stored leaf of the nb_window positions before them, or a match
    threshold) excluded."""
    from treeattn_b200.config import Config
    from treeattn_b200.seg import select_seg
    rng = np.random.default_rng(11)
    B, H, T, dh = 2, 3, 1024, 64
    q = torch.as_tensor(rng.standard_normal((B, H, T, dh)).astype(np.float32)).to(dt)
    k = torch.as_tensor(rng.standard_normal((B, H, T, dh)).astype(np.float32)).to(dt)
    lhat = torch.as_tensor(rng.integers(2, 9, (B, H, T)))
    cfg = Config(attn='seg', seq_len=T, wmax=8, beam=4, beam_mode='fixed', leaf=8)
    sel = select_seg(q.to(DEV), k.to(DEV), lhat.to(DEV), cfg)
    nb = dict(nb_window=cfg.nb_window, nb_store=cfg.nb_store, nb_rho=cfg.nb_rho, nb_probe=cfg.nb_probe,
              nb_cap_min=cfg.nb_cap_min)
    ref = oracle.select_seg(q.float().numpy(), k.float().numpy(), lhat.numpy(), 8, L0=3, with_margin=True, nb=nb)
    tie = ref['margin'] <= 1e-6
    near = np.zeros_like(tie)
    for d in range(0, cfg.nb_window + 1):  # a tie at any of the positions a query borrows from
        near[..., d:] |= tie[..., :T - d]
    excl = near | (ref['nb_margin'] <= 1e-6)
    srt = lambda a: np.sort(a, -1)
    ok = ~excl
    record(int(ok.sum()), int(excl.sum()), 0, 'descent + neighbours')
    for key in ('tree_pos', 'nb_pos'):
        eq = (srt(sel[key].cpu().numpy()) == srt(ref[key])).all(-1)
        assert eq[ok].all(), (key, int((~eq & ok).sum()))
    assert (sel['nb_leaves'].cpu().numpy() == ref['nb_leaves'])[ok].all()
    assert (sel['n_tree'].cpu().numpy() == ref['n_tree'])[ok].all()
    assert ok.mean() > 0.95 and (ref['nb_pos'] >= 0).sum() > 1000
    _no_device_error()


def test_seg_attention_neighbours_autograd_matches_inference():
    """With neighbours on, the fused inference path (tree + borrowed leaves deduplicated, one attention kernel)
    and the training form (explicit candidate list + sparse_attn) give the same output."""
    from treeattn_b200.config import Config
    from treeattn_b200.fastseg import SegAttention
    cfg = Config(vocab_size=64, seq_len=256, n_layer=1, n_head=2, n_embd=64, attn='seg', wmax=4, beam=3, local=16,
                 neighbors=True, beam_mode='fixed', leaf=4)
    torch.manual_seed(3)
    m = SegAttention(cfg).to(DEV)
    x = torch.randn(2, 256, 64, device=DEV)
    with torch.no_grad():
        y_fast = m(x)
        aux_fast = {k: float(v) for k, v in m.aux.items()}
    y = m(x.clone().requires_grad_(True))
    aux_train = {k: float(v) for k, v in m.aux.items()}
    assert float((y.detach() - y_fast).abs().max()) < 1e-5
    for k in ('keys_total', 'keys_tree', 'keys_nb', 'nb_leaves', 'leaves_used'):
        assert abs(aux_fast[k] - aux_train[k]) < 1e-4, (k, aux_fast[k], aux_train[k])
    assert aux_fast['keys_nb'] > 0


def test_engine_neighbours_golden():
    """The reference engine's token-by-token decoding with neighbour borrowing (each position stores its best
    leaves, later positions borrow the matched ones): our Decoder (general-selection step, CUDA graph) gives the
    reference's logits within 1e-4 and the same keys read per step."""
    from treeattn_b200.config import Config
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    g = load('tiny_gpt_nb')
    cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=32, attn='seg', wmax=4, beam=3,
                 neighbors=True, beam_mode='fixed')
    torch.manual_seed(6)
    m = GPT(cfg).eval()
    dec = Decoder(weights_from_ours(m.state_dict(), cfg), cfg.n_layer, cfg.n_head, cfg.n_embd, 128, 'seg', cfg, DEV)
    idx = g['idx'][0]
    worst, kw = 0.0, 0.0
    for t in range(128):
        lg, keys = dec.step(int(idx[t]), t)
        worst = max(worst, float(np.abs(lg.cpu().numpy() - g['dec_logits'][t]).max()))
        kw = max(kw, abs(float(keys) - float(g['dec_keys'][t])))
    assert worst < 1e-4 and kw < 1e-4, (worst, kw)
    _no_device_error()


@pytest.mark.parametrize('global_pool', [False, True])
def test_engine_pred_neighbours_matches_forward(global_pool):
    """Learned budget head + neighbour borrowing on 4-token leaf blocks, batch 3: prefill of the first half and
    token-by-token steps give the whole-sequence forward's logits (the property of the reference's
    test_seg.test_engine_matches_forward), 1e-4."""
    from treeattn_b200.config import Config
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=64, attn='seg', wmax=8, beam=4, local=8,
                 neighbors=True, beam_mode='pred', beam_classes=(2, 4, 8), global_pool=global_pool, leaf=4)
    torch.manual_seed(12)
    m = GPT(cfg).eval().to(DEV)
    idx = torch.randint(0, 64, (3, 128), device=DEV)
    with torch.no_grad():
        ref = m(idx)[0]
    dec = Decoder(weights_from_ours(m.state_dict(), cfg), cfg.n_layer, cfg.n_head, cfg.n_embd, 128, 'seg', cfg, DEV,
                  batch=3)
    last = dec.prefill(idx[:, :64])
    np.testing.assert_allclose(last.float().cpu().numpy(), ref[:, 63].cpu().numpy(), atol=1e-4)
    for t in range(64, 128):
        lg, _ = dec.step(idx[:, t], t)
        np.testing.assert_allclose(lg.float().cpu().numpy(), ref[:, t].cpu().numpy(), atol=1e-4)
    _no_device_error()


# ------------------------------------------------------------------------------------------------ mean-log gate
@pytest.mark.parametrize('dt,L0,dh', [(torch.float32, 1, 32), (torch.bfloat16, 3, 64), (torch.float16, 4, 128)])
def test_gate_levels_vs_oracle(dt, L0, dh):
    """Log-magnitude tree and gated nodes (ta_build_log_levels, ta_gate_levels) vs the oracle: sums bit-exact,
    log sums within fp32 rounding of the logarithm, and the gated nodes equal wherever the gate keeps the same
    dimensions (the q-quantile cut can move only where two dimensions' mean logs tie to an ulp)."""
    from treeattn_b200 import _ops
    from treeattn_b200.seg import gated_tree
    rng = np.random.default_rng(L0 + dh)
    B, H, T = 2, 3, 512
    k = torch.as_tensor(rng.standard_normal((B, H, T, dh)).astype(np.float32)).to(dt)
    Lm = int(math.log2(T)) - 1
    raw, lg, gated = gated_tree(k.to(DEV), T, L0, Lm, 0.25, L0 + 1)
    kf = k.float().numpy()
    S = oracle.level_sums(kf, L0, Lm)
    G = oracle.log_sums(kf, L0, Lm)
    R = oracle.gated_levels(kf, L0, Lm, 0.25, L0 + 1)
    bad = total = 0
    for l in range(L0, Lm + 1):
        np.testing.assert_array_equal(raw.level(l).cpu().numpy(), S[l])
        np.testing.assert_allclose(lg.level(l).cpu().numpy(), G[l], rtol=2e-6, atol=2e-6 * (1 << l))
        got = gated.level(l).cpu().numpy()
        same = (got == R[l]).all(-1)
        bad += int((~same).sum())
        total += same.size
    assert bad <= max(1, total // 200), (bad, total)
    _no_device_error()


def test_gate_append_matches_bulk():
    """Decoding with the gate: the log-magnitude and gated nodes formed step by step (ta_append + ta_gate_append,
    across several leaf-block boundaries) equal the bulk build of the same cache, bit for bit."""
    from treeattn_b200.config import Config
    from treeattn_b200.engine import SegState
    cfg = Config(attn='seg', seq_len=256, n_head=2, n_embd=128, gate=True, gate_q=0.25, gate_min_level=3, leaf=4,
                 neighbors=False)
    rng = np.random.default_rng(5)
    B, H, dh, T0, steps = 2, 2, 64, 37, 40
    st = SegState(cfg, 256, H, dh, DEV, batch=B, dtype=torch.bfloat16)
    K0 = torch.as_tensor(rng.standard_normal((B, H, T0, dh)).astype(np.float32)).to(DEV, torch.bfloat16)
    st.fill(K0, K0)
    for s_i in range(steps):
        kk = torch.as_tensor(rng.standard_normal((B, H, dh)).astype(np.float32)).to(DEV, torch.bfloat16)
        st.add(T0 + s_i, kk, kk)
    ref = SegState(cfg, 256, H, dh, DEV, batch=B, dtype=torch.bfloat16)
    n = T0 + steps
    ref.fill(st.K[:, :, :n].clone(), st.V[:, :, :n].clone())
    for l in range(st.L0, st.Lm + 1):
        m = n >> l
        for a, b_ in ((st.levels, ref.levels), (st.lg, ref.lg), (st.gated, ref.gated)):
            assert torch.equal(a.level(l)[:, :, :m], b_.level(l)[:, :, :m]), l
    _no_device_error()


def test_select_seg_fast_gate_golden():
    """fastseg.select_seg_fast on mean-log gated levels (gate_min_level 2, neighbours on), the reference's fixture:
    tree and neighbour positions, budgets and nb_leaves equal on every query."""
    from treeattn_b200.config import Config
    from treeattn_b200.fastseg import select_seg_fast
    g = load('sel_gate')
    cfg = Config(attn='seg', seq_len=128, wmax=int(g['wmax']), beam=4, beam_mode='fixed', gate=True,
                 gate_q=float(g['gate_q']), gate_min_level=int(g['gate_min']))
    sel = select_seg_fast(torch.as_tensor(g['q']).to(DEV), torch.as_tensor(g['k']).to(DEV),
                          torch.as_tensor(g['lhat']).to(DEV), cfg)
    srt = lambda a: np.sort(a, -1)
    assert (srt(sel['tree_pos'].cpu().numpy()) == srt(g['tree_pos'])).all()
    assert (srt(sel['nb_pos'].cpu().numpy()) == srt(g['nb_pos'])).all()
    assert (sel['n_tree'].cpu().numpy() == g['n_tree']).all()
    assert (sel['nb_leaves'].cpu().numpy() == g['nb_leaves']).all()
    _no_device_error()


def test_gpt_gate_golden():
    """The reference's tiny GPT with the gate (gate_min_level 1) and neighbours: forward logits and statistics, and
    the engine's token-by-token logits, within 1e-4."""
    from treeattn_b200.config import Config
    from treeattn_b200.engine import Decoder, weights_from_ours
    from treeattn_b200.model import GPT
    g = load('tiny_gpt_gate')
    cfg = Config(vocab_size=64, seq_len=128, n_layer=2, n_head=2, n_embd=32, attn='seg', wmax=4, beam=3,
                 neighbors=True, beam_mode='fixed', gate=True, gate_q=0.25, gate_min_level=1)
    torch.manual_seed(8)
    m = GPT(cfg).eval()
    W = weights_from_ours(m.state_dict(), cfg)
    m = m.to(DEV)
    with torch.no_grad():
        logits, _, stats = m(torch.as_tensor(g['idx']).to(DEV))
    np.testing.assert_allclose(logits.cpu().numpy(), g['logits'], atol=1e-4)
    for k in ('keys_total', 'keys_tree', 'keys_nb', 'nb_leaves', 'leaves_used'):
        assert abs(stats[k] - float(g['stat_' + k])) < 1e-4, (k, stats[k], float(g['stat_' + k]))
    dec = Decoder(W, cfg.n_layer, cfg.n_head, cfg.n_embd, 128, 'seg', cfg, DEV)
    worst = 0.0
    for t in range(128):
        lg, keys = dec.step(int(g['idx'][0, t]), t)
        worst = max(worst, float(np.abs(lg.cpu().numpy() - g['dec_logits'][t]).max()))
        assert abs(float(keys) - float(g['dec_keys'][t])) < 1e-4, t
    assert worst < 1e-4, worst
    _no_device_error()


# ------------------------------------------------------------------------------------------------ checkpoint interop
GOLDEN_DIR = __import__('os').path.join(__import__('os').path.dirname(__import__('os').path.abspath(__file__)),
                                        'golden')


def test_checkpoint_forward_and_decoder_golden():
    """A checkpoint saved the way the reference's training scripts save it (train.py:144): the loaded GPT's logits and
    the Decoder's token-by-token logits (learned budget, neighbours) within 1e-4 of the reference's."""
    import os
    from treeattn_b200.engine import Decoder
    from treeattn_b200.model import load_checkpoint
    g = load('interop')
    path = os.path.join(GOLDEN_DIR, 'ckpt_tiny_seg.pt')
    m, cfg = load_checkpoint(path, DEV)
    with torch.no_grad():
        logits, _, _ = m(torch.as_tensor(g['idx']).to(DEV))
    assert (logits.cpu() - torch.as_tensor(g['logits'])).abs().max().item() < 1e-4
    dec = Decoder.from_checkpoint(path, 128, DEV)
    got = torch.stack([dec.step(int(g['idx'][0, t]), t)[0].float().cpu() for t in range(128)])
    assert (got - torch.as_tensor(g['seg_steps'])).abs().max().item() < 1e-4
    _no_device_error()


def test_nanogpt_dense_decoder_golden():
    """engine.weights_from_nanogpt (engine.py:137-146, torch.compile's '_orig_mod.' prefix) and the dense-mode
    Decoder (engine.py:74-81 DenseState): token-by-token logits within 1e-4 of the reference's; a prefill of the
    first 100 tokens continues to the same logits."""
    import os
    from treeattn_b200.engine import Decoder, weights_from_nanogpt
    g = load('interop')
    sd = torch.load(os.path.join(GOLDEN_DIR, 'ckpt_tiny_nanogpt.pt'), map_location='cpu', weights_only=True)
    W = weights_from_nanogpt(sd, 2)
    dec = Decoder(W, 2, 2, 32, 128, 'dense', None, DEV)
    got = torch.stack([dec.step(int(g['idx'][0, t]), t)[0].float().cpu() for t in range(128)])
    assert (got - torch.as_tensor(g['dense_steps'])).abs().max().item() < 1e-4
    dec2 = Decoder(W, 2, 2, 32, 128, 'dense', None, DEV)
    last = dec2.prefill(torch.as_tensor(g['idx'][:, :100]).to(DEV))
    assert (last[0].float().cpu() - torch.as_tensor(g['dense_steps'][99])).abs().max().item() < 1e-4
    nxt = dec2.step(int(g['idx'][0, 100]), 100)[0].float().cpu()
    assert (nxt - torch.as_tensor(g['dense_steps'][100])).abs().max().item() < 1e-4
    _no_device_error()
