"""CPU checks of the C-ABI library: it loads, exports every symbol the header declares, and rejects bad
arguments before touching the GPU. Plus the host-side helpers of the Python layer."""
import ctypes
import os
import re

import numpy as np
import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, 'include', 'treeattn_b200.h')


def _declared():
    src = open(HEADER).read()
    src = re.sub(r'/\*.*?\*/', '', src, flags=re.S)
    return sorted(set(re.findall(r'\b(ta_[a-z0-9_]+)\s*\(', src)))


def test_library_exports_every_declared_symbol():
    from treeattn_b200 import _lib
    lib = _lib.load()
    declared = _declared()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(_lib.SIGNATURES) == declared
    assert lib.ta_version() >= 100


def test_level_nodes():
    from treeattn_b200 import _lib, _ops
    lib = _lib.load()
    for cap, L0, Lm in [(4352, 6, 12), (65536, 7, 15), (512, 1, 8), (300, 2, 9)]:
        want = sum(cap >> l for l in range(L0, Lm + 1))
        assert lib.ta_level_nodes(cap, L0, Lm) == want
        counts = _ops.level_counts(cap, L0, Lm)
        assert sum(c for _, c in counts.values()) == want


def test_argument_validation_without_gpu():
    """Rejected arguments return TA_ERR_ARG with a message; no CUDA call is made on these paths."""
    from treeattn_b200 import _lib
    lib = _lib.load()
    # wait probe: limit outside [1 us, 10 s]
    for limit in (0, 999, 10 ** 10 + 1):
        rc = lib.ta_wait_probe(limit, None)
        assert rc == _lib.TA_ERR_ARG and 'ta_wait_probe' in _lib.last_error()
    # bad head dim
    rc = lib.ta_build_levels(None, 1, 1, 1, 16, 48, 0, 0, 0, 16, 1, 3, 1, None, 0, 0, None)
    assert rc == _lib.TA_ERR_ARG and 'head dim' in _lib.last_error()
    # wmax out of range
    rc = lib.ta_select(None, 1, 1, 1, 1, 64, 0, 0, 0, None, 0, 0, None, 0, 0, 16, 1, 3, 0, 1, None, None, None, None)
    assert rc == _lib.TA_ERR_ARG and 'wmax' in _lib.last_error()
    # top level below the leaf level
    rc = lib.ta_decode_step(None, 1, 1, 1, 64, 0, 0, 0, None, None, 0, 0, 0, None, 0, 0, 64, 6, 5, None, 16, 16, 128,
                            ctypes.c_float(0.125), None, 0, None, None, None, 1, None, None, None)
    assert rc == _lib.TA_ERR_ARG and 'Lm' in _lib.last_error()
    # cluster size limit
    rc = lib.ta_decode_step(None, 1, 1, 1, 64, 0, 0, 0, None, None, 0, 0, 0, None, 0, 0, 64, 3, 5, None, 16, 16, 128,
                            ctypes.c_float(0.125), None, 0, None, None, None, 9, None, None, None)
    assert rc == _lib.TA_ERR_ARG and 'splits' in _lib.last_error()
    # misaligned rows
    buf = (ctypes.c_char * 256)()
    addr = ctypes.addressof(buf)
    addr += (16 - addr % 16) % 16
    rc = lib.ta_seg_attn(addr + 2, addr, addr, 1, 1, 1, 1, 64, 0, 0, 64, 0, 0, 64, 0, 0, 64, 16, addr, 0, 1, addr,
                         addr, 1, None, 1, 2, 3, ctypes.c_float(0.125), addr, 0, 0, 64, None, None, None)
    assert rc == _lib.TA_ERR_ARG and 'aligned' in _lib.last_error()
    # training backward: bad head dim, null pointers
    rc = lib.ta_sparse_attn_bwd(addr, addr, addr, addr, addr, addr, 1, 1, 1, 4, 4, 48, addr, 0, 2,
                                ctypes.c_float(0.125), addr, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'head dim' in _lib.last_error()
    rc = lib.ta_sparse_attn_bwd(addr, addr, addr, addr, None, addr, 1, 1, 1, 4, 4, 64, addr, 0, 2,
                                ctypes.c_float(0.125), addr, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'null' in _lib.last_error()
    # dynamic-tree search: width above the beam, depth out of range
    rc = lib.ta_lane_search(addr, addr, addr, 4, 3, 64, 4, 5, addr, addr, None, None)
    assert rc == _lib.TA_ERR_ARG and 'wl' in _lib.last_error()
    rc = lib.ta_lane_search(addr, addr, addr, 4, 0, 64, 4, 4, addr, addr, None, None)
    assert rc == _lib.TA_ERR_ARG and 'D=' in _lib.last_error()
    # dynamic tree: capacity not a power of two, too many levels, neighbour store above the beam
    rc = lib.ta_lane_order(addr, 1, 1000 * 16, addr, 1, 2, 1000, 16, 3, 3, addr, addr, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'power of two' in _lib.last_error()
    rc = lib.ta_lane_order(addr, 1, 1024 * 16, addr, 1, 2, 1024, 16, 3, 10, addr, addr, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'levels' in _lib.last_error()
    rc = lib.ta_lane_order(addr + 4, 1, 1024 * 16, addr, 1, 2, 1024, 16, 3, 9, addr, addr, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'aligned' in _lib.last_error()
    rc = lib.ta_lane_select(addr, addr, addr, 1, 1, 64, 16, 16, 4, 4, 8, 2, 1, ctypes.c_float(0.35), 1, addr, addr,
                            addr, addr, addr, addr, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'nb_store' in _lib.last_error()
    rc = lib.ta_lane_insert(addr, addr, addr, 2, 48, 16, addr, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'power of two' in _lib.last_error()
    # block forest: depth not log2(B / 2), T not a multiple of the block, bad dtype
    ptrs = (ctypes.c_void_p * 8)(*([addr] * 8))
    rc = lib.ta_forest_levels(addr, 1, 4, 32, 16, 3, 2, 1, addr, 0, ctypes.c_float(0.25), ctypes.c_float(0.3),
                              ptrs, None)
    assert rc == _lib.TA_ERR_ARG and 'depth' in _lib.last_error()
    rc = lib.ta_forest_select(addr, 1, 1, 1, 100, 16, 0, 0, 16, ptrs, addr, 32, 4, None, 4, 8, addr, addr, addr,
                              addr, None, None, None)
    assert rc == _lib.TA_ERR_ARG and 'multiple' in _lib.last_error()
    rc = lib.ta_soft_gate(addr, addr, 7, 4, 8, 16, ctypes.c_float(0.25), ctypes.c_float(0.3), addr, None)
    assert rc == _lib.TA_ERR_ARG and 'dtype' in _lib.last_error()
    # neighbour pass: more than 32 stored leaves per query
    rc = lib.ta_neighbor_pass(addr, 1, 1, 1, 4, 64, 0, 0, 64, addr, 0, 1, addr, 0, 0, 8, 3, addr, addr, addr, 16,
                              9, 4, ctypes.c_float(0.35), 3, 2, 1, addr, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'nb_window' in _lib.last_error()


def test_python_layer_rejects_cpu_tensors():
    import torch
    from treeattn_b200 import _ops
    k = torch.randn(1, 2, 16, 64)
    with pytest.raises(ValueError, match='CUDA'):
        _ops.build_levels(k, 16, 1, 3)


@pytest.mark.parametrize('n_levels,wmax', [(1, 4), (2, 4), (3, 4), (8, 16), (12, 8)])
def test_output_width_matches_reference_rule(n_levels, wmax):
    """The slot count the reference's tree_pass returns (min(wmax, #candidates) at the last level)."""
    from treeattn_b200._ops import output_width
    T = 1 << (n_levels + 1)
    q = np.random.default_rng(0).standard_normal((1, 1, 4, 8)).astype(np.float32)
    k = np.random.default_rng(1).standard_normal((1, 1, T, 8)).astype(np.float32)
    S = oracle.level_sums(k, 1, n_levels)
    ids, _, _ = oracle.tree_pass(q, S, np.arange(T - 4, T), 1, n_levels, wmax)
    assert ids.shape[-1] == output_width(n_levels, wmax)


def test_n_tree_fixed_matches_finish():
    from treeattn_b200.fastseg import n_tree_fixed
    for wmax in (1, 4, 16):
        for beam in range(0, 20):
            r = oracle.finish(np.zeros((1, 1), np.int64), np.ones((1, 1), bool), np.zeros((1, 0), np.int64),
                              np.zeros((1, 0), bool), np.zeros(1, np.int64), np.array([beam]), wmax)
            assert n_tree_fixed(beam, wmax) == int(r['n_tree'][0]), (beam, wmax)


def test_config_fields_match_reference_defaults():
    from treeattn_b200.config import Config
    c = Config()
    assert (c.wmax, c.beam, c.local, c.nb_window, c.nb_store, c.leaf) == (8, 4, 3, 8, 2, 2)
    assert Config(**c.to_dict()) == c


def test_block_and_dyn_paths_need_cuda():
    """The block forest and the dynamic tree have no CPU path: CPU tensors are refused before any kernel call."""
    import torch
    from treeattn_b200.config import Config
    from treeattn_b200.dyntree import LaneTree, select_keys
    from treeattn_b200.forest import build_forest
    from treeattn_b200.model import GPT
    m = GPT(Config(attn='block', vocab_size=64, seq_len=128, n_layer=1, n_head=2, n_embd=32, tree_block=32)).eval()
    with pytest.raises(ValueError, match='CUDA'):
        with torch.no_grad():
            m(torch.zeros(1, 128, dtype=torch.long))
    k = torch.zeros(1, 2, 64, 16)
    with pytest.raises(ValueError, match='CUDA'):
        build_forest(k, 32, 4, Config())
    with pytest.raises(ValueError, match='CUDA'):
        select_keys(k, k, torch.ones(1, 2, 64, dtype=torch.long), Config(attn='dyn', seq_len=64, chunk=16))
    with pytest.raises(ValueError, match='CUDA'):
        LaneTree(torch.zeros(2, 64, 16), torch.tensor([0, 5]))


def test_checkpoint_loads_unchanged():
    """A checkpoint written by the reference's training script format loads into this package's GPT unchanged."""
    import torch
    from treeattn_b200.model import load_checkpoint
    path = os.path.join(ROOT, 'tests', 'golden', 'ckpt_tiny_seg.pt')
    m, cfg = load_checkpoint(path, 'cpu')
    ck = torch.load(path, map_location='cpu', weights_only=True)
    sd = m.state_dict()
    assert sorted(sd) == sorted(ck['model'])
    for name, t in ck['model'].items():
        assert torch.equal(sd[name], t), name
    assert cfg.beam_mode == 'pred' and tuple(cfg.beam_classes) == (2, 3, 4)


def test_block_tail_plan_and_linear_shapes_without_gpu():
    """The host-side planning of the decode step's fused callers: ta_block_tail_plan sizes the workspace and sync
    words for the shapes the block tail takes (and names why it refuses the others), ta_block_tail refuses missing
    pointers and a short workspace before any CUDA call, ta_linear_supported answers from the shapes alone."""
    from treeattn_b200 import _lib
    lib = _lib.load()
    ws, ns = ctypes.c_int64(0), ctypes.c_int(0)
    for B, C, q in [(64, 768, 1), (64, 768, 0), (8, 768, 1), (128, 768, 1), (3, 128, 1), (20, 2048, 1)]:
        assert lib.ta_block_tail_plan(1, B, C, q, ctypes.byref(ws), ctypes.byref(ns)) == _lib.TA_OK, _lib.last_error()
        # sync words: 8 fixed, two per c_fc tile, one per c_attn tile
        assert ns.value == 8 + 2 * (4 * C // 128) + 3 * C // 128
        # the workspace holds at least the 16-bit ln_2 and GELU rows, each piece 256-byte aligned
        assert ws.value >= B * C * 2 + B * 4 * C * 2 and ws.value % 256 == 0
    for dt, B, C in [(0, 64, 768), (1, 64, 96), (1, 129, 768), (1, 20, 4096), (1, 0, 768)]:
        rc = lib.ta_block_tail_plan(dt, B, C, 1, ctypes.byref(ws), ctypes.byref(ns))
        assert rc == _lib.TA_ERR_ARG and 'ta_block_tail' in _lib.last_error()
    f = ctypes.c_float(1e-5)
    rc = lib.ta_block_tail(None, None, None, None, None, None, None, None, f, 1, 64, 768, None, None, None, 0, None, None)
    assert rc == _lib.TA_ERR_ARG and 'null' in _lib.last_error()
    fake = 1 << 20  # aligned addresses that are never dereferenced: the workspace check comes first
    rc = lib.ta_block_tail(fake, fake, fake, fake, fake, fake, fake, fake, f, 1, 64, 768, fake, fake, fake, 256, fake,
                           None)
    assert rc == _lib.TA_ERR_ARG and 'workspace' in _lib.last_error()
    assert lib.ta_linear_supported(1, 64, 2304, 768, 1) == 1
    assert lib.ta_linear_supported(1, 64, 768, 3072, 16) == 1
    assert lib.ta_linear_supported(0, 64, 2304, 768, 1) == 0   # fp32 operands
    assert lib.ta_linear_supported(1, 300, 2304, 768, 1) == 0  # more than 256 rows
    assert lib.ta_linear_supported(1, 64, 2300, 768, 1) == 0   # N not a multiple of 8
    assert lib.ta_linear_supported(1, 64, 768, 768, 5) == 0    # K not a multiple of 64 x splits
