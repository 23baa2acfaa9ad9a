"""treeattn_b200: treeattn's segment-tree sparse attention on NVIDIA B200 (sm_100a).

Drop-in modules mirroring the reference package: config (Config), seg (level_sums, tree_pass, finish,
select_seg), fastseg (gather_dot, sparse_attn, dedupe_fast, select_seg_fast, SegAttention), attention_dyn
(dedupe, DynAttention), engine (SegState, seg_attend, Decoder), model (GPT). The kernels live in
lib/libtreeattn_b200.so (C ABI: include/treeattn_b200.h)."""
from .config import Config  # noqa: F401

__version__ = '0.1.0'
