"""Model / search configuration (the reference's Config, config.py:4-38, field for field, plus `leaf`)."""
from dataclasses import asdict, dataclass


@dataclass
class Config:
    vocab_size: int = 8192
    seq_len: int = 512          # training window (power of two); also the learned-position table size
    n_layer: int = 6
    n_head: int = 6
    n_embd: int = 384
    attn: str = 'block'         # 'seg' = segment tree (this package), 'dyn' = dynamic tree, 'block' = block forest
    tree_block: int = 64
    wmax: int = 8               # beam width of the tree descent (max leaves kept per level)
    beam: int = 4               # leaf budget when beam_mode == 'fixed'
    beam_mode: str = 'fixed'    # 'fixed' or 'pred' (learned budget head)
    beam_classes: tuple = (2, 3, 4, 6, 8)
    global_pool: bool = False
    gate: bool = False
    gate_q: float = 0.25
    gate_min_level: int = 0
    gate_temp: float = 0.3
    kmeans_iters: int = 3
    route_weight: float = 0.0
    pred_weight: float = 0.1
    chunk: int = 64
    local: int = 3              # static recent keys t, t-1, ... (window length max(local, 3))
    neighbors: bool = True
    nb_window: int = 8
    nb_store: int = 2
    nb_rho: float = 0.35
    nb_probe: int = 3
    nb_cap_min: int = 2
    leaf: int = 2               # tokens per tree leaf block (power of two); 2 = the reference's level-1 leaves

    def to_dict(self):
        return asdict(self)
