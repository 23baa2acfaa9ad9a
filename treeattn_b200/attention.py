"""Block-forest attention (reference attention.py, attn='block'): not part of this package.

The name is kept so that model code that imports it keeps importing; constructing it raises."""
import torch.nn as nn


class TreeAttention(nn.Module):
    def __init__(self, cfg):
        raise NotImplementedError("attn='block' (block-forest TreeAttention) is not implemented in treeattn_b200; "
                                  "use attn='seg'")
