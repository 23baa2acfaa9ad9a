"""forest.gather_nodes (reference forest.py:4-9): the only forest helper the segment-tree path uses.

The block-forest attention (build_forest, two_means_order, soft_gate; attn='block') is not part of this
package."""


def gather_nodes(S, idx):
    """S: (b, H, M, d); idx: (b, H, T, W) long -> (b, H, T, W, d)."""
    b, H, T, W = idx.shape
    d = S.shape[-1]
    out = S.gather(2, idx.reshape(b, H, T * W, 1).expand(-1, -1, -1, d))
    return out.reshape(b, H, T, W, d)
