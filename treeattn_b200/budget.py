"""The learned leaf budget (beam_mode='pred'): how many of the leaves the descent found a query actually uses.

One small head per layer maps a query to one of cfg.beam_classes. Its inputs and its training target are the same
for the three attention forms that carry it - the segment tree (fastseg.SegAttention, engine.Decoder) and the
block forest (attention.TreeAttention) - so both live here:

* inputs: the query, the logarithm of its norm, the one-hot index of its head and, with cfg.global_pool, the mean of
  the keys the query comes after (reference fastseg.py:352-365, attention.py:96-111, engine.py:89-94);
* target: the smallest budget class that covers 90 % of the attention weight the query puts on its leaves, counted
  best-first (reference fastseg.py:394-405, attention.py:145-159).
"""
import torch


def budget_features(q, kmean=None):
    """Input rows of the budget head for queries q (B, H, N, dh), in q's dtype: [q | log(||q|| + 1e-6) | one-hot
    head | kmean], where kmean (B, H, N, dh), given with global pooling, is the mean key before each query."""
    B, H, N, _ = q.shape
    log_norm = torch.log(torch.linalg.vector_norm(q.float(), dim=-1, keepdim=True) + 1e-6).to(q.dtype)
    head = torch.eye(H, device=q.device, dtype=q.dtype).view(1, H, 1, H).expand(B, H, N, H)
    parts = [q, log_norm, head]
    if kmean is not None:
        parts.append(kmean.to(q.dtype))
    return torch.cat(parts, -1)


def mean_before(x, dim=2):
    """Mean of the rows of x before each position along `dim` (zero for the first position): the running key mean
    the budget head sees with global pooling."""
    n = x.shape[dim]
    shape = [1] * x.dim()
    shape[dim] = n
    count = torch.arange(n, device=x.device).clamp(min=1).view(shape).to(x.dtype)
    return (x.cumsum(dim) - x) / count


def budget_label(leaf_mass, classes, cover=0.9):
    """Training target of the budget head. leaf_mass (..., wl) >= 0 is the attention weight on each of a query's
    leaves, best-first. Walking the leaves in that order, n is the count it takes before the running weight
    reaches `cover` of the total (plus the leaf that reaches it); the target is the first class not below n,
    i.e. the number of classes below n, and the last class when n is above them all.
    Returns (label (...) int64, has_mass (...) bool: queries whose leaves carry any weight)."""
    total = leaf_mass.sum(-1, keepdim=True)
    # the running weight never decreases, so the count of leaves still short of the cover is a sorted search
    short = torch.searchsorted(leaf_mass.cumsum(-1).contiguous(), (cover * total).contiguous())
    n = short.squeeze(-1) + 1
    ladder = torch.sort(classes.to(n.device)).values
    label = torch.bucketize(n, ladder).clamp(max=ladder.numel() - 1)
    return label, total.squeeze(-1) > 0
