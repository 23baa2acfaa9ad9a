"""Selection comparator shared by the parity tests.

The reference's torch.topk leaves the order of tied scores undefined, and two fp32 dot-product reductions
round differently, so selected sets are compared only for queries with no near-tie at any cut: a query is
excluded when, at some level, the best dropped valid candidate scores within TIE_REL (relative) of the last
kept one. Only valid slots are compared (invalid slots of torch.topk carry arbitrary ids)."""
import numpy as np

TIE_REL = 1e-6


def valid_sets(ids, vld):
    """(…, w) ids + validity -> (…, w) int64 array of the valid ids sorted ascending, padded with a sentinel."""
    ids = np.asarray(ids, np.int64)
    vld = np.asarray(vld, bool)
    big = np.iinfo(np.int64).max
    return np.sort(np.where(vld, ids, big), -1)


def compare_sets(ids_a, vld_a, ids_b, vld_b, exclude=None):
    """Returns (n_mismatch, n_compared, n_excluded) over the leading query dims."""
    sa, sb = valid_sets(ids_a, vld_a), valid_sets(ids_b, vld_b)
    w = max(sa.shape[-1], sb.shape[-1])
    big = np.iinfo(np.int64).max
    pad = lambda s: np.concatenate([s, np.full(s.shape[:-1] + (w - s.shape[-1],), big)], -1)
    eq = (pad(sa) == pad(sb)).all(-1)
    if exclude is None:
        exclude = np.zeros(eq.shape, bool)
    comp = ~exclude
    return int((~eq & comp).sum()), int(comp.sum()), int(exclude.sum())


def tied(margin):
    return np.asarray(margin) <= TIE_REL
