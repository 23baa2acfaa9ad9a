"""Selection comparator shared by the parity tests.

The reference's torch.topk leaves the order of tied scores undefined, and two fp32 dot-product reductions
round differently, so selected sets are compared only for queries with no near-tie at any cut: a query is
excluded when, at some level, the best dropped valid candidate scores within TIE_REL (relative) of the last
kept one. Only valid slots are compared (invalid slots of torch.topk carry arbitrary ids).

Every comparison is logged (test, queries compared, queries excluded as ties, mismatches) so that the exclusions
can be audited: tests/conftest.py prints the log at the end of the run."""
import os

import numpy as np

TIE_REL = 1e-6
TIE_LOG = []


def record(n_compared, n_excluded, n_mismatch=0, what=''):
    """Adds one selection comparison to the run's log."""
    test = os.environ.get('PYTEST_CURRENT_TEST', '?').split(' ')[0]
    TIE_LOG.append((test, what, int(n_compared), int(n_excluded), int(n_mismatch)))


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
    res = int((~eq & comp).sum()), int(comp.sum()), int(exclude.sum())
    record(res[1], res[2], res[0])
    return res


def tied(margin):
    return np.asarray(margin) <= TIE_REL
