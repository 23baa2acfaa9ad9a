import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200, sm_100a) and the built library')


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason='no CUDA GPU in this environment')
    for it in items:
        if 'gpu' in it.keywords:
            it.add_marker(skip)


def pytest_terminal_summary(terminalreporter):
    """Selection comparisons of the run: per test, the queries compared, those excluded as fp32 ties at a cut
    (tests/_compare.py) and the mismatches."""
    try:
        from tests._compare import TIE_LOG
    except Exception:  # pragma: no cover
        return
    if not TIE_LOG:
        return
    agg = {}
    for test, what, n, x, bad in TIE_LOG:
        a = agg.setdefault((test, what), [0, 0, 0])
        a[0] += n
        a[1] += x
        a[2] += bad
    tr = terminalreporter
    tr.section('selection comparisons (queries compared / excluded as fp32 ties / mismatches)')
    tot = [0, 0, 0]
    for (test, what), (n, x, bad) in sorted(agg.items()):
        frac = x / max(n + x, 1)
        tr.write_line('%-90s compared %8d  excluded %6d (%.4f%%)  mismatches %d' % (
            test + (' [%s]' % what if what else ''), n, x, 100 * frac, bad))
        tot = [tot[0] + n, tot[1] + x, tot[2] + bad]
    tr.write_line('%-90s compared %8d  excluded %6d (%.4f%%)  mismatches %d' % (
        'TOTAL', tot[0], tot[1], 100 * tot[1] / max(tot[0] + tot[1], 1), tot[2]))
