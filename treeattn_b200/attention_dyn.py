"""DynAttention (reference attention_dyn.py) on this package's kernels.

attention_dyn.py:31-121: the budget (fixed, or the learned head), the non-differentiable key selection - the
segment tree's (attn='seg', the parity twin of SegAttention that reference test_fast.py:47-64 checks) or the
dynamic content tree's (attn='dyn', dyntree.select_keys: ta_lane_order / ta_lane_sums / ta_lane_select) - then
exact softmax attention over [tree positions, neighbour positions, sink + local window], deduplicated, through
the differentiable sparse_attn (ta_sparse_attn / ta_sparse_attn_bwd), and the budget head's loss in training."""
from . import _ops
from .dyntree import select_keys
from .fastseg import SegAttention


def dedupe(cand, valid):
    """attention_dyn.py:12-17: keep only the first copy of every key position among the valid candidates."""
    return _ops.dedupe(cand, valid)


class DynAttention(SegAttention):
    def _select(self, q, k, lhat):
        if self.cfg.attn == 'dyn':
            return select_keys(q, k, lhat, self.cfg)
        return super()._select(q, k, lhat)

    def sparse_attend(self, q, k, v, out=None):
        if self.cfg.attn != 'dyn':
            return super().sparse_attend(q, k, v, out=out)
        o = self._sparse_attend_autograd(q, k, v)
        if out is not None:
            out.copy_(o)
            return out
        return o
