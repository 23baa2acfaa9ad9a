"""DynAttention (reference attention_dyn.py) on this package's kernels.

With attn='seg' DynAttention is the parity twin of SegAttention (same parameters, same selection, same exact
attention; reference test_fast.py:47-64 checks exactly that), so it shares SegAttention's implementation.
The dynamic content tree (attn='dyn', dyntree.select_keys) is not implemented here and raises."""
from . import _ops
from .fastseg import SegAttention


def dedupe(cand, valid):
    """attention_dyn.py:12-17: keep only the first copy of every key position among the valid candidates."""
    return _ops.dedupe(cand, valid)


class DynAttention(SegAttention):
    def sparse_attend(self, q, k, v, out=None):
        if self.cfg.attn != 'seg':
            raise NotImplementedError("DynAttention with attn='%s' (dynamic content tree) is not implemented in "
                                      "treeattn_b200; attn='seg' is" % self.cfg.attn)
        return super().sparse_attend(q, k, v, out=out)
