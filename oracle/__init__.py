"""CPU oracle of treeattn's segment-tree sparse-attention path, its dynamic content tree and the block forest
(numpy, fp32).

TEST INFRASTRUCTURE ONLY. The product (treeattn_b200) never imports this package; only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference legs use it, and only as the checker or
as the timed CPU baseline. It is pinned against golden vectors produced by the reference itself
(tests/golden/make_golden.py, tests/test_oracle_golden.py).
"""
from .seg_oracle import *  # noqa: F401,F403
from .dyn_oracle import *  # noqa: F401,F403
from .forest_oracle import *  # noqa: F401,F403
