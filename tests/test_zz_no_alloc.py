"""ta_lane_order_noalloc: the dynamic tree's slot ordering for callers that cannot allocate device memory (a program
that reserved the GPU's memory for its own pool and gives the library only views into it). Its scratch is a static
array inside the library instead of a caller buffer; it must give ta_lane_order's result, call after call, and leave
torch's allocator untouched.

This file is collected last on purpose, so that a run stopping at its first failure has already run every other
test; it also passes when run alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch


def test_noalloc_rejects_oversize_without_gpu():
    """More slots than the static scratch holds: TA_ERR_ARG with a message, before any CUDA call."""
    from treeattn_b200 import _lib
    lib = _lib.load()
    buf = (ctypes.c_char * 64)()
    addr = ctypes.addressof(buf)
    addr += (16 - addr % 16) % 16
    rc = lib.ta_lane_order_noalloc(addr, 1, 1024 * 16, addr, 1, 4096, 1024, 16, 3, 9, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'static scratch' in _lib.last_error()


def _inputs(rng, P, C, dh, dev):
    keys = torch.as_tensor(rng.standard_normal((P, C, dh)).astype(np.float32)).to(dev)
    n = torch.as_tensor(rng.integers(0, C + 1, P)).to(dev)
    return keys, n


@pytest.mark.gpu
@pytest.mark.parametrize('P,C,dh', [(8, 1024, 64), (96, 512, 32), (3, 16384, 16)])
def test_noalloc_matches_lane_order_twice(P, C, dh):
    """Two calls in a row on different inputs (the second sees the scratch the first left behind), each equal to
    ta_lane_order with caller scratch. Neither call allocates through torch; the second (after the first has loaded
    the library's kernels and looked up the scratch) leaves the device's free memory unchanged as well, which also
    catches an allocation inside the library that torch's counters cannot see."""
    from treeattn_b200 import _lib, _ops
    dev = 'cuda'
    rng = np.random.default_rng(C + dh)
    D = C.bit_length() - 2
    for call in range(2):
        keys, n = _inputs(rng, P, C, dh, dev)
        perm = torch.empty(P, C, device=dev, dtype=torch.int32)
        valid = torch.empty(P, C, device=dev, dtype=torch.uint8)
        pt, vt = torch.empty_like(perm), torch.empty_like(valid)
        _lib.call('ta_lane_order', _ops._p(keys), 1, C * dh, _ops._p(n), 1, P, C, dh, 3, D, _ops._p(perm),
                  _ops._p(valid), _ops._p(pt), _ops._p(vt), _ops._stream(keys))
        perm2 = torch.full_like(perm, -7)
        valid2 = torch.full_like(valid, 9)
        torch.cuda.synchronize()
        before = torch.cuda.memory_allocated()
        free_before = torch.cuda.mem_get_info()[0]
        _lib.call('ta_lane_order_noalloc', _ops._p(keys), 1, C * dh, _ops._p(n), 1, P, C, dh, 3, D, _ops._p(perm2),
                  _ops._p(valid2), _ops._stream(keys))
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == before
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free_before
        assert torch.equal(perm, perm2) and torch.equal(valid, valid2)
    assert _ops.device_error()[0] == 0
