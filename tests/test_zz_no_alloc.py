"""ta_lane_order_noalloc: the 2-means build's slot ordering with its scratch in the library's static device memory
(cudaGetSymbolAddress) instead of caller buffers. It must give exactly ta_lane_order's result and allocate nothing."""
import ctypes

import numpy as np
import pytest
import torch


def test_noalloc_rejects_oversize_without_gpu():
    """More slots than the static scratch holds: TA_ERR_ARG before any CUDA call."""
    from treeattn_b200 import _lib
    lib = _lib.load()
    buf = (ctypes.c_char * 64)()
    addr = ctypes.addressof(buf)
    addr += (16 - addr % 16) % 16
    rc = lib.ta_lane_order_noalloc(addr, 1, 1024 * 16, addr, 1, 4096, 1024, 16, 3, 9, addr, addr, None)
    assert rc == _lib.TA_ERR_ARG and 'static scratch' in _lib.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize('P,C,dh', [(8, 1024, 64), (96, 512, 32), (3, 16384, 16)])
def test_noalloc_matches_lane_order(P, C, dh):
    from treeattn_b200 import _lib, _ops
    dev = 'cuda'
    rng = np.random.default_rng(C + dh)
    keys = torch.as_tensor(rng.standard_normal((P, C, dh)).astype(np.float32)).to(dev)
    n = torch.as_tensor(rng.integers(0, C + 1, P)).to(dev)
    D = C.bit_length() - 2
    perm = torch.empty(P, C, device=dev, dtype=torch.int32)
    valid = torch.empty(P, C, device=dev, dtype=torch.uint8)
    pt, vt = torch.empty_like(perm), torch.empty_like(valid)
    _lib.call('ta_lane_order', _ops._p(keys), 1, C * dh, _ops._p(n), 1, P, C, dh, 3, D, _ops._p(perm),
              _ops._p(valid), _ops._p(pt), _ops._p(vt), _ops._stream(keys))
    perm2 = torch.empty_like(perm)
    valid2 = torch.empty_like(valid)
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    _lib.call('ta_lane_order_noalloc', _ops._p(keys), 1, C * dh, _ops._p(n), 1, P, C, dh, 3, D, _ops._p(perm2),
              _ops._p(valid2), _ops._stream(keys))
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == before
    assert torch.equal(perm, perm2) and torch.equal(valid, valid2)
    assert _ops.device_error()[0] == 0
