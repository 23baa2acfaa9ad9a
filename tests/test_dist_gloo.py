"""Multi-process (gloo, world size 2, CPU) tests of the sharding and gather helpers used by bench.py."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from treeattn_b200 import dist as tdist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        tdist.init('gloo', timeout_s=60)
        r, lr, w = tdist.env_rank_world()
        assert (r, w) == (rank, world)
        a, b = tdist.shard(13, rank, world)
        # each rank "decodes" its own sequences: token = sequence index * 10 + rank marker
        toks = torch.arange(a, b, dtype=torch.int64) * 10
        allt = tdist.gather_rows(toks.view(-1, 1))
        mx = tdist.max_over_ranks([float(rank + 1), -float(rank)], torch.device('cpu'))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, (a, b), allt.view(-1).tolist(), mx))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, 'error', repr(e), None))


def _worker_leaves(rank, world, port, q):
    """Rank 1 leaves between steps (before the gather, with nothing in flight); rank 0's gather must end with an
    error within the process group's short timeout instead of waiting for good."""
    import time
    import torch.distributed as dist
    from treeattn_b200 import dist as tdist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    tdist.init('gloo', timeout_s=5)
    dist.barrier()
    if rank == 1:
        q.put((rank, 'left', 0.0))
        return
    t0 = time.time()
    try:
        tdist.gather_rows(torch.zeros(3, 1, dtype=torch.int64))
        q.put((rank, 'no error', time.time() - t0))
    except Exception as e:  # the expected path: a closed connection or the timeout
        q.put((rank, 'error: ' + type(e).__name__, time.time() - t0))


def test_shard_partition():
    from treeattn_b200.dist import shard
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            parts = [shard(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in parts) - min(b - a for a, b in parts) <= 1


@pytest.mark.timeout(180)
def test_gloo_two_ranks():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=150) for _ in procs]
    for p in procs:
        p.join(timeout=30)
    res.sort()
    for rank, shard_, toks, mx in res:
        assert shard_ != 'error', toks
        assert toks == [i * 10 for i in range(13)]  # both ranks see all 13 sequences in order
        assert mx == [2.0, 0.0]
    assert res[0][1] == (0, 7) and res[1][1] == (7, 13)


@pytest.mark.timeout(180)
def test_gloo_rank_leaving_is_detected():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_leaves, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=150) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    assert res[1][1] == 'left'
    assert res[0][1].startswith('error'), res[0]
    assert res[0][2] < 60, res[0]
