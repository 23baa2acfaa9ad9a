"""Multi-GPU decode: one process per GPU, sequences sharded across ranks.

The segment-tree path shards by sequence: every tree, KV cache and selection belongs to one (b, h), so a rank
decodes its own sequences with no communication in the decode step. Collectives (NCCL on GPUs, gloo in CPU tests)
are used only outside the step: gathering generated tokens and reducing timings / metrics.
"""
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def env_rank_world():
    """(rank, local_rank, world_size) from the torchrun environment (defaults for a single process)."""
    return (int(os.environ.get('RANK', '0')), int(os.environ.get('LOCAL_RANK', '0')),
            int(os.environ.get('WORLD_SIZE', '1')))


def init(backend='nccl', timeout_s=600, device=None):
    """Initialise the default process group from the environment (MASTER_ADDR/PORT set by torchrun)."""
    if dist.is_initialized():
        return
    kw = dict(timeout=timedelta(seconds=timeout_s))
    if device is not None and backend == 'nccl':
        kw['device_id'] = device
    dist.init_process_group(backend, **kw)


def shard(n, rank, world):
    """Contiguous [start, end) of n items owned by `rank` (sizes differ by at most one)."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_rows(t, group=None):
    """All-gather a (B_local, ...) tensor whose B_local may differ per rank -> (sum B, ...) in rank order."""
    world = dist.get_world_size(group)
    n = torch.tensor([t.shape[0]], device=t.device, dtype=torch.int64)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    m = max(sizes)
    pad = torch.zeros((m,) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
    pad[:t.shape[0]] = t
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], 0)


def max_over_ranks(values, device):
    """Elementwise maximum of a list of floats over all ranks (timings are reported as the max over ranks)."""
    t = torch.tensor(list(values), device=device, dtype=torch.float64)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()
