"""One process per GPU (torchrun): each rank runs its token-balanced shard of the requests and the results come
back to every rank in request order through a host gather. There is no device collective on the data path: the
requests are independent, and a pass's outputs are a few hundred KB."""
from __future__ import annotations

import torch
import torch.distributed as dist

from .decision import shard


def run_sharded(requests, sizes, engine_fn):
    """Runs engine_fn on this rank's shard of `requests` (sizes: tokens per request) and returns the results of
    all ranks, in request order. A rank that fails makes the gather fail on the others (their process group's
    timeout bounds the wait), so a batch never hangs."""
    rank, world = dist.get_rank(), dist.get_world_size()
    a, b = shard(sizes, world)[rank]
    local = list(engine_fn(requests[a:b])) if b > a else []
    parts = [None] * world
    dist.all_gather_object(parts, (a, local))
    out = []
    for _, loc in sorted(parts, key=lambda p: p[0]):
        out.extend(loc)
    return out


def max_over_ranks(x: float, device=None) -> float:
    """The largest value of x over the ranks (timings are reported as the slowest rank's)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
