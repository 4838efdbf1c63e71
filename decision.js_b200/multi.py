"""One process per GPU (torchrun): each rank runs its token-balanced shard of the requests and the results come
back to every rank in request order through a host gather. There is no device collective on the data path: the
requests are independent, and a pass's outputs are a few hundred KB."""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .decision import shard


def _rows(local):
    """(width, dtype) when every result is a 1-D numpy array of one width and dtype (pooled embeddings, per-option
    logits of one width), else None."""
    if not local or not all(isinstance(x, np.ndarray) and x.ndim == 1 for x in local):
        return None
    w, dt = local[0].shape[0], local[0].dtype
    if dt not in (np.float32, np.float64) or any(x.shape[0] != w or x.dtype != dt for x in local):
        return None
    return w, dt


def run_sharded(requests, sizes, engine_fn):
    """Runs engine_fn on this rank's shard of `requests` (sizes: tokens per request) and returns the results of
    all ranks, in request order. Every rank computes the same shards, so it knows how many results each rank
    holds: results that are rows of one width (embeddings) are gathered as one tensor (one small agreement on the
    width, then one all-gather of the rows, padded to the largest shard); anything else as pickled objects. A rank
    that fails makes the gather fail on the others (their process group's timeout bounds the wait), so a batch
    never hangs."""
    rank, world = dist.get_rank(), dist.get_world_size()
    shards = shard(sizes, world)
    a, b = shards[rank]
    local = list(engine_fn(requests[a:b])) if b > a else []
    # every rank takes the same collective steps: agree first on whether all hold rows of one width
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    rows = _rows(local)
    big = 1 << 40  # an empty shard takes part without a width: its entries never win the maxima
    if rows:
        vals = [rows[0], -rows[0], int(rows[1] == np.float64), -int(rows[1] == np.float64), -1]
    elif b == a:
        vals = [0, -big, 0, -big, -1]
    else:
        vals = [0, -big, 0, -big, 0]  # results that are not rows: everyone takes the object path
    agree = torch.tensor(vals, dtype=torch.int64, device=dev)
    dist.all_reduce(agree, op=dist.ReduceOp.MAX)
    wmax, wmin, fmax, fmin = int(agree[0]), -int(agree[1]), int(agree[2]), -int(agree[3])
    all_rows = -int(agree[4]) == 1  # the minimum over ranks of "rows or empty"
    if all_rows and wmax > 0 and wmin == wmax and fmin == fmax:
        counts = [e - s for s, e in shards]
        most = max(counts)
        dt = torch.float64 if fmax else torch.float32
        buf = torch.zeros((most, wmax), dtype=dt, device=dev)
        if local:
            buf[:len(local)] = torch.from_numpy(np.stack(local)).to(dev)
        gathered = torch.empty((world * most, wmax), dtype=dt, device=dev)
        dist.all_gather_into_tensor(gathered, buf)
        host = gathered.cpu().numpy()
        out = []
        for r, c in enumerate(counts):
            out.extend(host[r * most:r * most + c])
        return [np.array(x) for x in out]
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
