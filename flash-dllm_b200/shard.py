"""Sequence sharding across the GPUs of one node.

Sequences are independent work units (their own cache rows, block-table rows
and acceptance decisions), so N GPUs each take a contiguous shard of the
prompts and run the decode driver on a full model replica; nothing crosses
GPUs while decoding.  These helpers only split the prompts and gather the
results once at the end, over any ``torch.distributed`` backend (NCCL on the
GPUs, gloo for CPU tests).
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def shard_range(n_items: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous shard [start, end) of ``n_items`` for ``rank``; the first
    ``n_items % world`` ranks take one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def reduce_counters(times: Sequence[float], counts: Sequence[float], device=None, group=None) -> Tuple[List[float],
                                                                                                   List[float]]:
    """Max over ranks of each time and sum over ranks of each count (the
    whole-job throughput is sum(tokens) / max(time))."""
    dev = device if device is not None else torch.device("cpu")
    t = torch.tensor(list(times), dtype=torch.float64, device=dev)
    c = torch.tensor(list(counts), dtype=torch.float64, device=dev)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        dist.all_reduce(c, op=dist.ReduceOp.SUM, group=group)
    return t.tolist(), c.tolist()


def gather_responses(local: Sequence[Sequence[int]], start: int, n_items: int, device=None,
                     group=None) -> Optional[List[List[int]]]:
    """All ranks' token responses, ordered by global prompt index (every rank
    gets the full list); ``local[i]`` is the response of prompt ``start + i``."""
    dev = device if device is not None else torch.device("cpu")
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    longest = torch.tensor([max([len(r) for r in local], default=0)], dtype=torch.int64, device=dev)
    if world > 1:
        dist.all_reduce(longest, op=dist.ReduceOp.MAX, group=group)
    width = int(longest.item()) + 2
    buf = torch.full((n_items, width), -1, dtype=torch.int64, device=dev)
    for i, r in enumerate(local):
        buf[start + i, 0] = 1
        buf[start + i, 1] = len(r)
        buf[start + i, 2:2 + len(r)] = torch.tensor(list(r), dtype=torch.int64, device=dev)
    if world > 1:
        # each row is written by exactly one rank; the others hold -1 there
        mask = (buf[:, 0] == 1).to(torch.int64)
        contrib = (buf + 1) * mask[:, None]
        dist.all_reduce(contrib, op=dist.ReduceOp.SUM, group=group)
        buf = contrib - 1
    out = []
    for i in range(n_items):
        n = int(buf[i, 1])
        out.append(buf[i, 2:2 + n].tolist() if int(buf[i, 0]) == 1 else [])
    return out
