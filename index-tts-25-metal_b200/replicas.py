"""Request-parallel serving across GPUs: one decoder replica per GPU.

Batch-1 decode of the GPT does not shard (every layer's GEMV needs the previous
layer's full output), so several GPUs serve independent synthesis requests,
each GPU with its own weights, KV arena and stream, and nothing on the data
path crosses GPUs.  This module holds the host logic of that mode:

* ``serving_requests`` - the synthetic request mix of the serving workload
  (text length uniform in [20, 400], target code count uniform in [100, 1500]);
* ``partition`` - which requests a rank serves (round-robin by request index,
  or longest-first greedy balancing of the decode work);
* ``aggregate`` - whole-job throughput from per-rank token counts and times:
  tokens summed, wall time the maximum over ranks (the slowest replica ends the
  job).  It runs over any ``torch.distributed`` process group (NCCL on the GPU
  box, gloo in the CPU tests); a rank that died or never joined makes the
  collective fail within the group's timeout, which surfaces here as
  ``ReplicaFailure``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np


@dataclass(frozen=True)
class Request:
    index: int
    text_len: int
    codes: int


class ReplicaFailure(RuntimeError):
    """A peer replica failed or left before the collective completed."""


def serving_requests(n: int = 64, seed: int = 7) -> List[Request]:
    """The serving workload's requests: seeded text lengths in [20, 400] and
    target code counts in [100, 1500] (both inclusive)."""
    r = np.random.default_rng(seed)
    text = r.integers(20, 401, n)
    codes = r.integers(100, 1501, n)
    return [Request(i, int(t), int(c)) for i, (t, c) in enumerate(zip(text, codes))]


def partition(requests: Sequence[Request], world: int, rank: int, policy: str = "round_robin") -> List[Request]:
    """The requests rank `rank` of `world` serves, in serving order.

    ``round_robin``: request i goes to rank i % world.  ``longest_first``:
    requests sorted by decreasing decode work (codes, then text length, then
    index) go one by one to the rank with the least work so far (ties: lowest
    rank), which bounds the imbalance of ragged lengths.  Every rank computes
    the same assignment locally; no communication is needed."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    if policy == "round_robin":
        return [q for q in requests if q.index % world == rank]
    if policy != "longest_first":
        raise ValueError(f"unknown policy {policy!r}")
    load = [0] * world
    mine: List[Request] = []
    for q in sorted(requests, key=lambda q: (-q.codes, -q.text_len, q.index)):
        k = min(range(world), key=lambda i: (load[i], i))
        load[k] += q.codes
        if k == rank:
            mine.append(q)
    return mine


def aggregate(tokens: int, seconds: float, group=None, device: Optional[str] = None) -> dict:
    """Whole-job throughput: total tokens over all ranks divided by the
    slowest rank's time.  Without an initialised process group this is the
    single-rank value."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return {"tokens": int(tokens), "seconds": float(seconds), "value": tokens / seconds if seconds > 0 else 0.0,
                "world": 1}
    t = torch.tensor([float(tokens)], dtype=torch.float64, device=device)
    s = torch.tensor([float(seconds)], dtype=torch.float64, device=device)
    try:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(s, op=dist.ReduceOp.MAX, group=group)
    except Exception as e:  # a peer died, left or timed out
        raise ReplicaFailure(f"replica collective failed: {e}") from e
    total, slowest = float(t.item()), float(s.item())
    return {"tokens": int(total), "seconds": slowest, "value": total / slowest if slowest > 0 else 0.0,
            "world": dist.get_world_size(group)}
