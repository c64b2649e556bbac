"""Env sharding across GPUs: one process per GPU, contiguous env ranges, no collective
on the plan path.

Independent environments are the natural partition of the planning hot path
(the reference plans env batches serially on one GPU,
``lewm/solvers/icem.py:501``). Each rank owns ``env_range(n_envs, rank, world)``
and plans it on its own device; results are gathered to rank 0 on the host
after the plans finish (``gather_plans``), outside any timed region.
"""

from __future__ import annotations

from typing import Callable, Dict, List, Optional, Tuple

import torch


def env_range(n_envs: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, end) of the envs owned by ``rank`` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    if n_envs < 0:
        raise ValueError("n_envs must be >= 0")
    base, extra = divmod(n_envs, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_inputs(tensors: Dict[str, torch.Tensor], rank: int, world: int) -> Dict[str, torch.Tensor]:
    """Slice every (n_envs, ...) tensor to this rank's env range."""
    n = None
    for v in tensors.values():
        if n is None:
            n = int(v.shape[0])
        elif int(v.shape[0]) != n:
            raise ValueError("all sharded tensors need the same leading env dimension")
    s, e = env_range(n or 0, rank, world)
    return {k: v[s:e] for k, v in tensors.items()}


def plan_shard(plan_fn: Callable[..., Tuple[torch.Tensor, ...]], inputs: Dict[str, torch.Tensor], rank: int,
               world: int, **kw) -> Tuple[torch.Tensor, ...]:
    """Run ``plan_fn`` on this rank's envs. ``plan_fn(**shard, **kw)`` returns per-env tensors."""
    shard = shard_inputs(inputs, rank, world)
    if next(iter(shard.values())).shape[0] == 0:
        return tuple()
    return plan_fn(**shard, **kw)


def gather_plans(local: Tuple[torch.Tensor, ...], n_envs: int, tail_shapes: List[Tuple[int, ...]],
                 group=None) -> Optional[List[torch.Tensor]]:
    """Host-side gather of per-env outputs to rank 0 (pads uneven shards, then trims).

    ``local[i]`` has shape (envs of this rank,) + ``tail_shapes[i]``; an empty
    tuple means this rank owns no env. Runs after planning; it is the only
    communication and is not on the plan path. Returns the outputs concatenated
    in env order on rank 0 and None elsewhere.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    per = -(-n_envs // world)
    out: Optional[List[torch.Tensor]] = [] if rank == 0 else None
    for i, tail in enumerate(tail_shapes):
        buf = torch.zeros((per,) + tuple(tail), dtype=torch.float32)
        if local:
            t = local[i].detach().to("cpu", torch.float32)
            buf[: t.shape[0]] = t
        parts = [torch.zeros_like(buf) for _ in range(world)] if rank == 0 else None
        dist.gather(buf, parts, dst=0, group=group)
        if rank == 0:
            rows = []
            for r in range(world):
                s, e = env_range(n_envs, r, world)
                rows.append(parts[r][: e - s])
            out.append(torch.cat(rows, 0))
    return out
