"""Env sharding over GPUs: one process per GPU, no collective on the step path.

Games are independent, so rank r of W owns a contiguous range of global env
indices and steps it with its own buffer; every random stream (setup deal,
action sampling, Gumbel noise, belief deals) is keyed by the *global* env
index (``env_base + e``), so each game plays out identically for any W.
The only exchange is at the end of a rollout: the int64[5] episode counters
(finished, red wins, blue wins, draws, sum of lengths) are all-gathered.

Works with any ``torch.distributed`` backend: NCCL on GPUs, gloo on CPU
(what the multi-rank CPU tests use).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """(env_base, n) of rank ``rank``: ``total`` envs split into ``world``
    contiguous ranges whose sizes differ by at most one (the first
    ``total % world`` ranks take one more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if total < 0:
        raise ValueError("total must be >= 0")
    q, r = divmod(total, world)
    n = q + (1 if rank < r else 0)
    base = rank * q + min(rank, r)
    return base, n


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1


def gather_episode_stats(stats: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather each rank's int64[5] episode counters: returns int64[W,5]
    (row r = rank r), on ``stats``'s device.  One collective, called by every
    rank at the same point (end of a rollout)."""
    if stats.dtype != torch.int64 or stats.numel() != 5:
        raise ValueError("stats must be int64[5]")
    w = _world(group)
    s = stats.reshape(5).contiguous()
    if w == 1:
        return s.reshape(1, 5).clone()
    out = torch.empty((w, 5), dtype=torch.int64, device=s.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, s, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), s, group=group)
    return out


def max_over_ranks(value: float, device: torch.device | str = "cpu", group=None) -> float:
    """The maximum of a per-rank scalar (timings are reported as the slowest
    rank's)."""
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if _world(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
