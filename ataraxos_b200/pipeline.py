"""Asynchronous host-driven stepping: a GPU's games split into groups that
take turns, so the host's round trip of one group hides behind the kernels
of the others.

A host-side loop over ``step_host`` is synchronous: the host waits for a
ply's results before it can send the next ply's actions, and the GPU idles
for the launch, completion and host wake-up of every step.  ``StepPipeline``
splits the games into ``groups`` buffers (contiguous global env ranges, each
with its own CUDA stream) and exposes the send / receive form of a batched
environment: ``send(g, actions)`` queues group ``g``'s next ply and returns
at once, ``recv(g)`` waits for that ply's results.  A loop that receives one
group, computes its actions and sends it, then turns to the next group keeps
the GPU busy with the other groups' plies meanwhile.

Every random stream is keyed by the global env index, so a game plays out
exactly as it does in one buffer of all the games, whatever the number of
groups.  Each group's ply is one ``sb_step_host`` call (actions read from
page-locked host memory, reward / done / next action written into page-locked
memory), so the data crossing PCIe per ply is that of ``step_host``.

This is the host loop of ``SelfPlayGenerator.generate_games``
(stratego/training/selfplay.py:190-268) with its games split into groups that
the policy serves in turn.
"""

from __future__ import annotations

import torch

from . import sharding
from .buffer import HostStepOutput, StrategoRolloutBuffer


class StepPipeline:
    """``n_games`` games on one GPU in ``groups`` independently stepped buffers."""

    def __init__(self, n_games: int, device_id: int = 0, *, groups: int = 2, env_base: int = 0,
                 **buffer_kwargs) -> None:
        if groups < 1:
            raise RuntimeError("groups must be >= 1")
        if n_games < groups:
            raise RuntimeError("every group needs at least one game")
        self.n_games, self.device = int(n_games), torch.device("cuda", int(device_id))
        self.buffers: list[StrategoRolloutBuffer] = []
        self.ranges: list[tuple[int, int]] = []
        for g in range(groups):
            off, n = sharding.shard_range(self.n_games, groups, g)
            self.buffers.append(StrategoRolloutBuffer(n, device_id, env_base=env_base + off, **buffer_kwargs))
            self.ranges.append((off, n))
        self.streams = [torch.cuda.Stream(self.device) for _ in range(groups)]
        # page-locked int64 action staging, one per group (read in place by the kernel)
        self.actions = [torch.zeros(max(n, 1), dtype=torch.int64, pin_memory=True)[:n] for _, n in self.ranges]
        self._pending = [None] * groups

    @property
    def groups(self) -> int:
        return len(self.buffers)

    def reset_all_from_pool(self) -> None:
        for b, s in zip(self.buffers, self.streams):
            with torch.cuda.stream(s):
                b.reset_all_from_pool()

    def send(self, g: int, actions: torch.Tensor | None = None, *, policy: str = "uniform",
             auto_reset: bool = True, observe: bool = True) -> None:
        """Queue one ply of group ``g`` and return without waiting.  ``actions``:
        CPU int64 [n_g] (copied into the group's page-locked staging, which the
        kernel reads in place) or None (the device's own proposals).  The
        group must have no ply in flight."""
        if self._pending[g] is not None:
            raise RuntimeError(f"group {g} has a ply in flight: recv({g}) first")
        a = None
        if actions is not None:
            a = self.actions[g]
            if actions.data_ptr() != a.data_ptr():
                a.copy_(actions)
        self._pending[g] = self.buffers[g].step_host(a, policy=policy, auto_reset=auto_reset, observe=observe,
                                                     sync=False, stream=self.streams[g])

    def recv(self, g: int) -> HostStepOutput:
        """Wait for group ``g``'s ply in flight and return its results (valid
        until the group's next ``send``)."""
        r = self._pending[g]
        if r is None:
            raise RuntimeError(f"group {g} has no ply in flight")
        self.streams[g].synchronize()
        self._pending[g] = None
        return r

    def synchronize(self) -> None:
        for s in self.streams:
            s.synchronize()
