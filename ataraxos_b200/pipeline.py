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
groups.  Each group's ply is one ``sb_step_host`` call on prebuilt arguments
(actions read in place from the pipeline's page-locked staging, reward / done /
next action written by the kernel into the group buffer's page-locked result
block), so the data crossing PCIe per ply is that of ``step_host``.

This is the host loop of ``SelfPlayGenerator.generate_games``
(stratego/training/selfplay.py:190-268) with its games split into groups that
the policy serves in turn.
"""

from __future__ import annotations

import ctypes

import torch

from . import _capi as C
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
        # per (group, policy, host actions?): the prebuilt arguments of its
        # sb_step_host call (the pipeline's own io blocks, the buffer's mapped
        # result block), so a send is one native call
        self._fast: dict = {}

    def _fast_call(self, g: int, policy: str, host_actions: bool):
        key = (g, policy, host_actions)
        c = self._fast.get(key)
        if c is None:
            b = self.buffers[g]
            h = b._host_io()
            io = C.SbHostIo(actions_host=self.actions[g].data_ptr() if host_actions else None, actions_dev=None,
                            back_dev=None, back_host=None, back_bytes=0, sync=0, reserved=0)
            pol = b._policy(policy, None)
            c = self._fast[key] = (h["fn"], h["st"], io, ctypes.byref(io), pol, ctypes.byref(pol),
                                   h["out"]["mapped"][True], self.streams[g].cuda_stream, h["ret"]["mapped"][True])
        return c

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
                if actions.shape != a.shape:
                    raise RuntimeError(f"group {g} takes actions of shape {tuple(a.shape)}")
                a.copy_(actions)
        b = self.buffers[g]
        if not (auto_reset and observe):
            self._pending[g] = b.step_host(a, policy=policy, auto_reset=auto_reset, observe=observe, sync=False,
                                           stream=self.streams[g])
            return
        # (the io block and the policy ride along in the tuple to stay alive)
        fn, st, _, io, _, pol, out, stream, ret = self._fast_call(g, policy, a is not None)
        if torch.cuda.current_device() != self.device.index:
            with torch.cuda.device(self.device):
                rc = fn(st, io, b._ply, pol, 1, out, stream)
        else:
            rc = fn(st, io, b._ply, pol, 1, out, stream)
        if rc:
            C.check(rc)
        b._ply += 1
        self._pending[g] = ret

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
