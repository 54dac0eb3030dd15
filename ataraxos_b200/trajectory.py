"""Trajectory ring and search rollouts on top of StrategoRolloutBuffer.

``TrajectoryBuffer`` is the self-play ring of the north-star contract
(benchmark config 4): T slots x N envs, each slot holding the observation
(bf16 infostate, compact 76-plane layout by default), the bit-packed legal
mask, the sampled action (int16 src*100+dst), its log-prob, and the reward /
done of the transition taken from that slot.  ``rollout(k)`` runs k plies in
ONE kernel launch per call: every env's record stays on chip while the ply
loop writes straight into the ring.

``BeliefRollouts`` is the search batch (benchmark config 5): each root is
copied into ``samples_per_root`` envs whose opponent identities are re-dealt
consistently with the side to move's information, then every sample plays
``depth`` plies; per-ply legal masks and the terminal values come back.
The intended callers are the batched versions of
stratego/training/selfplay.py:190-268 (self-play) and
stratego/search/rollouts.py:46-118 (search rollouts).
"""

from __future__ import annotations

import ctypes

import torch

from . import _capi as C
from .buffer import COMPACT_CHANNELS, MASK_BITS_BYTES, NUM_CHANNELS, NUM_SQUARES, StrategoRolloutBuffer, _POLICIES


class TrajectoryBuffer:
    """T x N ring of (observation, mask, action, log-prob, reward, done)."""

    def __init__(
        self,
        buffer: StrategoRolloutBuffer,
        T: int,
        *,
        obs_dtype: torch.dtype | None = torch.bfloat16,
        obs_layout: str = "compact",
        mask_format: str = "bits",
        policy: str = "gumbel",
        store_hash: bool = False,
    ) -> None:
        if T < 1:
            raise RuntimeError("T must be >= 1")
        if policy not in _POLICIES:
            raise RuntimeError(f"unknown policy {policy!r}")
        self.buf = buffer
        self.T = int(T)
        self.policy = policy
        n, dev = buffer.n_games, buffer.device
        self.obs_layout = obs_layout
        self.obs = None
        if obs_dtype is not None:
            chans = COMPACT_CHANNELS if obs_layout == "compact" else NUM_CHANNELS
            self.obs = torch.zeros((T, n, chans, 10, 10), dtype=obs_dtype, device=dev)
        self.mask_format = mask_format
        self.mask = None
        if mask_format == "bits":
            self.mask = torch.zeros((T, n, MASK_BITS_BYTES), dtype=torch.uint8, device=dev)
        elif mask_format == "u8":
            self.mask = torch.zeros((T, n, NUM_SQUARES, NUM_SQUARES), dtype=torch.uint8, device=dev)
        self.action = torch.full((T, n), -1, dtype=torch.int16, device=dev)
        self.logprob = torch.zeros((T, n), dtype=torch.float32, device=dev)
        self.reward = torch.zeros((T, n), dtype=torch.float32, device=dev)
        self.done = torch.zeros((T, n), dtype=torch.uint8, device=dev)
        self.hash = torch.zeros((T, n), dtype=torch.int64, device=dev) if store_hash else None
        self.stats = torch.zeros(5, dtype=torch.int64, device=dev)
        self.slot = 0  # slot holding the current state

    def _traj(self) -> C.SbTraj:
        obs = self.obs
        return C.SbTraj(
            infostate=None if obs is None else obs.data_ptr(),
            info_dtype=C.SB_DTYPE_F32 if obs is None or obs.dtype == torch.float32 else C.SB_DTYPE_BF16,
            info_layout=C.SB_LAYOUT_COMPACT if self.obs_layout == "compact" else C.SB_LAYOUT_DENSE_LIVE,
            mask_u8=self.mask.data_ptr() if self.mask_format == "u8" else None,
            mask_bits=self.mask.data_ptr() if self.mask_format == "bits" else None,
            action=self.action.data_ptr(),
            logprob=self.logprob.data_ptr(),
            reward=self.reward.data_ptr(),
            done=self.done.data_ptr(),
            hash=None if self.hash is None else self.hash.data_ptr(),
            stats=self.stats.data_ptr(),
            n_slots=self.T,
            slot0=self.slot,
        )

    def _run(self, n_plies: int, auto_reset: bool) -> None:
        b = self.buf
        pol = C.SbPolicy(kind=_POLICIES[self.policy], reserved=0, logits=None)
        tr = self._traj()
        if b.n_games:
            b._call("sb_rollout", b.ply, ctypes.byref(pol), int(auto_reset), int(n_plies), ctypes.byref(tr))

    def prime(self) -> None:
        """Observe the current state into the current slot (and sample its action)."""
        self._run(0, False)

    def rollout(self, n_plies: int, auto_reset: bool = True) -> None:
        """Play n_plies plies in one launch, filling slots slot+1 .. slot+n_plies (mod T)."""
        if n_plies < 1:
            raise RuntimeError("n_plies must be >= 1")
        self._run(n_plies, auto_reset)
        self.buf.ply += n_plies
        self.slot = (self.slot + n_plies) % self.T


class BeliefRollouts:
    """Search batch: belief-resampled copies of root states rolled out for ``depth`` plies."""

    def __init__(self, roots: StrategoRolloutBuffer, samples_per_root: int, depth: int = 40, *,
                 policy: str = "uniform", seed: int = 0, mask_format: str = "bits") -> None:
        self.roots = roots
        self.k = int(samples_per_root)
        self.depth = int(depth)
        n = roots.n_games * self.k
        self.samples = StrategoRolloutBuffer(
            n, roots.device_id, seed=seed, zobrist=roots._zobrist.cpu(), no_attack_limit=roots.no_attack_limit,
            max_game_length=roots.max_game_length, two_square_limit=roots.two_square_limit, rules=roots.rules)
        self.root_of = torch.arange(roots.n_games, device=roots.device).repeat_interleave(self.k)
        self.traj = TrajectoryBuffer(self.samples, self.depth + 1, obs_dtype=None, mask_format=mask_format,
                                     policy=policy)

    def resample(self) -> None:
        self.samples.resample_from(self.roots, self.root_of)

    def run(self) -> dict[str, torch.Tensor]:
        """Resample beliefs, then roll every sample ``depth`` plies without auto-reset.

        Returns per-rollout ``masks`` [depth+1, n, ...] (legal masks of every
        visited state, slot 0 = the resampled root), ``actions`` [depth+1, n],
        ``terminal_value`` [n] (player-0 reward at the end: +1/-1, 0 for a
        draw or an unfinished rollout) and ``done`` [n].
        """
        self.resample()
        self.traj.slot = 0
        self.traj.prime()
        self.traj.rollout(self.depth, auto_reset=False)
        return {
            "masks": self.traj.mask,
            "actions": self.traj.action,
            "terminal_value": self.traj.reward[self.depth - 1] if self.depth else self.samples.compute_reward_pl0(),
            "done": self.traj.done[self.depth - 1].view(torch.bool) if self.depth else self.samples.get_terminated(),
        }
