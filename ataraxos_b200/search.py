"""Batched test-time search over the B200 simulator.

``BatchedSearch.search(roots)`` is the batched counterpart of
``SearchEngine.search`` (stratego/search/mirror_descent.py:115-154), run for
every game of a ``StrategoRolloutBuffer`` of root positions at once:

  1. the legal moves of each root (ascending ``src*100+dst``) and
     ``n_configs = max(1, n_rollouts // n_legal)`` per root (:127, :135);
  2. one simulator game per (root, legal move, config): a copy of the root
     whose hidden opponent identities are re-dealt by the simulator's belief
     resampling (``resample_from``; with ``resample=False`` a plain copy, which
     is what the reference's loop amounts to, since it never applies its
     sampled configs, :139-146);
  3. the move applied, then ``depth - 1`` plies sampled from the move
     network's policy and the value head's ``P(win) - P(loss)`` at the end
     (``BatchedRolloutEngine.rollout``, rollouts.py:106-118);
  4. ``q`` = the mean over a move's configs (:146), the network's legal
     probabilities at the root (:120-126), the magnet policy (uniform piece,
     then uniform move of that piece, :156-177), the closed-form mirror-descent
     policy :func:`compute_search_policy` (:32-76) and one move sampled from it.

Differences from the reference, all deliberate: configurations come from the
simulator's uniform belief resampling (every deal consistent with what the
side to move has seen), not from a belief network's autoregressive decoder
(stratego/search/belief_sampler.py:36-105); rollouts keep the simulator's own
move history and trackers; the final move is drawn with a seeded torch
generator instead of ``np.random.choice``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .buffer import NUM_ACTIONS, NUM_SQUARES, StrategoRolloutBuffer
from .selfplay import BatchedRolloutEngine, NetFn, _net_out

R_PROPPLY = 160  # record byte offset of the cached proposal's ply (int32; -1 = no cached proposal)


def compute_search_policy(q: torch.Tensor, net_probs: torch.Tensor, magnet_probs: torch.Tensor,
                          alpha: float = 0.002, beta: float = 0.02, legal: torch.Tensor | None = None) -> torch.Tensor:
    """``pi proportional to [exp(q) rho^alpha pi_theta^beta]^(1/(alpha+beta))``
    row by row (mirror_descent.py:32-76), in float64 like the reference's
    numpy arrays: log-space, ``eps = 1e-8`` inside both logs, the row maximum
    subtracted before exponentiation, normalised to sum to 1.  ``legal``
    (bool, same shape) marks the entries of each row; the rest are 0."""
    eps = 1e-8
    q, net, mag = (x.to(torch.float64) for x in (q, net_probs, magnet_probs))
    log_unnorm = (q + alpha * torch.log(mag + eps) + beta * torch.log(net + eps)) / (alpha + beta)
    if legal is not None:
        log_unnorm = log_unnorm.masked_fill(~legal, float("-inf"))
    log_unnorm = log_unnorm - log_unnorm.max(dim=-1, keepdim=True).values
    pi = torch.exp(log_unnorm)
    return pi / pi.sum(dim=-1, keepdim=True)


def magnet_policy(mask: torch.Tensor) -> torch.Tensor:
    """``rho`` over the flat actions of legal masks ``[R,100,100]`` (bool):
    every movable piece gets ``1 / n_pieces``, split evenly over its legal
    moves (mirror_descent.py:156-177); float64 ``[R,10000]``."""
    m = mask.to(torch.float64)
    per_src = m.sum(-1)                                   # [R,100] moves of each source square
    n_pieces = (per_src > 0).sum(-1, keepdim=True)        # [R,1]
    rho = m / (per_src.clamp(min=1) * n_pieces.clamp(min=1)).unsqueeze(-1)
    return rho.reshape(mask.shape[0], NUM_ACTIONS)


def copy_games(dst: StrategoRolloutBuffer, src: StrategoRolloutBuffer, src_of: torch.Tensor) -> None:
    """Game ``e`` of ``dst`` becomes a copy of game ``src_of[e]`` of ``src``
    (record, chase rings, ISF two-square state), its cached proposal dropped."""
    idx = src_of.to(src.device, torch.int64)
    n = dst.n_games
    dst._records[:n] = src._records.index_select(0, idx)
    dst._records[:n, R_PROPPLY:R_PROPPLY + 4] = 255
    dst._ring[:n] = src._ring.index_select(0, idx)
    if src._isf is not None and dst._isf is not None:
        dst._isf[:n] = src._isf.index_select(0, idx)


@dataclass
class SearchResult:
    """Outcome of one batched search over R roots."""

    action: torch.Tensor       # [R] int64 chosen move src*100+dst (-1: no legal move)
    policy: torch.Tensor       # [R,10000] float64 search policy over flat actions (0 off the legal moves)
    q: torch.Tensor            # [R,10000] float64 mean rollout value per legal move (0 elsewhere)
    net_probs: torch.Tensor    # [R,10000] float64 renormalised network probabilities of the legal moves
    magnet: torch.Tensor       # [R,10000] float64 magnet policy
    n_configs: torch.Tensor    # [R] int64 configs (rollouts) per legal move
    values: torch.Tensor       # [S] float32 value of every rollout, samples ordered (root, move, config)
    legal: torch.Tensor        # [S] int64 the first move of every rollout
    root_of: torch.Tensor      # [S] int64 the root of every rollout


class BatchedSearch:
    """Search for every root game at once (mirror_descent.py:82-154)."""

    def __init__(self, move_net: NetFn, *, n_rollouts: int = 1000, depth: int = 40, alpha: float = 0.002,
                 beta: float = 0.02, resample: bool = True, seed: int = 0,
                 obs_dtype: torch.dtype = torch.float32) -> None:
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.move_net = move_net
        self.n_rollouts, self.depth = int(n_rollouts), int(depth)
        self.alpha, self.beta = float(alpha), float(beta)
        self.resample = bool(resample)
        self.seed = int(seed)
        self.obs_dtype = obs_dtype
        self.rollouts = BatchedRolloutEngine(move_net, obs_dtype=obs_dtype)
        self._calls = 0

    def _samples(self, roots: StrategoRolloutBuffer, root_of: torch.Tensor) -> StrategoRolloutBuffer:
        s = StrategoRolloutBuffer(
            int(root_of.numel()), roots.device_id, seed=self.seed + self._calls, zobrist=roots._zobrist,
            no_attack_limit=roots.no_attack_limit, max_game_length=roots.max_game_length,
            two_square_limit=roots.two_square_limit, obs_dtype=self.obs_dtype, obs_layout="dense",
            mask_format="none", rules=roots.rules)
        if self.resample:
            s.resample_from(roots, root_of)
        else:
            copy_games(s, roots, root_of)
        return s

    def search(self, roots: StrategoRolloutBuffer, player: torch.Tensor | None = None,
               trace: list[torch.Tensor] | None = None) -> SearchResult:
        """One search per root game; ``player`` (optional, [R]) must be the side
        to move of each root (the reference searches for the player to move).
        ``trace``, when given, receives the rollouts' actions ply by ply (see
        ``BatchedRolloutEngine.rollout``)."""
        dev = roots.device
        R = roots.n_games
        if player is not None and not torch.equal(player.to(dev, torch.int8), roots.get_current_player()):
            raise RuntimeError("search runs for the side to move of each root")
        mask = roots.compute_legal_action_mask()                       # [R,100,100] bool
        flat = mask.reshape(R, NUM_ACTIONS)
        n_legal = flat.sum(-1)                                          # [R]
        # network probabilities of the legal moves at the root (:120-126)
        info = roots.compute_infostate_tensor(self.obs_dtype)
        _, policy = _net_out(self.move_net, info, None)
        probs = torch.softmax(policy.reshape(R, NUM_ACTIONS).to(torch.float64), dim=-1) * flat
        net_probs = probs / (probs.sum(-1, keepdim=True) + 1e-8)
        magnet = magnet_policy(mask)
        # one rollout per (root, legal move, config)
        n_cfg = torch.clamp(self.n_rollouts // n_legal.clamp(min=1), min=1) * (n_legal > 0)
        per_root = n_legal * n_cfg
        root_of = torch.repeat_interleave(torch.arange(R, device=dev), per_root)
        acts = flat.nonzero()                                           # [sum n_legal, 2] (root, action), ascending
        move_of = torch.repeat_interleave(acts[:, 1], n_cfg[acts[:, 0]])
        S = int(root_of.numel())
        q = torch.zeros((R, NUM_ACTIONS), dtype=torch.float64, device=dev)
        values = torch.zeros(S, dtype=torch.float32, device=dev)
        if S:
            samples = self._samples(roots, root_of)
            samples.apply_actions(move_of)
            values = self.rollouts.rollout(samples, self.depth - 1, trace=trace)
            q.index_put_((root_of, move_of), values.to(torch.float64), accumulate=True)
            q = q / n_cfg.clamp(min=1).to(torch.float64).unsqueeze(-1)
        self._calls += 1
        pi = compute_search_policy(q, net_probs, magnet, self.alpha, self.beta, legal=flat)
        pi = torch.where(n_legal.unsqueeze(-1) > 0, pi, torch.zeros_like(pi))
        gen = torch.Generator(device=dev)
        gen.manual_seed(self.seed * 1_000_003 + self._calls)
        choice = torch.full((R,), -1, dtype=torch.int64, device=dev)
        has = n_legal > 0
        if bool(has.any()):
            choice[has] = torch.multinomial(pi[has], 1, generator=gen).squeeze(-1)
        return SearchResult(action=choice, policy=pi, q=q * flat, net_probs=net_probs, magnet=magnet,
                            n_configs=n_cfg, values=values, legal=move_of, root_of=root_of)


__all__ = ["BatchedSearch", "SearchResult", "compute_search_policy", "magnet_policy", "copy_games", "NUM_SQUARES"]
