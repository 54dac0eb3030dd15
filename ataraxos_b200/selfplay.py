"""Batched self-play and search rollouts driven by a move network.

``BatchedSelfPlay`` is the batched counterpart of
``SelfPlayGenerator.generate_games`` (stratego/training/selfplay.py:190-268):
N games advance together, one fused kernel per ply.  Each ply the move
network scores every game's infostate ``[N,488,10,10]`` and the kernel samples
one legal move per game from the network's policy restricted to the legal
moves, applies it and writes the next infostate.  The kernel samples by
Gumbel-max over the legal entries of the logits, whose distribution is the
softmax of the logits renormalised over the legal moves: the reference's
``softmax`` + ``_map_policy_to_actions`` + ``np.random.choice``
(selfplay.py:221-228, 301-317, 331-353).

``BatchedRolloutEngine`` is the batched counterpart of
``RolloutEngine.rollout`` / ``rollout_for_move`` (stratego/search/rollouts.py:
46-118): every game of a buffer plays up to ``depth`` plies sampled from the
network's policy, then the network's value head scores the final position
as ``P(win) - P(loss)``.

The network is any callable ``net(infostate[, legal_move_mask])`` returning
``(value_logits [N,3], policy_logits [N,10000])`` like
``stratego/networks/move_net.py:153-185`` (a bare policy tensor also works
where no value is needed).

Differences from the reference, all deliberate:
  * move history and moved / revealed squares are the simulator's own
    trackers (the reference CUDA class's semantics), carried through the whole
    game; the reference rollout engine restarts them at the rollout root and
    scores the final position with empty trackers (rollouts.py:59-61, 97-99);
  * sampling from logits cannot underflow, so the reference's uniform
    fallback for near-zero probabilities (selfplay.py:348-350) never applies;
  * setups come from the buffer's seeded setup pool instead of
    ``random.shuffle`` (selfplay.py:291-322), and squares are plain indices
    ``row * 10 + col`` instead of ``Square`` objects.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import numpy as np
import torch

from .buffer import NUM_ACTIONS, NUM_SQUARES, StrategoRolloutBuffer

NetFn = Callable[..., object]

TRAINING_NO_ATTACK_LIMIT = 100  # stratego/constants.py:55
EVAL_NO_ATTACK_LIMIT = 200      # stratego/constants.py:56


def _net_out(net: NetFn, info: torch.Tensor, mask: torch.Tensor | None) -> tuple[torch.Tensor | None, torch.Tensor]:
    with torch.no_grad():
        out = net(info) if mask is None else net(info, mask)
    if isinstance(out, (tuple, list)):
        return out[0], out[-1]
    return None, out


def _logits(policy: torch.Tensor, n: int) -> torch.Tensor:
    if policy.shape[0] != n or policy.numel() != n * NUM_ACTIONS:
        raise RuntimeError(f"the network's policy must be [{n},{NUM_ACTIONS}], got {tuple(policy.shape)}")
    return policy.reshape(n, NUM_ACTIONS).float().contiguous()


@dataclass
class SelfPlayTransition:
    """One move of a self-play game (stratego/training/selfplay.py:43-61)."""

    infostate: np.ndarray | None  # (488,10,10) float32 before the move (None unless stored)
    action: tuple[int, int]       # (src, dst) square indices, row * 10 + col
    player: int                   # 0 Red, 1 Blue
    move_idx: int                 # src * 100 + dst
    is_attack: bool               # the destination held an opponent piece


@dataclass
class SelfPlayGame:
    """A complete self-play game (stratego/training/selfplay.py:64-77)."""

    transitions: list[SelfPlayTransition]
    outcome: int                              # 1 Red wins, -1 Blue wins, 0 draw
    setup_red: list[tuple[tuple[int, int], int]]   # ((row, col), piece type 1..12)
    setup_blue: list[tuple[tuple[int, int], int]]


class BatchedSelfPlay:
    """Self-play games sampled from a move network, N games per kernel launch."""

    def __init__(
        self,
        move_net: NetFn,
        num_envs: int = 1536,
        device_id: int = 0,
        *,
        seed: int = 0,
        env_base: int = 0,
        no_attack_limit: int = TRAINING_NO_ATTACK_LIMIT,
        max_game_length: int = 4000,
        pool_size: int = 65536,
        setup_pool: torch.Tensor | np.ndarray | None = None,
        obs_dtype: torch.dtype = torch.float32,
        pass_legal_mask: bool = False,
    ) -> None:
        self.move_net = move_net
        self.num_envs = int(num_envs)
        self.pass_legal_mask = bool(pass_legal_mask)
        self.obs_dtype = obs_dtype
        self.buf = StrategoRolloutBuffer(
            self.num_envs, device_id, seed=seed, env_base=env_base,
            pool_size=None if setup_pool is not None else pool_size, setup_pool=setup_pool,
            no_attack_limit=no_attack_limit, max_game_length=max_game_length, obs_dtype=obs_dtype,
            obs_layout="dense", mask_format="u8" if pass_legal_mask else "none")
        self.device = self.buf.device

    # -- helpers ---------------------------------------------------------
    def _observe_fresh(self) -> tuple[torch.Tensor, torch.Tensor | None]:
        info = self.buf.compute_infostate_tensor(self.obs_dtype)
        mask = self.buf.compute_legal_action_mask() if self.pass_legal_mask else None
        return info, mask

    def _policy(self, info: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
        _, policy = _net_out(self.move_net, info, mask)
        return _logits(policy, self.num_envs)

    def _setups(self) -> tuple[np.ndarray, np.ndarray]:
        return self.buf.get_board_owner().cpu().numpy(), self.buf.get_board_piece().cpu().numpy()

    # -- tensor-native collection ------------------------------------------
    def collect(self, plies: int, *, store_obs: bool = True, auto_reset: bool = True) -> dict[str, torch.Tensor]:
        """Play ``plies`` plies of every game from the current positions (new
        games start from the pool as old ones end when ``auto_reset``).

        Returns device tensors stacked over plies ``[P, N]``: ``action``
        (int64, -1 for a game that had ended), ``logprob`` (log-prob of the
        sampled move under the network's legal softmax), ``player`` (int8,
        side that moved), ``reward`` (player-0 reward of the transition),
        ``done`` (bool), and with ``store_obs`` the infostate before each move
        as its 75 live planes ``obs [P, N, 75, 10, 10]`` (channels 0-42 and
        456-487; 43-455 are zero).
        """
        n = self.num_envs
        info, mask = self._observe_fresh()
        live = torch.cat([torch.arange(43), torch.arange(456, 488)]).to(self.device)
        keys = ("action", "logprob", "player", "reward", "done")
        res: dict[str, list[torch.Tensor]] = {k: [] for k in keys}
        obs: list[torch.Tensor] = []
        for _ in range(int(plies)):
            if store_obs:
                obs.append(info.index_select(1, live))
            player = self.buf.get_current_player()
            out = self.buf.step(None, policy="gumbel", logits=self._policy(info, mask), auto_reset=auto_reset)
            res["action"].append(out.action.clone())
            res["logprob"].append(out.logprob.clone())
            res["player"].append(player)
            res["reward"].append(out.reward.clone())
            res["done"].append(out.done.clone())
            info = out.infostate
            mask = out.legal_mask
        ret = {k: torch.stack(v) if v else torch.empty((0, n), device=self.device) for k, v in res.items()}
        if store_obs:
            ret["obs"] = torch.stack(obs) if obs else torch.empty((0, n, 75, 10, 10), device=self.device)
        return ret

    # -- the reference's list-of-games API -----------------------------------
    def generate_games(self, n_games: int = 16, *, store_infostate: bool = True) -> list[SelfPlayGame]:
        """Play ``n_games`` complete games (selfplay.py:190-268), in waves of
        ``num_envs`` games that each play exactly one game to its end, so the
        returned games are not biased towards short ones."""
        games: list[SelfPlayGame] = []
        while len(games) < n_games:
            m = min(self.num_envs, n_games - len(games))
            games.extend(self._wave(m, store_infostate))
        return games

    def _wave(self, m: int, store_infostate: bool) -> list[SelfPlayGame]:
        b, n = self.buf, self.num_envs
        b.reset_all_from_pool()
        owner0, piece0 = self._setups()
        info, mask = self._observe_fresh()
        trans: list[list[SelfPlayTransition]] = [[] for _ in range(m)]
        outcome = [0] * m
        active = np.ones(n, dtype=bool)
        player = np.zeros(n, dtype=np.int64)
        rows = torch.arange(n, device=self.device)
        while active.any():
            owner = b.get_board_owner().reshape(n, NUM_SQUARES)
            host_info = info[:m].float().cpu().numpy() if store_infostate else None
            out = b.step(None, policy="gumbel", logits=self._policy(info, mask), auto_reset=False)
            act = out.action
            dst = act.clamp(min=0) % NUM_SQUARES
            attack = (owner[rows, dst] == torch.from_numpy(1 - player).to(self.device)).cpu().numpy()
            act_h = act.cpu().numpy()
            done_h = out.done.cpu().numpy()
            rew_h = out.reward.cpu().numpy()
            for e in np.nonzero(active[:m])[0]:
                a = int(act_h[e])
                if a >= 0:
                    trans[e].append(SelfPlayTransition(
                        infostate=None if host_info is None else host_info[e].copy(),
                        action=(a // NUM_SQUARES, a % NUM_SQUARES), player=int(player[e]), move_idx=a,
                        is_attack=bool(attack[e])))
                if done_h[e]:
                    outcome[e] = int(round(float(rew_h[e])))
            player = np.where(act_h >= 0, 1 - player, player)
            active &= ~done_h.astype(bool)
            info, mask = out.infostate, out.legal_mask
        games = []
        for e in range(m):
            red = [((q // 10, q % 10), int(piece0[e].reshape(-1)[q])) for q in range(NUM_SQUARES)
                   if owner0[e].reshape(-1)[q] == 0]
            blue = [((q // 10, q % 10), int(piece0[e].reshape(-1)[q])) for q in range(NUM_SQUARES)
                    if owner0[e].reshape(-1)[q] == 1]
            games.append(SelfPlayGame(transitions=trans[e], outcome=outcome[e], setup_red=red, setup_blue=blue))
        return games


class BatchedRolloutEngine:
    """Depth-limited rollouts of every game of a buffer, sampled from a move
    network (stratego/search/rollouts.py:22-118)."""

    def __init__(self, move_net: NetFn, *, obs_dtype: torch.dtype = torch.float32) -> None:
        self.move_net = move_net
        self.obs_dtype = obs_dtype

    def _info(self, states: StrategoRolloutBuffer, out=None) -> torch.Tensor:
        if out is not None and out.infostate is not None and out.infostate.shape[1] == 488:
            return out.infostate if out.infostate.dtype == self.obs_dtype else out.infostate.to(self.obs_dtype)
        return states.compute_infostate_tensor(self.obs_dtype)

    def rollout(self, states: StrategoRolloutBuffer, depth: int = 40,
                trace: list[torch.Tensor] | None = None) -> torch.Tensor:
        """Advance every game of ``states`` in place by up to ``depth`` plies
        (a game that ends stops), then return ``P(win) - P(loss)`` of the
        network's value head at each final position, for the side to move
        there (rollouts.py:46-104).  float32 [N] on the buffer's device.
        ``trace``, when given, receives each ply's applied actions ([N] int64,
        -1 for a game that had ended)."""
        n = states.n_games
        info = self._info(states)
        for _ in range(int(depth)):
            if bool(states.get_terminated().all()):
                break
            _, policy = _net_out(self.move_net, info, None)
            out = states.step(None, policy="gumbel", logits=_logits(policy, n), auto_reset=False)
            if trace is not None:
                trace.append(out.action.clone())
            info = self._info(states, out)
        value, _ = _net_out(self.move_net, info, None)
        if value is None:
            raise RuntimeError("the network must return (value_logits, policy_logits)")
        p = torch.softmax(value.float(), dim=-1)
        return p[:, 0] - p[:, 1]

    def rollout_for_move(self, states: StrategoRolloutBuffer, actions: torch.Tensor, depth: int = 40) -> torch.Tensor:
        """Apply ``actions`` [N] to a copy of ``states`` and roll ``depth - 1``
        more plies (rollouts.py:106-118); ``states`` is left unchanged."""
        c = states.clone()
        c.apply_actions(actions)
        return self.rollout(c, depth - 1)
