"""Shared test helpers: reference-test constants, the oracle adapter, comparisons.

``OracleRolloutBuffer`` presents the reference's StrategoRolloutBuffer API
(csrc/stratego_buffer.cpp:341-411) on top of the CPU oracle, returning CPU
torch tensors, so the scenario functions in ``scenarios.py`` run unchanged on
the oracle (CPU tests) and on the B200 buffer (GPU tests).
"""

from __future__ import annotations

import hashlib

import numpy as np
import torch

import oracle

PT_NONE, PT_SPY, PT_SCOUT, PT_MINER, PT_SERGEANT = 0, 1, 2, 3, 4
PT_CAPTAIN, PT_MARSHAL, PT_FLAG, PT_BOMB = 6, 10, 11, 12
PLAYER_RED, PLAYER_BLUE, PLAYER_EMPTY = 0, 1, -1
OUTCOME_ONGOING, OUTCOME_RED_WIN, OUTCOME_BLUE_WIN, OUTCOME_DRAW = -1, 0, 1, 2
NUM_SQUARES = 100
NUM_INFOSTATE_CHANNELS = 488
UNIFORM_PROB = 1.0 / 12.0


def encode_action(src_r: int, src_c: int, dst_r: int, dst_c: int) -> int:
    """(src_row, src_col, dst_row, dst_col) -> src_idx*100 + dst_idx."""
    return (src_r * 10 + src_c) * NUM_SQUARES + (dst_r * 10 + dst_c)


def make_setup(pieces_red, pieces_blue, n_games: int = 1):
    """(N,10,10) int8 setup planes from lists of (row, col, piece)."""
    red = torch.zeros((n_games, 10, 10), dtype=torch.int8)
    blue = torch.zeros((n_games, 10, 10), dtype=torch.int8)
    for r, c, p in pieces_red:
        red[:, r, c] = p
    for r, c, p in pieces_blue:
        blue[:, r, c] = p
    return red, blue


def digest(a: np.ndarray) -> np.int64:
    """blake2b-64 of an array's bytes, as tests/golden/make_golden.py computes it."""
    return np.frombuffer(hashlib.blake2b(np.ascontiguousarray(a).tobytes(), digest_size=8).digest(), dtype=np.int64)[0]


def board_code(owner: np.ndarray, piece: np.ndarray) -> np.ndarray:
    ow = owner.reshape(owner.shape[0], 100).astype(np.int16)
    pc = piece.reshape(piece.shape[0], 100).astype(np.int16)
    return np.where(ow >= 0, pc | (ow << 4) | 32, 0).astype(np.uint8)


class OracleRolloutBuffer:
    """The reference buffer API over the CPU oracle (tensors on the CPU)."""

    def __init__(self, n_games: int = 1, device_id: int = 0, **kw) -> None:
        self._o = oracle.OracleState(n_games, **kw)
        self.n_games = n_games
        self.device_id = device_id

    def _t(self, name: str) -> torch.Tensor:
        return torch.from_numpy(self._o.a[name].copy())

    def hello_world(self) -> torch.Tensor:
        return torch.tensor([42], dtype=torch.int32)

    def apply_actions(self, actions: torch.Tensor) -> None:
        if actions.dim() != 1 or actions.size(0) != self.n_games or actions.dtype != torch.int64:
            raise RuntimeError("bad actions")
        self._o.apply(actions.numpy())

    def compute_legal_action_mask(self) -> torch.Tensor:
        return torch.from_numpy(self._o.legal_mask_u8()).view(torch.bool)

    def compute_reward_pl0(self) -> torch.Tensor:
        return torch.from_numpy(self._o.reward_pl0())

    def compute_infostate_tensor(self) -> torch.Tensor:
        return torch.from_numpy(self._o.infostate_f32())

    def compute_two_square_rule_applies(self) -> torch.Tensor:
        return self._t("two_square_violation").view(torch.bool)

    def is_chasing_violation(self) -> torch.Tensor:
        return self._t("chasing_violation").view(torch.bool)

    def hash_board(self) -> torch.Tensor:
        return torch.from_numpy(self._o.hash_board())

    def get_terminated(self):
        return self._t("terminated").view(torch.bool)

    def get_outcomes(self):
        return self._t("outcome")

    def get_board_owner(self):
        return self._t("board_owner")

    def get_board_piece(self):
        return self._t("board_piece")

    def get_current_player(self):
        return self._t("current_player")

    def get_move_number(self):
        return self._t("move_number")

    def get_num_moves(self):
        return self._t("move_number")

    def get_num_moves_since_last_attack(self):
        return self._t("moves_since_attack")

    def get_flag_captured(self):
        return self._t("flag_captured").view(torch.bool)

    def get_has_legal_movement(self):
        return torch.from_numpy(self._o.legal_mask_u8().reshape(self.n_games, -1).any(1))

    def get_terminated_since(self):
        return self._t("terminated_since")

    def board_strs(self) -> list[str]:
        ow, pc = self._o.a["board_owner"], self._o.a["board_piece"]
        out = []
        for g in range(self.n_games):
            s = ""
            for r in range(10):
                for c in range(10):
                    o, p = int(ow[g, r, c]), int(pc[g, r, c])
                    s += ". " if o < 0 else ("R" if o == 0 else "B") + str(p) + (" " if p < 10 else "")
                s += "\n"
            out.append(s)
        return out

    def reset_terminated(self, red, blue) -> None:
        self._o.reset_planes(red.numpy(), blue.numpy(), force_all=False)

    def reset_all(self, red, blue) -> None:
        self._o.reset_planes(red.numpy(), blue.numpy(), force_all=True)

    def current_step(self) -> int:
        return int(self._o.a["move_number"].sum())

    def export_state(self) -> dict[str, torch.Tensor]:
        d = {k: torch.from_numpy(v.copy()) for k, v in self._o.a.items()}
        d["chase_hashes"] = d["chase_hashes"]
        return d


def export_np(buf) -> dict[str, np.ndarray]:
    """A buffer's full state (GPU or oracle adapter) as numpy, oracle naming."""
    d = buf.export_state()
    out = {k: v.cpu().numpy() for k, v in d.items() if k != "reward"}
    out["board_owner"] = out["board_owner"].reshape(-1, 10, 10)
    out["board_piece"] = out["board_piece"].reshape(-1, 10, 10)
    return out


def assert_state_equal(gpu: dict[str, np.ndarray], ora: dict[str, np.ndarray], ctx: str = "") -> None:
    for k, v in ora.items():
        g = gpu[k]
        if k == "chase_hashes":
            g = g.astype(np.int64)
        assert g.shape == v.shape, f"{ctx} {k}: shape {g.shape} vs {v.shape}"
        if not np.array_equal(g.astype(v.dtype), v):
            bad = np.argwhere(g.astype(v.dtype) != v)[:5]
            raise AssertionError(f"{ctx} field {k} differs at {bad.tolist()}")
