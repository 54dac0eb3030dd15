"""Generate the golden traces in tests/golden/ from the reference's Python engine.

Run in a container that holds the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/ataraxos

The rules (legal moves, movement, combat, terminal order, outcome) and the
488-channel infostate come from the reference itself:
``stratego.env.rules.StrategoState`` (rules.py:27-500) and
``stratego.env.infostate.compute_infostate`` (infostate.py:37-109).
Setups are validated by the reference's ``apply_setup`` (rules.py:94-145).

The caller-side state that the reference keeps only inside its CUDA class is
tracked here in Python with the CUDA kernel's semantics, because the Python
engine has no such state (stratego/training/selfplay.py keeps a different
variant):
  * moved / revealed squares and the 32-move history ring
    (csrc/stratego_buffer.cu:243-260);
  * two-square tracker, per mover (cu:272-296);
  * chasing tracker with a 64-entry Zobrist ring per side (cu:306-381),
    hashing with the seed-42 table of stratego/env/chasing.py:17-31;
  * flag_captured / terminated_since (csrc/stratego_buffer.cpp:80-119).

Seeded inputs (no reference counterpart; the product and the oracle define
them the same way): Philox4x32-10 (Salmon et al., SC'11) restated here in
pure Python, setup pool entries by a Philox-driven Fisher-Yates shuffle of
the 40-piece roster, uniform action choice k = (u32 * n) >> 32 over the legal
actions in ascending src*100+dst order.

Two traces are written:
  * ``config1.npz``: 64 games, 200 plies, no auto-reset;
  * ``autoreset.npz``: 16 games, 400 plies, auto-reset from the pool, with
    no_attack_limit=20 and max game length 150 so that draws by both caps and
    resets happen inside the trace.  The max game length is a module constant
    in the reference (constants.py:60); the script sets it on the two modules
    that read it (rules.py, infostate.py) for this trace only.
Per snapshot the fixtures hold compact state, digests (blake2b-64) of the
float32 infostate, of the packed legal mask and of the chase ring, and full
arrays for a few envs.
"""

from __future__ import annotations

import argparse
import os
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# ---------------------------------------------------------------------------
# Philox4x32-10 and the seeded inputs (pure Python)
# ---------------------------------------------------------------------------
M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
MASK32 = 0xFFFFFFFF
TAG_SETUP, TAG_RESET, TAG_ACTION = 1, 2, 3
ROSTER = [1] + [2] * 8 + [3] * 5 + [4] * 4 + [5] * 4 + [6] * 4 + [7] * 3 + [8] * 2 + [9, 10, 11] + [12] * 6


def philox(c0: int, c1: int, c2: int, c3: int, seed: int) -> tuple[int, int, int, int]:
    k0, k1 = seed & MASK32, (seed >> 32) & MASK32
    for _ in range(10):
        p0, p1 = M0 * c0, M1 * c2
        c0, c1, c2, c3 = ((p1 >> 32) ^ c1 ^ k0) & MASK32, p1 & MASK32, ((p0 >> 32) ^ c3 ^ k1) & MASK32, p0 & MASK32
        k0, k1 = (k0 + W0) & MASK32, (k1 + W1) & MASK32
    return c0, c1, c2, c3


def make_setup(seed: int, index: int) -> list[int]:
    p = list(ROSTER)
    w: list[int] = []
    for blk in range(10):
        w.extend(philox(index & MASK32, blk, index >> 32, TAG_SETUP, seed))
    for d in range(39):
        i = 39 - d
        j = (w[d] * (i + 1)) >> 32
        p[i], p[j] = p[j], p[i]
    return p


def reset_indices(seed: int, genv: int, episode: int, pool_size: int) -> tuple[int, int]:
    w = philox(genv & MASK32, episode, genv >> 32, TAG_RESET, seed)
    return (w[0] * pool_size) >> 32, (w[1] * pool_size) >> 32


def choose_index(seed: int, genv: int, ply: int, n: int) -> int:
    w = philox(genv & MASK32, ply & MASK32, ply >> 32, TAG_ACTION, seed)
    return (w[0] * n) >> 32


def digest(a: np.ndarray) -> np.int64:
    return np.frombuffer(hashlib.blake2b(np.ascontiguousarray(a).tobytes(), digest_size=8).digest(), dtype=np.int64)[0]


# ---------------------------------------------------------------------------
# One game: reference engine + CUDA-semantics trackers
# ---------------------------------------------------------------------------


class Game:
    def __init__(self, ref, zobrist: np.ndarray, no_attack_limit: int) -> None:
        self.ref = ref
        self.z = zobrist
        self.no_attack_limit = no_attack_limit
        self.state = None

    def reset(self, red: list[int], blue: list[int]) -> None:
        R = self.ref
        st = R.StrategoState(no_attack_limit=self.no_attack_limit)
        st.apply_setup(R.Player.RED, [(R.Square(i // 10, i % 10), R.PieceType(p)) for i, p in enumerate(red)])
        st.apply_setup(R.Player.BLUE, [(R.Square(6 + i // 10, i % 10), R.PieceType(p)) for i, p in enumerate(blue)])
        self.state = st
        self.moved = np.zeros(100, np.uint8)
        self.revealed = np.zeros(100, np.uint8)
        self.hist = np.zeros(32, np.int32)
        self.hist_head = 0
        self.hist_len = 0
        self.history: list = []
        self.ts_count = [0, 0]
        self.ts_lo = [-1, -1]
        self.ts_hi = [-1, -1]
        self.ts_violation = 0
        self.chase = np.zeros((2, 64), np.int64)
        self.chase_head = [0, 0]
        self.chase_len = [0, 0]
        self.chase_last_src = [-1, -1]
        self.chase_violation = 0
        self.flag_captured = 0
        self.terminated_since = 0

    def legal_sorted(self) -> list[int]:
        return sorted(a.src.idx * 100 + a.dst.idx for a in self.state.legal_actions())

    def board_hash(self) -> int:
        ow, pc = self.state.board_owner, self.state.board_piece
        h = np.int64(0)
        for r in range(10):
            for c in range(10):
                if ow[r, c] >= 0:
                    h ^= self.z[r, c, ow[r, c], pc[r, c]]
        return int(h)

    def apply(self, a: int) -> None:
        R, st = self.ref, self.state
        src, dst = a // 100, a % 100
        sq_s, sq_d = R.Square.from_idx(src), R.Square.from_idx(dst)
        player = int(st.current_player)
        opp = 1 - player
        dst_owner = int(st.board_owner[sq_d.row, sq_d.col])
        attack = dst_owner not in (-1, player)
        flag = attack and int(st.board_piece[sq_d.row, sq_d.col]) == 11
        st.apply_action(R.Action(sq_s, sq_d))
        # moved / revealed / history (cu:243-260)
        if attack:
            self.revealed[src] = 1
            self.revealed[dst] = 1
        else:
            self.moved[src] = 1
            self.moved[dst] = 1
            self.revealed[dst] = self.revealed[src]
            self.revealed[src] = 0
        self.hist[self.hist_head] = a
        self.hist_head = (self.hist_head + 1) % 32
        self.hist_len = min(self.hist_len + 1, 32)
        self.history.append(R.Action(sq_s, sq_d))
        # two-square, per mover (cu:272-296)
        if attack:
            self.ts_count[player], self.ts_lo[player], self.ts_hi[player] = 0, -1, -1
        else:
            lo, hi = min(src, dst), max(src, dst)
            if self.ts_lo[player] == lo and self.ts_hi[player] == hi:
                self.ts_count[player] += 1
            else:
                self.ts_count[player], self.ts_lo[player], self.ts_hi[player] = 1, lo, hi
            if self.ts_count[player] > 3:
                self.ts_violation = 1
        # chasing (cu:306-381)
        dr, dc = sq_d.row, sq_d.col
        threat = False
        for rr, cc in ((dr - 1, dc), (dr + 1, dc), (dr, dc - 1), (dr, dc + 1)):
            if 0 <= rr < 10 and 0 <= cc < 10 and not R.Square(rr, cc).is_lake:
                if int(st.board_owner[rr, cc]) == opp:
                    threat = True
                    break
        if threat:
            h = self.board_hash()
            found = any(int(self.chase[player, i]) == h for i in range(self.chase_len[player]))
            exc = self.chase_last_src[player] >= 0 and dst == self.chase_last_src[player]
            if found and not exc:
                self.chase_violation = 1
            if self.chase_len[player] < 64:
                self.chase[player, self.chase_len[player]] = h
                self.chase_len[player] += 1
            else:
                self.chase[player, self.chase_head[player]] = h
                self.chase_head[player] = (self.chase_head[player] + 1) % 64
            self.chase_last_src[player] = src
        else:
            self.chase_len[player], self.chase_head[player], self.chase_last_src[player] = 0, 0, -1
        if flag:
            self.flag_captured = 1

    def infostate(self) -> np.ndarray:
        R, st = self.ref, self.state
        moved = {R.Square.from_idx(i) for i in np.nonzero(self.moved)[0]}
        rev = {R.Square.from_idx(i) for i in np.nonzero(self.revealed)[0]}
        return R.compute_infostate(
            st, st.current_player, move_history=self.history, moved_squares=moved, revealed_squares=rev
        )


# ---------------------------------------------------------------------------
# Traces
# ---------------------------------------------------------------------------


def run_trace(ref, *, n: int, plies: int, seed: int, pool_size: int, auto_reset: bool, no_attack_limit: int,
              full_envs: int, full_plies: list[int]) -> dict[str, np.ndarray]:
    z = np.random.default_rng(42).integers(low=0, high=2**63, size=(10, 10, 2, 13), dtype=np.int64)
    pool = np.array([make_setup(seed, i) for i in range(pool_size)], dtype=np.uint8)
    games = [Game(ref, z, no_attack_limit) for _ in range(n)]
    episode = np.zeros(n, np.int32)

    def new_game(g: int) -> None:
        ri, bi = reset_indices(seed, g, int(episode[g]), pool_size)
        games[g].reset(list(pool[ri]), list(pool[bi]))
        episode[g] += 1

    for g in range(n):
        new_game(g)

    T = plies + 1
    rec: dict[str, list] = {k: [] for k in (
        "board", "moved", "revealed", "current_player", "outcome", "flag_captured", "move_number",
        "moves_since_attack", "terminated_since", "hist_head", "hist_len", "hist_digest", "ts_count", "ts_lo",
        "ts_hi", "ts_violation", "chase_head", "chase_len", "chase_last_src", "chase_digest", "chase_violation",
        "hash", "n_legal", "mask_digest", "info_digest", "episode")}
    full_info, full_mask = [], []
    actions = np.full((plies, n), -1, np.int64)
    reward = np.zeros((plies, n), np.float32)
    done = np.zeros((plies, n), np.uint8)

    def snapshot(t: int) -> None:
        rows = {k: [] for k in rec}
        for g, gm in enumerate(games):
            st = gm.state
            ow = st.board_owner.reshape(100).astype(np.int16)
            pc = st.board_piece.reshape(100).astype(np.int16)
            code = np.where(ow >= 0, pc | (ow << 4) | 32, 0).astype(np.uint8)
            rows["board"].append(code)
            rows["moved"].append(np.packbits(gm.moved, bitorder="little"))
            rows["revealed"].append(np.packbits(gm.revealed, bitorder="little"))
            rows["current_player"].append(int(st.current_player))
            rows["outcome"].append(int(st.outcome))
            rows["flag_captured"].append(gm.flag_captured)
            rows["move_number"].append(st.move_number)
            rows["moves_since_attack"].append(st.moves_since_last_attack)
            rows["terminated_since"].append(gm.terminated_since)
            rows["hist_head"].append(gm.hist_head)
            rows["hist_len"].append(gm.hist_len)
            rows["hist_digest"].append(digest(gm.hist.astype(np.int32)))
            rows["ts_count"].append(list(gm.ts_count))
            rows["ts_lo"].append(list(gm.ts_lo))
            rows["ts_hi"].append(list(gm.ts_hi))
            rows["ts_violation"].append(gm.ts_violation)
            rows["chase_head"].append(list(gm.chase_head))
            rows["chase_len"].append(list(gm.chase_len))
            rows["chase_last_src"].append(list(gm.chase_last_src))
            rows["chase_digest"].append(digest(gm.chase))
            rows["chase_violation"].append(gm.chase_violation)
            rows["hash"].append(gm.board_hash())
            legal = gm.legal_sorted()
            m = np.zeros(10000, np.uint8)
            m[legal] = 1
            bits = np.packbits(m, bitorder="little")
            rows["n_legal"].append(len(legal))
            rows["mask_digest"].append(digest(bits))
            info = gm.infostate()
            rows["info_digest"].append(digest(info.astype(np.float32)))
            rows["episode"].append(int(episode[g]))
            if g < full_envs and t in full_plies:
                full_info.append(info.astype(np.float32))
                full_mask.append(bits)
        for k in rec:
            rec[k].append(rows[k])

    snapshot(0)
    for t in range(plies):
        for g, gm in enumerate(games):
            if not gm.state.is_terminal:
                legal = gm.legal_sorted()
                if legal:
                    a = legal[choose_index(seed, g, t, len(legal))]
                    gm.apply(a)
                    actions[t, g] = a
            gm.terminated_since += 1 if gm.state.is_terminal else 0
            o = int(gm.state.outcome)
            reward[t, g] = 1.0 if o == 0 else (-1.0 if o == 1 else 0.0)
            done[t, g] = 1 if gm.state.is_terminal else 0
            if auto_reset and gm.state.is_terminal:
                new_game(g)
        snapshot(t + 1)

    out = {k: np.asarray(v) for k, v in rec.items()}
    for k in ("current_player", "outcome", "flag_captured", "ts_violation", "chase_violation"):
        out[k] = out[k].astype(np.int8)
    for k in ("move_number", "moves_since_attack", "terminated_since", "hist_head", "hist_len", "n_legal", "episode"):
        out[k] = out[k].astype(np.int32)
    for k in ("ts_count", "ts_lo", "ts_hi", "chase_head", "chase_len", "chase_last_src"):
        out[k] = out[k].astype(np.int32)
    out["hash"] = out["hash"].astype(np.int64)
    out["actions"] = actions
    out["reward"] = reward
    out["done"] = done
    out["pool"] = pool
    out["full_info"] = np.asarray(full_info, np.float32).reshape(len(full_plies), full_envs, 488, 10, 10)
    out["full_mask"] = np.asarray(full_mask, np.uint8).reshape(len(full_plies), full_envs, 1250)
    out["full_plies"] = np.asarray(full_plies, np.int32)
    out["meta"] = np.asarray([n, plies, seed, pool_size, int(auto_reset), no_attack_limit], np.int64)
    return out


class _Ref:
    """The reference modules the traces use."""

    def __init__(self, root: Path) -> None:
        sys.path.insert(0, str(root))
        from stratego.env import infostate as infostate_mod
        from stratego.env import rules as rules_mod
        from stratego.env.infostate import compute_infostate
        from stratego.env.rules import StrategoState
        from stratego.types import Action, PieceType, Player, Square

        self.rules_mod, self.infostate_mod = rules_mod, infostate_mod
        self.StrategoState, self.compute_infostate = StrategoState, compute_infostate
        self.Action, self.PieceType, self.Player, self.Square = Action, PieceType, Player, Square

    def set_max_game_length(self, v: int) -> None:
        self.rules_mod.MAX_GAME_LENGTH = v
        self.infostate_mod.MAX_GAME_LENGTH = v


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ATARAXOS_REFERENCE"),
                    required="ATARAXOS_REFERENCE" not in os.environ,
                    help="checkout of the reference project (or set ATARAXOS_REFERENCE)")
    args = ap.parse_args()
    ref = _Ref(Path(args.reference))

    ref.set_max_game_length(4000)
    c1 = run_trace(ref, n=64, plies=200, seed=20251107, pool_size=1024, auto_reset=False, no_attack_limit=100,
                   full_envs=4, full_plies=[0, 1, 2, 100, 200])
    c1["max_game_length"] = np.asarray(4000)
    np.savez_compressed(HERE / "config1.npz", **c1)

    ref.set_max_game_length(150)
    ar = run_trace(ref, n=16, plies=400, seed=7, pool_size=64, auto_reset=True, no_attack_limit=20,
                   full_envs=2, full_plies=[0, 37, 150, 400])
    ar["max_game_length"] = np.asarray(150)
    np.savez_compressed(HERE / "autoreset.npz", **ar)
    ref.set_max_game_length(4000)
    for f in ("config1.npz", "autoreset.npz"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
