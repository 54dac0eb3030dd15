"""Generate tests/golden/isf.npz: the ISF repetition trackers of the reference.

Run in a container that holds the reference checkout (read-only is fine):

    python tests/golden/make_golden_isf.py --reference /path/to/ataraxos

The reference's Python engine plays the games (``stratego.env.rules.
StrategoState``, rules.py:27-500) and the reference's own ISF trackers judge
every move before it is recorded:

  * ``TwoSquareTracker.is_violation`` / ``record_move``
    (stratego/env/two_square.py:27-94), per piece, scout moves contributing
    every pair of the squares they cover;
  * ``ChasingTracker.is_chasing_violation`` / ``record_move``
    (stratego/env/chasing.py:54-109), per chaser, gated on the opponent's
    last move being an evasion, hashing with the seed-42 table.

Two kinds of game:
  * ``full``: standard 40-piece setups from the Philox setup pool, uniform
    random legal moves (the same seeded inputs as make_golden.py);
  * ``sparse``: a few pieces per side placed at random, moves picked by a
    chase-seeking policy (oscillate the piece that just moved, threaten,
    evade) so that both rules fire often, a variant with one to three
    movable pieces per side that never oscillates on purpose, and duels where
    every move evades or re-threatens, going back where that does it.

Per game the fixture stores the initial board, the action of every ply (-1
once the game is over) and, per ply, whether the move violated each rule.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from make_golden import make_setup  # noqa: E402


def _path(src: int, dst: int) -> list[int]:
    """Squares from src (exclusive) to dst (inclusive) along the line."""
    step = (10 if dst > src else -10) if src // 10 != dst // 10 else (1 if dst > src else -1)
    return list(range(src + step, dst + step, step))


def play(R, owner0: np.ndarray, piece0: np.ndarray, plies: int, policy: str, rng: np.random.Generator,
         no_attack_limit: int):
    st = R.StrategoState(no_attack_limit=no_attack_limit)
    st.board_owner[:] = owner0.reshape(10, 10)
    st.board_piece[:] = piece0.reshape(10, 10)
    st._red_setup_done = st._blue_setup_done = True
    ts, ch = R.TwoSquareTracker(), R.ChasingTracker()
    acts = np.full(plies, -1, np.int32)
    ev_ts = np.zeros(plies, np.uint8)
    ev_ch = np.zeros(plies, np.uint8)
    last_own = {0: None, 1: None}
    for t in range(plies):
        if st.is_terminal:
            break
        legal = sorted(a.src.idx * 100 + a.dst.idx for a in st.legal_actions())
        if not legal:
            break
        player = int(st.current_player)
        opp = 1 - player
        ow = st.board_owner.reshape(100)
        if policy == "uniform":
            a = legal[int(rng.integers(len(legal)))]
        else:
            back = last_own[player]
            threatened_me = [q for q in range(100) if ow[q] == player and any(
                0 <= q // 10 + dr < 10 and 0 <= q % 10 + dc < 10 and ow[(q // 10 + dr) * 10 + q % 10 + dc] == opp
                for dr, dc in ((-1, 0), (1, 0), (0, -1), (0, 1)))]
            evade = [x for x in legal if x // 100 in threatened_me and ow[x % 100] == -1]
            threat = [x for x in legal if ow[x % 100] == -1 and any(
                0 <= (x % 100) // 10 + dr < 10 and 0 <= x % 10 + dc < 10
                and ow[((x % 100) // 10 + dr) * 10 + x % 10 + dc] == opp
                for dr, dc in ((-1, 0), (1, 0), (0, -1), (0, 1)))]
            u = rng.random()
            if policy == "chase2":  # chase first, oscillate less
                u = 0.45 + 0.55 * u
            if policy == "duel":  # evade or re-threaten, by going back when that does it
                if evade and u < 0.9:
                    a = back if back in evade and rng.random() < 0.7 else evade[int(rng.integers(len(evade)))]
                elif threat and u < 0.95:
                    a = back if back in threat and rng.random() < 0.7 else threat[int(rng.integers(len(threat)))]
                else:
                    a = legal[int(rng.integers(len(legal)))]
            elif back is not None and back in legal and u < 0.45:
                a = back
            elif evade and u < 0.7:
                a = evade[int(rng.integers(len(evade)))]
            elif threat and u < 0.9:
                a = threat[int(rng.integers(len(threat)))]
            else:
                a = legal[int(rng.integers(len(legal)))]
        src, dst = a // 100, a % 100
        S = R.Square
        action = R.Action(S.from_idx(src), S.from_idx(dst))
        bo, bp = st.board_owner.copy(), st.board_piece.copy()
        attack = int(bo.reshape(100)[dst]) not in (-1, player)
        scout = int(bp.reshape(100)[src]) == 2
        path = [S.from_idx(q) for q in _path(src, dst)]
        ev_ts[t] = ts.is_violation(R.Player(player), S.from_idx(src), action, scout, path, attack)
        ev_ch[t] = ch.is_chasing_violation(R.Player(player), action, bo, bp)
        st.apply_action(action)
        ts.record_move(R.Player(player), S.from_idx(src), action, scout, path, attack)
        ch.record_move(R.Player(player), action, bo, bp, st.board_owner, st.board_piece)
        acts[t] = a
        last_own[player] = dst * 100 + src
    return acts, ev_ts, ev_ch


def sparse_board(rng: np.random.Generator, lo: int = 3, hi: int = 6) -> tuple[np.ndarray, np.ndarray]:
    owner = np.full(100, -1, np.int8)
    piece = np.zeros(100, np.int8)
    free = [q for q in range(20, 80) if not (q // 10 in (4, 5) and q % 10 in (2, 3, 6, 7))]
    rng.shuffle(free)
    k = 0
    for p in (0, 1):
        kinds = [11, 12] + list(rng.choice([1, 2, 2, 3, 4, 5, 6, 7, 8, 9, 10], size=int(rng.integers(lo, hi))))
        for pt in kinds:
            q = free[k]
            k += 1
            owner[q], piece[q] = p, pt
    return owner, piece


class _Ref:
    def __init__(self, root: Path) -> None:
        sys.path.insert(0, str(root))
        from stratego.env.chasing import ChasingTracker
        from stratego.env.rules import StrategoState
        from stratego.env.two_square import TwoSquareTracker
        from stratego.types import Action, Player, Square

        self.StrategoState, self.TwoSquareTracker, self.ChasingTracker = StrategoState, TwoSquareTracker, ChasingTracker
        self.Action, self.Player, self.Square = Action, Player, Square


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ATARAXOS_REFERENCE"),
                    required="ATARAXOS_REFERENCE" not in os.environ,
                    help="checkout of the reference project (or set ATARAXOS_REFERENCE)")
    args = ap.parse_args()
    R = _Ref(Path(args.reference))
    rng = np.random.default_rng(20251201)
    plies = 300
    owners, pieces, acts, ets, ech, kind, nal = [], [], [], [], [], [], []
    for g in range(24):  # full boards, uniform play
        red, blue = make_setup(11, 2 * g), make_setup(11, 2 * g + 1)
        ow = np.full(100, -1, np.int8)
        pc = np.zeros(100, np.int8)
        for i in range(40):
            ow[i], pc[i] = 0, red[i]
            ow[60 + i], pc[60 + i] = 1, blue[i]
        a, t, c = play(R, ow, pc, plies, "uniform", rng, 100)
        owners.append(ow), pieces.append(pc), acts.append(a), ets.append(t), ech.append(c)
        kind.append(0), nal.append(100)
    for g in range(72):  # sparse boards, chase-seeking play
        ow, pc = sparse_board(rng)
        a, t, c = play(R, ow, pc, plies, "chase", rng, 200)
        owners.append(ow), pieces.append(pc), acts.append(a), ets.append(t), ech.append(c)
        kind.append(1), nal.append(200)
    for g in range(64):  # very sparse boards, mostly chasing
        ow, pc = sparse_board(rng, 1, 3)
        a, t, c = play(R, ow, pc, plies, "chase2", rng, 200)
        owners.append(ow), pieces.append(pc), acts.append(a), ets.append(t), ech.append(c)
        kind.append(2), nal.append(200)
    for g in range(96):  # one or two movable pieces per side chasing each other
        ow, pc = sparse_board(rng, 1, 3)
        a, t, c = play(R, ow, pc, plies, "duel", rng, 200)
        owners.append(ow), pieces.append(pc), acts.append(a), ets.append(t), ech.append(c)
        kind.append(3), nal.append(200)
    out = {
        "owner": np.stack(owners), "piece": np.stack(pieces), "actions": np.stack(acts),
        "ev_two_square": np.stack(ets), "ev_chasing": np.stack(ech), "kind": np.asarray(kind, np.int8),
        "no_attack_limit": np.asarray(nal, np.int32),
    }
    np.savez_compressed(HERE / "isf.npz", **out)
    print("isf.npz", (HERE / "isf.npz").stat().st_size, "bytes;",
          "two-square events", int(out["ev_two_square"].sum()), "chasing events", int(out["ev_chasing"].sum()),
          "games with either", int(((out["ev_two_square"] | out["ev_chasing"]).sum(1) > 0).sum()))


if __name__ == "__main__":
    main()
