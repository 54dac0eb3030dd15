"""Generate tests/golden/isf_long_chase.npz: long chases judged by the
reference's own ISF chasing tracker.

Run in a container that holds the reference checkout (read-only is fine):

    python tests/golden/make_golden_isf_chase.py --reference /path/to/ataraxos

The reference's ``ChasingTracker`` (stratego/env/chasing.py:54-109) keeps
every position of a chase in an unbounded set; this build keeps the last 64
(a ring of hashes).  Each game here is a chase around a closed loop of L
free squares: a Red sergeant follows a Blue sergeant one square behind, Blue
evading every time, so the chase revisits its first position after L chaser
moves.  The reference flags that move and every later one; a 64-position
memory flags it only when L <= 64.  Loops of L = 60, 62, 64, 66 and 84
squares pin the bound from both sides.

The loop: a serpentine over columns 0..W of rows 0-3 and 6-9 joined through
(4,1), (5,1) and column 0 (8W + 12 squares, no lake on it), plus detours of
two squares ("bumps" into column W+1) that lengthen it by 2 each.  Squares at
loop distance two are never 4-adjacent (the grid is bipartite), so Blue's
moves threaten nothing and Red's always threaten Blue.

Per game the fixture stores the initial board, the actions (-1 after the
end), the reference's per-ply chasing and two-square verdicts (each taken
before the move is recorded, as in make_golden_isf.py) and L.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LAKES = {42, 43, 46, 47, 52, 53, 56, 57}


def serpentine(W: int) -> list[int]:
    """The closed loop of 8W + 12 squares described above (square = r*10 + c)."""
    sq = [c for c in range(0, W + 1)]                      # row 0: 0 -> W
    sq += [10 + c for c in range(W, 0, -1)]                # row 1: W -> 1
    sq += [20 + c for c in range(1, W + 1)]                # row 2: 1 -> W
    sq += [30 + c for c in range(W, 0, -1)]                # row 3: W -> 1
    sq += [41, 51]                                         # down column 1
    sq += [60 + c for c in range(1, W + 1)]                # row 6: 1 -> W
    sq += [70 + c for c in range(W, 0, -1)]                # row 7: W -> 1
    sq += [80 + c for c in range(1, W + 1)]                # row 8: 1 -> W
    sq += [90 + c for c in range(W, -1, -1)]               # row 9: W -> 0
    sq += [r * 10 for r in range(8, 0, -1)]                # column 0 up: 8 -> 1
    return sq


def with_bumps(loop: list[int], W: int, bumps: int) -> list[int]:
    """Replace the loop's vertical edges (r,W)-(r+1,W) at r = 0, 2, 6 by the
    detour (r,W) (r,W+1) (r+1,W+1) (r+1,W): +2 squares each."""
    out = list(loop)
    for r in (0, 2, 6)[:bumps]:
        a, b = r * 10 + W, (r + 1) * 10 + W
        i = out.index(a)
        assert out[(i + 1) % len(out)] == b
        out[i + 1:i + 1] = [a + 1, b + 1]
    return out


def check_loop(loop: list[int]) -> None:
    assert len(set(loop)) == len(loop) and not LAKES & set(loop)
    for i, a in enumerate(loop):
        b = loop[(i + 1) % len(loop)]
        assert abs(a // 10 - b // 10) + abs(a % 10 - b % 10) == 1, (a, b)


LOOPS = {60: (6, 0), 62: (6, 1), 64: (6, 2), 66: (6, 3), 84: (9, 0)}


def play(R, loop: list[int], plies: int, no_attack_limit: int):
    L = len(loop)
    st = R.StrategoState(no_attack_limit=no_attack_limit)
    owner = np.full(100, -1, np.int8)
    piece = np.zeros(100, np.int8)
    owner[loop[0]], piece[loop[0]] = 0, 4   # Red sergeant, the chaser
    owner[loop[2]], piece[loop[2]] = 1, 4   # Blue sergeant, the evader
    st.board_owner[:] = owner.reshape(10, 10)
    st.board_piece[:] = piece.reshape(10, 10)
    st._red_setup_done = st._blue_setup_done = True
    ts, ch = R.TwoSquareTracker(), R.ChasingTracker()
    acts = np.full(plies, -1, np.int32)
    ev_ts = np.zeros(plies, np.uint8)
    ev_ch = np.zeros(plies, np.uint8)
    pos = {0: 0, 1: 2}  # loop index of each side's sergeant
    S = R.Square
    for t in range(plies):
        assert not st.is_terminal
        player = int(st.current_player)
        src, dst = loop[pos[player] % L], loop[(pos[player] + 1) % L]
        a = src * 100 + dst
        legal = {x.src.idx * 100 + x.dst.idx for x in st.legal_actions()}
        assert a in legal, (t, a)
        action = R.Action(S.from_idx(src), S.from_idx(dst))
        bo, bp = st.board_owner.copy(), st.board_piece.copy()
        ev_ts[t] = ts.is_violation(R.Player(player), S.from_idx(src), action, False, [S.from_idx(dst)], False)
        ev_ch[t] = ch.is_chasing_violation(R.Player(player), action, bo, bp)
        st.apply_action(action)
        ts.record_move(R.Player(player), S.from_idx(src), action, False, [S.from_idx(dst)], False)
        ch.record_move(R.Player(player), action, bo, bp, st.board_owner, st.board_piece)
        acts[t] = a
        pos[player] += 1
    return owner, piece, acts, ev_ts, ev_ch


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
    plies, nal = 2 * 84 + 20, 1000
    out = {k: [] for k in ("owner", "piece", "actions", "ev_two_square", "ev_chasing", "cycle_len")}
    for L, (W, bumps) in LOOPS.items():
        loop = with_bumps(serpentine(W), W, bumps)
        check_loop(loop)
        assert len(loop) == L
        ow, pc, a, t, c = play(R, loop, plies, nal)
        for k, v in zip(out, (ow, pc, a, t, c, L)):
            out[k].append(v)
    res = {k: np.stack(v) if k != "cycle_len" else np.asarray(v, np.int32) for k, v in out.items()}
    res["no_attack_limit"] = np.full(len(LOOPS), nal, np.int32)
    np.savez_compressed(HERE / "isf_long_chase.npz", **res)
    first = [int(np.argmax(c)) if c.any() else -1 for c in res["ev_chasing"]]
    print("isf_long_chase.npz", (HERE / "isf_long_chase.npz").stat().st_size, "bytes; loops",
          list(LOOPS), "first chasing verdict at ply", first)


if __name__ == "__main__":
    main()
