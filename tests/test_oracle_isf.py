"""The oracle's ISF repetition rules against the reference's own trackers.

``tests/golden/isf.npz`` (made by ``tests/golden/make_golden_isf.py``) holds
games played by the reference's Python engine, each move judged by the
reference's ``TwoSquareTracker`` (stratego/env/two_square.py:27-94) and
``ChasingTracker`` (stratego/env/chasing.py:54-109) before it was recorded.
The oracle (rules=RULES_ISF) replays every game from its initial board and
must flag exactly the same moves, rule by rule, and end every game the same
way.  Two scenarios of the reference's unit tests
(tests/test_two_square.py, tests/test_chasing.py) are restated as real
games on top.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "isf.npz"


def _planes(owner, piece):
    red = np.where(owner == 0, piece, 0).astype(np.int8).reshape(-1, 10, 10)
    blue = np.where(owner == 1, piece, 0).astype(np.int8).reshape(-1, 10, 10)
    return red, blue


@pytest.fixture(scope="module")
def golden():
    with np.load(GOLDEN) as f:
        return {k: f[k] for k in f.files}


@pytest.mark.parametrize("kind", [0, 1, 2, 3])
def test_oracle_isf_events_match_reference_trackers(golden, kind):
    sel = np.nonzero(golden["kind"] == kind)[0]
    g = {k: v[sel] for k, v in golden.items()}
    n, plies = g["actions"].shape
    nal = int(g["no_attack_limit"][0])
    o = oracle.OracleState(n, no_attack_limit=nal, rules=oracle.RULES_ISF)
    o.reset_planes(*_planes(g["owner"], g["piece"]), force_all=True)
    for t in range(plies):
        acts = g["actions"][:, t].astype(np.int64)
        live = acts >= 0
        if not live.any():
            break
        before_ts = o.a["two_square_violation"].copy()
        o.apply(np.where(live, acts, 0))
        ev = o.isf_event
        np.testing.assert_array_equal((ev[live] & 1), g["ev_two_square"][live, t], err_msg=f"two-square ply {t}")
        np.testing.assert_array_equal((ev[live] >> 1) & 1, g["ev_chasing"][live, t], err_msg=f"chasing ply {t}")
        assert (o.a["invalid_count"] == 0).all()
        assert (o.a["two_square_violation"] >= before_ts).all()
    # every recorded game ended where the reference's did
    ended = (g["actions"] >= 0).sum(1) < plies
    assert (o.a["terminated"][ended] == 1).all()
    if kind:
        assert g["ev_two_square"].sum() > 0
    if kind == 3:
        assert g["ev_chasing"].sum() > 0


def _board(pieces):
    owner = np.full((1, 100), -1, np.int8)
    piece = np.zeros((1, 100), np.int8)
    for sq, ow, pt in pieces:
        owner[0, sq], piece[0, sq] = ow, pt
    return _planes(owner, piece)


def _play(o, moves):
    ev = []
    for src, dst in moves:
        o.apply(np.array([src * 100 + dst]))
        assert int(o.a["invalid_count"][0]) == 0, (src, dst)
        ev.append(int(o.isf_event[0]))
    return ev


def test_isf_two_square_fourth_crossing_and_attack_reset():
    """test_two_square.py TestBasicRule / attack-resets, as a game: a Red
    Sergeant oscillates 30<->31 while Blue shuffles far away."""
    o = oracle.OracleState(1, rules=oracle.RULES_ISF)
    o.reset_planes(*_board([(30, 0, 4), (0, 0, 11), (99, 1, 11), (80, 1, 4)]), force_all=True)
    ev = _play(o, [(30, 31), (80, 81), (31, 30), (81, 80), (30, 31), (80, 81), (31, 30)])
    assert [e & 1 for e in ev] == [0, 0, 0, 0, 0, 0, 1]


def test_isf_scout_long_moves_share_pairs():
    """test_two_square.py TestScoutSpecialCase: a scout oscillating A<->D on
    row 3 breaks the rule on the 4th long move, and a plain D->C move after
    three long moves hits the counted pair {C, D}."""
    o = oracle.OracleState(1, rules=oracle.RULES_ISF)
    o.reset_planes(*_board([(30, 0, 2), (0, 0, 11), (99, 1, 11), (80, 1, 4)]), force_all=True)
    ev = _play(o, [(30, 33), (80, 81), (33, 30), (81, 80), (30, 33), (80, 81), (33, 30)])
    assert [e & 1 for e in ev] == [0, 0, 0, 0, 0, 0, 1]
    o2 = oracle.OracleState(1, rules=oracle.RULES_ISF)
    o2.reset_planes(*_board([(30, 0, 2), (0, 0, 11), (99, 1, 11), (80, 1, 4)]), force_all=True)
    ev = _play(o2, [(30, 33), (80, 81), (33, 30), (81, 80), (30, 33), (80, 81), (33, 32)])
    assert [e & 1 for e in ev] == [0, 0, 0, 0, 0, 0, 1]


def test_isf_chase_needs_an_evasion():
    """chasing.py:66-72: a repeated threatening position counts only during a
    chase, i.e. while the opponent keeps evading.  A Red sergeant circles
    through squares that each threaten a Blue piece that never moves (Blue
    shuffles another piece): the CUDA class's rule flags the repeated
    position, the ISF rule does not."""
    pieces = [(25, 0, 4), (24, 1, 4), (27, 1, 4), (37, 1, 4), (34, 1, 4), (80, 1, 4), (0, 0, 11), (99, 1, 11)]
    # Red circles 25 -> 26 -> 36 -> 35 -> 25 -> 26, every square next to a Blue
    # piece and never back to the square it just left
    moves = [(25, 26), (80, 81), (26, 36), (81, 80), (36, 35), (80, 81), (35, 25), (81, 80), (25, 26)]
    cuda = oracle.OracleState(1)
    cuda.reset_planes(*_board(pieces), force_all=True)
    _play(cuda, moves)
    assert int(cuda.a["chasing_violation"][0]) == 1
    isf = oracle.OracleState(1, rules=oracle.RULES_ISF)
    isf.reset_planes(*_board(pieces), force_all=True)
    ev = _play(isf, moves)
    assert int(isf.a["chasing_violation"][0]) == 0 and not any(e & 2 for e in ev)


LONG_CHASE = Path(__file__).resolve().parent / "golden" / "isf_long_chase.npz"


def test_isf_chase_memory_bound_against_reference():
    """The one place the ISF chasing rule departs from the reference: a chase
    remembers its last 64 positions (the reference's set, chasing.py:54-109,
    is unbounded).  ``isf_long_chase.npz`` (tests/golden/make_golden_isf_chase.py)
    holds chases around loops of L squares judged by the reference's own
    tracker, which flags the chaser's return to the chase's first position
    (ply 2L + 2) and every chasing move after it.  The oracle agrees move for
    move while L <= 64 and flags nothing once L > 64; two-square verdicts
    agree everywhere."""
    with np.load(LONG_CHASE) as f:
        g = {k: f[k] for k in f.files}
    n, plies = g["actions"].shape
    o = oracle.OracleState(n, no_attack_limit=int(g["no_attack_limit"][0]), rules=oracle.RULES_ISF)
    o.reset_planes(*_planes(g["owner"], g["piece"]), force_all=True)
    ev = np.zeros((n, plies), np.uint8)
    for t in range(plies):
        o.apply(g["actions"][:, t].astype(np.int64))
        ev[:, t] = o.isf_event
    assert (o.a["invalid_count"] == 0).all() and (o.a["terminated"] == 0).all()
    np.testing.assert_array_equal(ev & 1, g["ev_two_square"])
    for i, L in enumerate(g["cycle_len"]):
        ref = g["ev_chasing"][i]
        first = 2 * int(L) + 2
        # the reference: every Red (chaser) move from ply 2L + 2 on, nothing before
        assert not ref[:first].any() and ref[first::2].all() and not ref[first + 1::2].any()
        if L <= 64:
            np.testing.assert_array_equal((ev[i] >> 1) & 1, ref, err_msg=f"loop {L}")
        else:
            assert not ((ev[i] >> 1) & 1).any(), f"loop {L}"
    assert sorted(g["cycle_len"].tolist()) == [60, 62, 64, 66, 84]
