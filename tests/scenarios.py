"""Known-answer scenarios of the reference simulator, runnable on any buffer.

Each ``sc_*`` function takes ``make(n_games, **kw)`` returning an object with
the reference StrategoRolloutBuffer API.  The scenarios restate the
reference's own CUDA tests (file:line of each cited) plus edge cases the
reference engine defines (stratego/env/rules.py) but those tests do not reach.
``tests/test_oracle_scenarios.py`` runs them on the CPU oracle and
``tests/test_gpu_scenarios.py`` on the B200 buffer.
"""

from __future__ import annotations

import torch

from _helpers import (
    NUM_INFOSTATE_CHANNELS,
    NUM_SQUARES,
    OUTCOME_BLUE_WIN,
    OUTCOME_DRAW,
    OUTCOME_ONGOING,
    OUTCOME_RED_WIN,
    PLAYER_BLUE,
    PLAYER_EMPTY,
    PLAYER_RED,
    PT_BOMB,
    PT_CAPTAIN,
    PT_FLAG,
    PT_MARSHAL,
    PT_MINER,
    PT_NONE,
    PT_SCOUT,
    PT_SERGEANT,
    PT_SPY,
    UNIFORM_PROB,
    encode_action as enc,
    make_setup,
)

A = lambda *xs: torch.tensor(list(xs), dtype=torch.int64)  # noqa: E731

# Blue shuttles used by tests/test_cuda_rules.py:83-95
SHUTTLE_CYCLE = [enc(8, 8, 8, 9), enc(8, 9, 9, 9), enc(9, 9, 9, 8), enc(9, 8, 8, 8)]
SHUTTLE_OSC = [enc(8, 8, 8, 9), enc(8, 9, 8, 8)]


def alternate(buf, red_moves, blue_moves, n=1):
    for i in range(max(len(red_moves), len(blue_moves))):
        if i < len(red_moves):
            buf.apply_actions(torch.tensor([red_moves[i]] * n, dtype=torch.int64))
        if i < len(blue_moves):
            buf.apply_actions(torch.tensor([blue_moves[i]] * n, dtype=torch.int64))


def approx(x: float, y: float, tol: float = 1e-6) -> bool:
    return abs(float(x) - float(y)) <= tol


# ---------------------------------------------------------------------------
# tests/test_cuda_sim.py:108-260
# ---------------------------------------------------------------------------
def sc_construction(make):
    buf = make(4)
    assert buf.n_games == 4 and buf.device_id == 0


def sc_simple_move(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 0, PT_SPY)], []))
    buf.apply_actions(A(enc(3, 0, 4, 0)))
    ow, pc = buf.get_board_owner(), buf.get_board_piece()
    assert ow[0, 4, 0].item() == PLAYER_RED and pc[0, 4, 0].item() == PT_SPY
    assert ow[0, 3, 0].item() == PLAYER_EMPTY and pc[0, 3, 0].item() == PT_NONE


def sc_mask_shape_empty(make):
    buf = make(4)
    m = buf.compute_legal_action_mask()
    assert tuple(m.shape) == (4, NUM_SQUARES, NUM_SQUARES) and m.dtype == torch.bool
    assert not m.any().item()


def sc_mask_with_pieces(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 0, PT_SPY)], []))
    m = buf.compute_legal_action_mask()
    assert m[0, 30, 20].item() and m[0, 30, 40].item() and m[0, 30, 31].item()
    assert not m[0, 30, 39].item()
    assert int(m.sum().item()) == 3


def sc_spy_defeats_marshal(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 0, PT_SPY)], [(4, 0, PT_MARSHAL)]))
    buf.apply_actions(A(enc(3, 0, 4, 0)))
    ow, pc = buf.get_board_owner(), buf.get_board_piece()
    assert ow[0, 4, 0].item() == PLAYER_RED and pc[0, 4, 0].item() == PT_SPY
    assert ow[0, 3, 0].item() == PLAYER_EMPTY


def sc_marshal_defeats_attacking_spy_reverse(make):
    # Marshal attacking Spy wins by rank (rules.py:344-359)
    buf = make(1)
    buf.reset_all(*make_setup([(3, 0, PT_MARSHAL)], [(4, 0, PT_SPY), (9, 9, PT_FLAG)]))
    buf.apply_actions(A(enc(3, 0, 4, 0)))
    ow, pc = buf.get_board_owner(), buf.get_board_piece()
    assert ow[0, 4, 0].item() == PLAYER_RED and pc[0, 4, 0].item() == PT_MARSHAL


def sc_miner_defeats_bomb(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 1, PT_MINER)], [(4, 1, PT_BOMB)]))
    buf.apply_actions(A(enc(3, 1, 4, 1)))
    ow, pc = buf.get_board_owner(), buf.get_board_piece()
    assert ow[0, 4, 1].item() == PLAYER_RED and pc[0, 4, 1].item() == PT_MINER
    assert ow[0, 3, 1].item() == PLAYER_EMPTY


def sc_bomb_kills_non_miner(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 1, PT_CAPTAIN), (0, 0, PT_SPY)], [(4, 1, PT_BOMB), (9, 9, PT_SPY)]))
    buf.apply_actions(A(enc(3, 1, 4, 1)))
    ow, pc = buf.get_board_owner(), buf.get_board_piece()
    assert ow[0, 3, 1].item() == PLAYER_EMPTY
    assert ow[0, 4, 1].item() == PLAYER_BLUE and pc[0, 4, 1].item() == PT_BOMB
    assert buf.get_num_moves_since_last_attack()[0].item() == 0


def sc_equal_rank_both_die(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 4, PT_SERGEANT)], [(4, 4, PT_SERGEANT)]))
    buf.apply_actions(A(enc(3, 4, 4, 4)))
    ow, pc = buf.get_board_owner(), buf.get_board_piece()
    assert ow[0, 3, 4].item() == PLAYER_EMPTY and pc[0, 3, 4].item() == PT_NONE
    assert ow[0, 4, 4].item() == PLAYER_EMPTY and pc[0, 4, 4].item() == PT_NONE


def sc_defender_wins(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 4, PT_SERGEANT), (0, 0, PT_SPY)], [(4, 4, PT_CAPTAIN), (9, 9, PT_SPY)]))
    buf.apply_actions(A(enc(3, 4, 4, 4)))
    ow, pc = buf.get_board_owner(), buf.get_board_piece()
    assert ow[0, 3, 4].item() == PLAYER_EMPTY
    assert ow[0, 4, 4].item() == PLAYER_BLUE and pc[0, 4, 4].item() == PT_CAPTAIN


def sc_flag_capture_wins(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 5, PT_SPY)], [(4, 5, PT_FLAG)]))
    buf.apply_actions(A(enc(3, 5, 4, 5)))
    assert buf.get_outcomes()[0].item() == OUTCOME_RED_WIN
    assert buf.get_terminated()[0].item() is True
    assert buf.compute_reward_pl0()[0].item() == 1.0


def sc_outcomes_initial(make):
    buf = make(4)
    o = buf.get_outcomes()
    assert tuple(o.shape) == (4,) and o.dtype == torch.int8 and torch.all(o == OUTCOME_ONGOING).item()
    t = buf.get_terminated()
    assert tuple(t.shape) == (4,) and t.dtype == torch.bool and not t.any().item()


def sc_current_step(make):
    buf = make(2)
    buf.reset_all(*make_setup([(3, 0, PT_SPY), (3, 1, PT_SPY)], [(6, 0, PT_FLAG), (6, 1, PT_FLAG)], n_games=2))
    assert buf.current_step() == 0
    buf.apply_actions(A(enc(3, 0, 4, 0), enc(3, 1, 4, 1)))
    assert buf.current_step() == 2


def sc_hello_world(make):
    r = make(1).hello_world()
    assert tuple(r.shape) == (1,) and r.dtype == torch.int32 and r.item() == 42


# ---------------------------------------------------------------------------
# tests/test_cuda_api.py:78-162
# ---------------------------------------------------------------------------
def sc_getters_initial(make):
    buf = make(3)
    for t, dt in ((buf.get_num_moves(), torch.int32), (buf.get_num_moves_since_last_attack(), torch.int32),
                  (buf.get_terminated_since(), torch.int32)):
        assert tuple(t.shape) == (3,) and t.dtype == dt and torch.all(t == 0).item()
    fc = buf.get_flag_captured()
    assert fc.dtype == torch.bool and not fc.any().item()


def sc_flag_captured(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 5, PT_SPY)], [(4, 5, PT_FLAG)]))
    buf.apply_actions(A(enc(3, 5, 4, 5)))
    assert buf.get_flag_captured()[0].item() is True
    assert buf.get_terminated_since()[0].item() >= 1
    buf2 = make(1)
    buf2.reset_all(*make_setup([(3, 0, PT_SPY)], []))
    buf2.apply_actions(A(enc(3, 0, 4, 0)))
    assert not buf2.get_flag_captured()[0].item()


def sc_has_legal_movement(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 0, PT_SPY)], []))
    h = buf.get_has_legal_movement()
    assert tuple(h.shape) == (1,) and h.dtype == torch.bool and h[0].item() is True
    assert not make(1).get_has_legal_movement()[0].item()


def sc_board_strs(make):
    buf = make(1)
    buf.reset_all(*make_setup([(3, 0, PT_SPY)], [(9, 9, PT_MARSHAL)]))
    s = buf.board_strs()
    assert len(s) == 1 and isinstance(s[0], str) and "R1" in s[0] and "B10" in s[0]
    lines = s[0].split("\n")
    assert lines[3].startswith("R1 . ") and lines[9].endswith("B10")
    s2 = make(2).board_strs()
    assert len(s2) == 2 and all(isinstance(x, str) for x in s2)


# ---------------------------------------------------------------------------
# tests/test_cuda_rules.py:112-424
# ---------------------------------------------------------------------------
def sc_two_square(make):
    buf = make(3)
    v = buf.compute_two_square_rule_applies()
    assert tuple(v.shape) == (3,) and v.dtype == torch.bool and not v.any().item()
    red, blue = make_setup([(3, 0, PT_SERGEANT)], [(8, 8, PT_SERGEANT)])
    osc = [enc(3, 0, 4, 0), enc(4, 0, 3, 0), enc(3, 0, 4, 0), enc(4, 0, 3, 0)]
    b = make(1)
    b.reset_all(red, blue)
    b.apply_actions(A(osc[0]))
    assert not b.compute_two_square_rule_applies()[0].item()
    b = make(1)
    b.reset_all(red, blue)
    alternate(b, osc[:3], SHUTTLE_CYCLE[:3])
    assert not b.compute_two_square_rule_applies()[0].item()
    b = make(1)
    b.reset_all(red, blue)
    alternate(b, osc, SHUTTLE_CYCLE[:4])
    assert b.compute_two_square_rule_applies()[0].item()
    b.reset_all(red, blue)  # reset clears (test_cuda_rules.py:200-214)
    assert not b.compute_two_square_rule_applies()[0].item()
    b = make(1)
    b.reset_all(red, blue)
    alternate(b, [enc(3, 0, 4, 0), enc(4, 0, 4, 1), enc(4, 1, 3, 1)], SHUTTLE_CYCLE[:3])
    assert not b.compute_two_square_rule_applies()[0].item()
    b = make(1)  # sticky (test_cuda_rules.py:185-198)
    b.reset_all(red, blue)
    alternate(b, osc + [enc(3, 0, 3, 1)], SHUTTLE_CYCLE[:5] + [SHUTTLE_CYCLE[0]])
    assert b.compute_two_square_rule_applies()[0].item()


def sc_two_square_attack_resets(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_MARSHAL)], [(5, 0, PT_SERGEANT), (8, 8, PT_SERGEANT)]))
    alternate(b, [enc(3, 0, 4, 0), enc(4, 0, 3, 0), enc(3, 0, 4, 0), enc(4, 0, 5, 0)], SHUTTLE_CYCLE[:4])
    assert not b.compute_two_square_rule_applies()[0].item()
    st = b.export_state()
    assert st["two_square_count"][0, 0].item() == 0
    assert st["two_square_pair_lo"][0, 0].item() == -1


def sc_hash_board(make):
    b = make(2)
    b.reset_all(*make_setup([(3, 0, PT_SERGEANT)], [(6, 0, PT_SERGEANT)], n_games=2))
    h1, h2 = b.hash_board(), b.hash_board()
    assert tuple(h1.shape) == (2,) and h1.dtype == torch.int64 and torch.equal(h1, h2)
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SERGEANT)], [(6, 0, PT_SERGEANT)]))
    h0 = b.hash_board()[0].item()
    b.apply_actions(A(enc(3, 0, 4, 0)))
    assert b.hash_board()[0].item() != h0
    assert make(1).hash_board()[0].item() == 0  # empty board (test_chasing.py:369-374)


def sc_chasing(make):
    b = make(3)
    v = b.is_chasing_violation()
    assert tuple(v.shape) == (3,) and v.dtype == torch.bool and not v.any().item()
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SERGEANT)], [(8, 8, PT_SERGEANT)]))
    b.apply_actions(A(enc(3, 0, 4, 0)))
    assert not b.is_chasing_violation()[0].item()
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SERGEANT)], [(5, 0, PT_SERGEANT), (8, 8, PT_SERGEANT)]))
    b.apply_actions(A(enc(3, 0, 4, 0)))
    assert not b.is_chasing_violation()[0].item()


CHASE_BLUE = [(5, 0, PT_SERGEANT), (5, 1, PT_SERGEANT), (2, 1, PT_SERGEANT), (2, 0, PT_SERGEANT), (8, 8, PT_SERGEANT)]
CHASE_RED_CYCLE = [enc(3, 0, 4, 0), enc(4, 0, 4, 1), enc(4, 1, 3, 1), enc(3, 1, 3, 0), enc(3, 0, 4, 0)]


def sc_chasing_violation_4cycle(make):
    b = make(1)
    red, blue = make_setup([(3, 0, PT_SERGEANT)], CHASE_BLUE)
    b.reset_all(red, blue)
    alternate(b, CHASE_RED_CYCLE, SHUTTLE_CYCLE[:4])
    assert b.is_chasing_violation()[0].item()
    b.reset_all(red, blue)
    assert not b.is_chasing_violation()[0].item()


def sc_chasing_exception(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SERGEANT)], [(5, 0, PT_SERGEANT), (2, 0, PT_SERGEANT), (8, 8, PT_SERGEANT)]))
    alternate(b, [enc(3, 0, 4, 0), enc(4, 0, 3, 0), enc(3, 0, 4, 0)], SHUTTLE_OSC[:2])
    assert not b.is_chasing_violation()[0].item()


def sc_two_square_in_one_game(make):
    n = 2
    b = make(n)
    b.reset_all(*make_setup([(3, 0, PT_SERGEANT)], [(8, 8, PT_SERGEANT)], n_games=n))
    red = [A(enc(3, 0, 4, 0), enc(3, 0, 4, 0)), A(enc(4, 0, 3, 0), enc(4, 0, 4, 1)),
           A(enc(3, 0, 4, 0), enc(4, 1, 3, 1)), A(enc(4, 0, 3, 0), enc(3, 1, 3, 0))]
    for i in range(4):
        b.apply_actions(red[i])
        b.apply_actions(torch.tensor([SHUTTLE_CYCLE[i]] * n, dtype=torch.int64))
    v = b.compute_two_square_rule_applies()
    assert v[0].item() and not v[1].item()


# ---------------------------------------------------------------------------
# tests/test_cuda_infostate.py:98-304
# ---------------------------------------------------------------------------
def sc_info_shape(make):
    b = make(3)
    b.reset_all(*make_setup([(3, 0, PT_SPY)], [(6, 0, PT_FLAG)], n_games=3))
    info = b.compute_infostate_tensor()
    assert tuple(info.shape) == (3, NUM_INFOSTATE_CHANNELS, 10, 10) and info.dtype == torch.float32


def sc_info_initial(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SPY)], [(6, 0, PT_FLAG)]))
    info = b.compute_infostate_tensor()
    assert approx(info[0, 0, 3, 0].item(), 1.0) and approx(info[0, 10].sum().item(), 0.0)
    for ch in range(12, 24):
        assert approx(info[0, ch, 6, 0].item(), UNIFORM_PROB)
    assert approx(info[0, 12:24, 6, 0].sum().item(), 1.0, 1e-5)
    assert approx(info[0, 36, 3, 0].item(), 1.0) and approx(info[0, 37, 6, 0].item(), 1.0)
    assert approx(info[0, 38, 0, 0].item(), 1.0) and approx(info[0, 38, 3, 0].item(), 0.0)
    assert approx(info[0, 38, 4, 2].item(), 1.0)  # lakes count as empty
    assert info[0, 43:456].abs().sum().item() == 0.0
    assert info[0, 456:488].abs().sum().item() == 0.0


def sc_info_after_move(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SPY)], [(6, 0, PT_FLAG)]))
    b.apply_actions(A(enc(3, 0, 4, 0)))
    info = b.compute_infostate_tensor()
    assert info[0, 456, 4, 0].item() == 1.0 and info[0, 456, 3, 0].item() == -1.0
    assert info[0, 40, 4, 0].item() == 1.0 and info[0, 40, 3, 0].item() == 0.0
    assert info[0, 37, 4, 0].item() == 1.0
    assert info[0, 457:488].abs().sum().item() == 0.0


def sc_info_after_attack(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SPY)], [(4, 0, PT_MARSHAL), (6, 9, PT_SCOUT)]))
    b.apply_actions(A(enc(3, 0, 4, 0)))
    info = b.compute_infostate_tensor()
    assert info[0, 37, 4, 0].item() == 0.0 and info[0, 12, 4, 0].item() == 1.0
    for ch in range(13, 24):
        assert info[0, ch, 4, 0].item() == 0.0
    assert info[0, 456, 4, 0].item() == 1.0 and info[0, 456, 3, 0].item() == -1.0


def sc_info_scalars(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SPY)], [(6, 0, PT_FLAG)]))
    i0 = b.compute_infostate_tensor()
    assert i0[0, 41].sum().item() == 0.0 and i0[0, 42].sum().item() == 0.0
    b.apply_actions(A(enc(3, 0, 4, 0)))
    i1 = b.compute_infostate_tensor()
    # exact float32 quotients, as numpy makes them from Python floats
    assert torch.equal(i1[0, 41], torch.full((10, 10), 1.0 / 4000.0, dtype=torch.float32, device=i1.device))
    assert torch.equal(i1[0, 42], torch.full((10, 10), 1.0 / 100.0, dtype=torch.float32, device=i1.device))


def sc_info_history(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SCOUT)], [(6, 0, PT_SCOUT)]))
    b.apply_actions(A(enc(3, 0, 2, 0)))
    b.apply_actions(A(enc(6, 0, 7, 0)))
    info = b.compute_infostate_tensor()
    assert info[0, 456, 7, 0].item() == 1.0 and info[0, 456, 6, 0].item() == -1.0
    assert info[0, 457, 2, 0].item() == 1.0 and info[0, 457, 3, 0].item() == -1.0
    assert info[0, 458:488].abs().sum().item() == 0.0


def sc_info_history_overflow(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SCOUT)], [(6, 0, PT_SCOUT)]))
    for i in range(33):
        if i % 2 == 0:
            r, d = (3, 2) if i % 4 == 0 else (2, 3)
        else:
            r, d = (6, 7) if i % 4 == 1 else (7, 6)
        b.apply_actions(A(enc(r, 0, d, 0)))
    info = b.compute_infostate_tensor()
    assert (info[0, 456:488] != 0).any(dim=2).any(dim=1).sum().item() == 32
    assert info[0, 456, 2, 0].item() == 1.0 and info[0, 456, 3, 0].item() == -1.0
    assert info[0, 487, 7, 0].item() == 1.0 and info[0, 487, 6, 0].item() == -1.0


def sc_info_reset_clears(make):
    b = make(1)
    red, blue = make_setup([(3, 0, PT_SPY)], [(6, 0, PT_FLAG)])
    b.reset_all(red, blue)
    b.apply_actions(A(enc(3, 0, 4, 0)))
    assert b.compute_infostate_tensor()[0, 456].abs().sum().item() > 0
    b.reset_all(red, blue)
    after = b.compute_infostate_tensor()
    for ch in (39, 40, 41):
        assert after[0, ch].sum().item() == 0.0
    assert after[0, 456:488].abs().sum().item() == 0.0


# ---------------------------------------------------------------------------
# Edge cases of the rules the reference defines (rules.py, cu:111-399)
# ---------------------------------------------------------------------------
def sc_invalid_actions_ignored(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SCOUT), (3, 5, PT_BOMB)], [(6, 0, PT_SERGEANT), (9, 9, PT_FLAG)]))
    before = b.get_board_owner().clone()
    bad = [-1, 10000, 12345, enc(3, 0, 3, 0),   # out of range / src == dst
           enc(6, 0, 5, 0),                      # not the mover's piece
           enc(3, 5, 4, 5),                      # bomb cannot move
           enc(3, 0, 4, 1),                      # diagonal
           enc(3, 0, 7, 0),                      # scout path blocked by (6,0)
           enc(2, 2, 3, 2)]                      # empty source
    for a in bad:
        b.apply_actions(A(a))
    assert torch.equal(b.get_board_owner(), before)
    assert b.get_current_player()[0].item() == PLAYER_RED and b.get_move_number()[0].item() == 0
    st = b.export_state()
    assert st["invalid_count"][0].item() == len(bad)


def sc_scout_slides(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SCOUT)], [(8, 0, PT_SERGEANT), (9, 9, PT_FLAG)]))
    m = b.compute_legal_action_mask()[0]
    # up 3 squares, right 9, down to and including the enemy at (8,0)
    assert sorted(int(d) for d in torch.nonzero(m[30]).flatten()) == sorted(
        [20, 10, 0] + [31 + i for i in range(9)] + [40, 50, 60, 70, 80])
    b.apply_actions(A(enc(3, 0, 8, 0)))  # long-range attack, scout loses
    assert b.get_board_owner()[0, 8, 0].item() == PLAYER_BLUE
    b2 = make(1)
    b2.reset_all(*make_setup([(4, 1, PT_SCOUT)], [(9, 9, PT_FLAG)]))
    m2 = b2.compute_legal_action_mask()[0]
    assert not m2[41, 42].item() and not m2[41, 43].item()  # lake blocks


def sc_no_legal_move_loses(make):
    # after Red's move Blue has only a bomb and a flag: Blue loses (rules.py:406-413)
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_SERGEANT)], [(9, 0, PT_BOMB), (9, 9, PT_FLAG)]))
    b.apply_actions(A(enc(3, 0, 4, 0)))
    assert b.get_outcomes()[0].item() == OUTCOME_RED_WIN and b.get_terminated()[0].item()
    assert b.compute_reward_pl0()[0].item() == 1.0


def sc_both_immobile_side_to_move_loses(make):
    # rules.py:406-413 via test_rules.py:532-550 style: Red captures the last
    # movable blue piece while Red has movers left -> Blue to move, cannot
    b = make(1)
    b.reset_all(*make_setup([(3, 0, PT_MARSHAL)], [(4, 0, PT_SERGEANT), (9, 9, PT_BOMB), (9, 8, PT_FLAG)]))
    b.apply_actions(A(enc(3, 0, 4, 0)))
    assert b.get_outcomes()[0].item() == OUTCOME_RED_WIN


def sc_no_attack_draw(make):
    b = make(1, no_attack_limit=4)
    b.reset_all(*make_setup([(3, 0, PT_SERGEANT)], [(8, 8, PT_SERGEANT)]))
    alternate(b, [enc(3, 0, 4, 0), enc(4, 0, 4, 1)], SHUTTLE_CYCLE[:2])
    assert b.get_outcomes()[0].item() == OUTCOME_DRAW and b.get_terminated()[0].item()
    assert b.compute_reward_pl0()[0].item() == 0.0
    # terminated games ignore further actions and count terminated_since
    b.apply_actions(A(SHUTTLE_CYCLE[2]))
    assert b.get_move_number()[0].item() == 4 and b.get_terminated_since()[0].item() == 2


def sc_max_length_draw(make):
    b = make(1, max_game_length=3)
    b.reset_all(*make_setup([(3, 0, PT_SERGEANT)], [(8, 8, PT_SERGEANT)]))
    alternate(b, [enc(3, 0, 4, 0), enc(4, 0, 4, 1)], SHUTTLE_CYCLE[:1])
    assert b.get_outcomes()[0].item() == OUTCOME_DRAW


def sc_reset_terminated_only(make):
    b = make(2)
    red, blue = make_setup([(3, 5, PT_SPY)], [(4, 5, PT_FLAG), (9, 9, PT_SPY)], n_games=2)
    b.reset_all(red, blue)
    b.apply_actions(A(enc(3, 5, 4, 5), enc(3, 5, 2, 5)))  # game 0 captures, game 1 moves away
    assert b.get_terminated().tolist() == [True, False]
    b.reset_terminated(red, blue)
    assert b.get_terminated().tolist() == [False, False]
    assert b.get_move_number().tolist() == [0, 1]
    assert b.get_flag_captured().tolist() == [False, False]
    assert b.get_terminated_since().tolist() == [0, 0]
    assert b.get_current_player().tolist() == [PLAYER_RED, PLAYER_BLUE]


def sc_blue_wins_reward(make):
    b = make(1)
    b.reset_all(*make_setup([(3, 3, PT_SPY), (0, 9, PT_FLAG)], [(5, 5, PT_SCOUT), (1, 9, PT_SCOUT)]))
    b.apply_actions(A(enc(3, 3, 3, 4)))
    b.apply_actions(A(enc(19 // 10, 9, 0, 9)))  # blue scout (1,9) takes the flag at (0,9)
    assert b.get_outcomes()[0].item() == OUTCOME_BLUE_WIN
    assert b.compute_reward_pl0()[0].item() == -1.0
    assert b.get_flag_captured()[0].item()


SCENARIOS = [v for k, v in sorted(globals().items()) if k.startswith("sc_") and callable(v)]
