"""Pin the CPU oracle against the golden traces made by the reference's Python engine.

tests/golden/make_golden.py ran ``stratego.env.rules.StrategoState`` and
``stratego.env.infostate.compute_infostate`` (with the CUDA simulator's
tracker semantics restated in Python) on seeded setups and Philox-chosen
uniform legal actions.  This test replays the same seeds through the C oracle
and requires every snapshot to match: board, trackers, Zobrist hash, the
legal-move set (digest of the packed mask), the float32 infostate (digest,
plus full arrays for a few envs), actions, rewards and dones.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from _helpers import board_code, digest

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


def _snapshot(o: oracle.OracleState) -> dict[str, np.ndarray]:
    a = o.a
    n = o.n
    info = o.infostate_f32()
    bits = o.legal_mask_bits()
    return {
        "board": board_code(a["board_owner"], a["board_piece"]),
        "moved": np.packbits(a["moved_squares"], axis=1, bitorder="little"),
        "revealed": np.packbits(a["revealed_squares"], axis=1, bitorder="little"),
        "current_player": a["current_player"].astype(np.int8),
        "outcome": a["outcome"].astype(np.int8),
        "flag_captured": a["flag_captured"].astype(np.int8),
        "move_number": a["move_number"],
        "moves_since_attack": a["moves_since_attack"],
        "terminated_since": a["terminated_since"],
        "hist_head": a["move_history_head"],
        "hist_len": a["move_history_len"],
        "hist_digest": np.array([digest(a["move_history"][g]) for g in range(n)]),
        "ts_count": a["two_square_count"],
        "ts_lo": a["two_square_pair_lo"],
        "ts_hi": a["two_square_pair_hi"],
        "ts_violation": a["two_square_violation"].astype(np.int8),
        "chase_head": a["chase_hash_head"],
        "chase_len": a["chase_hash_len"],
        "chase_last_src": a["chase_last_src"],
        "chase_digest": np.array([digest(a["chase_hashes"][g]) for g in range(n)]),
        "chase_violation": a["chasing_violation"].astype(np.int8),
        "hash": o.hash_board(),
        "n_legal": np.unpackbits(bits, axis=1).sum(1).astype(np.int32),
        "mask_digest": np.array([digest(bits[g]) for g in range(n)]),
        "info_digest": np.array([digest(info[g]) for g in range(n)]),
        "episode": a["episode"],
        "_info": info,
        "_bits": bits,
    }


@pytest.mark.parametrize("name", ["config1", "autoreset"])
def test_oracle_matches_reference_trace(name):
    g = _load(name)
    n, plies, seed, pool_size, auto_reset, no_attack_limit = (int(x) for x in g["meta"])
    pool = oracle.make_setup_pool(seed, pool_size)
    np.testing.assert_array_equal(pool, g["pool"], err_msg="setup pool differs from the Python restatement")
    o = oracle.OracleState(n, seed=seed, pool=pool, no_attack_limit=no_attack_limit,
                           max_game_length=int(g["max_game_length"]))
    o.reset_pool(force_all=True)
    full_plies = list(g["full_plies"])
    for t in range(plies + 1):
        if t > 0:
            r = o.step(None, auto_reset=bool(auto_reset))
            np.testing.assert_array_equal(r["action"], g["actions"][t - 1], err_msg=f"actions at ply {t - 1}")
            np.testing.assert_array_equal(r["reward"], g["reward"][t - 1], err_msg=f"reward at ply {t - 1}")
            np.testing.assert_array_equal(r["done"], g["done"][t - 1], err_msg=f"done at ply {t - 1}")
        s = _snapshot(o)
        for k, v in s.items():
            if k.startswith("_"):
                continue
            np.testing.assert_array_equal(v, g[k][t], err_msg=f"{name}: field {k} at snapshot {t}")
        if t in full_plies:
            i = full_plies.index(t)
            ne = g["full_info"].shape[1]
            np.testing.assert_array_equal(s["_info"][:ne], g["full_info"][i])
            np.testing.assert_array_equal(s["_bits"][:ne], g["full_mask"][i])


def test_golden_trace_exercises_the_rules():
    """The fixtures are only useful if they reach the interesting paths."""
    c1 = _load("config1")
    assert (c1["outcome"][-1] >= 0).sum() > 5           # games ended (flag captures)
    assert c1["ts_violation"][-1].sum() > 0             # two-square violations
    assert c1["chase_len"].max() > 2                     # chase rings in use
    ar = _load("autoreset")
    assert ar["done"].sum() > 50 and ar["episode"][-1].min() > 1  # auto-resets happened
