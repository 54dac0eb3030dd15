"""The oracle against fixtures made by the reference's own CUDA kernels.

``tests/golden/refcuda.npz`` was produced on a B200 by
``tests/golden/make_golden_refcuda.py``, which ran the reference's
``csrc/stratego_buffer.cu`` (compiled from its source) on two committed
action streams.  The fields it pins are the ones that only the reference's
CUDA class defines -- moved / revealed squares, the move-history ring, the
per-mover two-square tracker, the 64-entry chase rings and the chasing flag
-- together with boards, counters, hashes, masks and infostate digests.  The
oracle (and through the GPU tests, this repository's kernels) must match
them; channels 41 / 42, which the reference divides with fast math, to 1e-6.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from _helpers import board_code, digest

GOLDEN = Path(__file__).resolve().parent / "golden"
FIX = GOLDEN / "refcuda.npz"

pytestmark = pytest.mark.skipif(not FIX.exists(), reason="refcuda.npz not generated yet")


def _snapshot(o: oracle.OracleState) -> dict[str, np.ndarray]:
    a = o.a
    n = o.n
    mask = o.legal_mask_u8().reshape(n, -1)
    info = o.infostate_f32().reshape(n, 488, 100)
    bits = np.packbits(mask, axis=1, bitorder="little")
    planes = np.concatenate([info[:, :41], info[:, 43:]], axis=1)
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
        "hist_digest": np.array([digest(a["move_history"][g].astype(np.int32)) for g in range(n)]),
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
        "n_legal": mask.sum(1).astype(np.int32),
        "mask_digest": np.array([digest(bits[g]) for g in range(n)]),
        "planes_digest": np.array([digest(planes[g]) for g in range(n)]),
        "ch41": info[:, 41, 0].copy(),
        "ch42": info[:, 42, 0].copy(),
    }


def _compare(snap, fix, prefix, t):
    for k, v in snap.items():
        ref = fix[f"{prefix}{k}"] if t is None else fix[f"{prefix}{k}"][t]
        if k in ("ch41", "ch42"):
            np.testing.assert_allclose(v, ref, atol=1e-6, rtol=0, err_msg=f"{prefix}{k} at {t}")
        else:
            np.testing.assert_array_equal(v, ref, err_msg=f"{prefix}{k} at snapshot {t}")


@pytest.fixture(scope="module")
def fix():
    with np.load(FIX) as f:
        return {k: f[k] for k in f.files}


def test_oracle_replays_reference_kernels_config1(fix):
    with np.load(GOLDEN / "config1.npz") as f:
        g = {k: f[k] for k in f.files}
    n, plies, seed = (int(x) for x in g["meta"][:3])
    o = oracle.OracleState(n, seed=seed, pool=g["pool"])
    o.reset_pool(force_all=True)
    o.a["episode"][:] = 0
    _compare(_snapshot(o), fix, "c1_", 0)
    for t in range(plies):
        o.apply(g["actions"][t])
        _compare(_snapshot(o), fix, "c1_", t + 1)


def test_config1_restatement_equals_reference_kernels(fix):
    """The Python restatement of the CUDA-only trackers that made
    config1.npz gives what the reference kernels give."""
    with np.load(GOLDEN / "config1.npz") as f:
        for k in ("board", "moved", "revealed", "current_player", "outcome", "flag_captured", "move_number",
                  "moves_since_attack", "terminated_since", "hist_head", "hist_len", "hist_digest", "ts_count",
                  "ts_lo", "ts_hi", "ts_violation", "chase_head", "chase_len", "chase_last_src", "chase_digest",
                  "chase_violation", "hash", "n_legal", "mask_digest"):
            np.testing.assert_array_equal(f[k], fix[f"c1_{k}"], err_msg=k)


def test_oracle_replays_reference_kernels_chase_streams(fix):
    with np.load(GOLDEN / "isf.npz") as f:
        g = {k: f[k] for k in f.files}
    n, plies = g["actions"].shape
    o = oracle.OracleState(n)  # the reference class's limits: no-attack 100, length 4000
    ow, pc = g["owner"], g["piece"]
    o.reset_planes(np.where(ow == 0, pc, 0), np.where(ow == 1, pc, 0), force_all=True)
    for t in range(plies):
        o.apply(g["actions"][:, t].astype(np.int64))
        np.testing.assert_array_equal(o.a["two_square_violation"], fix["isf_ts_violation"][t], err_msg=f"ply {t}")
        np.testing.assert_array_equal(o.a["chasing_violation"], fix["isf_chase_violation"][t], err_msg=f"ply {t}")
    _compare(_snapshot(o), fix, "isf_end_", None)
    np.testing.assert_array_equal(o.a["chase_hashes"], fix["isf_end_chase_hashes"])
    np.testing.assert_array_equal(o.a["move_history"], fix["isf_end_move_history"])
    assert fix["isf_chase_violation"][-1].sum() >= 10  # the streams reach the chasing rule (10 games)
    assert fix["isf_ts_violation"][-1].sum() >= 100
