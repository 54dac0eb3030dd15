"""The ISF repetition rules (rules='isf') on the B200, against the oracle and
the reference's own trackers.

* the games of ``tests/golden/isf.npz`` (judged move by move by the
  reference's ``TwoSquareTracker`` / ``ChasingTracker``) replayed through the
  fused step kernel and through ``apply_actions``: the sticky violation flags
  rise exactly when the reference's first violation happens, and the full
  state (per-square two-square intervals, threat lists, evasion bits, chase
  rings) equals the oracle's after every ply;
* random games under the ISF rules: uniform and Gumbel steps, multi-ply
  trajectory launches and belief resampling, bit-exact with the oracle.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from _helpers import assert_state_equal, export_np

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "isf.npz"


def _planes(owner, piece):
    red = np.where(owner == 0, piece, 0).astype(np.int8).reshape(-1, 10, 10)
    blue = np.where(owner == 1, piece, 0).astype(np.int8).reshape(-1, 10, 10)
    return red, blue


@pytest.fixture(scope="module")
def golden():
    with np.load(GOLDEN) as f:
        return {k: f[k] for k in f.files}


@pytest.mark.parametrize("kind,path", [(0, "step"), (1, "step"), (2, "apply"), (3, "step"), (3, "apply")])
def test_isf_golden_games(golden, kind, path):
    from ataraxos_b200 import StrategoRolloutBuffer

    sel = np.nonzero(golden["kind"] == kind)[0]
    g = {k: v[sel] for k, v in golden.items()}
    n, plies = g["actions"].shape
    nal = int(g["no_attack_limit"][0])
    b = StrategoRolloutBuffer(n, 0, no_attack_limit=nal, rules="isf")
    o = oracle.OracleState(n, no_attack_limit=nal, rules=oracle.RULES_ISF)
    red, blue = _planes(g["owner"], g["piece"])
    b.reset_all(torch.from_numpy(red), torch.from_numpy(blue))
    o.reset_planes(red, blue, force_all=True)
    seen_ts = np.zeros(n, bool)
    seen_ch = np.zeros(n, bool)
    for t in range(plies):
        acts = g["actions"][:, t].astype(np.int64)
        live = acts >= 0
        if not live.any():
            break
        a = np.where(live, acts, 0)
        if path == "step":
            b.step(torch.from_numpy(a), auto_reset=False)
        else:
            b.apply_actions(torch.from_numpy(a))
        o.apply(a)
        seen_ts |= live & (g["ev_two_square"][:, t] > 0)
        seen_ch |= live & (g["ev_chasing"][:, t] > 0)
        st = export_np(b)
        np.testing.assert_array_equal(st["two_square_violation"].astype(bool), seen_ts, err_msg=f"ply {t}")
        np.testing.assert_array_equal(st["chasing_violation"].astype(bool), seen_ch, err_msg=f"ply {t}")
        if t % 25 == 0:
            assert_state_equal(st, o.export(), f"kind {kind} ply {t}")
    assert_state_equal(export_np(b), o.export(), f"kind {kind} end")
    assert (export_np(b)["invalid_count"] == 0).all()


@pytest.mark.parametrize("path", ["step", "apply"])
def test_isf_long_chases_match_oracle(path):
    """Chases around loops of 60-84 squares (tests/golden/isf_long_chase.npz):
    the kernel's sticky chasing flag rises where the oracle's does -- the
    reference's verdict while the loop is at most 64 squares long (the chase
    memory), never for the longer loops -- and the full state, chase rings
    included, equals the oracle's."""
    from ataraxos_b200 import StrategoRolloutBuffer

    with np.load(Path(__file__).resolve().parent / "golden" / "isf_long_chase.npz") as f:
        g = {k: f[k] for k in f.files}
    n, plies = g["actions"].shape
    nal = int(g["no_attack_limit"][0])
    b = StrategoRolloutBuffer(n, 0, no_attack_limit=nal, rules="isf")
    o = oracle.OracleState(n, no_attack_limit=nal, rules=oracle.RULES_ISF)
    red, blue = _planes(g["owner"], g["piece"])
    b.reset_all(torch.from_numpy(red), torch.from_numpy(blue))
    o.reset_planes(red, blue, force_all=True)
    seen = np.zeros(n, bool)
    short = g["cycle_len"] <= 64
    for t in range(plies):
        a = g["actions"][:, t].astype(np.int64)
        if path == "step":
            b.step(torch.from_numpy(a), auto_reset=False)
        else:
            b.apply_actions(torch.from_numpy(a))
        o.apply(a)
        seen |= short & (g["ev_chasing"][:, t] > 0)
        st = export_np(b)
        np.testing.assert_array_equal(st["chasing_violation"].astype(bool), seen, err_msg=f"ply {t}")
        if t % 20 == 0:
            assert_state_equal(st, o.export(), f"ply {t}")
    assert seen[short].all() and not seen[~short].any()
    assert_state_equal(export_np(b), o.export(), "end")


@pytest.mark.parametrize("policy", ["uniform", "gumbel"])
def test_isf_random_games_match_oracle(policy):
    from ataraxos_b200 import StrategoRolloutBuffer

    n, plies = 500, 400
    pool = oracle.make_setup_pool(31, 1024)
    b = StrategoRolloutBuffer(n, 0, seed=31, setup_pool=torch.from_numpy(pool), no_attack_limit=60, rules="isf")
    o = oracle.OracleState(n, seed=31, pool=pool, no_attack_limit=60, rules=oracle.RULES_ISF)
    b.reset_all_from_pool()
    o.reset_pool(force_all=True)
    pol = oracle.POLICY_UNIFORM if policy == "uniform" else oracle.POLICY_GUMBEL
    for t in range(1, plies + 1):
        if policy == "uniform":
            b.step(None)
            o.step(None)
        else:
            out = b.step(None, policy="gumbel")
            o.step(out.action.cpu().numpy(), policy=pol)
        if t % 100 == 0:
            assert_state_equal(export_np(b), o.export(), f"ply {t}")
    st = export_np(b)
    assert st["two_square_violation"].sum() > 0


def test_isf_trajectory_and_belief_match_oracle():
    from ataraxos_b200 import StrategoRolloutBuffer
    from ataraxos_b200.trajectory import TrajectoryBuffer

    n = 256
    pool = oracle.make_setup_pool(8, 512)
    b = StrategoRolloutBuffer(n, 0, seed=8, setup_pool=torch.from_numpy(pool), no_attack_limit=40, rules="isf")
    o = oracle.OracleState(n, seed=8, pool=pool, no_attack_limit=40, rules=oracle.RULES_ISF)
    b.reset_all_from_pool()
    o.reset_pool(force_all=True)
    tr = TrajectoryBuffer(b, 16, policy="uniform", obs_dtype=None)
    tr.prime()
    for chunk in (9, 16, 5):
        tr.rollout(chunk)
        for _ in range(chunk):
            o.step(None)
    assert_state_equal(export_np(b), o.export(), "after trajectory launches")
    # belief samples keep the roots' per-square two-square state
    k = 4
    s = StrategoRolloutBuffer(n * k, 0, seed=77, rules="isf", no_attack_limit=40)
    os_ = oracle.OracleState(n * k, seed=77, rules=oracle.RULES_ISF, no_attack_limit=40)
    root_of = np.repeat(np.arange(n), k)
    s.resample_from(b, torch.from_numpy(root_of))
    os_.resample_from(o, root_of)
    assert_state_equal(export_np(s), os_.export(), "belief samples")
    with pytest.raises(RuntimeError):
        StrategoRolloutBuffer(4, 0).resample_from(b, torch.zeros(4, dtype=torch.int64))
