"""This repository's kernels against the reference's own CUDA kernels, on the B200.

``oracle/_ref/libref_stratego_cuda.so`` is the reference's
``csrc/stratego_buffer.cu`` compiled from its source (``oracle/refcuda.py``);
``RefCudaBuffer`` drives it as the reference's pybind class does.  Here:

* the known-answer scenarios of ``tests/scenarios.py`` (restated from the
  reference's tests/test_cuda_*.py) run on the reference kernels themselves,
  which pins the restatement;
* random play on both simulators with the same actions: the full state
  (board, counters, moved / revealed squares, history ring, two-square and
  chasing trackers, chase rings), Zobrist hashes, legal masks and infostate
  must agree after every ply, through the reference API
  (``apply_actions``, ``reset_terminated``) and through the fused step.

Channels 41 and 42 of the infostate are compared to 1e-6: the reference
divides with ``--use_fast_math``, this build rounds the exact quotient as the
reference's Python engine does.  Every other value must be identical.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle import refcuda
from scenarios import SCENARIOS

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not refcuda.available(), reason="reference CUDA library not built here")]

# Scenarios that set limits the reference class hard-codes (no-attack 100, length 4000),
# or read a field only this build keeps (the per-game count of ignored actions).
_NOT_IN_REFERENCE = {"sc_no_attack_draw": "the reference class has no configurable limits",
                     "sc_max_length_draw": "the reference class has no configurable limits",
                     "sc_invalid_actions_ignored": "counts ignored actions, which the reference class does not"}


@pytest.mark.parametrize("scenario", SCENARIOS, ids=[s.__name__ for s in SCENARIOS])
def test_reference_kernels_pass_the_scenarios(scenario):
    if scenario.__name__ in _NOT_IN_REFERENCE:
        pytest.skip(_NOT_IN_REFERENCE[scenario.__name__])

    def make(n, **kw):
        assert not kw
        return refcuda.RefCudaBuffer(n, 0)

    scenario(make)


def _planes(pool: np.ndarray, idx: np.ndarray):
    n = len(idx)
    red = np.zeros((n, 100), np.int8)
    blue = np.zeros((n, 100), np.int8)
    red[:, :40] = pool[idx % len(pool)]
    blue[:, 60:] = pool[(idx * 7 + 3) % len(pool)]
    return torch.from_numpy(red.reshape(n, 10, 10)), torch.from_numpy(blue.reshape(n, 10, 10))


_FIELDS = ("board_owner", "board_piece", "current_player", "outcome", "terminated", "flag_captured", "move_number",
           "moves_since_attack", "terminated_since", "moved_squares", "revealed_squares", "move_history",
           "move_history_head", "move_history_len", "two_square_count", "two_square_pair_lo", "two_square_pair_hi",
           "two_square_violation", "chase_hash_head", "chase_hash_len", "chase_last_src", "chasing_violation",
           "chase_hashes")


def _compare_state(ours, ref, ctx):
    a = ours.export_state()
    b = ref.export_state()
    for k in _FIELDS:
        x = a[k].cpu().numpy().reshape(b[k].shape).astype(np.int64)
        y = b[k].cpu().numpy().astype(np.int64)
        if not np.array_equal(x, y):
            bad = np.argwhere(x != y)[:5].tolist()
            raise AssertionError(f"{ctx}: {k} differs at {bad}")


def _compare_obs(ours, ref, ctx):
    np.testing.assert_array_equal(ours.hash_board().cpu().numpy(), ref.hash_board().cpu().numpy(),
                                  err_msg=f"{ctx}: hash")
    np.testing.assert_array_equal(ours.compute_legal_action_mask().cpu().numpy(),
                                  ref.compute_legal_action_mask().cpu().numpy(), err_msg=f"{ctx}: mask")
    x = ours.compute_infostate_tensor().cpu().numpy()
    y = ref.compute_infostate_tensor().cpu().numpy()
    keep = np.r_[0:41, 43:488]
    np.testing.assert_array_equal(x[:, keep], y[:, keep], err_msg=f"{ctx}: infostate")
    np.testing.assert_allclose(x[:, 41:43], y[:, 41:43], atol=1e-6, rtol=0, err_msg=f"{ctx}: channels 41-42")


@pytest.mark.parametrize("path", ["apply_actions", "fused_step"])
def test_random_play_matches_reference_kernels(path):
    from ataraxos_b200 import StrategoRolloutBuffer

    n, plies, seed = 2048, 400, 4242
    pool = oracle.make_setup_pool(seed, 4096)
    ours = StrategoRolloutBuffer(n, 0, seed=seed, obs_dtype=torch.float32)
    ref = refcuda.RefCudaBuffer(n, 0)
    red, blue = _planes(pool, np.arange(n))
    ours.reset_all(red, blue)
    ref.reset_all(red, blue)
    _compare_state(ours, ref, "after reset_all")
    _compare_obs(ours, ref, "after reset_all")
    ended = 0
    for t in range(plies):
        if path == "apply_actions":
            acts, _ = ours.sample_actions("uniform", ply=t)
            ours.apply_actions(acts)
        else:
            acts = ours.step(None, auto_reset=False, observe=False).action
        ref.apply_actions(acts)
        _compare_state(ours, ref, f"{path} ply {t}")
        if t % 25 == 24:
            _compare_obs(ours, ref, f"{path} ply {t}")
        if t % 100 == 99:  # new games where games ended, on both
            ended += int(ref.get_terminated().sum())
            red, blue = _planes(pool, np.arange(n) + 977 * (t + 1))
            ours.reset_terminated(red, blue)
            ref.reset_terminated(red, blue)
            _compare_state(ours, ref, f"{path} reset after ply {t}")
    assert ended > 0
    assert int(ref.two_square_violation.sum()) > 0 and int(ref.chase_hash_len.max()) > 2
