"""The oracle's threaded runners, which the full-size GPU parity tests use.

``OracleState.run`` (plies of ``step`` on host threads) and
``OracleState.observe`` (masks and infostate on host threads) must give
exactly what the single-threaded calls give, for any thread count, and a
subsample replayed with its global env indices (``genv``) must follow the
same games as the full batch.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle


def _pair(n, seed, pool, **kw):
    a = oracle.OracleState(n, seed=seed, pool=pool, **kw)
    b = oracle.OracleState(n, seed=seed, pool=pool, **kw)
    a.reset_pool(force_all=True)
    b.reset_pool(force_all=True)
    return a, b


@pytest.mark.parametrize("policy", [oracle.POLICY_UNIFORM, oracle.POLICY_GUMBEL])
def test_threaded_run_equals_sequential_steps(policy):
    pool = oracle.make_setup_pool(5, 300)
    a, b = _pair(97, 5, pool, no_attack_limit=30, max_game_length=120)
    hist = a.run(160, policy=policy, threads=7)
    for t in range(160):
        r = b.step(None, policy=policy)
        for k, v in r.items():
            np.testing.assert_array_equal(v, hist[k][t], err_msg=f"{k} at ply {t}")
    for k in a.a:
        np.testing.assert_array_equal(a.a[k], b.a[k], err_msg=k)
    assert hist["done"].sum() > 0


def test_threaded_observe_equals_single_thread():
    pool = oracle.make_setup_pool(6, 100)
    a, b = _pair(41, 6, pool)
    a.run(30, threads=3, record=False)
    b.run(30, threads=1, record=False)
    obs = a.observe(mask_u8=True, mask_bits=True, info="dense", threads=5)
    np.testing.assert_array_equal(obs["mask_u8"], b.legal_mask_u8())
    np.testing.assert_array_equal(obs["mask_bits"], b.legal_mask_bits())
    np.testing.assert_array_equal(obs["info"], b.infostate_bf16_bits())
    compact = a.observe(info="compact", threads=2)["info"]
    np.testing.assert_array_equal(compact[:, :44], obs["info"][:, :44])
    np.testing.assert_array_equal(compact[:, 44:], obs["info"][:, 456:])


def test_subsample_by_global_index_follows_the_full_batch():
    pool = oracle.make_setup_pool(8, 400)
    full = oracle.OracleState(300, seed=8, pool=pool, env_base=1000, no_attack_limit=40)
    full.reset_pool(force_all=True)
    sub_idx = np.arange(5, 300, 11)
    sub = oracle.OracleState(len(sub_idx), seed=8, pool=pool, genv=1000 + sub_idx, no_attack_limit=40)
    sub.reset_pool(force_all=True)
    hf = full.run(120, policy=oracle.POLICY_GUMBEL, threads=6)
    hs = sub.run(120, policy=oracle.POLICY_GUMBEL, threads=4)
    for k in hs:
        np.testing.assert_array_equal(hs[k], hf[k][:, sub_idx], err_msg=k)
    for k in sub.a:
        np.testing.assert_array_equal(sub.a[k], full.a[k][sub_idx], err_msg=k)
