"""Batched search-rollouts on the B200, replayed on the oracle.

``BatchedRolloutEngine.rollout`` (rollouts.py:46-104) and
``BatchedSearch.search`` (mirror_descent.py:115-154) run on the GPU with a
small deterministic move network; every rollout's actions are recorded and
replayed on the CPU oracle from the same copies (plain, or re-dealt by the
same belief resampling), and the oracle's final float32 infostates, scored
by the same network, must give the same values bit for bit; ``q`` must be
their mean per (root, move), and the policy the closed form over them.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _helpers import assert_state_equal, export_np

pytestmark = pytest.mark.gpu


class TinyNet:
    """(value_logits [N,3], policy_logits [N,10000]) as a fixed function of the
    infostate, computed in float64 on the host so that the same input always
    gives the same bits whatever the batch."""

    def __init__(self, seed=5):
        g = torch.Generator().manual_seed(seed)
        self.table = torch.randn(10000, generator=g, dtype=torch.float64)

    def __call__(self, info):
        x = info.detach().double().cpu().reshape(info.shape[0], 488, 100)
        own = x[:, :12].sum(1)                                            # own pieces per square
        pol = self.table[None, :] + 0.7 * own.repeat_interleave(100, dim=1)
        v = torch.stack([0.02 * x[:, :43].sum((1, 2)), 0.05 * x[:, 36].sum(1), 0.05 * x[:, 37].sum(1)], 1)
        return v.float().to(info.device), pol.float().to(info.device)


def _value(net, info_f32: torch.Tensor) -> torch.Tensor:
    v, _ = net(info_f32)
    p = torch.softmax(v.float(), dim=-1)
    return p[:, 0] - p[:, 1]


def _roots(n, plies, seed):
    from ataraxos_b200 import StrategoRolloutBuffer

    pool = oracle.make_setup_pool(seed, 256)
    b = StrategoRolloutBuffer(n, 0, seed=seed, setup_pool=torch.from_numpy(pool), obs_dtype=torch.float32)
    o = oracle.OracleState(n, seed=seed, pool=pool)
    b.reset_all_from_pool()
    o.reset_pool(force_all=True)
    for _ in range(plies):
        b.step(None)
    o.run(plies, threads=4, record=False)
    assert_state_equal(export_np(b), o.export(), "roots")
    return b, o


def _replay(net, o: oracle.OracleState, trace, dev) -> torch.Tensor:
    for acts in trace:
        o.step(acts.cpu().numpy(), auto_reset=False)
    return _value(net, torch.from_numpy(o.infostate_f32()).to(dev))


def test_rollout_engine_replays_on_oracle():
    from ataraxos_b200.selfplay import BatchedRolloutEngine

    net = TinyNet()
    roots, oroots = _roots(48, 20, 21)
    states = roots.clone()
    trace: list[torch.Tensor] = []
    vals = BatchedRolloutEngine(net).rollout(states, depth=12, trace=trace)
    assert len(trace) == 12
    ref = _replay(net, oroots, trace, roots.device)
    assert torch.equal(vals, ref)
    assert_state_equal(export_np(states), oroots.export(), "after the rollouts")


@pytest.mark.parametrize("resample", [False, True])
def test_batched_search_values_q_and_policy(resample):
    from ataraxos_b200.search import BatchedSearch, compute_search_policy

    net = TinyNet()
    roots, oroots = _roots(3, 30, 7)
    s = BatchedSearch(net, n_rollouts=90, depth=8, resample=resample, seed=11)
    trace: list[torch.Tensor] = []
    res = s.search(roots, player=roots.get_current_player(), trace=trace)
    root_of = res.root_of.cpu().numpy()
    first = res.legal.cpu().numpy()
    S = len(root_of)
    # the rollouts: every legal move of every root, n_configs times
    mask = roots.compute_legal_action_mask().reshape(3, -1).cpu().numpy()
    for r in range(3):
        legal = np.nonzero(mask[r])[0]
        k = int(res.n_configs[r])
        assert k == max(1, 90 // len(legal))
        np.testing.assert_array_equal(first[root_of == r], np.repeat(legal, k))
    # replay every rollout on the oracle from the same starting copies
    o = oracle.OracleState(S, seed=s.seed)
    if resample:
        o.resample_from(oroots, root_of)
    else:
        for key, arr in o.a.items():
            arr[...] = oroots.a[key][root_of]
    o.apply(first)
    ref = _replay(net, o, trace, roots.device)
    assert torch.equal(res.values, ref)
    # q: the mean value per (root, move); the policy: the closed form over it
    q = torch.zeros((3, 10000), dtype=torch.float64, device=roots.device)
    q.index_put_((res.root_of, res.legal), ref.double(), accumulate=True)
    q /= res.n_configs.double().unsqueeze(-1)
    flat = torch.from_numpy(mask).to(roots.device)
    torch.testing.assert_close(res.q, q * flat, rtol=1e-12, atol=1e-12)
    pi = compute_search_policy(q, res.net_probs, res.magnet, s.alpha, s.beta, legal=flat)
    torch.testing.assert_close(res.policy, pi, rtol=1e-12, atol=1e-12)
    assert torch.allclose(res.policy.sum(-1), torch.ones(3, dtype=torch.float64, device=roots.device))
    a = res.action.cpu().numpy()
    assert all(mask[r, a[r]] for r in range(3))
