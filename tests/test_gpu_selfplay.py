"""Batched self-play and search-rollout adapters on the B200, checked on the oracle.

* ``BatchedSelfPlay.generate_games`` returns complete games whose moves
  replay legally on the CPU oracle from the recorded setups, with the same
  infostate before every move (float32, bit-exact), side to move, attack
  flags and outcome;
* the kernel's sampling from network logits follows the softmax of the
  logits restricted to the legal moves (chi-square over 16,384 games in one
  position);
* ``BatchedRolloutEngine`` scores the final positions with the network's
  value head, leaves the caller's buffer alone in ``rollout_for_move`` and
  stops games that end.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


class ToyMoveNet(torch.nn.Module):
    """(value [N,3], policy [N,10000]) from a seeded 1x1 convolution."""

    def __init__(self, seed: int = 0) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.w = torch.nn.Parameter(torch.randn(2, 488, generator=g) * 0.5)
        self.v = torch.nn.Parameter(torch.randn(3, 488, generator=g) * 0.5)

    def forward(self, info, legal_move_mask=None):
        x = info.float().flatten(2)                       # [N,488,100]
        h = torch.einsum("cd,ndq->ncq", self.w, x)        # [N,2,100]
        policy = (h[:, 0, :, None] + h[:, 1, None, :]).flatten(1)
        value = torch.einsum("kd,nd->nk", self.v, x.mean(2))
        return value, policy


def _planes(setup, n_sq=100):
    p = np.zeros(n_sq, dtype=np.int8)
    for (r, c), pt in setup:
        p[r * 10 + c] = pt
    return p.reshape(1, 10, 10)


def test_generate_games_replay_on_oracle():
    from ataraxos_b200.selfplay import BatchedSelfPlay

    net = ToyMoveNet(1).cuda()
    pool = torch.from_numpy(oracle.make_setup_pool(9, 256))
    sp = BatchedSelfPlay(net, num_envs=24, seed=9, setup_pool=pool, no_attack_limit=30, max_game_length=300)
    games = sp.generate_games(30)  # two waves: 24 + 6
    assert len(games) == 30
    outcomes = set()
    for gi, g in enumerate(games):
        assert len(g.setup_red) == 40 and len(g.setup_blue) == 40
        o = oracle.OracleState(1, no_attack_limit=30, max_game_length=300)
        o.reset_planes(_planes(g.setup_red), _planes(g.setup_blue), force_all=True)
        for t, tr in enumerate(g.transitions):
            assert int(o.a["current_player"][0]) == tr.player, (gi, t)
            np.testing.assert_array_equal(tr.infostate, o.infostate_f32()[0], err_msg=f"game {gi} move {t}")
            owner = o.a["board_owner"][0].reshape(-1)
            assert tr.is_attack == (owner[tr.move_idx % 100] == 1 - tr.player)
            assert tr.action == (tr.move_idx // 100, tr.move_idx % 100)
            assert not bool(o.a["terminated"][0])
            o.apply(np.array([tr.move_idx]))
            assert int(o.a["invalid_count"][0]) == 0, (gi, t)
        assert bool(o.a["terminated"][0]), gi
        oc = int(o.a["outcome"][0])
        assert g.outcome == {0: 1, 1: -1}.get(oc, 0)
        outcomes.add(g.outcome)
    assert len(outcomes) >= 2


def test_sampling_follows_legal_softmax_of_logits():
    from ataraxos_b200.selfplay import BatchedSelfPlay

    n = 16384
    pool = oracle.make_setup_pool(4, 1)  # every game starts from the same setup
    fixed = torch.randn(1, 10000, generator=torch.Generator().manual_seed(3)).cuda() * 1.5

    def net(info, mask=None):
        return fixed.expand(info.shape[0], -1)

    sp = BatchedSelfPlay(net, num_envs=n, seed=21, setup_pool=torch.from_numpy(pool))
    sp.buf.reset_all_from_pool()
    first = sp.collect(1, store_obs=False)["action"][0].cpu().numpy()
    o = oracle.OracleState(1, seed=21, pool=pool)
    o.reset_pool(force_all=True)
    legal = o.legal_list(0)
    z = fixed[0].cpu().double().numpy()[legal]
    p = np.exp(z - z.max())
    p /= p.sum()
    counts = np.array([(first == a).sum() for a in legal], dtype=np.float64)
    assert counts.sum() == n  # every sampled move is legal
    exp = n * p
    keep = exp >= 5
    chi2 = (((counts - exp) ** 2 / exp)[keep]).sum() + ((counts[~keep].sum() - exp[~keep].sum()) ** 2
                                                         / max(exp[~keep].sum(), 1e-9) if (~keep).any() else 0.0)
    dof = int(keep.sum()) + (1 if (~keep).any() else 0) - 1
    assert chi2 < dof + 6 * np.sqrt(2 * dof), (chi2, dof)


def test_collect_shapes_and_logprobs():
    from ataraxos_b200.selfplay import BatchedSelfPlay

    net = ToyMoveNet(2).cuda()
    sp = BatchedSelfPlay(net, num_envs=64, seed=5, pool_size=512, no_attack_limit=20, obs_dtype=torch.bfloat16)
    sp.buf.reset_all_from_pool()
    r = sp.collect(40)
    assert tuple(r["obs"].shape) == (40, 64, 75, 10, 10) and r["obs"].dtype == torch.bfloat16
    assert tuple(r["action"].shape) == (40, 64)
    assert (r["action"] >= 0).all()  # auto-reset keeps every env playing
    assert (r["logprob"] <= 0).all()
    assert int(r["done"].sum()) > 0
    # players alternate within a game and restart with Red after a reset
    pl = r["player"].cpu().numpy().astype(int)
    dn = r["done"].cpu().numpy()
    for t in range(1, 40):
        np.testing.assert_array_equal(pl[t], np.where(dn[t - 1], 0, 1 - pl[t - 1]))


def test_rollout_engine_values_and_isolation():
    from ataraxos_b200 import StrategoRolloutBuffer
    from ataraxos_b200.selfplay import BatchedRolloutEngine

    net = ToyMoveNet(3).cuda()
    roots = StrategoRolloutBuffer(48, 0, seed=2, pool_size=512, no_attack_limit=200)
    roots.reset_all_from_pool()
    for _ in range(120):
        roots.step(None)
    eng = BatchedRolloutEngine(net)
    # depth 0: the value head on the roots' own infostate
    v0 = eng.rollout(roots.clone(), depth=0)
    val, _ = net(roots.compute_infostate_tensor())
    p = torch.softmax(val.float(), -1)
    torch.testing.assert_close(v0, p[:, 0] - p[:, 1])
    before = roots.export_state()
    c = roots.clone()
    moves0 = c.get_move_number().clone()
    v = eng.rollout(c, depth=40)
    assert v.shape == (48,) and bool(((v >= -1) & (v <= 1)).all())
    adv = (c.get_move_number() - moves0).cpu().numpy()
    term = c.get_terminated().cpu().numpy()
    assert ((adv == 40) | term).all() and (adv <= 40).all()
    # rollout_for_move leaves the caller's buffer unchanged
    acts, _ = roots.sample_actions()
    eng.rollout_for_move(roots, acts, depth=10)
    after = roots.export_state()
    for k in before:
        assert torch.equal(before[k], after[k]), k
