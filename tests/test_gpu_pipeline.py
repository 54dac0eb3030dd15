"""``StepPipeline`` on the B200: games split into asynchronously stepped
groups play exactly as one buffer of all the games.

* a host loop that receives, acts on and re-sends each group in turn gives,
  per ply and per game, the reward / done / next action and the final state
  of ``step_host`` on one buffer (random streams are keyed by the global env
  index, so the split is invisible), for 1, 2, 3 and 5 groups and ragged
  group sizes, with uniform and Gumbel-max (virtual logits) sampling;
* host actions (some illegal: ignored and counted) and device proposals mix;
* misuse (a second send before recv, recv with nothing in flight, actions of
  the wrong shape, more groups than games) is refused;
* the grouped forms bench.py times for configs 4 and 5 (trajectory rings and
  belief rollouts split into groups on their own streams) equal one batch of
  all the games.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _helpers import assert_state_equal, export_np

pytestmark = pytest.mark.gpu


def _pool(seed):
    return torch.from_numpy(oracle.make_setup_pool(seed, 512))


@pytest.mark.parametrize("n,groups,policy", [(1000, 1, "uniform"), (1000, 2, "uniform"), (1001, 3, "uniform"),
                                             (4096, 5, "uniform"), (1001, 3, "gumbel")])
def test_groups_equal_one_buffer(n, groups, policy):
    from ataraxos_b200 import StrategoRolloutBuffer
    from ataraxos_b200.pipeline import StepPipeline

    seed, pool = 7, _pool(7)
    one = StrategoRolloutBuffer(n, 0, seed=seed, setup_pool=pool, no_attack_limit=40)
    one.reset_all_from_pool()
    p = StepPipeline(n, 0, groups=groups, seed=seed, setup_pool=pool, no_attack_limit=40)
    p.reset_all_from_pool()
    assert sum(m for _, m in p.ranges) == n
    ref = one.step_host(None, policy=policy)
    acts = ref.next_action.to(torch.int64)
    for g in range(groups):
        p.send(g, None, policy=policy)
    for t in range(50):
        for g, (off, m) in enumerate(p.ranges):
            r = p.recv(g)
            sl = slice(off, off + m)
            np.testing.assert_array_equal(r.reward.numpy(), ref.reward.numpy()[sl], err_msg=f"ply {t} group {g}")
            np.testing.assert_array_equal(r.done.numpy(), ref.done.numpy()[sl], err_msg=f"ply {t} group {g}")
            np.testing.assert_array_equal(r.next_action.numpy(), ref.next_action.numpy()[sl],
                                          err_msg=f"ply {t} group {g}")
            nxt = acts[sl].clone()
            if t % 9 == 4:
                nxt[::6] = 0  # illegal for those games: ignored and counted
            p.send(g, None if t % 11 == 10 else nxt, policy=policy)
        x = torch.cat([p.actions[g] for g in range(groups)])
        if t % 11 == 10:
            ref = one.step_host(None, policy=policy)
        else:
            ref = one.step_host(x.contiguous(), policy=policy)
        acts = ref.next_action.to(torch.int64)
    for g in range(groups):
        p.recv(g)
    p.synchronize()
    whole = export_np(one)
    for g, (off, m) in enumerate(p.ranges):
        part = export_np(p.buffers[g])
        assert_state_equal(part, {k: v[off:off + m] for k, v in whole.items()}, f"group {g}")
        assert p.buffers[g].status() == 0


def test_pipeline_refuses_misuse():
    from ataraxos_b200.pipeline import StepPipeline

    with pytest.raises(RuntimeError):
        StepPipeline(2, 0, groups=3, seed=1, setup_pool=_pool(1))
    p = StepPipeline(64, 0, groups=2, seed=1, setup_pool=_pool(1))
    p.reset_all_from_pool()
    with pytest.raises(RuntimeError):
        p.recv(0)
    p.send(0, None)
    with pytest.raises(RuntimeError):
        p.send(0, None)
    with pytest.raises(RuntimeError):
        p.send(1, torch.zeros(5, dtype=torch.int64))  # group 1 holds 32 games
    p.recv(0)
    p.synchronize()


def test_grouped_trajectory_rings_equal_one_ring():
    """Config 4 as bench.py steps it: the games as 2 buffers over contiguous
    global env ranges, each with its own trajectory ring and stream, fill
    exactly the slots one ring of all the games fills (Gumbel proposals,
    compact bf16 infostate, bit-packed masks), across a ring wrap."""
    from ataraxos_b200 import StrategoRolloutBuffer, sharding
    from ataraxos_b200.trajectory import TrajectoryBuffer

    n, T, R, launches, seed = 3001, 11, 4, 4, 41
    pool = _pool(seed)
    one_buf = StrategoRolloutBuffer(n, 0, seed=seed, setup_pool=pool)
    one_buf.reset_all_from_pool()
    one = TrajectoryBuffer(one_buf, T, policy="gumbel")
    one.prime()
    parts = []
    for g in range(2):
        off, m = sharding.shard_range(n, 2, g)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            b = StrategoRolloutBuffer(m, 0, seed=seed, env_base=off, setup_pool=pool)
            b.reset_all_from_pool()
            tr = TrajectoryBuffer(b, T, policy="gumbel")
            tr.prime()
        parts.append((tr, s, off, m))
    for _ in range(launches):
        one.rollout(R)
        for tr, s, _, _ in parts:
            with torch.cuda.stream(s):
                tr.rollout(R)
    torch.cuda.synchronize()
    for tr, _, off, m in parts:
        for name in ("obs", "mask", "action", "logprob", "reward", "done"):
            assert torch.equal(getattr(tr, name), getattr(one, name)[:, off:off + m]), name
        assert tr.slot == one.slot
    assert int(sum(tr.stats[0] for tr, _, _, _ in parts)) == int(one.stats[0])


def test_grouped_belief_rollouts_equal_one_batch():
    """Config 5 as bench.py steps it: the roots as 2 groups (their own root
    buffers and sample buffers over contiguous global ranges, own streams)
    resample and roll exactly the samples of one batch over all roots."""
    from ataraxos_b200 import StrategoRolloutBuffer, sharding
    from ataraxos_b200.trajectory import BeliefRollouts

    n_roots, k, depth, seed = 6, 50, 12, 43
    pool = _pool(seed)
    roots = StrategoRolloutBuffer(n_roots, 0, seed=seed, setup_pool=pool)
    roots.reset_all_from_pool()
    for _ in range(30):
        roots.step(None)
    one = BeliefRollouts(roots, k, depth, seed=seed + 1).run()
    got = []
    for g in range(2):
        off, nr = sharding.shard_range(n_roots, 2, g)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            r = StrategoRolloutBuffer(nr, 0, seed=seed, env_base=off, setup_pool=pool)
            r.reset_all_from_pool()
            for _ in range(30):
                r.step(None)
            br = BeliefRollouts(r, k, depth, seed=seed + 1)
            br.samples.env_base = off * k
            br.samples._st = br.samples._make_state()
            got.append((br.run(), off * k, nr * k))
    torch.cuda.synchronize()
    for out, a, m in got:
        for name in ("masks", "actions"):
            assert torch.equal(out[name], one[name][:, a:a + m]), name
        assert torch.equal(out["terminal_value"], one["terminal_value"][a:a + m])
        assert torch.equal(out["done"], one["done"][a:a + m])
