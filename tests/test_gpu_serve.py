"""The persistent step server (``StrategoRolloutBuffer.serve``) on the B200.

* served plies equal ``step()`` plies on a twin buffer: per-step reward,
  done and next action in page-locked host memory, the device infostate and
  u8 mask, and the final state;
* device proposals (``host_actions=False``) equal ``step(None)``;
* a server that gets no step within its limit gives up on its own, raises
  SB_STATUS_WAIT_TIMEOUT and leaves a usable buffer (the wait that runs out
  is the host's next step, which the test never publishes);
* more envs than can be resident at once is refused before any launch.
"""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle
from _helpers import assert_state_equal, export_np

pytestmark = pytest.mark.gpu


def _twins(n, seed, **kw):
    from ataraxos_b200 import StrategoRolloutBuffer

    pool = torch.from_numpy(oracle.make_setup_pool(seed, 512))
    a = StrategoRolloutBuffer(n, 0, seed=seed, setup_pool=pool, **kw)
    b = StrategoRolloutBuffer(n, 0, seed=seed, setup_pool=pool, **kw)
    a.reset_all_from_pool()
    b.reset_all_from_pool()
    return a, b


@pytest.mark.parametrize("n,dtype", [(1000, torch.bfloat16), (4096, torch.bfloat16), (77, torch.float32)])
def test_served_plies_equal_step(n, dtype):
    a, b = _twins(n, 5, no_attack_limit=40, obs_dtype=dtype)
    first = a.step_host(None)
    b.step(None)
    acts = first.next_action.to(torch.int64)
    fed, got = [], []
    # the server keeps every CTA resident: the twin replays afterwards
    with a.serve() as srv:
        for t in range(60):
            if t % 7 == 3:
                acts[::5] = 0  # illegal for those games: ignored and counted
            fed.append(acts.clone())
            r = srv.step(acts)
            got.append((r.reward.clone(), r.done.clone(), r.next_action.clone()))
            acts = r.next_action.to(torch.int64)
    for t, (acts, (rew, done, nxt)) in enumerate(zip(fed, got)):
        ref = b.step(acts.to("cuda"))
        np.testing.assert_array_equal(rew.numpy(), ref.reward.cpu().numpy(), err_msg=f"step {t}")
        np.testing.assert_array_equal(done.numpy(), ref.done.cpu().numpy(), err_msg=f"step {t}")
        np.testing.assert_array_equal(nxt.numpy(), ref.next_action.cpu().numpy(), err_msg=f"step {t}")
    da, db = a._ensure_outputs(), b._ensure_outputs()
    assert torch.equal(da["infostate"], db["infostate"]) and torch.equal(da["mask"], db["mask"])
    assert a.ply == b.ply
    assert_state_equal(export_np(a), export_np(b), "served vs stepped")
    assert a.status() == 0


def test_served_device_proposals_equal_step_none():
    a, b = _twins(512, 9, no_attack_limit=30)
    got = []
    with a.serve(host_actions=False) as srv:
        for t in range(50):
            r = srv.step(None)
            got.append((r.next_action.clone(), r.done.clone()))
    for t, (nxt, done) in enumerate(got):
        ref = b.step(None)
        np.testing.assert_array_equal(nxt.numpy(), ref.next_action.cpu().numpy(), err_msg=f"step {t}")
        np.testing.assert_array_equal(done.numpy(), ref.done.cpu().numpy())
    assert_state_equal(export_np(a), export_np(b), "served proposals")


def test_server_gives_up_without_steps():
    import ataraxos_b200._capi as C

    a, b = _twins(256, 13)
    srv = a.serve(host_actions=False, limit_s=0.2)
    srv.start()
    srv.step(None)
    time.sleep(0.6)  # no second step: every CTA's bounded wait runs out
    srv.close()
    b.step(None)
    assert a.status() & C.SB_STATUS_WAIT_TIMEOUT
    assert_state_equal(export_np(a), export_np(b), "after a timed-out server")
    a.step(None)  # the buffer is usable afterwards
    b.step(None)
    assert_state_equal(export_np(a), export_np(b), "stepping after the server")


def test_server_refuses_more_envs_than_resident():
    from ataraxos_b200 import StrategoRolloutBuffer

    big = StrategoRolloutBuffer(60000, 0, seed=1, pool_size=64)
    big.reset_all_from_pool()
    with pytest.raises(RuntimeError, match="resident"):
        big.serve().start()
