"""sb_step_host_noalloc on the B200, called through the C ABI.

The entry point stages the host actions in the library's own device array
instead of a caller-allocated buffer.  Two calls in a row (and a few more
plies after them) must give exactly what sb_step_host gives with a staging
buffer of the caller's on a twin buffer; oversized shards and a caller
staging buffer are refused before any launch.  The file name sorts last so
that the suite also runs it after every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from _helpers import assert_state_equal, export_np

pytestmark = pytest.mark.gpu


def _twins(n, seed, **kw):
    from ataraxos_b200 import StrategoRolloutBuffer

    pool = torch.from_numpy(oracle.make_setup_pool(seed, 512))
    a = StrategoRolloutBuffer(n, 0, seed=seed, setup_pool=pool, no_attack_limit=30, **kw)
    b = StrategoRolloutBuffer(n, 0, seed=seed, setup_pool=pool, no_attack_limit=30, **kw)
    a.reset_all_from_pool()
    b.reset_all_from_pool()
    return a, b


def _noalloc_step(buf, actions, observe=True):
    """One ply of ``buf`` through sb_step_host_noalloc: ``actions`` is a CPU
    int64 array (pageable or page-locked) or None; reward / done /
    next_action come back into the buffer's page-locked result block."""
    import ataraxos_b200._capi as C

    h = buf._host_io()
    cp = h["io"]["copy"]
    io = C.SbHostIo(actions_host=None if actions is None else actions.data_ptr(), actions_dev=None,
                    back_dev=cp.back_dev, back_host=cp.back_host, back_bytes=cp.back_bytes, sync=1, reserved=0)
    pol = C.SbPolicy(kind=C.SB_POLICY_UNIFORM, reserved=0, logits=None)
    rc = C.lib().sb_step_host_noalloc(ctypes.byref(buf._st), ctypes.byref(io), buf.ply, ctypes.byref(pol), 1,
                                      h["out"]["copy"][observe], torch.cuda.current_stream().cuda_stream)
    assert rc == 0, C.lib().sb_last_error()
    buf._ply += 1
    return h["ret"]["copy"][observe]


def _same(r, ref, t):
    np.testing.assert_array_equal(r.reward.numpy(), ref.reward.numpy(), err_msg=f"ply {t}")
    np.testing.assert_array_equal(r.done.numpy(), ref.done.numpy(), err_msg=f"ply {t}")
    np.testing.assert_array_equal(r.next_action.numpy(), ref.next_action.numpy(), err_msg=f"ply {t}")
    assert torch.equal(r.device.infostate, ref.device.infostate), f"ply {t}"
    assert torch.equal(r.device.legal_mask, ref.device.legal_mask), f"ply {t}"


def test_noalloc_equals_step_host_two_calls_in_a_row():
    n = 1000
    a, b = _twins(n, 23)
    ref = b.step_host(None, mapped=False)
    r = _noalloc_step(a, None)
    _same(r, ref, "first")
    acts = r.next_action.to(torch.int64)
    acts[::9] = 0  # illegal for those games: ignored and counted
    # two host-action calls in a row: page-locked, then pageable actions
    for t, pin in enumerate((True, False)):
        x = acts.pin_memory() if pin else acts.clone()
        r_ref = b.step_host(x, mapped=False)
        r = _noalloc_step(a, x)
        _same(r, r_ref, t)
        acts = r.next_action.to(torch.int64)
    for t in range(40):  # more plies, including device sampling, on the same staging array
        x = None if t % 4 == 3 else acts
        r_ref = b.step_host(x, mapped=False)
        r = _noalloc_step(a, x)
        _same(r, r_ref, t + 2)
        acts = r.next_action.to(torch.int64)
    assert a.ply == b.ply
    assert_state_equal(export_np(a), export_np(b), "noalloc vs step_host")
    assert a.status() == 0


def test_noalloc_refuses_before_launch():
    import ataraxos_b200._capi as C

    a, b = _twins(64, 29)
    h = a._host_io()
    acts = torch.zeros(64, dtype=torch.int64)
    pol = C.SbPolicy(kind=C.SB_POLICY_UNIFORM, reserved=0, logits=None)
    stream = torch.cuda.current_stream().cuda_stream
    fn = C.lib().sb_step_host_noalloc
    # a caller staging buffer is not taken
    io = C.SbHostIo(actions_host=acts.data_ptr(), actions_dev=h["io"]["copy"].actions_dev, back_dev=None,
                    back_host=None, back_bytes=0, sync=1, reserved=0)
    assert fn(ctypes.byref(a._st), ctypes.byref(io), 0, ctypes.byref(pol), 1, h["out"]["copy"][True], stream) \
        == C.SB_E_ARG
    # more envs than the staging array holds: refused by size alone, nothing is read
    big = C.SbState.from_buffer_copy(a._st)
    big.n = C.SB_NOALLOC_MAX_ENVS + 1
    io.actions_dev = None
    assert fn(ctypes.byref(big), ctypes.byref(io), 0, ctypes.byref(pol), 1, h["out"]["copy"][True], stream) \
        == C.SB_E_ARG
    assert b"at most" in C.lib().sb_last_error()
    torch.cuda.synchronize()
    # neither refusal touched the game
    assert_state_equal(export_np(a), export_np(b), "after refusals")
    ra, rb = _noalloc_step(a, None), b.step_host(None, mapped=False)
    _same(ra, rb, "after refusals")


def test_noalloc_full_staging_array():
    """A shard of exactly SB_NOALLOC_MAX_ENVS games fills the staging array:
    accepted, and equal to sb_step_host on a twin buffer."""
    import ataraxos_b200._capi as C

    n = C.SB_NOALLOC_MAX_ENVS
    a, b = _twins(n, 31, obs_layout="compact", mask_format="none")
    acts = b.step_host(None, mapped=False, observe=False).next_action.to(torch.int64)
    _noalloc_step(a, None, observe=False)
    acts[::7] = 0  # illegal for those games: ignored and counted
    for t in range(3):
        r_ref = b.step_host(acts, mapped=False, observe=False)
        r = _noalloc_step(a, acts, observe=False)
        np.testing.assert_array_equal(r.reward.numpy(), r_ref.reward.numpy(), err_msg=f"ply {t}")
        np.testing.assert_array_equal(r.done.numpy(), r_ref.done.numpy(), err_msg=f"ply {t}")
        np.testing.assert_array_equal(r.next_action.numpy(), r_ref.next_action.numpy(), err_msg=f"ply {t}")
        acts = r.next_action.to(torch.int64)
    assert torch.equal(a._records, b._records)
    assert a.status() == 0
