"""Parity of the B200 kernels (through libstratego_b200.so) with the reference.

* golden traces of the reference's Python engine (tests/golden/*.npz),
  replayed through the fused step kernel and through the reference-facing API;
* the CPU oracle on larger seeded random workloads: full state, Zobrist hash,
  masks (u8 and bit-packed), infostate (float32 and bfloat16, dense and
  compact), bit-exact;
* softmax (Gumbel-max) sampling: the oracle's choices and bit-identical
  log-probs;
* shard invariance (env_base), checkpoint round trip, episode statistics.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from _helpers import assert_state_equal, board_code, digest, export_np

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name):
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


def _buf(n, **kw):
    from ataraxos_b200 import StrategoRolloutBuffer

    return StrategoRolloutBuffer(n, 0, **kw)


def _gpu_snapshot(buf, mask_u8: np.ndarray, info: np.ndarray) -> dict[str, np.ndarray]:
    st = export_np(buf)
    n = st["board_owner"].shape[0]
    bits = np.packbits(mask_u8.reshape(n, -1).astype(np.uint8), axis=1, bitorder="little")
    return {
        "board": board_code(st["board_owner"], st["board_piece"]),
        "moved": np.packbits(st["moved_squares"], axis=1, bitorder="little"),
        "revealed": np.packbits(st["revealed_squares"], axis=1, bitorder="little"),
        "current_player": st["current_player"].astype(np.int8),
        "outcome": st["outcome"].astype(np.int8),
        "flag_captured": st["flag_captured"].astype(np.int8),
        "move_number": st["move_number"],
        "moves_since_attack": st["moves_since_attack"],
        "terminated_since": st["terminated_since"],
        "hist_head": st["move_history_head"],
        "hist_len": st["move_history_len"],
        "hist_digest": np.array([digest(st["move_history"][g].astype(np.int32)) for g in range(n)]),
        "ts_count": st["two_square_count"],
        "ts_lo": st["two_square_pair_lo"],
        "ts_hi": st["two_square_pair_hi"],
        "ts_violation": st["two_square_violation"].astype(np.int8),
        "chase_head": st["chase_hash_head"],
        "chase_len": st["chase_hash_len"],
        "chase_last_src": st["chase_last_src"],
        "chase_digest": np.array([digest(st["chase_hashes"][g]) for g in range(n)]),
        "chase_violation": st["chasing_violation"].astype(np.int8),
        "hash": buf.hash_board().cpu().numpy(),
        "n_legal": mask_u8.reshape(n, -1).sum(1).astype(np.int32),
        "mask_digest": np.array([digest(bits[g]) for g in range(n)]),
        "info_digest": np.array([digest(info[g]) for g in range(n)]),
        "episode": st["episode"],
    }


def _compare(snap, g, t, name):
    for k, v in snap.items():
        np.testing.assert_array_equal(v, g[k][t], err_msg=f"{name}: field {k} at snapshot {t}")


@pytest.mark.parametrize("name", ["config1", "autoreset"])
def test_fused_step_replays_reference_trace(name):
    """Device-sampled uniform actions, the fused step kernel, float32 dense outputs."""
    g = _load(name)
    n, plies, seed, pool_size, auto_reset, nal = (int(x) for x in g["meta"])
    buf = _buf(n, seed=seed, setup_pool=torch.from_numpy(g["pool"]), no_attack_limit=nal,
               max_game_length=int(g["max_game_length"]), obs_dtype=torch.float32)
    buf.reset_all_from_pool()
    snap = _gpu_snapshot(buf, buf.compute_legal_action_mask().cpu().numpy(),
                         buf.compute_infostate_tensor().cpu().numpy())
    _compare(snap, g, 0, name)
    fp = list(g["full_plies"])
    for t in range(1, plies + 1):
        out = buf.step(None, auto_reset=bool(auto_reset))
        np.testing.assert_array_equal(out.action.cpu().numpy(), g["actions"][t - 1])
        np.testing.assert_array_equal(out.reward.cpu().numpy(), g["reward"][t - 1])
        np.testing.assert_array_equal(out.done.cpu().numpy().astype(np.uint8), g["done"][t - 1])
        info = out.infostate.cpu().numpy()
        snap = _gpu_snapshot(buf, out.legal_mask.cpu().numpy(), info)
        _compare(snap, g, t, name)
        if t in fp:
            ne = g["full_info"].shape[1]
            np.testing.assert_array_equal(info[:ne], g["full_info"][fp.index(t)])


def test_reference_api_replays_reference_trace():
    """reset_all(planes) + apply_actions + compute_* (the reference's own API)."""
    g = _load("config1")
    n, plies, seed, pool_size, _, nal = (int(x) for x in g["meta"])
    o = oracle.OracleState(n, seed=seed, pool=g["pool"])
    o.reset_pool(force_all=True)
    ow, pc = o.a["board_owner"], o.a["board_piece"]
    red = torch.from_numpy(np.where(ow == 0, pc, 0).astype(np.int8))
    blue = torch.from_numpy(np.where(ow == 1, pc, 0).astype(np.int8))
    buf = _buf(n)
    buf.reset_all(red, blue)
    for t in range(plies + 1):
        if t > 0:
            buf.apply_actions(torch.from_numpy(g["actions"][t - 1]))
        if t % 10 and t != plies:
            continue
        mask = buf.compute_legal_action_mask()
        assert mask.dtype == torch.bool and tuple(mask.shape) == (n, 100, 100)
        info = buf.compute_infostate_tensor()
        assert info.dtype == torch.float32 and tuple(info.shape) == (n, 488, 10, 10)
        snap = _gpu_snapshot(buf, mask.cpu().numpy(), info.cpu().numpy())
        snap.pop("episode")
        _compare(snap, g, t, "config1/api")
        np.testing.assert_array_equal(buf.compute_reward_pl0().cpu().numpy(),
                                      np.where(g["outcome"][t] == 0, 1.0, np.where(g["outcome"][t] == 1, -1.0, 0.0)))


def _paired(n, seed, pool, **kw):
    b = _buf(n, seed=seed, setup_pool=torch.from_numpy(pool), **kw)
    o = oracle.OracleState(n, seed=seed, pool=pool, **{k: v for k, v in kw.items() if k in (
        "no_attack_limit", "max_game_length", "two_square_limit", "env_base")})
    b.reset_all_from_pool()
    o.reset_pool(force_all=True)
    return b, o


@pytest.mark.parametrize("n,plies,nal,maxlen", [(1000, 400, 100, 4000), (333, 600, 12, 90), (1, 50, 100, 4000)])
def test_random_rollout_matches_oracle(n, plies, nal, maxlen):
    rng = np.random.default_rng(n)
    seed = int(rng.integers(1, 2**62))
    pool = oracle.make_setup_pool(seed ^ 0x5A5A, 4096)
    b, o = _paired(n, seed, pool, no_attack_limit=nal, max_game_length=maxlen, obs_dtype=torch.bfloat16)
    for t in range(1, plies + 1):
        out = b.step(None)
        r = o.step(None)
        np.testing.assert_array_equal(out.action.cpu().numpy(), r["action"], err_msg=f"ply {t}")
        np.testing.assert_array_equal(out.reward.cpu().numpy(), r["reward"])
        np.testing.assert_array_equal(out.done.cpu().numpy().astype(np.uint8), r["done"])
        if t % 50 == 0 or t == plies:
            assert_state_equal(export_np(b), o.export(), f"ply {t}")
            np.testing.assert_array_equal(b.hash_board().cpu().numpy(), o.hash_board())
            np.testing.assert_array_equal(out.legal_mask.cpu().numpy().view(np.uint8), o.legal_mask_u8())
            bits = out.infostate.view(torch.int16).cpu().numpy().view(np.uint16)
            np.testing.assert_array_equal(bits, o.infostate_bf16_bits())
            np.testing.assert_array_equal(b.compute_legal_action_mask_bits().cpu().numpy(), o.legal_mask_bits())
            np.testing.assert_array_equal(b.compute_infostate_tensor().cpu().numpy(), o.infostate_f32())
            np.testing.assert_array_equal(b.get_has_legal_movement().cpu().numpy(),
                                          o.legal_mask_u8().reshape(n, -1).any(1))
    assert int(b.episode_stats()[0]) > 0 or plies < 100


def test_layouts_and_bit_packed_masks_agree():
    n = 200
    pool = oracle.make_setup_pool(11, 512)
    dense = _buf(n, seed=5, setup_pool=torch.from_numpy(pool), obs_dtype=torch.bfloat16, mask_format="u8")
    comp = _buf(n, seed=5, setup_pool=torch.from_numpy(pool), obs_dtype=torch.bfloat16, obs_layout="compact",
                mask_format="bits")
    f32c = _buf(n, seed=5, setup_pool=torch.from_numpy(pool), obs_dtype=torch.float32, obs_layout="compact",
                mask_format="none")
    for b in (dense, comp, f32c):
        b.reset_all_from_pool()
    for _ in range(120):
        d, c, f = dense.step(None), comp.step(None), f32c.step(None)
    di, ci, fi = d.infostate, c.infostate, f.infostate
    assert tuple(ci.shape) == (n, 76, 10, 10)
    assert torch.equal(ci[:, :43], di[:, :43]) and torch.equal(ci[:, 44:], di[:, 456:])
    assert not ci[:, 43].any() and not di[:, 43:456].any()
    assert torch.equal(fi[:, :43].to(torch.bfloat16), di[:, :43])
    packed = np.packbits(d.legal_mask.cpu().numpy().reshape(n, -1).astype(np.uint8), axis=1, bitorder="little")
    np.testing.assert_array_equal(c.legal_mask.cpu().numpy(), packed)
    full = dense.compute_infostate_tensor(torch.float32)
    assert torch.equal(full[:, :43].to(torch.bfloat16), di[:, :43])
    assert torch.equal(full[:, 456:].to(torch.bfloat16), di[:, 456:])


def test_gumbel_sampling_matches_oracle():
    n, plies = 256, 120
    pool = oracle.make_setup_pool(3, 1024)
    b, o = _paired(n, 99, pool)
    for t in range(plies):
        acts, lp = b.sample_actions("gumbel")
        oa, olp, _ = o.sample(ply=b.ply, policy=oracle.POLICY_GUMBEL)
        acts, lp = acts.cpu().numpy(), lp.cpu().numpy()
        # the noise's float functions are reproduced bit for bit: same
        # choices and bit-identical log-probs
        np.testing.assert_array_equal(acts, oa, err_msg=f"ply {t}")
        np.testing.assert_array_equal(lp.view(np.uint32), olp.astype(np.float32).view(np.uint32), err_msg=f"ply {t}")
        # legal: replaying the GPU's choices on the oracle is never rejected
        before = o.a["invalid_count"].copy()
        out = b.step(torch.from_numpy(acts), auto_reset=True)
        o.step(acts, auto_reset=True)
        np.testing.assert_array_equal(o.a["invalid_count"], before)
        np.testing.assert_array_equal(out.action.cpu().numpy(), acts)
    assert_state_equal(export_np(b), o.export(), "after gumbel replay")


def test_sampling_with_many_legal_moves_matches_oracle():
    """Custom setups of 28 Scouts give 130-165 legal moves (five or more per
    lane): uniform and Gumbel choices and log-probs stay bit-identical to the
    oracle over a few plies."""
    rng = np.random.default_rng(5)
    n = 6
    red = np.zeros((n, 10, 10), np.int8)
    blue = np.zeros((n, 10, 10), np.int8)
    lakes = {(4, 2), (4, 3), (5, 2), (5, 3), (4, 6), (4, 7), (5, 6), (5, 7)}
    for g in range(n):
        sqs = [(r, c) for r in range(10) for c in range(10) if (r, c) not in lakes]
        rng.shuffle(sqs)
        for r, c in sqs[:28]:
            red[g, r, c] = 2  # Scout
        blue[g, sqs[28][0], sqs[28][1]] = 11  # Flag
        for r, c in sqs[29:31]:
            blue[g, r, c] = 10  # Marshal
    for policy, opol in (("uniform", oracle.POLICY_UNIFORM), ("gumbel", oracle.POLICY_GUMBEL)):
        b = _buf(n, seed=41)
        o = oracle.OracleState(n, seed=41)
        b.reset_all(torch.from_numpy(red), torch.from_numpy(blue))
        o.reset_planes(red, blue, force_all=True)
        assert min(len(o.legal_list(g)) for g in range(n)) > 128
        for t in range(6):
            acts, lp = b.sample_actions(policy)
            oa, olp, _ = o.sample(ply=b.ply, policy=opol)
            np.testing.assert_array_equal(acts.cpu().numpy(), oa, err_msg=f"{policy} ply {t}")
            np.testing.assert_array_equal(lp.cpu().numpy().view(np.uint32), olp.view(np.uint32),
                                          err_msg=f"{policy} ply {t}")
            b.step(acts.cpu(), auto_reset=False)
            o.step(oa, auto_reset=False)
        assert_state_equal(export_np(b), o.export(), f"{policy} many moves")


def test_gumbel_with_logits_in_memory_follows_logits():
    n = 64
    pool = oracle.make_setup_pool(4, 256)
    b = _buf(n, seed=4, setup_pool=torch.from_numpy(pool))
    b.reset_all_from_pool()
    logits = torch.randn(n, 10000, device="cuda") * 1e4
    acts, lp = b.sample_actions("gumbel", logits=logits)
    mask = b.compute_legal_action_mask().reshape(n, -1)
    best = torch.where(mask, logits, torch.full_like(logits, -float("inf"))).argmax(1)
    assert torch.equal(acts, best)
    assert torch.all(lp <= 0) and torch.all(lp > -1e-3)


def test_host_actions_step_equals_reference_api():
    n = 128
    pool = oracle.make_setup_pool(8, 512)
    a = _buf(n, seed=8, setup_pool=torch.from_numpy(pool))
    c = _buf(n, seed=8, setup_pool=torch.from_numpy(pool))
    a.reset_all_from_pool()
    c.reset_all_from_pool()
    for _ in range(60):
        acts, _ = a.sample_actions()
        host = acts.cpu().pin_memory()
        a.step(host, auto_reset=False)
        c.apply_actions(acts.cpu())
    assert_state_equal(export_np(a), export_np(c), "step vs apply_actions")


@pytest.mark.parametrize("pinned,mapped", [(True, True), (False, True), (True, False), (False, False)])
def test_step_host_equals_step(pinned, mapped):
    """sb_step_host (host actions in, reward/done/next_action back into pinned
    memory in one call: by copies, or read / written in place by the kernel)
    drives the game exactly as step() with device tensors, for host-chosen
    actions (the previous proposals) and device sampling."""
    n = 300
    pool = torch.from_numpy(oracle.make_setup_pool(17, 512))
    h = _buf(n, seed=17, setup_pool=pool, no_attack_limit=30)
    d = _buf(n, seed=17, setup_pool=pool, no_attack_limit=30)
    h.reset_all_from_pool()
    d.reset_all_from_pool()
    r = h.step_host(None, mapped=mapped)
    ref = d.step(None)
    for t in range(80):
        np.testing.assert_array_equal(r.next_action.numpy(), ref.next_action.cpu().numpy(), err_msg=f"ply {t}")
        np.testing.assert_array_equal(r.reward.numpy(), ref.reward.cpu().numpy())
        np.testing.assert_array_equal(r.done.numpy(), ref.done.cpu().numpy())
        if t % 3 == 2:
            r, ref = h.step_host(None, mapped=mapped), d.step(None)
            continue
        acts = r.next_action.to(torch.int64)
        if pinned:
            acts = acts.pin_memory()
        if t % 5 == 0:
            acts[::7] = 0  # illegal: ignored and counted for those games
        r = h.step_host(acts, mapped=mapped)
        ref = d.step(acts.to("cuda"))
        assert torch.equal(r.device.infostate, ref.infostate)
        assert torch.equal(r.device.legal_mask, ref.legal_mask)
    assert_state_equal(export_np(h), export_np(d), "step_host vs step")
    with pytest.raises(RuntimeError):
        h.step_host(torch.zeros(n, dtype=torch.int64, device="cuda"))
    with pytest.raises(RuntimeError):
        h.step_host(torch.zeros(n - 1, dtype=torch.int64))


def test_step_host_rejects_pageable_memory_for_in_place_reads():
    """The C ABI refuses, with an error and before any launch, a pageable host
    pointer where the kernel would read in place."""
    import ctypes

    import ataraxos_b200._capi as C

    n = 64
    b = _buf(n, seed=3, pool_size=256)
    b.reset_all_from_pool()
    h = b._host_io()
    pageable = np.zeros(n, dtype=np.int64)
    io = C.SbHostIo(actions_host=pageable.ctypes.data, actions_dev=None, back_dev=None, back_host=None,
                    back_bytes=0, sync=1, reserved=0)
    pol = C.SbPolicy(kind=C.SB_POLICY_UNIFORM, reserved=0, logits=None)
    rc = C.lib().sb_step_host(ctypes.byref(b._st), ctypes.byref(io), 0, ctypes.byref(pol), 1,
                              h["out"]["copy"][True], torch.cuda.current_stream().cuda_stream)
    assert rc == C.SB_E_ARG
    assert b"page-locked" in C.lib().sb_last_error()
    b.step(None)  # the buffer still works


def test_shard_invariance_env_base():
    """A buffer owning envs [64,128) reproduces those envs of a 128-env buffer."""
    pool = oracle.make_setup_pool(21, 1024)
    whole = _buf(128, seed=21, setup_pool=torch.from_numpy(pool))
    lo = _buf(64, seed=21, setup_pool=torch.from_numpy(pool), env_base=0)
    hi = _buf(64, seed=21, setup_pool=torch.from_numpy(pool), env_base=64)
    for b in (whole, lo, hi):
        b.reset_all_from_pool()
    for _ in range(300):
        for b in (whole, lo, hi):
            b.step(None)
    w = export_np(whole)
    for part, sl in ((export_np(lo), slice(0, 64)), (export_np(hi), slice(64, 128))):
        assert_state_equal(part, {k: v[sl] for k, v in w.items()}, "shard")


def test_state_dict_round_trip():
    pool = oracle.make_setup_pool(2, 256)
    b = _buf(96, seed=2, setup_pool=torch.from_numpy(pool))
    b.reset_all_from_pool()
    for _ in range(40):
        b.step(None)
    sd = b.state_dict()
    for _ in range(40):
        b.step(None)
    ref = export_np(b)
    c = _buf(96, seed=0)
    c.load_state_dict(sd)
    for _ in range(40):
        c.step(None)
    assert_state_equal(export_np(c), ref, "resumed")


def test_episode_stats_count_finished_games():
    n = 500
    pool = oracle.make_setup_pool(6, 512)
    b, o = _paired(n, 6, pool, no_attack_limit=30)
    fin = red = blue = draw = length = 0
    for _ in range(300):
        mn = o.a["move_number"].copy()
        r = o.step(None)
        d = r["done"].astype(bool)
        fin += int(d.sum())
        red += int((d & (r["reward"] == 1)).sum())
        blue += int((d & (r["reward"] == -1)).sum())
        draw += int((d & (r["reward"] == 0)).sum())
        length += int((mn[d] + 1).sum())
        b.step(None)
    s = b.episode_stats().cpu().tolist()
    assert s[:4] == [fin, red, blue, draw] and fin > 0
    assert s[4] == length


def test_bad_inputs_raise():
    b = _buf(2)
    with pytest.raises(RuntimeError):
        b.apply_actions(torch.zeros(3, dtype=torch.int64))
    with pytest.raises(RuntimeError):
        b.apply_actions(torch.zeros(2, dtype=torch.int32))
    with pytest.raises(RuntimeError):
        b.apply_actions(torch.zeros((2, 1), dtype=torch.int64))
    bad = torch.zeros((2, 10, 10), dtype=torch.int8)
    bad[0, 0, 0] = 13
    with pytest.raises(RuntimeError):
        b.reset_all(bad, torch.zeros((2, 10, 10), dtype=torch.int8))
    with pytest.raises(RuntimeError):
        b.reset_all(torch.zeros((2, 10, 9), dtype=torch.int8), torch.zeros((2, 10, 10), dtype=torch.int8))
    with pytest.raises(RuntimeError):
        b.step(None)  # auto_reset without a setup pool


def test_empty_buffer():
    b = _buf(0, pool_size=16)
    b.reset_all_from_pool()
    out = b.step(None)
    assert out.infostate.shape == (0, 488, 10, 10) and out.legal_mask.shape == (0, 100, 100)
    assert b.compute_legal_action_mask().shape == (0, 100, 100)
    assert b.compute_infostate_tensor().shape == (0, 488, 10, 10)
    assert b.hash_board().shape == (0,)
    r = b.step_host(None)
    assert r.reward.shape == (0,)
    assert b.current_step() == 0


def test_full_size_config3_properties_and_subsample_parity():
    """Benchmark config 3 at full size on one GPU (262,144 envs, Gumbel): every
    proposed move is set in its game's legal mask, and a subsample of 257
    games, rebuilt on the oracle from the exported state, has bit-identical
    masks and bfloat16 infostates."""
    n = 262144
    b = _buf(n, seed=3, pool_size=1 << 20)
    b.reset_all_from_pool()
    for _ in range(3):
        out = b.step(None, policy="gumbel")
    nxt = out.next_action.long()
    flat = out.legal_mask.view(n, -1)
    live = nxt >= 0
    assert int(live.sum()) == n
    assert bool(flat.gather(1, nxt.clamp(min=0)[:, None]).squeeze(1)[live].all())
    idx = torch.arange(0, n, 1021, device="cuda")
    st = export_np(b)
    sub = idx.cpu().numpy()
    o = oracle.OracleState(len(sub))
    for k, v in o.a.items():
        np.copyto(v, st[k][sub].astype(v.dtype).reshape(v.shape))
    np.testing.assert_array_equal(flat[idx].cpu().numpy().reshape(-1, 100, 100).view(np.uint8), o.legal_mask_u8())
    bits = out.infostate[idx].view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(bits, o.infostate_bf16_bits())
