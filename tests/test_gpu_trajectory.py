"""Trajectory ring (multi-ply launches) and belief resampling on the B200, vs the oracle.

* ``TrajectoryBuffer.rollout(k)`` runs k plies in one launch; every slot of
  the ring must equal what the oracle produces ply by ply (uniform policy:
  bit-exact observations, masks, actions, rewards, dones; log-probs to 1e-6),
  including wrap-around of the ring;
* Gumbel-policy rollouts: the oracle's proposals with bit-identical
  log-probs ply by ply (which also match log-softmax of the virtual logits),
  replayed legally on the oracle;
* ``resample_from`` (belief resampling) is bit-exact with the oracle's
  restatement and keeps everything the side to move knows.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _helpers import assert_state_equal, export_np

pytestmark = pytest.mark.gpu


def _pair(n, seed, pool_n=1024, **kw):
    from ataraxos_b200 import StrategoRolloutBuffer

    pool = oracle.make_setup_pool(seed + 1, pool_n)
    b = StrategoRolloutBuffer(n, 0, seed=seed, setup_pool=torch.from_numpy(pool), **kw)
    o = oracle.OracleState(n, seed=seed, pool=pool, **kw)
    b.reset_all_from_pool()
    o.reset_pool(force_all=True)
    return b, o


def _compact(bf16_bits: np.ndarray) -> np.ndarray:
    n = bf16_bits.shape[0]
    out = np.zeros((n, 76, 10, 10), dtype=np.uint16)
    out[:, :43] = bf16_bits[:, :43]
    out[:, 44:] = bf16_bits[:, 456:]
    return out


def test_trajectory_ring_matches_oracle_uniform():
    from ataraxos_b200.trajectory import TrajectoryBuffer

    n, T = 300, 16
    b, o = _pair(n, 31, no_attack_limit=40)
    tr = TrajectoryBuffer(b, T, policy="uniform", store_hash=True)
    ref = {}  # ply index -> dict of oracle values for the state observed at that ply

    def observe(t):
        acts, lp, _ = o.sample(ply=t, policy=oracle.POLICY_UNIFORM)
        ref[t] = {"obs": _compact(o.infostate_bf16_bits()), "mask": o.legal_mask_bits(), "action": acts,
                  "logprob": lp, "hash": o.hash_board()}

    tr.prime()
    observe(0)
    t = 0
    for chunk in (7, 13, 1, 19):
        tr.rollout(chunk)
        for _ in range(chunk):
            r = o.step(None)
            ref[t]["reward"], ref[t]["done"] = r["reward"], r["done"]
            t += 1
            observe(t)
    assert tr.slot == t % T and b.ply == t
    got = {k: getattr(tr, k).cpu().numpy() for k in ("action", "logprob", "reward", "done", "hash")}
    got["obs"] = tr.obs.view(torch.int16).cpu().numpy().view(np.uint16)
    got["mask"] = tr.mask.cpu().numpy()
    for ply in range(t - T + 1, t + 1):
        s = ply % T
        for k in ("obs", "mask", "action", "hash"):
            np.testing.assert_array_equal(got[k][s], ref[ply][k].astype(got[k].dtype), err_msg=f"{k} ply {ply}")
        np.testing.assert_allclose(got["logprob"][s], ref[ply]["logprob"], atol=1e-6)
        if ply < t:
            np.testing.assert_array_equal(got["reward"][s], ref[ply]["reward"])
            np.testing.assert_array_equal(got["done"][s], ref[ply]["done"])
    assert_state_equal(export_np(b), o.export(), "after trajectory rollout")
    assert int(tr.stats[0]) > 0


def test_trajectory_gumbel_replays_on_oracle():
    from ataraxos_b200.trajectory import TrajectoryBuffer

    n, T, plies = 128, 64, 50
    b, o = _pair(n, 77)
    tr = TrajectoryBuffer(b, T, policy="gumbel", obs_dtype=None)
    tr.prime()
    tr.rollout(plies)
    acts = tr.action.cpu().numpy().astype(np.int64)
    lps = tr.logprob.cpu().numpy()
    dones = tr.done.cpu().numpy()
    for p in range(plies):
        # the rollout's proposals are the oracle's, bit for bit
        oa, olp, _ = o.sample(ply=p, policy=oracle.POLICY_GUMBEL)
        np.testing.assert_array_equal(acts[p], oa, err_msg=f"ply {p}")
        np.testing.assert_array_equal(lps[p].view(np.uint32), olp.view(np.uint32), err_msg=f"ply {p}")
        if p % 10 == 0:  # log-prob of the chosen action = log-softmax of the virtual logits
            for g in range(0, n, 17):
                legal = o.legal_list(g)
                z = np.array([oracle.logit_noise(b.seed, g, p, int(a))[0] for a in legal], dtype=np.float64)
                i = int(np.nonzero(legal == acts[p, g])[0][0])
                ref_lp = z[i] - (z.max() + np.log(np.exp(z - z.max()).sum()))
                assert abs(lps[p, g] - ref_lp) < 1e-4
        before = o.a["invalid_count"].copy()
        r = o.step(acts[p], auto_reset=True)
        np.testing.assert_array_equal(o.a["invalid_count"], before)
        np.testing.assert_array_equal(r["done"], dones[p])
    assert_state_equal(export_np(b), o.export(), "after gumbel trajectory")


def _advanced_roots(n_roots, plies, seed):
    b, o = _pair(n_roots, seed)
    for _ in range(plies):
        b.step(None)
        o.step(None)
    return b, o


def test_belief_resample_matches_oracle():
    from ataraxos_b200 import StrategoRolloutBuffer

    roots, oroots = _advanced_roots(8, 150, 5)
    k = 50
    root_of = np.repeat(np.arange(8), k)
    s = StrategoRolloutBuffer(8 * k, 0, seed=1234)
    os_ = oracle.OracleState(8 * k, seed=1234)
    s.resample_from(roots, torch.from_numpy(root_of))
    os_.resample_from(oroots, root_of)
    assert_state_equal(export_np(s), os_.export(), "belief samples")
    np.testing.assert_array_equal(s.hash_board().cpu().numpy(), os_.hash_board())
    # samples are playable and keep their proposal cache coherent
    s.step(torch.from_numpy(s.sample_actions()[0].cpu().numpy()), auto_reset=False)


def test_belief_resample_keeps_information_and_is_uniform():
    from ataraxos_b200 import StrategoRolloutBuffer

    roots, _ = _advanced_roots(2, 150, 9)
    k = 4000
    s = StrategoRolloutBuffer(2 * k, 0, seed=99)
    s.resample_from(roots, torch.arange(2, device="cuda").repeat_interleave(k))
    R = export_np(roots)
    S = export_np(s)
    for r in range(2):
        sl = slice(r * k, (r + 1) * k)
        me = int(R["current_player"][r])
        ow, pc = R["board_owner"][r].reshape(100), R["board_piece"][r].reshape(100)
        rv, mv = R["revealed_squares"][r].astype(bool), R["moved_squares"][r].astype(bool)
        so, sp = S["board_owner"][sl].reshape(k, 100), S["board_piece"][sl].reshape(k, 100)
        assert (so == ow).all()
        known = (ow == me) | rv | (ow < 0)
        assert (sp[:, known] == pc[known]).all()
        hidden = (ow == 1 - me) & ~rv
        assert (np.sort(sp[:, hidden], axis=1) == np.sort(pc[hidden])).all()
        hm = hidden & mv
        assert ((sp[:, hm] >= 1) & (sp[:, hm] <= 10)).all()
        # the Flag lands uniformly on the unmoved hidden squares
        hu = np.nonzero(hidden & ~mv)[0]
        if len(hu) >= 2 and (pc[hidden] == 11).any():
            counts = np.array([(sp[:, q] == 11).sum() for q in hu], dtype=np.float64)
            assert counts.sum() == k
            exp = k / len(hu)
            chi2 = ((counts - exp) ** 2 / exp).sum()
            assert chi2 < len(hu) + 6 * np.sqrt(2 * len(hu)), chi2
        assert len({bytes(x) for x in sp[:200, hidden]}) > 150  # the deals differ


def test_search_rollouts_shapes_and_values():
    from ataraxos_b200.trajectory import BeliefRollouts

    roots, _ = _advanced_roots(4, 150, 13)
    br = BeliefRollouts(roots, 100, depth=40, seed=3)
    out = br.run()
    assert tuple(out["masks"].shape) == (41, 400, 1250)
    assert tuple(out["actions"].shape) == (41, 400)
    v = out["terminal_value"].cpu().numpy()
    assert set(np.unique(v)).issubset({-1.0, 0.0, 1.0})
    d = out["done"].cpu().numpy()
    assert ((v != 0) <= d).all()
    # every recorded action of an unfinished rollout is legal in its slot's mask
    m = out["masks"].cpu().numpy()
    a = out["actions"].cpu().numpy().astype(np.int64)
    for p in range(0, 40, 7):
        live = a[p] >= 0
        idx = np.nonzero(live)[0]
        bits = (m[p, idx, a[p, idx] >> 3] >> (a[p, idx] & 7)) & 1
        assert bits.all()
