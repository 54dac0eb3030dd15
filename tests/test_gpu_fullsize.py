"""The benchmarked workloads at their full sizes, replayed on the oracle.

Each test builds the kernel instantiation that ``bench.py`` times, at the
shape it times, and checks it against the CPU oracle (``oracle/``, the C
restatement of the reference simulator) bit for bit:

* config 2 exactly as benched: 4096 games, the single-ply production step
  (uniform actions, auto-reset from a 65,536-entry pool, bf16 dense
  infostate, u8 mask), 1000 plies; every ply's action / log-prob / reward /
  done, and every 100 plies the full state, hashes, masks and infostate of
  every game; and the same 4096 games as the bench steps them, in 3 groups
  on their own streams inside CUDA graphs, 300 plies;
* config 3: 262,144 games on one GPU, Gumbel-max over virtual N(0,1)
  logits, a 1M-entry pool, 200 plies; a subsample of 4,096 games spread over
  the whole batch is replayed with its global indices, checked every ply
  (action / log-prob / reward / done) and every 50 plies (state, masks,
  infostate);
* config 4: 32,768 games, T=128 trajectory ring (compact bf16 infostate,
  bit-packed masks), 8 plies per launch, 17 launches (the ring wraps);
* config 5: 64 roots advanced 150 plies, 1000 belief samples each, 40-ply
  rollouts; a subsample of 4,000 samples replayed (resample, per-ply masks
  and actions, terminal values);
* the distribution of the Gumbel sampler over virtual logits (the path that
  configs 3 and 4 time) against the softmax of the same logits (chi-square
  over the rank of the chosen action).
"""

from __future__ import annotations

import gc
import os

import numpy as np
import pytest
import torch

import oracle
from _helpers import assert_state_equal, export_np

pytestmark = pytest.mark.gpu

SEED = 20251107  # the bench's seed
THREADS = os.cpu_count() or 1


@pytest.fixture(autouse=True)
def _release_device_memory():
    """These workloads hold up to ~70 GB each: return it between tests."""
    yield
    gc.collect()
    torch.cuda.empty_cache()


def _buf(n, **kw):
    from ataraxos_b200 import StrategoRolloutBuffer

    return StrategoRolloutBuffer(n, 0, **kw)


def _bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> its uint16 bit patterns on the host."""
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _check_state(buf, o, idx, ctx):
    st = export_np(buf)
    if idx is not None:
        st = {k: v[idx] for k, v in st.items()}
    assert_state_equal(st, o.export(), ctx)
    h = buf.hash_board().cpu().numpy()
    np.testing.assert_array_equal(h if idx is None else h[idx], o.hash_board(), err_msg=f"{ctx}: hash")


def _check_history(got: dict[str, np.ndarray], ref: dict[str, np.ndarray], ctx: str):
    for k in ("action", "reward", "done"):
        np.testing.assert_array_equal(got[k], ref[k].astype(got[k].dtype), err_msg=f"{ctx}: {k}")
    np.testing.assert_array_equal(got["logprob"].view(np.uint32), ref["logprob"].view(np.uint32),
                                  err_msg=f"{ctx}: logprob bits")


def test_config2_as_benched_matches_oracle_1000_plies():
    B, plies, chunk = 4096, 1000, 100
    buf = _buf(B, seed=SEED, env_base=0, pool_size=65536, pool_seed=SEED, obs_dtype=torch.bfloat16,
               obs_layout="dense", mask_format="u8")
    pool = buf.setup_pool.cpu().numpy()
    np.testing.assert_array_equal(pool, oracle.make_setup_pool(SEED, 65536))
    buf.reset_all_from_pool()
    o = oracle.OracleState(B, seed=SEED, pool=pool)
    o.reset_pool(force_all=True)
    dev = buf.device
    hist = {"action": torch.empty((chunk, B), dtype=torch.int64, device=dev),
            "logprob": torch.empty((chunk, B), dtype=torch.float32, device=dev),
            "reward": torch.empty((chunk, B), dtype=torch.float32, device=dev),
            "done": torch.empty((chunk, B), dtype=torch.uint8, device=dev)}
    finished = 0
    for c in range(plies // chunk):
        for t in range(chunk):
            out = buf.step(None)
            hist["action"][t].copy_(out.action)
            hist["logprob"][t].copy_(out.logprob)
            hist["reward"][t].copy_(out.reward)
            hist["done"][t].copy_(out.done.view(torch.uint8))
        ref = o.run(chunk, threads=THREADS)
        got = {k: v.cpu().numpy() for k, v in hist.items()}
        ctx = f"config2 plies {c * chunk}-{(c + 1) * chunk - 1}"
        _check_history(got, ref, ctx)
        finished += int(ref["done"].sum())
        _check_state(buf, o, None, ctx)
        obs = o.observe(mask_u8=True, info="dense", threads=THREADS)
        np.testing.assert_array_equal(out.legal_mask.view(torch.uint8).cpu().numpy(), obs["mask_u8"],
                                      err_msg=f"{ctx}: u8 mask")
        for a in range(0, B, 1024):  # infostate bits in slices of 1024 games (400 MB in all)
            np.testing.assert_array_equal(_bits(out.infostate[a:a + 1024]), obs["info"][a:a + 1024],
                                          err_msg=f"{ctx}: infostate games {a}-{a + 1023}")
    st = buf.episode_stats().cpu().numpy()
    assert st[0] == finished and finished > 1000, (st, finished)
    assert buf.status() == 0


def test_config2_grouped_graph_as_benched_matches_oracle():
    """Config 2 the way bench.py times it: the 4096 games as 3 buffers over
    contiguous global env ranges, each stepped on its own stream and writing
    4 output sets in turn, the steps captured in one CUDA graph per 100 plies
    (the groups' launches run concurrently); after every 100 plies the full
    state, hashes, u8 masks and infostate bits of every game equal the
    oracle's one run of all 4096 games."""
    from ataraxos_b200 import sharding

    B, G, plies, chunk = 4096, 3, 300, 100
    main = torch.cuda.Stream()
    parts = []
    for g in range(G):
        off, n = sharding.shard_range(B, G, g)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            b = _buf(n, seed=SEED, env_base=off, pool_size=65536, pool_seed=SEED, obs_dtype=torch.bfloat16,
                     obs_layout="dense", mask_format="u8")
            b.reset_all_from_pool()
            sets = [b._ensure_outputs()] + [b.new_outputs() for _ in range(3)]
        parts.append((b, s, sets, off, n))
    torch.cuda.synchronize()
    o = oracle.OracleState(B, seed=SEED, pool=oracle.make_setup_pool(SEED, 65536))
    o.reset_pool(force_all=True)
    outs = [None] * G
    for c in range(plies // chunk):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=main):
            fork = torch.cuda.Event()
            fork.record(main)
            for _, s, _, _, _ in parts:
                s.wait_event(fork)
            for i in range(c * chunk, (c + 1) * chunk):
                for g, (b, s, sets, _, _) in enumerate(parts):
                    with torch.cuda.stream(s):
                        outs[g] = b.step(None, outputs=sets[i % 4])
            for _, s, _, _, _ in parts:
                join = torch.cuda.Event()
                join.record(s)
                main.wait_event(join)
        with torch.cuda.stream(main):
            graph.replay()
        torch.cuda.synchronize()
        del graph
        o.run(chunk, threads=THREADS)
        ctx = f"grouped config2 after {(c + 1) * chunk} plies"
        ref = o.export()
        obs = o.observe(mask_u8=True, info="dense", threads=THREADS)
        h_ref = o.hash_board()
        for g, (b, _, _, off, n) in enumerate(parts):
            sl = slice(off, off + n)
            assert_state_equal(export_np(b), {k: v[sl] for k, v in ref.items()}, f"{ctx}, group {g}")
            np.testing.assert_array_equal(b.hash_board().cpu().numpy(), h_ref[sl], err_msg=f"{ctx}: hash")
            np.testing.assert_array_equal(outs[g].legal_mask.view(torch.uint8).cpu().numpy(), obs["mask_u8"][sl],
                                          err_msg=f"{ctx}, group {g}: u8 mask")
            np.testing.assert_array_equal(_bits(outs[g].infostate), obs["info"][sl],
                                          err_msg=f"{ctx}, group {g}: infostate")
            assert b.status() == 0


def _spread(n_all: int, n_sub: int) -> np.ndarray:
    """n_sub indices spread over [0, n_all), the last CTA's games included."""
    idx = np.unique(np.concatenate([np.linspace(0, n_all - 1, n_sub - 16).astype(np.int64),
                                    np.arange(n_all - 16, n_all)]))
    return idx


def test_config3_full_size_gumbel_subsample_matches_oracle():
    B, plies, every = 262144, 200, 50
    buf = _buf(B, seed=SEED, env_base=0, pool_size=1 << 20, pool_seed=SEED, obs_dtype=torch.bfloat16,
               obs_layout="dense", mask_format="u8")
    pool = buf.setup_pool.cpu().numpy()
    np.testing.assert_array_equal(pool, oracle.make_setup_pool(SEED, 1 << 20))
    buf.reset_all_from_pool()
    sub = _spread(B, 4096)
    o = oracle.OracleState(len(sub), seed=SEED, pool=pool, genv=sub)
    o.reset_pool(force_all=True)
    dev = buf.device
    si = torch.from_numpy(sub).to(dev)
    hist = {"action": torch.empty((every, len(sub)), dtype=torch.int64, device=dev),
            "logprob": torch.empty((every, len(sub)), dtype=torch.float32, device=dev),
            "reward": torch.empty((every, len(sub)), dtype=torch.float32, device=dev),
            "done": torch.empty((every, len(sub)), dtype=torch.uint8, device=dev)}
    for c in range(plies // every):
        for t in range(every):
            out = buf.step(None, policy="gumbel")
            hist["action"][t].copy_(out.action[si])
            hist["logprob"][t].copy_(out.logprob[si])
            hist["reward"][t].copy_(out.reward[si])
            hist["done"][t].copy_(out.done.view(torch.uint8)[si])
        ref = o.run(every, policy=oracle.POLICY_GUMBEL, threads=THREADS)
        ctx = f"config3 plies {c * every}-{(c + 1) * every - 1}"
        _check_history({k: v.cpu().numpy() for k, v in hist.items()}, ref, ctx)
        _check_state(buf, o, sub, ctx)
        obs = o.observe(mask_u8=True, info="dense", threads=THREADS)
        np.testing.assert_array_equal(out.legal_mask.view(torch.uint8)[si].cpu().numpy(), obs["mask_u8"],
                                      err_msg=f"{ctx}: u8 mask")
        np.testing.assert_array_equal(_bits(out.infostate[si]), obs["info"], err_msg=f"{ctx}: infostate")
    assert buf.status() == 0


def test_config4_full_size_ring_wraps_and_matches_oracle():
    from ataraxos_b200.trajectory import TrajectoryBuffer

    B, T, R, launches = 32768, 128, 8, 17  # 136 plies: the ring wraps
    buf = _buf(B, seed=SEED, env_base=0, pool_size=65536, pool_seed=SEED)
    pool = buf.setup_pool.cpu().numpy()
    buf.reset_all_from_pool()
    tr = TrajectoryBuffer(buf, T, policy="gumbel")
    assert tr.obs.shape == (T, B, 76, 10, 10) and tr.mask.shape == (T, B, 1250)
    sub = _spread(B, 4096)
    si = torch.from_numpy(sub).to(buf.device)
    o = oracle.OracleState(len(sub), seed=SEED, pool=pool, genv=sub)
    o.reset_pool(force_all=True)

    def check_obs(slot, ctx):
        obs = o.observe(mask_bits=True, info="compact", threads=THREADS)
        np.testing.assert_array_equal(tr.mask[slot][si].cpu().numpy(), obs["mask_bits"], err_msg=f"{ctx}: mask bits")
        np.testing.assert_array_equal(_bits(tr.obs[slot][si]), obs["info"], err_msg=f"{ctx}: compact infostate")

    tr.prime()
    check_obs(0, "config4 primed slot 0")
    t = 0
    for L in range(launches):
        tr.rollout(R)
        got = {k: getattr(tr, k)[:, si].cpu().numpy() for k in ("action", "logprob", "reward", "done")}
        for p in range(R):
            s = t % T
            ref = o.run(1, policy=oracle.POLICY_GUMBEL, threads=THREADS)
            ctx = f"config4 launch {L} ply {t} (slot {s})"
            np.testing.assert_array_equal(got["action"][s].astype(np.int64), ref["action"][0], err_msg=ctx)
            np.testing.assert_array_equal(got["logprob"][s].view(np.uint32), ref["logprob"][0].view(np.uint32),
                                          err_msg=ctx)
            np.testing.assert_array_equal(got["reward"][s], ref["reward"][0], err_msg=ctx)
            np.testing.assert_array_equal(got["done"][s], ref["done"][0], err_msg=ctx)
            t += 1
            if p in (3, R - 1):
                check_obs(t % T, f"config4 state after ply {t - 1} (slot {t % T})")
    assert t > T and tr.slot == t % T
    _check_state(buf, o, sub, "config4 final")
    assert int(tr.stats[0]) > 0 and buf.status() == 0


def test_config5_full_size_search_subsample_matches_oracle():
    from ataraxos_b200.trajectory import BeliefRollouts

    n_roots, k, depth = 64, 1000, 40
    roots = _buf(n_roots, seed=SEED, env_base=0, pool_size=65536, pool_seed=SEED)
    pool = roots.setup_pool.cpu().numpy()
    roots.reset_all_from_pool()
    oroots = oracle.OracleState(n_roots, seed=SEED, pool=pool)
    oroots.reset_pool(force_all=True)
    for _ in range(150):
        roots.step(None)
    oroots.run(150, threads=THREADS, record=False)
    _check_state(roots, oroots, None, "config5 roots after 150 plies")
    br = BeliefRollouts(roots, k, depth, seed=SEED + 1, policy="uniform")
    out = br.run()
    sub = np.arange(0, n_roots * k, 16)  # 4,000 samples, every root
    si = torch.from_numpy(sub).to(roots.device)
    o = oracle.OracleState(len(sub), seed=SEED + 1, genv=sub)
    o.resample_from(oroots, sub // k)
    masks = out["masks"][:, si].cpu().numpy()
    acts = out["actions"][:, si].cpu().numpy().astype(np.int64)
    rew = br.traj.reward[:, si].cpu().numpy()
    done = br.traj.done[:, si].cpu().numpy()
    for p in range(depth):
        obs = o.observe(mask_bits=True, threads=THREADS)
        np.testing.assert_array_equal(masks[p], obs["mask_bits"], err_msg=f"config5 mask at ply {p}")
        ref = o.run(1, auto_reset=False, threads=THREADS)
        np.testing.assert_array_equal(acts[p], ref["action"][0], err_msg=f"config5 action at ply {p}")
        np.testing.assert_array_equal(rew[p], ref["reward"][0], err_msg=f"config5 reward at ply {p}")
        np.testing.assert_array_equal(done[p], ref["done"][0], err_msg=f"config5 done at ply {p}")
    np.testing.assert_array_equal(masks[depth], o.observe(mask_bits=True)["mask_bits"], err_msg="config5 last mask")
    np.testing.assert_array_equal(out["terminal_value"][si].cpu().numpy(), o.reward_pl0())
    _check_state(br.samples, o, sub, "config5 samples after the rollouts")


def test_gumbel_virtual_logits_sample_their_softmax():
    """Chi-square: the rank (by logit) of the action the Gumbel sampler picks
    over virtual N(0,1) logits, against the ranks' softmax probabilities."""
    n, plies = 65536, 24
    buf = _buf(n, seed=SEED, pool_size=4096, pool_seed=SEED, obs_layout="compact", mask_format="none")
    pool = buf.setup_pool.cpu().numpy()
    buf.reset_all_from_pool()
    o = oracle.OracleState(n, seed=SEED, pool=pool)
    o.reset_pool(force_all=True)
    edges = [0, 1, 2, 3, 4, 5, 6, 8, 11, 16, 10_000]  # rank bins (0 = the largest logit)
    obs_count = np.zeros(len(edges) - 1)
    exp_count = np.zeros(len(edges) - 1)
    trials = 0
    for t in range(plies):
        if t % 4 == 0:  # sample at the current state with several RNG plies
            acts, z, cnt = o.virtual_logits(t)
            a_gpu, lp_gpu = buf.sample_actions("gumbel", ply=t)
            a_gpu = a_gpu.cpu().numpy()
            live = (cnt >= 2) & (cnt <= z.shape[1])
            zz = np.where(np.arange(z.shape[1])[None, :] < cnt[:, None], z.astype(np.float64), -np.inf)[live]
            aa = acts[live].astype(np.int64)
            order = np.argsort(-zz, axis=1, kind="stable")
            p = np.exp(zz - zz.max(1, keepdims=True))
            p /= p.sum(1, keepdims=True)
            p_rank = np.take_along_axis(p, order, axis=1)
            chosen = np.take_along_axis(aa, order, axis=1) == a_gpu[live][:, None]
            assert chosen.sum(1).min() == 1  # the sampled action is legal
            rank = np.argmax(chosen, axis=1)
            for b in range(len(edges) - 1):
                obs_count[b] += ((rank >= edges[b]) & (rank < edges[b + 1])).sum()
                exp_count[b] += p_rank[:, edges[b]:edges[b + 1]].sum()
            trials += int(live.sum())
            # the reported log-prob is the log-softmax of the chosen logit (float32 arithmetic)
            lp_ref = np.log(p_rank[np.arange(len(rank)), rank])
            np.testing.assert_allclose(lp_gpu.cpu().numpy()[live], lp_ref, atol=2e-5)
        buf.step(None, policy="gumbel", observe=False)
        o.run(1, policy=oracle.POLICY_GUMBEL, threads=THREADS, record=False)
    assert trials > 300_000
    keep = exp_count >= 20
    chi2 = float(((obs_count[keep] - exp_count[keep]) ** 2 / exp_count[keep]).sum())
    dof = int(keep.sum()) - 1
    # p < 1e-6 for chi-square with dof <= 9 needs chi2 > 46
    assert chi2 < 46.0, (chi2, dof, obs_count.tolist(), exp_count.round(1).tolist())
