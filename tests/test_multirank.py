"""Multi-rank host logic on CPU (gloo, world_size 2): env sharding keyed by the
global env index, the end-of-rollout episode-statistics all-gather, the
max-over-ranks timing reduction, and a rank that dies between steps.

The kernels need a GPU, so the per-rank games here are played by the CPU
oracle with each rank's ``env_base``; the GPU counterpart of the shard check
is ``test_shard_invariance_env_base`` (several buffers on one B200) and
``test_gpu_multigpu.py`` (NCCL ranks, when the box has two GPUs).
"""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ataraxos_b200 import sharding

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn_name, q, timeout_s):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
        q.put((rank, "ok", globals()[fn_name](rank, world)))
    except Exception as e:  # reported to the parent, which asserts on it
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(fn_name, world=WORLD, timeout_s=30, join_s=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn_name, q, timeout_s)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, status, val = q.get(timeout=join_s)
            out[rank] = (status, val)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    return out


# ---- rank bodies (module level so spawn can pickle them by name) ----------

def _stats_body(rank, world):
    stats = torch.tensor([rank + 1, 10 * rank, 7, 0, 1000 + rank], dtype=torch.int64)
    g = sharding.gather_episode_stats(stats)
    m = sharding.max_over_ranks(0.5 + rank)
    return g.numpy(), m


def _oracle_shard_body(rank, world):
    import oracle

    total, plies, seed = 37, 120, 5
    base, n = sharding.shard_range(total, world, rank)
    pool = oracle.make_setup_pool(seed, 256)
    o = oracle.OracleState(n, seed=seed, pool=pool, env_base=base, no_attack_limit=25)
    o.reset_pool(force_all=True)
    acc = np.zeros(5, dtype=np.int64)
    for _ in range(plies):
        acc += _episode_counts(o.step(None))
    h = torch.from_numpy(o.hash_board().astype(np.int64))
    moves = torch.from_numpy(o.export()["move_number"].astype(np.int64))
    # ragged shards: pad to the largest shard, gather, and cut back by shard_range
    width = sharding.shard_range(total, world, 0)[1]
    pad = torch.full((2, width), -1, dtype=torch.int64)
    pad[0, :n], pad[1, :n] = h, moves
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    stats = sharding.gather_episode_stats(torch.from_numpy(acc))
    hashes, mv = [], []
    for r, p in enumerate(parts):
        nr = sharding.shard_range(total, world, r)[1]
        hashes.append(p[0, :nr])
        mv.append(p[1, :nr])
    return torch.cat(hashes).numpy(), torch.cat(mv).numpy(), stats.numpy()


def _episode_counts(r) -> np.ndarray:
    """finished, red wins, blue wins, draws of one ply's step results (last slot unused)."""
    d = r["done"].astype(bool)
    return np.array([d.sum(), (d & (r["reward"] > 0)).sum(), (d & (r["reward"] < 0)).sum(),
                     (d & (r["reward"] == 0)).sum(), 0], dtype=np.int64)


def _dies_body(rank, world):
    stats = torch.tensor([1, 0, 0, 1, 5], dtype=torch.int64)
    sharding.gather_episode_stats(stats)  # step 1: both ranks present
    if rank == 1:
        raise RuntimeError("rank 1 leaves between steps")
    sharding.gather_episode_stats(stats)  # step 2: rank 1 is gone
    return "unreachable"


# ---- tests ----------------------------------------------------------------

@pytest.mark.parametrize("total", [0, 1, 7, 64, 262144, 262147])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_range_partitions(total, world):
    spans = [sharding.shard_range(total, world, r) for r in range(world)]
    assert spans[0][0] == 0
    for (b0, n0), (b1, _) in zip(spans, spans[1:]):
        assert b0 + n0 == b1
    assert sum(n for _, n in spans) == total
    sizes = [n for _, n in spans]
    assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(total, world, world)


def test_single_process_collectives_are_identity():
    s = torch.arange(5, dtype=torch.int64)
    assert torch.equal(sharding.gather_episode_stats(s), s.reshape(1, 5))
    assert sharding.max_over_ranks(3.0) == 3.0
    with pytest.raises(ValueError):
        sharding.gather_episode_stats(torch.zeros(4, dtype=torch.int64))


def test_gloo_stats_gather_and_max():
    out = _run("_stats_body")
    for rank in range(WORLD):
        status, val = out[rank]
        assert status == "ok", val
        g, m = val
        assert g.shape == (WORLD, 5)
        for r in range(WORLD):
            np.testing.assert_array_equal(g[r], [r + 1, 10 * r, 7, 0, 1000 + r])
        assert m == 0.5 + (WORLD - 1)


def test_gloo_sharded_games_equal_one_rank():
    """Ragged shards (37 games over 2 ranks) play exactly the games of one
    37-game run: same hashes, move numbers and summed episode statistics."""
    import oracle

    out = _run("_oracle_shard_body")
    whole = oracle.OracleState(37, seed=5, pool=oracle.make_setup_pool(5, 256), no_attack_limit=25)
    whole.reset_pool(force_all=True)
    acc = np.zeros(5, dtype=np.int64)
    for _ in range(120):
        acc += _episode_counts(whole.step(None))
    for rank in range(WORLD):
        status, val = out[rank]
        assert status == "ok", val
        h, mv, stats = val
        np.testing.assert_array_equal(h, whole.hash_board().astype(np.int64))
        np.testing.assert_array_equal(mv, whole.export()["move_number"].astype(np.int64))
        np.testing.assert_array_equal(stats.sum(0), acc)
        assert stats.sum(0)[0] > 0  # games did finish (no-attack limit 25)


def test_gloo_rank_leaving_between_steps_ends_peer_collective_with_error():
    out = _run("_dies_body", timeout_s=5, join_s=120)
    assert out[1][0] == "error" and "leaves between steps" in out[1][1]
    assert out[0][0] == "error", out[0]
