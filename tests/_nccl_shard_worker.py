"""One NCCL rank of ``test_gpu_multigpu.py`` (launched by torch.distributed.run).

Rank r steps its shard of a ragged game range on GPU r; the per-game Zobrist
hashes and move numbers are all-gathered (padded to the largest shard), the
episode counters are gathered with ``sharding.gather_episode_stats``, and rank
0 checks both against a one-GPU buffer holding every game.  Exit code 0 on
agreement.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from ataraxos_b200 import StrategoRolloutBuffer, sharding  # noqa: E402

TOTAL, PLIES, SEED = 1001, 300, 23


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    base, n = sharding.shard_range(TOTAL, world, rank)
    kw = dict(seed=SEED, pool_size=4096, pool_seed=SEED, no_attack_limit=30)
    buf = StrategoRolloutBuffer(n, local, env_base=base, **kw)
    buf.reset_all_from_pool()
    for _ in range(PLIES):
        buf.step(None)
    width = sharding.shard_range(TOTAL, world, 0)[1]
    pad = torch.full((2, width), -1, dtype=torch.int64, device=dev)
    pad[0, :n] = buf.hash_board()
    pad[1, :n] = buf.get_move_number().to(torch.int64)
    parts = torch.empty((world, 2, width), dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(parts, pad)
    stats = sharding.gather_episode_stats(buf.episode_stats().clone())
    ok = True
    if rank == 0:
        whole = StrategoRolloutBuffer(TOTAL, local, **kw)
        whole.reset_all_from_pool()
        for _ in range(PLIES):
            whole.step(None)
        got = torch.cat([parts[r, :, :sharding.shard_range(TOTAL, world, r)[1]] for r in range(world)], dim=1)
        ok = bool(torch.equal(got[0], whole.hash_board()))
        ok &= bool(torch.equal(got[1], whole.get_move_number().to(torch.int64)))
        ok &= bool(torch.equal(stats.sum(0), whole.episode_stats()))
        ok &= int(stats.sum(0)[0]) > 0
        print(f"multigpu shard check world={world}: {'ok' if ok else 'MISMATCH'}", flush=True)
    flag = torch.tensor([int(ok)], dtype=torch.int32, device=dev)
    dist.broadcast(flag, 0)
    dist.destroy_process_group()
    return 0 if int(flag.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
