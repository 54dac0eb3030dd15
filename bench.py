"""Benchmark of the B200 StrategoRolloutBuffer hot path.

Metric: env state updates per second, one update = one ply of one env (sample a
uniform legal action, apply it with combat / trackers / terminal check,
auto-reset from the seeded setup pool, emit the uint8 legal mask and the
bfloat16 [488,10,10] infostate of the new state).

Default workload = benchmark config 2: 4096 envs per GPU, seeded random setups
(pool of 65536), uniform random legal actions, auto-reset, bf16 infostate
[B,488,10,10] (channels 43-455 are zero planes written once at allocation;
every ply rewrites the 75 live channels), uint8 mask [B,100,100].  One step =
one ply over all envs = one launch of the fused step kernel.  Synthetic data:
there is no dataset; setups and actions come from Philox.

Timing (config 2, default ``--timing graph``): W untimed warm-up steps, then
the K timed steps, launched back to back as one CUDA graph (captured after the
warm-up, each node one fused-step launch with its own ply number) and
replayed once between two CUDA events on the buffer's stream; barrier +
synchronize on both sides; max over ranks.  The steps write their outputs
into 4 output sets in turn (4 x 441 MB, 14x the 126 MB L2), so no step
writes lines still held in L2 and every step's 104.6 MB of writes reaches
HBM inside the timed region (the game records, 1 MB, stay in L2 from ply to
ply, as in any rollout).  ``--timing flush`` is the per-launch form: each
step bracketed by its own events, with a 512 MiB write and a 256 MiB read
between steps (outside the bracketed interval) to flush L2.
Multi-GPU (torchrun): each rank owns its own 4096 envs (global env indices
rank*4096 ...), no collective on the step path (weak scaling); an NCCL
all-gather of the episode statistics follows the timed region.

e2e: the same steps through the public host API (``step_host``: int64 actions
from page-locked host memory in, reward / done / next action back into
page-locked memory, the call returning when they have landed), CUDA events
around the loop; ``--e2e-api serve`` uses the persistent step server instead.

``--impl reference`` times the reference algorithm's CPU implementation on the
host cores: the C restatement in oracle/ (the reference's own code is Python
and cannot run on the GPU box), same config (the 4096-game batch per step),
all host threads; under torchrun rank 0 alone runs it.

``--impl reference-cuda`` times the reference's own CUDA kernels
(csrc/stratego_buffer.cu compiled from its source into oracle/_ref/, driven as
its pybind class drives them: apply_actions with its flag-count reductions,
then compute_legal_action_mask and compute_infostate_tensor, each a zeroed
fresh output plus a kernel) at config 2's 4096 games per ply, on the same
games and actions as this build's step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from ataraxos_b200 import sharding  # noqa: E402

SEED = 20251107
POOL = 65536
FALLBACK_HBM_GBS = 6650.0
METRIC = "env state updates/sec (step+mask+infostate)"

# Algorithmic bytes per update of the fused step (config 2 outputs):
#   record read + write ............... 256 + 256
#   uint8 legal mask .................. 10,000
#   bf16 infostate, 75 live planes .... 75 * 200 = 15,000
#   reward f32, done u8, action i64, logprob f32, next action i16,
#   next logprob f32 .................. 23
# (chase-ring reads on threatening moves and pool reads on resets are left out.)
BYTES_PER_UPDATE = 256 + 256 + 10_000 + 15_000 + 23
NUM_CH_DENSE = 488


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons via NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device: torch.device) -> None:
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            try:
                uuid = str(torch.cuda.get_device_properties(device).uuid)
                self._h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
                pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
        except Exception:
            self._h = None

    def _run(self) -> None:
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = self._reasons_fn(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._h is not None:
            self._stop.set()
            self._t.join()

    def summary(self) -> dict:
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


def cpu_baseline(envs: int, plies: int | None = None, seconds: float = 12.0) -> dict:
    """The reference algorithm on the host cores (oracle/ C restatement, all threads)."""
    import oracle

    threads = os.cpu_count() or 1
    pool = oracle.make_setup_pool(SEED, 4096)
    o = oracle.OracleState(envs, seed=SEED, pool=pool)
    o.reset_pool(force_all=True)
    t0 = time.perf_counter()
    o.bench_rollout(1, threads)
    t1 = time.perf_counter() - t0
    if plies is None:
        plies = max(2, min(400, int(seconds / max(t1, 1e-6))))
    t0 = time.perf_counter()
    o.bench_rollout(plies, threads)
    dt = time.perf_counter() - t0
    return {
        "value": envs * plies / dt,
        "unit": "updates/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{envs} envs x {plies} plies of the config-2 ply (uniform action, apply, auto-reset, "
                  f"u8 mask, dense bf16 [488,10,10] infostate) by the C restatement of the reference "
                  f"algorithm, {threads} threads, {dt:.1f} s",
    }


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    import oracle

    threads = os.cpu_count() or 1
    envs = args.envs  # the config-2 batch itself; one step is one ply of every game
    pool = oracle.make_setup_pool(SEED, 4096)
    o = oracle.OracleState(envs, seed=SEED, pool=pool)
    o.reset_pool(force_all=True)
    o.bench_rollout(args.warmup, threads)
    t0 = time.perf_counter()
    o.bench_rollout(args.steps, threads)
    dt = time.perf_counter() - t0
    value = envs * args.steps / dt
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "updates/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8/int32 state, bf16 infostate",
        "data": "synthetic (Philox setups and actions)",
        "config": {"workload": f"config2: {args.envs} envs/GPU, uniform random legal actions, auto-reset, "
                               f"u8 mask + bf16 dense infostate; reference arm steps {envs} envs (bounded sample)",
                   "envs_per_step": envs, "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": value, "unit": "updates/s", "cores": threads, "kind": "port",
                         "sample": f"{envs} envs x {args.steps} plies, C restatement of the reference algorithm "
                                   f"(oracle/stratego_oracle.c), {threads} threads"},
        "e2e": {"value": value, "unit": "updates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_cuda(args, rank: int) -> None:
    """The reference's own CUDA kernels at config 2 (rank 0 only): per ply,
    apply_actions + compute_legal_action_mask + compute_infostate_tensor of
    the reference class (oracle/refcuda.py), on the games and actions this
    build's step plays from the same setups (without auto-reset: the
    reference class resets only from caller-supplied planes)."""
    if rank != 0:
        return
    from oracle import refcuda

    if not refcuda.available():
        print(json.dumps({"impl": "reference-cuda", "unavailable": "oracle/_ref/libref_stratego_cuda.so was not "
                          "built (it is compiled where the reference checkout is present)"}), flush=True)
        return
    from ataraxos_b200 import StrategoRolloutBuffer

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    B, W, K = args.envs, args.warmup, args.steps
    ours = StrategoRolloutBuffer(B, dev.index, seed=SEED, pool_size=POOL, pool_seed=SEED, obs_layout="compact",
                                 mask_format="none")
    ours.reset_all_from_pool()
    ow, pc = ours.get_board_owner(), ours.get_board_piece()
    red = torch.where(ow == 0, pc, torch.zeros_like(pc))
    blue = torch.where(ow == 1, pc, torch.zeros_like(pc))
    acts = torch.empty((W + K, B), dtype=torch.int64, device=dev)
    for t in range(W + K):
        acts[t].copy_(ours.step(None, auto_reset=False, observe=False).action)
    ref = refcuda.RefCudaBuffer(B, dev.index)
    ref.reset_all(red, blue)

    def ply(t):
        ref.apply_actions(acts[t])
        ref.compute_legal_action_mask()
        ref.compute_infostate_tensor()

    for t in range(W):
        ply(t)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for t in range(W, W + K):
        ply(t)
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    value = B * K / (ms / 1e3)
    bpu = 2 * (NUM_CH_DENSE * 100 * 4 + 10_000)  # zero fill + kernel write of the f32 infostate and bool mask
    peak, _ = _peaks()
    print(json.dumps({
        "impl": "reference-cuda", "metric": METRIC, "value": value, "unit": "updates/s", "n_gpus": 1, "steps": K,
        "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "config": {"workload": f"config2: {B} envs, reference kernels (csrc/stratego_buffer.cu, -O3 --use_fast_math, "
                               "sm_100a) driven as its pybind class drives them; f32 [B,488,10,10] infostate + bool "
                               "[B,100,100] mask per ply, each zero-filled then written",
                   "l2": "outputs of one ply (841 MB) exceed L2; no flush"},
        "roofline": {"bound": "hbm", "bytes_per_update": bpu, "achieved": bpu * B / (ms / K / 1e3) / 1e9,
                     "peak": peak, "unit": "GB/s"},
        "gpu_launches": None,
    }), flush=True)


def _profile_traffic(name: str, updates_per_launch: int | None = None) -> float | None:
    """DRAM bytes (read + write) per launch from the ncu capture summarised in
    profiles/<name>: its dram_bytes_per_launch, or, for a capture taken on a
    smaller case, its dram_bytes_per_update times the updates of this launch."""
    f = ROOT / "profiles" / name
    try:
        for line in f.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch:") and updates_per_launch is None:
                return float(line.split(":", 1)[1].split()[0])
            if line.startswith("dram_bytes_per_update:") and updates_per_launch is not None:
                return float(line.split(":", 1)[1].split()[0]) * updates_per_launch
    except Exception:
        return None
    return None


class Ctx:
    def __init__(self, args):
        import torch.distributed as dist

        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = dist
        if self.world > 1:
            from datetime import timedelta

            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=self.dev)
        self.stream = torch.cuda.current_stream(self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, v: float) -> float:
        return sharding.max_over_ranks(v, self.dev)

    def gather_stats(self, stats: torch.Tensor) -> list[int]:
        """End-of-rollout NCCL all-gather of each rank's int64[5] episode statistics."""
        return sharding.gather_episode_stats(stats).sum(0).tolist()


def timed_graph(ctx: Ctx, launch, first: int, k: int):
    """launch(first) .. launch(first + k - 1) captured into one CUDA graph,
    then replayed once between CUDA events (no host work between steps)."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(first, first + k):
            launch(i)
    torch.cuda.synchronize(ctx.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    torch.cuda.nvtx.range_push("timed")
    with ClockSampler(ctx.dev) as clocks:
        e0.record(ctx.stream)
        g.replay()
        e1.record(ctx.stream)
        torch.cuda.synchronize(ctx.dev)
        ctx.barrier()
    torch.cuda.nvtx.range_pop()
    total_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    del g
    return total_ms, clocks.summary()


def timed_launches(ctx: Ctx, launch, k: int, flush_mib: int):
    """k launches, each bracketed by CUDA events; L2 flushed between them when flush_mib > 0."""
    flush = flush_rd = None
    if flush_mib > 0:
        flush = torch.empty(flush_mib << 20, dtype=torch.uint8, device=ctx.dev)
        flush_rd = torch.ones((flush_mib << 20) // 16, dtype=torch.int64, device=ctx.dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(k)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(k)]
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    # the NVTX range lets a profiler select the timed launches (ncu --nvtx --nvtx-include timed/)
    torch.cuda.nvtx.range_push("timed")
    with ClockSampler(ctx.dev) as clocks:
        for i in range(k):
            if flush is not None:
                # write a buffer larger than the 126 MB L2, then read another, so
                # the L2 holds only clean unrelated lines when the launch starts
                flush.fill_(i & 0xFF)
                flush_rd.max()
            starts[i].record(ctx.stream)
            launch(i)
            ends[i].record(ctx.stream)
        torch.cuda.synchronize(ctx.dev)
        ctx.barrier()
    torch.cuda.nvtx.range_pop()
    total_ms = ctx.max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)))
    return total_ms, clocks.summary()


def e2e_loop(ctx: Ctx, buf, steps: int, policy: str = "uniform", total_envs: int | None = None
             ) -> tuple[float, int, int, str]:
    """The public host-side API with host buffers: per step the actions
    (int64[B], page-locked host memory) cross to the device, the fused step
    runs, and reward, done and the next proposed actions cross back into
    page-locked host memory; the host takes the proposals as its next actions.
    By default (``--e2e-api step_host``) every step is one ``step_host`` call
    (the kernel reads / writes the page-locked memory in place, CUDA events
    around the loop).  ``--e2e-api serve`` runs uniform steps through the
    persistent step server instead (``StrategoRolloutBuffer.serve``: no launch
    or stream synchronisation per step, CUDA events around the server
    kernel's whole life).  Returns (updates/s, h2d, d2h bytes, api)."""
    from ataraxos_b200.serve import StepServer

    B = buf.n_games
    total = ctx.world * B if total_envs is None else total_envs
    r = buf.step_host(None, policy=policy)
    # untimed warm-up of the same host loop for about half a second (the
    # host round trips of a process that has just started run slower)
    h_act = torch.empty(B, dtype=torch.int64, pin_memory=True)
    t_end, i = time.perf_counter() + 0.5, 0
    while i < ctx.args.warmup or time.perf_counter() < t_end:
        h_act.copy_(r.next_action)
        r = buf.step_host(h_act, policy=policy)
        i += 1
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ctx.args.e2e_api == "serve" and policy == "uniform" and B <= StepServer.max_envs(buf.device):
        st = torch.cuda.Stream(ctx.dev)
        e0.record(st)
        with StepServer(buf, stream=st) as srv:
            acts = srv.actions
            acts.copy_(r.next_action)
            for _ in range(steps):
                r = srv.step(acts)
                acts.copy_(r.next_action)
        e1.record(st)
        api = "StrategoRolloutBuffer.serve().step (persistent step server)"
    else:
        e0.record(ctx.stream)
        for _ in range(steps):
            h_act.copy_(r.next_action)
            r = buf.step_host(h_act, policy=policy)
        e1.record(ctx.stream)
        api = "StrategoRolloutBuffer.step_host"
    torch.cuda.synchronize(ctx.dev)
    ctx.barrier()
    ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    return total * steps / (ms / 1e3), B * 8, int(r.reward.numel() * 4 + r.next_action.numel() * 2
                                                  + r.done.numel()), api


def run_step_config(ctx: Ctx, cfg: int) -> dict:
    """Configs 2 (4096 envs/GPU, uniform) and 3 (262144 envs split over the GPUs, Gumbel-max
    over virtual N(0,1) logits, 1M-entry pool): one fused-kernel ply per step."""
    from ataraxos_b200 import StrategoRolloutBuffer

    a = ctx.args
    if cfg == 2:
        B, pool, policy, env_base = a.envs, POOL, "uniform", ctx.rank * a.envs
    else:
        total = a.envs if a.envs != 4096 else 262144
        env_base, B = sharding.shard_range(total, ctx.world, ctx.rank)
        pool, policy = 1 << 20, "gumbel"
    buf = StrategoRolloutBuffer(B, ctx.local, seed=SEED, env_base=env_base, pool_size=pool, pool_seed=SEED,
                                obs_dtype=torch.bfloat16, obs_layout="dense", mask_format="u8")
    buf.reset_all_from_pool()
    graph = cfg == 2 and a.timing == "graph"
    # config 2 under graph timing: the steps write 4 output sets in turn (see the module docstring)
    sets = [buf._ensure_outputs()] + [buf.new_outputs() for _ in range(3)] if graph else [None]

    def launch(i):
        buf.step(None, policy=policy, outputs=sets[i % len(sets)])

    for i in range(a.warmup):
        launch(i)
    if graph:
        total_ms, clocks = timed_graph(ctx, launch, a.warmup, a.steps)
    else:
        flush = a.flush_mib if cfg == 2 else 0  # config 3 writes 6.7 GB/GPU per step: far above L2
        total_ms, clocks = timed_launches(ctx, launch, a.steps, flush)
    launch_ms = total_ms / a.steps
    stats = ctx.gather_stats(buf.episode_stats().clone())
    if cfg == 2:
        e2e, h2d, d2h, api = e2e_loop(ctx, buf, a.e2e_steps)
        workload = (f"config2: {B} envs/GPU, seeded random setups (pool {pool}), uniform random legal actions, "
                    "auto-reset, bf16 [B,488,10,10] infostate (75 live planes rewritten per ply), u8 [B,100,100] "
                    "mask; one step = one fused-kernel ply over all envs")
        if graph:
            l2 = ("back-to-back steps (one CUDA graph of the K timed launches); outputs written to 4 sets in turn "
                  "(4 x 441 MB, 14x L2): no step rewrites lines held in L2, every step's writes reach HBM in the "
                  "timed region")
        else:
            l2 = f"flushed between timed steps ({a.flush_mib} MiB write, then {a.flush_mib // 2} MiB read)"
        scaling = "weak"
    else:
        e2e, h2d, d2h, api = e2e_loop(ctx, buf, max(10, a.e2e_steps // 10), policy, total)
        workload = (f"config3: {total} envs split over {ctx.world} GPU(s) ({B}/GPU), actions by Gumbel-max "
                    "over virtual Philox N(0,1) logits of the legal moves (logits never materialised), setups from "
                    f"a {pool}-entry pool, auto-reset, bf16 dense infostate + u8 mask")
        l2 = "outputs of one step (25.5 KB/env) exceed L2 many times; no flush"
        scaling = "strong"
    return {
        "value": (ctx.world * B if cfg == 2 else total) * a.steps / (total_ms / 1e3), "ms_per_step": launch_ms,
        "launch_ms": launch_ms,
        "envs_per_launch": B, "plies_per_launch": 1, "bytes_per_update": BYTES_PER_UPDATE, "clocks": clocks,
        "stats": stats, "e2e": {"value": e2e, "unit": "updates/s", "h2d_bytes_per_step": h2d,
                                "d2h_bytes_per_step": d2h, "api": api},
        "gpu_launches": a.steps, "config": {"workload": workload, "envs_per_gpu": B, "l2": l2,
                                            "parallelism": f"env-sharded x{ctx.world}, no step-path collective"},
        "scaling": scaling,
        "traffic": _profile_traffic("step_kernel_config2.txt") if cfg == 2 else _profile_traffic("step_kernel_config3.txt", B),
    }


def run_traj_config(ctx: Ctx) -> dict:
    """Config 4: 32768 envs/GPU, T=128 ring of compact bf16 infostate, bit-packed masks,
    int16 actions, f32 log-probs (Gumbel over virtual N(0,1) logits), f32 rewards, u8 dones.
    One timed launch = `plies_per_launch` plies with every record kept on chip."""
    from ataraxos_b200 import StrategoRolloutBuffer
    from ataraxos_b200.trajectory import TrajectoryBuffer

    a = ctx.args
    B = a.envs if a.envs != 4096 else 32768
    T, R = a.ring_slots, a.plies_per_launch
    if T <= R:
        raise SystemExit("--ring-slots must exceed --plies-per-launch")
    buf = StrategoRolloutBuffer(B, ctx.local, seed=SEED, env_base=ctx.rank * B, pool_size=POOL, pool_seed=SEED)
    buf.reset_all_from_pool()
    tr = TrajectoryBuffer(buf, T, policy="gumbel")
    tr.prime()
    for _ in range(a.warmup):
        tr.rollout(R)
    total_ms, clocks = timed_launches(ctx, lambda i: tr.rollout(R), a.steps, 0)
    stats = ctx.gather_stats(tr.stats.clone())
    # e2e: each launch is followed by a device->host read of the last ply's rewards and dones
    h_rew = torch.empty(B, dtype=torch.float32, pin_memory=True)
    h_done = torch.empty(B, dtype=torch.uint8, pin_memory=True)
    steps = max(5, a.steps // 4)
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ctx.stream)
    for _ in range(steps):
        tr.rollout(R)
        last = (tr.slot - 1) % T
        h_rew.copy_(tr.reward[last], non_blocking=True)
        h_done.copy_(tr.done[last], non_blocking=True)
        ctx.stream.synchronize()
    e1.record(ctx.stream)
    torch.cuda.synchronize(ctx.dev)
    e2e_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    bpu = 15_000 + 1_250 + 2 + 4 + 4 + 1 + 512 / R
    return {
        "value": ctx.world * B * R * a.steps / (total_ms / 1e3), "ms_per_step": total_ms / a.steps,
        "launch_ms": total_ms / a.steps, "envs_per_launch": B, "plies_per_launch": R, "bytes_per_update": bpu,
        "clocks": clocks, "stats": stats,
        "e2e": {"value": ctx.world * B * R * steps / (e2e_ms / 1e3), "unit": "updates/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": B * 5},
        "gpu_launches": a.steps,
        "config": {"workload": f"config4: {B} envs/GPU, T={T} ring (compact bf16 [76,10,10] infostate, bit-packed "
                               f"mask, i16 action, f32 log-prob from virtual N(0,1) logits, f32 reward, u8 done); "
                               f"{R} plies per launch", "envs_per_gpu": B,
                   "l2": f"ring of {T} slots ({T * B * 16.5 / 1e9:.0f} GB) far above L2; no flush",
                   "parallelism": f"env-sharded x{ctx.world}, no step-path collective"},
        "scaling": "weak", "traffic": _profile_traffic("rollout_kernel_config4.txt", B * R),
    }


def run_search_config(ctx: Ctx) -> dict:
    """Config 5: 64 roots/GPU advanced 150 random plies, 1000 belief samples each
    (64,000 envs), 40-ply rollouts in one launch; bit-packed legal masks per ply
    and terminal values per rollout."""
    from ataraxos_b200 import StrategoRolloutBuffer
    from ataraxos_b200.trajectory import BeliefRollouts

    a = ctx.args
    n_roots, k, depth = 64, a.samples, 40
    roots = StrategoRolloutBuffer(n_roots, ctx.local, seed=SEED, env_base=ctx.rank * n_roots, pool_size=POOL,
                                  pool_seed=SEED)
    roots.reset_all_from_pool()
    for _ in range(150):
        roots.step(None)
    br = BeliefRollouts(roots, k, depth, seed=SEED + 1 + ctx.rank, policy="uniform")
    br.samples.env_base = ctx.rank * n_roots * k
    br.samples._st = br.samples._make_state()
    for _ in range(a.warmup):
        br.run()

    def one(i):
        br.run()

    total_ms, clocks = timed_launches(ctx, one, a.steps, 0)
    n = n_roots * k
    h_val = torch.empty(n, dtype=torch.float32, pin_memory=True)
    steps = max(3, a.steps // 4)
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ctx.stream)
    for _ in range(steps):
        out = br.run()
        h_val.copy_(out["terminal_value"], non_blocking=True)
        ctx.stream.synchronize()
    e1.record(ctx.stream)
    torch.cuda.synchronize(ctx.dev)
    e2e_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    return {
        "value": ctx.world * n * depth * a.steps / (total_ms / 1e3), "ms_per_step": total_ms / a.steps,
        "launch_ms": total_ms / a.steps, "envs_per_launch": n, "plies_per_launch": depth,
        "bytes_per_update": 1250 + 2 + 4 + 4 + 1 + 512 / depth, "clocks": clocks,
        "stats": [0, 0, 0, 0, 0],
        "e2e": {"value": ctx.world * n * depth * steps / (e2e_ms / 1e3), "unit": "updates/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": n * 4},
        "gpu_launches": 3 * a.steps,
        "config": {"workload": f"config5: {n_roots} roots/GPU (seeded setups + 150 random plies) x {k} belief samples, "
                               f"{depth}-ply uniform rollouts in one launch; per-ply bit-packed masks, terminal values; "
                               "one step = resample + prime + rollout", "envs_per_gpu": n,
                   "l2": "n/a: per-launch outputs 3.2 GB/GPU", "parallelism": f"root-sharded x{ctx.world}"},
        "scaling": "weak", "traffic": _profile_traffic("search_kernels_config5.txt", n * depth),
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference", "reference-cuda"], default="b200")
    ap.add_argument("--config", type=int, choices=[2, 3, 4, 5], default=2)
    ap.add_argument("--envs", type=int, default=4096, help="envs per GPU (config 2)")
    ap.add_argument("--plies-per-launch", type=int, default=8, help="config 4 rollout launch length")
    ap.add_argument("--ring-slots", type=int, default=128, help="config 4 ring length T (smaller: profiling cases)")
    ap.add_argument("--samples", type=int, default=1000, help="config 5 belief samples per root")
    ap.add_argument("--e2e-steps", type=int, default=500)
    ap.add_argument("--e2e-api", choices=["serve", "step_host"], default="step_host",
                    help="host API of the e2e loop: the persistent step server or step_host")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--flush-mib", type=int, default=512)
    ap.add_argument("--timing", choices=["graph", "flush"], default="graph",
                    help="config 2: K back-to-back steps as one CUDA graph over 4 output sets, or per-launch events "
                         "with an L2 flush between launches")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {2: 3000, 3: 100, 4: 40, 5: 10}[args.config]
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args, int(os.environ.get("RANK", "0")))
        return
    if args.impl == "reference-cuda":
        run_reference_cuda(args, int(os.environ.get("RANK", "0")))
        return

    ctx = Ctx(args)
    if args.config in (2, 3):
        r = run_step_config(ctx, args.config)
    elif args.config == 4:
        r = run_traj_config(ctx)
    else:
        r = run_search_config(ctx)

    if ctx.rank == 0:
        peak, peak_kind = _peaks()
        achieved = r["bytes_per_update"] * r["envs_per_launch"] * r["plies_per_launch"] / (r["launch_ms"] / 1e3) / 1e9
        line = {
            "metric": METRIC,
            "value": r["value"],
            "unit": "updates/s",
            "n_gpus": ctx.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": r["ms_per_step"],
            "higher_is_better": True,
            "scaling": r["scaling"],
            "vs_baseline": None,
            "dtype": "u8/int32 state, bf16 infostate",
            "data": "synthetic (Philox setups and actions, no dataset)",
            "config": r["config"],
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": r["traffic"],
                "bytes_per_update": r["bytes_per_update"],
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "kernel": "env_kernel (fused step)",
            },
            "e2e": r["e2e"],
            "gpu_launches": r["gpu_launches"],
            "clocks": r["clocks"],
            "episode_stats": dict(zip(["finished", "red_wins", "blue_wins", "draws", "sum_lengths"], r["stats"])),
        }
        if ctx.world == 1 and not args.no_cpu_baseline and args.config == 2:
            line["cpu_baseline"] = cpu_baseline(args.envs)
        print(json.dumps(line), flush=True)
    if ctx.world > 1:
        ctx.dist.destroy_process_group()


if __name__ == "__main__":
    main()
