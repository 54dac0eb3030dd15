"""Benchmark of the B200 StrategoRolloutBuffer hot path.

Metric: env state updates per second, one update = one ply of one env (sample a
uniform legal action, apply it with combat / trackers / terminal check,
auto-reset from the seeded setup pool, emit the uint8 legal mask and the
bfloat16 [488,10,10] infostate of the new state).

Default workload = benchmark config 2: 4096 envs per GPU, seeded random setups
(pool of 65536), uniform random legal actions, auto-reset, bf16 infostate
[B,488,10,10] (channels 43-455 are zero planes written once at allocation;
every ply rewrites the 75 live channels), uint8 mask [B,100,100].  One step =
one ply over all envs.  The GPU's envs form ``--groups`` groups (default 3 for
config 2, 2 for config 3): contiguous global env ranges, each a buffer stepped
on its own CUDA stream, so one step is one fused-step launch per group and the
groups' launches run concurrently (one launch's ramp and drain overlap the
others' work).  Every random stream is keyed by the global env index, so the
games are the same for any number of groups.  Synthetic data: there is no
dataset; setups and actions come from Philox.

Timing (config 2, default ``--timing graph``): W untimed warm-up steps, then
the K timed steps, launched back to back as one CUDA graph (captured after the
warm-up; each group's launches a chain on its own stream, each node with its
own ply number, and two CUDA events recorded in the graph on the stream the
chains fork from and join, before the fork and after the join), uploaded to
the device, and replayed once; barrier + synchronize on both sides; max over
ranks.  Each group writes its outputs into 4 output sets
in turn (4 x 441 MB in all, 14x the 126 MB L2), so no step writes lines still
held in L2 and every step's 104.6 MB of writes reaches HBM inside the timed
region (the game records, 1 MB, stay in L2 from ply to ply, as in any
rollout).  ``--timing flush`` (one group only) is the per-launch form: each
step bracketed by its own events, with a 512 MiB write and a 256 MiB read
between steps (outside the bracketed interval) to flush L2.  Config 3 (6.7 GB
written per step) launches the groups' chains from the host between two
events.
Multi-GPU (torchrun): each rank owns its own 4096 envs (global env indices
rank*4096 ...), no collective on the step path (weak scaling); an NCCL
all-gather of the episode statistics follows the timed region.

e2e: the same games through the public host API with host buffers: int64
actions from page-locked host memory in, reward / done / next action back into
page-locked memory every step, the host playing the proposals it received.
Default ``--e2e-api pipeline``: ``ataraxos_b200.pipeline.StepPipeline`` with
``--e2e-groups`` groups received and re-sent in turn (each group's ply one
``sb_step_host`` call); ``step_host``: one synchronous call per step over all
envs; ``serve``: the persistent step server.  CUDA events around the loop.

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
    """DRAM bytes (read + write) per step from the ncu capture summarised in
    profiles/<name>: its dram_bytes_per_step (config 2: the step's launches,
    one per group), or, for a capture taken on a smaller case, its
    dram_bytes_per_update times the updates of the step."""
    f = ROOT / "profiles" / name
    try:
        for line in f.read_text().splitlines():
            if line.startswith("dram_bytes_per_step:") and updates_per_launch is None:
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


def fork(main: torch.cuda.Stream, streams) -> None:
    """Every stream in ``streams`` waits for the work queued on ``main`` so far."""
    ev = torch.cuda.Event()
    ev.record(main)
    for s in streams:
        s.wait_event(ev)


def join(main: torch.cuda.Stream, streams) -> None:
    """``main`` waits for the work queued on every stream in ``streams`` so far."""
    for s in streams:
        ev = torch.cuda.Event()
        ev.record(s)
        main.wait_event(ev)


class Groups:
    """The rank's games as ``G`` buffers (contiguous global env ranges), each
    stepped on its own CUDA stream, so the groups' launches run concurrently:
    one group's launch ramp and drain overlap the others' work.  Every random
    stream is keyed by the global env index, so the games play exactly as in
    one buffer of all of them; one step = one ply of every game = one launch
    per group."""

    def __init__(self, ctx: Ctx, B: int, env_base: int, G: int, n_sets: int, **buf_kw) -> None:
        from ataraxos_b200 import StrategoRolloutBuffer

        if not 1 <= G <= B:
            raise SystemExit(f"--groups must be in 1..{B}")
        self.parts = []
        for g in range(G):
            off, n = sharding.shard_range(B, G, g)
            s = torch.cuda.Stream(ctx.dev)
            with torch.cuda.stream(s):
                b = StrategoRolloutBuffer(n, ctx.local, env_base=env_base + off, **buf_kw)
                b.reset_all_from_pool()
                sets = [b._ensure_outputs()] + [b.new_outputs() for _ in range(n_sets - 1)] if n_sets > 1 else [None]
            self.parts.append((b, s, sets))
        torch.cuda.synchronize(ctx.dev)

    def step(self, i: int, policy: str) -> None:
        for b, s, sets in self.parts:
            with torch.cuda.stream(s):
                b.step(None, policy=policy, outputs=sets[i % len(sets)])

    def fork(self, main: torch.cuda.Stream) -> None:
        fork(main, [s for _, s, _ in self.parts])

    def join(self, main: torch.cuda.Stream) -> None:
        join(main, [s for _, s, _ in self.parts])

    def stats(self) -> torch.Tensor:
        return sum(b.episode_stats().clone() for b, _, _ in self.parts)

    def status(self) -> int:
        st = 0
        for b, _, _ in self.parts:
            st |= int(b.status())
        return st


def _graph_upload(graph: torch.cuda.CUDAGraph, stream: torch.cuda.Stream) -> bool:
    """Upload an instantiated graph to the device before its first launch
    (cuGraphUpload), so the timed launch does not pay for it.  False (and the
    graph is uploaded by its first launch instead) if the driver call is not
    available or fails."""
    import ctypes

    try:
        cu = ctypes.CDLL("libcuda.so.1")
        rc = cu.cuGraphUpload(ctypes.c_void_p(graph.raw_cuda_graph_exec()), ctypes.c_void_p(stream.cuda_stream))
    except (OSError, AttributeError):
        return False
    stream.synchronize()
    return rc == 0


def timed_graph(ctx: Ctx, groups: Groups, first: int, k: int, policy: str):
    """Steps first .. first + k - 1 of every group captured into one CUDA graph
    (each group's launches a chain on its own stream, forked from and joined
    to one stream, with a CUDA event recorded on that stream before the fork
    and after the join), uploaded, then replayed once (no host work between
    steps)."""
    main = torch.cuda.Stream(ctx.dev)
    g = torch.cuda.CUDAGraph()
    # the timing events are nodes of the graph (external events): they bracket
    # the K steps on the device, not the host's launch of the graph
    e0, e1 = torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True)
    with torch.cuda.graph(g, stream=main):
        e0.record(main)
        groups.fork(main)
        for i in range(first, first + k):
            groups.step(i, policy)
        groups.join(main)
        e1.record(main)
    torch.cuda.synchronize(ctx.dev)
    _graph_upload(g, main)
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    # for the record: the same replay bracketed by events the host records
    # around its launch of the graph (includes the graph's launch latency)
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    with ClockSampler(ctx.dev) as clocks:
        with torch.cuda.stream(main):
            h0.record(main)
            g.replay()
            h1.record(main)
        torch.cuda.synchronize(ctx.dev)
        ctx.barrier()
    torch.cuda.nvtx.range_pop()
    total_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    host_ms = ctx.max_over_ranks(h0.elapsed_time(h1))
    del g
    return total_ms, clocks.summary(), host_ms


def timed_streams(ctx: Ctx, groups: Groups, first: int, k: int, policy: str):
    """k steps of every group launched from the host (each group's chain on
    its own stream), forked from and joined to one stream whose CUDA events
    bracket the whole interval."""
    main = torch.cuda.Stream(ctx.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    torch.cuda.nvtx.range_push("timed")
    with ClockSampler(ctx.dev) as clocks:
        e0.record(main)
        groups.fork(main)
        for i in range(first, first + k):
            groups.step(i, policy)
        groups.join(main)
        e1.record(main)
        torch.cuda.synchronize(ctx.dev)
        ctx.barrier()
    torch.cuda.nvtx.range_pop()
    return ctx.max_over_ranks(e0.elapsed_time(e1)), clocks.summary()


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


def e2e_loop(ctx: Ctx, B: int, env_base: int, buf_kw: dict, steps: int, policy: str, total: int
             ) -> tuple[float, int, int, str]:
    """The public host-side API with host buffers, on the same games as the
    device-timed steps (same global env indices, seed and pool): per step every
    game's int64 action crosses from page-locked host memory to the device, the
    fused ply runs, and reward, done and the next proposed action cross back
    into page-locked host memory; the host takes the proposals as its next
    actions, so a game's ply waits on the host for its previous ply.

    ``--e2e-api pipeline`` (default): ``StepPipeline`` with ``--e2e-groups``
    groups; per step every group is received and re-sent in turn, so one
    group's host round trip overlaps the other groups' plies.  ``step_host``:
    one synchronous ``StrategoRolloutBuffer.step_host`` call per step (the
    kernel reads / writes the page-locked memory in place).  ``serve``: uniform
    steps through the persistent step server.  CUDA events around the loop.
    Returns (updates/s, h2d, d2h bytes per step, api)."""
    from ataraxos_b200 import StrategoRolloutBuffer
    from ataraxos_b200.pipeline import StepPipeline
    from ataraxos_b200.serve import StepServer

    a = ctx.args
    api = a.e2e_api
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if api == "pipeline":
        G = a.e2e_groups
        p = StepPipeline(B, ctx.local, groups=G, env_base=env_base, **buf_kw)
        p.reset_all_from_pool()
        for g in range(G):
            p.send(g, None, policy=policy)

        def loop(k: int) -> None:
            for _ in range(k):
                for g in range(G):
                    r = p.recv(g)
                    p.send(g, r.next_action, policy=policy)

        # untimed warm-up of the same host loop for about half a second (the
        # host round trips of a process that has just started run slower)
        t_end = time.perf_counter() + 0.5
        while time.perf_counter() < t_end:
            loop(a.warmup)
        p.synchronize()
        ctx.barrier()
        torch.cuda.synchronize(ctx.dev)
        e0.record(ctx.stream)
        loop(steps)
        p.synchronize()
        e1.record(ctx.stream)
        for g in range(G):
            p.recv(g)
        name = f"ataraxos_b200.pipeline.StepPipeline ({G} groups; each group's ply one sb_step_host call)"
    else:
        buf = StrategoRolloutBuffer(B, ctx.local, env_base=env_base, **buf_kw)
        buf.reset_all_from_pool()
        r = buf.step_host(None, policy=policy)
        h_act = torch.empty(B, dtype=torch.int64, pin_memory=True)
        t_end, i = time.perf_counter() + 0.5, 0
        while i < a.warmup or time.perf_counter() < t_end:
            h_act.copy_(r.next_action)
            r = buf.step_host(h_act, policy=policy)
            i += 1
        ctx.barrier()
        torch.cuda.synchronize(ctx.dev)
        if api == "serve" and policy == "uniform" and B <= StepServer.max_envs(buf.device):
            st = torch.cuda.Stream(ctx.dev)
            e0.record(st)
            with StepServer(buf, stream=st) as srv:
                acts = srv.actions
                acts.copy_(r.next_action)
                for _ in range(steps):
                    r = srv.step(acts)
                    acts.copy_(r.next_action)
            e1.record(st)
            name = "StrategoRolloutBuffer.serve().step (persistent step server)"
        else:
            e0.record(ctx.stream)
            for _ in range(steps):
                h_act.copy_(r.next_action)
                r = buf.step_host(h_act, policy=policy)
            e1.record(ctx.stream)
            name = "StrategoRolloutBuffer.step_host"
    torch.cuda.synchronize(ctx.dev)
    ctx.barrier()
    ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    # per game and step: the int64 action in; f32 reward, i16 next action, u8 done out
    return total * steps / (ms / 1e3), B * 8, B * (4 + 2 + 1), name


def run_step_config(ctx: Ctx, cfg: int) -> dict:
    """Configs 2 (4096 envs/GPU, uniform) and 3 (262144 envs split over the GPUs, Gumbel-max
    over virtual N(0,1) logits, 1M-entry pool): one fused-kernel ply per group per step."""
    a = ctx.args
    if cfg == 2:
        B, pool, policy, env_base = a.envs, POOL, "uniform", ctx.rank * a.envs
        total = ctx.world * B
    else:
        total = a.envs if a.envs != 4096 else 262144
        env_base, B = sharding.shard_range(total, ctx.world, ctx.rank)
        pool, policy = 1 << 20, "gumbel"
    G = a.groups if a.groups else (3 if cfg == 2 else 2)
    buf_kw = dict(seed=SEED, pool_size=pool, pool_seed=SEED, obs_dtype=torch.bfloat16, obs_layout="dense",
                  mask_format="u8")
    graph = cfg == 2 and a.timing == "graph"
    if cfg == 2 and a.timing == "flush" and G != 1:
        raise SystemExit("--timing flush times launches one by one: use --groups 1")
    # config 2 under graph timing: each group writes 4 output sets in turn (see the module docstring)
    groups = Groups(ctx, B, env_base, G, 4 if graph else 1, **buf_kw)
    for i in range(a.warmup):
        groups.step(i, policy)
    torch.cuda.synchronize(ctx.dev)
    host_ms = None
    if graph:
        total_ms, clocks, host_ms = timed_graph(ctx, groups, a.warmup, a.steps, policy)
    elif cfg == 2 and a.timing == "flush":
        buf, _, _ = groups.parts[0]
        total_ms, clocks = timed_launches(ctx, lambda i: buf.step(None, policy=policy), a.steps, a.flush_mib)
    else:
        # config 3 writes 6.7 GB per GPU per step: far above L2, no flush
        total_ms, clocks = timed_streams(ctx, groups, a.warmup, a.steps, policy)
    if groups.status():
        raise SystemExit(f"device status {groups.status():#x} after the timed steps")
    stats = ctx.gather_stats(groups.stats())
    del groups
    torch.cuda.synchronize(ctx.dev)
    torch.cuda.empty_cache()
    step_ms = total_ms / a.steps
    e2e_steps = a.e2e_steps if cfg == 2 else max(10, a.e2e_steps // 10)
    e2e, h2d, d2h, api = e2e_loop(ctx, B, env_base, buf_kw, e2e_steps, policy, total)
    split = (f"{G} groups of ~{B // G} envs, each on its own CUDA stream (their launches run concurrently)"
             if G > 1 else "one launch per step")
    if cfg == 2:
        workload = (f"config2: {B} envs/GPU, seeded random setups (pool {pool}), uniform random legal actions, "
                    "auto-reset, bf16 [B,488,10,10] infostate (75 live planes rewritten per ply), u8 [B,100,100] "
                    f"mask; one step = one fused-kernel ply over all envs ({split})")
        if graph:
            l2 = ("back-to-back steps (one CUDA graph of the K timed steps); each group writes 4 output sets in turn "
                  "(4 x 441 MB in all, 14x L2): no step rewrites lines held in L2, every step's writes reach HBM in "
                  "the timed region")
        else:
            l2 = f"flushed between timed steps ({a.flush_mib} MiB write, then {a.flush_mib // 2} MiB read)"
        scaling = "weak"
    else:
        workload = (f"config3: {total} envs split over {ctx.world} GPU(s) ({B}/GPU), actions by Gumbel-max "
                    "over virtual Philox N(0,1) logits of the legal moves (logits never materialised), setups from "
                    f"a {pool}-entry pool, auto-reset, bf16 dense infostate + u8 mask; one step = one ply of "
                    f"every env ({split})")
        l2 = "outputs of one step (25.5 KB/env) exceed L2 many times; no flush"
        scaling = "strong"
    return {
        "value": (ctx.world * B if cfg == 2 else total) * a.steps / (total_ms / 1e3), "ms_per_step": step_ms,
        "launch_ms": step_ms, "host_ms_per_step": None if host_ms is None else host_ms / a.steps,
        "envs_per_launch": B, "plies_per_launch": 1, "bytes_per_update": BYTES_PER_UPDATE, "clocks": clocks,
        "stats": stats, "e2e": {"value": e2e, "unit": "updates/s", "h2d_bytes_per_step": h2d,
                                "d2h_bytes_per_step": d2h, "api": api},
        "gpu_launches": a.steps * G, "config": {"workload": workload, "envs_per_gpu": B, "groups": G, "l2": l2,
                                                "parallelism": f"env-sharded x{ctx.world}, no step-path collective"},
        "scaling": scaling,
        "kernel": ("env_kernel (fused step)" if G == 1 else
                   f"env_kernel (fused step), {G} concurrent launches per step (one per group): achieved = the "
                   "step's algorithmic bytes / the step's time"),
        "traffic": _profile_traffic("step_kernel_config2.txt") if cfg == 2 else _profile_traffic("step_kernel_config3.txt", B),
    }


def run_traj_config(ctx: Ctx) -> dict:
    """Config 4: 32768 envs/GPU, T=128 ring of compact bf16 infostate, bit-packed masks,
    int16 actions, f32 log-probs (Gumbel over virtual N(0,1) logits), f32 rewards, u8 dones.
    One step = `plies_per_launch` plies of every env: one launch per group (the
    GPU's envs as ``--groups`` buffers, each with its own ring and stream, the
    launches running concurrently), every record kept on chip in the launch."""
    from ataraxos_b200 import StrategoRolloutBuffer
    from ataraxos_b200.trajectory import TrajectoryBuffer

    a = ctx.args
    B = a.envs if a.envs != 4096 else 32768
    T, R = a.ring_slots, a.plies_per_launch
    G = a.groups if a.groups else 2
    if T <= R:
        raise SystemExit("--ring-slots must exceed --plies-per-launch")
    if not 1 <= G <= B:
        raise SystemExit(f"--groups must be in 1..{B}")
    parts = []
    for g in range(G):
        off, n = sharding.shard_range(B, G, g)
        s = torch.cuda.Stream(ctx.dev)
        with torch.cuda.stream(s):
            buf = StrategoRolloutBuffer(n, ctx.local, seed=SEED, env_base=ctx.rank * B + off, pool_size=POOL,
                                        pool_seed=SEED)
            buf.reset_all_from_pool()
            tr = TrajectoryBuffer(buf, T, policy="gumbel")
            tr.prime()
        parts.append((tr, s, off, n))

    def step() -> None:
        for tr, s, _, _ in parts:
            with torch.cuda.stream(s):
                tr.rollout(R)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize(ctx.dev)
    main = torch.cuda.Stream(ctx.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    streams = [s for _, s, _, _ in parts]
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    torch.cuda.nvtx.range_push("timed")
    with ClockSampler(ctx.dev) as clocks:
        e0.record(main)
        fork(main, streams)
        for _ in range(a.steps):
            step()
        join(main, streams)
        e1.record(main)
        torch.cuda.synchronize(ctx.dev)
        ctx.barrier()
    torch.cuda.nvtx.range_pop()
    total_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    stats = ctx.gather_stats(sum(tr.stats.clone() for tr, _, _, _ in parts))
    # e2e: each step (every group's launch) is followed by a device->host read of
    # the last ply's rewards and dones of every env, then the host waits for them
    h_rew = torch.empty(B, dtype=torch.float32, pin_memory=True)
    h_done = torch.empty(B, dtype=torch.uint8, pin_memory=True)
    steps = max(5, a.steps // 4)
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    e0.record(main)
    fork(main, streams)
    for _ in range(steps):
        for tr, s, off, n in parts:
            with torch.cuda.stream(s):
                tr.rollout(R)
                last = (tr.slot - 1) % T
                h_rew[off:off + n].copy_(tr.reward[last], non_blocking=True)
                h_done[off:off + n].copy_(tr.done[last], non_blocking=True)
        for s in streams:
            s.synchronize()
    join(main, streams)
    e1.record(main)
    torch.cuda.synchronize(ctx.dev)
    e2e_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    bpu = 15_000 + 1_250 + 2 + 4 + 4 + 1 + 512 / R
    split = (f"{G} groups of ~{B // G} envs, each with its own ring and CUDA stream (their launches run "
             "concurrently)" if G > 1 else "one launch per step")
    return {
        "value": ctx.world * B * R * a.steps / (total_ms / 1e3), "ms_per_step": total_ms / a.steps,
        "launch_ms": total_ms / a.steps, "envs_per_launch": B, "plies_per_launch": R, "bytes_per_update": bpu,
        "clocks": clocks.summary(), "stats": stats,
        "e2e": {"value": ctx.world * B * R * steps / (e2e_ms / 1e3), "unit": "updates/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": B * 5},
        "gpu_launches": a.steps * G,
        "config": {"workload": f"config4: {B} envs/GPU, T={T} ring (compact bf16 [76,10,10] infostate, bit-packed "
                               f"mask, i16 action, f32 log-prob from virtual N(0,1) logits, f32 reward, u8 done); "
                               f"one step = {R} plies of every env ({split})", "envs_per_gpu": B, "groups": G,
                   "l2": f"ring of {T} slots ({T * B * 16.5 / 1e9:.0f} GB) far above L2; no flush",
                   "parallelism": f"env-sharded x{ctx.world}, no step-path collective"},
        "scaling": "weak", "traffic": _profile_traffic("rollout_kernel_config4.txt", B * R),
        "kernel": ("env_kernel (rollout)" if G == 1 else
                   f"env_kernel (rollout), {G} concurrent launches per step (one per group): achieved = the "
                   "step's algorithmic bytes / the step's time"),
    }


def run_search_config(ctx: Ctx) -> dict:
    """Config 5: 64 roots/GPU advanced 150 random plies, 1000 belief samples each
    (64,000 envs), 40-ply rollouts in one launch; bit-packed legal masks per ply
    and terminal values per rollout.  The roots form ``--groups`` groups, each
    with its own sample buffer and CUDA stream (their launches run
    concurrently); one step = resample + prime + rollout of every group."""
    from ataraxos_b200 import StrategoRolloutBuffer
    from ataraxos_b200.trajectory import BeliefRollouts

    a = ctx.args
    n_roots, k, depth = 64, a.samples, 40
    G = a.groups if a.groups else 2
    if not 1 <= G <= n_roots:
        raise SystemExit(f"--groups must be in 1..{n_roots}")
    parts = []
    for g in range(G):
        off, nr = sharding.shard_range(n_roots, G, g)
        s = torch.cuda.Stream(ctx.dev)
        with torch.cuda.stream(s):
            roots = StrategoRolloutBuffer(nr, ctx.local, seed=SEED, env_base=ctx.rank * n_roots + off,
                                          pool_size=POOL, pool_seed=SEED)
            roots.reset_all_from_pool()
            for _ in range(150):
                roots.step(None)
            br = BeliefRollouts(roots, k, depth, seed=SEED + 1 + ctx.rank, policy="uniform")
            br.samples.env_base = (ctx.rank * n_roots + off) * k
            br.samples._st = br.samples._make_state()
        parts.append((br, s, off * k, nr * k))

    def step(outs=None) -> None:
        for br, s, _, _ in parts:
            with torch.cuda.stream(s):
                o = br.run()
                if outs is not None:
                    outs.append(o)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize(ctx.dev)
    main = torch.cuda.Stream(ctx.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    streams = [s for _, s, _, _ in parts]
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    torch.cuda.nvtx.range_push("timed")
    with ClockSampler(ctx.dev) as clocks:
        e0.record(main)
        fork(main, streams)
        for _ in range(a.steps):
            step()
        join(main, streams)
        e1.record(main)
        torch.cuda.synchronize(ctx.dev)
        ctx.barrier()
    torch.cuda.nvtx.range_pop()
    total_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    n = n_roots * k
    h_val = torch.empty(n, dtype=torch.float32, pin_memory=True)
    steps = max(3, a.steps // 4)
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    e0.record(main)
    fork(main, streams)
    for _ in range(steps):
        for br, s, off, m in parts:
            with torch.cuda.stream(s):
                out = br.run()
                h_val[off:off + m].copy_(out["terminal_value"], non_blocking=True)
        for s in streams:
            s.synchronize()
    join(main, streams)
    e1.record(main)
    torch.cuda.synchronize(ctx.dev)
    e2e_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    split = (f"{G} groups of ~{n_roots // G} roots, each with its own samples and CUDA stream (their launches run "
             "concurrently)" if G > 1 else "one launch of each kernel per step")
    return {
        "value": ctx.world * n * depth * a.steps / (total_ms / 1e3), "ms_per_step": total_ms / a.steps,
        "launch_ms": total_ms / a.steps, "envs_per_launch": n, "plies_per_launch": depth,
        "bytes_per_update": 1250 + 2 + 4 + 4 + 1 + 512 / depth, "clocks": clocks.summary(),
        "stats": [0, 0, 0, 0, 0],
        "e2e": {"value": ctx.world * n * depth * steps / (e2e_ms / 1e3), "unit": "updates/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": n * 4},
        "gpu_launches": 3 * a.steps * G,
        "config": {"workload": f"config5: {n_roots} roots/GPU (seeded setups + 150 random plies) x {k} belief samples, "
                               f"{depth}-ply uniform rollouts in one launch; per-ply bit-packed masks, terminal values; "
                               f"one step = resample + prime + rollout ({split})", "envs_per_gpu": n, "groups": G,
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
    ap.add_argument("--e2e-api", choices=["pipeline", "serve", "step_host"], default="pipeline",
                    help="host API of the e2e loop: groups stepped in turn (StepPipeline), the persistent step "
                         "server, or one synchronous step_host call per step")
    ap.add_argument("--e2e-groups", type=int, default=2, help="groups of the e2e pipeline")
    ap.add_argument("--groups", type=int, default=0,
                    help="the GPU's envs (config 5: roots) as this many concurrently stepped groups, one CUDA "
                         "stream each (0: 3 for config 2, 2 for configs 3-5)")
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
                "kernel": r.get("kernel", "env_kernel (fused step)"),
            },
            "e2e": r["e2e"],
            "gpu_launches": r["gpu_launches"],
            "timing": ("device span of the K steps: CUDA events recorded inside the CUDA graph, before the fork "
                       "and after the join of the groups' chains; ms_per_step_with_graph_launch: the same replay "
                       "bracketed by events the host records around its launch of the graph"
                       if r.get("host_ms_per_step") is not None else "CUDA events on the host-launched stream"),
            "clocks": r["clocks"],
            "episode_stats": dict(zip(["finished", "red_wins", "blue_wins", "draws", "sum_lengths"], r["stats"])),
        }
        if r.get("host_ms_per_step") is not None:
            line["ms_per_step_with_graph_launch"] = r["host_ms_per_step"]
        if ctx.world == 1 and not args.no_cpu_baseline and args.config == 2:
            line["cpu_baseline"] = cpu_baseline(args.envs)
        print(json.dumps(line), flush=True)
    if ctx.world > 1:
        ctx.dist.destroy_process_group()


if __name__ == "__main__":
    main()
