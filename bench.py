"""Benchmark of the B200 StrategoRolloutBuffer hot path.

Metric: env state updates per second, one update = one ply of one env (sample a
uniform legal action, apply it with combat / trackers / terminal check,
auto-reset from the seeded setup pool, emit the uint8 legal mask and the
bfloat16 [488,10,10] infostate of the new state).

Default workload = BASELINE config 2: 4096 envs per GPU, seeded random setups
(pool of 65536), uniform random legal actions, auto-reset, bf16 infostate
[B,488,10,10] (channels 43-455 are zero planes written once at allocation;
every ply rewrites the 75 live channels), uint8 mask [B,100,100].  One step =
one ply over all envs = one launch of the fused step kernel.  Synthetic data:
there is no dataset; setups and actions come from Philox.

Timing: W untimed warm-up steps; then K steps, each bracketed by CUDA events
on the buffer's stream, with a 512 MiB write and a 256 MiB read between timed
steps to flush the 126 MB L2 (outside the bracketed interval); barrier +
synchronize on both
sides; max over ranks.  Multi-GPU (torchrun): each rank owns its own 4096 envs
(global env indices rank*4096 ...), no collective on the step path (weak
scaling); an NCCL all-gather of the episode statistics follows the timed
region.

``--impl reference`` times the reference algorithm's CPU implementation on the
host cores: the C restatement in oracle/ (the reference's own code is Python
and cannot run on the GPU box), same config, a bounded sample of envs per step.
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
    envs = min(args.envs, 64 * threads)
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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--envs", type=int, default=4096, help="envs per GPU")
    ap.add_argument("--e2e-steps", type=int, default=500)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--flush-mib", type=int, default=512)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch.distributed as dist

    from ataraxos_b200 import StrategoRolloutBuffer

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    B = args.envs
    buf = StrategoRolloutBuffer(B, local, seed=SEED, env_base=rank * B, pool_size=POOL, pool_seed=SEED,
                                obs_dtype=torch.bfloat16, obs_layout="dense", mask_format="u8")
    buf.reset_all_from_pool()
    for _ in range(args.warmup):
        buf.step(None)
    # L2 flush between timed steps: write a buffer larger than the 126 MB L2,
    # then read another one, so the L2 holds only clean unrelated lines when
    # the timed step starts (its write-backs do not land inside the step).
    flush = torch.empty(args.flush_mib << 20, dtype=torch.uint8, device=dev)
    flush_rd = torch.ones((args.flush_mib << 20) // 8 // 2, dtype=torch.int64, device=dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stream = torch.cuda.current_stream(dev)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(dev) as clocks:
        for k in range(args.steps):
            flush.fill_(k & 0xFF)
            flush_rd.max()
            starts[k].record(stream)
            buf.step(None)
            ends[k].record(stream)
        torch.cuda.synchronize(dev)
        barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    value = world * B * args.steps / (total_ms / 1e3)
    launch_ms = total_ms / args.steps

    # end-of-rollout statistics: NCCL all-gather of int64[5] per rank (off the step path)
    stats = buf.episode_stats().clone()
    if world > 1:
        gathered = torch.empty((world, 5), dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(gathered, stats)
        stats_all = gathered.sum(0).tolist()
    else:
        stats_all = stats.tolist()

    # e2e through the public API with host buffers: each step copies the
    # actions (int64[B]) from pinned host memory to the device, runs the fused
    # step, and reads reward, done and the next proposed actions back into
    # pinned host memory (the host picks the next actions from them).
    h_act = torch.empty(B, dtype=torch.int64, pin_memory=True)
    h_rew = torch.empty(B, dtype=torch.float32, pin_memory=True)
    h_done = torch.empty(B, dtype=torch.uint8, pin_memory=True)
    h_next = torch.empty(B, dtype=torch.int16, pin_memory=True)
    out = buf.step(None)
    h_next.copy_(out.next_action)
    e2e_steps = args.e2e_steps
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        h_act.copy_(h_next)  # host-side policy: take the proposals
        out = buf.step(h_act)
        h_rew.copy_(out.reward, non_blocking=True)
        h_done.copy_(out.done.view(torch.uint8), non_blocking=True)
        h_next.copy_(out.next_action, non_blocking=True)
        stream.synchronize()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    e2e = world * B * e2e_steps / (e2e_ms / 1e3)

    if rank == 0:
        peak, peak_kind = _peaks()
        achieved = BYTES_PER_UPDATE * B / (launch_ms / 1e3) / 1e9
        traffic = None
        tf = ROOT / "profiles" / "step_kernel_traffic.json"
        if tf.exists():
            try:
                traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch_4096")
            except Exception:
                traffic = None
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "updates/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": launch_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "u8/int32 state, bf16 infostate",
            "data": "synthetic (Philox setups and actions, no dataset)",
            "config": {
                "workload": f"config2: {B} envs/GPU, seeded random setups (pool {POOL}), uniform random legal "
                            "actions, auto-reset, bf16 [B,488,10,10] infostate (75 live planes rewritten per ply), "
                            "u8 [B,100,100] mask; one step = one fused-kernel ply over all envs",
                "envs_per_gpu": B,
                "parallelism": f"env-sharded x{world}, no step-path collective",
                "l2": f"flushed between timed steps ({args.flush_mib} MiB write, then {args.flush_mib // 2} MiB read)",
            },
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "bytes_per_update": BYTES_PER_UPDATE,
                "peak_source": peak_kind,
            },
            "e2e": {
                "value": e2e,
                "unit": "updates/s",
                "h2d_bytes_per_step": B * 8,
                "d2h_bytes_per_step": B * (4 + 1 + 2),
                "steps": e2e_steps,
            },
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "episode_stats": dict(zip(["finished", "red_wins", "blue_wins", "draws", "sum_lengths"], stats_all)),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(B)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
