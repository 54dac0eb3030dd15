"""Generate tests/golden/refcuda.npz by running the reference's own CUDA kernels.

Needs a CUDA GPU and ``oracle/_ref/libref_stratego_cuda.so`` (the
reference's ``csrc/stratego_buffer.cu`` compiled from its source, see
``oracle/refcuda.py``); the reference checkout itself is not read here.

    python tests/golden/make_golden_refcuda.py [--out tests/golden/refcuda.npz]

Two action streams already committed as fixtures are replayed through
``oracle.refcuda.RefCudaBuffer`` (the reference pybind class restated over
its kernels, with the seed-42 Zobrist table injected):

* ``c1_*``: config 1 of the benchmark (tests/golden/config1.npz: 64 games
  from the seeded pool, 200 plies of uniform random legal actions).  Per
  snapshot (before the first ply and after each ply) the fields that only
  the reference CUDA class defines -- moved / revealed squares, the 32-move
  history ring, the per-mover two-square tracker, the chase rings -- plus
  board, counters, hash, legal mask and infostate digests, in the layout of
  config1.npz;
* ``isf_*``: the 256 games of tests/golden/isf.npz (full boards with uniform
  play, and sparse boards whose pieces chase and shuttle), 300 plies each,
  under the reference class's fixed limits (no-attack 100, length 4000):
  the sticky two-square / chasing violation flags after every ply, and the
  full tracker state at the end.

Infostate planes are digested without channels 41 and 42, which the
reference computes with ``--use_fast_math`` division; those two channels are
stored as values.
"""

from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def digest(a: np.ndarray) -> np.int64:
    return np.frombuffer(hashlib.blake2b(np.ascontiguousarray(a).tobytes(), digest_size=8).digest(), dtype=np.int64)[0]


def board_code(owner: np.ndarray, piece: np.ndarray) -> np.ndarray:
    ow = owner.reshape(owner.shape[0], 100).astype(np.int16)
    pc = piece.reshape(piece.shape[0], 100).astype(np.int16)
    return np.where(ow >= 0, pc | (ow << 4) | 32, 0).astype(np.uint8)


def snapshot(buf) -> dict[str, np.ndarray]:
    st = {k: v.cpu().numpy() for k, v in buf.export_state().items()}
    n = buf.n_games
    mask = buf.compute_legal_action_mask().cpu().numpy().reshape(n, -1).astype(np.uint8)
    info = buf.compute_infostate_tensor().cpu().numpy().reshape(n, 488, 100)
    bits = np.packbits(mask, axis=1, bitorder="little")
    planes = np.concatenate([info[:, :41], info[:, 43:]], axis=1)
    return {
        "board": board_code(st["board_owner"], st["board_piece"]),
        "moved": np.packbits(st["moved_squares"].astype(np.uint8), axis=1, bitorder="little"),
        "revealed": np.packbits(st["revealed_squares"].astype(np.uint8), axis=1, bitorder="little"),
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
        "n_legal": mask.sum(1).astype(np.int32),
        "mask_digest": np.array([digest(bits[g]) for g in range(n)]),
        "planes_digest": np.array([digest(planes[g]) for g in range(n)]),
        "ch41": info[:, 41, 0].copy(),
        "ch42": info[:, 42, 0].copy(),
    }


def planes_from(owner: np.ndarray, piece: np.ndarray):
    import torch

    n = owner.shape[0]
    ow, pc = owner.reshape(n, 10, 10), piece.reshape(n, 10, 10)
    red = torch.from_numpy(np.where(ow == 0, pc, 0).astype(np.int8))
    blue = torch.from_numpy(np.where(ow == 1, pc, 0).astype(np.int8))
    return red, blue


def run_config1(lib_oracle) -> dict[str, np.ndarray]:
    import torch

    from oracle.refcuda import RefCudaBuffer

    g = np.load(HERE / "config1.npz")
    n, plies, seed = (int(x) for x in g["meta"][:3])
    o = lib_oracle.OracleState(n, seed=seed, pool=g["pool"])
    o.reset_pool(force_all=True)  # the trace's starting boards
    buf = RefCudaBuffer(n, 0)
    buf.reset_all(*planes_from(o.a["board_owner"], o.a["board_piece"]))
    snaps = [snapshot(buf)]
    for t in range(plies):
        buf.apply_actions(torch.from_numpy(g["actions"][t]))
        snaps.append(snapshot(buf))
    return {f"c1_{k}": np.stack([s[k] for s in snaps]) for k in snaps[0]}


def run_isf_streams() -> dict[str, np.ndarray]:
    import torch

    from oracle.refcuda import RefCudaBuffer

    g = np.load(HERE / "isf.npz")
    n, plies = g["actions"].shape
    buf = RefCudaBuffer(n, 0)
    buf.reset_all(*planes_from(g["owner"], g["piece"]))
    ts, ch = [], []
    for t in range(plies):
        buf.apply_actions(torch.from_numpy(g["actions"][:, t].astype(np.int64)))
        ts.append(buf.compute_two_square_rule_applies().cpu().numpy().astype(np.uint8))
        ch.append(buf.is_chasing_violation().cpu().numpy().astype(np.uint8))
    end = snapshot(buf)
    st = {k: v.cpu().numpy() for k, v in buf.export_state().items()}
    out = {"isf_ts_violation": np.stack(ts), "isf_chase_violation": np.stack(ch)}
    out.update({f"isf_end_{k}": v for k, v in end.items()})
    out["isf_end_chase_hashes"] = st["chase_hashes"]
    out["isf_end_move_history"] = st["move_history"]
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE / "refcuda.npz"))
    args = ap.parse_args()
    import oracle
    from oracle import refcuda

    if not refcuda.available():
        raise SystemExit(f"{refcuda.LIB_PATH} is missing: build it where the reference checkout is present")
    out = run_config1(oracle)
    out.update(run_isf_streams())
    np.savez_compressed(args.out, **out)
    print(args.out, Path(args.out).stat().st_size, "bytes;",
          "config1 two-square violations", int(out["c1_ts_violation"][-1].sum()),
          "isf-stream chasing violations", int(out["isf_chase_violation"][-1].sum()),
          "two-square", int(out["isf_ts_violation"][-1].sum()))


if __name__ == "__main__":
    main()
