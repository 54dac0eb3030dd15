"""The reference's own CUDA kernels, built from its source -- TEST INFRASTRUCTURE.

The reference project's simulator kernels (``csrc/stratego_buffer.cu``) are
compiled here with nvcc from that one source file, together with
``oracle/refcuda/ref_driver.cu`` (an ``extern "C"`` layer over the launchers
of ``csrc/stratego_buffer.cuh:72-267``) and ``oracle/refcuda/shim/`` (a
stand-in for the single c10 macro that ``csrc/utils.cuh`` uses), into
``oracle/_ref/libref_stratego_cuda.so``.  The flags are the reference's own
(``setup.py:27-35``: ``-O3 --use_fast_math``) with ``sm_100a`` as the target.

:class:`RefCudaBuffer` restates the reference's pybind class
(``csrc/stratego_buffer.cpp:7-303``) in Python with torch: the same state
tensors, the same per-method host work (the four flag-count reductions and
the ``terminated_since`` update around ``apply_actions``, the zero-filled
output tensors, the masked fills of ``reset_terminated``), calling the
reference kernels through the driver.  One deliberate difference: the
Zobrist table is passed in (default: the seed-42 table of
``stratego/env/chasing.py:17-22``) instead of ``torch::randint``
(``cpp:46-49``), so that hashes and chase rings can be compared.

Only ``tests/``, ``tests/golden/make_golden_refcuda.py`` and ``bench.py``'s
``--impl reference-cuda`` arm use this module; the product never does.  The
library exists where it was built in a container holding the reference
checkout (``build()``, run by ``__graft_entry__.build()``); elsewhere
:func:`available` is False.
"""

from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_DIR = HERE / "_ref"
LIB_PATH = LIB_DIR / "libref_stratego_cuda.so"
DRIVER = HERE / "refcuda" / "ref_driver.cu"
SHIM = HERE / "refcuda" / "shim"

NSQ, NACT, NCH, NRING, NHIST = 100, 10000, 488, 64, 32


def reference_root() -> Path | None:
    """The reference checkout (``ATARAXOS_REFERENCE``, else a checkout named
    ``reference`` beside this repository), or None when absent."""
    for cand in (os.environ.get("ATARAXOS_REFERENCE"), HERE.parent.parent / "reference"):
        if cand and (Path(cand) / "csrc" / "stratego_buffer.cu").exists():
            return Path(cand)
    return None


def build(force: bool = False) -> Path | None:
    """Compile the reference kernels + driver into oracle/_ref/ (None when
    the reference checkout is not present)."""
    ref = reference_root()
    if ref is None:
        return LIB_PATH if LIB_PATH.exists() else None
    src = ref / "csrc" / "stratego_buffer.cu"
    deps = [src, ref / "csrc" / "stratego_buffer.cuh", ref / "csrc" / "utils.cuh", DRIVER,
            SHIM / "c10" / "cuda" / "CUDAException.h"]
    if not force and LIB_PATH.exists() and all(d.stat().st_mtime <= LIB_PATH.stat().st_mtime for d in deps):
        return LIB_PATH
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_name(f".{LIB_PATH.name}.{os.getpid()}.tmp")
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--use_fast_math", "-std=c++17",
                    "-shared", "-Xcompiler", "-fPIC", f"-I{SHIM}", f"-I{ref / 'csrc'}", "-o", str(tmp), str(src),
                    str(DRIVER)], check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def available() -> bool:
    return LIB_PATH.exists()


class _RefState(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "board_owner", "board_piece", "current_player", "move_number", "moves_since_attack", "outcome",
        "terminated", "moved_squares", "revealed_squares", "move_history", "move_history_head",
        "move_history_len", "two_square_count", "two_square_pair_lo", "two_square_pair_hi",
        "two_square_violation", "zobrist_table", "chase_hashes", "chase_hash_head", "chase_hash_len",
        "chase_last_src", "chasing_violation")] + [("n", ctypes.c_int32)]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it where the reference checkout is present")
        _lib = ctypes.CDLL(str(LIB_PATH))
        S, vp = ctypes.POINTER(_RefState), ctypes.c_void_p
        for name, args in {
            "ref_hello_world": [vp, vp],
            "ref_apply_actions": [S, vp, vp],
            "ref_legal_action_mask": [S, vp, vp],
            "ref_reset": [S, vp, vp, vp],
            "ref_infostate": [S, vp, vp],
            "ref_hash_board": [S, vp, vp],
        }.items():
            f = getattr(_lib, name)
            f.restype = ctypes.c_int
            f.argtypes = args
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what}: CUDA error {rc}")


def zobrist_table(seed: int = 42) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(low=0, high=2**63, size=(10, 10, 2, 13), dtype=np.int64)


class RefCudaBuffer:
    """The reference pybind class's API over the reference's own kernels."""

    def __init__(self, n_games: int = 1, device_id: int = 0, zobrist: np.ndarray | None = None) -> None:
        import torch

        self.torch = torch
        self.n_games, self.device_id = int(n_games), int(device_id)
        d = self.device = torch.device("cuda", self.device_id)
        n = self.n_games
        i8, i32, i64, b = torch.int8, torch.int32, torch.int64, torch.bool
        # cpp:24-55
        self.board_owner = torch.full((n, 10, 10), -1, dtype=i8, device=d)
        self.board_piece = torch.zeros((n, 10, 10), dtype=i8, device=d)
        self.current_player = torch.zeros(n, dtype=i8, device=d)
        self.move_number = torch.zeros(n, dtype=i32, device=d)
        self.moves_since_attack = torch.zeros(n, dtype=i32, device=d)
        self.outcome = torch.full((n,), -1, dtype=i8, device=d)
        self.terminated = torch.zeros(n, dtype=b, device=d)
        self.flag_captured = torch.zeros(n, dtype=b, device=d)
        self.terminated_since = torch.zeros(n, dtype=i32, device=d)
        self.moved_squares = torch.zeros((n, NSQ), dtype=b, device=d)
        self.revealed_squares = torch.zeros((n, NSQ), dtype=b, device=d)
        self.move_history = torch.zeros((n, NHIST), dtype=i32, device=d)
        self.move_history_head = torch.zeros(n, dtype=i32, device=d)
        self.move_history_len = torch.zeros(n, dtype=i32, device=d)
        self.two_square_count = torch.zeros((n, 2), dtype=i32, device=d)
        self.two_square_pair_lo = torch.full((n, 2), -1, dtype=i32, device=d)
        self.two_square_pair_hi = torch.full((n, 2), -1, dtype=i32, device=d)
        self.two_square_violation = torch.zeros(n, dtype=b, device=d)
        z = zobrist_table() if zobrist is None else np.asarray(zobrist, dtype=np.int64)
        self.zobrist_table = torch.from_numpy(np.ascontiguousarray(z)).to(d)
        self.chase_hashes = torch.zeros((n, 2, NRING), dtype=i64, device=d)
        self.chase_hash_head = torch.zeros((n, 2), dtype=i32, device=d)
        self.chase_hash_len = torch.zeros((n, 2), dtype=i32, device=d)
        self.chase_last_src = torch.full((n, 2), -1, dtype=i32, device=d)
        self.chasing_violation = torch.zeros(n, dtype=b, device=d)
        self._st = _RefState(n=n, **{f: getattr(self, f).data_ptr() for f, _ in _RefState._fields_ if f != "n"})

    def _stream(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream(self.device).cuda_stream)

    # -- cpp:59-303 ------------------------------------------------------
    def hello_world(self):
        out = self.torch.zeros(1, dtype=self.torch.int32, device=self.device)
        _check(lib().ref_hello_world(out.data_ptr(), self._stream()), "hello_world")
        return out

    def _flag_counts(self, player: int):
        t = self.torch
        return ((self.board_owner == player) & (self.board_piece == 11)).view(self.n_games, -1).sum(1).to(t.int32)

    def apply_actions(self, actions) -> None:
        t = self.torch
        if actions.dim() != 1 or actions.size(0) != self.n_games or actions.dtype != t.int64:
            raise RuntimeError("actions must be int64 (N,)")
        a = actions.to(self.device, non_blocking=False)
        blue_before, red_before = self._flag_counts(1), self._flag_counts(0)
        if self.n_games:
            _check(lib().ref_apply_actions(ctypes.byref(self._st), a.data_ptr(), self._stream()), "apply_actions")
        blue_after, red_after = self._flag_counts(1), self._flag_counts(0)
        self.flag_captured |= (blue_before > blue_after) | (red_before > red_after)
        self.terminated_since += self.terminated.to(t.int32)

    def compute_legal_action_mask(self):
        m = self.torch.zeros((self.n_games, NSQ, NSQ), dtype=self.torch.bool, device=self.device)
        if self.n_games:
            _check(lib().ref_legal_action_mask(ctypes.byref(self._st), m.data_ptr(), self._stream()), "mask")
        return m

    def compute_reward_pl0(self):
        r = self.torch.zeros(self.n_games, dtype=self.torch.float32, device=self.device)
        r.masked_fill_(self.outcome == 0, 1.0)
        r.masked_fill_(self.outcome == 1, -1.0)
        return r

    def compute_infostate_tensor(self):
        out = self.torch.zeros((self.n_games, NCH, 10, 10), dtype=self.torch.float32, device=self.device)
        if self.n_games:
            _check(lib().ref_infostate(ctypes.byref(self._st), out.data_ptr(), self._stream()), "infostate")
        return out

    def compute_two_square_rule_applies(self):
        return self.two_square_violation.clone()

    def is_chasing_violation(self):
        return self.chasing_violation.clone()

    def hash_board(self):
        out = self.torch.zeros(self.n_games, dtype=self.torch.int64, device=self.device)
        if self.n_games:
            _check(lib().ref_hash_board(ctypes.byref(self._st), out.data_ptr(), self._stream()), "hash_board")
        return out

    def get_terminated(self):
        return self.terminated.clone()

    def get_outcomes(self):
        return self.outcome.clone()

    def get_board_owner(self):
        return self.board_owner.clone()

    def get_board_piece(self):
        return self.board_piece.clone()

    def get_current_player(self):
        return self.current_player.clone()

    def get_move_number(self):
        return self.move_number.clone()

    def get_num_moves(self):
        return self.move_number.clone()

    def get_num_moves_since_last_attack(self):
        return self.moves_since_attack.clone()

    def get_flag_captured(self):
        return self.flag_captured.clone()

    def get_has_legal_movement(self):
        return self.compute_legal_action_mask().view(self.n_games, -1).any(-1)

    def get_terminated_since(self):
        return self.terminated_since.clone()

    def board_strs(self) -> list[str]:
        ow, pc = self.board_owner.cpu().numpy(), self.board_piece.cpu().numpy()
        out = []
        for g in range(self.n_games):
            s = ""
            for r in range(10):
                for c in range(10):
                    o, p = int(ow[g, r, c]), int(pc[g, r, c])
                    s += ". " if o < 0 else ("R" if o == 0 else "B") + str(p) + (" " if p < 10 else "")
                s += "\n"
            out.append(s)
        return out

    def reset_terminated(self, setup_red, setup_blue) -> None:
        t = self.torch
        for x, nm in ((setup_red, "setup_red"), (setup_blue, "setup_blue")):
            if x.dim() != 3 or x.size(0) != self.n_games or x.shape[1:] != (10, 10) or x.dtype != t.int8:
                raise RuntimeError(f"{nm} must be int8 (N, 10, 10)")
        red = setup_red.to(self.device).contiguous()
        blue = setup_blue.to(self.device).contiguous()
        was = self.terminated.clone()
        if self.n_games:
            _check(lib().ref_reset(ctypes.byref(self._st), red.data_ptr(), blue.data_ptr(), self._stream()), "reset")
        reset = was & ~self.terminated
        self.flag_captured.masked_fill_(reset, False)
        self.terminated_since.masked_fill_(reset, 0)

    def reset_all(self, setup_red, setup_blue) -> None:
        self.terminated.fill_(True)
        self.reset_terminated(setup_red, setup_blue)

    def current_step(self) -> int:
        return int(self.move_number.sum().item())

    # -- for comparisons --------------------------------------------------
    def export_state(self) -> dict:
        """The state tensors under the names ``StrategoRolloutBuffer.export_state`` uses."""
        names = ("board_owner", "board_piece", "current_player", "outcome", "terminated", "flag_captured",
                 "move_number", "moves_since_attack", "terminated_since", "moved_squares", "revealed_squares",
                 "move_history", "move_history_head", "move_history_len", "two_square_count",
                 "two_square_pair_lo", "two_square_pair_hi", "two_square_violation", "chase_hash_head",
                 "chase_hash_len", "chase_last_src", "chasing_violation")
        d = {k: getattr(self, k).clone() for k in names}
        d["chase_hashes"] = self.chase_hashes.clone()
        return d
