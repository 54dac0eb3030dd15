"""ctypes binding of libstratego_b200.so (the C ABI declared in include/stratego_b200.h).

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises.  Build it with ``python -m ataraxos_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_LIB_DIR = Path(__file__).resolve().parent / "_lib"
# ATARAXOS_B200_DEBUG=1 selects the debug build, whose kernels check every game
# record's indices first and skip a bad game (SB_STATUS_BAD_STATE) instead of
# reading or writing out of range; it is slower and meant for loaded records.
DEBUG = os.environ.get("ATARAXOS_B200_DEBUG", "0") not in ("", "0")
LIB_PATH = _LIB_DIR / ("libstratego_b200_debug.so" if DEBUG else "libstratego_b200.so")

SB_OK, SB_E_ARG, SB_E_CUDA, SB_E_NOPOOL = 0, -1, -2, -3
SB_DTYPE_F32, SB_DTYPE_BF16 = 0, 1
SB_LAYOUT_DENSE_ALL, SB_LAYOUT_DENSE_LIVE, SB_LAYOUT_COMPACT = 0, 1, 2
SB_POLICY_UNIFORM, SB_POLICY_GUMBEL = 0, 1
SB_RULES_CUDA, SB_RULES_ISF = 0, 1
SB_NOALLOC_MAX_ENVS = 262144
SB_STATUS_BAD_SETUP = 1
SB_STATUS_WAIT_TIMEOUT = 2
SB_STATUS_BAD_STATE = 4
RECORD_BYTES = 256
ISF_TS_BYTES = 600  # per env under SB_RULES_ISF: 100 squares x 3 intervals x (lo, hi)

vp = ctypes.c_void_p


class SbState(ctypes.Structure):
    _fields_ = [
        ("records", vp),
        ("chase_ring", vp),
        ("zobrist", vp),
        ("setup_pool", vp),
        ("pool_size", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("env_base", ctypes.c_int64),
        ("seed", ctypes.c_uint64),
        ("no_attack_limit", ctypes.c_int32),
        ("max_game_length", ctypes.c_int32),
        ("two_square_limit", ctypes.c_int32),
        ("rules", ctypes.c_int32),
        ("status", vp),
        ("isf_two_square", vp),
    ]


class SbStepOut(ctypes.Structure):
    _fields_ = [
        ("mask_u8", vp),
        ("mask_bits", vp),
        ("infostate", vp),
        ("info_dtype", ctypes.c_int32),
        ("info_layout", ctypes.c_int32),
        ("reward", vp),
        ("done", vp),
        ("action_taken", vp),
        ("logprob_taken", vp),
        ("next_action", vp),
        ("next_logprob", vp),
        ("hash", vp),
        ("stats", vp),
    ]


class SbTraj(ctypes.Structure):
    _fields_ = [
        ("infostate", vp),
        ("info_dtype", ctypes.c_int32),
        ("info_layout", ctypes.c_int32),
        ("mask_u8", vp),
        ("mask_bits", vp),
        ("action", vp),
        ("logprob", vp),
        ("reward", vp),
        ("done", vp),
        ("hash", vp),
        ("stats", vp),
        ("n_slots", ctypes.c_int64),
        ("slot0", ctypes.c_int64),
    ]


class SbPolicy(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("reserved", ctypes.c_int32), ("logits", vp)]


EXPORT_FIELDS = [
    "board_owner", "board_piece", "current_player", "outcome", "terminated", "flag_captured", "move_number",
    "moves_since_attack", "terminated_since", "moved_squares", "revealed_squares", "move_history",
    "move_history_head", "move_history_len", "two_square_count", "two_square_pair_lo", "two_square_pair_hi",
    "two_square_violation", "chase_hash_head", "chase_hash_len", "chase_last_src", "chasing_violation", "episode",
    "invalid_count", "reward", "isf_two_square", "isf_threats", "isf_evasion",
]


class SbExport(ctypes.Structure):
    _fields_ = [(f, vp) for f in EXPORT_FIELDS]


class SbServe(ctypes.Structure):
    _fields_ = [("ctl", vp), ("dev", vp), ("back_dev", vp), ("back_host", vp), ("back_bytes", ctypes.c_int64),
                ("n_ctas", ctypes.c_int64), ("limit_ns", ctypes.c_int64)]


class SbHostIo(ctypes.Structure):
    _fields_ = [
        ("actions_host", vp),
        ("actions_dev", vp),
        ("back_dev", vp),
        ("back_host", vp),
        ("back_bytes", ctypes.c_int64),
        ("sync", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


# name -> (restype, argtypes)
_SIGS = {
    "sb_abi_version": (ctypes.c_int, []),
    "sb_last_error": (ctypes.c_char_p, []),
    "sb_debug_bounds": (ctypes.c_int, []),
    "sb_init_state": (ctypes.c_int, [ctypes.POINTER(SbState), vp]),
    "sb_hello_world": (ctypes.c_int, [vp, vp]),
    "sb_reset_planes": (ctypes.c_int, [ctypes.POINTER(SbState), vp, vp, ctypes.c_int, vp]),
    "sb_reset_pool": (ctypes.c_int, [ctypes.POINTER(SbState), ctypes.c_int, vp]),
    "sb_make_setup_pool": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64, vp, vp]),
    "sb_apply_actions": (ctypes.c_int, [ctypes.POINTER(SbState), vp, vp]),
    "sb_step": (ctypes.c_int, [ctypes.POINTER(SbState), vp, ctypes.c_int64, ctypes.POINTER(SbPolicy), ctypes.c_int,
                               ctypes.POINTER(SbStepOut), vp]),
    "sb_step_host": (ctypes.c_int, [ctypes.POINTER(SbState), ctypes.POINTER(SbHostIo), ctypes.c_int64,
                                    ctypes.POINTER(SbPolicy), ctypes.c_int, ctypes.POINTER(SbStepOut), vp]),
    "sb_step_host_noalloc": (ctypes.c_int, [ctypes.POINTER(SbState), ctypes.POINTER(SbHostIo), ctypes.c_int64,
                                            ctypes.POINTER(SbPolicy), ctypes.c_int, ctypes.POINTER(SbStepOut), vp]),
    "sb_serve_start": (ctypes.c_int, [ctypes.POINTER(SbState), ctypes.c_int64, ctypes.c_int, vp,
                                      ctypes.POINTER(SbStepOut), ctypes.POINTER(SbServe), vp]),
    "sb_serve_step": (ctypes.c_int, [ctypes.POINTER(SbServe), ctypes.c_int64, ctypes.c_int64]),
    "sb_serve_stop": (ctypes.c_int, [ctypes.POINTER(SbServe), ctypes.c_int64, vp]),
    "sb_rollout": (ctypes.c_int, [ctypes.POINTER(SbState), ctypes.c_int64, ctypes.POINTER(SbPolicy), ctypes.c_int,
                                  ctypes.c_int32, ctypes.POINTER(SbTraj), vp]),
    "sb_belief_resample": (ctypes.c_int, [ctypes.POINTER(SbState), ctypes.POINTER(SbState), vp, vp]),
    "sb_sample_actions": (ctypes.c_int, [ctypes.POINTER(SbState), ctypes.c_int64, ctypes.POINTER(SbPolicy), vp, vp, vp]),
    "sb_legal_mask_u8": (ctypes.c_int, [ctypes.POINTER(SbState), vp, vp]),
    "sb_legal_mask_bits": (ctypes.c_int, [ctypes.POINTER(SbState), vp, vp]),
    "sb_infostate": (ctypes.c_int, [ctypes.POINTER(SbState), vp, ctypes.c_int, ctypes.c_int, vp]),
    "sb_hash_board": (ctypes.c_int, [ctypes.POINTER(SbState), vp, vp]),
    "sb_has_legal_movement": (ctypes.c_int, [ctypes.POINTER(SbState), vp, vp]),
    "sb_export_state": (ctypes.c_int, [ctypes.POINTER(SbState), ctypes.POINTER(SbExport), vp]),
    "sb_sum_move_number": (ctypes.c_int, [ctypes.POINTER(SbState), vp, vp]),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: the B200 simulator has no CPU fallback. "
                "Build it with `python -m ataraxos_b200.build`."
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.sb_abi_version() != 2:
            raise ImportError("libstratego_b200.so ABI version mismatch")
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(rc: int) -> None:
    if rc != SB_OK:
        msg = lib().sb_last_error().decode(errors="replace")
        raise RuntimeError(f"libstratego_b200 error {rc}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
