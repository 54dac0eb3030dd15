"""StrategoRolloutBuffer: the B200 batched Stratego simulator behind the reference's API.

``StrategoRolloutBuffer(n_games, device_id)`` is a drop-in for the reference's
pybind class ``_stratego_cuda.StrategoRolloutBuffer``
(``csrc/stratego_buffer.cpp:7-411``): same constructor, same method names,
same return shapes and dtypes, same "getters return copies" ownership and the
same errors (``RuntimeError`` on shape/dtype misuse, as ``TORCH_CHECK`` gives;
illegal actions are ignored per game).  Every method launches native code from
``libstratego_b200.so`` on the current torch stream of ``device_id``; there is
no CPU or eager-torch fallback.

On top of that API the north-star contract adds:
  * ``step(actions=None)``: the fused ply (sample or take actions, apply,
    auto-reset from a seeded device setup pool, legal mask and infostate of
    the new state) in one kernel, writing into persistent output buffers;
  * the setup pool (``pool_size=``, ``reset_all_from_pool()``);
  * uniform and Gumbel-max action sampling (``sample_actions``);
  * bit-packed masks, bf16 / compact infostate layouts, trajectory slots
    (``ataraxos_b200.trajectory``);
  * ``export_state()`` / ``state_dict()`` / ``load_state_dict()``.

Differences from the reference, all deliberate:
  * the Zobrist table is the seed-42 numpy table of
    ``stratego/env/chasing.py:17-22`` (the reference CUDA class draws a
    non-reproducible one with ``torch::randint``, ``cpp:46-49``);
  * setup planes must hold piece codes 0..12 (the reference does not check;
    a larger code made its hash kernel read out of bounds);
  * channels 41/42 are exact float32 quotients (the reference divides with
    ``--use_fast_math``; the Python engine rounds the exact quotient, which
    is what this build matches).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _capi as C

NUM_SQUARES = 100
NUM_ACTIONS = 10000
NUM_CHANNELS = 488
COMPACT_CHANNELS = 76
MASK_BITS_BYTES = 1250


def zobrist_table(seed: int = 42) -> np.ndarray:
    """Zobrist table [10,10,2,13] int64 drawn exactly as ``ZobristHasher(seed)``
    does (``stratego/env/chasing.py:17-22``): numpy ``default_rng(seed)``,
    integers in [0, 2**63)."""
    rng = np.random.default_rng(seed)
    return rng.integers(low=0, high=2**63, size=(10, 10, 2, 13), dtype=np.int64)


def _vp(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


_get_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _raw_stream(index: int) -> int:
    """cudaStream_t of the current torch stream of device ``index`` (as an int)."""
    if _get_raw_stream is not None:
        return _get_raw_stream(index)
    return torch.cuda.current_stream(index).cuda_stream


_POLICIES = {"uniform": C.SB_POLICY_UNIFORM, "gumbel": C.SB_POLICY_GUMBEL}
_RULES = {"cuda": C.SB_RULES_CUDA, "isf": C.SB_RULES_ISF}

_RESULT_FIELDS = (("reward", torch.float32, 4), ("next_action", torch.int16, 2), ("done", torch.uint8, 1))


def _results_layout(n: int) -> dict[str, int]:
    """Byte offsets of reward f32[n], next_action i16[n] and done u8[n] in one
    block, each 16-byte aligned."""
    lay, off = {}, 0
    for name, _, size in _RESULT_FIELDS:
        lay[name] = off
        off += (n * size + 15) // 16 * 16
    lay["bytes"] = max(off, 16)
    return lay


def _results_view(block: torch.Tensor, lay: dict[str, int], name: str, n: int) -> torch.Tensor:
    dtype, size = {f: (d, s) for f, d, s in _RESULT_FIELDS}[name]
    return block[lay[name]:lay[name] + n * size].view(dtype)


@dataclass
class StepOutput:
    """Views into the buffer's persistent outputs (overwritten by the next step)."""

    infostate: torch.Tensor | None   # [N,488,10,10] (or [N,76,10,10] compact)
    legal_mask: torch.Tensor | None  # [N,100,100] bool, or [N,1250] uint8 bit-packed
    reward: torch.Tensor             # [N] float32, player-0 reward of this transition
    done: torch.Tensor               # [N] bool, the transition ended the game
    action: torch.Tensor             # [N] int64, action applied (-1 none)
    logprob: torch.Tensor            # [N] float32, log-prob of the applied action when sampled
    next_action: torch.Tensor        # [N] int16, action proposed for the new state (-1: none, game over)
    next_logprob: torch.Tensor       # [N] float32


@dataclass
class HostStepOutput:
    """Pinned host copies of one step's per-game results, plus the step's
    device outputs (all overwritten by the next ``step_host``)."""

    reward: torch.Tensor       # [N] float32, player-0 reward of the transition
    done: torch.Tensor         # [N] bool
    next_action: torch.Tensor  # [N] int16, action proposed for the new state (-1: none, game over)
    device: StepOutput


class StrategoRolloutBuffer:
    """N parallel Stratego games on one B200 (csrc/stratego_buffer.cpp:7-337)."""

    def __init__(
        self,
        n_games: int = 1,
        device_id: int = 0,
        *,
        seed: int = 0,
        env_base: int = 0,
        pool_size: int | None = None,
        setup_pool: torch.Tensor | np.ndarray | None = None,
        pool_seed: int | None = None,
        no_attack_limit: int = 100,
        max_game_length: int = 4000,
        two_square_limit: int = 3,
        zobrist: np.ndarray | torch.Tensor | None = None,
        obs_dtype: torch.dtype = torch.bfloat16,
        obs_layout: str = "dense",
        mask_format: str = "u8",
        rules: str = "cuda",
    ) -> None:
        if n_games < 0:
            raise RuntimeError("n_games must be >= 0")
        C.lib()  # fail loudly before allocating anything
        self._n = int(n_games)
        self._device_id = int(device_id)
        self.device = torch.device("cuda", self._device_id)
        self.seed = int(seed)
        self.env_base = int(env_base)
        self.no_attack_limit = int(no_attack_limit)
        self.max_game_length = int(max_game_length)
        self.two_square_limit = int(two_square_limit)
        if obs_dtype not in (torch.bfloat16, torch.float32):
            raise RuntimeError("obs_dtype must be torch.bfloat16 or torch.float32")
        if obs_layout not in ("dense", "compact"):
            raise RuntimeError("obs_layout must be 'dense' or 'compact'")
        if mask_format not in ("u8", "bits", "none"):
            raise RuntimeError("mask_format must be 'u8', 'bits' or 'none'")
        self.obs_dtype, self.obs_layout, self.mask_format = obs_dtype, obs_layout, mask_format
        if rules not in _RULES:
            raise RuntimeError("rules must be 'cuda' (the reference CUDA class's trackers) or 'isf' (the ISF rules "
                               "of stratego/env/two_square.py and chasing.py)")
        if rules == "isf" and not 1 <= self.two_square_limit <= 3:
            raise RuntimeError("rules='isf' supports two_square_limit 1..3")
        self.rules = rules
        n, dev = self._n, self.device
        with torch.cuda.device(dev):
            self._records = torch.empty((max(n, 1), C.RECORD_BYTES), dtype=torch.uint8, device=dev)
            self._ring = torch.empty((max(n, 1), 2, 64), dtype=torch.int64, device=dev)
            z = zobrist_table() if zobrist is None else zobrist
            z = torch.as_tensor(np.asarray(z) if not isinstance(z, torch.Tensor) else z, dtype=torch.int64)
            if tuple(z.shape) != (10, 10, 2, 13):
                raise RuntimeError("zobrist table must be [10,10,2,13] int64")
            self._zobrist = z.contiguous().to(dev)
            self._status = torch.zeros(1, dtype=torch.int32, device=dev)
            # per-square two-square state of the ISF rules (none under the CUDA rules)
            self._isf = (torch.empty((max(n, 1), C.ISF_TS_BYTES), dtype=torch.uint8, device=dev)
                         if rules == "isf" else None)
            self._pool: torch.Tensor | None = None
            if setup_pool is not None:
                self.set_setup_pool(setup_pool)
            elif pool_size:
                self.make_setup_pool(int(pool_size), self.seed if pool_seed is None else int(pool_seed))
            self._st = self._make_state()
            C.call("sb_init_state", ctypes.byref(self._st), _stream(dev))
        self._ply = 0
        self._outs: dict[str, torch.Tensor] | None = None
        self._host: dict | None = None
        self._pol_cache: dict = {}

    # ------------------------------------------------------------------
    # plumbing
    # ------------------------------------------------------------------
    def _make_state(self) -> C.SbState:
        return C.SbState(
            records=self._records.data_ptr(),
            chase_ring=self._ring.data_ptr(),
            zobrist=self._zobrist.data_ptr(),
            setup_pool=_vp(self._pool),
            pool_size=0 if self._pool is None else self._pool.shape[0],
            n=self._n,
            env_base=self.env_base,
            seed=self.seed,
            no_attack_limit=self.no_attack_limit,
            max_game_length=self.max_game_length,
            two_square_limit=self.two_square_limit,
            rules=_RULES[self.rules],
            status=self._status.data_ptr(),
            isf_two_square=_vp(self._isf),
        )

    def _call(self, name: str, *args) -> None:
        with torch.cuda.device(self.device):
            C.call(name, ctypes.byref(self._st), *args, _stream(self.device))

    def _alloc(self, shape, dtype) -> torch.Tensor:
        return torch.empty(shape, dtype=dtype, device=self.device)

    def _export_one(self, field: str, shape, dtype) -> torch.Tensor:
        out = self._alloc(shape, dtype)
        ex = C.SbExport(**{field: out.data_ptr()})
        self._call("sb_export_state", ctypes.byref(ex))
        return out

    # ------------------------------------------------------------------
    # reference API (csrc/stratego_buffer.cpp:341-411)
    # ------------------------------------------------------------------
    @property
    def n_games(self) -> int:
        return self._n

    @property
    def device_id(self) -> int:
        return self._device_id

    def hello_world(self) -> torch.Tensor:
        """int32 [1] CUDA tensor holding 42 (cpp:59-67)."""
        out = torch.zeros(1, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            C.call("sb_hello_world", out.data_ptr(), _stream(self.device))
        return out

    def _actions_dev(self, actions: torch.Tensor, non_blocking: bool = False) -> torch.Tensor:
        if not isinstance(actions, torch.Tensor):
            raise RuntimeError("actions must be a torch.Tensor")
        if actions.dim() != 1:
            raise RuntimeError("actions must be 1D (N,)")
        if actions.size(0) != self._n:
            raise RuntimeError(f"actions size mismatch: expected {self._n}, got {actions.size(0)}")
        if actions.dtype != torch.int64:
            raise RuntimeError("actions must be int64")
        return actions.to(self.device, non_blocking=non_blocking).contiguous()

    def apply_actions(self, actions: torch.Tensor) -> None:
        """Apply (N,) int64 actions src*100+dst to all games (cpp:70-120)."""
        a = self._actions_dev(actions)
        if self._n:
            self._call("sb_apply_actions", a.data_ptr())
        self._ply += 1

    def compute_legal_action_mask(self) -> torch.Tensor:
        """(N,100,100) bool legal-move mask of the side to move (cpp:123-139)."""
        out = self._alloc((self._n, NUM_SQUARES, NUM_SQUARES), torch.uint8)
        if self._n:
            self._call("sb_legal_mask_u8", out.data_ptr())
        return out.view(torch.bool)

    def compute_legal_action_mask_bits(self) -> torch.Tensor:
        """(N,1250) uint8 bit-packed mask; bit j of byte k is flat action 8k+j."""
        out = self._alloc((self._n, MASK_BITS_BYTES), torch.uint8)
        if self._n:
            self._call("sb_legal_mask_bits", out.data_ptr())
        return out

    def compute_reward_pl0(self) -> torch.Tensor:
        """(N,) float32: +1 Red win, -1 Blue win, else 0 (cpp:142-151)."""
        return self._export_one("reward", (self._n,), torch.float32)

    def compute_infostate_tensor(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """(N,488,10,10) infostate from the side to move's view (cpp:154-176)."""
        code = C.SB_DTYPE_F32 if dtype == torch.float32 else C.SB_DTYPE_BF16
        if dtype not in (torch.float32, torch.bfloat16):
            raise RuntimeError("dtype must be float32 or bfloat16")
        out = self._alloc((self._n, NUM_CHANNELS, 10, 10), dtype)
        if self._n:
            self._call("sb_infostate", out.data_ptr(), code, C.SB_LAYOUT_DENSE_ALL)
        return out

    def compute_two_square_rule_applies(self) -> torch.Tensor:
        return self._export_one("two_square_violation", (self._n,), torch.uint8).view(torch.bool)

    def is_chasing_violation(self) -> torch.Tensor:
        return self._export_one("chasing_violation", (self._n,), torch.uint8).view(torch.bool)

    def hash_board(self) -> torch.Tensor:
        """(N,) int64 Zobrist hash of each board (cu:805-845)."""
        out = self._alloc((self._n,), torch.int64)
        if self._n:
            self._call("sb_hash_board", out.data_ptr())
        return out

    def get_terminated(self) -> torch.Tensor:
        return self._export_one("terminated", (self._n,), torch.uint8).view(torch.bool)

    def get_outcomes(self) -> torch.Tensor:
        return self._export_one("outcome", (self._n,), torch.int8)

    def get_board_owner(self) -> torch.Tensor:
        return self._export_one("board_owner", (self._n, 10, 10), torch.int8)

    def get_board_piece(self) -> torch.Tensor:
        return self._export_one("board_piece", (self._n, 10, 10), torch.int8)

    def get_current_player(self) -> torch.Tensor:
        return self._export_one("current_player", (self._n,), torch.int8)

    def get_move_number(self) -> torch.Tensor:
        return self._export_one("move_number", (self._n,), torch.int32)

    def get_num_moves(self) -> torch.Tensor:
        return self.get_move_number()

    def get_num_moves_since_last_attack(self) -> torch.Tensor:
        return self._export_one("moves_since_attack", (self._n,), torch.int32)

    def get_flag_captured(self) -> torch.Tensor:
        return self._export_one("flag_captured", (self._n,), torch.uint8).view(torch.bool)

    def get_has_legal_movement(self) -> torch.Tensor:
        """(N,) bool: the side to move has a legal move (cpp:216-219)."""
        out = self._alloc((self._n,), torch.uint8)
        if self._n:
            self._call("sb_has_legal_movement", out.data_ptr())
        return out.view(torch.bool)

    def get_terminated_since(self) -> torch.Tensor:
        return self._export_one("terminated_since", (self._n,), torch.int32)

    def board_strs(self) -> list[str]:
        """One text board per game, 'R<piece>'/'B<piece>'/'.' (cpp:222-242)."""
        ow = self.get_board_owner().cpu().numpy()
        pc = self.get_board_piece().cpu().numpy()
        out = []
        for g in range(self._n):
            rows = []
            for r in range(10):
                s = ""
                for c in range(10):
                    o, p = int(ow[g, r, c]), int(pc[g, r, c])
                    if o < 0:
                        s += ". "
                    else:
                        s += ("R" if o == 0 else "B") + str(p) + (" " if p < 10 else "")
                rows.append(s + "\n")
            out.append("".join(rows))
        return out

    def _setup_plane(self, t: torch.Tensor, name: str) -> torch.Tensor:
        if not isinstance(t, torch.Tensor):
            raise RuntimeError(f"{name} must be a torch.Tensor")
        if t.dim() != 3:
            raise RuntimeError(f"{name} must be (N, 10, 10)")
        if t.size(0) != self._n:
            raise RuntimeError(f"{name} N mismatch")
        if t.size(1) != 10 or t.size(2) != 10:
            raise RuntimeError(f"{name} must be (N, 10, 10)")
        if t.dtype != torch.int8:
            raise RuntimeError(f"{name} must be int8")
        if t.numel() and (int(t.min()) < 0 or int(t.max()) > 12):
            raise RuntimeError(f"{name} holds piece codes outside 0..12")
        return t.to(self.device).contiguous()

    def reset_terminated(self, setup_red: torch.Tensor, setup_blue: torch.Tensor) -> None:
        """Reset terminated games from setup planes (cpp:245-292)."""
        r = self._setup_plane(setup_red, "setup_red")
        b = self._setup_plane(setup_blue, "setup_blue")
        if self._n:
            self._call("sb_reset_planes", r.data_ptr(), b.data_ptr(), 0)

    def reset_all(self, setup_red: torch.Tensor, setup_blue: torch.Tensor) -> None:
        """Force-reset every game from setup planes (cpp:295-298)."""
        r = self._setup_plane(setup_red, "setup_red")
        b = self._setup_plane(setup_blue, "setup_blue")
        if self._n:
            self._call("sb_reset_planes", r.data_ptr(), b.data_ptr(), 1)

    def current_step(self) -> int:
        """Sum of move numbers over all games (cpp:301-303)."""
        out = self._alloc((1,), torch.int64)
        self._call("sb_sum_move_number", out.data_ptr())
        return int(out.item())

    # ------------------------------------------------------------------
    # north-star additions
    # ------------------------------------------------------------------
    @property
    def ply(self) -> int:
        """Number of apply_actions/step calls so far (keys the action RNG)."""
        return self._ply

    @ply.setter
    def ply(self, v: int) -> None:
        self._ply = int(v)

    @property
    def setup_pool(self) -> torch.Tensor | None:
        return self._pool

    def set_setup_pool(self, pool) -> None:
        p = torch.as_tensor(np.asarray(pool) if not isinstance(pool, torch.Tensor) else pool)
        if p.dim() != 2 or p.size(1) != 40 or p.size(0) < 1:
            raise RuntimeError("setup pool must be [P,40] with P >= 1")
        p = p.to(torch.uint8)
        if int(p.min()) < 1 or int(p.max()) > 12:
            raise RuntimeError("setup pool entries must hold piece codes 1..12")
        self._pool = p.to(self.device).contiguous()
        if hasattr(self, "_st"):
            self._st = self._make_state()

    def make_setup_pool(self, size: int, seed: int) -> torch.Tensor:
        """Generate ``size`` seeded random setups on the device (Philox Fisher-Yates)."""
        p = torch.empty((size, 40), dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            C.call("sb_make_setup_pool", ctypes.c_uint64(seed), 0, size, p.data_ptr(), _stream(self.device))
        self._pool = p
        if hasattr(self, "_st"):
            self._st = self._make_state()
        return p

    def reset_all_from_pool(self) -> None:
        """Start a new game in every env from the setup pool."""
        if self._n:
            self._call("sb_reset_pool", 1)

    def reset_terminated_from_pool(self) -> None:
        if self._n:
            self._call("sb_reset_pool", 0)

    def status(self) -> int:
        """Device status bits (SB_STATUS_*) raised since construction."""
        return int(self._status.item())

    def _alloc_outputs(self, stats: torch.Tensor | None) -> dict[str, torch.Tensor]:
        n, dev = self._n, self.device
        chans = NUM_CHANNELS if self.obs_layout == "dense" else COMPACT_CHANNELS
        # reward, next_action and done share one block (see _results_layout) so
        # that step_host brings all three back with a single copy.
        lay = _results_layout(n)
        res = torch.zeros(lay["bytes"], dtype=torch.uint8, device=dev)
        o: dict = {
            "infostate": torch.zeros((n, chans, 10, 10), dtype=self.obs_dtype, device=dev),
            "results": res,
            "reward": _results_view(res, lay, "reward", n),
            "done": _results_view(res, lay, "done", n),
            "action": torch.zeros(n, dtype=torch.int64, device=dev),
            "logprob": torch.zeros(n, dtype=torch.float32, device=dev),
            "next_action": _results_view(res, lay, "next_action", n),
            "next_logprob": torch.zeros(n, dtype=torch.float32, device=dev),
            "stats": torch.zeros(5, dtype=torch.int64, device=dev) if stats is None else stats,
        }
        if self.mask_format == "u8":
            o["mask"] = torch.zeros((n, NUM_SQUARES, NUM_SQUARES), dtype=torch.uint8, device=dev)
        elif self.mask_format == "bits":
            o["mask"] = torch.zeros((n, MASK_BITS_BYTES), dtype=torch.uint8, device=dev)
        o["_args"] = {}  # prebuilt ctypes arguments of step(), per observe flag
        return o

    def _ensure_outputs(self) -> dict[str, torch.Tensor]:
        if self._outs is None:
            self._outs = self._alloc_outputs(None)
        return self._outs

    def new_outputs(self) -> dict[str, torch.Tensor]:
        """A further set of step outputs for ``step(outputs=...)``: infostate,
        legal mask and per-game results laid out as the buffer's own (their
        zero infostate planes written once, here).  With two or more sets a
        consumer can read one ply's observations while the next ply writes
        another set.  The episode statistics stay shared with the buffer's
        own outputs."""
        return self._alloc_outputs(self._ensure_outputs()["stats"])

    def _policy(self, policy: str, logits: torch.Tensor | None) -> C.SbPolicy:
        if policy not in _POLICIES:
            raise RuntimeError(f"unknown policy {policy!r}")
        lp = None
        if logits is not None:
            if policy != "gumbel":
                raise RuntimeError("logits need policy='gumbel'")
            if logits.dtype != torch.float32 or logits.device != self.device or logits.numel() != self._n * NUM_ACTIONS:
                raise RuntimeError("logits must be float32 [N,10000] on the buffer's device")
            lp = logits.contiguous().data_ptr()
        return C.SbPolicy(kind=_POLICIES[policy], reserved=0, logits=lp)

    def step_raw(
        self,
        actions: torch.Tensor | None = None,
        *,
        policy: str = "uniform",
        logits: torch.Tensor | None = None,
        auto_reset: bool = True,
        outputs: C.SbStepOut | None = None,
    ) -> None:
        """One fused ply writing into caller-provided ``outputs`` (an SbStepOut)."""
        a = None if actions is None else self._actions_dev(actions, non_blocking=True)
        pol = self._policy(policy, logits)
        if self._n:
            self._call("sb_step", _vp(a), self._ply, ctypes.byref(pol), int(auto_reset),
                       None if outputs is None else ctypes.byref(outputs))
        self._ply += 1

    def step(
        self,
        actions: torch.Tensor | None = None,
        *,
        policy: str = "uniform",
        logits: torch.Tensor | None = None,
        auto_reset: bool = True,
        observe: bool = True,
        outputs: dict | None = None,
    ) -> StepOutput:
        """One ply for every game, fused in one kernel.

        ``actions`` (N,) int64 (host or device) or None to sample each game's
        action on the device (``policy`` 'uniform' or 'gumbel'; ``logits``
        [N,10000] float32 for 'gumbel', else virtual Philox N(0,1) logits).
        Then: apply, per-game auto-reset from the setup pool for games that
        ended, and the legal mask / infostate of the new state into the
        buffer's persistent outputs (or into ``outputs``, a set made by
        :meth:`new_outputs`).  The returned tensors are views of those outputs
        and are overwritten by the next step that writes the same set.
        """
        o = self._ensure_outputs() if outputs is None else outputs
        if logits is None and actions is None and self._n:
            # the common device-sampled step: one native call on prebuilt arguments
            args = o["_args"].get(observe)
            if args is None:
                args = o["_args"][observe] = (ctypes.byref(self._step_out(o, observe)),
                                              self._step_views(o, observe))
            pol = self._pol_cache.get(policy)
            if pol is None:
                pol = self._pol_cache[policy] = ctypes.byref(self._policy(policy, None))
            dev = self._device_id
            fn = C.lib().sb_step
            if torch.cuda.current_device() != dev:
                with torch.cuda.device(self.device):
                    rc = fn(ctypes.byref(self._st), None, self._ply, pol, 1 if auto_reset else 0, args[0],
                            _raw_stream(dev))
            else:
                rc = fn(ctypes.byref(self._st), None, self._ply, pol, 1 if auto_reset else 0, args[0],
                        _raw_stream(dev))
            if rc:
                C.check(rc)
            self._ply += 1
            return args[1]
        self.step_raw(actions, policy=policy, logits=logits, auto_reset=auto_reset,
                      outputs=self._step_out(o, observe))
        return self._step_views(o, observe)

    def _step_out(self, o: dict[str, torch.Tensor], observe: bool) -> C.SbStepOut:
        info = o["infostate"] if observe else None
        mask = o.get("mask") if observe else None
        return C.SbStepOut(
            mask_u8=_vp(mask) if self.mask_format == "u8" else None,
            mask_bits=_vp(mask) if self.mask_format == "bits" else None,
            infostate=_vp(info),
            info_dtype=C.SB_DTYPE_BF16 if self.obs_dtype == torch.bfloat16 else C.SB_DTYPE_F32,
            info_layout=C.SB_LAYOUT_DENSE_LIVE if self.obs_layout == "dense" else C.SB_LAYOUT_COMPACT,
            reward=o["reward"].data_ptr(),
            done=o["done"].data_ptr(),
            action_taken=o["action"].data_ptr(),
            logprob_taken=o["logprob"].data_ptr(),
            next_action=o["next_action"].data_ptr(),
            next_logprob=o["next_logprob"].data_ptr(),
            hash=None,
            stats=o["stats"].data_ptr(),
        )

    def _step_views(self, o: dict[str, torch.Tensor], observe: bool) -> StepOutput:
        mask = o.get("mask") if observe else None
        legal = None
        if mask is not None:
            legal = mask.view(torch.bool) if self.mask_format == "u8" else mask
        return StepOutput(
            infostate=o["infostate"] if observe else None,
            legal_mask=legal,
            reward=o["reward"],
            done=o["done"].view(torch.bool),
            action=o["action"],
            logprob=o["logprob"],
            next_action=o["next_action"],
            next_logprob=o["next_logprob"],
        )

    def step_host(
        self,
        actions: torch.Tensor | None = None,
        *,
        policy: str = "uniform",
        auto_reset: bool = True,
        observe: bool = True,
        sync: bool = True,
        mapped: bool = True,
        stream: torch.cuda.Stream | None = None,
    ) -> HostStepOutput:
        """``step`` for a host-side caller, in one native call: the (N,) int64
        CPU ``actions`` (None: sample on the device) go host->device, the fused
        ply runs, and reward / done / next_action come back into pinned host
        memory with one copy.  The returned host tensors (and ``.device``, the
        step's device outputs) are overwritten by the next call; with
        ``sync=False`` they are valid once the stream (``stream``, else the
        current stream) has reached this call's end.

        ``mapped=True`` moves the data without copy-engine transfers: the
        kernel reads the actions from page-locked host memory and writes
        reward / done / next_action straight into the pinned result block
        (the device copies of those three are then not written).
        ``mapped=False`` copies actions in and the result block back with
        ``cudaMemcpyAsync``."""
        h = self._host_io()
        mode = "mapped" if mapped else "copy"
        io = h["io"][mode]
        if actions is None:
            io.actions_host = None
        else:
            if type(actions) is not torch.Tensor or actions.device.type != "cpu":
                raise RuntimeError("step_host takes CPU actions (use step() for device tensors)")
            if actions.shape != h["shape"] or actions.dtype is not torch.int64:
                raise RuntimeError(f"actions must be int64 ({self._n},)")
            ptr = actions.data_ptr()
            if ptr != h["pinned_ptr"]:  # pinned-ness checked once per buffer address
                if not (actions.is_contiguous() and actions.is_pinned()):
                    h["act"].copy_(actions)
                    ptr = h["act"].data_ptr()
                else:
                    h["pinned_ptr"] = ptr
            io.actions_host = ptr
        io.sync = 1 if sync else 0
        pol = h["pol"].get(policy)
        if pol is None:
            pol = h["pol"][policy] = ctypes.byref(self._policy(policy, None))
        dev = self._device_id
        if torch.cuda.current_device() != dev:
            with torch.cuda.device(self.device):
                rc = h["fn"](h["st"], h["bio"][mode], self._ply, pol, 1 if auto_reset else 0,
                             h["out"][mode][bool(observe)],
                             _raw_stream(dev) if stream is None else stream.cuda_stream)
        else:
            rc = h["fn"](h["st"], h["bio"][mode], self._ply, pol, 1 if auto_reset else 0,
                         h["out"][mode][bool(observe)], _raw_stream(dev) if stream is None else stream.cuda_stream)
        if rc:
            C.check(rc)
        self._ply += 1
        return h["ret"][mode][bool(observe)]

    def _host_io(self) -> dict:
        if self._host is None:
            o = self._ensure_outputs()
            n, lay = self._n, _results_layout(self._n)
            back = torch.zeros(lay["bytes"], dtype=torch.uint8, pin_memory=True)
            host = {f: _results_view(back, lay, f, n) for f in ("reward", "next_action", "done")}
            d_act = self._alloc((max(n, 1),), torch.int64)
            io = {
                "copy": C.SbHostIo(actions_host=None, actions_dev=d_act.data_ptr(), back_dev=o["results"].data_ptr(),
                                   back_host=back.data_ptr(), back_bytes=lay["bytes"], sync=1, reserved=0),
                "mapped": C.SbHostIo(actions_host=None, actions_dev=None, back_dev=None, back_host=None, back_bytes=0,
                                     sync=1, reserved=0),
            }
            outs, rets = {"copy": {}, "mapped": {}}, {"copy": {}, "mapped": {}}
            for observe in (False, True):
                dev_views = self._step_views(o, observe)
                outs["copy"][observe] = self._step_out(o, observe)
                m = self._step_out(o, observe)
                m.reward, m.done, m.next_action = (host["reward"].data_ptr(), host["done"].data_ptr(),
                                                   host["next_action"].data_ptr())
                outs["mapped"][observe] = m
                for mode in ("copy", "mapped"):
                    dv = dev_views if mode == "copy" else StepOutput(
                        **{**dev_views.__dict__, "reward": host["reward"], "done": host["done"].view(torch.bool),
                           "next_action": host["next_action"]})
                    rets[mode][observe] = HostStepOutput(reward=host["reward"], done=host["done"].view(torch.bool),
                                                         next_action=host["next_action"], device=dv)
            # the per-call path reuses prebuilt ctypes arguments
            self._host = {
                "back": back, "d_act": d_act, "ret": rets, "pol": {}, "io": io, "shape": torch.Size([n]),
                "act": torch.zeros(max(n, 1), dtype=torch.int64, pin_memory=True)[:n], "pinned_ptr": None,
                "fn": C.lib().sb_step_host, "st": ctypes.byref(self._st),
                "bio": {k: ctypes.byref(v) for k, v in io.items()},
                "out": {k: {b: ctypes.byref(x) for b, x in v.items()} for k, v in outs.items()}, "outs": outs,
            }
        return self._host

    def serve(self, **kw):
        """A persistent step server over this buffer (``ataraxos_b200.serve.StepServer``)."""
        from .serve import StepServer

        return StepServer(self, **kw)

    def episode_stats(self) -> torch.Tensor:
        """int64 [5]: games finished in step(), red wins, blue wins, draws, Σ lengths."""
        return self._ensure_outputs()["stats"]

    def sample_actions(self, policy: str = "uniform", logits: torch.Tensor | None = None,
                       ply: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Sample one legal action per game for the current state: (int64 [N], log-prob [N])."""
        acts = self._alloc((self._n,), torch.int64)
        lp = self._alloc((self._n,), torch.float32)
        pol = self._policy(policy, logits)
        if self._n:
            self._call("sb_sample_actions", self._ply if ply is None else int(ply), ctypes.byref(pol),
                       acts.data_ptr(), lp.data_ptr())
        return acts, lp

    def resample_from(self, roots: "StrategoRolloutBuffer", root_of: torch.Tensor) -> None:
        """Belief resampling: env e becomes a copy of ``roots`` env ``root_of[e]`` with
        the side-not-to-move's unrevealed identities re-dealt uniformly among the
        deals consistent with what the side to move has seen (moved pieces are
        never a Bomb or the Flag).  Keyed by this buffer's seed and env indices."""
        if root_of.dtype != torch.int64 or root_of.numel() != self._n:
            raise RuntimeError("root_of must be int64 [n_games]")
        r = root_of.to(self.device).contiguous()
        with torch.cuda.device(self.device):
            C.call("sb_belief_resample", ctypes.byref(roots._st), ctypes.byref(self._st), r.data_ptr(),
                   _stream(self.device))

    def export_state(self) -> dict[str, torch.Tensor]:
        """Every state field in the reference's tensor layout (cpp:24-55), plus
        ``chase_hashes`` [N,2,64], ``episode`` and ``invalid_count``."""
        shapes = {
            "board_owner": ((self._n, 10, 10), torch.int8), "board_piece": ((self._n, 10, 10), torch.int8),
            "current_player": ((self._n,), torch.int8), "outcome": ((self._n,), torch.int8),
            "terminated": ((self._n,), torch.uint8), "flag_captured": ((self._n,), torch.uint8),
            "move_number": ((self._n,), torch.int32), "moves_since_attack": ((self._n,), torch.int32),
            "terminated_since": ((self._n,), torch.int32), "moved_squares": ((self._n, 100), torch.uint8),
            "revealed_squares": ((self._n, 100), torch.uint8), "move_history": ((self._n, 32), torch.int32),
            "move_history_head": ((self._n,), torch.int32), "move_history_len": ((self._n,), torch.int32),
            "two_square_count": ((self._n, 2), torch.int32), "two_square_pair_lo": ((self._n, 2), torch.int32),
            "two_square_pair_hi": ((self._n, 2), torch.int32), "two_square_violation": ((self._n,), torch.uint8),
            "chase_hash_head": ((self._n, 2), torch.int32), "chase_hash_len": ((self._n, 2), torch.int32),
            "chase_last_src": ((self._n, 2), torch.int32), "chasing_violation": ((self._n,), torch.uint8),
            "episode": ((self._n,), torch.int32), "invalid_count": ((self._n,), torch.int32),
            "reward": ((self._n,), torch.float32),
            "isf_two_square": ((self._n, 100, 6), torch.uint8), "isf_threats": ((self._n, 2, 4), torch.int8),
            "isf_evasion": ((self._n, 2), torch.uint8),
        }
        outs = {k: self._alloc(s, d) for k, (s, d) in shapes.items()}
        ex = C.SbExport(**{k: v.data_ptr() for k, v in outs.items()})
        if self._n:
            self._call("sb_export_state", ctypes.byref(ex))
        outs["chase_hashes"] = self._ring[: self._n].clone()
        return outs

    def clone(self) -> "StrategoRolloutBuffer":
        """A new buffer on the same device holding a copy of every game (same
        seed, env indices, limits, pool and Zobrist table); the two then
        evolve independently."""
        c = StrategoRolloutBuffer(
            self._n, self._device_id, seed=self.seed, env_base=self.env_base, setup_pool=self._pool,
            no_attack_limit=self.no_attack_limit, max_game_length=self.max_game_length,
            two_square_limit=self.two_square_limit, zobrist=self._zobrist, obs_dtype=self.obs_dtype,
            obs_layout=self.obs_layout, mask_format=self.mask_format, rules=self.rules)
        c.load_state_dict(self.state_dict())
        return c

    def state_dict(self) -> dict:
        """Everything needed to resume bit-exactly."""
        return {
            "records": self._records.clone(),
            "chase_ring": self._ring.clone(),
            "ply": self._ply,
            "seed": self.seed,
            "env_base": self.env_base,
            "setup_pool": None if self._pool is None else self._pool.clone(),
            "zobrist": self._zobrist.clone(),
            "limits": (self.no_attack_limit, self.max_game_length, self.two_square_limit),
            "rules": self.rules,
            "isf_two_square": None if self._isf is None else self._isf.clone(),
        }

    def load_state_dict(self, sd: dict) -> None:
        if tuple(sd["records"].shape) != tuple(self._records.shape):
            raise RuntimeError("state_dict was saved from a buffer with a different n_games")
        self._records.copy_(sd["records"])
        self._ring.copy_(sd["chase_ring"])
        self._ply = int(sd["ply"])
        self.seed = int(sd["seed"])
        self.env_base = int(sd["env_base"])
        self.no_attack_limit, self.max_game_length, self.two_square_limit = map(int, sd["limits"])
        self._zobrist.copy_(sd["zobrist"])
        if sd.get("setup_pool") is not None:
            self._pool = sd["setup_pool"].to(self.device).contiguous()
        if sd.get("rules", "cuda") != self.rules:
            raise RuntimeError("state_dict was saved from a buffer with other repetition rules")
        if self._isf is not None:
            self._isf.copy_(sd["isf_two_square"])
        self._st = self._make_state()
