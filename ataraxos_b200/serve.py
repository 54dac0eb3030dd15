"""Persistent step server: a host-driven loop of fused plies without a kernel
launch or a stream synchronisation per ply.

``StepServer(buf)`` (or ``buf.serve()``) launches one persistent kernel that
plays a ply of every game each time ``step()`` publishes one in a control
block of mapped page-locked host memory: it reads that step's actions from
page-locked host memory (or plays the cached device proposals when the step
has none), applies them with auto-reset and writes every output to the
buffer's device outputs; the CTA that completes the step copies the result
block (reward / next action / done) into page-locked host memory and tells
the host.  ``step()`` returns then.  The kernel ends on ``close()`` (or when no step comes for
``limit_s``).  While it runs, nothing else may use the buffer, and other
kernels on the GPU wait for free SMs (the server keeps every CTA resident);
it runs on a stream of its own (``stream``).

This is the host loop of ``SelfPlayGenerator.generate_games``
(stratego/training/selfplay.py:190-268) when its policy lives on the host:
one call per ply, each ply's actions in and results out.
"""

from __future__ import annotations

import ctypes

import torch

from . import _capi as C
from .buffer import HostStepOutput, _results_layout, _results_view, _vp

TIMEOUT_NS = 10_000_000_000  # the host's wait for one step


class StepServer:
    """Context manager around the persistent step kernel of one buffer."""

    def __init__(self, buf, *, auto_reset: bool = True, limit_s: float = 2.0, host_actions: bool = True,
                 stream: torch.cuda.Stream | None = None) -> None:
        if buf.mask_format not in ("u8", "none") or buf.obs_layout != "dense":
            raise RuntimeError("the step server writes the dense infostate and the u8 mask")
        if buf.rules != "cuda":
            raise RuntimeError("the step server runs the CUDA repetition rules")
        self.buf = buf
        n = buf.n_games
        o = buf._ensure_outputs()
        lay = _results_layout(n)
        self._back = torch.zeros(lay["bytes"], dtype=torch.uint8, pin_memory=True)
        self.actions = torch.zeros(max(n, 1), dtype=torch.int64, pin_memory=True)[:n]
        self._host_actions = bool(host_actions)
        self._ctl = torch.zeros(17, dtype=torch.int64, pin_memory=True)
        self._dev = torch.zeros(4, dtype=torch.int64, device=buf.device)
        # the device results block (reward | next_action | done) is copied
        # whole into the page-locked block of the same layout after each step
        self._sv = C.SbServe(ctl=self._ctl.data_ptr(), dev=self._dev.data_ptr(), back_dev=o["results"].data_ptr(),
                             back_host=self._back.data_ptr(), back_bytes=lay["bytes"], n_ctas=0,
                             limit_ns=int(limit_s * 1e9))
        self._out = buf._step_out(o, True)
        host = {f: _results_view(self._back, lay, f, n) for f in ("reward", "next_action", "done")}
        self._ret = HostStepOutput(reward=host["reward"], done=host["done"].view(torch.bool),
                                   next_action=host["next_action"], device=buf._step_views(o, True))
        self._t = 0
        self._ply0 = buf.ply
        self._open = False
        self._auto_reset = bool(auto_reset)
        self.stream = stream

    @staticmethod
    def max_envs(device) -> int:
        """Envs one server can hold on `device`: every CTA (7 games each) resident, 4 per SM."""
        return torch.cuda.get_device_properties(device).multi_processor_count * 4 * 7

    def __enter__(self) -> "StepServer":
        self.start()
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def start(self) -> None:
        b = self.buf
        with torch.cuda.device(b.device):
            # the server's inputs and outputs must be ready before it starts
            torch.cuda.current_stream(b.device).synchronize()
            if self.stream is None:
                self.stream = torch.cuda.Stream(b.device)
            C.call("sb_serve_start", ctypes.byref(b._st), self._ply0, int(self._auto_reset),
                   _vp(self.actions) if self._host_actions else None, ctypes.byref(self._out),
                   ctypes.byref(self._sv), ctypes.c_void_p(self.stream.cuda_stream))
        self._open = True
        self._lib = C.lib()

    def step(self, actions: torch.Tensor | None = None) -> HostStepOutput:
        """One ply of every game.  ``actions``: CPU int64 [N] (copied into the
        server's page-locked ``actions`` unless it is that tensor) or None to
        play the cached proposals (the server must then have been made with
        ``host_actions=False``)."""
        if not self._open:
            raise RuntimeError("the step server is not running")
        if actions is not None:
            if not self._host_actions:
                raise RuntimeError("this server plays device proposals (host_actions=False)")
            if actions.data_ptr() != self.actions.data_ptr():
                if actions.device.type != "cpu" or actions.dtype != torch.int64 or actions.shape != self.actions.shape:
                    raise RuntimeError(f"actions must be CPU int64 ({self.buf.n_games},)")
                self.actions.copy_(actions)
        elif self._host_actions:
            raise RuntimeError("this server reads host actions every step")
        self._t += 1
        rc = self._lib.sb_serve_step(ctypes.byref(self._sv), self._t, TIMEOUT_NS)
        if rc:
            C.check(rc)
        return self._ret

    def close(self) -> None:
        if not self._open:
            return
        self._open = False
        b = self.buf
        with torch.cuda.device(b.device):
            C.call("sb_serve_stop", ctypes.byref(self._sv), self._t, ctypes.c_void_p(self.stream.cuda_stream))
        b.ply = self._ply0 + self._t
