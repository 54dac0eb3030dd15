"""The debug build's bounds checks (libstratego_b200_debug.so, SB_DEBUG_BOUNDS).

A child process loads the debug library (``ATARAXOS_B200_DEBUG=1``), plays
two identical buffers, then overwrites four game records of one of them with
indices no kernel may use (a piece code of 13, a history-ring head of 40, a
chase-ring head of 70, a history entry of 20000).  Further steps must skip
exactly those games -- their records untouched, SB_STATUS_BAD_STATE raised --
and play every other game exactly as the twin buffer does.  The corrupted
records are only ever given to the debug build, whose checks run before any
use of a record.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

CHILD = r"""
import os, sys
sys.path.insert(0, sys.argv[1])
import numpy as np
import torch
from ataraxos_b200 import StrategoRolloutBuffer, _capi as C
import oracle

assert C.DEBUG and C.lib().sb_debug_bounds() == 1
pool = torch.from_numpy(oracle.make_setup_pool(3, 256))
bufs = [StrategoRolloutBuffer(64, 0, seed=3, setup_pool=pool) for _ in range(2)]
for b in bufs:
    b.reset_all_from_pool()
    for _ in range(12):
        b.step(None)
a, b = bufs
rec = a._records
R_BOARD, R_HHEAD, R_HLEN, R_CHHEAD, R_HIST = 0, 116, 117, 136, 176
rec[3, R_BOARD + 11] = 32 | 13                   # occupied, piece code 13
rec[5, R_HHEAD] = 40                             # history head beyond the 32-entry ring
rec[7, R_CHHEAD + 1] = 70                        # chase head beyond the 64-entry ring
hh, hl = int(rec[9, R_HHEAD]), int(rec[9, R_HLEN])
assert hl >= 1
slot = R_HIST + 2 * ((hh - 1) & 31)
rec[9, slot:slot + 2] = torch.tensor(np.frombuffer(np.int16(20000).tobytes(), np.uint8))
bad = [3, 5, 7, 9]
good = [g for g in range(64) if g not in bad]
before = rec.clone()
assert a.status() == 0
for _ in range(6):
    oa, ob = a.step(None), b.step(None)
    assert torch.equal(oa.action[good], ob.action[good])
    assert torch.equal(oa.infostate[good], ob.infostate[good])
    assert torch.equal(oa.legal_mask[good], ob.legal_mask[good])
torch.cuda.synchronize()
assert a.status() & C.SB_STATUS_BAD_STATE, a.status()
assert torch.equal(a._records[bad], before[bad]), "skipped games were modified"
assert torch.equal(a._records[good], b._records[good]), "the other games diverged"
assert b.status() == 0
print("debug bounds ok")
"""


def test_debug_build_skips_corrupt_records_and_plays_the_rest():
    lib = ROOT / "ataraxos_b200" / "_lib" / "libstratego_b200_debug.so"
    assert lib.exists(), "the debug library is built by ataraxos_b200.build"
    env = dict(os.environ, ATARAXOS_B200_DEBUG="1")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "debug bounds ok" in r.stdout
