"""The C ABI from a C program on the B200.

``tests/c_host/c_host_loop.c`` includes only ``include/stratego_b200.h`` and
links ``libstratego_b200.so`` and the CUDA runtime: it allocates the state and
the outputs itself, builds the setup pool, resets every game from it and plays
300 plies through ``sb_step_host`` with host actions and results in
page-locked memory, the games split into 1 or 3 states over contiguous slices
of the same arrays (each on its own stream, stepped in turn).  Every ply's
rewards, dones and proposed actions, and the final game records, must equal
what ``StrategoRolloutBuffer.step_host`` gives for the same games from Python.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
SRC = Path(__file__).resolve().parent / "c_host" / "c_host_loop.c"


@pytest.fixture(scope="module")
def c_host(tmp_path_factory):
    from ataraxos_b200 import _capi as C

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler on this machine")
    cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    lib_dir = Path(C.LIB_PATH).resolve().parent
    exe = tmp_path_factory.mktemp("c_host") / "c_host_loop"
    cmd = [gcc, "-O2", "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}", f"-I{cuda / 'include'}",
           str(SRC), f"-L{lib_dir}", "-lstratego_b200", f"-L{cuda / 'lib64'}", "-lcudart",
           f"-Wl,-rpath,{lib_dir}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def _python_run(n: int, plies: int):
    from ataraxos_b200 import StrategoRolloutBuffer

    buf = StrategoRolloutBuffer(n, 0, seed=7, pool_size=4096)
    buf.reset_all_from_pool()
    r = buf.step_host(None)
    log = []
    for t in range(plies):
        log.append((r.reward.numpy().copy(), r.done.view(torch.uint8).numpy().copy(), r.next_action.numpy().copy()))
        if t + 1 < plies:
            r = buf.step_host(r.next_action.to(torch.int64))
    torch.cuda.synchronize()
    return log, buf._records[:n].cpu().numpy()


@pytest.mark.parametrize("groups", [1, 3])
def test_c_program_equals_python_step_host(c_host, tmp_path, groups):
    from ataraxos_b200 import zobrist_table

    n, plies = 1000, 300
    zob = tmp_path / "zobrist.bin"
    zob.write_bytes(np.ascontiguousarray(zobrist_table(), dtype=np.int64).tobytes())
    out = tmp_path / "out.bin"
    r = subprocess.run([str(c_host), str(n), str(plies), str(groups), str(zob), str(out)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "status 0" in r.stdout
    raw = out.read_bytes()
    per_ply = n * (4 + 1 + 2)
    assert len(raw) == plies * per_ply + n * 256
    ref, ref_rec = _python_run(n, plies)
    for t in range(plies):
        b = raw[t * per_ply:(t + 1) * per_ply]
        rew = np.frombuffer(b[:4 * n], dtype=np.float32)
        done = np.frombuffer(b[4 * n:5 * n], dtype=np.uint8)
        nxt = np.frombuffer(b[5 * n:], dtype=np.int16)
        np.testing.assert_array_equal(rew, ref[t][0], err_msg=f"reward, ply {t}")
        np.testing.assert_array_equal(done, ref[t][1], err_msg=f"done, ply {t}")
        np.testing.assert_array_equal(nxt, ref[t][2], err_msg=f"next action, ply {t}")
    rec = np.frombuffer(raw[plies * per_ply:], dtype=np.uint8).reshape(n, 256)
    np.testing.assert_array_equal(rec, ref_rec, err_msg="final game records")
    assert sum(int(d.sum()) for _, d, _ in ref) > 0  # games ended (and were reset) on the way
