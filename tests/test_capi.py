"""The C ABI library: it loads without a GPU, exports every declared symbol, and
its structs have the layout the Python binding assumes.  No kernel is launched."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from ataraxos_b200 import _capi as C
from ataraxos_b200 import build as B

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "stratego_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char \*)\s*(sb_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_reports_abi():
    lib = C.lib()
    assert lib.sb_abi_version() == 2
    assert Path(C.LIB_PATH).exists()


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_functions()
    assert len(names) >= 15
    lib = ctypes.CDLL(str(C.LIB_PATH))
    for name in names:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
        assert name in C.exported_symbols(), f"{name} not bound in ataraxos_b200/_capi.py"
    out = subprocess.run(["nm", "-D", "--defined-only", str(C.LIB_PATH)], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
    assert set(names) <= exported


def test_library_is_built_for_sm100a():
    # the build command targets exactly sm_100a, no other architecture
    flags = " ".join(B.NVCC_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags
    assert flags.count("-gencode") == 1


def test_errors_are_reported_without_a_gpu():
    st = C.SbState(n=-1)
    rc = C.lib().sb_init_state(ctypes.byref(st), None)
    assert rc == C.SB_E_ARG
    assert b"n < 0" in C.lib().sb_last_error()
    rc = C.lib().sb_make_setup_pool(0, -1, 1, None, None)
    assert rc == C.SB_E_ARG


_LAYOUT_PROG = r"""
#include <stdio.h>
#include <stddef.h>
#include "stratego_b200.h"
int main(void) {
  printf("%zu %zu %zu %zu\n", sizeof(sb_state), sizeof(sb_step_out), sizeof(sb_policy), sizeof(sb_export));
  printf("%zu %zu %zu\n", offsetof(sb_state, seed), offsetof(sb_state, status), offsetof(sb_step_out, stats));
  return 0;
}
"""


def test_struct_layouts_match_the_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(_LAYOUT_PROG)
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), "-o", str(exe), str(src)], check=True)
    lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    sizes = [int(x) for x in lines[0].split()]
    offs = [int(x) for x in lines[1].split()]
    assert sizes == [ctypes.sizeof(C.SbState), ctypes.sizeof(C.SbStepOut), ctypes.sizeof(C.SbPolicy),
                     ctypes.sizeof(C.SbExport)]
    assert offs == [C.SbState.seed.offset, C.SbState.status.offset, C.SbStepOut.stats.offset]


@pytest.mark.parametrize("name", ["sb_step", "sb_apply_actions", "sb_infostate", "sb_legal_mask_u8"])
def test_null_state_is_rejected(name):
    fn = getattr(C.lib(), name)
    args = [0 if t in (ctypes.c_int, ctypes.c_int64) else None for t in fn.argtypes]
    assert fn(*args) == C.SB_E_ARG


def test_step_pipeline_refuses_bad_group_counts_before_allocating():
    """StepPipeline checks its group count before it builds any buffer (so
    these refusals need no GPU)."""
    from ataraxos_b200.pipeline import StepPipeline

    with pytest.raises(RuntimeError, match="groups must be >= 1"):
        StepPipeline(64, 0, groups=0)
    with pytest.raises(RuntimeError, match="at least one game"):
        StepPipeline(3, 0, groups=4)


def test_c_host_compiles_and_links_against_the_header_and_library(tmp_path):
    """A C program written only against include/stratego_b200.h
    (tests/c_host/c_host_loop.c) compiles warning-free as C11 and links against
    libstratego_b200.so; tests/test_gpu_c_host.py runs it on a GPU."""
    import os
    import shutil

    gcc = shutil.which("gcc")
    cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    if gcc is None or not (cuda / "include" / "cuda_runtime.h").exists():
        pytest.skip("no C compiler or CUDA runtime headers here")
    lib_dir = Path(C.LIB_PATH).resolve().parent
    exe = tmp_path / "c_host_loop"
    r = subprocess.run([gcc, "-O2", "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
                        f"-I{cuda / 'include'}", str(ROOT / "tests" / "c_host" / "c_host_loop.c"), f"-L{lib_dir}",
                        "-lstratego_b200", f"-L{cuda / 'lib64'}", "-lcudart", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert exe.exists()
