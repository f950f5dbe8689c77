"""Failure paths that need a GPU but fault none: an allocation that fails on
the host side (RT_FAULT_INJECT_ALLOC) and a peer all-reduce whose partner
rank never arrives (a bounded wait that gives up and reports)."""

import ctypes
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_INJECT = r"""
import sys
sys.path.insert(0, sys.argv[1])
from rich_triplet_b200 import RtError
from rich_triplet_b200._lib import RT_E_NOMEM
from rich_triplet_b200.decode import CudaDecodeContext
from rich_triplet_b200.model import Config4, synth_gemma3
from rich_triplet_b200.ops import Context
ctx = Context(0)  # allocation 1: the context's error word
w = synth_gemma3(Config4.tiny(), seed=3)
try:
    CudaDecodeContext(w, 16, ctx)
    print("RESULT no-error")
except RtError as e:
    print("RESULT", e.code, str(e).splitlines()[0])
ctx.close()
print("DONE")
"""


@pytest.mark.parametrize("nth", [2, 5, 40])
def test_injected_allocation_failure_is_reported(nth):
    """RT_FAULT_INJECT_ALLOC=N makes the library's N-th device allocation fail
    with RT_E_NOMEM.  Engine construction must return that status (no crash,
    no hang) and release what it had allocated."""
    env = dict(os.environ, RT_FAULT_INJECT_ALLOC=str(nth))
    out = subprocess.run([sys.executable, "-c", _INJECT, ROOT], capture_output=True, text=True, timeout=300, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    line = [ln for ln in out.stdout.splitlines() if ln.startswith("RESULT")][-1]
    from rich_triplet_b200._lib import RT_E_NOMEM
    assert line.split()[1] == str(RT_E_NOMEM), line
    assert "injected allocation failure" in line
    assert "DONE" in out.stdout


def test_peer_allreduce_wait_gives_up_and_reports(gpu_ctx):
    """Rank 0 of a two-rank peer all-reduce whose partner never raises its
    flag: the first call's bounded wait gives up after ~2 s and sets the error
    word to kErrGridTimeout (3); the second call sees the word and does not
    wait at all."""
    from rich_triplet_b200._lib import RT_OK, lib

    err = ctypes.c_int(0)
    t1, t2 = ctypes.c_float(0), ctypes.c_float(0)
    rc = lib().rt_test_peer_allreduce_lonely(gpu_ctx.h, ctypes.byref(err), ctypes.byref(t1), ctypes.byref(t2))
    assert rc == RT_OK, gpu_ctx.last_error()
    assert err.value == 3
    assert 1500.0 < t1.value < 10000.0, t1.value
    assert t2.value < 100.0, t2.value
