"""rt_gemv_bf16_argmax_static (the allocation-free greedy LM-head GEMV)
against the context-based rt_gemv_bf16 on the same device buffers and against
the CPU oracle (MatBf16::gemv_mt, src/autograd2.rs:954-1000, and
sample_token at temperature 0, src/transformer4.rs:3036-3091), two calls in a
row per shape.

Collected last on purpose (file name), and self-contained, so it passes both
alone in a fresh process and after the rest of the suite."""

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

from rich_triplet_b200._lib import RT_DEVICE, RT_E_INVAL, RT_E_SHAPE, RT_FMT_BF16, RT_OK, lib
from rich_triplet_b200.model import synth_normal, synth_normal_bf16
from rich_triplet_b200.spec import greedy_token

pytestmark = pytest.mark.gpu

RTOL = 1e-3  # the GEMV tolerance: floored relative error of y
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rel(y, ref):
    floor = np.abs(ref).max() * 1e-3
    return float((np.abs(y - ref) / np.maximum(np.abs(ref), floor)).max())


def _static(w_ptr, rows, cols, x, y, tok, stream=None):
    err = ctypes.create_string_buffer(256)
    rc = lib().rt_gemv_bf16_argmax_static(
        ctypes.c_void_p(w_ptr), rows, cols, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
        ctypes.c_void_p(tok.data_ptr()), stream, err, len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("rows, cols", [(40000, 2560), (262145, 2560), (17, 8)])
def test_static_argmax_matches_context_gemv_and_oracle_twice(orc, rows, cols):
    """Shapes: the common case; a 4B-sized LM head with rows % 16 != 0 (the
    last tile split); and a tiny one.  Two calls in a row with different
    activations show the counters return to zero between calls."""
    import torch

    from rich_triplet_b200.ops import Context, DeviceWeight

    ctx = Context(0)
    try:
        wh = synth_normal_bf16(77, 1, rows * cols, 0.0, 0.05)
        w = DeviceWeight.upload(ctx, RT_FMT_BF16, wh, rows, cols)
        ctx.sync()
        for call, seed in enumerate((5, 6)):
            xh = synth_normal(seed, 2, cols)
            x = torch.from_numpy(xh).cuda()
            y_ref = torch.empty(rows, dtype=torch.float32, device="cuda")
            y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
            tok = torch.full((1,), -2, dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            rc = lib().rt_gemv_bf16(ctx.h, w.h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y_ref.data_ptr()),
                                    RT_DEVICE)
            assert rc == RT_OK, ctx.last_error()
            ctx.sync()
            rc, msg = _static(w.device_ptr, rows, cols, x, y, tok)
            assert rc == RT_OK, msg
            torch.cuda.synchronize()
            yr, ys = y_ref.cpu().numpy(), y.cpu().numpy()
            assert _rel(ys, yr) < RTOL, (call, _rel(ys, yr))
            yo = orc.bf16_gemv(wh, rows, cols, xh)
            assert _rel(ys, yo) < RTOL, (call, _rel(ys, yo))
            t = int(tok.cpu().item())
            # the device token follows sample_token's rule on the device's own y ...
            assert t == orc.sample_greedy(ys) == greedy_token(ys), (call, t)
            # ... and on the oracle's y, unless the top two are closer than the GEMV tolerance
            top2 = np.sort(yo)[-2:]
            if top2[1] - top2[0] > 1e-5 * np.abs(yo).max():
                assert t == orc.sample_greedy(yo), (call, t)
    finally:
        ctx.close()


def test_static_argmax_near_tie_takes_the_later_row():
    """Logits one f32 ulp apart: at 0.125 exp() of their difference rounds to
    1, so sample_token's softmax ties them and the LATER row wins although its
    logit is smaller; at 4.0 the larger logit wins.  y = W x with x = (1,
    2^-20, 0, ...) makes row r's logit W[r,0] + 2^-20 W[r,1] exactly."""
    import torch

    rows, cols = 1000, 256
    w = torch.zeros((rows, cols), dtype=torch.bfloat16)
    w[:, 0] = -10.0
    x = torch.zeros(cols, dtype=torch.float32)
    x[0] = 1.0
    x[1] = 2.0 ** -20
    # (base, W[hi_row, 1], expected row): 2^-20 * 2^-6 = 2^-26 = ulp(0.125);
    # 2^-20 * 2^-1 = 2^-21 = ulp(4.0)
    for base, w1, want in ((0.125, 2.0 ** -6, 700), (4.0, 0.5, 10)):
        hi_row, lo_row = 10, 700
        wc = w.clone()
        wc[hi_row, 0] = base
        wc[hi_row, 1] = w1
        wc[lo_row, 0] = base
        wd, xd = wc.cuda(), x.cuda()
        y = torch.empty(rows, dtype=torch.float32, device="cuda")
        tok = torch.full((1,), -2, dtype=torch.int32, device="cuda")
        rc, msg = _static(wd.data_ptr(), rows, cols, xd, y, tok)
        assert rc == RT_OK, msg
        torch.cuda.synchronize()
        yh = y.cpu().numpy()
        assert yh[hi_row] == np.nextafter(np.float32(base), np.float32(np.inf)) and yh[lo_row] == base
        assert int(tok.item()) == want == greedy_token(yh), (base, int(tok.item()))


def test_static_argmax_rejects_bad_arguments():
    import torch

    x = torch.zeros(256, dtype=torch.float32, device="cuda")
    y = torch.zeros(16, dtype=torch.float32, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    w = torch.zeros(16 * 256, dtype=torch.bfloat16, device="cuda")
    rc, msg = _static(0, 16, 256, x, y, tok)
    assert rc == RT_E_INVAL and "null" in msg
    rc, msg = _static(w.data_ptr(), 16, 250, x, y, tok)
    assert rc == RT_E_SHAPE and "multiple of 8" in msg
    rc, msg = _static(w.data_ptr(), (1 << 20) + 1, 256, x, y, tok)
    assert rc == RT_E_SHAPE and "rows" in msg
    rc, msg = _static(w.data_ptr() + 2, 16, 256, x, y, tok)
    assert rc == RT_E_INVAL and "aligned" in msg


_GIVE_UP = r"""
import ctypes, json, os, sys
sys.path.insert(0, sys.argv[1])
import numpy as np, torch
from rich_triplet_b200._lib import lib
from rich_triplet_b200.spec import greedy_token
rows, cols = 65536, 2560
w = torch.randn(rows, cols, device="cuda").to(torch.bfloat16)
x = torch.randn(cols, device="cuda")
y = torch.empty(rows, device="cuda")
tok = torch.full((1,), -2, dtype=torch.int32, device="cuda")
err = ctypes.create_string_buffer(256)
def call():
    rc = lib().rt_gemv_bf16_argmax_static(ctypes.c_void_p(w.data_ptr()), rows, cols, ctypes.c_void_p(x.data_ptr()),
                                          ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(tok.data_ptr()), None, err, 256)
    assert rc == 0, err.value
    torch.cuda.synchronize()
    return int(tok.item()), greedy_token(y.cpu().numpy())
call()  # set-up outside the forced failure
os.environ["RT_TEST_MBAR_WAIT_ITERS"] = "1"
bad = call()[0]
del os.environ["RT_TEST_MBAR_WAIT_ITERS"]
good = [call(), call()]
print("RESULT " + json.dumps({"bad": bad, "good": good}))
"""


def test_static_argmax_reports_a_bounded_wait_that_gave_up():
    """With each weight-stream wait bounded to one poll (the test override
    RT_TEST_MBAR_WAIT_ITERS), the bounded waits give up: the launch reports
    token -1 and returns its counters to zero, so the next calls are right
    again.  Run in a child process: nothing of it leaks into the suite."""
    out = subprocess.run([sys.executable, "-c", _GIVE_UP, ROOT], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    import json

    line = [ln for ln in out.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    res = json.loads(line[len("RESULT "):])
    assert res["bad"] == -1
    (t1, r1), (t2, r2) = res["good"]
    assert t1 == r1 and t2 == r2 and t1 == t2
