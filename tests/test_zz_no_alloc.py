"""rt_gemv_bf16_argmax_static (the allocation-free greedy LM-head GEMV) against
the context-based rt_gemv_bf16 on the same device buffers, two calls in a row.

Collected last on purpose (file name), and self-contained, so it passes both
alone in a fresh process and after the rest of the suite."""

import ctypes

import numpy as np
import pytest

from rich_triplet_b200._lib import RT_DEVICE, RT_E_INVAL, RT_E_SHAPE, RT_FMT_BF16, RT_OK, lib
from rich_triplet_b200.model import synth_normal, synth_normal_bf16

pytestmark = pytest.mark.gpu

RTOL = 1e-3  # the GEMV tolerance: floored relative error of y


def _greedy(y):
    """Index of the largest value, ties to the higher index (sample_greedy)."""
    m = y.max()
    return int(np.nonzero(y == m)[0][-1])


def _static(w_ptr, rows, cols, x, y, tok, stream=None):
    err = ctypes.create_string_buffer(256)
    rc = lib().rt_gemv_bf16_argmax_static(
        ctypes.c_void_p(w_ptr), rows, cols, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
        ctypes.c_void_p(tok.data_ptr()), stream, err, len(err))
    return rc, err.value.decode()


def test_static_argmax_matches_context_gemv_twice():
    import torch

    from rich_triplet_b200.ops import Context, DeviceWeight

    rows, cols = 40000, 2560
    ctx = Context(0)
    try:
        w = DeviceWeight.upload(ctx, RT_FMT_BF16, synth_normal_bf16(77, 1, rows * cols, 0.0, 0.05), rows, cols)
        ctx.sync()
        for call, seed in enumerate((5, 6)):  # two calls in a row, different activations
            x = torch.from_numpy(synth_normal(seed, 2, cols)).cuda()
            y_ref = torch.empty(rows, dtype=torch.float32, device="cuda")
            y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
            tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            rc = lib().rt_gemv_bf16(ctx.h, w.h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y_ref.data_ptr()),
                                    RT_DEVICE)
            assert rc == RT_OK, ctx.last_error()
            ctx.sync()
            rc, msg = _static(w.device_ptr, rows, cols, x, y, tok)
            assert rc == RT_OK, msg
            torch.cuda.synchronize()
            yr, ys = y_ref.cpu().numpy(), y.cpu().numpy()
            floor = np.abs(yr).max() * 1e-3
            rel = np.abs(ys - yr) / np.maximum(np.abs(yr), floor)
            assert rel.max() < RTOL, (call, rel.max())
            t = int(tok.cpu().item())
            assert t == _greedy(ys), (call, t)
            assert t == _greedy(yr), (call, t)
    finally:
        ctx.close()


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
