"""Q4_K and BF16 GEMV kernels vs the CPU oracle (Q4KMat / MatBf16 gemv_mt)."""

import ctypes

import numpy as np
import pytest

from rich_triplet_b200 import RtError
from rich_triplet_b200._lib import RT_DEVICE, RT_FMT_BF16, RT_FMT_Q4K, RT_HOST, lib
from rich_triplet_b200.model import MatBf16, Q4KMat, synth_normal, synth_normal_bf16, synth_q4k
from rich_triplet_b200.ops import DeviceWeight, cuda_gemv_bf16_t, cuda_gemv_q4k_t

pytestmark = pytest.mark.gpu

# Tolerance: the reference's GEMV test bound, max relative error 1e-3
# (src/metal_ops.rs:1171-1178).  For random data the denominator is floored at
# 1e-2 * rms(y): a dot product whose terms cancel to ~0 has no meaningful
# relative error, and its absolute error is bounded by the terms' scale.
REL_TOL = 1e-3


def _rel(got, ref):
    floor = 1e-2 * float(np.sqrt(np.mean(ref.astype(np.float64) ** 2))) + 1e-30
    return np.abs(got - ref) / np.maximum(np.abs(ref), floor)


def _hex(h, dt):
    return np.frombuffer(bytes.fromhex(h), dtype=dt).copy()


def test_q4k_gemv_reference_kats(golden):
    for case in golden["q4k_gemv"]:
        q = Q4KMat(case["rows"], case["cols"], _hex(case["blocks_hex"], np.uint8))
        y = cuda_gemv_q4k_t(np.array(case["x"], np.float32), q)[0]
        exp = np.array(case["expected"], np.float32)
        rel = np.abs(y - exp) / (np.abs(exp) + 1e-6)
        assert rel.max() < case["rel_tol"], (case["name"], rel.max())


def test_q4k_gemv_cache_reuse_different_activations(golden):
    # src/metal_ops.rs:1210-1235: second call reuses the uploaded weight.
    a1, a2 = golden["q4k_gemv"][2], golden["q4k_gemv"][3]
    q = Q4KMat(a1["rows"], a1["cols"], _hex(a1["blocks_hex"], np.uint8))
    r1 = cuda_gemv_q4k_t(np.array(a1["x"], np.float32), q)[0]
    r2 = cuda_gemv_q4k_t(np.array(a2["x"], np.float32), q)[0]
    assert not np.array_equal(r1, r2)
    for r, c in ((r1, a1), (r2, a2)):
        exp = np.array(c["expected"], np.float32)
        assert (np.abs(r - exp) / (np.abs(exp) + 1e-6)).max() < 1e-3


def test_bf16_gemv_reference_kats(golden):
    for case in golden["bf16_gemv"]:
        m = MatBf16(case["rows"], case["cols"], _hex(case["w_hex"], np.uint16))
        y = cuda_gemv_bf16_t(np.array(case["x"], np.float32), m)[0]
        assert np.abs(y - np.array(case["expected"], np.float32)).max() < case["abs_tol"]


@pytest.mark.parametrize("rows,cols", [
    (10240, 2560), (2560, 10240),            # BASELINE config 0 and its transpose
    (4096, 2560), (2560, 2048), (20480, 2560),  # fused QKV, o, gate/up shapes
    (1, 256), (3, 256), (7, 512), (65, 768), (129, 1280), (300, 5376), (33, 21504), (1000, 2304),
])
def test_q4k_gemv_random_vs_oracle(orc, rows, cols):
    blocks = synth_q4k(77, rows * 7 + cols, rows, cols)
    x = synth_normal(78, rows + cols, cols)
    y = cuda_gemv_q4k_t(x, Q4KMat(rows, cols, blocks))[0]
    ref = orc.q4k_gemv(blocks, rows, cols, x)
    assert np.all(np.isfinite(y))
    assert _rel(y, ref).max() < REL_TOL


@pytest.mark.parametrize("rows,cols", [(262144 // 64, 2560), (1, 8), (5, 64), (128, 256), (77, 1000), (513, 2560),
                                       (64, 5376), (9, 4104)])
def test_bf16_gemv_random_vs_oracle(orc, rows, cols):
    w = synth_normal_bf16(91, rows + 3 * cols, rows * cols, 0.0, 0.02)
    x = synth_normal(92, cols, cols)
    y = cuda_gemv_bf16_t(x, MatBf16(rows, cols, w))[0]
    ref = orc.bf16_gemv(w, rows, cols, x)
    assert _rel(y, ref).max() < REL_TOL


def test_q4k_gemv_device_pointers(gpu_ctx, orc):
    import torch
    rows, cols = 2560, 10240
    blocks = synth_q4k(5, 5, rows, cols)
    x = synth_normal(6, 6, cols)
    w = DeviceWeight.upload(gpu_ctx, RT_FMT_Q4K, blocks, rows, cols)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(rows, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    rc = lib().rt_gemv_q4k(gpu_ctx.h, w.h, ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(yd.data_ptr()), RT_DEVICE)
    assert rc == 0
    gpu_ctx.sync()
    ref = orc.q4k_gemv(blocks, rows, cols, x)
    assert _rel(yd.cpu().numpy(), ref).max() < REL_TOL
    w.free()


def test_gemv_rejects_bad_input(gpu_ctx):
    blocks = synth_q4k(1, 1, 4, 256)
    w = DeviceWeight.upload(gpu_ctx, RT_FMT_Q4K, blocks, 4, 256)
    x = np.zeros(256, np.float32)
    y = np.zeros(4, np.float32)
    # wrong entry point for the format
    assert lib().rt_gemv_bf16(gpu_ctx.h, w.h, x.ctypes.data, y.ctypes.data, RT_HOST) == -5
    assert "format" in gpu_ctx.last_error()
    # unknown flag
    assert lib().rt_gemv_q4k(gpu_ctx.h, w.h, x.ctypes.data, y.ctypes.data, 7) == -1
    # byte count that does not match the shape
    h = ctypes.c_void_p()
    assert lib().rt_weight_upload(gpu_ctx.h, RT_FMT_Q4K, blocks.ctypes.data, blocks.nbytes - 144, 4, 256,
                                  ctypes.byref(h)) == -4
    # Q4_K needs whole super-blocks
    assert lib().rt_weight_upload(gpu_ctx.h, RT_FMT_Q4K, blocks.ctypes.data, blocks.nbytes, 4, 250,
                                  ctypes.byref(h)) == -4
    with pytest.raises(ValueError):
        cuda_gemv_q4k_t(np.zeros(255, np.float32), Q4KMat(4, 256, blocks))
    w.free()


def test_q4k_gemv_zero_and_extreme_blocks(orc):
    # d = dmin = 0 blocks give exact zeros; large d / all-15 nibbles stay finite.
    rows, cols = 40, 512
    blocks = synth_q4k(3, 3, rows, cols).reshape(rows, -1, 144)
    blocks[:10, :, 0:4] = 0
    blocks[10:20, :, 16:] = 0xFF
    blocks[10:20, :, 1] = 0x5B  # d ~ 224
    blocks = np.ascontiguousarray(blocks.reshape(-1))
    x = synth_normal(4, 4, cols)
    y = cuda_gemv_q4k_t(x, Q4KMat(rows, cols, blocks))[0]
    ref = orc.q4k_gemv(blocks, rows, cols, x)
    assert np.all(y[:10] == 0.0)
    assert _rel(y, ref).max() < REL_TOL


@pytest.mark.parametrize("ctas_per_sm", [1, 2])
def test_gemv_bench_graph_matches_gemv(ctas_per_sm):
    # rt_gemv_bench replays a graph of chained GEMVs over rotating weights; the
    # last launch's y must equal a plain GEMV of the same weight.
    import torch

    from rich_triplet_b200.ops import Context, gemv_bench, gemv_device

    rows, cols = 1000, 2304
    ctx = Context(0)
    try:
        ws = [DeviceWeight.upload(ctx, RT_FMT_Q4K, synth_q4k(5, 40 + c, rows, cols), rows, cols) for c in range(3)]
        x = torch.from_numpy(synth_normal(6, 1, cols)).cuda()
        y = torch.empty(rows, dtype=torch.float32, device="cuda")
        y_ref = torch.empty(rows, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        launches = 5  # last launch reads ws[4 % 3] = ws[1]
        us = gemv_bench(ctx, ws, x.data_ptr(), y.data_ptr(), launches=launches, ctas_per_sm=ctas_per_sm, reps=2)
        assert us > 0.0
        gemv_device(ctx, ws[1], x.data_ptr(), y_ref.data_ptr())
        ctx.sync()
        assert np.allclose(y.cpu().numpy(), y_ref.cpu().numpy(), rtol=1e-5, atol=1e-4)
        for w in ws:
            w.free()
    finally:
        ctx.close()
