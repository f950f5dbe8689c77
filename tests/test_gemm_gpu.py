"""Q4_K prefill GEMM (tcgen05 tensor cores) vs the CPU oracle's
Q4KMat::matmul_q4k_t (src/autograd2.rs:1437-1457, no-BLAS order).

A is bf16 (A = bf16(N(0,1))); the oracle multiplies the same
bf16 values widened to f32.  The tensor cores take fp16 operands: each row of A
is scaled by a power of two into fp16's range (exact for these bf16 values),
and each weight is dequantised as fma(q, fp16(d*sc), fp16(-dmin*m)) with one
fp16 rounding.  Two checks:
  * exact arithmetic: against the float64 product of those fp16 operands,
    emulated here from the raw blocks (q4k_f16_weights),
    max |C - C_f16| <= 1e-5 of the row's L2 norm (f32 accumulation order is
    the only difference);
  * against the oracle's f32 weights: max |C - C_ref| / ||C_ref row||_2 <= 1e-3
    and relative L2 <= 1e-3 (fp16 operand rounding gives about 3e-4).
"""

import numpy as np
import pytest

from rich_triplet_b200.model import Q4KMat, synth_normal_bf16, synth_q4k
from rich_triplet_b200.ops import cuda_matmul_q4k_t

pytestmark = pytest.mark.gpu

EXACT_TOL = 1e-5
ROW_TOL = 1e-3
L2_TOL = 1e-3


def _bf16_to_f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _row_err(c, ref):
    c64, r64 = c.astype(np.float64), ref.astype(np.float64)
    return (np.abs(c64 - r64) / (np.linalg.norm(r64, axis=1, keepdims=True) + 1e-30)).max()


def q4k_parts(blocks, n, k):
    """q [n, k] (0..15), d1 = d*sc and m1 = dmin*m [n, k/32] (f32, one rounding
    each) of Q4_K blocks (Q4KMat::scale_min and dequantize_row_into,
    src/autograd2.rs:1075-1085, 1326-1366)."""
    b = blocks.reshape(n, k // 256, 144)
    d = b[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    dmin = b[:, :, 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    sc = b[:, :, 4:16].astype(np.uint32)
    qs = b[:, :, 16:144]
    scale = np.empty((n, k // 256, 8), np.uint32)
    mins = np.empty((n, k // 256, 8), np.uint32)
    for j in range(8):
        if j < 4:
            scale[..., j], mins[..., j] = sc[..., j] & 63, sc[..., j + 4] & 63
        else:
            scale[..., j] = (sc[..., j + 4] & 0xF) | ((sc[..., j - 4] >> 6) << 4)
            mins[..., j] = (sc[..., j + 4] >> 4) | ((sc[..., j] >> 6) << 4)
    d1 = (d[..., None] * scale.astype(np.float32)).astype(np.float32).reshape(n, k // 32)
    m1 = (dmin[..., None] * mins.astype(np.float32)).astype(np.float32).reshape(n, k // 32)
    q = np.empty((n, k // 256, 256), np.uint8)
    for ch in range(4):
        byt = qs[:, :, 32 * ch:32 * ch + 32]
        q[:, :, 64 * ch:64 * ch + 32] = byt & 0xF
        q[:, :, 64 * ch + 32:64 * ch + 64] = byt >> 4
    return q.reshape(n, k), d1, m1


def q4k_f16_weights(blocks, n, k):
    """The fp16 weights the GEMM's tensor cores read: fma(q, fp16(d1), fp16(-m1))
    rounded once to fp16 (float64 holds the exact value)."""
    q, d1, m1 = q4k_parts(blocks, n, k)
    d1h = np.repeat(d1.astype(np.float16).astype(np.float64), 32, axis=1)
    m1h = np.repeat((-m1).astype(np.float16).astype(np.float64), 32, axis=1)
    return (q.astype(np.float64) * d1h + m1h).astype(np.float16).astype(np.float64)


def f16_rows(a):
    """A as the GEMM's fp16 rows, scaled back: fp16(a * 2^-e) * 2^e with the
    row's largest magnitude in [2^14, 2^15) after scaling."""
    a = np.asarray(a, np.float64)
    mx = np.abs(a).max(axis=1, keepdims=True)
    e = np.where(mx > 0, np.floor(np.log2(np.where(mx > 0, mx, 1.0))), 0.0)
    up = np.where(mx > 0, np.minimum(14 - e, 126), 0.0)
    return (a * 2.0 ** up).astype(np.float16).astype(np.float64) * 2.0 ** -up


def _check(orc, blocks, n, k, a_bits, c):
    assert np.all(np.isfinite(c))
    a = _bf16_to_f32(a_bits).astype(np.float64)
    w = orc.q4k_dequantize(blocks, n, k)
    q, d1, m1 = q4k_parts(blocks, n, k)
    assert np.array_equal((np.repeat(d1, 32, axis=1) * q - np.repeat(m1, 32, axis=1)).astype(np.float32),
                          w.reshape(n, k))
    exact = f16_rows(a) @ q4k_f16_weights(blocks, n, k).T
    assert _row_err(c, exact) <= EXACT_TOL, _row_err(c, exact)
    ref = a @ w.astype(np.float64).reshape(n, k).T
    assert _row_err(c, ref) <= ROW_TOL, _row_err(c, ref)
    l2 = np.linalg.norm(c.astype(np.float64) - ref) / (np.linalg.norm(ref) + 1e-30)
    assert l2 <= L2_TOL, l2


@pytest.fixture(params=["128", "256"])
def tile(request, monkeypatch):
    """Both CTA tiles (128 x 128 with one accumulator, 256 x 256 with two),
    forced through RT_GEMM_TILE; the plan otherwise picks by grid size."""
    monkeypatch.setenv("RT_GEMM_TILE", request.param)
    return int(request.param)


@pytest.mark.parametrize("m,n,k", [
    (1, 128, 256), (5, 256, 512), (128, 128, 256), (200, 300, 512),  # ragged M and N tiles
    (130, 384, 2560), (64, 256, 10240), (300, 600, 2048),             # hidden and FFN widths
])
def test_gemm_q4k_vs_oracle(orc, tile, m, n, k):
    blocks = synth_q4k(21, m * 3 + n + k, n, k)
    a = synth_normal_bf16(22, m + n, m * k).reshape(m, k)
    c = cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks))
    _check(orc, blocks, n, k, a, c)
    if m * n * k <= 2 ** 24:  # the oracle's own GEMM (matmul_q4k_t) on the small cases
        ref = orc.q4k_gemm(blocks, n, k, _bf16_to_f32(a))
        assert _row_err(c, ref) <= ROW_TOL


@pytest.mark.parametrize("m,n,k", [(512, 2560, 2560), (512, 2560, 2048), (256, 4096, 2560)])
def test_gemm_q4k_config2_shapes(orc, tile, m, n, k):
    # BASELINE config 2 shapes at the smaller M
    blocks = synth_q4k(31, n + k, n, k)
    a = synth_normal_bf16(32, m, m * k).reshape(m, k)
    c = cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks))
    _check(orc, blocks, n, k, a, c)


def test_gemm_q4k_device_pointers_and_reuse():
    # Device pointers through rt_gemm_q4k (RT_DEVICE), two calls on the same
    # weight with different A: results differ and each matches the host path.
    import torch

    from rich_triplet_b200._lib import RT_FMT_Q4K
    from rich_triplet_b200.ops import Context, DeviceWeight, gemm_device

    m, n, k = 256, 512, 2560
    blocks = synth_q4k(41, 1, n, k)
    ctx = Context(0)
    try:
        w = DeviceWeight.upload(ctx, RT_FMT_Q4K, blocks, n, k)
        outs = []
        for seed in (42, 43):
            a = synth_normal_bf16(seed, 1, m * k).reshape(m, k)
            da = torch.from_numpy(a.view(np.int16)).cuda()
            dc = torch.empty((m, n), dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            gemm_device(ctx, w, da.data_ptr(), m, dc.data_ptr())
            ctx.sync()
            outs.append(dc.cpu().numpy())
            host = cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks))
            assert np.array_equal(outs[-1], host)
        assert not np.array_equal(outs[0], outs[1])
        w.free()
    finally:
        ctx.close()


def test_gemm_q4k_rejects_bad_shapes():
    from rich_triplet_b200 import RtError

    blocks = synth_q4k(51, 1, 16, 256)
    with pytest.raises(ValueError):
        cuda_matmul_q4k_t(np.zeros((4, 128), np.float32), Q4KMat(16, 256, blocks))
    with pytest.raises(RtError):
        cuda_matmul_q4k_t(np.zeros((0, 256), np.float32), Q4KMat(16, 256, blocks))


@pytest.mark.parametrize("splits", [2, 3])
@pytest.mark.parametrize("m,n,k", [(64, 256, 2560), (200, 300, 2048)])
def test_gemm_q4k_split_k(orc, tile, monkeypatch, splits, m, n, k):
    # K split across CTAs (RT_GEMM_SPLITS forces the count); the partial
    # products are added in split order.
    monkeypatch.setenv("RT_GEMM_SPLITS", str(splits))
    blocks = synth_q4k(61, m + n + k, n, k)
    a = synth_normal_bf16(62, m, m * k).reshape(m, k)
    c = cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks))
    _check(orc, blocks, n, k, a, c)


@pytest.mark.parametrize("splits", [1, 2])
@pytest.mark.parametrize("m,n,k", [(8, 512, 2560), (48, 1000, 2560), (64, 4096, 2560), (130, 1000, 512)])
def test_gemm_bf16_weights(tile, monkeypatch, splits, m, n, k):
    # BF16 weights (the LM head of a many-sequence step): both operands are
    # bf16 values, exact in fp16 (A after its row scale), so the product
    # matches float64 to f32 accumulation.
    from rich_triplet_b200.model import MatBf16
    from rich_triplet_b200.ops import cuda_matmul_bf16_t

    monkeypatch.setenv("RT_GEMM_SPLITS", str(splits))
    wb = synth_normal_bf16(71, n, n * k, 0.0, 0.05)
    a = synth_normal_bf16(72, m, m * k).reshape(m, k)
    c = cuda_matmul_bf16_t(a, MatBf16(n, k, wb))
    ref = _bf16_to_f32(a).astype(np.float64) @ _bf16_to_f32(wb).reshape(n, k).astype(np.float64).T
    assert np.all(np.isfinite(c))
    assert _row_err(c, ref) <= EXACT_TOL, _row_err(c, ref)
