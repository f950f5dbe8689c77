"""Q4_K prefill GEMM (tcgen05 tensor cores) vs the CPU oracle's
Q4KMat::matmul_q4k_t (src/autograd2.rs:1437-1457, no-BLAS order).

A is bf16 (A = bf16(N(0,1))); the oracle multiplies the same
bf16 values widened to f32.  The GEMM dequantises each weight in f32 in the
reference's order and rounds it to bf16 for the tensor cores (the design the
north star names: Q4_K -> bf16 in shared memory), so two checks:
  * exact arithmetic: against the float64 product with the oracle's
    dequantised weights rounded to bf16, max |C - C_bf16| <= 1e-5 of the row's
    L2 norm (f32 accumulation order is the only difference);
  * against the oracle's f32 weights: max |C - C_ref| / ||C_ref row||_2 <= 2.5e-3
    and relative L2 <= 4e-3 (bf16 weight rounding alone gives up to 1.7e-3 and
    about 1.6e-3 here); at the config-2 shapes (K >= 2048, N >= 2560) the
    row-normalised error also meets 1e-3.
"""

import numpy as np
import pytest

from rich_triplet_b200.model import Q4KMat, synth_normal_bf16, synth_q4k
from rich_triplet_b200.ops import bf16_bits, cuda_matmul_q4k_t

pytestmark = pytest.mark.gpu

EXACT_TOL = 1e-5
ROW_TOL = 2.5e-3
L2_TOL = 4e-3
ROW_TOL_CONFIG2 = 1e-3


def _bf16_to_f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _row_err(c, ref):
    c64, r64 = c.astype(np.float64), ref.astype(np.float64)
    return (np.abs(c64 - r64) / (np.linalg.norm(r64, axis=1, keepdims=True) + 1e-30)).max()


def _check(orc, blocks, n, k, a_bits, c, row_tol=ROW_TOL):
    assert np.all(np.isfinite(c))
    a = _bf16_to_f32(a_bits).astype(np.float64)
    w = orc.q4k_dequantize(blocks, n, k)
    exact = a @ _bf16_to_f32(bf16_bits(w)).astype(np.float64).T
    assert _row_err(c, exact) <= EXACT_TOL, _row_err(c, exact)
    ref = a @ w.astype(np.float64).T
    assert _row_err(c, ref) <= row_tol, _row_err(c, ref)
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
    _check(orc, blocks, n, k, a, c, row_tol=ROW_TOL_CONFIG2)


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
@pytest.mark.parametrize("m,n,k", [(8, 512, 2560), (130, 1000, 512)])
def test_gemm_bf16_weights(tile, monkeypatch, splits, m, n, k):
    # BF16 weights (the LM head of a many-sequence step): both operands are
    # exact bf16, so the product matches float64 to f32 accumulation.
    from rich_triplet_b200.model import MatBf16
    from rich_triplet_b200.ops import cuda_matmul_bf16_t

    monkeypatch.setenv("RT_GEMM_SPLITS", str(splits))
    wb = synth_normal_bf16(71, n, n * k, 0.0, 0.05)
    a = synth_normal_bf16(72, m, m * k).reshape(m, k)
    c = cuda_matmul_bf16_t(a, MatBf16(n, k, wb))
    ref = _bf16_to_f32(a).astype(np.float64) @ _bf16_to_f32(wb).reshape(n, k).astype(np.float64).T
    assert np.all(np.isfinite(c))
    assert _row_err(c, ref) <= EXACT_TOL, _row_err(c, ref)
