"""The multi-row GEMV (csrc/gemm_rows.cu): the Q4_K product at M <= 16 rows
that rt_gemm_q4k, QLinear and the many-sequence engines plan for small M,
against Q4KMat::matmul_q4k_t (src/autograd2.rs:1437-1457).

A reaches the kernel as fp16 rows scaled by a power of two (as for the
tensor-core GEMM); the kernel splits each 256-column segment of a row into two
int8 planes (error at most max|a_seg| / 64516 per element) and multiplies them
by the exact Q4_K weights (q * d * sc - dmin * m) in integer MMAs.  Checks:
  * against the float64 product of the fp16 rows and the exact weights:
    relative L2 <= 1e-4 and max |C - C_exact| <= 3e-4 of the row's rms
    (the planes' rounding gives about 3e-5 relative);
  * against the oracle's f32 product of the bf16 rows: max |C - C_ref| over
    the row's L2 norm <= 1e-3 and relative L2 <= 1e-3, as the other GEMMs.
"""

import numpy as np
import pytest

from rich_triplet_b200.model import Q4KMat, synth_normal_bf16, synth_q4k
from rich_triplet_b200.ops import cuda_matmul_q4k_t
from test_gemm_gpu import _bf16_to_f32, _row_err, f16_rows, q4k_parts

pytestmark = pytest.mark.gpu

PLANE_L2_TOL = 1e-4
PLANE_MAX_TOL = 3e-4
ROW_TOL = 1e-3
L2_TOL = 1e-3


@pytest.fixture(autouse=True)
def _plan_defaults(monkeypatch):
    for v in ("RT_GEMM_TILE", "RT_GEMM_SPLITS", "RT_GEMM_ROWS"):
        monkeypatch.delenv(v, raising=False)


def exact_weights(blocks, n, k):
    """float64 q * (d * sc) - dmin * m of every weight (exact)."""
    q, d1, m1 = q4k_parts(blocks, n, k)
    return q.astype(np.float64) * np.repeat(d1.astype(np.float64), 32, axis=1) - np.repeat(m1.astype(np.float64), 32, axis=1)


def _check(orc, blocks, n, k, a_bits, c):
    assert c.shape == (a_bits.shape[0], n)
    assert np.all(np.isfinite(c))
    a = _bf16_to_f32(a_bits).astype(np.float64)
    exact = f16_rows(a) @ exact_weights(blocks, n, k).T
    c64 = c.astype(np.float64)
    l2 = np.linalg.norm(c64 - exact) / np.linalg.norm(exact)
    rms = np.sqrt(np.mean(exact ** 2, axis=1, keepdims=True))
    mx = (np.abs(c64 - exact) / rms).max()
    assert l2 <= PLANE_L2_TOL and mx <= PLANE_MAX_TOL, (l2, mx)
    w = orc.q4k_dequantize(blocks, n, k).reshape(n, k).astype(np.float64)
    ref = a @ w.T
    assert _row_err(c, ref) <= ROW_TOL, _row_err(c, ref)
    l2r = np.linalg.norm(c64 - ref) / np.linalg.norm(ref)
    assert l2r <= L2_TOL, l2r


@pytest.mark.parametrize("m", [1, 2, 4, 5, 8, 11, 16])
@pytest.mark.parametrize("n,k", [(1000, 2560), (17, 256), (300, 5376), (4096, 2560)])
def test_rows_gemm_vs_oracle(orc, m, n, k):
    blocks = synth_q4k(81, m + n + k, n, k)
    a = synth_normal_bf16(82, m * 7 + k, m * k).reshape(m, k)
    _check(orc, blocks, n, k, a, cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks)))


@pytest.mark.parametrize("m,n,k", [(8, 512, 21504), (16, 2048, 5376), (3, 5376, 10240)])
def test_rows_gemm_long_k(orc, m, n, k):
    # K longer than one part's planes: the plan cuts K into parts, added by
    # rt_gemm_q4k in part order.
    blocks = synth_q4k(83, m + n, n, k)
    a = synth_normal_bf16(84, m + k, m * k).reshape(m, k)
    _check(orc, blocks, n, k, a, cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks)))


@pytest.mark.parametrize("parts", [1, 2, 5, 8])
def test_rows_gemm_forced_parts_agree(orc, monkeypatch, parts):
    # Any K split gives the same product up to the f32 order of the parts.
    m, n, k = 8, 700, 5120
    blocks = synth_q4k(85, 1, n, k)
    a = synth_normal_bf16(86, 2, m * k).reshape(m, k)
    monkeypatch.setenv("RT_GEMM_SPLITS", str(parts))
    c = cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks))
    _check(orc, blocks, n, k, a, c)
    monkeypatch.delenv("RT_GEMM_SPLITS")
    base = cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks))
    assert np.abs(c.astype(np.float64) - base).max() <= 1e-5 * np.abs(base).max()


def test_rows_gemm_deterministic_and_matches_tensor_core_path(orc, monkeypatch):
    # Two calls give identical bits (pieces of split tiles are added in warp
    # order); the tcgen05 kernel (RT_GEMM_ROWS=0) computes the same product
    # from fp16 weights, within the fp16 operand error.
    m, n, k = 6, 2000, 2560
    blocks = synth_q4k(87, 2, n, k)
    a = synth_normal_bf16(88, 3, m * k).reshape(m, k)
    c1 = cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks))
    c2 = cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks))
    assert np.array_equal(c1, c2)
    monkeypatch.setenv("RT_GEMM_ROWS", "0")
    tc = cuda_matmul_q4k_t(a, Q4KMat(n, k, blocks))
    l2 = np.linalg.norm(c1.astype(np.float64) - tc) / np.linalg.norm(tc.astype(np.float64))
    assert l2 <= 1e-3, l2


def test_rows_gemm_zero_and_scaled_rows(orc):
    # A zero row (plane scale 0) and rows of very different magnitudes (the
    # power-of-two row scales and per-segment plane scales keep each exact).
    m, n, k = 5, 256, 1024
    blocks = synth_q4k(89, 4, n, k)
    a = _bf16_to_f32(synth_normal_bf16(90, 5, m * k).reshape(m, k)).copy()
    a[1] = 0.0
    a[2] *= 1e-6
    a[3] *= 3e4
    a[4, 256:512] = 0.0  # one zero segment
    bits = (a.view(np.uint32) >> 16).astype(np.uint16)  # truncated to bf16: the kernel's input
    a_b = _bf16_to_f32(bits)
    c = cuda_matmul_q4k_t(bits, Q4KMat(n, k, blocks))
    assert np.all(c[1] == 0.0)
    exact = f16_rows(a_b.astype(np.float64)) @ exact_weights(blocks, n, k).T
    for r in (0, 2, 3, 4):
        err = np.abs(c[r].astype(np.float64) - exact[r]).max() / np.sqrt(np.mean(exact[r] ** 2))
        assert err <= PLANE_MAX_TOL, (r, err)
