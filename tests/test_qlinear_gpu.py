"""QLinear on the GPU (rich_triplet_b200.qlinear, rt_qlinear_forward) against
the CPU oracle: QLinear::forward (src/qlinear.rs:83-111) with a Q4_K weight is
matmul_q4k_t_exact plus add_bias_rows (src/qlinear.rs:49-61), with a BF16
weight matmul_by_t plus the bias.

Tolerances, as in the GEMV and GEMM tests:
  * one row (the GEMV path): max relative error 1e-3, floored at 1% of the
    output's rms (the x planes carry f32-level precision);
  * several rows (the tensor-core GEMM, fp16 operands): max |y - ref| over the
    row's L2 norm <= 1e-3 and relative L2 <= 1e-3.
The bias test mirrors the reference's applies_its_bias_once_per_row
(src/qlinear.rs:178-190), the state test reports_whether_a_weight_is_present
(:192-200).
"""

import numpy as np
import pytest

from rich_triplet_b200.model import MatBf16, Q4KMat, synth_normal, synth_q4k
from rich_triplet_b200.qlinear import QLinear

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3
ROW_TOL = 1e-3
L2_TOL = 1e-3


def _spread(rows, cols, scale, salt):
    """The reference tests' deterministic fill (src/qlinear.rs:144-150)."""
    r = np.arange(rows)[:, None]
    c = np.arange(cols)[None, :]
    i = ((r * 131 + c * 37 + salt * 7919) % 251).astype(np.float32)
    return ((np.sin(i * np.float32(0.41)) * np.float32(0.7) + np.cos(i * np.float32(0.13)) * np.float32(0.3))
            * np.float32(scale)).astype(np.float32)


def _check(y, ref):
    if y.shape[0] == 1:
        r64 = ref.astype(np.float64)
        floor = 1e-2 * np.sqrt(np.mean(r64 ** 2))
        rel = (np.abs(y - r64) / np.maximum(np.abs(r64), floor)).max()
        assert rel < GEMV_TOL, rel
    else:
        y64, r64 = y.astype(np.float64), ref.astype(np.float64)
        row = (np.abs(y64 - r64) / (np.linalg.norm(r64, axis=1, keepdims=True) + 1e-30)).max()
        l2 = np.linalg.norm(y64 - r64) / np.linalg.norm(r64)
        assert row < ROW_TOL and l2 < L2_TOL, (row, l2)


@pytest.mark.parametrize("t,out,inp", [(1, 1024, 2560), (3, 1024, 2560), (64, 3072, 512), (300, 2560, 2048),
                                       (1, 17, 256), (5, 17, 256)])
def test_q4k_qlinear_matches_oracle(gpu_ctx, orc, t, out, inp):
    blocks = synth_q4k(31, t + out, out, inp)
    x = synth_normal(32, t * inp, t * inp).reshape(t, inp)
    bias = synth_normal(33, out, out) * np.float32(0.5)
    ql = QLinear.from_q4k(gpu_ctx, Q4KMat(out, inp, blocks), out, inp, bias)
    y = ql.forward(x)
    assert y.shape == (t, out)
    if t == 1:
        ref = orc.q4k_gemv(blocks, out, inp, x[0])[None, :]
    else:
        ref = orc.q4k_gemm(blocks, out, inp, x)
    _check(y, ref + bias[None, :])
    ql.free_weight()


@pytest.mark.parametrize("t", [1, 4, 40])
def test_bf16_qlinear_matches_oracle(gpu_ctx, orc, t):
    out, inp = 384, 1024
    w = _spread(out, inp, 0.05, 5)
    wb = ((w.view(np.uint32) + 0x7FFF + ((w.view(np.uint32) >> 16) & 1)) >> 16).astype(np.uint16)  # RNE to bf16
    x = _spread(t, inp, 1.0, 7)
    bias = _spread(1, out, 0.5, 6)[0]
    ql = QLinear.from_bf16(gpu_ctx, MatBf16(out, inp, wb), bias)
    y = ql.forward(x)
    wf = (wb.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    ref = x.astype(np.float64) @ wf.T + bias[None, :]
    _check(y, ref.astype(np.float32))


def test_applies_its_bias_once_per_row(gpu_ctx):
    out, inp, t = 48, 256, 4
    blocks = synth_q4k(41, 1, out, inp)
    x = _spread(t, inp, 1.0, 9)
    b = np.tile(np.array([1.0, -2.0, 0.5], dtype=np.float32), out // 3)
    plain = QLinear.from_q4k(gpu_ctx, Q4KMat(out, inp, blocks), out, inp).forward(x)
    biased = QLinear.from_q4k(gpu_ctx, Q4KMat(out, inp, blocks), out, inp, b).forward(x)
    np.testing.assert_allclose(biased, plain + b[None, :], rtol=1e-6, atol=1e-5)


def test_reports_whether_a_weight_is_present(gpu_ctx):
    empty = QLinear()
    assert not empty.loaded()
    ql = QLinear.from_q4k(gpu_ctx, Q4KMat(16, 256, synth_q4k(5, 5, 16, 256)), 16, 256)
    assert ql.loaded() and ql.size_bytes() == 16 * 144
    ql.free_weight()
    assert not ql.loaded() and ql.size_bytes() == 0


def test_qlinear_device_pointers(gpu_ctx, orc):
    import torch
    out, inp, t = 512, 1024, 8
    blocks = synth_q4k(51, 2, out, inp)
    x = synth_normal(52, t * inp, t * inp).reshape(t, inp)
    bias = synth_normal(53, out, out)
    ql = QLinear.from_q4k(gpu_ctx, Q4KMat(out, inp, blocks), out, inp)
    dx = torch.from_numpy(x).cuda()
    db = torch.from_numpy(bias).cuda()
    dy = torch.empty((t, out), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ql.forward_device(dx.data_ptr(), t, dy.data_ptr(), db.data_ptr())
    gpu_ctx.sync()
    _check(dy.cpu().numpy(), orc.q4k_gemm(blocks, out, inp, x) + bias[None, :])


def test_qlinear_rejects_bad_input(gpu_ctx):
    ql = QLinear.from_q4k(gpu_ctx, Q4KMat(16, 256, synth_q4k(6, 6, 16, 256)), 16, 256)
    with pytest.raises(ValueError):
        ql.forward(np.zeros((2, 255), dtype=np.float32))
    with pytest.raises(ValueError):
        QLinear(gpu_ctx, None, 256, 16, bias=np.zeros(15, dtype=np.float32))
    with pytest.raises(NotImplementedError):
        QLinear.from_f32(np.zeros((2, 2), dtype=np.float32), ())
