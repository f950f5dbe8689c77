"""Load-time conversions on the GPU are bit-exact with the reference CPU code."""

import numpy as np
import pytest

from rich_triplet_b200.model import synth_bytes
from rich_triplet_b200.ops import convert_q4_0_to_q4k, convert_q6k_to_bf16

pytestmark = pytest.mark.gpu


def _hex(h, dt):
    return np.frombuffer(bytes.fromhex(h), dtype=dt).copy()


def _finite_f16(rng, n, lo, hi, neg=False):
    v = rng.uniform(lo, hi, size=n).astype(np.float16)
    if neg:
        v[::3] *= -1
    return v.view(np.uint16)


def _q4_0_blocks(seed, rows, cols, neg=False):
    n_blocks = rows * cols // 32
    raw = synth_bytes(seed, 1, n_blocks * 18).reshape(n_blocks, 18)
    rng = np.random.default_rng(seed)
    d = _finite_f16(rng, n_blocks, 1e-4, 5e-2, neg)
    raw[:, 0] = d & 0xFF
    raw[:, 1] = d >> 8
    return np.ascontiguousarray(raw.reshape(-1))


def test_q4_0_to_q4k_golden(golden, gpu_ctx):
    c = golden["q4_0_to_q4k"]
    w = convert_q4_0_to_q4k(gpu_ctx, _hex(c["q4_0_hex"], np.uint8), c["rows"], c["cols"])
    assert w.download().tobytes().hex() == c["q4k_hex"]
    w.free()


@pytest.mark.parametrize("rows,cols,neg", [(64, 2560, False), (37, 768, True), (1, 256, False), (256, 10240, True)])
def test_q4_0_to_q4k_bit_exact(gpu_ctx, orc, rows, cols, neg):
    src = _q4_0_blocks(rows + cols, rows, cols, neg)
    w = convert_q4_0_to_q4k(gpu_ctx, src, rows, cols)
    got = w.download()
    ref = orc.q4_0_to_q4k(src, rows, cols)
    assert got.tobytes() == ref.tobytes()
    w.free()


def test_q4_0_to_q4k_edge_blocks(gpu_ctx, orc):
    # all-zero nibbles (every value -8*d), all-8 nibbles (zeros), denormal and
    # zero scales, and a constant sub-block: the min/max and scale==0 branches.
    rows, cols = 4, 512
    n_blocks = rows * cols // 32
    raw = np.zeros((n_blocks, 18), dtype=np.uint8)
    raw[:, 2:] = 0x88                      # nibble 8 -> value 0
    raw[0:8, 2:] = 0x00                    # -8 * d everywhere
    raw[8:16, 2:] = 0xFF                   # +7 * d
    scales = np.array([0x3C00, 0x0001, 0x0000, 0x8400, 0x1234, 0x7BFF, 0x03FF, 0xBC00] * (n_blocks // 8),
                      dtype=np.uint16)     # 1, denormal, 0, -6e-5, small, max, denormal, -1
    raw[:, 0] = scales & 0xFF
    raw[:, 1] = scales >> 8
    src = np.ascontiguousarray(raw.reshape(-1))
    w = convert_q4_0_to_q4k(gpu_ctx, src, rows, cols)
    assert w.download().tobytes() == orc.q4_0_to_q4k(src, rows, cols).tobytes()
    w.free()


def test_q6k_to_bf16_golden(golden, gpu_ctx):
    c = golden["q6k"]
    w = convert_q6k_to_bf16(gpu_ctx, _hex(c["bytes_hex"], np.uint8), 2, 256)
    np.testing.assert_array_equal(w.download(), np.array(c["bf16"], np.uint16))
    w.free()


@pytest.mark.parametrize("rows,cols", [(64, 2560), (3, 256), (512, 10240)])
def test_q6k_to_bf16_bit_exact(gpu_ctx, orc, rows, cols):
    n_blocks = rows * cols // 256
    raw = synth_bytes(rows * 31 + cols, 2, n_blocks * 210).reshape(n_blocks, 210)
    rng = np.random.default_rng(rows)
    d = _finite_f16(rng, n_blocks, 1e-5, 3e-2, neg=True)
    raw[:, 208] = d & 0xFF
    raw[:, 209] = d >> 8
    src = np.ascontiguousarray(raw.reshape(-1))
    w = convert_q6k_to_bf16(gpu_ctx, src, rows, cols)
    np.testing.assert_array_equal(w.download(), orc.q6k_to_bf16(src, rows * cols))
    w.free()
