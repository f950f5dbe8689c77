"""The GEMM launch plan (rt_gemm_plan, the host logic behind rt_gemm_q4k /
rt_gemm_bf16 and the many-sequence engines) on the shapes its rules were
measured on: no GPU needed.  Each case states the rule it pins."""

import ctypes

import pytest

SMS = 148  # B200


def _plan(rtlib, m, n, k, bf16=False):
    out = (ctypes.c_int32 * 4)()
    rc = rtlib.rt_gemm_plan(m, n, k, SMS, 1 if bf16 else 0, out)
    return rc, tuple(out)


@pytest.fixture(autouse=True)
def _no_overrides(monkeypatch):
    for v in ("RT_GEMM_TILE", "RT_GEMM_SPLITS", "RT_GEMM_ROWS"):
        monkeypatch.delenv(v, raising=False)


@pytest.mark.parametrize("m,n,k,want", [
    # Q4_K at M <= 16: the multi-row GEMV (tile 16); one K part while the
    # part's planes fit, since an extra part costs the pass that adds them
    (8, 20480, 2560, (16, 1, 16, 2560)),        # 4B gate/up
    (8, 43008, 5376, (16, 1, 16, 5376)),        # 27B gate/up
    (1, 43008, 5376, (16, 1, 16, 5376)),
    (3, 8192, 5376, (16, 1, 16, 5376)),         # 27B qkv, odd M
    # long K: parts chosen to balance the CTAs' whole tiles (336 tiles over
    # 7 x 21 CTAs), measured faster than the fewest parts
    (8, 5376, 21504, (16, 7, 16, 3072)),        # 27B down
    (16, 43008, 5376, (16, 3, 16, 1792)),       # 16 rows: planes of 7 segments per part
    # M = 17: the tensor-memory kernel again
    (17, 20480, 2560, (128, 1, 64, 2560)),
])
def test_rows_plan_rules(rtlib, m, n, k, want):
    rc, got = _plan(rtlib, m, n, k)
    assert rc == 0 and got == want, (rc, got)


@pytest.mark.parametrize("m,n,k,bf16,want", [
    # M <= 64: the swapped 128 tile, 16 or 64 activation rows per tile
    (8, 20480, 2560, False, (128, 1, 16, 2560)),      # 4B gate/up: K of 10 super-blocks is not split
    (64, 20480, 2560, False, (128, 1, 64, 2560)),     # config 3 gate/up
    (8, 262144, 5376, True, (128, 1, 16, 5376)),      # 27B LM head (BF16)
    (64, 262144, 2560, True, (128, 1, 64, 2560)),     # 4B LM head at 64 sequences
    # long K, tiles filling half a wave to two waves of 296 slots: 3 splits above one wave, 4 below
    (8, 43008, 5376, False, (128, 3, 16, 1792)),      # 27B gate/up, 336 tiles
    (1, 43008, 5376, False, (128, 3, 16, 1792)),
    (8, 21504, 5376, False, (128, 4, 16, 1536)),      # its 2-rank shard, 168 tiles
    # few tiles: split until the slots are filled (at most 8)
    (8, 5376, 21504, False, (128, 7, 16, 3072)),      # 27B down, 42 tiles
    # large M: the 256 x 256 tile when it halves the waves, no split
    (2048, 20480, 2560, False, (256, 1, 128, 2560)),
])
def test_plan_rules(rtlib, monkeypatch, m, n, k, bf16, want):
    # the tensor-memory kernel's rules (RT_GEMM_ROWS=0 keeps it at M <= 16)
    monkeypatch.setenv("RT_GEMM_ROWS", "0")
    rc, got = _plan(rtlib, m, n, k, bf16)
    assert rc == 0 and got == want, (rc, got)


def test_plan_rejects_k_off_the_super_block(rtlib):
    from rich_triplet_b200._lib import RT_E_SHAPE
    rc, _ = _plan(rtlib, 8, 512, 300)
    assert rc == RT_E_SHAPE


def test_plan_overrides(rtlib, monkeypatch):
    monkeypatch.setenv("RT_GEMM_SPLITS", "2")
    assert _plan(rtlib, 8, 43008, 5376)[1][:2] == (16, 2)   # the multi-row GEMV, 2 parts
    monkeypatch.setenv("RT_GEMM_TILE", "256")               # a forced tile: the tcgen05 kernel
    assert _plan(rtlib, 8, 43008, 5376)[1][:2] == (256, 2)
    monkeypatch.delenv("RT_GEMM_TILE")
    monkeypatch.delenv("RT_GEMM_SPLITS")
    monkeypatch.setenv("RT_GEMM_ROWS", "0")
    assert _plan(rtlib, 8, 43008, 5376)[1][:2] == (128, 3)
