"""GGUF reading (rich_triplet_b200.gguf, GgufFile / read_tensor_bytes,
src/gguf_loader.rs:142-252) on files written by write_gguf: every metadata
type, tensor infos and bytes, alignment; header errors; the f32 -> bf16
rounding of MatBf16::f32_to_bf16 (src/autograd2.rs:709-719)."""

import numpy as np
import pytest

from rich_triplet_b200.gguf import (GGML_BF16, GGML_F16, GGML_F32, GGML_Q4K, GgufError, GgufFile, f32_to_bf16_bits,
                                    write_gguf)


def test_round_trip(tmp_path):
    rng = np.random.default_rng(3)
    f32 = rng.standard_normal(96).astype(np.float32)
    f16 = rng.standard_normal((4, 64)).astype(np.float16)
    q4k = rng.integers(0, 256, 3 * 144, dtype=np.uint8)
    bf = rng.integers(0, 65535, 512, dtype=np.uint16)
    meta = [("general.architecture", 8, "gemma3"), ("general.alignment", 4, 64), ("u8", 0, 7), ("i8", 1, -3),
            ("u16", 2, 60000), ("i16", 3, -20000), ("i32", 5, -7), ("f32", 6, 0.5), ("flag", 7, True),
            ("u64", 10, 1 << 40), ("i64", 11, -(1 << 40)), ("f64", 12, 0.25),
            ("arr", 9, (4, [1, 2, 3])), ("names", 9, (8, ["a", "bc"]))]
    tensors = [("blk.0.attn_norm.weight", [96], GGML_F32, f32), ("h", [64, 4], GGML_F16, f16),
               ("blk.0.attn_q.weight", [256, 3], GGML_Q4K, q4k), ("e", [32, 16], GGML_BF16, bf)]
    path = tmp_path / "m.gguf"
    write_gguf(str(path), tensors, meta, alignment=64)
    g = GgufFile(str(path))
    try:
        assert g.version == 3 and g.data_start % 64 == 0
        want = {k: v for k, _, v in meta}
        want["arr"], want["names"] = [1, 2, 3], ["a", "bc"]
        assert g.metadata == want
        for i, (name, dims, gtype, data) in enumerate(tensors):
            t = g.tensor_info[i]
            assert (t.name, t.shape, t.gguf_type) == (name, dims, gtype)
            assert t.data_offset % 64 == 0
            assert np.array_equal(g.tensor_bytes(i), np.ascontiguousarray(data).view(np.uint8).reshape(-1))
        assert g.find_tensor("e") == 3 and g.find_tensor("nope") is None
    finally:
        g.close()


def test_header_errors(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUX" + bytes(20))
    with pytest.raises(GgufError):
        GgufFile(str(p))
    p.write_bytes(b"GGUF" + (4).to_bytes(4, "little") + bytes(16))
    with pytest.raises(GgufError):
        GgufFile(str(p))
    write_gguf(str(p), [("x", [8], GGML_F32, np.zeros(8, np.float32))])
    data = p.read_bytes()
    p.write_bytes(data[:30])
    with pytest.raises(GgufError):
        GgufFile(str(p))


def test_f32_to_bf16_rounding():
    bits = np.array([0x3F800000, 0x3F808000, 0x3F818000, 0x3F80FFFF, 0x7F800000, 0xFF800000, 0x7FC00001, 0x7F800001],
                    dtype=np.uint32)
    got = f32_to_bf16_bits(bits.view(np.float32))
    # 1.0; ties to even (stays, rounds up to even); above half; +-inf; NaN keeps a set mantissa bit
    assert [int(x) for x in got] == [0x3F80, 0x3F80, 0x3F82, 0x3F81, 0x7F80, 0xFF80, 0x7FC0, 0x7FC0]
