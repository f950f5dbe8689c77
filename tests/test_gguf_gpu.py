"""Gemma 3 from a GGUF file (rich_triplet_b200.gguf.load_gemma3,
Gemma3Model::load_weights_from_gguf, src/transformer4.rs:757-1010) against
an engine built from the same weights in memory.

The file holds the tiny model with Q4_K projections, two of them as Q4_0
(converted to Q4_K on the GPU), norms stored as 1 + gamma (F32, one F16), a
vision-tower tensor that the loader skips, and the embedding as BF16 or Q6_K
(converted on the GPU).  The in-memory engine gets the oracle's conversions
of the same bytes, so the two engines' logits must be bit-identical."""

from dataclasses import replace

import numpy as np
import pytest

from rich_triplet_b200.gguf import (GGML_BF16, GGML_F16, GGML_F32, GGML_Q4_0, GGML_Q4K, GGML_Q6K, GgufError,
                                    load_gemma3, write_gguf)
from rich_triplet_b200.model import Config4, synth_gemma3, synth_tokens

pytestmark = pytest.mark.gpu

PROJ = (("attn_q", "q"), ("attn_k", "k"), ("attn_v", "v"), ("attn_output", "o"), ("ffn_gate", "gate"),
        ("ffn_up", "up"), ("ffn_down", "down"))
NORMS = (("attn_norm", "attn_norm"), ("post_attention_norm", "post_attn_norm"), ("ffn_norm", "pre_ffn_norm"),
         ("post_ffw_norm", "post_ffn_norm"), ("attn_q_norm", "q_norm"), ("attn_k_norm", "k_norm"))
Q4_0_AT = {(0, "q"), (1, "down")}


def _q4_0_blocks(rng, rows, cols):
    nb = rows * cols // 32
    b = np.empty((nb, 18), np.uint8)
    b[:, :2] = np.float16(rng.uniform(1e-3, 1e-2, nb)).view(np.uint8).reshape(nb, 2)
    b[:, 2:] = rng.integers(0, 256, (nb, 16), dtype=np.uint8)
    return b.reshape(-1)


def _q6k_blocks(rng, rows, cols):
    nb = rows * cols // 256
    b = rng.integers(0, 256, (nb, 210), dtype=np.uint8)
    b[:, 192:208] = rng.integers(-32, 32, (nb, 16)).astype(np.int8).view(np.uint8)  # scales
    b[:, 208:210] = np.float16(rng.uniform(1e-4, 1e-3, nb)).view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def _model_file(path, orc, cfg, embed_type, extra=()):
    """Write the GGUF; return the host weights an in-memory engine should get."""
    rng = np.random.default_rng(17)
    w = synth_gemma3(cfg, seed=29)
    H, D, F = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
    q, kv = cfg.num_attention_heads * D, cfg.num_key_value_heads * D
    shapes = {"q": (q, H), "k": (kv, H), "v": (kv, H), "o": (H, q), "gate": (F, H), "up": (F, H), "down": (H, F)}
    tensors = []
    if embed_type == GGML_BF16:
        tensors.append(("token_embd.weight", [H, cfg.vocab_size], GGML_BF16, w.embed))
    else:
        raw = _q6k_blocks(rng, cfg.vocab_size, H)
        tensors.append(("token_embd.weight", [H, cfg.vocab_size], GGML_Q6K, raw))
        w.embed = orc.q6k_to_bf16(raw, cfg.vocab_size * H)
    tensors.append(("output_norm.weight", [H], GGML_F32, (w.final_norm + np.float32(1)).astype(np.float32)))
    for i, L in enumerate(w.layers):
        for gname, f in PROJ:
            rows, cols = shapes[f]
            if (i, f) in Q4_0_AT:
                raw = _q4_0_blocks(rng, rows, cols)
                tensors.append((f"blk.{i}.{gname}.weight", [cols, rows], GGML_Q4_0, raw))
                setattr(L, f, orc.q4_0_to_q4k(raw, rows, cols))
            else:
                tensors.append((f"blk.{i}.{gname}.weight", [cols, rows], GGML_Q4K, getattr(L, f)))
        for gname, f in NORMS:
            g = getattr(L, f)
            if i == 1 and f == "attn_norm":  # an F16 norm: the gamma the engine gets is f16(1 + g) - 1
                h = (g + np.float32(1)).astype(np.float16)
                tensors.append((f"blk.{i}.{gname}.weight", [g.size], GGML_F16, h))
                setattr(L, f, (h.astype(np.float32) - np.float32(1)).astype(np.float32))
            else:
                tensors.append((f"blk.{i}.{gname}.weight", [g.size], GGML_F32, (g + np.float32(1)).astype(np.float32)))
    tensors.append(("v.blk.0.attn_q.weight", [H, 256], GGML_F32, np.zeros(H * 256, np.float32)))  # vision tower
    tensors.extend(extra)
    write_gguf(str(path), tensors, [("general.architecture", 8, "gemma3")])
    return w


@pytest.mark.parametrize("embed_type", [GGML_BF16, GGML_Q6K])
def test_gguf_model_matches_in_memory(tmp_path, orc, embed_type):
    from rich_triplet_b200.decode import CudaDecodeContext
    from rich_triplet_b200.ops import Context

    cfg = Config4.tiny().with_layers(2)
    path = tmp_path / "tiny.gguf"
    w = _model_file(path, orc, cfg, embed_type)
    ctx = Context(0)
    a = load_gemma3(str(path), cfg, 32, ctx)
    b = CudaDecodeContext(w, 32, ctx)
    try:
        for pos, tok in enumerate(synth_tokens(3, 3, 8, cfg.vocab_size)):
            la, lb = a.decode_step(int(tok), pos), b.decode_step(int(tok), pos)
            assert np.array_equal(la, lb), pos
    finally:
        a.close()
        b.close()
        ctx.close()


def test_gguf_refuses_what_the_engine_cannot_run(tmp_path, orc):
    from rich_triplet_b200.ops import Context

    cfg = Config4.tiny().with_layers(1)
    ctx = Context(0)
    try:
        p = tmp_path / "lm.gguf"
        _model_file(p, orc, cfg, GGML_BF16, extra=[("output.weight", [cfg.hidden_size, cfg.vocab_size], GGML_BF16,
                                                    np.zeros(cfg.vocab_size * cfg.hidden_size, np.uint16))])
        with pytest.raises(GgufError):
            load_gemma3(str(p), cfg, 16, ctx)
        # a BF16 projection
        p2 = tmp_path / "bf16proj.gguf"
        _model_file(p2, orc, cfg, GGML_BF16)
        from rich_triplet_b200.gguf import GgufFile
        g = GgufFile(str(p2))
        tensors = []
        for i, t in enumerate(g.tensor_info):
            data = np.array(g.tensor_bytes(i))
            if t.name == "blk.0.attn_k.weight":
                n = t.shape[0] * t.shape[1]
                tensors.append((t.name, t.shape, GGML_BF16, np.zeros(n, np.uint16)))
            else:
                tensors.append((t.name, t.shape, t.gguf_type, data))
        g.close()
        write_gguf(str(p2), tensors)
        with pytest.raises(GgufError):
            load_gemma3(str(p2), cfg, 16, ctx)
        # wrong hidden size for the config
        with pytest.raises(GgufError):
            load_gemma3(str(p), replace(cfg, hidden_size=512), 16, ctx)
    finally:
        ctx.close()
