"""The Qwen 3.5 decode engine (rt_qwen35_*, rich_triplet_b200.qwen35) against
the CPU oracle's restatement of the reference's cached decode
(oracle/qwen35.py, src/transformer_qwen35.rs:905-924, 1124-1133).

Both run the same synthetic Q4_K model token by token; the oracle's greedy
token drives both.  The bar is the decode tests': logits within relative L2
2e-3 at every step and the same greedy token (the GPU's projections carry
f32-level accuracy; the DeltaNet recurrence and the attention sum in a
different order)."""

import numpy as np
import pytest

from oracle import qwen35 as oq
from rich_triplet_b200.qwen35 import CudaQwen35Decoder, Qwen35Config, greedy, synth_qwen35

pytestmark = pytest.mark.gpu

REL_L2 = 2e-3

TINY = Qwen35Config(vocab_size=512, hidden_size=256, num_hidden_layers=4, num_attention_heads=2,
                    num_key_value_heads=1, head_dim=128, linear_num_key_heads=2, linear_num_value_heads=4,
                    linear_key_head_dim=64, linear_value_head_dim=64, intermediate_size=512)
# the 0.8B preset's widths (head dims of the real models), fewer layers and a smaller vocabulary
WIDTH_08B = Qwen35Config.qwen35_0_8b().with_layers(4)
WIDTH_08B = Qwen35Config(**{**WIDTH_08B.__dict__, "vocab_size": 4096})


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / np.linalg.norm(b)


def _run(cfg, prompt, n_new, seed):
    w = synth_qwen35(cfg, seed=seed)
    orc = oq.OracleQwen35(w)
    dec = CudaQwen35Decoder(w, len(prompt) + n_new + 4)
    worst = 0.0
    try:
        toks = list(prompt)
        for p in range(len(prompt) + n_new):
            lo = orc.step(toks[p], p)
            lg = dec.step(toks[p], p)
            assert np.all(np.isfinite(lg))
            worst = max(worst, _rel(lg, lo))
            assert _rel(lg, lo) < REL_L2, (p, _rel(lg, lo))
            if p >= len(prompt) - 1:
                t_o, t_g = greedy(lo), greedy(lg)
                assert t_o == t_g, (p, t_o, t_g)
                toks.append(t_o)
    finally:
        dec.close()
    return worst


def test_tiny_qwen35_decode_matches_oracle():
    _run(TINY, [3, 17, 250, 9, 400], 12, seed=21)


def test_qwen35_08b_width_decode_matches_oracle():
    # DeltaNet heads of 128 x 128, attention heads of 256 with partial RoPE over 64 dims
    _run(WIDTH_08B, [11, 2048, 7], 6, seed=22)


def test_reset_starts_a_new_sequence():
    w = synth_qwen35(TINY, seed=23)
    dec = CudaQwen35Decoder(w, 16)
    try:
        first = [dec.step(t, p) for p, t in enumerate([5, 6, 7])]
        dec.reset()
        again = [dec.step(t, p) for p, t in enumerate([5, 6, 7])]
        for a, b in zip(first, again):
            np.testing.assert_array_equal(a, b)
        gen = dec.generate([5, 6], 4)
        assert len(gen) == 4 and all(0 <= t < TINY.vocab_size for t in gen)
    finally:
        dec.close()


def test_qwen35_rejects_bad_input():
    from rich_triplet_b200 import RtError
    w = synth_qwen35(TINY, seed=24)
    dec = CudaQwen35Decoder(w, 4)
    try:
        with pytest.raises(RtError):
            dec.step(TINY.vocab_size, 0)   # token out of range
        with pytest.raises(RtError):
            dec.step(1, 4)                 # position past the cache
    finally:
        dec.close()
    # 4 value heads over 3 key heads: valid Q4_K shapes, but no whole number of
    # value heads per key head (the repeat-interleave of src/transformer_qwen35.rs:367-374)
    bad = Qwen35Config(**{**TINY.__dict__, "linear_num_key_heads": 3})
    with pytest.raises(RtError):
        CudaQwen35Decoder(synth_qwen35(bad, seed=25), 4)
