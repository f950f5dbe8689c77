"""Many-sequence decode (CudaBatchDecoder, rt_batch_*) against the
single-sequence engine and the CPU oracle.

Every sequence of a batch must decode exactly as it would alone: per-step
logits within the tolerances below of the single-sequence CUDA engine (itself
within 2e-6 of the oracle), identical greedy tokens, and rows that depend only on
their own sequence (bit-identical rows for identical inputs, outputs that
follow a permutation of the sequences).

Tolerances.  The batch engine's projections are tensor-core GEMMs over fp16
operands (activation rows scaled by a power of two, dequantised Q4_K weights
rounded once to fp16; f32 accumulation): each operand is within 2^-11 relative,
about 3e-4 relative L2 on one projection.  REL_L2 (2e-3) is the north star's
bar for full-model logits; the full 34-layer 4B model measures 2.9e-4 against
the single-sequence engine and tiny 3.1e-4 against the oracle.
REL_L2_REDUCED (5e-3) bounds the 2-layer 4B-width slice, whose logits move
more under the same operand error (up to 3.5e-3 measured over 20 greedy steps).
"""

import numpy as np
import pytest

from rich_triplet_b200.decode import CudaBatchDecoder, CudaDecodeContext
from rich_triplet_b200._lib import RtError
from rich_triplet_b200.model import Config4, synth_gemma3, synth_tokens
from rich_triplet_b200.ops import Context

pytestmark = pytest.mark.gpu

REL_L2 = 2e-3
REL_L2_REDUCED = 5e-3
TOP2_MARGIN = 0.05  # greedy tokens compared where the single engine's top-2 gap exceeds this


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / (np.linalg.norm(b.astype(np.float64)) + 1e-30))


def top2_gap(logits):
    s = np.sort(logits)
    return float(s[-1] - s[-2])


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def tiny():
    cfg = Config4.tiny()
    return cfg, synth_gemma3(cfg, seed=1234)


@pytest.fixture(scope="module")
def w4b_2l():
    cfg = Config4.gemma3_4b(vocab_size=262144).with_layers(2)
    return cfg, synth_gemma3(cfg, seed=1234)


def _vs_singles(ctx, cfg, w, nseq, prompt_len, n_gen, cap=64):
    prompts = [synth_tokens(7 + b, 3, prompt_len, cfg.vocab_size) for b in range(nseq)]
    singles = [CudaDecodeContext(w, cap, ctx) for _ in range(nseq)]
    bat = CudaBatchDecoder(singles[0], nseq, cap)
    worst, compared = 0.0, 0
    try:
        cur = [int(p[0]) for p in prompts]
        for t in range(prompt_len + n_gen):
            bat.set(cur, [t] * nseq)
            lb, nb = bat.step()
            ls = [singles[b].decode_step(cur[b], t) for b in range(nseq)]
            for b in range(nseq):
                worst = max(worst, rel_l2(lb[b], ls[b]))
                assert int(nb[b]) == int(np.argmax(lb[b]))
                if t >= prompt_len - 1 and top2_gap(ls[b]) > TOP2_MARGIN:
                    assert int(nb[b]) == int(np.argmax(ls[b])), (t, b)
                    compared += 1
            if t + 1 < prompt_len:
                cur = [int(p[t + 1]) for p in prompts]
            else:
                cur = [int(x) for x in nb]
    finally:
        bat.close()
        for s in singles:
            s.close()
    return worst, compared


def test_batch_matches_single_engine_tiny(ctx, tiny):
    cfg, w = tiny
    # 12 prompt tokens exceed the sliding window (8) on the local layers.
    worst, compared = _vs_singles(ctx, cfg, w, 3, 12, 8)
    assert worst < REL_L2, worst
    assert compared > 0


def test_batch_matches_single_engine_4b_width(ctx, w4b_2l):
    cfg, w = w4b_2l
    worst, compared = _vs_singles(ctx, cfg, w, 3, 6, 4)
    assert worst < REL_L2_REDUCED, worst
    assert compared > 0


def test_batch_matches_single_engine_full_4b(ctx):
    # The full 34-layer Gemma 3 4B (synthetic weights): the north star's bar.
    cfg = Config4.gemma3_4b(vocab_size=262144)
    w = synth_gemma3(cfg, seed=1234)
    worst, compared = _vs_singles(ctx, cfg, w, 3, 4, 4)
    assert worst < REL_L2, worst
    assert compared > 0


def test_batch_rows_independent(ctx, tiny):
    cfg, w = tiny
    dec = CudaDecodeContext(w, 16, ctx)
    toks = synth_tokens(3, 9, 4, cfg.vocab_size)
    try:
        # identical inputs -> bit-identical rows
        bat = CudaBatchDecoder(dec, 4, 32)
        bat.set([int(toks[0])] * 4, [0] * 4)
        lb, _ = bat.step()
        bat.close()
        for b in range(1, 4):
            assert np.array_equal(lb[b], lb[0])
        # a permutation of the sequences permutes the outputs exactly
        outs = []
        for order in ([0, 1, 2, 3], [2, 0, 3, 1]):
            bat = CudaBatchDecoder(dec, 4, 32)
            steps = []
            for t in range(3):
                bat.set([int(toks[(o + t) % 4]) for o in order], [t] * 4)
                lb, _ = bat.step()
                steps.append(lb)
            bat.close()
            outs.append((order, steps))
        (o0, s0), (o1, s1) = outs
        for t in range(3):
            for i, o in enumerate(o1):
                assert np.array_equal(s1[t][i], s0[t][o0.index(o)]), (t, i)
    finally:
        dec.close()


def test_batch_vs_oracle_tiny(ctx, orc, tiny):
    cfg, w = tiny
    dec = CudaDecodeContext(w, 16, ctx)
    bat = CudaBatchDecoder(dec, 2, 40)
    oms = [orc.OracleModel(cfg, w, 40) for _ in range(2)]
    prompts = [synth_tokens(21 + b, 1, 10, cfg.vocab_size) for b in range(2)]
    worst = 0.0
    try:
        for t in range(10):
            cur = [int(p[t]) for p in prompts]
            bat.set(cur, [t] * 2)
            lb, _ = bat.step()
            for b in range(2):
                worst = max(worst, rel_l2(lb[b], oms[b].step(cur[b])))
    finally:
        bat.close()
        dec.close()
        for om in oms:
            om.close()
    assert worst < REL_L2, worst


def test_batch_synthetic_context_generate(ctx, w4b_2l):
    # The benchmark's form: synthetic caches at a long context, then device-side
    # greedy steps; every row advances and stays in the vocabulary.
    cfg, w = w4b_2l
    dec = CudaDecodeContext(w, 16, ctx)
    bat = CudaBatchDecoder(dec, 8, 600)
    try:
        mem, launches = bat.info()
        assert mem > 8 * 600 * cfg.num_hidden_layers * 2 * cfg.num_key_value_heads * cfg.head_dim * 4
        assert launches > 0
        bat.synth_kv(5, 512)
        bat.generate(4)
        lb, nb = bat.step()
        assert np.all(np.isfinite(lb))
        assert np.all((nb >= 0) & (nb < cfg.vocab_size))
        assert [int(x) for x in nb] == [int(np.argmax(r)) for r in lb]
    finally:
        bat.close()
        dec.close()


def test_batch_rejects_bad_input(ctx, tiny):
    cfg, w = tiny
    dec = CudaDecodeContext(w, 16, ctx)
    try:
        with pytest.raises(RtError):
            CudaBatchDecoder(dec, 0, 32)
        bat = CudaBatchDecoder(dec, 2, 32)
        with pytest.raises(RtError):
            bat.set([1, cfg.vocab_size], [0, 0])
        with pytest.raises(RtError):
            bat.set([1, 2], [0, 32])
        with pytest.raises(ValueError):
            bat.set([1, 2, 3], [0, 0, 0])
        with pytest.raises(RtError):
            bat.synth_kv(1, 32)
        bat.set([1, 2], [0, 1])
        lb, nb = bat.step()
        assert lb.shape == (2, cfg.vocab_size)
        bat.close()
    finally:
        dec.close()
