"""All-positions prefill (rt_decoder_prefill_gemm) and the batched verify
step (rt_decoder_step_batch, MetalDecodeContext::decode_step_batch,
src/metal_decode.rs:2079) against the CPU oracle and the token-by-token
engine.

Both paths run every projection as a tensor-core GEMM over the positions with
fp16 operands (each within 2^-11 relative; about 3e-4 relative L2 per
projection), so the KV cache they leave and the logits they return sit near,
not on, the token-by-token values.  Tolerances: logits within REL_L2 (2e-3,
the north star's bar for full-model logits; measured 2.2e-4 on the full
34-layer 4B model after 512 tokens and on a 6-layer slice after 640), the KV
cache within KV_L2 (2e-3, measured 5.2e-4) relative L2 per layer, and greedy
tokens that agree when the decode continues from the prefilled cache.
"""

import numpy as np
import pytest

from rich_triplet_b200._lib import RtError
from rich_triplet_b200.decode import CudaDecodeContext
from rich_triplet_b200.model import Config4, synth_gemma3, synth_tokens
from rich_triplet_b200.ops import Context

pytestmark = pytest.mark.gpu

REL_L2 = 2e-3
KV_L2 = 2e-3


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / (np.linalg.norm(b.astype(np.float64)) + 1e-30))


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def tiny():
    cfg = Config4.tiny()
    return cfg, synth_gemma3(cfg, seed=1234)


def _kv_err(dec, ref_kv, n):
    worst = 0.0
    for layer, (rk, rv) in enumerate(ref_kv):
        k, v = dec.read_kv(layer, n)
        worst = max(worst, rel_l2(k, rk), rel_l2(v, rv))
    return worst


def test_prefill_gemm_vs_oracle_tiny(ctx, orc, tiny):
    cfg, w = tiny
    cap = 64
    prompt = synth_tokens(31, 2, 20, cfg.vocab_size)  # > window 8: local layers slide
    om = orc.OracleModel(cfg, w, cap)
    dec = CudaDecodeContext(w, cap, ctx)
    try:
        ol = None
        for t in prompt:
            ol = om.step(int(t))
        gl = dec.prefill_gemm(prompt)
        assert rel_l2(gl, ol) < REL_L2, rel_l2(gl, ol)
        kvd = cfg.num_key_value_heads * cfg.head_dim
        ref = []
        for layer in range(cfg.num_hidden_layers):
            k = np.ctypeslib.as_array(orc.lib.or_model_kcache(om._h, layer), shape=(cap * kvd,))[: len(prompt) * kvd]
            v = np.ctypeslib.as_array(orc.lib.or_model_vcache(om._h, layer), shape=(cap * kvd,))[: len(prompt) * kvd]
            ref.append((k.copy(), v.copy()))
        assert _kv_err(dec, ref, len(prompt)) < KV_L2
        # greedy decode continues from the prefilled cache
        tok_o, tok_g = int(np.argmax(ol)), int(np.argmax(gl))
        assert tok_o == tok_g
        pos = len(prompt)
        for _ in range(10):
            ol = om.step(tok_o)
            gl = dec.decode_step(tok_g, pos)
            pos += 1
            assert rel_l2(gl, ol) < REL_L2
            tok_o, tok_g = int(np.argmax(ol)), int(np.argmax(gl))
            assert tok_o == tok_g
    finally:
        dec.close()
        om.close()


def _vs_token_by_token(ctx, cfg, w, n, tol, start=0):
    cap = start + n + 8
    prompt = synth_tokens(41, 4, n, cfg.vocab_size)
    a = CudaDecodeContext(w, cap, ctx)
    b = CudaDecodeContext(w, cap, ctx)
    try:
        if start:
            head = synth_tokens(42, 4, start, cfg.vocab_size)
            a.prefill(head, want_logits=False)
            b.prefill(head, want_logits=False)
        la = a.prefill(prompt, start_pos=start)
        lb = b.prefill_gemm(prompt, start_pos=start)
        assert rel_l2(lb, la) < tol, rel_l2(lb, la)
        assert int(np.argmax(lb)) == int(np.argmax(la))
        ref = [a.read_kv(layer, start + n) for layer in range(cfg.num_hidden_layers)]
        assert _kv_err(b, ref, start + n) < KV_L2
    finally:
        a.close()
        b.close()


def test_prefill_gemm_two_pieces_4b_width(ctx):
    # 600 tokens: two pieces (512 + 88), attention over up to 600 positions
    # (several 256-position chunks on the global layer), after a 40-token head
    # prefilled token by token.
    cfg = Config4.gemma3_4b(vocab_size=262144).with_layers(6)
    w = synth_gemma3(cfg, seed=1234)
    _vs_token_by_token(ctx, cfg, w, 600, REL_L2, start=40)


def test_prefill_gemm_full_4b(ctx):
    # BASELINE config 1's prompt: 512 tokens through the full 34-layer model.
    cfg = Config4.gemma3_4b(vocab_size=262144)
    w = synth_gemma3(cfg, seed=1234)
    _vs_token_by_token(ctx, cfg, w, 512, REL_L2)


def test_step_batch_matches_steps(ctx, tiny):
    cfg, w = tiny
    head = synth_tokens(51, 1, 9, cfg.vocab_size)
    draft = synth_tokens(52, 1, 6, cfg.vocab_size)
    a = CudaDecodeContext(w, 32, ctx)
    b = CudaDecodeContext(w, 32, ctx)
    try:
        a.prefill(head, want_logits=False)
        b.prefill(head, want_logits=False)
        seq = np.stack([a.decode_step(int(t), len(head) + i) for i, t in enumerate(draft)])
        bat = b.decode_step_batch(draft, len(head))
        assert bat.shape == (len(draft), cfg.vocab_size)
        for i in range(len(draft)):
            assert rel_l2(bat[i], seq[i]) < REL_L2, (i, rel_l2(bat[i], seq[i]))
            assert int(np.argmax(bat[i])) == int(np.argmax(seq[i]))
        # the verified positions are in the cache: the next single step agrees
        la = a.decode_step(3, len(head) + len(draft))
        lb = b.decode_step(3, len(head) + len(draft))
        assert rel_l2(lb, la) < REL_L2
    finally:
        a.close()
        b.close()


def test_prefill_gemm_rejects_bad_input(ctx, tiny):
    cfg, w = tiny
    dec = CudaDecodeContext(w, 16, ctx)
    try:
        with pytest.raises(RtError):
            dec.prefill_gemm([1, cfg.vocab_size])
        with pytest.raises(RtError):
            dec.prefill_gemm(list(range(17)))
        with pytest.raises(RtError):
            dec.prefill_gemm([1, 2], start_pos=15)
        with pytest.raises(RtError):
            dec.decode_step_batch(list(range(65)), 0)
        assert dec.prefill_gemm([], want_logits=False) is None
        assert np.all(np.isfinite(dec.prefill_gemm([1, 2, 3])))
    finally:
        dec.close()


def test_speculative_generate_matches_greedy(ctx, tiny):
    # The reference's n-gram speculative loop over decode_step_batch emits the
    # plain greedy sequence (src/transformer4.rs:2244-2330).
    from rich_triplet_b200.spec import greedy_token, speculative_generate

    cfg, w = tiny
    unit = synth_tokens(61, 1, 8, cfg.vocab_size)
    prompt = np.concatenate([unit, unit, unit])
    a = CudaDecodeContext(w, 128, ctx)
    b = CudaDecodeContext(w, 128, ctx)
    try:
        first = greedy_token(a.prefill(prompt))
        b.prefill(prompt, want_logits=False)
        plain = [first] + [int(x) for x in a.generate(first, len(prompt), 39)]
        spec, stats = speculative_generate(b, [int(x) for x in prompt], first, len(prompt), 40, draft_len=4)
        assert spec == plain
        assert stats["rounds"] > 0
    finally:
        a.close()
        b.close()
