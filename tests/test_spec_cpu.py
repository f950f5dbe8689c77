"""NgramDraftEngine against the reference's own known-answer test
(test_ngram_draft_engine, src/transformer4.rs:3457-3490), plus the
speculative loop's bookkeeping on a fake decode context (CPU only)."""

import numpy as np

from rich_triplet_b200.spec import NgramDraftEngine, greedy_token, speculative_generate


def test_ngram_draft_engine_reference_vectors():
    ng = NgramDraftEngine(4, 4)
    assert ng.draft() == []
    for t in (10, 20, 30, 40, 10, 20, 30, 40, 50, 60):
        ng.record(t)
    assert ng.draft() == []
    ng.record(10)
    assert ng.draft() == []
    ng.record(20)
    assert ng.draft() == [30, 40, 10, 20]


def test_ngram_draft_prefers_longest_suffix_and_caps_length():
    ng = NgramDraftEngine(4, 3)
    ng.record_many([1, 2, 3, 9, 2, 3, 7, 1, 2, 3])
    # suffix [1, 2, 3] first occurs at 0 -> continuation [9, 2, 3]
    assert ng.draft() == [9, 2, 3]
    ng2 = NgramDraftEngine(2, 8)
    ng2.record_many([5, 6, 7, 5, 6])
    # only n = 2: [5, 6] at 0 -> continuation up to the end of the history
    assert ng2.draft() == [7, 5, 6]


class _FakeDecoder:
    """Next token = (token * 3 + position) % V as a one-hot logit row."""

    V = 17

    def _row(self, tok, pos):
        r = np.zeros(self.V, np.float32)
        r[(tok * 3 + pos) % self.V] = 1.0
        return r

    def decode_step(self, tok, pos):
        return self._row(tok, pos)

    def decode_step_batch(self, toks, pos):
        return np.stack([self._row(t, pos + i) for i, t in enumerate(toks)])


def _plain(dec, first, start, n):
    out, prev = [first], first
    for i in range(n - 1):
        prev = greedy_token(dec.decode_step(prev, start + i))
        out.append(prev)
    return out


def test_speculative_loop_emits_the_greedy_sequence():
    dec = _FakeDecoder()
    prompt = [1, 2, 3, 4, 1, 2, 3, 4]
    first = greedy_token(dec.decode_step(prompt[-1], len(prompt) - 1))
    toks, stats = speculative_generate(dec, prompt, first, len(prompt), 40, draft_len=4)
    assert toks == _plain(dec, first, len(prompt), 40)
    assert stats["rounds"] > 0 and stats["accepted"] >= stats["rounds"]


def test_greedy_token_ties_to_higher_index():
    assert greedy_token(np.array([1.0, 3.0, 3.0, 0.0])) == 2


def test_greedy_token_follows_sample_token_on_near_ties(orc):
    """Two logits one f32 ulp apart: below ~0.25 in magnitude exp() of their
    difference rounds to 1, so sample_token (softmax, last index of the
    largest probability) takes the LATER index; at magnitude 4 the
    probabilities differ and the larger logit wins.  greedy_token must agree
    with the oracle's restatement in both cases, and on random rows."""
    y = np.full(1000, -10.0, np.float32)
    y[10] = np.float32(0.125) + np.float32(2.0 ** -26)  # one ulp above 0.125
    y[20] = np.float32(0.125)
    assert orc.sample_greedy(y) == 20 and greedy_token(y) == 20 and int(np.argmax(y)) == 10
    y = np.full(1000, -10.0, np.float32)
    y[10] = np.float32(4.0) + np.float32(2.0 ** -21)  # one ulp above 4
    y[20] = np.float32(4.0)
    assert orc.sample_greedy(y) == 10 and greedy_token(y) == 10
    rng = np.random.default_rng(3)
    for scale in (0.01, 1.0, 30.0):
        for _ in range(20):
            v = (rng.standard_normal(4096) * scale).astype(np.float32)
            assert greedy_token(v) == orc.sample_greedy(v)
