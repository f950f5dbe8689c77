"""Greedy speculative decoding with n-gram drafts: the host loop of the
reference's Metal path (Gemma3Model::generate_cached_streaming,
src/transformer4.rs:2244-2330) over CudaDecodeContext.decode_step_batch.

Each round drafts up to `draft_len` tokens from the generated history
(NgramDraftEngine), runs [prev] + draft[:k-1] through one batched step, and
accepts drafts while the greedy token of each logits row equals the draft
token; the first mismatch emits the sampled token instead and ends the round.
With no draft the round is one ordinary decode step.  The emitted sequence is
the plain greedy sequence whenever each position's greedy token is the same in
both paths.
"""

import numpy as np


class NgramDraftEngine:
    """NgramDraftEngine (src/transformer4.rs:1985-2036): the continuation, up
    to `max_draft` tokens, of the earliest earlier occurrence of the longest
    suffix (n from max_n down to 2) of the token history."""

    def __init__(self, max_n, max_draft):
        self.history = []
        self.max_n = max_n
        self.max_draft = max_draft

    def record(self, token):
        self.history.append(int(token))

    def record_many(self, tokens):
        self.history.extend(int(t) for t in tokens)

    def draft(self):
        h = self.history
        n_hist = len(h)
        if n_hist < 2:
            return []
        for n in range(min(self.max_n, n_hist), 1, -1):
            suffix = h[n_hist - n:]
            for start in range(n_hist - n):
                if h[start:start + n] == suffix:
                    c0 = start + n
                    c1 = min(c0 + self.max_draft, n_hist)
                    if c0 < c1:
                        return h[c0:c1]
        return []


GREEDY_TAU = np.float32(2.0 ** -21)


def greedy_token(logits):
    """sample_token at temperature 0 (src/transformer4.rs:3036-3091): the LAST
    index of the largest softmax probability p_i = exp(y_i - M) / S, computed
    the way the device kernels compute it.  Only rows within 2^-21 of the
    maximum M can share its probability; for them p_i is formed as the
    reference does (f32 difference, exp rounded to f32, one f32 division by
    S), and the highest such row whose p_i equals 1/S wins.  Logits of
    magnitude below ~0.25 one f32 ulp apart therefore tie (exp rounds to 1)
    and the later index wins, where a plain argmax would take the larger."""
    row = np.asarray(logits, dtype=np.float32)
    m = row.max()
    s = np.float32(np.exp((row - m).astype(np.float64)).astype(np.float32).sum(dtype=np.float32))
    q = np.float32(1.0) / s
    cand = np.flatnonzero(row >= m - GREEDY_TAU)
    e = np.exp((row[cand] - m).astype(np.float64)).astype(np.float32)
    ties = cand[(e / s).astype(np.float32) == q]
    return int(ties[-1])


def speculative_generate(dec, prompt, first_token, start_pos, max_new, draft_len=4, max_n=4):
    """Tokens after `prompt` (already in the cache at positions
    start_pos - len(prompt) .. start_pos - 1), `first_token` being the greedy
    token of the prompt's last position; returns (tokens, stats) with
    len(tokens) == max_new, tokens[0] == first_token."""
    ngram = NgramDraftEngine(max_n, draft_len)
    ngram.record_many(prompt)
    ngram.record(first_token)
    out = [int(first_token)]
    prev = int(first_token)
    seq_len = start_pos
    stats = {"rounds": 0, "drafted": 0, "accepted": 0, "single_steps": 0}
    while len(out) < max_new:
        draft = ngram.draft() if draft_len > 0 else []
        if draft:
            k = min(len(draft), max_new - len(out))
            verify = [prev] + draft[:k - 1]
            logits = dec.decode_step_batch(verify, seq_len)
            stats["rounds"] += 1
            stats["drafted"] += k
            accepted = 0
            for i in range(k):
                sampled = greedy_token(logits[i])
                out.append(sampled)
                ngram.record(sampled)
                prev = sampled
                accepted += 1
                if sampled != draft[i]:
                    break
            stats["accepted"] += accepted
            seq_len += accepted
        else:
            logits = dec.decode_step(prev, seq_len)
            sampled = greedy_token(logits)
            out.append(sampled)
            ngram.record(sampled)
            prev = sampled
            seq_len += 1
            stats["single_steps"] += 1
    return out[:max_new], stats
