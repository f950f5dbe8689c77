"""Qwen 3.5 decode restated on the CPU -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's single-token path for its hybrid
Gated DeltaNet / full-attention model (src/transformer_qwen35.rs), the
checker of rich_triplet_b200.qwen35's CUDA engine.  Only tests/ and bench.py's
CPU legs use it.  The projections and the tied LM head run on the C oracle's
Q4_K / BF16 GEMVs (oracle.c, the reference's x86 dot products); the rest is
float32 numpy in the reference's order of operations.

Parity unpinned: the reference holds no known-answer test for this model, and
the reference itself (Rust) cannot run here, so this restatement is checked
against the cited lines by reading and, in tests/test_qwen35_cpu.py, against
a literal transcription of the reference's loops on small cases.
"""

import numpy as np

from . import oracle as orc

_F = np.float32


def sigmoid(x):
    """src/transformer_qwen35.rs:1737-1739 (exp(-x) may overflow to inf, giving 0,
    as f32 does in the reference)."""
    x = np.asarray(x, dtype=_F)
    with np.errstate(over="ignore"):
        return (_F(1.0) / (_F(1.0) + np.exp(-x))).astype(_F)


def softplus(x):
    """src/transformer_qwen35.rs:1742-1748."""
    x = np.asarray(x, dtype=_F)
    return np.where(x > _F(20.0), x, np.log(_F(1.0) + np.exp(np.minimum(x, _F(20.0))))).astype(_F)


def silu(x):
    """src/transformer_qwen35.rs:1751-1753."""
    x = np.asarray(x, dtype=_F)
    return (x * sigmoid(x)).astype(_F)


def l2_normalize_heads(x, n_heads, dim):
    """src/transformer_qwen35.rs:1756-1766."""
    x = np.asarray(x, dtype=_F).reshape(n_heads, dim)
    norm = np.maximum(np.sqrt((x * x).sum(axis=1, dtype=_F)), _F(1e-12))
    return (x / norm[:, None]).astype(_F).reshape(-1)


def per_head_norm(x, gamma, n_heads, dim, eps):
    """apply_per_head_norm_raw (src/transformer_qwen35.rs:1768-1781):
    (x / rms) * (1 + gamma) per head."""
    x = np.asarray(x, dtype=_F).reshape(n_heads, dim)
    rms = np.sqrt((x * x).sum(axis=1, dtype=_F) / _F(dim) + _F(eps))
    return ((x / rms[:, None]) * (_F(1.0) + np.asarray(gamma, dtype=_F))[None, :]).astype(_F).reshape(-1)


def partial_rope(x, n_heads, head_dim, rope_dim, theta, pos):
    """apply_partial_rope (src/transformer_qwen35.rs:1783-1812): pairs
    (i, i + rope_dim / 2) of the first rope_dim dims of each head."""
    x = np.asarray(x, dtype=_F).reshape(n_heads, head_dim).copy()
    half = rope_dim // 2
    i = np.arange(half, dtype=_F)
    freq = (_F(1.0) / np.power(_F(theta), _F(2.0) * i / _F(rope_dim))).astype(_F)
    ang = (_F(pos) * freq).astype(_F)
    c, s = np.cos(ang).astype(_F), np.sin(ang).astype(_F)
    x0, x1 = x[:, :half].copy(), x[:, half:2 * half].copy()
    x[:, :half] = x0 * c - x1 * s
    x[:, half:2 * half] = x1 * c + x0 * s
    return x.reshape(-1)


def deltanet_heads(q, k, v, z, a, b, a_log, dt_bias, norm_w, S, nk, nv, kd, vd):
    """Steps 4-9 of Qwen35DeltaNet::forward_cached (src/transformer_qwen35.rs:346-453)
    on the conv outputs q [nk kd], k [nk kd], v [nv vd]; S [nv, kd, vd] is
    updated in place.  Returns the gated output [nv vd]."""
    beta = sigmoid(b)
    g = (-np.exp(np.asarray(a_log, dtype=_F)) * softplus(np.asarray(a, dtype=_F) + np.asarray(dt_bias, dtype=_F))).astype(_F)
    qn = l2_normalize_heads(q, nk, kd).reshape(nk, kd)
    kn = l2_normalize_heads(k, nk, kd).reshape(nk, kd)
    rep = nv // nk
    q_exp = np.repeat(qn, rep, axis=0) * _F(1.0 / np.sqrt(np.float32(kd)))  # repeat-interleave: head g -> g*rep..
    k_exp = np.repeat(kn, rep, axis=0)
    v = np.asarray(v, dtype=_F).reshape(nv, vd)
    z = np.asarray(z, dtype=_F).reshape(nv, vd)
    out = np.zeros((nv, vd), dtype=_F)
    for h in range(nv):
        Sh = S[h]
        Sh *= np.exp(g[h]).astype(_F)
        kv = (Sh * k_exp[h][:, None]).sum(axis=0, dtype=_F)
        delta = ((v[h] - kv) * beta[h]).astype(_F)
        Sh += np.outer(k_exp[h], delta).astype(_F)
        out[h] = (Sh * q_exp[h][:, None].astype(_F)).sum(axis=0, dtype=_F)
    rms = np.sqrt((out * out).sum(axis=1, dtype=_F) / _F(vd) + _F(1e-6))
    normed = out / rms[:, None]
    return ((normed * np.asarray(norm_w, dtype=_F)[None, :]) * silu(z)).astype(_F).reshape(-1)


def conv1d_step(inp, w, state, ks):
    """Qwen35DeltaNet::apply_conv1d (src/transformer_qwen35.rs:589-617):
    state [C, ks - 1] shifted in place.  Returns silu(conv)."""
    C = inp.shape[0]
    w = np.asarray(w, dtype=_F).reshape(C, ks)
    hist = ks - 1
    val = np.zeros(C, dtype=_F)
    for t in range(hist):
        val = (val + w[:, t] * state[:, t]).astype(_F)
    val = (val + w[:, hist] * inp).astype(_F)
    if hist > 0:
        state[:, :-1] = state[:, 1:].copy()
        state[:, hist - 1] = inp
    return silu(val)


class OracleQwen35:
    """Qwen35Model's cached decode (src/transformer_qwen35.rs:1124-1133,
    905-924): step(token, position) -> logits, with per-layer DeltaNet states
    and K/V caches."""

    def __init__(self, weights):
        self.w = weights
        self.cfg = weights.cfg
        self.reset()

    def reset(self):
        c = self.cfg
        self.S, self.conv, self.K, self.V = {}, {}, {}, {}
        for i, L in enumerate(self.w.layers):
            if L.full:
                self.K[i], self.V[i] = [], []
            else:
                self.S[i] = np.zeros((c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim), _F)
                self.conv[i] = np.zeros((c.qkv_dim, c.linear_conv_kernel_dim - 1), _F)

    def _gemv(self, L, name, rows, cols, x):
        return orc.q4k_gemv(L.proj[name], rows, cols, np.ascontiguousarray(x, dtype=_F))

    def _deltanet(self, i, L, x):
        """Qwen35DeltaNet::forward_cached (src/transformer_qwen35.rs:315-456)."""
        c = self.cfg
        H, nk, nv = c.hidden_size, c.linear_num_key_heads, c.linear_num_value_heads
        kd, vd = c.linear_key_head_dim, c.linear_value_head_dim
        qkv = self._gemv(L, "in_qkv", c.qkv_dim, H, x)
        z = self._gemv(L, "in_z", c.value_dim, H, x)
        a = self._gemv(L, "in_a", nv, H, x)
        b = self._gemv(L, "in_b", nv, H, x)
        conv = conv1d_step(qkv, L.vec["conv1d_weight"], self.conv[i], c.linear_conv_kernel_dim)
        key_dim = nk * kd
        out = deltanet_heads(conv[:key_dim], conv[key_dim:2 * key_dim], conv[2 * key_dim:], z, a, b,
                             L.vec["a_log"], L.vec["dt_bias"], L.vec["norm_weight"], self.S[i], nk, nv, kd, vd)
        return self._gemv(L, "out_proj", H, c.value_dim, out)

    def _full_attn(self, i, L, x, pos):
        """Qwen35FullAttention::forward_cached (src/transformer_qwen35.rs:663-724)."""
        c = self.cfg
        H, nq, nkv, d = c.hidden_size, c.num_attention_heads, c.num_key_value_heads, c.head_dim
        qg = self._gemv(L, "q", 2 * nq * d, H, x).reshape(nq, 2 * d)
        k = self._gemv(L, "k", nkv * d, H, x)
        v = self._gemv(L, "v", nkv * d, H, x)
        q = per_head_norm(qg[:, :d].reshape(-1), L.vec["q_norm"], nq, d, c.rms_norm_eps)
        gate = qg[:, d:].reshape(-1)
        k = per_head_norm(k, L.vec["k_norm"], nkv, d, c.rms_norm_eps)
        q = partial_rope(q, nq, d, c.rope_dim, c.rope_theta, pos)
        k = partial_rope(k, nkv, d, c.rope_dim, c.rope_theta, pos)
        self.K[i].append(k)
        self.V[i].append(np.asarray(v, dtype=_F))
        kc = np.ascontiguousarray(np.stack(self.K[i]), dtype=_F)
        vc = np.ascontiguousarray(np.stack(self.V[i]), dtype=_F)
        att = orc.gqa_attention_decode(q, kc, vc, 0, kc.shape[0], nq, nkv, d, 1.0 / float(np.sqrt(np.float32(d))))
        gated = (np.asarray(att, dtype=_F) * sigmoid(gate)).astype(_F)
        return self._gemv(L, "o", H, nq * d, gated)

    def step(self, token, pos):
        c = self.cfg
        H, F = c.hidden_size, c.intermediate_size
        x = ((self.w.embed[token * H:(token + 1) * H].astype(np.uint32) << 16).view(np.float32)).astype(_F)
        for i, L in enumerate(self.w.layers):
            xn = orc.rms_norm_gemma3(x, L.vec["input_norm"], c.rms_norm_eps)
            y = self._full_attn(i, L, xn, pos) if L.full else self._deltanet(i, L, xn)
            x = (x + y).astype(_F)
            xn = orc.rms_norm_gemma3(x, L.vec["post_attn_norm"], c.rms_norm_eps)
            g = silu(self._gemv(L, "gate", F, H, xn))
            u = self._gemv(L, "up", F, H, xn)
            x = (x + self._gemv(L, "down", H, F, (g * u).astype(_F))).astype(_F)
        xn = orc.rms_norm_gemma3(x, self.w.final_norm, c.rms_norm_eps)
        return orc.bf16_gemv(self.w.embed, c.vocab_size, H, xn)
