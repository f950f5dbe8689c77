"""The Qwen 3.5 oracle (oracle/qwen35.py) against literal transcriptions of
the reference's loops (src/transformer_qwen35.rs) on small cases: no GPU.
The reference holds no known-answer test for this model, so these loops,
written element by element as the reference writes them, are what pins the
vectorised restatement."""

import math

import numpy as np

from oracle import qwen35 as oq


def _sig(x):
    return 1.0 / (1.0 + math.exp(-x))


def _softplus(x):
    return x if x > 20.0 else math.log(1.0 + math.exp(x))


def _literal_deltanet(q, k, v, z, a, b, a_log, dt_bias, norm_w, S, nk, nv, kd, vd):
    """src/transformer_qwen35.rs:346-453, one element at a time (float64)."""
    beta = [_sig(b[h]) for h in range(nv)]
    g = [-math.exp(a_log[h]) * _softplus(a[h] + dt_bias[h]) for h in range(nv)]

    def l2(x, n, d):
        out = list(x)
        for hh in range(n):
            norm = max(math.sqrt(sum(out[hh * d + j] ** 2 for j in range(d))), 1e-12)
            for j in range(d):
                out[hh * d + j] /= norm
        return out

    q, k = l2(q, nk, kd), l2(k, nk, kd)
    rep = nv // nk
    qe = [q[(h // rep) * kd + i] / math.sqrt(kd) for h in range(nv) for i in range(kd)]
    ke = [k[(h // rep) * kd + i] for h in range(nv) for i in range(kd)]
    out = [0.0] * (nv * vd)
    for h in range(nv):
        s = S[h]
        dec = math.exp(g[h])
        for i in range(kd):
            for j in range(vd):
                s[i][j] *= dec
        kv = [sum(s[i][j] * ke[h * kd + i] for i in range(kd)) for j in range(vd)]
        for i in range(kd):
            for j in range(vd):
                s[i][j] += ke[h * kd + i] * (v[h * vd + j] - kv[j]) * beta[h]
        for j in range(vd):
            out[h * vd + j] = sum(s[i][j] * qe[h * kd + i] for i in range(kd))
    res = []
    for h in range(nv):
        o = out[h * vd:(h + 1) * vd]
        rms = math.sqrt(sum(x * x for x in o) / vd + 1e-6)
        for j in range(vd):
            zz = z[h * vd + j]
            res.append(o[j] / rms * norm_w[j] * zz * _sig(zz))
    return res


def test_deltanet_matches_the_reference_loops():
    rng = np.random.default_rng(3)
    nk, nv, kd, vd = 2, 4, 4, 6
    args = [rng.normal(size=n).astype(np.float32) for n in (nk * kd, nk * kd, nv * vd, nv * vd, nv, nv, nv, nv, vd)]
    S0 = rng.normal(size=(nv, kd, vd)).astype(np.float32)
    S_lit = [[[float(S0[h, i, j]) for j in range(vd)] for i in range(kd)] for h in range(nv)]
    S_or = S0.copy()
    for step in range(3):  # the state carries over steps
        got = oq.deltanet_heads(*args, S_or, nk, nv, kd, vd)
        want = _literal_deltanet(*[a.astype(np.float64).tolist() for a in args], S_lit, nk, nv, kd, vd)
        np.testing.assert_allclose(got, np.array(want), rtol=2e-5, atol=2e-6)
        np.testing.assert_allclose(S_or, np.array(S_lit), rtol=2e-5, atol=2e-6)
        args[2] = rng.normal(size=nv * vd).astype(np.float32)


def test_conv1d_shifts_its_history():
    rng = np.random.default_rng(4)
    C, ks = 5, 4
    w = rng.normal(size=C * ks).astype(np.float32)
    state = np.zeros((C, ks - 1), np.float32)
    hist = [[0.0] * (ks - 1) for _ in range(C)]
    for t in range(6):
        x = rng.normal(size=C).astype(np.float32)
        got = oq.conv1d_step(x, w, state, ks)
        for c in range(C):  # src/transformer_qwen35.rs:595-613
            val = sum(float(w[c * ks + j]) * hist[c][j] for j in range(ks - 1)) + float(w[c * ks + ks - 1]) * float(x[c])
            assert abs(got[c] - val * _sig(val)) <= 1e-5 * (1 + abs(val))
            hist[c] = hist[c][1:] + [float(x[c])]
        np.testing.assert_allclose(state, np.array(hist, np.float32))


def test_partial_rope_rotates_only_the_first_dims():
    rng = np.random.default_rng(5)
    nh, d, rd, theta, pos = 2, 16, 8, 10_000_000.0, 37
    x = rng.normal(size=nh * d).astype(np.float32)
    got = oq.partial_rope(x, nh, d, rd, theta, pos)
    half = rd // 2
    for h in range(nh):
        for i in range(half):  # src/transformer_qwen35.rs:1795-1810
            f = 1.0 / theta ** (2.0 * i / rd)
            c, s = math.cos(pos * f), math.sin(pos * f)
            x0, x1 = x[h * d + i], x[h * d + i + half]
            assert abs(got[h * d + i] - (x0 * c - x1 * s)) < 1e-4
            assert abs(got[h * d + i + half] - (x1 * c + x0 * s)) < 1e-4
        np.testing.assert_array_equal(got[h * d + rd:(h + 1) * d], x[h * d + rd:(h + 1) * d])


def test_layer_pattern_and_presets():
    from rich_triplet_b200.qwen35 import Qwen35Config
    c = Qwen35Config.qwen35_4b()
    assert [i for i in range(c.num_hidden_layers) if c.is_full_attention_layer(i)] == list(range(3, 32, 4))
    assert c.qkv_dim == 16 * 128 * 2 + 32 * 128 and c.rope_dim == 64
    s = Qwen35Config.qwen35_0_8b()
    assert (s.hidden_size, s.num_hidden_layers, s.linear_num_value_heads, s.intermediate_size) == (1024, 24, 16, 3584)


def test_oracle_model_is_deterministic():
    from rich_triplet_b200.qwen35 import Qwen35Config, synth_qwen35
    cfg = Qwen35Config(vocab_size=512, hidden_size=256, num_hidden_layers=4, num_attention_heads=2,
                       num_key_value_heads=1, head_dim=128, linear_num_key_heads=2, linear_num_value_heads=4,
                       linear_key_head_dim=64, linear_value_head_dim=64, intermediate_size=512)
    w = synth_qwen35(cfg, seed=11)
    a, b = oq.OracleQwen35(w), oq.OracleQwen35(w)
    for p, t in enumerate([1, 5, 9]):
        la, lb = a.step(t, p), b.step(t, p)
        assert np.all(np.isfinite(la)) and np.array_equal(la, lb)
