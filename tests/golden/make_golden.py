"""Generate tests/golden/golden.json: known-answer vectors for the Q4_K decode path.

The inputs are the ones the reference crate's own tests use; the expected
outputs are computed here by an independent numpy float32 restatement of the
inline CPU formulas those tests (and the functions they exercise) contain.
The C oracle (oracle/oracle.c) and the CUDA kernels are both checked against
this file, so a mistake shared by the C restatement and the kernels would have
to be repeated a third time here to go unnoticed.

Reference tests whose inputs are used (paths relative to the reference crate):
  src/metal_ops.rs:1121-1152  make_test_q4k (d=0.1, dmin=0.05, scales 2/mins 1, nibbles 0x55)
  src/metal_ops.rs:1154-1235  Q4_K GEMV cases (N=4/K=256, N=64/K=512, two activations)
  src/metal_ops.rs:1239-1305  BF16 GEMV cases (N=8/K=64, N=128/K=256)
  src/metal_decode.rs:2698-2740 rms_norm_gemma3, 2743-2800 rope (pos 3, theta 1e4),
      2804-2842 gelu_tanh (incl. |x| = 100), 2915-2965 rms_norm_per_head,
      3049-3157 attention_decode
  src/autograd2.rs:5658-5729  Q4_K quantize round trips, 5732-5746 f16 round trip,
      5752-5765 bf16 round trip, 6046-6054 bf16 special values
Q6_K decode and Q4_0 -> Q4_K have no reference test; their vectors use seeded
random blocks and the restatement of src/gguf_loader.rs:282-350, 482-533 and
src/autograd2.rs:1171-1320 below.

Run:  python tests/golden/make_golden.py   (writes golden.json beside this file)
"""

import json
import math
import os
import struct

import numpy as np

f32 = np.float32


def f16_bits_trunc_metal_test(val):
    """f32_to_f16_bits from src/metal_ops.rs:1106-1118 (test helper: truncating, no denormals)."""
    bits = struct.unpack("<I", struct.pack("<f", float(f32(val))))[0]
    sign = (bits >> 31) & 1
    exp = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    if exp == 0:
        return sign << 15
    new_exp = exp - 127 + 15
    if new_exp <= 0:
        return sign << 15
    if new_exp >= 31:
        return (sign << 15) | 0x7C00
    return (sign << 15) | (new_exp << 10) | (mant >> 13)


def f16_to_f32(bits):
    """src/gguf_loader.rs:947-976."""
    return f32(np.array([bits], dtype=np.uint16).view(np.float16)[0])


def q4k_f32_to_f16(val):
    """Q4KMat::f32_to_f16, src/autograd2.rs:1090-1115 (mantissa truncated)."""
    bits = int(np.array([val], dtype=np.float32).view(np.uint32)[0])
    sign = (bits >> 16) & 0x8000
    exp = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    if exp == 0xFF:
        return sign | 0x7C00 | (mant >> 13)
    new_exp = exp - 127 + 15
    if new_exp >= 0x1F:
        return sign | 0x7C00
    if new_exp <= 0:
        if new_exp < -10:
            return sign
        m = mant | 0x800000
        shift = (1 - new_exp) + 13
        return sign | (m >> shift)
    return sign | (new_exp << 10) | (mant >> 13)


def f32_to_bf16(v):
    """MatBf16::f32_to_bf16, src/autograd2.rs:709-719."""
    bits = int(np.array([v], dtype=np.float32).view(np.uint32)[0])
    if math.isnan(float(v)):
        return ((bits >> 16) | 0x0040) & 0xFFFF
    bias = 0x7FFF + ((bits >> 16) & 1)
    return ((bits + bias) & 0xFFFFFFFF) >> 16


def bf16_to_f32(b):
    return f32(np.array([int(b) << 16], dtype=np.uint32).view(np.float32)[0])


def scale_min(sc, j):
    """src/autograd2.rs:1075-1085."""
    if j < 4:
        return f32(sc[j] & 0x3F), f32(sc[j + 4] & 0x3F)
    return (f32((sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4)),
            f32((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)))


def q4k_dequant_row(blocks, cols, row):
    """Q4KMat::dequantize_row_into x86 branch, src/autograd2.rs:1326-1366."""
    nb = cols // 256
    out = np.zeros(cols, dtype=np.float32)
    for b in range(nb):
        off = (row * nb + b) * 144
        d = f16_to_f32(int(blocks[off]) | (int(blocks[off + 1]) << 8))
        dmin = f16_to_f32(int(blocks[off + 2]) | (int(blocks[off + 3]) << 8))
        sc = [int(v) for v in blocks[off + 4:off + 16]]
        qs = [int(v) for v in blocks[off + 16:off + 144]]
        for c in range(4):
            s1, m1 = scale_min(sc, 2 * c)
            s2, m2 = scale_min(sc, 2 * c + 1)
            scale1, min1, scale2, min2 = f32(d * s1), f32(dmin * m1), f32(d * s2), f32(dmin * m2)
            for l in range(32):
                q = int(qs[c * 32 + l])
                out[b * 256 + c * 64 + l] = f32(f32(scale1 * f32(q & 0xF)) - min1)
                out[b * 256 + c * 64 + 32 + l] = f32(f32(scale2 * f32(q >> 4)) - min2)
    return out


def seq_dot(w, x):
    acc = f32(0.0)
    for a, b in zip(w, x):
        acc = f32(acc + f32(f32(a) * f32(b)))
    return acc


def make_test_q4k(n_rows, k):
    """src/metal_ops.rs:1121-1152."""
    nb = k // 256
    blocks = np.zeros(n_rows * nb * 144, dtype=np.uint8)
    d_bits = f16_bits_trunc_metal_test(0.1)
    dmin_bits = f16_bits_trunc_metal_test(0.05)
    for j in range(n_rows):
        for b in range(nb):
            off = (j * nb + b) * 144
            blocks[off] = d_bits & 0xFF
            blocks[off + 1] = d_bits >> 8
            blocks[off + 2] = dmin_bits & 0xFF
            blocks[off + 3] = dmin_bits >> 8
            for i in range(4):
                blocks[off + 4 + i] = 2
            for i in range(4, 8):
                blocks[off + 4 + i] = 1
            for i in range(8, 12):
                blocks[off + 4 + i] = 0
            blocks[off + 16:off + 144] = 0x55
    return blocks


def q4k_gemv_case(name, n, k, a):
    blocks = make_test_q4k(n, k)
    exp = [float(seq_dot(q4k_dequant_row(blocks, k, j), a)) for j in range(n)]
    return {"name": name, "rows": n, "cols": k, "blocks_hex": blocks.tobytes().hex(),
            "x": [float(v) for v in a], "expected": exp, "rel_tol": 1e-3}


def bf16_gemv_case(name, n, k, wfun, afun):
    w = np.array([f32_to_bf16(f32(wfun(i))) for i in range(n * k)], dtype=np.uint16)
    a = np.array([afun(c) for c in range(k)], dtype=np.float32)
    exp = []
    for j in range(n):
        acc = f32(0.0)
        for p in range(k):
            acc = f32(acc + f32(bf16_to_f32(w[j * k + p]) * a[p]))
        exp.append(float(acc))
    return {"name": name, "rows": n, "cols": k, "w_hex": w.tobytes().hex(),
            "x": [float(v) for v in a], "expected": exp, "abs_tol": 1e-2}


def rust_as_u8(x):
    x = float(x)
    if math.isnan(x) or x <= 0.0:
        return 0
    if x >= 255.0:
        return 255
    return int(x)


def pack_scales(sv, mv):
    """src/autograd2.rs:1119-1132."""
    sc = [0] * 12
    for j in range(4):
        sc[j] = (sv[j] & 0x3F) | ((sv[j + 4] & 0x30) << 2)
        sc[j + 4] = (mv[j] & 0x3F) | ((mv[j + 4] & 0x30) << 2)
    for j in range(4):
        sc[8 + j] = (sv[j + 4] & 0x0F) | ((mv[j + 4] & 0x0F) << 4)
    return [v & 0xFF for v in sc]


def quantize_block(data):
    """Q4KMat::quantize_block, src/autograd2.rs:1171-1246."""
    data = np.asarray(data, dtype=np.float32)
    sub_scales, sub_mins = [], []
    for sb in range(8):
        sub = data[sb * 32:(sb + 1) * 32]
        smin, smax = f32(np.inf), f32(-np.inf)
        for v in sub:
            if v < smin:
                smin = v
            if v > smax:
                smax = v
        if smin >= 0.0:
            sub_mins.append(f32(0.0))
            sub_scales.append(f32(smax / f32(15.0)) if smax > 0.0 else f32(0.0))
        else:
            sub_mins.append(smin)
            sub_scales.append(f32(f32(smax - smin) / f32(15.0)) if smax > smin else f32(0.0))
    max_scale = f32(0.0)
    max_min = f32(0.0)
    for j in range(8):
        max_scale = max(max_scale, sub_scales[j])
        max_min = max(max_min, f32(-sub_mins[j]))
    d = f32(max_scale / f32(63.0)) if max_scale > 0.0 else f32(0.0)
    dmin = f32(max_min / f32(63.0)) if max_min > 0.0 else f32(0.0)
    sv, mv = [0] * 8, [0] * 8
    if d > 0.0:
        inv_d = f32(f32(1.0) / d)
        for j in range(8):
            sv[j] = min(rust_as_u8(f32(f32(sub_scales[j] * inv_d) + f32(0.5))), 63)
    if dmin > 0.0:
        inv_dmin = f32(f32(1.0) / dmin)
        for j in range(8):
            mv[j] = min(rust_as_u8(f32(f32(f32(-sub_mins[j]) * inv_dmin) + f32(0.5))), 63)
    d16, dmin16 = q4k_f32_to_f16(d), q4k_f32_to_f16(dmin)
    out = [d16 & 0xFF, d16 >> 8, dmin16 & 0xFF, dmin16 >> 8] + pack_scales(sv, mv)
    d_val, dmin_val = f16_to_f32(d16), f16_to_f32(dmin16)
    qs = [0] * 128
    for c in range(4):
        scale1 = f32(d_val * f32(sv[2 * c]))
        min1 = f32(dmin_val * f32(mv[2 * c]))
        scale2 = f32(d_val * f32(sv[2 * c + 1]))
        min2 = f32(dmin_val * f32(mv[2 * c + 1]))
        for l in range(32):
            q_lo = min(rust_as_u8(f32(f32(f32(data[c * 64 + l] + min1) / scale1) + f32(0.5))), 15) if scale1 > 0.0 else 0
            q_hi = min(rust_as_u8(f32(f32(f32(data[c * 64 + 32 + l] + min2) / scale2) + f32(0.5))), 15) if scale2 > 0.0 else 0
            qs[c * 32 + l] = q_lo | (q_hi << 4)
    return bytes(out + qs)


def quantize_case(name, rows, cols, fn):
    m = np.array([[fn(r, c) for c in range(cols)] for r in range(rows)], dtype=np.float32)
    blocks = b"".join(quantize_block(m[r, b * 256:(b + 1) * 256]) for r in range(rows) for b in range(cols // 256))
    blk = np.frombuffer(blocks, dtype=np.uint8)
    max_err = 0.0
    for r in range(rows):
        row = q4k_dequant_row(blk, cols, r)
        max_err = max(max_err, float(np.max(np.abs(row - m[r]))))
    return {"name": name, "rows": rows, "cols": cols, "input": m.reshape(-1).tolist(),
            "blocks_hex": blocks.hex(), "max_err": max_err, "max_err_bound": 0.15}


def q6k_decode(data, n_elem):
    """GgufFile::decode_q6k_to_f32, src/gguf_loader.rs:482-533."""
    out = np.zeros(n_elem, dtype=np.float32)
    for b in range((n_elem + 255) // 256):
        blk = data[b * 210:(b + 1) * 210]
        ql_all, qh_all, sc_all = blk[0:128], blk[128:192], blk[192:208]
        d = f16_to_f32(int(blk[208]) | (int(blk[209]) << 8))
        base = b * 256
        for j in range(2):
            ql, qh, sc = ql_all[j * 64:(j + 1) * 64], qh_all[j * 32:(j + 1) * 32], sc_all[j * 8:(j + 1) * 8]
            yb = base + j * 128
            for l in range(32):
                is_ = l // 16
                q1 = ((int(ql[l]) & 0xF) | (((int(qh[l]) >> 0) & 3) << 4)) - 32
                q2 = ((int(ql[l + 32]) & 0xF) | (((int(qh[l]) >> 2) & 3) << 4)) - 32
                q3 = ((int(ql[l]) >> 4) | (((int(qh[l]) >> 4) & 3) << 4)) - 32
                q4 = ((int(ql[l + 32]) >> 4) | (((int(qh[l]) >> 6) & 3) << 4)) - 32
                s = [f32(d * f32(np.int8(np.uint8(sc[is_ + 2 * t])))) for t in range(4)]
                for t, q in enumerate((q1, q2, q3, q4)):
                    if yb + l + 32 * t < n_elem:
                        out[yb + l + 32 * t] = f32(s[t] * f32(q))
    return out


def q4_0_to_q4k(data, rows, cols):
    """decode_q4_0_to_q4mat (src/gguf_loader.rs:282-350) + Q4KMat::from_q4mat
    (src/autograd2.rs:1291-1320) via Q4Mat::dequantize_row_into (:2390-2410)."""
    n = rows * cols
    vals = np.zeros(n, dtype=np.float32)
    for b in range((n + 31) // 32):
        blk = data[b * 18:(b + 1) * 18]
        scale = f16_to_f32(int(blk[0]) | (int(blk[1]) << 8))
        for k in range(16):
            src = int(blk[2 + k])
            for e, nib in ((b * 32 + k, src & 0xF), (b * 32 + k + 16, (src >> 4) & 0xF)):
                if e < n:
                    v = (nib - 8) & 0xF
                    q = v - 16 if v >= 8 else v
                    vals[e] = f32(f32(q) * scale)
    out = b""
    for r in range(rows):
        for bb in range(cols // 256):
            out += quantize_block(vals[r * cols + bb * 256:r * cols + (bb + 1) * 256])
    return out


def main():
    rng = np.random.default_rng(20241201)
    cases = {}
    cases["q4k_gemv"] = [
        q4k_gemv_case("metal_ops_1154_small", 4, 256, np.array([(c + 1.0) * 0.01 for c in range(256)], dtype=np.float32)),
        q4k_gemv_case("metal_ops_1185_larger", 64, 512, np.array([((c % 7) - 3.0) * 0.1 for c in range(512)], dtype=np.float32)),
        q4k_gemv_case("metal_ops_1210_reuse_a1", 4, 256, np.array([c * 0.01 for c in range(256)], dtype=np.float32)),
        q4k_gemv_case("metal_ops_1210_reuse_a2", 4, 256, np.array([(256 - c) * 0.01 for c in range(256)], dtype=np.float32)),
    ]
    cases["bf16_gemv"] = [
        bf16_gemv_case("metal_ops_1239_small", 8, 64, lambda i: ((i % 17) - 8.0) * 0.1, lambda c: (c + 1.0) * 0.05),
        bf16_gemv_case("metal_ops_1270_larger", 128, 256, lambda i: ((i % 31) - 15.0) * 0.01, lambda c: ((c % 13) - 6.0) * 0.1),
    ]
    # rms_norm_gemma3 (src/metal_decode.rs:2698-2740), test-formula expected values.
    x = np.array([1, 2, 3, 4, 5, 6, 7, 8], dtype=np.float32)
    g = np.array([0.1, 0.2, 0.0, -0.1, 0.05, 0.0, 0.0, 0.15], dtype=np.float32)
    sq = f32(0.0)
    for v in x:
        sq = f32(sq + f32(v * v))
    rms = f32(np.sqrt(f32(f32(sq / f32(8)) + f32(1e-6))))
    cases["rms_norm"] = {"x": x.tolist(), "gamma": g.tolist(), "eps": 1e-6,
                         "expected": [float(f32(f32(xi / rms) * f32(f32(1.0) + gi))) for xi, gi in zip(x, g)],
                         "abs_tol": 1e-5}
    # rms_norm_per_head (src/metal_decode.rs:2915-2965).
    gh = np.array([0.1, 0.2, 0.0, -0.1], dtype=np.float32)
    exp = []
    for h in range(2):
        xs = x[h * 4:(h + 1) * 4]
        sq = f32(0.0)
        for v in xs:
            sq = f32(sq + f32(v * v))
        rms = f32(np.sqrt(f32(f32(sq / f32(4)) + f32(1e-6))))
        exp += [float(f32(f32(xs[i] / rms) * f32(f32(1.0) + gh[i]))) for i in range(4)]
    cases["per_head_norm"] = {"x": x.tolist(), "gamma": gh.tolist(), "n_heads": 2, "head_dim": 4, "eps": 1e-6,
                              "expected": exp, "abs_tol": 1e-4}
    # rope_neox (src/metal_decode.rs:2743-2800): 2 heads x 4, theta 1e4, pos 3.
    exp = x.copy()
    for h in range(2):
        for i in range(2):
            angle = f32(f32(f32(3.0) * f32(1.0)) / f32(np.power(f32(10000.0), f32(f32(2.0 * i) / f32(4.0)))))
            ca, sa = math.cos(float(angle)), math.sin(float(angle))
            c0, c1 = h * 4 + i, h * 4 + i + 2
            exp[c0] = f32(x[c0] * ca - x[c1] * sa)
            exp[c1] = f32(x[c0] * sa + x[c1] * ca)
    cases["rope"] = {"x": x.tolist(), "n_heads": 2, "head_dim": 4, "theta": 10000.0, "freq_scale": 1.0, "pos": 3,
                     "expected": exp.tolist(), "abs_tol": 1e-5}
    # gelu_tanh (src/metal_decode.rs:2804-2842), computed in float64.
    gx = [-2.0, -1.0, 0.0, 0.5, 1.0, 2.0, 3.0, 4.0, 10.0, 12.655, -15.0, 20.0, -25.0, 100.0]
    cases["gelu"] = {"x": gx, "expected": [0.5 * v * (1.0 + math.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3))) for v in gx],
                     "abs_tol": 1e-5}
    # attention_decode (src/metal_decode.rs:3049-3157): 2 q heads, 1 kv head, d=4, 3 positions.
    q = [1.0, 0.0, 1.0, 0.0, 0.0, 1.0, 0.0, 1.0]
    kc = [1.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0]
    vc = [10.0, 20.0, 30.0, 40.0, 50.0, 60.0, 70.0, 80.0, 90.0, 100.0, 110.0, 120.0]
    out = [0.0] * 8
    for qh in range(2):
        sc = [sum(q[qh * 4 + d] * kc[c * 4 + d] for d in range(4)) * 0.5 for c in range(3)]
        mx = max(sc)
        e = [math.exp(s - mx) for s in sc]
        ssum = sum(e)
        for c in range(3):
            for d in range(4):
                out[qh * 4 + d] += e[c] / ssum * vc[c * 4 + d]
    cases["attention"] = {"q": q, "k_cache": kc, "v_cache": vc, "n_q_heads": 2, "n_kv_heads": 1, "head_dim": 4,
                          "k_start": 0, "k_end": 3, "scale": 0.5, "expected": out, "abs_tol": 1e-4}
    # Q4_K quantize round trips (src/autograd2.rs:5658-5729).
    cases["q4k_quantize"] = [
        quantize_case("autograd2_5658_ramp", 4, 256, lambda r, c: ((r * 256 + c) / 1024.0) * 2.0 - 1.0),
        quantize_case("autograd2_5689_zeros", 2, 256, lambda r, c: 0.0),
        quantize_case("autograd2_5706_sin", 16, 512, lambda r, c: math.sin((r * 512 + c) * 0.001)),
    ]
    # f16 round trip (src/autograd2.rs:5732-5746) through Q4KMat::f32_to_f16 / f16_to_f32.
    vals = [0.0, 1.0, -1.0, 0.5, 65504.0, -65504.0, 0.001, 100.0, 1e-5, 3e-8, 1e-9, -7e-6, 70000.0]
    cases["f16"] = {"values": vals, "bits": [q4k_f32_to_f16(f32(v)) for v in vals],
                    "back": [float(f16_to_f32(q4k_f32_to_f16(f32(v)))) for v in vals]}
    # bf16 (src/autograd2.rs:5752-5765, 6046-6054) plus rounding-tie values.
    bvals = [0.0, 1.0, -1.0, 2.0, 0.5, 16.0, -8.0, 0.125, 3.14159, float("inf"), float("-inf"),
             1.00390625, 1.01171875, -2.00781250, 1e-30]
    cases["bf16"] = {"values": [str(v) for v in bvals], "bits": [f32_to_bf16(f32(v)) for v in bvals]}
    # Q6_K -> f32 -> bf16 on seeded random blocks (2 blocks).
    q6 = rng.integers(0, 256, size=2 * 210, dtype=np.uint8)
    for b in range(2):  # keep d finite and modest
        dbits = q4k_f32_to_f16(f32(rng.uniform(1e-3, 2e-2)))
        q6[b * 210 + 208] = dbits & 0xFF
        q6[b * 210 + 209] = dbits >> 8
    dec = q6k_decode(q6, 512)
    cases["q6k"] = {"n_elem": 512, "bytes_hex": q6.tobytes().hex(), "f32": dec.tolist(),
                    "bf16": [f32_to_bf16(v) for v in dec]}
    # Q4_0 -> Q4_K on seeded random blocks (2 rows x 256).
    q40 = rng.integers(0, 256, size=16 * 18, dtype=np.uint8)
    for b in range(16):
        sbits = q4k_f32_to_f16(f32(rng.uniform(1e-3, 5e-2)))
        q40[b * 18] = sbits & 0xFF
        q40[b * 18 + 1] = sbits >> 8
    cases["q4_0_to_q4k"] = {"rows": 2, "cols": 256, "q4_0_hex": q40.tobytes().hex(),
                            "q4k_hex": q4_0_to_q4k(q40, 2, 256).hex()}
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.json")
    with open(path, "w") as f:
        json.dump(cases, f, indent=1, sort_keys=True)
    print("wrote", path)


if __name__ == "__main__":
    main()
