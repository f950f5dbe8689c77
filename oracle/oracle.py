"""ctypes binding of liboracle.so -- TEST INFRASTRUCTURE ONLY.

The CPU oracle restates rich-triplet's reference CPU path (see oracle.c).  It
is the checker for the CUDA product path and the timed CPU baseline; only
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg
import this module.  The product package never does.
"""

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_u8p = ctypes.POINTER(ctypes.c_uint8)
_c_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64 = ctypes.c_int64


def build():
    """Compile liboracle.so with the committed Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)


_SOURCES = (os.path.join(_HERE, "oracle.c"), os.path.join(_HERE, "..", "rich_triplet_b200", "csrc", "synth.cpp"))


def _load():
    stale = not os.path.exists(_LIB_PATH) or any(
        os.path.exists(src) and os.path.getmtime(_LIB_PATH) < os.path.getmtime(src) for src in _SOURCES)
    if stale:
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    sig = {
        "or_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
        "or_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
        "or_bf16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
        "or_f32_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
        "or_q4k_quantize": (None, [_c_f32p, _i64, _i64, _c_u8p]),
        "or_q4k_dequantize_row": (None, [_c_u8p, _i64, _i64, _c_f32p]),
        "or_q4k_to_f32": (None, [_c_u8p, _i64, _c_f32p]),
        "or_q4k_dot_row": (ctypes.c_float, [_c_u8p, _i64, _i64, _c_f32p]),
        "or_bf16_dot_row": (ctypes.c_float, [_c_u16p, _i64, _i64, _c_f32p]),
        "or_q4k_gemv": (None, [_c_u8p, _i64, _i64, _c_f32p, _c_f32p, ctypes.c_int]),
        "or_bf16_gemv": (None, [_c_u16p, _i64, _i64, _c_f32p, _c_f32p, ctypes.c_int]),
        "or_q4k_gemm": (None, [_c_u8p, _i64, _i64, _c_f32p, _i64, _c_f32p]),
        "or_q4_0_to_q4k": (None, [_c_u8p, _i64, _i64, _c_u8p]),
        "or_q6k_to_f32": (None, [_c_u8p, _i64, _c_f32p]),
        "or_q6k_to_bf16": (None, [_c_u8p, _i64, _c_u16p]),
        "or_rms_norm_gemma3": (None, [_c_f32p, _c_f32p, _i64, ctypes.c_float, _c_f32p]),
        "or_per_head_norm": (None, [_c_f32p, _c_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, _c_f32p]),
        "or_rope": (None, [_c_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, _i64, ctypes.c_float]),
        "or_rope_cos_sin": (None, [ctypes.c_float, ctypes.c_int, _i64, ctypes.c_float, ctypes.c_int, _c_f32p, _c_f32p]),
        "or_gelu_tanh": (ctypes.c_float, [ctypes.c_float]),
        "or_gqa_attention_decode": (None, [_c_f32p, _c_f32p, _c_f32p, _i64, _i64, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_float, _c_f32p]),
        "or_sample_greedy": (_i64, [_c_f32p, _i64]),
        "or_set_threads": (None, [ctypes.c_int]),
        "or_model_create": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_void_p, _c_u16p, _c_f32p, _i64, ctypes.c_int]),
        "or_model_destroy": (None, [ctypes.c_void_p]),
        "or_model_step": (ctypes.c_int, [ctypes.c_void_p, _i64, _c_f32p, _c_f32p]),
        "or_model_seq_len": (_i64, [ctypes.c_void_p]),
        "or_model_set_seq_len": (None, [ctypes.c_void_p, _i64]),
        "or_model_kcache": (_c_f32p, [ctypes.c_void_p, ctypes.c_int]),
        "or_model_vcache": (_c_f32p, [ctypes.c_void_p, ctypes.c_int]),
        # the seeded generator (synth.cpp, linked in): the same bytes as the
        # product library's rt_synth_* for the same arguments
        "rt_synth_q4k": (None, [ctypes.c_uint64, ctypes.c_uint64, _i64, _i64, ctypes.c_void_p]),
        "rt_synth_normal_f32": (None, [ctypes.c_uint64, ctypes.c_uint64, _i64, ctypes.c_float, ctypes.c_float,
                                       ctypes.c_void_p]),
        "rt_synth_normal_bf16": (None, [ctypes.c_uint64, ctypes.c_uint64, _i64, ctypes.c_float, ctypes.c_float,
                                        ctypes.c_void_p]),
        "rt_synth_tokens": (None, [ctypes.c_uint64, ctypes.c_uint64, _i64, ctypes.c_int32, ctypes.c_void_p]),
        "rt_synth_bytes": (None, [ctypes.c_uint64, ctypes.c_uint64, _i64, ctypes.c_void_p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _p(a, t):
    return a.ctypes.data_as(t)


def f32p(a):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return _p(a, _c_f32p)


def u8p(a):
    assert a.dtype == np.uint8 and a.flags["C_CONTIGUOUS"]
    return _p(a, _c_u8p)


def u16p(a):
    assert a.dtype == np.uint16 and a.flags["C_CONTIGUOUS"]
    return _p(a, _c_u16p)


def q4k_gemv(blocks, rows, cols, x, nthreads=0):
    """Q4KMat::gemv_mt (x86 dot_row per row)."""
    y = np.empty(rows, dtype=np.float32)
    lib.or_q4k_gemv(u8p(blocks), rows, cols, f32p(np.ascontiguousarray(x, np.float32)), f32p(y), nthreads)
    return y


def bf16_gemv(w, rows, cols, x, nthreads=0):
    """MatBf16::gemv_mt."""
    y = np.empty(rows, dtype=np.float32)
    lib.or_bf16_gemv(u16p(w), rows, cols, f32p(np.ascontiguousarray(x, np.float32)), f32p(y), nthreads)
    return y


def q4k_gemm(blocks, n, k, a):
    """Q4KMat::matmul_q4k_t (no-BLAS order), C[M,N] = A[M,K] . W^T."""
    a = np.ascontiguousarray(a, np.float32)
    c = np.empty((a.shape[0], n), dtype=np.float32)
    lib.or_q4k_gemm(u8p(blocks), n, k, f32p(a), a.shape[0], f32p(c))
    return c


def q4k_dequantize(blocks, rows, cols):
    out = np.empty((rows, cols), dtype=np.float32)
    for r in range(rows):
        lib.or_q4k_dequantize_row(u8p(blocks), cols, r, f32p(out[r]))
    return out


def q4k_quantize(mat):
    mat = np.ascontiguousarray(mat, np.float32)
    rows, cols = mat.shape
    out = np.empty(rows * (cols // 256) * 144, dtype=np.uint8)
    lib.or_q4k_quantize(f32p(mat), rows, cols, u8p(out))
    return out


def q4_0_to_q4k(q4_0, rows, cols):
    out = np.empty(rows * (cols // 256) * 144, dtype=np.uint8)
    lib.or_q4_0_to_q4k(u8p(np.ascontiguousarray(q4_0, np.uint8)), rows, cols, u8p(out))
    return out


def q6k_to_f32(data, n):
    out = np.empty(n, dtype=np.float32)
    lib.or_q6k_to_f32(u8p(np.ascontiguousarray(data, np.uint8)), n, f32p(out))
    return out


def q6k_to_bf16(data, n):
    out = np.empty(n, dtype=np.uint16)
    lib.or_q6k_to_bf16(u8p(np.ascontiguousarray(data, np.uint8)), n, u16p(out))
    return out


def rms_norm_gemma3(x, gamma, eps=1e-6):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib.or_rms_norm_gemma3(f32p(x), f32p(np.ascontiguousarray(gamma, np.float32)), x.size, eps, f32p(out))
    return out


def per_head_norm(x, gamma, n_heads, head_dim, eps=1e-6):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib.or_per_head_norm(f32p(x), f32p(np.ascontiguousarray(gamma, np.float32)), n_heads, head_dim, eps, f32p(out))
    return out


def rope(x, n_heads, head_dim, theta, pos, freq_scale):
    x = np.array(x, dtype=np.float32)
    lib.or_rope(f32p(x), n_heads, head_dim, theta, pos, freq_scale)
    return x


def gelu_tanh(x):
    return np.array([lib.or_gelu_tanh(float(v)) for v in np.asarray(x, np.float32)], dtype=np.float32)


def gqa_attention_decode(q, k_cache, v_cache, k_start, k_end, n_q_heads, n_kv_heads, d_head, scale):
    out = np.empty(n_q_heads * d_head, dtype=np.float32)
    lib.or_gqa_attention_decode(f32p(np.ascontiguousarray(q, np.float32)), f32p(np.ascontiguousarray(k_cache, np.float32)),
                                f32p(np.ascontiguousarray(v_cache, np.float32)), k_start, k_end, n_q_heads, n_kv_heads,
                                d_head, scale, f32p(out))
    return out


def sample_greedy(logits):
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib.or_sample_greedy(f32p(logits), logits.size))


class _Cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("vocab", "hidden", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn",
                                            "sliding_window")] + \
               [(n, ctypes.c_float) for n in ("theta_local", "theta_global", "fs_local", "fs_global", "eps",
                                              "query_pre_attn_scalar")]


class _Layer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("q", "k", "v", "o", "gate", "up", "down", "attn_norm", "post_attn_norm",
                                               "pre_ffn_norm", "post_ffn_norm", "q_norm", "k_norm")]


class OracleModel:
    """CPU Gemma 3 decode (Gemma3Model::generate_cached_streaming's non-Metal loop,
    src/transformer4.rs:2357-2409), one token per step with an f32 KV cache.

    `weights` is a rich_triplet_b200.model.Gemma3Weights-like object holding host
    numpy arrays; the arrays must stay alive while this model exists.
    """

    def __init__(self, cfg, weights, cap, nthreads=0):
        self.cfg = cfg
        self._keep = weights
        c = _Cfg(cfg.vocab_size, cfg.hidden_size, cfg.num_hidden_layers, cfg.num_attention_heads,
                 cfg.num_key_value_heads, cfg.head_dim, cfg.intermediate_size, cfg.sliding_window or 0,
                 cfg.rope_theta_local, cfg.rope_theta_global, cfg.rope_freq_scale_local, cfg.rope_freq_scale_global,
                 cfg.rms_norm_eps, cfg.query_pre_attn_scalar)
        layers = (_Layer * cfg.num_hidden_layers)()
        for i, L in enumerate(weights.layers):
            for n in ("q", "k", "v", "o", "gate", "up", "down", "attn_norm", "post_attn_norm", "pre_ffn_norm",
                      "post_ffn_norm", "q_norm", "k_norm"):
                setattr(layers[i], n, getattr(L, n).ctypes.data)
        self._h = lib.or_model_create(ctypes.byref(c), layers, u16p(weights.embed), f32p(weights.final_norm), cap, nthreads)
        self.vocab = cfg.vocab_size
        self.hidden = cfg.hidden_size

    def step(self, token, want_hidden=False):
        logits = np.empty(self.vocab, dtype=np.float32)
        hid = np.empty(self.hidden, dtype=np.float32) if want_hidden else None
        rc = lib.or_model_step(self._h, int(token), f32p(logits), f32p(hid) if want_hidden else None)
        if rc != 0:
            raise RuntimeError("oracle KV cache full")
        return (logits, hid) if want_hidden else logits

    @property
    def seq_len(self):
        return int(lib.or_model_seq_len(self._h))

    def set_seq_len(self, s):
        lib.or_model_set_seq_len(self._h, s)

    def kv(self, layer, seq_len):
        n = seq_len * self.cfg.num_key_value_heads * self.cfg.head_dim
        k = np.ctypeslib.as_array(lib.or_model_kcache(self._h, layer), shape=(n,)).copy()
        v = np.ctypeslib.as_array(lib.or_model_vcache(self._h, layer), shape=(n,)).copy()
        return k, v

    def close(self):
        if self._h:
            lib.or_model_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()
