"""Gemma 3 configuration and host-side weight containers.

Mirrors the reference crate's Config4 (src/transformer4.rs:51-144), Q4KMat
(src/autograd2.rs:1036-1042) and MatBf16 (src/autograd2.rs:688-692), and
builds seeded synthetic models for benchmarks and parity tests with the
library's counter-based generators (rt_synth_*; host only, no GPU needed).
"""

import ctypes
from dataclasses import dataclass, field, replace
from typing import List, Optional

import numpy as np

from ._lib import lib


@dataclass
class Config4:
    """Gemma 3 hyperparameters (Config4, src/transformer4.rs:51-80)."""

    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    intermediate_size: int
    head_dim: int
    sliding_window: Optional[int]
    rope_theta_local: float
    rope_theta_global: float
    rope_freq_scale_local: float
    rope_freq_scale_global: float
    rms_norm_eps: float
    query_pre_attn_scalar: float
    eos_token_id: int = 1
    max_position_embeddings: int = 32768

    @staticmethod
    def gemma3_1b():
        """Config4::gemma3_1b (src/transformer4.rs:84-105)."""
        return Config4(262144, 1152, 26, 4, 1, 6912, 256, 512, 10_000.0, 1_000_000.0, 1.0, 1.0, 1e-6, 256.0)

    @staticmethod
    def gemma3_4b(vocab_size=262208):
        """Config4::gemma3_4b (src/transformer4.rs:112-131).  The reference sets
        vocab_size 262208 but sizes the LM head from the embedding table's rows
        (lm_head_vocab, src/metal_decode.rs:826, 1080); the benchmark's model
        has a 262144-row table, so callers pass vocab_size=262144."""
        return Config4(vocab_size, 2560, 34, 8, 4, 10240, 256, 1024, 10_000.0, 1_000_000.0, 1.0, 0.125, 1e-6, 256.0)

    @staticmethod
    def gemma3_27b(vocab_size=262144):
        """Gemma 3 27B.  The reference has no constructor for it; the sizes are
        BASELINE config 4 (62 layers, hidden 5376, FFN 21504, 32 / 16 heads,
        head_dim 128).  query_pre_attn_scalar = hidden / heads = 168 and the
        global-layer RoPE scale 1/8 follow the published model card; the
        local:global pattern and thetas are Config4's."""
        return Config4(vocab_size, 5376, 62, 32, 16, 21504, 128, 1024, 10_000.0, 1_000_000.0, 1.0, 0.125, 1e-6, 168.0)

    @staticmethod
    def tiny():
        """tiny_cfg of the reference's tests (src/transformer4.rs:3114-3133:
        2 query heads, 1 KV head, window 8), widened to the kernels' granularity
        (hidden and FFN multiples of 256 for Q4_K super-blocks, head_dim a
        multiple of 32) and given 6 layers so that layer 5 is a global layer."""
        return Config4(512, 256, 6, 2, 1, 512, 128, 8, 10_000.0, 1_000_000.0, 1.0, 0.125, 1e-6, 128.0,
                       max_position_embeddings=128)

    def is_global_layer(self, i):
        """Config4::is_global_layer (src/transformer4.rs:141-143)."""
        return i % 6 == 5

    def with_layers(self, n):
        return replace(self, num_hidden_layers=n)


@dataclass
class Q4KMat:
    """Raw GGUF Q4_K blocks of a [rows, cols] matrix, 144 bytes per 256 values."""

    rows: int
    cols: int
    blocks: np.ndarray  # uint8, rows * cols / 256 * 144

    def size_bytes(self):
        return self.blocks.nbytes


@dataclass
class MatBf16:
    """BF16 bits of a [rows, cols] matrix."""

    rows: int
    cols: int
    data: np.ndarray  # uint16, rows * cols

    def size_bytes(self):
        return self.data.nbytes


@dataclass
class Gemma3LayerWeights:
    q: np.ndarray
    k: np.ndarray
    v: np.ndarray
    o: np.ndarray
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray
    attn_norm: np.ndarray
    post_attn_norm: np.ndarray
    pre_ffn_norm: np.ndarray
    post_ffn_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray


@dataclass
class Gemma3Weights:
    """All decode-path weights of a Gemma 3 model, on the host.

    Projections are Q4_K blocks ([out, in] rows); norm vectors hold gamma as the
    kernels apply it (out = x_hat * (1 + gamma)); the BF16 embedding is tied with
    the LM head (src/transformer4.rs:1015-1029)."""

    cfg: Config4
    layers: List[Gemma3LayerWeights] = field(default_factory=list)
    embed: Optional[np.ndarray] = None  # uint16 [vocab * hidden]
    final_norm: Optional[np.ndarray] = None

    def q4k_bytes(self):
        return sum(getattr(L, n).nbytes for L in self.layers for n in ("q", "k", "v", "o", "gate", "up", "down"))


def _ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


# The generator functions below run in whichever loaded library `gen` names
# (default: librtcuda.so).  Any library that links synth.cpp exports the same
# rt_synth_* symbols and produces the same bytes; a CPU-only caller passes its
# own handle so that it never maps the CUDA library.
def _gen(gen):
    return gen if gen is not None else lib()


def synth_q4k(seed, stream, rows, cols, gen=None):
    """Seeded Q4_K blocks distributed as BASELINE config 0 describes."""
    out = np.empty(rows * (cols // 256) * 144, dtype=np.uint8)
    _gen(gen).rt_synth_q4k(seed, stream, rows, cols, _ptr(out))
    return out


def synth_normal(seed, stream, n, mean=0.0, std=1.0, gen=None):
    out = np.empty(n, dtype=np.float32)
    _gen(gen).rt_synth_normal_f32(seed, stream, n, mean, std, _ptr(out))
    return out


def synth_normal_bf16(seed, stream, n, mean=0.0, std=1.0, gen=None):
    out = np.empty(n, dtype=np.uint16)
    _gen(gen).rt_synth_normal_bf16(seed, stream, n, mean, std, _ptr(out))
    return out


def synth_tokens(seed, stream, n, vocab, gen=None):
    out = np.empty(n, dtype=np.int32)
    _gen(gen).rt_synth_tokens(seed, stream, n, vocab, _ptr(out))
    return out


def synth_bytes(seed, stream, n, gen=None):
    out = np.empty(n, dtype=np.uint8)
    _gen(gen).rt_synth_bytes(seed, stream, n, _ptr(out))
    return out


def synth_gemma3(cfg: Config4, seed=1234, norm_std=0.1, embed_std=0.02, gen=None):
    """Random-init Gemma 3 weights: Q4_K projections as BASELINE config 0,
    norm gamma ~ N(0, norm_std), embedding bf16 ~ N(0, embed_std).  `gen`: the
    library whose rt_synth_* generators to run (default librtcuda.so)."""
    H, D, F = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
    q, kv = cfg.num_attention_heads * D, cfg.num_key_value_heads * D
    w = Gemma3Weights(cfg)
    for i in range(cfg.num_hidden_layers):
        s = 1000 + 32 * i
        w.layers.append(Gemma3LayerWeights(
            q=synth_q4k(seed, s + 0, q, H, gen), k=synth_q4k(seed, s + 1, kv, H, gen),
            v=synth_q4k(seed, s + 2, kv, H, gen), o=synth_q4k(seed, s + 3, H, q, gen),
            gate=synth_q4k(seed, s + 4, F, H, gen), up=synth_q4k(seed, s + 5, F, H, gen),
            down=synth_q4k(seed, s + 6, H, F, gen),
            attn_norm=synth_normal(seed, s + 7, H, 0.0, norm_std, gen),
            post_attn_norm=synth_normal(seed, s + 8, H, 0.0, norm_std, gen),
            pre_ffn_norm=synth_normal(seed, s + 9, H, 0.0, norm_std, gen),
            post_ffn_norm=synth_normal(seed, s + 10, H, 0.0, norm_std, gen),
            q_norm=synth_normal(seed, s + 11, D, 0.0, norm_std, gen),
            k_norm=synth_normal(seed, s + 12, D, 0.0, norm_std, gen)))
    w.embed = synth_normal_bf16(seed, 7, cfg.vocab_size * H, 0.0, embed_std, gen)
    w.final_norm = synth_normal(seed, 8, H, 0.0, norm_std, gen)
    return w
