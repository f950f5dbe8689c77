"""Qwen 3.5 decode on the GPU: the hybrid Gated DeltaNet / full-attention
model of the reference's src/transformer_qwen35.rs behind rt_qwen35_* (the
engine the reference's MetalDecodeContextQwen35 provides on Metal,
src/metal_decode_qwen35.rs).

Qwen35Config mirrors ConfigQwen35 (src/transformer_qwen35.rs:32-151),
synth_qwen35 makes seeded random-init weights of that architecture (Q4_K
projections, f32 vectors, a BF16 embedding tied with the LM head), and
CudaQwen35Decoder runs one token per step() call, returning the logits.
"""

import ctypes
from dataclasses import dataclass, field, replace

import numpy as np

from ._lib import RT_FMT_BF16, RT_FMT_Q4K, RtQwen35Cfg, RtQwen35Layer, check, lib
from .model import synth_normal, synth_normal_bf16, synth_q4k
from .ops import Context, DeviceWeight


@dataclass(frozen=True)
class Qwen35Config:
    """ConfigQwen35 (src/transformer_qwen35.rs:32-58)."""
    vocab_size: int = 248320
    hidden_size: int = 2560
    num_hidden_layers: int = 32
    num_attention_heads: int = 16
    num_key_value_heads: int = 4
    head_dim: int = 256
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 32
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    intermediate_size: int = 9216
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10_000_000.0
    partial_rotary_factor: float = 0.25
    full_attention_interval: int = 4

    @classmethod
    def qwen35_4b(cls):
        """ConfigQwen35::qwen35_4b (src/transformer_qwen35.rs:61-83)."""
        return cls()

    @classmethod
    def qwen35_0_8b(cls):
        """ConfigQwen35::qwen35_0_8b (src/transformer_qwen35.rs:109-131)."""
        return cls(hidden_size=1024, num_hidden_layers=24, num_attention_heads=8, num_key_value_heads=2,
                   linear_num_value_heads=16, intermediate_size=3584)

    def with_layers(self, n):
        return replace(self, num_hidden_layers=n)

    def is_full_attention_layer(self, layer):
        """ConfigQwen35::is_full_attention_layer (src/transformer_qwen35.rs:133-135)."""
        return (layer + 1) % self.full_attention_interval == 0

    @property
    def qkv_dim(self):
        """deltanet_qkv_dim (src/transformer_qwen35.rs:138-142)."""
        return self.linear_num_key_heads * self.linear_key_head_dim * 2 + \
            self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def value_dim(self):
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def rope_dim(self):
        """rope_dim (src/transformer_qwen35.rs:144-146)."""
        return int(self.head_dim * self.partial_rotary_factor)

    def to_c(self):
        c = RtQwen35Cfg()
        for n in ("vocab_size", "hidden_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
                  "head_dim", "linear_num_key_heads", "linear_num_value_heads", "linear_key_head_dim",
                  "linear_value_head_dim", "linear_conv_kernel_dim", "intermediate_size", "full_attention_interval"):
            setattr(c, n, getattr(self, n))
        c.rope_dim = self.rope_dim
        c.rms_norm_eps = self.rms_norm_eps
        c.rope_theta = self.rope_theta
        return c


# projection name -> (rows, cols) of its [out, in] matrix
def _proj_shapes(cfg: Qwen35Config, full: bool):
    H, F = cfg.hidden_size, cfg.intermediate_size
    s = {"gate": (F, H), "up": (F, H), "down": (H, F)}
    if full:
        D = cfg.head_dim
        s.update(q=(2 * cfg.num_attention_heads * D, H), k=(cfg.num_key_value_heads * D, H),
                 v=(cfg.num_key_value_heads * D, H), o=(H, cfg.num_attention_heads * D))
    else:
        nv = cfg.linear_num_value_heads
        s.update(in_qkv=(cfg.qkv_dim, H), in_z=(cfg.value_dim, H), in_a=(nv, H), in_b=(nv, H),
                 out_proj=(H, cfg.value_dim))
    return s


@dataclass
class Qwen35Layer:
    """One Qwen35Block's weights: Q4_K bytes per projection, f32 vectors."""
    full: bool
    proj: dict = field(default_factory=dict)   # name -> Q4_K bytes
    vec: dict = field(default_factory=dict)    # name -> f32 array


@dataclass
class Qwen35Weights:
    cfg: Qwen35Config
    layers: list
    embed: np.ndarray       # bf16 bits [vocab * hidden]
    final_norm: np.ndarray  # f32 [hidden]


def synth_qwen35(cfg: Qwen35Config, seed=1234, norm_std=0.1, embed_std=0.02, gen=None):
    """Seeded random-init Qwen 3.5 weights (no checkpoint exists here): Q4_K
    projections distributed as the other synthetic models', norm gammas
    ~ N(0, norm_std), the DeltaNet output norm weight ~ N(1, norm_std),
    conv1d weights ~ N(0, 0.5), A_log and dt_bias ~ N(0, 0.5), the BF16
    embedding ~ N(0, embed_std).  `gen`: the library whose rt_synth_*
    generators to run (default librtcuda.so)."""
    H = cfg.hidden_size
    layers = []
    for i in range(cfg.num_hidden_layers):
        full = cfg.is_full_attention_layer(i)
        L = Qwen35Layer(full)
        base = 1000 + 100 * i
        for j, (name, (r, c)) in enumerate(sorted(_proj_shapes(cfg, full).items())):
            L.proj[name] = synth_q4k(seed, base + j, r, c, gen=gen)
        L.vec["input_norm"] = synth_normal(seed, base + 50, H, 0.0, norm_std, gen=gen)
        L.vec["post_attn_norm"] = synth_normal(seed, base + 51, H, 0.0, norm_std, gen=gen)
        if full:
            L.vec["q_norm"] = synth_normal(seed, base + 52, cfg.head_dim, 0.0, norm_std, gen=gen)
            L.vec["k_norm"] = synth_normal(seed, base + 53, cfg.head_dim, 0.0, norm_std, gen=gen)
        else:
            nv = cfg.linear_num_value_heads
            L.vec["conv1d_weight"] = synth_normal(seed, base + 54, cfg.qkv_dim * cfg.linear_conv_kernel_dim, 0.0, 0.5,
                                                  gen=gen)
            L.vec["a_log"] = synth_normal(seed, base + 55, nv, 0.0, 0.5, gen=gen)
            L.vec["dt_bias"] = synth_normal(seed, base + 56, nv, 0.0, 0.5, gen=gen)
            L.vec["norm_weight"] = synth_normal(seed, base + 57, cfg.linear_value_head_dim, 1.0, norm_std, gen=gen)
        layers.append(L)
    embed = synth_normal_bf16(seed, 7, cfg.vocab_size * H, 0.0, embed_std, gen=gen)
    final_norm = synth_normal(seed, 8, H, 0.0, norm_std, gen=gen)
    return Qwen35Weights(cfg, layers, embed, final_norm)


def greedy(logits):
    """The last index of the largest logit (sample_token at temperature 0,
    src/transformer4.rs:3084-3091, up to logits whose probabilities round
    equal without being equal)."""
    l = np.asarray(logits)
    return int(len(l) - 1 - np.argmax(l[::-1]))


class CudaQwen35Decoder:
    """Qwen 3.5 decode on one GPU (rt_qwen35_create / rt_qwen35_step), the
    counterpart of MetalDecodeContextQwen35: step(token, position) runs one
    token through every layer and returns its logits."""

    def __init__(self, weights: Qwen35Weights, max_tokens, ctx: Context = None):
        cfg = weights.cfg
        self.cfg = cfg
        self.ctx = ctx or Context(0)
        self.max_tokens = max_tokens
        staged, keep = [], []
        layers = (RtQwen35Layer * cfg.num_hidden_layers)()
        self.embed = None
        self.h = None
        try:
            for i, L in enumerate(weights.layers):
                for name, (r, c) in _proj_shapes(cfg, L.full).items():
                    w = DeviceWeight.upload(self.ctx, RT_FMT_Q4K, L.proj[name], r, c)
                    staged.append(w)
                    setattr(layers[i], name, w.h.value)
                for name, v in L.vec.items():
                    a = np.ascontiguousarray(v, dtype=np.float32)
                    keep.append(a)
                    setattr(layers[i], name, a.ctypes.data)
            self.embed = DeviceWeight.upload(self.ctx, RT_FMT_BF16, weights.embed, cfg.vocab_size, cfg.hidden_size)
            fnorm = np.ascontiguousarray(weights.final_norm, dtype=np.float32)
            c = cfg.to_c()
            h = ctypes.c_void_p()
            check(lib().rt_qwen35_create(self.ctx.h, ctypes.byref(c), layers, self.embed.h, fnorm.ctypes.data,
                                         int(max_tokens), ctypes.byref(h)), self.ctx.h)
            self.h = h
        except Exception:
            if self.embed is not None:
                self.embed.free()
            raise
        finally:
            for w in staged:
                w.free()
        self._logits = np.empty(cfg.vocab_size, dtype=np.float32)

    def reset(self):
        """A new sequence: zero the DeltaNet states and conv1d histories."""
        check(lib().rt_qwen35_reset(self.h), self.ctx.h)

    def step(self, token, position):
        """Logits of `token` at `position` (f32 [vocab]); the states advance."""
        check(lib().rt_qwen35_step(self.h, int(token), int(position), self._logits.ctypes.data), self.ctx.h)
        return self._logits.copy()

    def step_device(self, token, position):
        """The same, leaving the logits on the device (no host copy)."""
        check(lib().rt_qwen35_step(self.h, int(token), int(position), None), self.ctx.h)

    def generate(self, prompt, n):
        """Feed `prompt` token by token, then n greedy tokens (the decode loop
        of Qwen35Model::generate_cached_streaming, src/transformer_qwen35.rs:988-1168,
        at temperature 0).  Returns the generated tokens."""
        logits = None
        for p, t in enumerate(prompt):
            logits = self.step(t, p)
        out, pos = [], len(prompt)
        for _ in range(n):
            tok = greedy(logits)
            out.append(tok)
            logits = self.step(tok, pos)
            pos += 1
        return out

    def close(self):
        if self.h is not None:
            lib().rt_qwen35_destroy(self.h)
            self.h = None
        if self.embed is not None:
            self.embed.free()
            self.embed = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
