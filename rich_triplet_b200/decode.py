"""CudaDecodeContext: the CUDA counterpart of the reference's MetalDecodeContext.

    MetalDecodeContext::new(model, draft_len)   src/metal_decode.rs:971
    sync_kv_from_cpu(&cache)                    src/metal_decode.rs:1366
    decode_step(token_id, position) -> logits   src/metal_decode.rs:2028
    print_metal_memory()                        src/metal_decode.rs:1285
    lm_head_vocab                               src/metal_decode.rs:826

The engine lives in librtcuda.so (rt_decoder_*): weights, an f32 KV cache and
one captured CUDA graph per decode step.  This class only marshals host
buffers across the C ABI.
"""

import ctypes

import numpy as np

from ._lib import RT_DEVICE, RT_FMT_BF16, RT_FMT_Q4K, RT_HOST, RtGemma3Cfg, RtGemma3Layer, check, lib
from .model import Config4, Gemma3Weights
from .ops import Context, DeviceWeight

_PROJ = ("q", "k", "v", "o", "gate", "up", "down")
_NORMS = ("attn_norm", "post_attn_norm", "pre_ffn_norm", "post_ffn_norm", "q_norm", "k_norm")


def cfg_to_c(cfg: Config4):
    return RtGemma3Cfg(cfg.vocab_size, cfg.hidden_size, cfg.num_hidden_layers, cfg.num_attention_heads,
                       cfg.num_key_value_heads, cfg.head_dim, cfg.intermediate_size, cfg.sliding_window or 0,
                       cfg.rope_theta_local, cfg.rope_theta_global, cfg.rope_freq_scale_local,
                       cfg.rope_freq_scale_global, cfg.rms_norm_eps, cfg.query_pre_attn_scalar)


class CudaDecodeContext:
    """Gemma 3 decode on one GPU; one decode step is one CUDA graph launch."""

    def __init__(self, weights: Gemma3Weights, max_ctx, ctx: Context = None):
        cfg = weights.cfg
        self.cfg = cfg
        self.ctx = ctx or Context(0)
        self.max_ctx = max_ctx
        H, D, F = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
        q, kv = cfg.num_attention_heads * D, cfg.num_key_value_heads * D
        shapes = {"q": (q, H), "k": (kv, H), "v": (kv, H), "o": (H, q), "gate": (F, H), "up": (F, H), "down": (H, F)}
        staged = []  # device copies that only live until the engine has fused them
        layers = (RtGemma3Layer * cfg.num_hidden_layers)()
        keep = []
        try:
            for i, L in enumerate(weights.layers):
                for n in _PROJ:
                    r, c = shapes[n]
                    src = getattr(L, n)
                    # host Q4_K bytes, or a device weight (a GGUF load) that the engine copies and frees
                    w = src if isinstance(src, DeviceWeight) else DeviceWeight.upload(self.ctx, RT_FMT_Q4K, src, r, c)
                    staged.append(w)
                    setattr(layers[i], n, w.h.value)
                for n in _NORMS:
                    a = np.ascontiguousarray(getattr(L, n), dtype=np.float32)
                    keep.append(a)
                    setattr(layers[i], n, a.ctypes.data)
            emb = weights.embed if isinstance(weights.embed, DeviceWeight) else \
                DeviceWeight.upload(self.ctx, RT_FMT_BF16, weights.embed, cfg.vocab_size, H)
            staged.append(emb)
            fnorm = np.ascontiguousarray(weights.final_norm, dtype=np.float32)
            c = cfg_to_c(cfg)
            h = ctypes.c_void_p()
            check(lib().rt_decoder_create(self.ctx.h, ctypes.byref(c), layers, emb.h, fnorm.ctypes.data, max_ctx,
                                          ctypes.byref(h)), self.ctx.h)
            self.h = h
        finally:
            for w in staged:
                w.free()
        self.lm_head_vocab = cfg.vocab_size
        self._logits = np.empty(self.lm_head_vocab, dtype=np.float32)

    # --- MetalDecodeContext surface -------------------------------------
    def sync_kv_from_cpu(self, k_layers, v_layers, seq_len):
        """Load a CPU-prefilled f32 KV cache ([seq_len, nkv*D] per layer)."""
        for i, (k, v) in enumerate(zip(k_layers, v_layers)):
            k = np.ascontiguousarray(k, dtype=np.float32)
            v = np.ascontiguousarray(v, dtype=np.float32)
            check(lib().rt_decoder_load_kv(self.h, i, k.ctypes.data, v.ctypes.data, seq_len), self.ctx.h)

    def decode_step(self, token_id, position, out=None):
        """Logits (f32, lm_head_vocab) of `token_id` at absolute `position`."""
        logits = out if out is not None else np.empty(self.lm_head_vocab, dtype=np.float32)
        check(lib().rt_decoder_step(self.h, int(token_id), int(position), logits.ctypes.data), self.ctx.h)
        return logits

    def print_memory(self):
        b = ctypes.c_uint64()
        check(lib().rt_decoder_memory(self.h, ctypes.byref(b)), self.ctx.h)
        print(f"[ CUDA ] decode engine holds {b.value / 2**30:.2f} GiB of device memory")
        return b.value

    # --- extensions -------------------------------------------------------
    def prefill(self, tokens, start_pos=0, want_logits=True):
        """Run prompt tokens one position at a time (device-side); returns the
        last token's logits."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty(self.lm_head_vocab, dtype=np.float32) if want_logits else None
        check(lib().rt_decoder_prefill(self.h, t.ctypes.data, t.size, start_pos,
                                       logits.ctypes.data if want_logits else None), self.ctx.h)
        return logits

    def prefill_gemm(self, tokens, start_pos=0, want_logits=True):
        """Prompt tokens through the engine all positions at once (tensor-core
        GEMMs over the tokens, causal attention); returns the last token's
        logits."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty(self.lm_head_vocab, dtype=np.float32) if want_logits else None
        check(lib().rt_decoder_prefill_gemm(self.h, t.ctypes.data, t.size, start_pos,
                                            logits.ctypes.data if want_logits else None), self.ctx.h)
        return logits

    def decode_step_batch(self, token_ids, start_position):
        """Logits [m, vocab] of m consecutive positions in one pass
        (MetalDecodeContext::decode_step_batch, src/metal_decode.rs:2079)."""
        t = np.ascontiguousarray(token_ids, dtype=np.int32)
        logits = np.empty((t.size, self.lm_head_vocab), dtype=np.float32)
        check(lib().rt_decoder_step_batch(self.h, t.ctypes.data, t.size, start_position, logits.ctypes.data),
              self.ctx.h)
        return logits

    def generate(self, first_token, start_pos, n):
        """Greedy decode on the device; returns the n argmax tokens."""
        toks = np.empty(n, dtype=np.int32)
        check(lib().rt_decoder_generate(self.h, int(first_token), int(start_pos), n, toks.ctypes.data, RT_HOST),
              self.ctx.h)
        return toks

    def enqueue_generate(self, first_token, start_pos, n):
        """Enqueue n greedy steps on the context stream without waiting."""
        check(lib().rt_decoder_generate(self.h, int(first_token), int(start_pos), n, None, RT_DEVICE), self.ctx.h)

    def enqueue_q4k_gemvs(self):
        n = ctypes.c_int32()
        b = ctypes.c_uint64()
        check(lib().rt_decoder_enqueue_q4k_gemvs(self.h, ctypes.byref(n), ctypes.byref(b)), self.ctx.h)
        return n.value, b.value

    def read_kv(self, layer, seq_len):
        n = seq_len * self.cfg.num_key_value_heads * self.cfg.head_dim
        k = np.empty(n, dtype=np.float32)
        v = np.empty(n, dtype=np.float32)
        check(lib().rt_decoder_read_kv(self.h, layer, k.ctypes.data, v.ctypes.data, seq_len), self.ctx.h)
        return k, v

    def final_hidden(self):
        out = np.empty(self.cfg.hidden_size, dtype=np.float32)
        check(lib().rt_decoder_read_activation(self.h, 0, out.ctypes.data, out.size), self.ctx.h)
        return out

    @property
    def launches_per_step(self):
        n = ctypes.c_int32()
        check(lib().rt_decoder_launches_per_step(self.h, ctypes.byref(n)), self.ctx.h)
        return n.value

    def close(self):
        if getattr(self, "h", None):
            lib().rt_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaBatchDecoder:
    """Many-sequence decode on the weights of a
    CudaDecodeContext: `nseq` independent sequences, each with its own f32 KV
    cache of `cap` positions, advance together; every projection is one
    tensor-core GEMM over the sequences (fp16 operands, f32 accumulation).
    The reference decodes one sequence at a time; this has no counterpart
    there (its decode_step_batch, src/metal_decode.rs:2079, batches positions
    of one sequence)."""

    def __init__(self, dec: CudaDecodeContext, nseq, cap):
        self.dec = dec
        self.ctx = dec.ctx
        self.nseq = nseq
        self.cap = cap
        self.vocab = dec.lm_head_vocab
        h = ctypes.c_void_p()
        check(lib().rt_batch_create(dec.h, nseq, cap, ctypes.byref(h)), self.ctx.h)
        self.h = h

    def set(self, tokens, positions):
        """Each sequence's next input token and its position (arrays of nseq)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        if t.shape != (self.nseq,) or p.shape != (self.nseq,):
            raise ValueError(f"CudaBatchDecoder.set: need {self.nseq} tokens and positions")
        check(lib().rt_batch_set(self.h, t.ctypes.data, p.ctypes.data), self.ctx.h)

    def step(self, want_logits=True):
        """One step for every sequence; returns (logits [nseq, vocab] or None,
        greedy next tokens [nseq]).  Positions advance by one."""
        logits = np.empty((self.nseq, self.vocab), dtype=np.float32) if want_logits else None
        nxt = np.empty(self.nseq, dtype=np.int32)
        check(lib().rt_batch_step(self.h, logits.ctypes.data if want_logits else None, nxt.ctypes.data), self.ctx.h)
        return logits, nxt

    def generate(self, steps, wait=True):
        """`steps` greedy steps from the current tokens and positions."""
        check(lib().rt_batch_generate(self.h, steps, RT_HOST if wait else RT_DEVICE), self.ctx.h)

    def synth_kv(self, seed, seq_len):
        """Synthetic cache contents for benchmarks; every position = seq_len."""
        check(lib().rt_batch_synth_kv(self.h, seed, seq_len), self.ctx.h)

    def info(self):
        b = ctypes.c_uint64()
        n = ctypes.c_int32()
        check(lib().rt_batch_info(self.h, ctypes.byref(b), ctypes.byref(n)), self.ctx.h)
        return b.value, n.value

    def close(self):
        if getattr(self, "h", None):
            lib().rt_batch_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
