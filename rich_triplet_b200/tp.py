"""Tensor-parallel Gemma 3 decode: one process per GPU,
each holding 1/N of the model.

Sharding (the reference has no multi-GPU path; this follows the standard
Megatron split the north star names):
  q, k, v   rows by heads: rank r has query heads [r NQ/N, (r+1) NQ/N) and KV
            heads [r NKV/N, (r+1) NKV/N) (the GQA groups stay whole);
  o         columns by the same query heads;
  gate, up  rows by FFN index, in whole 256-column Q4_K super-blocks
            (rank r: super-blocks [r S/N, (r+1) S/N) of the S = FFN/256);
  down      columns by the same FFN index;
  norms, embedding (and so the tied LM head's weights) replicated.
A rank's shard is a Gemma 3 model of its own (NQ/N and NKV/N heads, its FFN
width), so the single-GPU engine builds it; rt_tp_create adds the NCCL
all-reduce of the o and down outputs and splits the LM head by vocab rows.
"""

import ctypes
from dataclasses import replace

import numpy as np

from ._lib import check, lib
from .decode import CudaBatchDecoder, CudaDecodeContext
from .model import Config4, Gemma3LayerWeights, Gemma3Weights, synth_normal, synth_normal_bf16

def shard_ranges(cfg: Config4, nranks, rank):
    """(q head range, KV head range, FFN column range) of `rank`."""
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    if nq % nranks or nkv % nranks:
        raise ValueError(f"tensor parallel: {nq} query / {nkv} KV heads do not split over {nranks} ranks")
    if cfg.intermediate_size % 256:
        raise ValueError("tensor parallel: FFN width must be a multiple of 256")
    nsb = cfg.intermediate_size // 256
    if nsb < nranks:
        raise ValueError(f"tensor parallel: {nsb} FFN super-blocks for {nranks} ranks")
    s0, s1 = nsb * rank // nranks, nsb * (rank + 1) // nranks
    return ((nq * rank // nranks, nq * (rank + 1) // nranks), (nkv * rank // nranks, nkv * (rank + 1) // nranks),
            (256 * s0, 256 * s1))


def shard_config(cfg: Config4, nranks, rank):
    (q0, q1), (k0, k1), (f0, f1) = shard_ranges(cfg, nranks, rank)
    return replace(cfg, num_attention_heads=q1 - q0, num_key_value_heads=k1 - k0, intermediate_size=f1 - f0)


def _rows(blocks, cols, r0, r1):
    per = cols // 256 * 144
    return np.ascontiguousarray(blocks[r0 * per:r1 * per])


def _cols(blocks, rows, cols, c0, c1):
    b = blocks.reshape(rows, cols // 256, 144)
    return np.ascontiguousarray(b[:, c0 // 256:c1 // 256]).reshape(-1)


def shard_weights(w: Gemma3Weights, nranks, rank):
    """Rank `rank`'s shard of host weights `w` (a copy of the slices)."""
    cfg = w.cfg
    D, H, F = cfg.head_dim, cfg.hidden_size, cfg.intermediate_size
    (q0, q1), (k0, k1), (f0, f1) = shard_ranges(cfg, nranks, rank)
    out = Gemma3Weights(shard_config(cfg, nranks, rank))
    for L in w.layers:
        out.layers.append(Gemma3LayerWeights(
            q=_rows(L.q, H, q0 * D, q1 * D), k=_rows(L.k, H, k0 * D, k1 * D), v=_rows(L.v, H, k0 * D, k1 * D),
            o=_cols(L.o, H, cfg.num_attention_heads * D, q0 * D, q1 * D),
            gate=_rows(L.gate, H, f0, f1), up=_rows(L.up, H, f0, f1), down=_cols(L.down, H, F, f0, f1),
            attn_norm=L.attn_norm, post_attn_norm=L.post_attn_norm, pre_ffn_norm=L.pre_ffn_norm,
            post_ffn_norm=L.post_ffn_norm, q_norm=L.q_norm, k_norm=L.k_norm))
    out.embed = w.embed
    out.final_norm = w.final_norm
    return out


def _synth_slice(seed, stream, rows, cols, r0, r1, c0, c1):
    out = np.empty((r1 - r0) * ((c1 - c0) // 256) * 144, dtype=np.uint8)
    lib().rt_synth_q4k_slice(seed, stream, rows, cols, r0, r1 - r0, c0, c1 - c0, out.ctypes.data)
    return out


class _LazyLayers:
    """The shard's layers, made one at a time as they are read (host memory
    holds one layer of the shard)."""

    def __init__(self, cfg, seed, nranks, rank, norm_std):
        self.cfg, self.seed, self.nranks, self.rank, self.norm_std = cfg, seed, nranks, rank, norm_std

    def __len__(self):
        return self.cfg.num_hidden_layers

    def __iter__(self):
        cfg, seed = self.cfg, self.seed
        D, H, F = cfg.head_dim, cfg.hidden_size, cfg.intermediate_size
        nq, nkv = cfg.num_attention_heads * D, cfg.num_key_value_heads * D
        (q0, q1), (k0, k1), (f0, f1) = shard_ranges(cfg, self.nranks, self.rank)
        sd = self.norm_std
        for i in range(cfg.num_hidden_layers):
            s = 1000 + 32 * i
            yield Gemma3LayerWeights(
                q=_synth_slice(seed, s + 0, nq, H, q0 * D, q1 * D, 0, H),
                k=_synth_slice(seed, s + 1, nkv, H, k0 * D, k1 * D, 0, H),
                v=_synth_slice(seed, s + 2, nkv, H, k0 * D, k1 * D, 0, H),
                o=_synth_slice(seed, s + 3, H, nq, 0, H, q0 * D, q1 * D),
                gate=_synth_slice(seed, s + 4, F, H, f0, f1, 0, H),
                up=_synth_slice(seed, s + 5, F, H, f0, f1, 0, H),
                down=_synth_slice(seed, s + 6, H, F, 0, H, f0, f1),
                attn_norm=synth_normal(seed, s + 7, H, 0.0, sd), post_attn_norm=synth_normal(seed, s + 8, H, 0.0, sd),
                pre_ffn_norm=synth_normal(seed, s + 9, H, 0.0, sd), post_ffn_norm=synth_normal(seed, s + 10, H, 0.0, sd),
                q_norm=synth_normal(seed, s + 11, D, 0.0, sd), k_norm=synth_normal(seed, s + 12, D, 0.0, sd))


def synth_shard_weights(cfg: Config4, seed, nranks, rank, norm_std=0.1, embed_std=0.02):
    """Rank `rank`'s shard of synth_gemma3(cfg, seed) made directly (the same
    bytes as shard_weights(synth_gemma3(cfg, seed), nranks, rank)), layers
    made lazily."""
    out = Gemma3Weights(shard_config(cfg, nranks, rank))
    out.layers = _LazyLayers(cfg, seed, nranks, rank, norm_std)
    out.embed = synth_normal_bf16(seed, 7, cfg.vocab_size * cfg.hidden_size, 0.0, embed_std)
    out.final_norm = synth_normal(seed, 8, cfg.hidden_size, 0.0, norm_std)
    return out


def nccl_unique_id():
    """128 bytes naming a new NCCL communicator (make on one rank, share)."""
    buf = ctypes.create_string_buffer(128)
    check(lib().rt_nccl_unique_id(buf))
    return buf.raw


class TpBatchDecoder(CudaBatchDecoder):
    """This rank's part of a tensor-parallel many-sequence decoder: `dec` is
    the CudaDecodeContext of the rank's shard; every rank creates its part
    together with the same `nccl_id` and then calls set / step / generate in
    step.  step() returns this rank's logits columns (vocab rows
    [vocab_lo, vocab_lo + vocab)) and every rank the same greedy tokens."""

    def __init__(self, dec: CudaDecodeContext, nseq, cap, nranks, rank, nccl_id=None):
        self.dec = dec
        self.ctx = dec.ctx
        self.nseq = nseq
        self.cap = cap
        h = ctypes.c_void_p()
        idbuf = ctypes.create_string_buffer(bytes(nccl_id), 128) if nccl_id is not None else None
        check(lib().rt_tp_create(dec.h, idbuf, nranks, rank, nseq, cap, ctypes.byref(h)), self.ctx.h)
        self.h = h
        v0, vr = ctypes.c_int32(), ctypes.c_int32()
        check(lib().rt_batch_vocab_slice(self.h, ctypes.byref(v0), ctypes.byref(vr)), self.ctx.h)
        self.vocab_lo, self.vocab = v0.value, vr.value

    def peer_handle(self):
        """64 bytes: the CUDA IPC handle of this rank's peer all-reduce buffer."""
        buf = ctypes.create_string_buffer(64)
        check(lib().rt_tp_peer_handle(self.h, buf), self.ctx.h)
        return buf.raw

    def peer_open(self, handles):
        """Map every rank's buffer (`handles` in rank order) and switch the
        per-layer sums from NCCL to the peer all-reduce kernel."""
        blob = b"".join(bytes(h) for h in handles)
        check(lib().rt_tp_peer_open(self.h, ctypes.create_string_buffer(blob, len(blob))), self.ctx.h)

    def enable_peer_allreduce(self, dist):
        """peer_handle on every rank, an all-gather of the handles over the
        torch.distributed group `dist` (any backend), then peer_open."""
        handles = [None] * dist.get_world_size()
        dist.all_gather_object(handles, self.peer_handle())
        self.peer_open(handles)


def share_nccl_id(dist, rank, make=nccl_unique_id):
    """The NCCL id made on rank 0, on every rank of the torch.distributed
    process group (any backend)."""
    box = [make() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return box[0]
