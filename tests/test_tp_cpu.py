"""Tensor-parallel sharding (rich_triplet_b200.tp) on the host: shards made
directly equal slices of the whole model, the row-split projections add up
to the whole product (dequantised with the oracle), and the NCCL id reaches
every rank and the peer all-reduce handles are gathered in rank order
(gloo, two processes)."""

import os

import numpy as np
import pytest

from rich_triplet_b200.model import Config4, synth_gemma3, synth_normal
from rich_triplet_b200.tp import shard_config, shard_ranges, shard_weights, share_nccl_id, synth_shard_weights

# 4 query / 2 KV heads of 128, FFN of 3 super-blocks (split 1 + 2 over 2 ranks)
CFG = Config4(512, 256, 2, 4, 2, 768, 128, 8, 10_000.0, 1_000_000.0, 1.0, 0.125, 1e-6, 128.0)
FIELDS = ("q", "k", "v", "o", "gate", "up", "down", "attn_norm", "post_attn_norm", "pre_ffn_norm", "post_ffn_norm",
          "q_norm", "k_norm")


def test_shard_ranges_cover_once():
    for n in (1, 2):
        qs, ks, fs = zip(*(shard_ranges(CFG, n, r) for r in range(n)))
        for rng, total in ((qs, 4), (ks, 2), (fs, 768)):
            assert rng[0][0] == 0 and rng[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(rng, rng[1:]))
    assert [shard_config(CFG, 2, r).intermediate_size for r in range(2)] == [256, 512]
    with pytest.raises(ValueError):
        shard_ranges(CFG, 4, 0)  # 2 KV heads over 4 ranks


def test_synth_shard_equals_slice():
    w = synth_gemma3(CFG, seed=5)
    for n in (1, 2):
        for r in range(n):
            a, b = shard_weights(w, n, r), synth_shard_weights(CFG, 5, n, r)
            for la, lb in zip(a.layers, b.layers):
                for f in FIELDS:
                    assert np.array_equal(getattr(la, f), getattr(lb, f)), (n, r, f)
            assert np.array_equal(a.embed, b.embed) and np.array_equal(a.final_norm, b.final_norm)


def test_row_split_products_add_up(orc):
    w = synth_gemma3(CFG, seed=6)
    D, H, F = CFG.head_dim, CFG.hidden_size, CFG.intermediate_size
    L = w.layers[0]
    xo = synth_normal(7, 1, CFG.num_attention_heads * D)
    xd = synth_normal(7, 2, F)
    full_o = orc.q4k_dequantize(L.o, H, CFG.num_attention_heads * D).reshape(H, -1).astype(np.float64) @ xo
    full_d = orc.q4k_dequantize(L.down, H, F).reshape(H, F).astype(np.float64) @ xd
    so = np.zeros(H)
    sd = np.zeros(H)
    for r in range(2):
        s = shard_weights(w, 2, r)
        (q0, q1), _, (f0, f1) = shard_ranges(CFG, 2, r)
        wo = orc.q4k_dequantize(s.layers[0].o, H, (q1 - q0) * D).reshape(H, -1).astype(np.float64)
        wd = orc.q4k_dequantize(s.layers[0].down, H, f1 - f0).reshape(H, -1).astype(np.float64)
        so += wo @ xo[q0 * D:q1 * D]
        sd += wd @ xd[f0:f1]
    assert np.allclose(so, full_o, rtol=1e-12, atol=1e-9)
    assert np.allclose(sd, full_d, rtol=1e-12, atol=1e-9)


def _id_worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got = share_nccl_id(dist, rank, make=lambda: bytes(range(128)))
        with open(os.path.join(out, f"id{rank}"), "wb") as f:
            f.write(got)
    finally:
        dist.destroy_process_group()


def test_nccl_id_reaches_every_rank(tmp_path):
    import torch.multiprocessing as mp
    port = 29500 + os.getpid() % 1000
    mp.spawn(_id_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert (tmp_path / f"id{r}").read_bytes() == bytes(range(128))


class _PeerStub:
    """TpBatchDecoder's handle exchange with the C-ABI calls replaced: each
    rank's handle is 64 bytes of its rank number; peer_open records what it
    was given."""

    def __init__(self, rank):
        self.rank = rank
        self.opened = None

    def peer_handle(self):
        return bytes([self.rank]) * 64

    def peer_open(self, handles):
        self.opened = b"".join(bytes(h) for h in handles)


def _peer_worker(rank, world, port, out):
    import torch.distributed as dist

    from rich_triplet_b200.tp import TpBatchDecoder

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        stub = _PeerStub(rank)
        TpBatchDecoder.enable_peer_allreduce(stub, dist)
        with open(os.path.join(out, f"peer{rank}"), "wb") as f:
            f.write(stub.opened)
    finally:
        dist.destroy_process_group()


def test_peer_handles_reach_every_rank_in_rank_order(tmp_path):
    # rt_tp_peer_open takes every rank's 64-byte handle, rank 0 first.
    import torch.multiprocessing as mp
    port = 29700 + os.getpid() % 1000
    mp.spawn(_peer_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert (tmp_path / f"peer{r}").read_bytes() == bytes([0]) * 64 + bytes([1]) * 64
