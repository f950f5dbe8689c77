"""Tensor-parallel many-sequence decode (rt_tp_create) against the
single-GPU engine on the same weights.

With one rank the engine is the many-sequence engine itself (bit-identical
logits).  With two ranks (two GPUs; skipped on a one-GPU machine) each rank
holds half of the heads and FFN columns; the o / down outputs are summed by
NCCL all-reduces and the greedy token comes from an all-gather.  The same
engine with the peer all-reduce (rt_tp_peer_open: NVLink stores into every
rank's buffer) must give the NCCL run's logits bit for bit: with two ranks
every element is one addition of the same two values.  Tolerance
REL_L2 (2e-3, the north star's bar for logits): the shards' GEMM operands are
rounded to fp16 with row scales taken over each rank's columns, so the sums
differ from the single-GPU ones at that rounding (about 3e-4).
"""

import os

import numpy as np
import pytest

from rich_triplet_b200.model import Config4, synth_gemma3, synth_tokens

pytestmark = pytest.mark.gpu

# 4 query / 2 KV heads of 128, FFN of 3 super-blocks (1 + 2 over two ranks),
# 6 layers (layer 5 global), window 8
CFG = Config4(512, 256, 6, 4, 2, 768, 128, 8, 10_000.0, 1_000_000.0, 1.0, 0.125, 1e-6, 128.0)
REL_L2 = 2e-3
NSEQ, STEPS, CAP = 3, 14, 64


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / (np.linalg.norm(b.astype(np.float64)) + 1e-30))


def _inputs():
    return [synth_tokens(70 + b, 1, STEPS, CFG.vocab_size) for b in range(NSEQ)]


def _run(bat, prompts):
    """Per step: the engine's logits and greedy tokens for the prompts' tokens."""
    logits, toks = [], []
    for t in range(STEPS):
        bat.set([int(p[t]) for p in prompts], [t] * NSEQ)
        lb, nb = bat.step()
        logits.append(lb.copy())
        toks.append(nb.copy())
    return logits, toks


def test_tp1_is_the_batch_engine():
    from rich_triplet_b200.decode import CudaBatchDecoder, CudaDecodeContext
    from rich_triplet_b200.ops import Context
    from rich_triplet_b200.tp import TpBatchDecoder

    w = synth_gemma3(CFG, seed=77)
    ctx = Context(0)
    dec = CudaDecodeContext(w, 16, ctx)
    try:
        a = CudaBatchDecoder(dec, NSEQ, CAP)
        la, ta = _run(a, _inputs())
        a.close()
        b = TpBatchDecoder(dec, NSEQ, CAP, 1, 0)
        assert (b.vocab_lo, b.vocab) == (0, CFG.vocab_size)
        lb, tb = _run(b, _inputs())
        b.close()
        for x, y in zip(la, lb):
            assert np.array_equal(x, y)
        for x, y in zip(ta, tb):
            assert np.array_equal(x, y)
    finally:
        dec.close()
        ctx.close()


def _tp_worker(rank, world, port, out):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank)
        from rich_triplet_b200.decode import CudaDecodeContext
        from rich_triplet_b200.ops import Context
        from rich_triplet_b200.tp import TpBatchDecoder, share_nccl_id, synth_shard_weights

        nccl_id = share_nccl_id(dist, rank)
        ctx = Context(rank)
        dec = CudaDecodeContext(synth_shard_weights(CFG, 77, world, rank), 16, ctx)
        bat = TpBatchDecoder(dec, NSEQ, CAP, world, rank, nccl_id)
        logits, toks = _run(bat, _inputs())
        v0 = bat.vocab_lo
        bat.close()
        peer = TpBatchDecoder(dec, NSEQ, CAP, world, rank, share_nccl_id(dist, rank))
        peer.enable_peer_allreduce(dist)
        dist.barrier()
        plog, ptok = _run(peer, _inputs())
        dist.barrier()  # no rank frees its buffer while a peer may still store into it
        peer.close()
        np.savez(os.path.join(out, f"rank{rank}.npz"), v0=v0, logits=np.stack(logits), toks=np.stack(toks),
                 peer_logits=np.stack(plog), peer_toks=np.stack(ptok))
        dec.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_tp2_matches_single_gpu(tmp_path):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    port = 29600 + os.getpid() % 1000
    mp.spawn(_tp_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(2)]
    assert np.array_equal(parts[0]["toks"], parts[1]["toks"])
    for p in parts:
        assert np.array_equal(p["peer_logits"], p["logits"])
        assert np.array_equal(p["peer_toks"], p["toks"])
    tp_logits = np.concatenate([p["logits"] for p in parts], axis=2)
    assert int(parts[1]["v0"]) == parts[0]["logits"].shape[2]

    from rich_triplet_b200.decode import CudaBatchDecoder, CudaDecodeContext
    from rich_triplet_b200.ops import Context

    ctx = Context(0)
    dec = CudaDecodeContext(synth_gemma3(CFG, seed=77), 16, ctx)
    try:
        bat = CudaBatchDecoder(dec, NSEQ, CAP)
        ref, ref_toks = _run(bat, _inputs())
        bat.close()
    finally:
        dec.close()
        ctx.close()
    worst = max(rel_l2(tp_logits[t, b], ref[t][b]) for t in range(STEPS) for b in range(NSEQ))
    assert worst < REL_L2, worst
    agree = np.mean([int(parts[0]["toks"][t][b]) == int(ref_toks[t][b]) for t in range(STEPS) for b in range(NSEQ)])
    assert agree == 1.0, agree
