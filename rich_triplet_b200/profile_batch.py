"""Profiling driver for many-sequence decode: `--seqs` sequences of a Gemma 3
4B-width model (synthetic weights) at a chosen depth, each with a synthetic KV
cache of `--context` positions, a few warm-up steps, then the steps to profile
(each step is one replay of the engine's CUDA graph).

    python -m rich_triplet_b200.profile_batch --seqs 64 --context 4096 --warmup 3 --steps 1
    python -m rich_triplet_b200.profile_batch --model 27b --seqs 1 --layers 62 --context 8192

`--model 27b` decodes the Gemma 3 27B shapes (config 4 on one GPU: the
tensor-parallel engine with one rank) instead of the 4B width.

Prints one line with the mean step time (CUDA events) when it is done.
"""

import argparse
import time


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--seqs", type=int, default=64)
    ap.add_argument("--layers", type=int, default=34)
    ap.add_argument("--context", type=int, default=4096, help="cached positions before the first profiled step")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--model", default="4b", choices=["4b", "27b"])
    a = ap.parse_args(argv)

    import torch

    from .decode import CudaBatchDecoder, CudaDecodeContext
    from .model import Config4, synth_gemma3
    from .ops import Context

    ctx = Context(0)
    cap = a.context + a.warmup + a.steps + 1
    if a.model == "27b":
        from .tp import TpBatchDecoder, synth_shard_weights

        cfg = Config4.gemma3_27b().with_layers(a.layers)
        dec = CudaDecodeContext(synth_shard_weights(cfg, a.seed, 1, 0), 16, ctx)
        bat = TpBatchDecoder(dec, a.seqs, cap, 1, 0)
    else:
        cfg = Config4.gemma3_4b(vocab_size=262144).with_layers(a.layers)
        dec = CudaDecodeContext(synth_gemma3(cfg, seed=a.seed), 16, ctx)
        bat = CudaBatchDecoder(dec, a.seqs, cap)
    bat.synth_kv(a.seed, a.context)
    bat.generate(a.warmup)
    ext = torch.cuda.ExternalStream(ctx.stream_ptr)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    bat.generate(a.steps, wait=False)
    e1.record(ext)
    e1.synchronize()
    ctx.sync()
    print(f"profile_batch: model={a.model} seqs={a.seqs} layers={a.layers} context={a.context} steps={a.steps} "
          f"ms_per_step={e0.elapsed_time(e1) / a.steps:.4f} at {time.strftime('%H:%M:%S')}", flush=True)
    bat.close()
    dec.close()
    ctx.close()


if __name__ == "__main__":
    main()
