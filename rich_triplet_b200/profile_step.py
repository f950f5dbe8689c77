"""Profiling driver for the decode step: a Gemma 3 4B-width model (synthetic
weights) at a chosen depth, a synthetic KV cache loaded straight into the
engine at the chosen context (no prefill, so a profiler sees only a few step
launches before the one it captures), a few warm-up steps, then the steps to
profile.

    python -m rich_triplet_b200.profile_step --layers 6 --context 512 --warmup 3 --steps 1

Prints one line with the mean step time (CUDA events) when it is done.
"""

import argparse
import time

import numpy as np


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--layers", type=int, default=6)
    ap.add_argument("--context", type=int, default=512, help="cached positions before the first profiled step")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--seed", type=int, default=1234)
    a = ap.parse_args(argv)

    import torch

    from .decode import CudaDecodeContext
    from .model import Config4, synth_gemma3
    from .ops import Context

    cfg = Config4.gemma3_4b(vocab_size=262144).with_layers(a.layers)
    w = synth_gemma3(cfg, seed=a.seed)
    ctx = Context(0)
    dec = CudaDecodeContext(w, a.context + a.warmup + a.steps + 1, ctx)
    rng = np.random.default_rng(a.seed)
    n = a.context * cfg.num_key_value_heads * cfg.head_dim
    kv = [rng.standard_normal(n, dtype=np.float32) for _ in range(2)]
    dec.sync_kv_from_cpu([kv[0]] * cfg.num_hidden_layers, [kv[1]] * cfg.num_hidden_layers, a.context)
    tok = 1
    pos = a.context
    for _ in range(a.warmup):
        tok = int(np.argmax(dec.decode_step(tok, pos)))
        pos += 1
    ctx.sync()
    ext = torch.cuda.ExternalStream(ctx.stream_ptr)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    dec.enqueue_generate(tok, pos, a.steps)
    e1.record(ext)
    e1.synchronize()
    ctx.sync()
    print(f"profile_step: layers={a.layers} context={a.context} steps={a.steps} "
          f"ms_per_step={e0.elapsed_time(e1) / a.steps:.4f} at {time.strftime('%H:%M:%S')}", flush=True)
    dec.close()
    ctx.close()


if __name__ == "__main__":
    main()
