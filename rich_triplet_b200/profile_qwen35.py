"""Profiling driver for the Qwen 3.5 decode engine: synthetic weights at the
4B widths (or `--layers` of them), `--warmup` steps, then `--steps` steps to
profile (each one CUDA graph launch).

    python -m rich_triplet_b200.profile_qwen35 --layers 8 --warmup 3 --steps 1

Prints one line with the mean step time when it is done.
"""

import argparse
import time


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--seed", type=int, default=1234)
    a = ap.parse_args(argv)

    from .qwen35 import CudaQwen35Decoder, Qwen35Config, synth_qwen35

    cfg = Qwen35Config.qwen35_4b().with_layers(a.layers)
    dec = CudaQwen35Decoder(synth_qwen35(cfg, seed=a.seed), a.warmup + a.steps + 1)
    for p in range(a.warmup):
        dec.step_device(p + 1, p)
    t = time.perf_counter()
    for p in range(a.warmup, a.warmup + a.steps):
        dec.step_device(p + 1, p)
    ms = (time.perf_counter() - t) * 1e3 / a.steps
    print(f"profile_qwen35: layers={a.layers} steps={a.steps} ms_per_step={ms:.4f}", flush=True)
    dec.close()
    dec.ctx.close()


if __name__ == "__main__":
    main()
