"""Profiling driver for the Q4_K prefill GEMM: one shape, a few warm-up
launches, then the launches to profile (device pointers, bf16 A ~ N(0,1)).

    python -m rich_triplet_b200.profile_gemm --m 2048 --k 2560 --n 20480 --warmup 2 --launches 1

Prints the mean device time per GEMM when it is done.
"""

import argparse

import numpy as np


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--m", type=int, default=2048)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--n", type=int, default=20480)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--launches", type=int, default=1)
    ap.add_argument("--seed", type=int, default=1234)
    a = ap.parse_args(argv)

    import torch

    from ._lib import RT_FMT_Q4K
    from .model import synth_normal_bf16, synth_q4k
    from .ops import Context, DeviceWeight, gemm_device

    ctx = Context(0)
    w = DeviceWeight.upload(ctx, RT_FMT_Q4K, synth_q4k(a.seed, a.n + a.k, a.n, a.k), a.n, a.k)
    x = torch.from_numpy(synth_normal_bf16(a.seed, a.m, a.m * a.k).view(np.int16)).cuda()
    c = torch.empty((a.m, a.n), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for _ in range(a.warmup):
        gemm_device(ctx, w, x.data_ptr(), a.m, c.data_ptr())
    ctx.sync()
    ext = torch.cuda.ExternalStream(ctx.stream_ptr)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for _ in range(a.launches):
        gemm_device(ctx, w, x.data_ptr(), a.m, c.data_ptr())
    e1.record(ext)
    e1.synchronize()
    ctx.sync()
    us = e0.elapsed_time(e1) * 1e3 / a.launches
    print(f"profile_gemm: M={a.m} K={a.k} N={a.n} us_per_gemm={us:.1f} "
          f"tflops={2.0 * a.m * a.n * a.k / us / 1e6:.1f}", flush=True)
    w.free()
    ctx.close()


if __name__ == "__main__":
    main()
