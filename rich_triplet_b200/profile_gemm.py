"""Profiling driver for the Q4_K prefill GEMM: one shape, a few warm-up
launches, then the launches to profile (device pointers, bf16 A ~ N(0,1)).

    python -m rich_triplet_b200.profile_gemm --m 2048 --k 2560 --n 20480 --warmup 2 --launches 1

Prints the mean device time per GEMM when it is done.  --copies C uploads C
copies of the weights and rotates over them, so that with C x the weight
bytes above the L2 (126 MB) every launch streams its weights from HBM.  The
library's RT_GEMM_SPLITS (split-K count) and RT_GEMM_TILE (128 / 256) force
the plan, for sweeps.
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
    ap.add_argument("--copies", type=int, default=1, help="weight copies to rotate over")
    a = ap.parse_args(argv)

    import torch

    from ._lib import RT_FMT_Q4K
    from .model import synth_normal_bf16, synth_q4k
    from .ops import Context, DeviceWeight, gemm_device

    ctx = Context(0)
    host = synth_q4k(a.seed, a.n + a.k, a.n, a.k)
    ws = [DeviceWeight.upload(ctx, RT_FMT_Q4K, host, a.n, a.k) for _ in range(max(1, a.copies))]
    x = torch.from_numpy(synth_normal_bf16(a.seed, a.m, a.m * a.k).view(np.int16)).cuda()
    c = torch.empty((a.m, a.n), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for i in range(a.warmup):
        gemm_device(ctx, ws[i % len(ws)], x.data_ptr(), a.m, c.data_ptr())
    ctx.sync()
    ext = torch.cuda.ExternalStream(ctx.stream_ptr)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for i in range(a.launches):
        gemm_device(ctx, ws[i % len(ws)], x.data_ptr(), a.m, c.data_ptr())
    e1.record(ext)
    e1.synchronize()
    ctx.sync()
    us = e0.elapsed_time(e1) * 1e3 / a.launches
    print(f"profile_gemm: M={a.m} K={a.k} N={a.n} us_per_gemm={us:.1f} "
          f"tflops={2.0 * a.m * a.n * a.k / us / 1e6:.1f}", flush=True)
    for w in ws:
        w.free()
    ctx.close()


if __name__ == "__main__":
    main()
