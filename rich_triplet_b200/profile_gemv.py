"""Profiling driver for the standalone Q4_K GEMV: uploads
16 copies of a synthetic Q4_K weight, then either runs a few plain launches
(for an ncu capture) or the CUDA-graph benchmark of bench.py.

    python -m rich_triplet_b200.profile_gemv --rows 10240 --cols 2560 --launches 3
    python -m rich_triplet_b200.profile_gemv --rows 10240 --cols 2560 --graph

Not imported by the package; a tool for measuring the GEMV kernel.
"""

import argparse


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--rows", type=int, default=10240)
    ap.add_argument("--cols", type=int, default=2560)
    ap.add_argument("--launches", type=int, default=3, help="plain launches (rotating weight copies)")
    ap.add_argument("--graph", action="store_true", help="run the 256-launch graph benchmark instead")
    ap.add_argument("--seed", type=int, default=1234)
    a = ap.parse_args(argv)

    import torch

    from ._lib import RT_FMT_Q4K
    from .model import synth_normal, synth_q4k
    from .ops import Context, DeviceWeight, gemv_bench, gemv_device

    ctx = Context(0)
    copies = [DeviceWeight.upload(ctx, RT_FMT_Q4K, synth_q4k(a.seed, 9000 + c, a.rows, a.cols), a.rows, a.cols)
              for c in range(16)]
    x = torch.from_numpy(synth_normal(a.seed, 9100, a.cols)).cuda()
    y = torch.empty(a.rows, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    if a.graph:
        us = gemv_bench(ctx, copies, x.data_ptr(), y.data_ptr(), launches=256, ctas_per_sm=1, reps=3)
        b = a.rows * a.cols // 256 * 144 + 4 * (a.rows + a.cols)
        print(f"profile_gemv: {a.rows}x{a.cols} {us:.2f} us per GEMV, {b / us / 1e3:.0f} GB/s", flush=True)
    else:
        for i in range(a.launches):
            gemv_device(ctx, copies[(5 * i) % 16], x.data_ptr(), y.data_ptr())
        ctx.sync()
        print(f"profile_gemv: {a.launches} launches of {a.rows}x{a.cols}", flush=True)
    for c in copies:
        c.free()
    ctx.close()


if __name__ == "__main__":
    main()
