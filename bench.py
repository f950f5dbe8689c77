#!/usr/bin/env python
"""bench.py -- Gemma 3 4B Q4_K batch-1 decode on B200.

A "step" is one decode step of the 4B model (34 layers + LM head) for one
sequence: prompt of 512 random token ids prefilled, then greedy steps at
positions 512..767.  Timed steps cycle through that 256-position span (every
span restarts at position 512 and overwrites the same cache rows), so every
timed step is a config-1 step whatever --steps is.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 runs under torchrun, one rank per GPU, each rank decoding its own
sequence with its own weight replica (sequences are independent: no
collective on the data path; the barrier and max-over-ranks timing use NCCL).
value = total tokens / max-over-ranks device time.  `--impl reference` times
the reference's CPU decode path (its restatement in oracle/, since the Rust
crate cannot be built here) on the host cores.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Gemma-3 4B Q4_K decode tok/s (bs=1) and Q4_K GEMV HBM GB/s vs 8 TB/s peak"
PROMPT = 512
SPAN = 256


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2048)
    p.add_argument("--warmup", type=int, default=16)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--layers", type=int, default=34, help="model depth (34 = Gemma 3 4B)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-config4", action="store_true", help="skip the 27B tensor-parallel section")
    p.add_argument("--no-qwen35", action="store_true", help="skip the Qwen 3.5 decode section")
    p.add_argument("--tp-allreduce", default="nccl", choices=["peer", "nccl"],
                   help="config 4's per-layer sums: peer all-reduce kernel over NVLink, or NCCL")
    p.add_argument("--cpu-steps", type=int, default=10)
    p.add_argument("--prompt", type=int, default=PROMPT,
                   help="prompt tokens prefilled before the timed steps (512 = BASELINE config 1; "
                        "shorter only for profiling)")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 8:
                    continue
                try:
                    rows.append((float(parts[0]), float(parts[1]), parts[4:8]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def step_traffic(cfg):
    """DRAM bytes per step-kernel launch from the committed ncu summary
    (profiles/step_kernel_traffic.json, measured on a reduced-depth model and
    scaled per layer), or None if there is none for this model."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", "step_kernel_traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
    except (OSError, ValueError):
        return None
    per_layer, fixed = t.get("bytes_per_layer"), t.get("bytes_fixed")
    if per_layer is None or fixed is None:
        return None
    return fixed + per_layer * cfg.num_hidden_layers


def argmax_last(v):
    import numpy as np
    return int(np.flatnonzero(v == v.max())[-1])


def config1_dict(cfg, world):
    """The `config` object of both arms' lines."""
    return {"workload": f"gemma3-4b Q4_K decode bs=1 (BASELINE config 1), layers={cfg.num_hidden_layers}",
            "prompt": PROMPT, "decode_positions": [PROMPT, PROMPT + SPAN - 1], "kv": "f32",
            "vocab": cfg.vocab_size, "l2": "inputs larger than L2: 3.3 GB of weights + KV per step",
            "parallelism": f"dp{world} (one sequence and weight replica per GPU)"}


REF_MAX_STEPS = 64


def run_reference(args):
    """Reference arm: the CPU decode step (oracle restatement of the reference's
    x86 path) on all host threads, on config 1's shapes.  Only liboracle.so is
    loaded: the synthetic model comes from its own copy of the seeded
    generator."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import numpy as np

    from oracle import oracle as orc
    from rich_triplet_b200.model import Config4, synth_gemma3, synth_normal, synth_tokens

    gen = orc.lib
    cfg = Config4.gemma3_4b(vocab_size=262144).with_layers(args.layers)
    w = synth_gemma3(cfg, seed=args.seed, gen=gen)
    cap = PROMPT + SPAN
    om = orc.OracleModel(cfg, w, cap, nthreads=0)
    kvd = cfg.num_key_value_heads * cfg.head_dim
    # Positions 0..511 of every layer's f32 cache hold N(0,1) values: prefilling
    # 512 tokens through the CPU path would take minutes, and a decode step
    # reads the same bytes whatever the cached values are.
    for layer in range(cfg.num_hidden_layers):
        kc = np.ctypeslib.as_array(orc.lib.or_model_kcache(om._h, layer), shape=(cap * kvd,))
        vc = np.ctypeslib.as_array(orc.lib.or_model_vcache(om._h, layer), shape=(cap * kvd,))
        kc[: PROMPT * kvd] = synth_normal(args.seed, 5000 + 2 * layer, PROMPT * kvd, gen=gen)
        vc[: PROMPT * kvd] = synth_normal(args.seed, 5001 + 2 * layer, PROMPT * kvd, gen=gen)
    tok = int(synth_tokens(args.seed, 100, 1, cfg.vocab_size, gen=gen)[0])
    n_warm = max(1, min(args.warmup, 8))
    n_steps = max(1, min(args.steps, REF_MAX_STEPS))
    om.set_seq_len(PROMPT)
    for _ in range(n_warm):
        tok = orc.sample_greedy(om.step(tok))
    om.set_seq_len(PROMPT)
    t0 = time.perf_counter()
    for _ in range(n_steps):
        tok = orc.sample_greedy(om.step(tok))
    dt = time.perf_counter() - t0
    value = n_steps / dt
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": n_steps, "warmup": n_warm, "ms_per_step": dt * 1e3 / n_steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config1_dict(cfg, world),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"{n_steps} CPU decode steps at positions 512.. (steps capped at {REF_MAX_STEPS}); "
                                   "reference is Rust (no toolchain here): oracle/ C restatement of its x86 path, "
                                   "row-parallel over all host threads; KV rows 0..511 synthetic"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    om.close()


def cpu_baselines_config0_config2(args, orc):
    """The reference CPU path of BASELINE configs 0 and 2 timed on the host:
    config 0's Q4_K GEMV (Q4KMat::gemv_mt: rows split over all host threads)
    and config 2's Q4_K GEMM at M = 512 (Q4KMat::matmul_q4k_t, single-threaded
    in the reference), the latter on a bounded sample of output rows."""
    import numpy as np

    from rich_triplet_b200.model import synth_normal, synth_q4k

    gen = orc.lib
    out = {}
    for rows, cols in ((10240, 2560), (2560, 10240)):
        blocks = synth_q4k(args.seed, 9000, rows, cols, gen=gen)
        x = synth_normal(args.seed, 9100, cols, gen=gen)
        orc.q4k_gemv(blocks, rows, cols, x)
        reps = 20
        t0 = time.perf_counter()
        for _ in range(reps):
            orc.q4k_gemv(blocks, rows, cols, x)
        us = (time.perf_counter() - t0) * 1e6 / reps
        b = rows * cols // 256 * 144 + cols * 4 + rows * 4
        out[f"config0_gemv_{rows}x{cols}"] = {"us": us, "gbs": b / (us * 1e-6) / 1e9, "cores": os.cpu_count(),
                                              "kind": "port", "sample": f"{reps} GEMVs, all host threads"}
    m = 512
    for name, k, n in (("qkv", 2560, 4096), ("o", 2048, 2560), ("gate_up", 2560, 20480), ("down", 10240, 2560)):
        ns = 16  # output rows sampled: the loop is the same for every row
        blocks = synth_q4k(args.seed, 9200 + n + k, ns, k, gen=gen)
        a = synth_normal(args.seed, 9300 + m, m * k, gen=gen).reshape(m, k)
        t0 = time.perf_counter()
        orc.q4k_gemm(blocks, ns, k, a)
        dt = time.perf_counter() - t0
        tf = 2.0 * m * ns * k / dt / 1e12
        out[f"config2_gemm_{name}_M{m}_K{k}_N{n}"] = {
            "tflops": tf, "est_ms_full": dt * n / ns * 1e3, "cores": 1, "kind": "port",
            "sample": f"{ns} of {n} output rows, f32 A (the reference's loop is single-threaded)"}
    return out


CONFIG3_SEQS, CONFIG3_CONTEXT, CONFIG3_STEPS = 64, 4096, 128


def batch_step_bytes(cfg, context, nseq, weight_bytes):
    """Bytes one many-sequence step must move: every weight once, plus each
    sequence's K and V rows at `context` cached positions (local layers read
    at most the sliding window)."""
    row = 2 * cfg.num_key_value_heads * cfg.head_dim * 4
    kv = 0
    for layer in range(cfg.num_hidden_layers):
        n = context + 1
        if not cfg.is_global_layer(layer) and cfg.sliding_window:
            n = min(n, cfg.sliding_window)
        kv += row * n
    return weight_bytes + nseq * kv


def batch_decode_config3(args, cfg, dec, ctx, ext, world, rank, dist, device, hbm_peak, weight_bytes):
    import torch

    from rich_triplet_b200 import dp
    from rich_triplet_b200.decode import CudaBatchDecoder

    s0, s1 = dp.shard(CONFIG3_SEQS, world, rank)
    nseq = s1 - s0
    warm = 3
    bat = CudaBatchDecoder(dec, nseq, CONFIG3_CONTEXT + warm + CONFIG3_STEPS + 1)
    try:
        bat.synth_kv(args.seed + rank, CONFIG3_CONTEXT)
        bat.generate(warm)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        bat.generate(CONFIG3_STEPS, wait=False)
        e1.record(ext)
        e1.synchronize()
        ctx.sync()
        ms = e0.elapsed_time(e1)
        mem, launches = bat.info()
    finally:
        bat.close()
    ms_max = dp.max_over_ranks(ms, dist, device)
    per_step = sum(batch_step_bytes(cfg, CONFIG3_CONTEXT + warm + i, nseq, weight_bytes)
                   for i in range(CONFIG3_STEPS)) / CONFIG3_STEPS
    gbs = per_step * CONFIG3_STEPS / (ms / 1e3) / 1e9
    return {
        "value": dp.job_rate(CONFIG3_SEQS * CONFIG3_STEPS, ms_max), "unit": "tok/s",
        "sequences": CONFIG3_SEQS, "sequences_per_gpu": nseq, "context": CONFIG3_CONTEXT, "steps": CONFIG3_STEPS,
        "ms_per_step": ms_max / CONFIG3_STEPS, "scaling": "strong (64 sequences in total, sharded by sequence)",
        "hbm_gbs_per_gpu": gbs, "frac": gbs / hbm_peak, "bytes_per_step_per_gpu": per_step,
        "device_bytes_per_gpu": mem, "gpu_launches_per_step": launches,
        "kv": "f32, synthetic contents at the 4096-token context (no prefill)",
        "gemm_operands": "fp16 activation rows (power-of-two row scales) and dequantised weights, f32 accumulation",
        "method": "one CUDA graph replay per step, CUDA events around 128 steps after 3 warm-up, max over ranks",
    }


CONFIG4_CONTEXT, CONFIG4_STEPS, CONFIG4_BATCHES = 8192, 16, (1, 8)


def tp_step_bytes(cfg, nranks, rank, context, nseq):
    """Bytes one tensor-parallel step must move on `rank`: its Q4_K shard, its
    slice of the BF16 LM head, and its KV heads' rows at `context`."""
    from rich_triplet_b200.tp import shard_config

    sc = shard_config(cfg, nranks, rank)
    H, D = cfg.hidden_size, cfg.head_dim
    q, kv, f = sc.num_attention_heads * D, sc.num_key_value_heads * D, sc.intermediate_size
    per_layer = (q * H + 2 * kv * H + H * q + 3 * f * H) // 256 * 144
    vr = cfg.vocab_size * (rank + 1) // nranks - cfg.vocab_size * rank // nranks
    kv_bytes = 0
    for layer in range(cfg.num_hidden_layers):
        n = context + 1
        if not cfg.is_global_layer(layer) and cfg.sliding_window:
            n = min(n, cfg.sliding_window)
        kv_bytes += 2 * kv * 4 * n
    return cfg.num_hidden_layers * per_layer + vr * H * 2 + nseq * kv_bytes


def all_ok(flag, dist, device):
    """True on every rank iff `flag` is true on every rank."""
    if dist is None:
        return bool(flag)
    import torch

    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def tp_decode_config4(args, world, rank, dist, device, hbm_peak):
    """Gemma 3 27B (synthetic weights), tensor parallel over
    the job's ranks, batch 1 and 8, each sequence at an 8192-token synthetic
    f32 KV cache; greedy steps timed with CUDA events, max over ranks."""
    import torch

    from rich_triplet_b200 import dp
    from rich_triplet_b200.decode import CudaDecodeContext
    from rich_triplet_b200.model import Config4
    from rich_triplet_b200.ops import Context
    from rich_triplet_b200.tp import TpBatchDecoder, share_nccl_id, synth_shard_weights

    cfg = Config4.gemma3_27b()
    out = {"model": "gemma3-27b (62 layers, hidden 5376, FFN 21504, 32/16 heads of 128), synthetic Q4_K weights",
           "parallelism": f"tp{world}: heads and FFN columns split, all-reduce after o and down, vocab-split LM head",
           "allreduce": ("none" if world == 1 else
                         "peer kernel (NVLink stores, one launch per sum)" if args.tp_allreduce == "peer" else "NCCL"),
           "context": CONFIG4_CONTEXT, "steps": CONFIG4_STEPS, "kv": "f32, synthetic contents (no prefill)",
           "gemm_operands": "fp16, f32 accumulation"}
    ctx = dec = None
    err = None
    try:
        ctx = Context(device)
        t0 = time.perf_counter()
        dec = CudaDecodeContext(synth_shard_weights(cfg, args.seed, world, rank), 16, ctx)
        out["setup_s"] = time.perf_counter() - t0
    except Exception as e:  # reported in the line; every rank learns of it below
        err = f"{type(e).__name__}: {e}"
    if not all_ok(err is None, dist, device):
        out["error"] = err or "another rank failed to build its shard"
        if dec is not None:
            dec.close()
        if ctx is not None:
            ctx.close()
        return out
    ext = torch.cuda.ExternalStream(ctx.stream_ptr)
    warm = 3
    for nseq in CONFIG4_BATCHES:
        nccl_id = share_nccl_id(dist, rank) if world > 1 else None
        bat = None
        try:
            bat = TpBatchDecoder(dec, nseq, CONFIG4_CONTEXT + warm + CONFIG4_STEPS + 1, world, rank, nccl_id)
            bat.synth_kv(args.seed + rank, CONFIG4_CONTEXT)
            if world > 1 and args.tp_allreduce == "peer":
                bat.enable_peer_allreduce(dist)
        except Exception as e:
            err = f"{type(e).__name__}: {e}"
        if not all_ok(err is None, dist, device):
            out[f"batch{nseq}"] = {"error": err or "another rank failed"}
            if bat is not None:
                bat.close()
            break
        bat.generate(warm)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        bat.generate(CONFIG4_STEPS, wait=False)
        e1.record(ext)
        e1.synchronize()
        ctx.sync()
        ms = e0.elapsed_time(e1)
        mem, launches = bat.info()
        bat.close()
        ms_max = dp.max_over_ranks(ms, dist, device)
        per_step = sum(tp_step_bytes(cfg, world, rank, CONFIG4_CONTEXT + warm + i, nseq)
                       for i in range(CONFIG4_STEPS)) / CONFIG4_STEPS
        gbs = per_step * CONFIG4_STEPS / (ms / 1e3) / 1e9
        out[f"batch{nseq}"] = {"value": dp.job_rate(nseq * CONFIG4_STEPS, ms_max), "unit": "tok/s",
                               "ms_per_step": ms_max / CONFIG4_STEPS, "hbm_gbs_rank0": gbs, "frac": gbs / hbm_peak,
                               "bytes_per_step_rank0": per_step, "device_bytes_engine_rank0": mem,
                               "launches_per_step": launches, "all_reduces_per_step": 2 * cfg.num_hidden_layers
                               if world > 1 else 0}
    dec.close()
    ctx.close()
    return out


def qwen35_decode(args, device, hbm_peak):
    """The Qwen 3.5 decode engine (rt_qwen35_*, the reference's
    MetalDecodeContextQwen35): the 4B widths (32 layers, 24 Gated DeltaNet +
    8 full attention, vocabulary 248320) on synthetic weights, greedy-free
    steps at positions 8..39 after 8 warm-up steps, CUDA events around them.
    Bytes per step: every Q4_K projection, the BF16 LM head, each DeltaNet
    state read and written, the K/V rows attended."""
    import torch

    from rich_triplet_b200.qwen35 import CudaQwen35Decoder, Qwen35Config, synth_qwen35

    cfg = Qwen35Config.qwen35_4b()
    w = synth_qwen35(cfg, seed=args.seed)
    dec = CudaQwen35Decoder(w, 1024)
    try:
        warm, n = 8, 32
        for p in range(warm):
            dec.step_device((p * 7919) % cfg.vocab_size, p)
        ext = torch.cuda.ExternalStream(dec.ctx.stream_ptr)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        for p in range(warm, warm + n):
            dec.step_device((p * 7919) % cfg.vocab_size, p)
        e1.record(ext)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / n
    finally:
        dec.close()
        dec.ctx.close()
    q4k = sum(b.size for L in w.layers for b in L.proj.values())
    n_dn = sum(1 for L in w.layers if not L.full)
    state = n_dn * cfg.linear_num_value_heads * cfg.linear_key_head_dim * cfg.linear_value_head_dim * 4 * 2
    kv = (cfg.num_hidden_layers - n_dn) * (warm + n / 2) * cfg.num_key_value_heads * cfg.head_dim * 4 * 2
    step_bytes = q4k + cfg.vocab_size * cfg.hidden_size * 2 + state + kv
    gbs = step_bytes / (ms / 1e3) / 1e9
    return {"model": "Qwen 3.5 4B widths (32 layers: 24 Gated DeltaNet, 8 full attention), synthetic Q4_K weights",
            "value": 1e3 / ms, "unit": "tok/s", "ms_per_step": ms, "positions": [warm, warm + n],
            "bytes_per_step": step_bytes, "hbm_gbs": gbs, "frac": gbs / hbm_peak,
            "method": "one CUDA graph launch per step (rt_qwen35_step), host sync per step, CUDA events around 32 steps"}


def run_ours(args):
    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180))
    else:
        torch.cuda.set_device(0)
    device = torch.cuda.current_device()

    from rich_triplet_b200 import dp
    from rich_triplet_b200.decode import CudaDecodeContext
    from rich_triplet_b200.model import Config4, synth_gemma3, synth_tokens
    from rich_triplet_b200.ops import Context

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    hbm_peak, tc_peak, peak_kind = peaks()
    cfg = Config4.gemma3_4b(vocab_size=262144).with_layers(args.layers)
    w = synth_gemma3(cfg, seed=args.seed)
    ctx = Context(device)
    cap = PROMPT + SPAN
    dec = CudaDecodeContext(w, cap, ctx)
    ext = torch.cuda.ExternalStream(ctx.stream_ptr)
    # one sequence per rank: the rank's share of `world` independent sequences
    seq0, _ = dp.shard(world, world, rank)
    prompt = synth_tokens(args.seed, dp.prompt_stream(seq0), PROMPT, cfg.vocab_size)
    t_pf = time.perf_counter()
    last = dec.prefill(prompt)
    prefill_token_ms = (time.perf_counter() - t_pf) * 1e3
    first = argmax_last(last)

    def enqueue(n):
        done = 0
        while done < n:
            m = min(SPAN, n - done)
            dec.enqueue_generate(first, PROMPT, m)
            done += m

    # ---- warm-up ----
    enqueue(max(3, args.warmup))
    ctx.sync()
    barrier()

    # ---- timed decode (inputs resident in HBM) ----
    clocks = ClockSampler(device)
    clocks.start()
    time.sleep(0.3)
    barrier()
    ctx.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    enqueue(args.steps)
    e1.record(ext)
    e1.synchronize()
    ctx.sync()
    ms = e0.elapsed_time(e1)
    barrier()
    clock_info = clocks.stop()
    ms_max = dp.max_over_ranks(ms, dist, device)
    value = dp.job_rate(world * args.steps, ms_max)

    # ---- whole-step bytes (weights + KV read), for the step roofline ----
    H, D, NKV = cfg.hidden_size, cfg.head_dim, cfg.num_key_value_heads
    q4k_bytes = w.q4k_bytes()
    lm_bytes = cfg.vocab_size * H * 2
    kv_per_pos = 2 * NKV * D * 4
    kv_avg = sum(kv_per_pos * (p + 1) * cfg.num_hidden_layers for p in range(PROMPT, PROMPT + SPAN)) / SPAN
    step_bytes = q4k_bytes + lm_bytes + kv_avg + H * 2
    step_gbs = step_bytes * args.steps / (ms / 1e3) / 1e9

    # ---- e2e through the public API: host token in, host logits out ----
    e2e = None
    if True:
        pinned = torch.empty(cfg.vocab_size, dtype=torch.float32).pin_memory()
        buf = pinned.numpy()
        n_e2e = min(args.steps, SPAN)
        tok, pos = first, PROMPT
        for _ in range(3):
            dec.decode_step(tok, pos, out=buf)
        barrier()
        t0 = time.perf_counter()
        for i in range(n_e2e):
            dec.decode_step(tok, PROMPT + i, out=buf)
            tok = int(buf.argmax())
        dt = time.perf_counter() - t0
        tt = torch.tensor([dt], device="cuda")
        if dist is not None:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e = {"value": world * n_e2e / float(tt.item()), "unit": "tok/s", "h2d_bytes_per_step": 8,
               "d2h_bytes_per_step": cfg.vocab_size * 4 + 4}

    # ---- 64 sequences at a 4096-token context, sharded by
    # sequence over the ranks, 128 greedy steps each (synthetic f32 caches) ----
    batch3 = batch_decode_config3(args, cfg, dec, ctx, ext, world, rank, dist, device, hbm_peak,
                                  w.q4k_bytes() + cfg.vocab_size * cfg.hidden_size * 2)

    # ---- Gemma 3 27B tensor parallel over the ranks ----
    tp4 = tp_decode_config4(args, world, rank, dist, device, hbm_peak) if not args.no_config4 else None

    # ---- the Qwen 3.5 decode engine (one GPU: a single-sequence engine) ----
    qwen = None
    if world == 1 and not args.no_qwen35:
        try:
            qwen = qwen35_decode(args, device, hbm_peak)
        except Exception as e:  # reported in the line
            qwen = {"error": f"{type(e).__name__}: {e}"}

    # ---- standalone Q4_K GEMV, CUDA graph of 256 chained
    # launches rotating over 16 weight copies (236 MB > L2) ----
    gemv0 = {}
    if rank == 0:
        from rich_triplet_b200._lib import RT_FMT_Q4K
        from rich_triplet_b200.model import synth_normal, synth_q4k
        from rich_triplet_b200.ops import DeviceWeight, gemv_bench
        for rows, cols in ((10240, 2560), (2560, 10240)):
            copies = [DeviceWeight.upload(ctx, RT_FMT_Q4K, synth_q4k(args.seed, 9000 + c, rows, cols), rows, cols)
                      for c in range(16)]
            x = torch.from_numpy(synth_normal(args.seed, 9100, cols)).cuda()
            y = torch.empty(rows, dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            b = rows * cols // 256 * 144 + cols * 4 + rows * 4
            modes = {}
            for cps in (1, 2):
                us = gemv_bench(ctx, copies, x.data_ptr(), y.data_ptr(), launches=256, ctas_per_sm=cps, reps=3)
                modes[f"ctas_per_sm={cps}"] = {"us": us, "gbs": b / (us * 1e-6) / 1e9}
            best = max(modes.values(), key=lambda m: m["gbs"])
            gemv0[f"{rows}x{cols}"] = {"us": best["us"], "gbs": best["gbs"], "frac": best["gbs"] / hbm_peak, "bytes": b,
                                       "modes": modes,
                                       "method": "CUDA graph of 256 GEMVs chained by programmatic dependent launch, "
                                                 "16 rotating weight copies (236 MB > L2), mean of 3 replays"}
            for c in copies:
                c.free()

    # ---- Q4_K prefill GEMM (tcgen05), bf16 A ~ N(0,1) ----
    gemm2 = {}
    if rank == 0:
        from rich_triplet_b200._lib import RT_FMT_Q4K
        from rich_triplet_b200.model import synth_normal_bf16, synth_q4k
        from rich_triplet_b200.ops import DeviceWeight, gemm_device
        shapes = (("qkv", 2560, 4096), ("o", 2048, 2560), ("gate_up", 2560, 20480), ("down", 10240, 2560))
        for name, k, n in shapes:
            gw = DeviceWeight.upload(ctx, RT_FMT_Q4K, synth_q4k(args.seed, 9200 + n + k, n, k), n, k)
            for m in (512, 2048):
                ga = torch.from_numpy(synth_normal_bf16(args.seed, 9300 + m, m * k).view(np.int16)).cuda()
                cm = torch.empty((m, n), dtype=torch.float32, device="cuda")
                torch.cuda.synchronize()
                for _ in range(3):
                    gemm_device(ctx, gw, ga.data_ptr(), m, cm.data_ptr())
                ctx.sync()
                reps = 5
                e0.record(ext)
                for _ in range(reps):
                    gemm_device(ctx, gw, ga.data_ptr(), m, cm.data_ptr())
                e1.record(ext)
                e1.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / reps
                tf = 2.0 * m * n * k / (us * 1e-6) / 1e12
                gemm2[f"{name}_M{m}_K{k}_N{n}"] = {"us": us, "tflops": tf, "frac": tf / tc_peak}
                del ga, cm
            gw.free()
        gemm2["peak_tflops"] = tc_peak
        gemm2["method"] = "device time per GEMM (CUDA events, mean of 5 after 3 warm-up), A bf16 ~ N(0,1) resident"

    # ---- CPU baseline: the oracle decode step on host cores (rank 0, N=1) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as orc
        om = orc.OracleModel(cfg, w, cap, nthreads=0)
        kvd = NKV * D
        for layer in range(cfg.num_hidden_layers):
            k, v = dec.read_kv(layer, PROMPT)
            np.ctypeslib.as_array(orc.lib.or_model_kcache(om._h, layer), shape=(cap * kvd,))[: PROMPT * kvd] = k
            np.ctypeslib.as_array(orc.lib.or_model_vcache(om._h, layer), shape=(cap * kvd,))[: PROMPT * kvd] = v
        om.set_seq_len(PROMPT)
        tok = first
        t0 = time.perf_counter()
        for _ in range(args.cpu_steps):
            tok = orc.sample_greedy(om.step(tok))
        dt = time.perf_counter() - t0
        cpu = {"value": args.cpu_steps / dt, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{args.cpu_steps} decode steps at positions 512..{511 + args.cpu_steps} of the same model, "
                         "KV cache copied from the GPU prefill; oracle/ restatement of the reference's x86 path"}
        om.close()
        cpu["per_config"] = cpu_baselines_config0_config2(args, orc)

    # ---- prefill of config 1's prompt with every position at once (tensor-core
    # GEMMs over the 512 tokens), against the token-by-token prefill above ----
    prefill = None
    if rank == 0:
        for _ in range(2):
            dec.prefill_gemm(prompt, want_logits=False)
        reps = 5
        t_pf = time.perf_counter()
        for _ in range(reps):
            lg = dec.prefill_gemm(prompt)
        gemm_ms = (time.perf_counter() - t_pf) * 1e3 / reps
        prefill = {"tokens": PROMPT, "gemm_ms": gemm_ms, "gemm_tok_s": PROMPT / (gemm_ms / 1e3),
                   "token_by_token_ms": prefill_token_ms, "token_by_token_tok_s": PROMPT / (prefill_token_ms / 1e3),
                   "same_greedy_token": argmax_last(lg) == first,
                   "method": "host wall time of rt_decoder_prefill_gemm (mean of 5 after 2 warm-up, host tokens in, "
                             "last logits out) vs one rt_decoder_prefill of the same prompt"}

    launches = dec.launches_per_step
    # The dominant kernel: the persistent step kernel (one launch per token),
    # or the per-projection GEMVs when the CUDA-graph path is selected.
    kernel_name = "step_kernel (one decode step per launch)" if launches == 1 else "decode graph (per-projection kernels)"
    traffic = step_traffic(cfg) if launches == 1 else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config1_dict(cfg, world),
            "roofline": {"bound": "hbm", "achieved": step_gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": step_gbs / hbm_peak, "traffic": traffic, "kernel": kernel_name,
                         "launch_us": ms / args.steps * 1e3, "bytes_per_launch": step_bytes, "peak_kind": peak_kind,
                         "bytes_model": "Q4_K weights + BF16 LM head + f32 KV read at the mean decode position + "
                                        "embedding row"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches * args.steps,
            "clocks": clock_info,
            "q4k_gemv_config0": gemv0,
            "q4k_gemm_config2": gemm2,
            "batch_decode_config3": batch3,
            "prefill_config1": prefill,
            "tp_decode_config4": tp4,
            "qwen35_decode": qwen,
        }
        print(json.dumps(line), flush=True)
    dec.close()
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    global PROMPT
    args = parse()
    PROMPT = args.prompt
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
