"""Data-parallel decode across ranks (one process per GPU, torch.distributed
for the plumbing).

Sequences are independent (BASELINE configs 1 and 3: one weight replica per
GPU, sequences sharded across GPUs), so each rank decodes its own share with no
collective on the data path.  Only the measurement is combined: the job's
device time is the maximum over ranks, and its rate is the units all ranks
processed over that time.  The reference has no multi-GPU path; this module is
the host logic `bench.py` uses and the gloo tests cover.
"""


def shard(n_items, world, rank):
    """The contiguous share [start, end) of `n_items` that `rank` owns; shares
    differ in size by at most one and cover every item exactly once."""
    if world < 1 or not 0 <= rank < world or n_items < 0:
        raise ValueError(f"shard: n_items={n_items} world={world} rank={rank}")
    return n_items * rank // world, n_items * (rank + 1) // world


def prompt_stream(sequence):
    """Synthetic-token stream id of global sequence `sequence` (its prompt is
    the same whichever rank decodes it)."""
    return 100 + sequence


def max_over_ranks(value, dist=None, device=None):
    """Maximum of a per-rank float (a device time) over the process group."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_rate(units_total, ms):
    """Whole-job throughput: units per second over `ms` milliseconds."""
    if ms <= 0:
        raise ValueError("job_rate: non-positive time")
    return units_total / (ms / 1e3)
