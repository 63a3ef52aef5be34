"""Rank plumbing shared by bench.py and the sharded CLI (torch.distributed).

Every rank calls these in the same order (collectives must match).  They
work on NCCL (CUDA tensors) and on gloo (CPU tensors), so the multi-rank
logic is tested on CPU with gloo ranks.
"""
from __future__ import annotations


def reduce_max(dist, value: float, device) -> float:
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_all(dist, flag: bool, device) -> bool:
    import torch
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def weak_scaling_rate(work_per_rank: float, world: int, steps: int, max_total_ms: float) -> float:
    """Whole-job rate (work units per second / 1e12): every rank processed
    `steps` units of `work_per_rank`; the job took the slowest rank's time."""
    return work_per_rank * world * steps / (max_total_ms / 1e3) / 1e12


def strong_scaling_rate(total_work: float, max_median_ms: float) -> float:
    """Rate of one GEMM split across ranks: total work / slowest rank."""
    return total_work / (max_median_ms / 1e3) / 1e12


def reduce_rows(dist, device, keys, measure):
    """Per key, this rank's measure(key) -> (median ms, parity ok, max rel),
    then one all-reduce (max) of [ms, rel, failed] over the ranks, taken
    whatever happened on this rank: an exception in measure counts as a
    failed row with an infinite time, so the other ranks are never left
    waiting in a collective that this rank skipped.  Returns, per key, the
    job's (max ms, max rel, every rank ok, this rank's error text or "")."""
    import torch
    out = []
    for key in keys:
        ms, ok, rel, err = float("inf"), False, float("inf"), ""
        try:
            ms, ok, rel = measure(key)
        except Exception as e:   # reported in the row; the collective below still runs
            ok, err = False, (str(e).splitlines() or [type(e).__name__])[0][:200]
        t = torch.tensor([float(ms), float(rel) if ok else float("inf"), 0.0 if ok else 1.0],
                         dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max, rel_max, failed = (float(v) for v in t.tolist())
        out.append((ms_max, rel_max, failed == 0.0, err))
    return out
