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
