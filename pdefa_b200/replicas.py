"""Data-parallel replicas: one process (rank) per GPU, images split into shards.

Images are independent (``pdefa/python/src/pdefa/batch.py:50-53`` runs one Session
per image), so N GPUs run N replicas of the model on contiguous shards and never
exchange activations. The only collective is the end-of-run reduction of the
per-rank device times (max over ranks, as the job finishes when the slowest rank
does) and of the per-rank image counts.

``shard_bounds`` is the split the native multi-GPU runner (``pdefa_batch_run``)
uses across devices of one process: ceil(n / world) images per shard, the last
shards shorter or empty.
"""
from __future__ import annotations

from typing import Tuple


def shard_bounds(n_images: int, rank: int, world: int) -> Tuple[int, int]:
    """[lo, hi) of rank's contiguous shard of n_images."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if n_images < 0:
        raise ValueError("n_images must be >= 0")
    per = (n_images + world - 1) // world
    lo = min(n_images, rank * per)
    return lo, min(n_images, lo + per)


def reduce_job(local_ms: float, local_images: int, device=None):
    """(max device ms over ranks, total images over ranks) of the current process
    group; (local_ms, local_images) when torch.distributed is not initialised.

    device: where the reduction tensors live (a CUDA device for NCCL, None = CPU
    for gloo)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(local_ms), int(local_images)
    t = torch.tensor([float(local_ms)], dtype=torch.float64, device=device)
    n = torch.tensor([int(local_images)], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(n, op=dist.ReduceOp.SUM)
    return float(t.item()), int(n.item())


def job_throughput(total_images: int, max_ms: float) -> float:
    """Whole-job images per second: all ranks' images over the slowest rank's time."""
    if max_ms <= 0:
        raise ValueError("max_ms must be > 0")
    return total_images / (max_ms / 1e3)
