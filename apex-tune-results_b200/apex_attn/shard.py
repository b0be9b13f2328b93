"""Batch x head sharding across ranks and the gather of the sharded output.

Every (b, h) pair is an independent attention problem, so the multi-GPU path gives each
rank a contiguous slice of the flattened b*h axis and runs the same persistent kernel on
it with no inter-GPU traffic inside the kernel; the only collective is the gather of
the per-rank outputs to rank 0 for checking (the reference is single-GPU only,
mls-bench_fused_attention/README.md:53).
"""
from __future__ import annotations

import torch


def shard_heads(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of the flattened b*h range owned by `rank` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def gather_to_rank0(local: torch.Tensor, total: int, world: int, rank: int, group=None):
    """Gathers per-rank [heads_r, ...] slices into a [total, ...] tensor on rank 0.

    Uses one torch.distributed.gather of equal-sized (padded) buffers, so it works on
    NCCL (CUDA tensors) and gloo (CPU tensors) alike. Returns None on other ranks."""
    import torch.distributed as dist

    counts = [shard_heads(total, world, r) for r in range(world)]
    width = max(e - s for s, e in counts)
    buf = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[: local.shape[0]].copy_(local)
    bufs = [torch.empty_like(buf) for _ in range(world)] if rank == 0 else None
    dist.gather(buf, gather_list=bufs, dst=0, group=group)
    if rank != 0:
        return None
    return torch.cat([b[: e - s] for b, (s, e) in zip(bufs, counts)], dim=0)
