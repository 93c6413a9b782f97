"""Batch data parallelism for the encoder plan: one process per GPU, each
rank runs its contiguous slice of the batch through its own EncoderPlan
(weights replicated), and the only exchange is the gather of the [B_local,
n_classes] logits to rank 0 over torch.distributed (NCCL on GPUs, gloo on
CPU). Sequences are independent, so no other collective is needed.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's rows; the first total % world ranks get one
    extra row, so shard sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if total < 0:
        raise ValueError("negative batch")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_logits(local: torch.Tensor, total: int, group=None) -> torch.Tensor | None:
    """Gathers every rank's [rows, C] logits into the full [total, C] tensor
    on rank 0 (None elsewhere). Uneven shards are padded to the largest one
    for the fixed-size all_gather and trimmed afterwards."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    C = local.shape[1]
    biggest = shard_rows(total, world, 0)[1]
    start, end = shard_rows(total, world, rank)
    if local.shape[0] != end - start:
        raise ValueError(f"rank {rank}: {local.shape[0]} logit rows, expected {end - start}")
    padded = torch.zeros(biggest, C, dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    out = torch.empty(world * biggest, C, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, padded, group=group)
    if rank != 0:
        return None
    parts = []
    for r in range(world):
        s, e = shard_rows(total, world, r)
        parts.append(out[r * biggest: r * biggest + (e - s)])
    return torch.cat(parts, 0)
