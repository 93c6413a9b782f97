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


def gather_logits(local: torch.Tensor, total: int, group=None,
                  out: torch.Tensor | None = None) -> torch.Tensor | None:
    """Gathers every rank's [rows, C] logits into the full [total, C] tensor
    on rank 0 (None elsewhere) with one gather to rank 0: only rank 0
    receives, each other rank sends its shard once. Uneven shards are padded
    to the largest one (the collective moves equal blocks) and rank 0 trims
    the padding. `out` (rank 0, optional) is a [world * largest, C] buffer
    reused across steps; with even shards the result is a view of it."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    C = local.shape[1]
    biggest = shard_rows(total, world, 0)[1]
    start, end = shard_rows(total, world, rank)
    if local.shape[0] != end - start:
        raise ValueError(f"rank {rank}: {local.shape[0]} logit rows, expected {end - start}")
    send = local.contiguous()
    if send.shape[0] != biggest:
        send = torch.zeros(biggest, C, dtype=local.dtype, device=local.device)
        send[: local.shape[0]] = local
    if rank != 0:
        dist.gather(send, None, dst=0, group=group)
        return None
    if out is None or out.shape != (world * biggest, C):
        out = torch.empty(world * biggest, C, dtype=local.dtype, device=local.device)
    dist.gather(send, [out[r * biggest:(r + 1) * biggest] for r in range(world)], dst=0,
                group=group)
    if total == world * biggest:
        return out
    parts = []
    for r in range(world):
        s, e = shard_rows(total, world, r)
        parts.append(out[r * biggest: r * biggest + (e - s)])
    return torch.cat(parts, 0)


class Membership:
    """Host-side record of which ranks are still serving, kept in the
    process group's key-value store. A rank that stops between steps calls
    leave(); every rank calls departed() before it launches its next step and
    stops (raising PeerLeft) instead of entering a collective that a missing
    peer would never join. Nothing here touches a device."""

    def __init__(self, store, world: int, rank: int, prefix: str = "inferc/left/"):
        self.store, self.world, self.rank, self.prefix = store, world, rank, prefix

    def leave(self) -> None:
        self.store.set(f"{self.prefix}{self.rank}", "1")

    def departed(self) -> list[int]:
        keys = [f"{self.prefix}{r}" for r in range(self.world) if r != self.rank]
        return [r for r, k in zip([r for r in range(self.world) if r != self.rank], keys)
                if self.store.check([k])]

    def check(self) -> None:
        gone = self.departed()
        if gone:
            raise PeerLeft(gone)


class PeerLeft(RuntimeError):
    """Raised on a rank whose peers have left the job between steps."""

    def __init__(self, ranks: list[int]):
        super().__init__(f"ranks {ranks} left the job; no further collective is issued")
        self.ranks = ranks
