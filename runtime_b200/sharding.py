"""Sequence sharding across GPUs (one process per GPU).

Independent sequences (and the prefix-state replicas they fork from) need no
exchange while they decode, so a multi-GPU run gives every rank a full
weight replica and a contiguous slice of the sequences: rank r of P serves
sequences [r * S // P, (r + 1) * S // P).  The only collectives are outside
the decode path: a barrier around the timed region and the max over ranks
of the measured time.  The reference has no multi-device code; its
executors are single-device and `!Send` (crates/engine-api/src/backend.rs:31-34),
so one process (or host thread) per device ordinal is the natural mapping.
"""
from __future__ import annotations

import os


def shard(n_items: int, world: int, rank: int) -> range:
    """The contiguous slice of `n_items` owned by `rank` of `world`
    (sizes differ by at most one; every item is owned exactly once)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if n_items < 0:
        raise ValueError("negative item count")
    return range(n_items * rank // world, n_items * (rank + 1) // world)


def env_rank() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from the torchrun environment."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Max of a per-rank measurement (no-op in a single process)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def head_shard_rows(vocab: int, world: int, rank: int) -> range:
    """The LM-head rows rank `rank` scores under mf_lfm2_set_head_split:
    contiguous shards of ceil(vocab / world) rounded up to 16 rows (the
    integer-MMA tile), the last one shorter."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    chunk = ((vocab + world - 1) // world + 15) // 16 * 16
    if world > 1 and chunk * (world - 1) >= vocab:
        raise ValueError("head has too few rows for this split")
    start = min(chunk * rank, vocab)
    return range(start, min(start + chunk, vocab))


def head_split_id(dist=None) -> bytes:
    """The NCCL id of a head split: made on rank 0, broadcast over the host
    process group (any backend, gloo included), identical on every rank."""
    from . import lfm2

    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return lfm2.nccl_unique_id()
    box = [lfm2.nccl_unique_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return box[0]
