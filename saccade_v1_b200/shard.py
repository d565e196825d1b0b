"""Batch sharding of the scan over the GPUs of one node (one process per GPU).

The selective scan has no exchange between (batch, channel) lanes (zero or
per-track carried state, reference tests/selective_scan_tests.cpp:250-261), so
each rank scans a contiguous slice of the batch with no collective on the scan
path.  The only collective is the optional assembly of the full output
(all-gather over NVLink with NCCL), preceded by a one-word all-reduce of the
ranks' failure flags so that every rank learns of a failed shard before any
rank waits on the gather.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    begin: int   # first batch row of this rank
    end: int     # one past the last
    rows: int    # rows every rank holds in the gathered layout (the largest shard)

    @property
    def size(self) -> int:
        return self.end - self.begin


def shard_rows(batch: int, world: int, rank: int) -> Shard:
    """Contiguous split of `batch` rows; the first batch % world ranks get one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if batch < 0:
        raise ValueError("batch must be non-negative")
    base, extra = divmod(batch, world)
    begin = rank * base + min(rank, extra)
    end = begin + base + (1 if rank < extra else 0)
    return Shard(rank, world, begin, end, base + (1 if extra else 0))


class ShardFailure(RuntimeError):
    """Raised on every rank when any rank's shard reported a failure."""


def agree_ok(local_flags: int, group=None, device=None) -> int:
    """MAX all-reduce of a failure word (0 = ok) so that all ranks see the same outcome."""
    t = torch.tensor([int(local_flags)], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return int(t.item())


def gather_batch(local: torch.Tensor, shard: Shard, batch: int, group=None) -> torch.Tensor:
    """All-gather batch shards (dim 0) into the full (batch, ...) tensor on every rank.

    Shards are padded to the largest shard for the collective and trimmed after.
    """
    if local.shape[0] != shard.size:
        raise ValueError("local tensor does not hold this rank's shard")
    padded = local
    if shard.size != shard.rows:
        padded = torch.zeros((shard.rows,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        padded[: shard.size] = local
    out = torch.empty((shard.rows * shard.world,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
    if shard.rows * shard.world == batch:
        return out
    parts = [out[r * shard.rows: r * shard.rows + shard_rows(batch, shard.world, r).size] for r in range(shard.world)]
    return torch.cat(parts, dim=0)


def run_sharded(scan_shard, batch: int, *, gather: bool = True, group=None, device=None):
    """Runs `scan_shard(shard) -> (y_local, flags)` on this rank's rows.

    Every rank then agrees on the failure word; on failure all ranks raise
    ShardFailure (no rank is left waiting in the gather), otherwise the full
    output is gathered (or the local shard returned when gather is False).
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    shard = shard_rows(batch, world, rank)
    try:
        y_local, flags = scan_shard(shard)
    except Exception:  # a rank that fails on the host still takes part in the agreement
        y_local, flags = None, 1 << 31
    if world > 1:
        flags = agree_ok(flags, group=group, device=device)
    if flags:
        raise ShardFailure(f"a shard reported failure flags {flags:#x}")
    if not gather or world == 1:
        return y_local
    return gather_batch(y_local, shard, batch, group=group)
