"""Request/batch sharding across ranks (one process per GPU).

Batch invariance makes every sample independent, so a batch is split into
contiguous row ranges, one per rank, with no collective on the compute path.
The collectives here (torch.distributed: NCCL on GPUs, gloo on CPU) only
serve measurement and verification: the max-over-ranks timing reduction, a
bitwise digest that must agree across ranks, and an optional gather of the
shards back to one tensor.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) rows of ``n`` owned by ``rank`` (sizes differ by
    at most one, lower ranks take the remainder)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} for world size {world}")
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """Maximum of a per-rank scalar (device time) over all ranks."""
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bit_digest(t: torch.Tensor) -> torch.Tensor:
    """Order-sensitive int64 digest of a tensor's bits (two sums of the 16-bit
    words, the second weighted by position), equal iff bit patterns match
    with overwhelming probability."""
    words = t.detach().contiguous().view(torch.int16).reshape(-1).to(torch.int64) & 0xFFFF
    pos = torch.arange(words.numel(), device=words.device, dtype=torch.int64) % 65521 + 1
    return torch.stack([words.sum(), (words * pos).remainder(2147483647).sum()])


def ranks_agree(digest: torch.Tensor) -> bool:
    """True when every rank holds the same digest."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return True
    gathered = [torch.empty_like(digest) for _ in range(dist.get_world_size())]
    dist.all_gather(gathered, digest)
    return all(torch.equal(gathered[0], g) for g in gathered)


def gather_rows(shard: torch.Tensor, n: int) -> torch.Tensor:
    """Reassemble the full ``n``-row tensor from every rank's contiguous shard
    (uneven shards are padded for the collective and trimmed)."""
    world = dist.get_world_size() if dist.is_initialized() else 1
    if world == 1:
        return shard
    longest = shard_range(n, world, 0)[1]
    padded = shard.new_zeros((longest, *shard.shape[1:]))
    padded[: shard.shape[0]] = shard
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded)
    rows = [parts[r][: shard_range(n, world, r)[1] - shard_range(n, world, r)[0]] for r in range(world)]
    return torch.cat(rows)
