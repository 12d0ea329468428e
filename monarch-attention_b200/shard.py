"""Batch x heads sharding across ranks (one process per GPU).

Every (e, h) pair of MonarchAttention is independent (ma/ma_torch.py never
mixes heads or batch rows; the mask is per batch row), so the forward shards
with no collective on the data path.  These helpers split the flattened
E * H index space into contiguous ranges (whole batch rows first, so a rank's
mask rows stay local when E >= world), time as the max over ranks, and gather
output shards after timing for verification.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(E: int, H: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) range of flattened (e, h) indices for `rank`.

    Balanced to within one head; when E is a multiple of `world` the ranges
    are whole batch rows.
    """
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    total = E * H
    if E % world == 0:
        per = (E // world) * H
        return rank * per, (rank + 1) * per
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_problem(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask, scales,
                  world: int, rank: int):
    """This rank's heads of an (E, H) problem as a smaller (E', H') problem.

    Returns ``(q, k, v, mask, scales, (start, stop))`` with contiguous copies.
    When E is a multiple of ``world`` the shard is whole batch rows
    (E / world, H) with their mask rows; otherwise it is laid out as
    (stop - start, 1) heads, each with the mask row of its batch row, so any
    shard runs through the same operator unchanged.  ``scales`` (e4m3
    per-(e, h) factors, each (E, H)) follow the heads.
    """
    E, H = q.shape[:2]
    a, b = shard_range(E, H, world, rank)
    if world == 1:
        return q, k, v, mask, scales, (a, b)
    if E % world == 0:
        e0, e1 = a // H, b // H
        sl = lambda t: t[e0:e1].contiguous()
        return (sl(q), sl(k), sl(v), None if mask is None else sl(mask),
                None if scales is None else tuple(sl(s) for s in scales), (a, b))
    n = b - a
    fl = lambda t: t.reshape(E * H, *t.shape[2:])[a:b].unsqueeze(1).contiguous()
    m = None
    if mask is not None:
        m = mask[torch.arange(a, b, device=mask.device) // H].contiguous()
    sc = None if scales is None else tuple(s.reshape(E * H)[a:b].reshape(n, 1).contiguous()
                                           for s in scales)
    return fl(q), fl(k), fl(v), m, sc, (a, b)


def take_shard(x: torch.Tensor, start: int, stop: int) -> torch.Tensor:
    """Rows [start, stop) of the flattened (E*H) leading dims of x, as (1, n, ...)."""
    E, H = x.shape[:2]
    return x.reshape(E * H, *x.shape[2:])[start:stop].unsqueeze(0)


def shard_mask(mask: torch.Tensor | None, H: int, start: int, stop: int):
    """Mask rows matching take_shard's heads: one (E, N) row per (e, h)."""
    if mask is None:
        return None
    e_idx = torch.arange(start, stop, device=mask.device) // H
    return mask[e_idx].unsqueeze(0).expand(1, stop - start, -1)


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (e.g. elapsed ms) over all ranks."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_shards(shard: torch.Tensor, E: int, H: int) -> torch.Tensor:
    """All-gather per-rank (E', H', N, D) output shards (E' * H' = the rank's
    head count) into the full (E, H, N, D) output on every rank."""
    world = dist.get_world_size()
    sizes = [shard_range(E, H, world, r) for r in range(world)]
    flat = shard.reshape(shard.shape[0] * shard.shape[1], *shard.shape[2:])
    maxn = max(b - a for a, b in sizes)
    pad = torch.zeros((maxn, *flat.shape[1:]), dtype=flat.dtype, device=flat.device)
    pad[: flat.shape[0]] = flat
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad)
    parts = [bufs[r][: b - a] for r, (a, b) in enumerate(sizes)]
    return torch.cat(parts).reshape(E, H, *flat.shape[1:])
