"""Request sharding across GPUs (one process per GPU, no per-step collective).

Every quantity of the select step is per request (``log_prior`` is
replicated), so rank r owns the contiguous request range
``[r*B/G, (r+1)*B/G)`` (the reference scales the same way: one worker process
per GPU behind a router, ``server/serve.py:1-5``).  The only collective is a
final gather of the committed block tokens.
"""
from __future__ import annotations

import torch


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous ``[lo, hi)`` of ``total`` requests for ``rank`` (sizes differ by at most one)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("bad world/rank")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_committed(xt_local: torch.Tensor, total: int, dist) -> torch.Tensor | None:
    """All-gather every rank's ``(B_local, L)`` committed tokens into ``(total, L)``
    int32 token ids (speech ids and MASK are below 2^31).

    Shards may be ragged; they are padded to the largest shard for the
    collective and trimmed afterwards.  Returns the full tensor on every rank.
    """
    world = dist.get_world_size()
    L = xt_local.shape[1]
    sizes = [shard_range(total, world, r)[1] - shard_range(total, world, r)[0] for r in range(world)]
    mx = max(sizes)
    pad = torch.full((mx, L), -1, dtype=torch.int32, device=xt_local.device)
    pad[: xt_local.shape[0]] = xt_local.to(torch.int32)
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    return torch.cat([p[:n] for p, n in zip(parts, sizes)], dim=0)
