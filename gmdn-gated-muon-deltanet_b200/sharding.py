"""Host-side sharding of the scan over (batch, head) across ranks.

Every (b, h) sequence is independent (fast_scan.py:72-95 loops over chunks
per (b, h) only), so a multi-GPU run splits the flattened B*H axis into
contiguous shards, one per rank, with no data-path collective.  The only
communication is the timing reduction (max over ranks).
"""

from __future__ import annotations

import torch


def shard_bh(total_bh: int, rank: int, world: int) -> tuple[int, int]:
    """[start, end) of rank's contiguous share of total_bh sequences; shares
    differ by at most one and cover the range exactly."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(total_bh, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def slice_heads(t: torch.Tensor, start: int, end: int) -> torch.Tensor:
    """View of the (B*H)-flattened slice [start, end) of a (B, H, ...) tensor,
    shaped (1, end - start, ...)."""
    B, H = t.shape[:2]
    return t.reshape(B * H, *t.shape[2:])[start:end].unsqueeze(0)


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """Max of a per-rank float over the default process group (identity when
    no group is initialised)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return value
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
