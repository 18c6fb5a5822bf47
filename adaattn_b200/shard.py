"""(batch x head) sharding of the attention path across ranks.

The (b, h) slices of one call are independent, so a job splits into
contiguous ranges of slices, one per rank, with no collective inside the
attention itself. Two host-side exchange steps exist:

* ``gather_slices`` -- all-gather of the per-rank outputs (the multi-GPU
  bench times it separately);
* ``global_decision`` -- the reference's single per-call decision
  (src/adaattn/attention/adaattn.py:262-289) when the slices live on several
  ranks: one all-reduce of {sum of normalised row entropies, row count,
  max |score|, max prob} followed by the same ladder on every rank.
"""

from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.distributed as dist


def shard_range(n_units: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous, balanced [start, stop) of n_units for this rank."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def local_slices(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's (b, h) slices of x [B, H, N, D] as a [1, n_local, N, D] view
    (requires the B and H strides to flatten, e.g. a contiguous tensor)."""
    b, h, n, d = x.shape
    start, stop = shard_range(b * h, rank, world)
    flat = x.reshape(b * h, n, d)
    return flat[start:stop].unsqueeze(0)


def gather_slices(local: torch.Tensor, batch: int, heads: int, group=None) -> torch.Tensor:
    """All-gather every rank's [1, n_local, N, D] slices into [B, H, N, D]."""
    world = dist.get_world_size(group)
    n, d = local.shape[2], local.shape[3]
    total = batch * heads
    counts = [shard_range(total, r, world) for r in range(world)]
    width = max(stop - start for start, stop in counts)
    buf = torch.zeros(1, width, n, d, dtype=local.dtype, device=local.device)
    buf[:, :local.shape[1]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    pieces = [p[0, :stop - start] for p, (start, stop) in zip(parts, counts)]
    return torch.cat(pieces, dim=0).view(batch, heads, n, d)


def _round_like(x: float, dtype: torch.dtype) -> float:
    return float(torch.tensor(x, dtype=torch.float32).to(dtype).float())


def global_decision(head_sum: torch.Tensor, head_stats: torch.Tensor, sample_rows: int,
                    min_seq: int, dtype: torch.dtype, *, rank_threshold: float = 0.95,
                    enable_adaptive_rank: bool = True, enable_adaptive_precision: bool = True,
                    default_precision: int = 1, allow_fp8: bool = False, group=None) -> dict:
    """The reference's per-call decision over slices spread across ranks.

    head_sum [n_local]: per-slice sum of normalised row entropies (the
    analyzer's scratch); head_stats [..., 4]: per-slice statistics.
    """
    local = torch.stack([
        head_sum.double().sum(),
        torch.tensor(float(head_sum.numel() * sample_rows), dtype=torch.float64,
                     device=head_sum.device),
    ])
    maxima = head_stats.reshape(-1, 4)[:, 1:3].double().amax(dim=0) if head_stats.numel() else \
        torch.zeros(2, dtype=torch.float64, device=head_sum.device)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(local, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(maxima, op=dist.ReduceOp.MAX, group=group)
    total, count = float(local[0]), float(local[1])
    ne = _round_like(float(torch.tensor(total, dtype=torch.float32) / count), dtype)
    max_score, max_prob = float(maxima[0]), float(maxima[1])
    low = bool(enable_adaptive_rank and ne < rank_threshold)
    if max_score > 50.0 or max_prob > 0.95:
        prec = 0
    elif ne > 0.8:
        prec = 3 if allow_fp8 else 1
    elif ne < 0.3:
        prec = 2
    else:
        prec = default_precision
    if not enable_adaptive_precision:
        prec = default_precision
    return {"low_rank": low, "precision": prec, "ne": ne, "max_score": max_score,
            "max_prob": max_prob, "effective_rank": ne * min_seq,
            "sample_rows": sample_rows, "log_s": math.log(sample_rows)}
