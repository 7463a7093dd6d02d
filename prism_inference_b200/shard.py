"""Frame sharding across GPUs (data parallelism over independent frames).

Each block of the stack mixes tokens only inside an 8x8 window of one frame
(split2_qkv_attn_d256.comp.glsl:25-33) and routes per token, so frames are
independent: a batch is split into contiguous frame ranges, one per rank, with the
weights replicated.  There is no exchange step on the data path; gathering the
outputs (if a caller wants them on one rank) happens after the forward.
"""
from __future__ import annotations

from typing import List, Tuple


def plan(total_frames: int, world_size: int) -> List[Tuple[int, int]]:
    """(first frame, frame count) per rank; counts differ by at most one."""
    if world_size < 1 or total_frames < 0:
        raise ValueError(f"plan({total_frames}, {world_size})")
    base, extra = divmod(total_frames, world_size)
    out, start = [], 0
    for r in range(world_size):
        n = base + (1 if r < extra else 0)
        out.append((start, n))
        start += n
    return out


def my_frames(total_frames: int, world_size: int, rank: int) -> Tuple[int, int]:
    if not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} of {world_size}")
    return plan(total_frames, world_size)[rank]


def gather_frames(local, total_frames: int, world_size: int, group=None):
    """All-gather every rank's [n_r, ...] frame slice into [total_frames, ...] on every
    rank (torch.distributed, any backend).  Ranks with fewer frames are padded for the
    collective and trimmed afterwards."""
    import torch
    import torch.distributed as dist
    p = plan(total_frames, world_size)
    n_max = max(n for _, n in p)
    pad = torch.zeros((n_max,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    # the collective moves bytes (every backend supports uint8), the caller's dtype is restored
    raw = pad.contiguous().view(torch.uint8)
    bufs = [torch.empty_like(raw) for _ in range(world_size)]
    dist.all_gather(bufs, raw, group=group)
    return torch.cat([b.view(local.dtype)[:n] for b, (_, n) in zip(bufs, p)], dim=0)
