"""Windows across GPUs: one process per GPU, no collective on the data path.

The 30 s windows of a batch are independent sequences, so a batch shards by
window: every rank holds a full weight replica and decodes a contiguous range
of windows with its own caches.  The only cross-rank traffic is host-side
bookkeeping -- the slowest rank's time, and the transcripts gathered back in
window order -- through torch.distributed (NCCL between GPUs, gloo on CPU).
"""
from __future__ import annotations

import numpy as np


def window_range(total: int, rank: int, world: int) -> range:
    """The contiguous windows rank `rank` of `world` decodes: the first
    total % world ranks take one window more than the rest."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is outside a world of {world}")
    if total < 0:
        raise ValueError("the window count must not be negative")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def max_over_ranks(values, device=None) -> list[float]:
    """Element-wise maximum of per-rank values (milliseconds) over every rank
    of the default process group; the values themselves with one rank."""
    import torch
    import torch.distributed as dist
    values = [float(v) for v in values]
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return values
    t = torch.tensor(values, dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def gather_transcripts(local: list[np.ndarray], total: int) -> list[np.ndarray] | None:
    """Every rank's transcripts, in window order, on rank 0 (None elsewhere)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(local)
    rank, world = dist.get_rank(), dist.get_world_size()
    mine = window_range(total, rank, world)
    if len(local) != len(mine):
        raise ValueError(f"rank {rank} holds {len(local)} transcripts for {len(mine)} windows")
    parts = [None] * world if rank == 0 else None
    dist.gather_object([np.asarray(t, dtype=np.uint32).tolist() for t in local], parts, dst=0)
    if rank != 0:
        return None
    return [np.asarray(t, dtype=np.uint32) for part in parts for t in part]


def transcribe_windows(decoder_factory, encoder_rows: np.ndarray, cross_positions: int = 0):
    """Decodes this rank's share of a window batch and gathers every
    transcript on rank 0.  decoder_factory(windows) returns a Decoder for
    that many windows on this rank's GPU, generation config already set."""
    import torch.distributed as dist
    ready = dist.is_available() and dist.is_initialized()
    rank, world = (dist.get_rank(), dist.get_world_size()) if ready else (0, 1)
    total = encoder_rows.shape[0]
    mine = window_range(total, rank, world)
    local: list[np.ndarray] = []
    if len(mine):
        decoder = decoder_factory(len(mine))
        try:
            local = decoder.transcribe(np.ascontiguousarray(encoder_rows[mine.start:mine.stop]), cross_positions)
        finally:
            decoder.close()
    return gather_transcripts(local, total)
