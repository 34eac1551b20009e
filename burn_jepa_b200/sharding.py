"""Stream sharding for one process per GPU.

The front end's units are independent video streams that share nothing but the read-only
patch-embed weight, so a multi-GPU job partitions streams across ranks and runs no
collective on the data path.  Each global stream has its own seed and its own token cache,
so a stream's results do not depend on how many ranks the job has or which rank owns it.
The only collectives are on the measurement path: the max over ranks of the timed region
and the sums of the units processed.
"""
from __future__ import annotations

from typing import Optional

_SEED_MIX = 0x9E3779B97F4A7C15


def shard_streams(total_streams: int, world: int, rank: int) -> range:
    """Global stream ids owned by `rank`: contiguous blocks, the first `total % world` ranks
    taking one more stream each."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if total_streams < 0:
        raise ValueError("stream count must be non-negative")
    base, extra = divmod(total_streams, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def stream_seed(base_seed: int, stream: int) -> int:
    """Seed of one global stream's synthetic input, independent of the rank layout."""
    return (int(base_seed) * 1_000_003 + (int(stream) + 1) * _SEED_MIX) & ((1 << 63) - 1)


class RankGroup:
    """Rank/world view and the scalar reductions of the measurement path.  With world 1 (or
    no process group) every reduction is the identity, so single-GPU runs need no group."""

    def __init__(self, device=None):
        import torch.distributed as dist

        self._dist = dist
        self.active = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size() if self.active else 1
        self.rank = dist.get_rank() if self.active else 0
        backend = dist.get_backend() if self.active else None
        # NCCL reduces device tensors; gloo host tensors
        self.device = device if backend == "nccl" else "cpu"

    def _reduce(self, value: float, op) -> float:
        if self.world == 1:
            return float(value)
        import torch

        t = torch.tensor([float(value)], dtype=torch.float64, device=self.device)
        self._dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, value: float) -> float:
        return self._reduce(value, self._dist.ReduceOp.MAX) if self.world > 1 else float(value)

    def sum(self, value: float) -> float:
        return self._reduce(value, self._dist.ReduceOp.SUM) if self.world > 1 else float(value)

    def barrier(self) -> None:
        if self.world > 1:
            self._dist.barrier()

    def broadcast_object(self, obj, src: int = 0):
        """`obj` of rank `src` on every rank."""
        if self.world == 1:
            return obj
        box = [obj]
        self._dist.broadcast_object_list(box, src=src)
        return box[0]

    def gather_objects(self, obj) -> Optional[list]:
        """Every rank's `obj`, in rank order (all ranks receive the list)."""
        if self.world == 1:
            return [obj]
        out = [None] * self.world
        self._dist.all_gather_object(out, obj)
        return out
