"""Chunk-sharded separation of one track over the GPUs of a node.

The reference separates a track chunk by chunk on one GPU
(src/inference_app.cpp:100-324).  Chunks carry no state between each other, so
here the chunk plan of the whole track is split into contiguous, balanced
ranges, one per rank; every rank runs its chunks (msst_model_forward_chunks),
the per-chunk stem outputs are gathered to rank 0 with one collective, and rank
0 overlap-adds all chunks in chunk order (msst_model_stitch).  The stitched
track is therefore the same as the single-GPU msst_model_separate result.

The compute functions are injectable so the sharding and gather logic can be
exercised with CPU tensors on a gloo process group.
"""
from __future__ import annotations


def shard(num_chunks: int, world: int, rank: int) -> tuple[int, int]:
    """(first chunk, count) of `rank`: contiguous ranges, sizes differing by at most one."""
    base, rem = divmod(num_chunks, world)
    count = base + (1 if rank < rem else 0)
    first = rank * base + min(rank, rem)
    return first, count


def max_shard(num_chunks: int, world: int) -> int:
    return -(-num_chunks // world)


class ShardedSeparator:
    """Separate one track with its chunks spread over the ranks of a process group.

    model:          msst_b200.Model on this rank's GPU (default compute), or None
    dist:           torch.distributed (initialised), or None for a single process
    forward_chunks: fn(track, overlap, first, count, chunk_batch, fix_tail_padding, out) -> out
    stitch:         fn(all_chunks, channels, length, overlap) -> [S, C, L] (S squeezed when 1)
    plan:           fn(length, overlap) -> dict(num_chunks=..., chunk_size=...)
    stems:          number of stems (from the model by default)
    """

    def __init__(self, model=None, dist=None, rank: int = 0, world: int = 1, forward_chunks=None, stitch=None,
                 plan=None, stems: int | None = None):
        self.model = model
        self.dist = dist
        self.rank = rank
        self.world = world
        self._forward = forward_chunks or (lambda track, overlap, first, count, cb, fix, out: model.forward_chunks(
            track, overlap, first, count, cb, fix, out=out))
        self._stitch = stitch or (lambda chunks, C, L, overlap: model.stitch(chunks, C, L, overlap))
        self._plan = plan or (lambda L, overlap: model.chunk_plan(L, overlap))
        self.stems = stems if stems is not None else model.info["num_stems"]

    def separate(self, track, overlap: float = 0.0, chunk_batch: int = 0, fix_tail_padding: bool = False):
        """track [C, L] (same on every rank) -> stems on rank 0, None on the other ranks."""
        import torch

        C, L = track.shape
        plan = self._plan(L, overlap)
        n, chunk = plan["num_chunks"], plan["chunk_size"]
        first, count = shard(n, self.world, self.rank)
        cap = max_shard(n, self.world)
        local = torch.zeros((cap, self.stems * C, chunk), dtype=torch.float32, device=track.device)
        if count:
            self._forward(track, overlap, first, count, chunk_batch, fix_tail_padding, local[:count])
        if self.world == 1:
            return self._stitch(local[:count], C, L, overlap)
        if self.rank == 0:
            bufs = [torch.empty_like(local) for _ in range(self.world)]
            self.dist.gather(local, bufs, dst=0)
            parts = [bufs[r][: shard(n, self.world, r)[1]] for r in range(self.world)]
            return self._stitch(torch.cat(parts, dim=0), C, L, overlap)
        self.dist.gather(local, dst=0)
        return None
