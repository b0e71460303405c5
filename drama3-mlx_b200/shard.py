"""Row sharding for multi-GPU sampling (one process per GPU).

Rows are independent, so a batch of N rows is split into contiguous ranges,
rank r taking rows [r*N/G, (r+1)*N/G); each rank samples its own rows with its
own per-row seeds (a row's seed is its global row index's seed, so the result
does not depend on G), and the int32 ids are gathered to one rank. There is no
other exchange.

On the GPUs the gather is d3s.Gather (the library's d3s_gather): each rank's
sampler writes its ids straight into rank 0's result over NVLink, so no
collective runs per step; `handle_exchange` is the one-time channel that hands
rank 0's IPC handle to the other ranks. `gather_ids` is the same gather as one
torch.distributed collective (any process group: gloo with CPU tensors in the
tests).
"""

from __future__ import annotations


def shard_range(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    """The contiguous rows [start, stop) of `rank` among `world` ranks."""
    if world < 1 or not 0 <= rank < world or n_rows < 0:
        raise ValueError(f"bad shard: n_rows={n_rows} world={world} rank={rank}")
    return n_rows * rank // world, n_rows * (rank + 1) // world


def handle_exchange(group=None, src: int = 0):
    """The exchange function d3s.Gather takes: rank `src` passes its handle
    (bytes), the others None, and every rank gets the source's handle back
    (one broadcast of a Python object over the process group)."""
    import torch.distributed as dist

    def exchange(mine):
        obj = [mine]
        dist.broadcast_object_list(obj, src=src, group=group)
        if not isinstance(obj[0], (bytes, bytearray)):
            raise RuntimeError("rank 0 sent no gather handle")
        return bytes(obj[0])

    return exchange


def gather_ids(ids, n_rows: int, world: int, rank: int, dst: int = 0, group=None):
    """Gather each rank's ids (int32 tensor of its shard, in row order) to `dst`.

    Shards may differ in size by one row: each is padded to the largest before
    the collective and trimmed after. Returns the N ids on `dst`, None elsewhere.
    Every rank must call it (it is one collective)."""
    import torch
    import torch.distributed as dist

    start, stop = shard_range(n_rows, world, rank)
    if ids.numel() != stop - start:
        raise ValueError(f"rank {rank}: {ids.numel()} ids for shard [{start}, {stop})")
    if world == 1:
        return ids
    width = -(-n_rows // world)  # the largest shard
    buf = torch.full((width,), -1, dtype=ids.dtype, device=ids.device)
    buf[: ids.numel()] = ids
    parts = [torch.empty_like(buf) for _ in range(world)] if rank == dst else None
    dist.gather(buf, parts, dst=dst, group=group)
    if rank != dst:
        return None
    out = []
    for r, part in enumerate(parts):
        s, e = shard_range(n_rows, world, r)
        out.append(part[: e - s])
    return torch.cat(out)
