"""The multi-GPU path's host logic on CPU: rows sharded over ranks, each rank
samples its own shard (here with the CPU oracle as the per-rank sampler), the
ids are gathered to rank 0 over a gloo process group of world size 2 and 3.
The gathered ids must equal one process sampling every row."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
ROOT = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def batch(N, V=1024, seed=5):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((N, V)) * 3.0).astype(np.float32)
    T = rng.uniform(0.5, 1.2, N).astype(np.float32)
    p = rng.uniform(0.5, 1.0, N).astype(np.float32)
    k = rng.integers(1, 65, N).astype(np.int32)
    seeds = (np.arange(N) + 1000).astype(np.uint64)  # a row's seed follows its global index
    return x, T, p, k, seeds


def _rank_main(rank, world, port, N, out_path):
    for p in (ROOT / "oracle", ROOT / "drama3-mlx_b200"):
        sys.path.insert(0, str(p))
    import torch.distributed as dist

    import oracle
    import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, T, p, k, seeds = batch(N)
        s, e = shard.shard_range(N, world, rank)
        ids = oracle.sample_rows(x[s:e], T[s:e], p[s:e], k[s:e], seeds[s:e], nthreads=1) \
            if e > s else np.zeros(0, np.int32)
        got = shard.gather_ids(torch.from_numpy(np.ascontiguousarray(ids, np.int32)), N, world, rank)
        if rank == 0:
            np.save(out_path, got.numpy())
        else:
            assert got is None
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,N", [(2, 300), (2, 301), (3, 100), (2, 1)])
def test_sharded_sampling_gathers_to_rank0(oracle, tmp_path, world, N):
    import torch.multiprocessing as mp
    out = tmp_path / "ids.npy"
    mp.spawn(_rank_main, args=(world, free_port(), N, str(out)), nprocs=world, join=True)
    x, T, p, k, seeds = batch(N)
    want = oracle.sample_rows(x, T, p, k, seeds)
    np.testing.assert_array_equal(np.load(out), want)


def test_shard_range_covers_rows_once():
    import shard
    for N in (0, 1, 7, 64, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            spans = [shard.shard_range(N, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == N
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and b - a >= d - c - 1 and d - c >= b - a - 1
    with pytest.raises(ValueError):
        shard.shard_range(10, 2, 2)


def _exchange_main(rank, world, port, out_path):
    for p in (ROOT / "drama3-mlx_b200",):
        sys.path.insert(0, str(p))
    import torch.distributed as dist

    import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        handle = bytes(range(64)) if rank == 0 else None
        got = shard.handle_exchange()(handle)
        Path(f"{out_path}.{rank}").write_bytes(got)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_handle_reaches_every_rank(tmp_path, world):
    """The one-time exchange of rank 0's 64-byte IPC handle that the NVLink id
    gather needs: every rank receives rank 0's bytes unchanged."""
    import torch.multiprocessing as mp
    out = tmp_path / "handle"
    mp.spawn(_exchange_main, args=(world, free_port(), str(out)), nprocs=world, join=True)
    for r in range(world):
        assert Path(f"{out}.{r}").read_bytes() == bytes(range(64))
