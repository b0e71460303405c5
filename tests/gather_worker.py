"""One rank of the two-GPU id-gather test (launched by tests/test_gather.py
under torch.distributed.run, one process per GPU): each rank samples its shard
of a seeded batch straight into rank 0's result through d3s.Gather, for
several steps with different seeds; rank 0 saves every step's gathered ids."""

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "drama3-mlx_b200"))


def main(out_dir: str, rows: int, steps: int) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    import d3s
    import shard
    import synth
    rank, world, local = (int(os.environ[k]) for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{local}"))
    try:
        ctx = d3s.Context(local)
        g = d3s.Gather(local, world, rank, rows, shard.handle_exchange())
        s, e = shard.shard_range(rows, world, rank)
        ids = torch.empty(rows, dtype=torch.int32, device="cuda")
        batches = [synth.c5_batch(rows, seed=300 + step, V=2049) for step in range(steps)]
        dist.barrier(device_ids=[local])
        g.line_up(1)  # both GPUs start the steps together
        for step, (x, T, p, k, seeds) in enumerate(batches):
            ptr = g.begin(step)
            ctx.sample_rows(x[s:e], ptr, temperature=T[s:e], top_p=p[s:e], top_k=k[s:e],
                            seeds=seeds[s:e])
            g.end(step)
            if rank == 0:
                g.copy_result(step, ids)
                np.save(Path(out_dir) / f"ids{step}.npy", ids.cpu().numpy())
            g.release(step)
        g.check()
        ctx.check()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        g.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], int(sys.argv[2]), int(sys.argv[3]))
