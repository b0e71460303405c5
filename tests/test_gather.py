"""The gather of sampled ids to rank 0 over NVLink peer memory (d3s_gather):
one rank (the result equals the sampler's own ids), a wait for a rank that
never arrives, at a step's end or at a start line (it gives up with an error
the host reads, and the device stays usable), and two GPUs (each rank's
sampler writes its shard into rank 0's result; every step equals the oracle),
the last only where two GPUs exist."""

import os
import socket
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def d3s():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    import d3s as m
    return m


def test_gather_one_rank_equals_local_ids(d3s):
    import synth
    ctx = d3s.Context(0)
    g = d3s.Gather(0, 1, 0, 3000, lambda mine: mine)
    out = torch.empty(3000, dtype=torch.int32, device="cuda")
    want = torch.empty_like(out)
    for line in (1, 2):  # one rank reaches every start line at once
        g.line_up(line)
    for step in range(5):
        x, T, p, k, seeds = synth.c5_batch(3000, seed=40 + step)
        ctx.sample_rows(x, want, temperature=T, top_p=p, top_k=k, seeds=seeds)
        ptr = g.begin(step)
        ctx.sample_rows(x, ptr, temperature=T, top_p=p, top_k=k, seeds=seeds)
        g.end(step)
        g.copy_result(step, out)
        g.release(step)
        torch.cuda.synchronize()
        assert torch.equal(out, want), f"step {step}"
    g.check()
    g.close()
    ctx.close()


def test_gather_wait_for_a_missing_rank_gives_up(d3s):
    """Rank 0 of a world of 2 whose peer never starts: its wait for the peer's
    arrival runs out (5 s), the gather reports it, and the device still works."""
    import synth
    g = d3s.Gather(0, 2, 0, 64, lambda mine: mine)
    ptr = g.begin(0)
    ctx = d3s.Context(0)
    x, T, p, k, seeds = synth.c5_batch(64, seed=50)
    ctx.sample_rows(x, ptr, temperature=T, top_p=p, top_k=k, seeds=seeds)
    t0 = time.time()
    g.end(0)  # waits for rank 1's arrival, which never comes
    with pytest.raises(d3s.D3SError) as e:
        g.check()
    assert e.value.code == d3s.D3S_ERR_CUDA
    assert time.time() - t0 < 30
    g.check()  # reported once, then cleared
    ids = torch.empty(64, dtype=torch.int32, device="cuda")
    ctx.sample_rows(x, ids, temperature=T, top_p=p, top_k=k, seeds=seeds)
    ctx.check()
    g.close()
    ctx.close()


def test_start_line_without_the_other_rank_gives_up(d3s):
    """Rank 0 of a world of 2 at a start line its peer never reaches: the wait
    runs out (5 s), the gather reports it once, and the device still works."""
    import synth
    g = d3s.Gather(0, 2, 0, 64, lambda mine: mine)
    t0 = time.time()
    g.line_up(1)
    with pytest.raises(d3s.D3SError) as e:
        g.check()
    assert e.value.code == d3s.D3S_ERR_CUDA
    assert time.time() - t0 < 30
    g.check()
    ctx = d3s.Context(0)
    x, T, p, k, seeds = synth.c5_batch(64, seed=51)
    ids = torch.empty(64, dtype=torch.int32, device="cuda")
    ctx.sample_rows(x, ids, temperature=T, top_p=p, top_k=k, seeds=seeds)
    ctx.check()
    g.close()
    ctx.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gpu_gather_equals_oracle(d3s, oracle, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import synth
    rows, steps = 4097, 4
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES="0,1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "gather_worker.py"), str(tmp_path), str(rows), str(steps)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    for step in range(steps):
        x, T, p, k, seeds = synth.c5_batch(rows, seed=300 + step, V=2049)
        want = oracle.sample_rows(synth.to_host_logits(x), T.cpu().numpy(), p.cpu().numpy(),
                                  k.cpu().numpy(), seeds.cpu().numpy().astype(np.uint64))
        got = np.load(tmp_path / f"ids{step}.npy")
        assert (got == want).all(), f"step {step}: {int((got != want).sum())} ids differ"
