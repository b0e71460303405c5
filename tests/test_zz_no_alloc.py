"""The entry point that allocates nothing (d3s_sample_rows_static), for callers
that cannot call cudaMalloc while they sample (budgeted serving engines,
real-time threads, code inside a stream capture). Its results must equal the
allocating entry point's (d3s_sample with per-row seeds) on two calls in a row,
which also shows the shared scratch starts each call clean. This file is
collected last, so a stop-at-first-failure run has run every other test."""

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_static_scratch_entry_point_matches_allocating_one():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    import d3s
    import synth
    ctx = d3s.Context(0)
    for call, (rows, seed) in enumerate([(3000, 21), (4096, 22)]):
        x, T, p, k, seeds = synth.c5_batch(rows, seed=seed)
        k[::97] = 300  # some rows take the wide kernel through the hand-off list
        want = torch.empty(rows, dtype=torch.int32, device="cuda")
        got = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
        ctx.sample_rows(x, want, temperature=T, top_p=p, top_k=k, seeds=seeds)
        d3s.sample_rows_static(x, got, T, p, k, seeds)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call}: {(got != want).sum().item()} rows differ"
    too_many = torch.zeros(d3s.STATIC_MAX_ROWS + 1, 8, device="cuda")
    one = torch.ones(d3s.STATIC_MAX_ROWS + 1, device="cuda")
    with pytest.raises(d3s.D3SError) as e:
        d3s.sample_rows_static(too_many, torch.empty(d3s.STATIC_MAX_ROWS + 1, dtype=torch.int32,
                                                     device="cuda"),
                               one, one, one.int(), one.long(), None)
    assert e.value.code == d3s.D3S_ERR_UNSUPPORTED
    ctx.close()
