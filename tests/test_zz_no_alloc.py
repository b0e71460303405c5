"""The entry point that allocates nothing (d3s_sample_rows_static), for callers
that cannot call cudaMalloc while they sample: a serving engine that budgets
every device byte before it serves, or a real-time audio thread that cannot
wait on cudaMalloc's implicit device synchronisation. Its results must equal
the allocating entry point's (d3s_sample with per-row seeds) on two calls in a
row, which also shows the shared scratch starts each call clean; a call must
leave the device's free memory unchanged; and a failure recorded in the
scratch's error word must reach the caller through d3s_static_check. This file
is collected last, so a stop-at-first-failure run has run every other test."""

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def d3s():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    import d3s as m
    return m


def test_static_scratch_entry_point_matches_allocating_one(d3s):
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
    d3s.static_check()
    too_many = torch.zeros(d3s.STATIC_MAX_ROWS + 1, 8, device="cuda")
    one = torch.ones(d3s.STATIC_MAX_ROWS + 1, device="cuda")
    with pytest.raises(d3s.D3SError) as e:
        d3s.sample_rows_static(too_many, torch.empty(d3s.STATIC_MAX_ROWS + 1, dtype=torch.int32,
                                                     device="cuda"),
                               one, one, one.int(), one.long(), None)
    assert e.value.code == d3s.D3S_ERR_UNSUPPORTED
    ctx.close()


def test_static_call_leaves_free_device_memory_unchanged(d3s):
    """Once the kernels it runs have been loaded (a first identical call), a
    call changes nothing in the device's free memory."""
    import synth
    x, T, p, k, seeds = synth.c5_batch(2048, seed=23)
    ids = torch.empty(2048, dtype=torch.int32, device="cuda")
    d3s.sample_rows_static(x, ids, T, p, k, seeds)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        d3s.sample_rows_static(x, ids, T, p, k, seeds)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    d3s.static_check()


def test_static_error_word_reaches_the_caller(d3s):
    """A recorded failure is set through the test hook (no copy is stalled):
    it survives a later call (the word is sticky), d3s_static_check reports it
    once and clears it."""
    import synth
    d3s.static_check()  # starts clean
    x, T, p, k, seeds = synth.c5_batch(64, seed=24)
    ids = torch.empty(64, dtype=torch.int32, device="cuda")
    d3s.static_debug_set_error(1)
    d3s.sample_rows_static(x, ids, T, p, k, seeds)
    with pytest.raises(d3s.D3SError) as e:
        d3s.static_check()
    assert e.value.code == d3s.D3S_ERR_CUDA
    d3s.static_check()  # cleared by the check that reported it
    d3s.sample_rows_static(x, ids, T, p, k, seeds)
    d3s.static_check()
