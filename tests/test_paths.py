"""Every kernel path that samples batches above the small-batch path (the
four-warp streaming stats kernel with the select kernel, the row-warp kernel
of one warp per row, the one-warp streaming stats kernel with the select
kernel) against the oracle on the same rows: forced in turn through the
d3s_debug_force_path test hook. Ids, kept counts, statuses and the bits of
the race probabilities must be identical on every path."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

PATHS = [("pair", 1), ("rowwarp", 3), ("pair1w", 4)]


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    import d3s
    c = d3s.Context(0)
    yield c
    d3s.force_path(0)
    c.close()


@pytest.fixture(params=PATHS, ids=[p[0] for p in PATHS])
def path(request, ctx):
    import d3s
    d3s.force_path(request.param[1])
    yield request.param[0]
    d3s.force_path(0)


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(x):
    import synth
    return synth.to_host_logits(x)


def rows_batch(N, V, seed, scale=3.0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((N, V)) * scale).astype(np.float32)
    T = rng.uniform(0.5, 1.2, N).astype(np.float32)
    p = rng.uniform(0.5, 1.0, N).astype(np.float32)
    k = rng.integers(1, 65, N).astype(np.int32)
    seeds = np.arange(N, dtype=np.int64) * 7 + seed
    return x, T, p, k, seeds


@pytest.mark.parametrize("dtype,V,N", [("f32", 4097, 3000), ("bf16", 4097, 3000), ("f32", 2049, 2600),
                                        ("f32", 3000, 2600), ("bf16", 6000, 2600)])
def test_per_row_params_equal_oracle(ctx, oracle, path, dtype, V, N):
    x, T, p, k, seeds = rows_batch(N, V, V + N)
    xt = dev(x, torch.bfloat16 if dtype == "bf16" else torch.float32)
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    kept = torch.empty_like(ids)
    status = torch.empty_like(ids)
    ctx.sample_rows(xt, ids, temperature=dev(T), top_p=dev(p), top_k=dev(k), seeds=dev(seeds),
                    kept=kept, status=status)
    want = oracle.sample_rows(host(xt), T, p, k, seeds.astype(np.uint64))
    got = ids.cpu().numpy()
    assert (got == want).all(), f"{path}: {int((got != want).sum())} of {N} rows differ"
    assert (status.cpu().numpy() == 0).all()
    ctx.check()


def test_diagnostics_and_uncertain_cuts(ctx, oracle, path):
    """Given noise with every diagnostic output, and top_p placed exactly on a
    cumsum of half of the rows (or one float below it), so the approximate
    sum cannot certify the cut and the exact sum decides."""
    import d3s
    rng = np.random.default_rng(31)
    N, V, k = 2600, 4097, 40
    x = (rng.standard_normal((N, V)) * 3).astype(np.float32)
    T = rng.uniform(0.5, 1.2, N).astype(np.float32)
    p = rng.uniform(0.5, 1.0, N).astype(np.float32)
    for i, r in enumerate(range(0, N, 2)):
        cums = oracle.row_cums(x[r], float(T[r]), k)
        c = np.float32(cums[int(rng.integers(1, k))])
        p[r] = c if i % 2 == 0 else np.nextafter(c, np.float32(0.0))
    u = rng.random((N, k), dtype=np.float32)
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    kept, status = torch.empty_like(ids), torch.empty_like(ids)
    probs = torch.zeros(N, k, dtype=torch.float32, device="cuda")
    topk = torch.zeros(N, k, dtype=torch.int32, device="cuda")
    req = ctx.request(dev(x), ids, temperature_rows=dev(T), top_p_rows=dev(p), top_k=k,
                      noise=d3s.NOISE_GIVEN, u=dev(u), status=status, kept=kept, probs=probs,
                      topk_ids=topk)
    ctx.sample(req)
    got_ids, got_kept, got_probs = ids.cpu().numpy(), kept.cpu().numpy(), probs.cpu().numpy()
    got_topk = topk.cpu().numpy()
    for r in range(N):
        rid, otk, oprobs, d = oracle.sample_row(x[r], float(T[r]), float(p[r]), k, u[r])
        assert got_ids[r] == rid and got_kept[r] == d.kept, (path, r)
        assert got_topk[r].tolist() == otk.tolist(), (path, r)
        assert got_probs[r].view(np.uint32).tolist() == oprobs.view(np.uint32).tolist(), (path, r)
    ctx.check()


def test_rows_outside_the_approximate_path_and_flags(ctx, oracle, path):
    """k in 129..256 (exact per-element path), k above 256 (handed to the wide
    kernel), T above 2^20, |x| above 2^60, NaN / +inf / all -inf rows
    (flagged), bad parameters (flagged)."""
    rng = np.random.default_rng(23)
    N, V = 2600, 4097
    x, T, p, k, seeds = rows_batch(N, V, 23)
    k[::5] = rng.integers(129, 257, len(k[::5]))
    k[2::13] = rng.integers(257, 2000, len(k[2::13]))
    T[1::7] = 2.0 ** 21
    x[3::11] *= np.float32(2.0 ** 61)
    x[4::97, 5] = np.nan
    x[6::101, 9] = np.inf
    x[8::103] = -np.inf
    k[10::107] = 0
    xt = dev(x)
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    status = torch.empty_like(ids)
    ctx.sample_rows(xt, ids, temperature=dev(T), top_p=dev(p), top_k=dev(k), seeds=dev(seeds),
                    status=status)
    want = oracle.sample_rows(x, T, p, k, seeds.astype(np.uint64))
    got = ids.cpu().numpy()
    assert (got == want).all(), f"{path}: rows {np.flatnonzero(got != want)[:10]}"
    st = status.cpu().numpy()
    assert (st[want == -1] != 0).all() and (st[want != -1] == 0).all()
    ctx.check()


@pytest.mark.parametrize("off", [1, 3])
def test_strided_unaligned_rows_and_ties(ctx, oracle, path, off):
    """Rows at element offsets that are not 16-byte aligned (ld = V + off), and
    rows of few distinct values (more candidates than a list holds)."""
    rng = np.random.default_rng(40 + off)
    N, V = 2600, 4097
    x, T, p, k, seeds = rows_batch(N, V, 40 + off)
    x[::17] = np.round(x[::17])
    x[5::19] = 1.0
    buf = np.zeros((N, V + off), np.float32)
    buf[:, :V] = x
    xt = dev(buf)[:, :V]
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    ctx.sample_rows(xt, ids, temperature=dev(T), top_p=dev(p), top_k=dev(k), seeds=dev(seeds))
    want = oracle.sample_rows(x, T, p, k, seeds.astype(np.uint64))
    got = ids.cpu().numpy()
    assert (got == want).all(), f"{path}: rows {np.flatnonzero(got != want)[:10]}"
    ctx.check()


def test_masked_rows_with_fewer_finite_logits_than_k(ctx, oracle, path):
    """Rows masked to a few finite logits (the rest -inf), fewer than k: the
    top k reaches into the -inf entries (ranked by id), which must not change
    the draw or the kept count."""
    rng = np.random.default_rng(51)
    N, V = 2600, 4097
    x, T, p, k, seeds = rows_batch(N, V, 51)
    for r in range(0, N, 9):
        keep = rng.choice(V, int(rng.integers(1, 20)), replace=False)
        row = np.full(V, -np.inf, np.float32)
        row[keep] = x[r, keep]
        x[r] = row
        k[r] = int(rng.integers(20, 65))
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    kept = torch.empty_like(ids)
    ctx.sample_rows(dev(x), ids, temperature=dev(T), top_p=dev(p), top_k=dev(k), seeds=dev(seeds),
                    kept=kept)
    want = oracle.sample_rows(x, T, p, k, seeds.astype(np.uint64))
    got = ids.cpu().numpy()
    assert (got == want).all(), f"{path}: rows {np.flatnonzero(got != want)[:10]}"
    ctx.check()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_tied_top_values(ctx, oracle, path, dtype):
    """Rows whose largest values repeat (the max at up to four ids, the next
    values twice or three times): the drawn rank often falls in a group of equal
    values, whose ranks go to increasing ids."""
    rng = np.random.default_rng(61)
    N, V = 2600, 4097
    x, T, p, k, seeds = rows_batch(N, V, 61)
    for r in range(N):
        order = np.argsort(-x[r])
        for t in range(int(rng.integers(1, 6))):
            src = order[t]
            dst = rng.choice(V, int(rng.integers(1, 4)), replace=False)
            x[r, dst] = x[r, src]
    T[::3] = 0.05  # sharp rows: the draw lands on the top values
    xt = dev(x, torch.bfloat16 if dtype == "bf16" else torch.float32)
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    kept = torch.empty_like(ids)
    ctx.sample_rows(xt, ids, temperature=dev(T), top_p=dev(p), top_k=dev(k), seeds=dev(seeds),
                    kept=kept)
    want = oracle.sample_rows(host(xt), T, p, k, seeds.astype(np.uint64))
    got = ids.cpu().numpy()
    assert (got == want).all(), f"{path}: rows {np.flatnonzero(got != want)[:10]}"
    ctx.check()
