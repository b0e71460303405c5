"""CUDA sampler vs the CPU oracle, through the C ABI (libd3s.so). Ids, kept
counts, ranked ids and probabilities must be bit-identical; the only tolerance
in this file is the statistical one of the distribution test."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    import d3s
    c = d3s.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def synth():
    import synth as s
    return s


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host_logits(x):
    import synth
    return synth.to_host_logits(x)


# ---- arithmetic ----

def float_range(lo_bits, hi_bits, stride):
    return np.arange(lo_bits, hi_bits, stride, dtype=np.uint64).astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("op,name", [(0, "exp"), (1, "log"), (2, "term")])
def test_math_bitwise(ctx, oracle, op, name):
    if name == "exp":  # every 7th float in [-104, 89] plus the edges
        xs = [float_range(0x80000000, 0xC2D00001, 7), float_range(0x00000000, 0x42B20001, 7)]
    elif name == "log":  # every 7th positive float, subnormals included
        xs = [float_range(0x00000001, 0x7F800001, 7)]
    else:  # every 3rd float in [-110, 0], dense around the -86 floor
        xs = [float_range(0x80000000, 0xC2DC0001, 3), np.linspace(-88.5, -86.5, 2_000_001).astype(np.float32)]
    extra = np.array([0.0, -0.0, 1.0, -1.0, -np.inf, 88.0, -86.33654, -86.33655, 1e-30, 3e38],
                     np.float32)
    x = np.concatenate(xs + [extra])
    if name == "term":
        x = -np.abs(x)
    ref = {"exp": oracle.exp, "log": oracle.log, "term": oracle.exp_term}[name]
    for chunk in np.array_split(x, max(1, len(x) // (1 << 24))):
        got = ctx.debug_math(op, dev(chunk)).cpu().numpy()
        want = ref(chunk)
        same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
        if not same.all():
            bad = np.flatnonzero(~same)[:5]
            pytest.fail(f"{name}: {len(np.flatnonzero(~same))} mismatches, e.g. "
                        f"{[(float(chunk[i]), float(got[i]), float(want[i])) for i in bad]}")


def test_reciprocal_division_is_ieee(ctx):
    """The stats kernel divides by a per-row reciprocal with one correction step
    when the row's range allows it; that quotient must equal the IEEE one for
    every float x with |x| in [2^-100, 2^60]: all 2^32 bit patterns for 64
    temperatures, every 61st pattern for 1024 more, T in [2^-17, 2^20]."""
    rng = np.random.default_rng(12)
    special = np.array([1e-5, 0.5, 0.7, 1.0, 1.2, 2.0 ** -17, 2.0 ** 20, 3.0, 1 / 3, 0.1, 10.0,
                        np.float32(1) - np.float32(2 ** -24), 2 - 2 ** -23, 1 + 2 ** -23, 1.5, 0.3],
                       np.float32)
    special = np.concatenate([special, np.array([0x3f7fffff, 0x3fffffff, 0x3effffff, 0x497fffff,
                                                 0x3f000001], np.uint32).view(np.float32)])
    full = np.concatenate([special, rng.uniform(0.5, 1.2, 64 - len(special)).astype(np.float32)])
    bad, ex = ctx.debug_div_check(torch.from_numpy(full).cuda())
    assert bad == 0, ex
    more = np.concatenate([rng.uniform(0.5, 1.2, 512), np.exp(rng.uniform(np.log(2.0 ** -17), np.log(2.0 ** 20), 512))])
    bad, ex = ctx.debug_div_check(torch.from_numpy(more.astype(np.float32)).cuda(), step=61)
    assert bad == 0, ex


@pytest.mark.parametrize("rows,V,top_k", [(1, 4097, 30), (3, 4097, 5), (7, 1024, 31), (256, 4097, 30),
                                          (1000, 100, 64), (5, 3, 30)])
def test_sample_noise_equals_oracle_uniform(ctx, oracle, rows, V, top_k):
    import d3s
    state = d3s.key_from_seed(rows * 1000 + top_k)
    ostate = oracle.key_from_seed(rows * 1000 + top_k)
    for _ in range(3):
        u = ctx.sample_noise(rows, V, top_k, state).cpu().numpy()
        want = oracle.uniform(oracle.next_key(ostate), rows * min(top_k, V)).reshape(rows, -1)
        assert np.array_equal(u, want)
    assert state.tolist() == ostate.tolist()


# ---- the reference's test entry point ----

def test_d3_sample_equals_oracle_and_golden(oracle):
    import d3s
    from pathlib import Path
    g = np.load(Path(__file__).resolve().parent / "golden" / "oracle_cases.npz")
    for pi, (T, k, p) in enumerate(g["d3_params"]):
        for s in range(4):
            ids = d3s.sample(g["d3_logits"], float(T), int(k), float(p), s)
            assert ids.tolist() == g["d3_ids"][pi, s].tolist()
        for s in range(4, 24):
            assert (d3s.sample(g["d3_logits"], float(T), int(k), float(p), s).tolist()
                    == oracle.d3_sample(g["d3_logits"], float(T), int(k), float(p), s).tolist())


def test_d3_sample_status_follows_each_call(oracle):
    """A call of N = 8 rows, then N = 1: each call's status belongs to its own
    rows (a smaller call must not read the larger call's ids as statuses)."""
    import d3s
    rng = np.random.default_rng(5)
    big = (rng.standard_normal((8, 4097)) * 3).astype(np.float32)
    big[:, 7] = 1e9  # large, finite: ids the status words must not be confused with
    d3s.sample(big, 0.7, 30, 0.7, 1)
    assert d3s.last_status() == d3s.D3S_OK
    one = (rng.standard_normal((1, 4097)) * 3).astype(np.float32)
    ids = d3s.sample(one, 0.7, 30, 0.7, 2)
    assert d3s.last_status() == d3s.D3S_OK
    assert ids.tolist() == oracle.d3_sample(one, 0.7, 30, 0.7, 2).tolist()
    bad = one.copy()
    bad[0, 3] = np.nan
    assert d3s.sample(bad, 0.7, 30, 0.7, 3).tolist() == [-1]
    assert d3s.last_status() == d3s.D3S_ERR_NONFINITE
    d3s.sample(one, 0.7, 30, 0.7, 4)
    assert d3s.last_status() == d3s.D3S_OK


def test_d3_sample_one_row_zero_copy_path(oracle):
    """One-row d3_sample calls run the one-CTA kernel on logits in mapped host
    memory and write the id there: every call equals the oracle across seeds,
    parameters and changes of V and top_k, a non-finite row is flagged, a row
    with fewer finite logits than k is handed on to the ordinary path, and a
    large call in between (the context's scratch regrown) changes nothing."""
    import d3s
    rng = np.random.default_rng(77)
    for V, k in [(4097, 30), (4097, 30), (1024, 5), (4097, 64), (4097, 30)]:
        x = (rng.standard_normal((24, V)) * 3).astype(np.float32)
        for i in range(24):
            T, p = float(rng.uniform(0.5, 1.2)), float(rng.uniform(0.5, 1.0))
            got = d3s.sample(x[i:i + 1], T, k, p, 1000 * V + i)
            assert d3s.last_status() == d3s.D3S_OK
            assert got.tolist() == oracle.d3_sample(x[i:i + 1], T, k, p, 1000 * V + i).tolist()
        bad = x[:1].copy()
        bad[0, 11] = np.inf
        assert d3s.sample(bad, 0.7, k, 0.7, 5).tolist() == [-1]
        assert d3s.last_status() == d3s.D3S_ERR_NONFINITE
        # a row with fewer finite logits than k is handed to the wide kernel
        masked = np.full((1, V), -np.inf, np.float32)
        masked[0, :3] = x[0, :3]
        assert d3s.sample(masked, 0.7, k, 0.9, 6).tolist() == oracle.d3_sample(masked, 0.7, k, 0.9, 6).tolist()
        assert d3s.last_status() == d3s.D3S_OK
    big = (rng.standard_normal((3000, 300)) * 3).astype(np.float32)
    assert d3s.sample(big, 0.8, 20, 0.9, 9).tolist() == oracle.d3_sample(big, 0.8, 20, 0.9, 9).tolist()
    one = (rng.standard_normal((1, 4097)) * 3).astype(np.float32)
    for s_ in range(5):
        assert d3s.sample(one, 0.7, 30, 0.7, s_).tolist() == oracle.d3_sample(one, 0.7, 30, 0.7, s_).tolist()


def test_config1_ten_thousand_sequential_draws(ctx, oracle, synth):
    """Config 1 as the reference's CLI runs it: m_seed(42) once
    (src/main.c:195), then 10,000 sequential sample_top_k_top_p calls on the
    global key (src/sampling.c:205-209), each on fresh f32 [1, 4097] logits
    ~N(0, 3) with one semantic logit +6; T 0.7, top_p 0.7, top_k 30. The ids of
    the global-key calls, and the kept sets (count, ranked ids, probabilities)
    of the same draws replayed with their subkeys, equal the oracle's."""
    import d3s
    n, V, k = 10_000, 4097, 30
    x = synth.c1_rows(n, seed=42)
    xh = host_logits(x)
    d3s.seed(42)
    ids = torch.empty(n, dtype=torch.int32, device="cuda")
    for i in range(n):
        ctx.sample_top_k_top_p(x[i:i + 1], 0.7, k, 0.7, None, ids[i:i + 1])
    got_ids = ids.cpu().numpy()
    # the subkeys of those draws, in order, then one batch that draws row i from subkey i
    state = d3s.key_from_seed(42)
    subs = np.array([d3s.next_key(state).tolist() for _ in range(n)], np.uint32)
    keys = torch.from_numpy(subs.view(np.int32)).cuda()
    b_ids = torch.empty(n, dtype=torch.int32, device="cuda")
    kept = torch.empty_like(b_ids)
    probs = torch.zeros(n, k, dtype=torch.float32, device="cuda")
    topk = torch.zeros(n, k, dtype=torch.int32, device="cuda")
    ctx.sample(ctx.request(x, b_ids, temperature=0.7, top_p=0.7, top_k=k, noise=d3s.NOISE_KEYS,
                           keys=keys, kept=kept, probs=probs, topk_ids=topk))
    ostate = oracle.key_from_seed(42)
    want_ids = np.zeros(n, np.int32)
    want_kept = np.zeros(n, np.int32)
    want_topk = np.zeros((n, k), np.int32)
    want_probs = np.zeros((n, k), np.float32)
    for i in range(n):
        sub = oracle.next_key(ostate)
        assert sub.tolist() == subs[i].tolist()
        r, tk, pr, dg = oracle.sample_row(xh[i], 0.7, 0.7, k, oracle.uniform(sub, k))
        want_ids[i], want_kept[i], want_topk[i], want_probs[i] = r, dg.kept, tk, pr
    assert (got_ids == want_ids).all(), f"{int((got_ids != want_ids).sum())} of {n} ids differ"
    assert (b_ids.cpu().numpy() == want_ids).all()
    assert (kept.cpu().numpy() == want_kept).all()
    assert (topk.cpu().numpy() == want_topk).all()
    assert (probs.cpu().numpy().view(np.uint32) == want_probs.view(np.uint32)).all()
    assert state.tolist() == ostate.tolist()
    ctx.check()


@pytest.mark.parametrize("V,top_k", [(4097, 30), (1024, 30), (4097, 5)])
def test_ties_match_oracle(oracle, V, top_k):
    """The reference's tests/test_decode.py:73-86 inputs: logits tied across the
    k-th place, seeds 0..39, top-p off; equal to the oracle and to itself."""
    import d3s
    rng = np.random.default_rng(1)
    logits = np.round(rng.standard_normal((8, V)) * 2).astype(np.float32)
    for seed in range(40):
        a = d3s.sample(logits, 1.0, top_k, 2.0, seed)
        b = d3s.sample(logits, 1.0, top_k, 2.0, seed)
        assert a.tolist() == b.tolist() == oracle.d3_sample(logits, 1.0, top_k, 2.0, seed).tolist()


@pytest.mark.parametrize("T,top_k,top_p", [(0.7, 30, 0.7), (1.0, 30, 0.9), (1.0, 5, 1.0),
                                           (0.3, 30, 0.95)])
def test_distribution(oracle, T, top_k, top_p):
    """tests/test_decode.py:89-114 restated on the GPU: 4000 seeds, frequencies
    within 4 sigma + 1e-3 of the exact kept-set probabilities."""
    import d3s
    from test_oracle import kept_set_definition
    rng = np.random.default_rng(0)
    logits = (rng.standard_normal((1, 4097)) * 3).astype(np.float32)
    n = 4000
    ours = np.array([d3s.sample(logits, T, top_k, top_p, s)[0] for s in range(n)])
    ids, probs, _ = kept_set_definition(logits[0], T, top_k, top_p)
    expected = dict(zip(ids.tolist(), probs.tolist()))
    for token, prob in expected.items():
        tol = 4 * np.sqrt(prob * (1 - prob) / n) + 1e-3
        assert abs(np.mean(ours == token) - prob) < tol
    assert set(np.unique(ours).tolist()) <= set(expected)


# ---- device API ----

def run_given(ctx, x, u, T, p):
    """sample_with_noise with every diagnostic output."""
    import d3s
    N, k = u.shape
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    status = torch.empty_like(ids)
    kept = torch.empty_like(ids)
    probs = torch.zeros(N, k, dtype=torch.float32, device="cuda")
    topk = torch.zeros(N, k, dtype=torch.int32, device="cuda")
    req = ctx.request(x, ids, temperature=T, top_p=p, top_k=k, noise=d3s.NOISE_GIVEN, u=u,
                      status=status, kept=kept, probs=probs, topk_ids=topk)
    ctx.sample(req)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), status.cpu().numpy(), kept.cpu().numpy(), probs.cpu().numpy(), topk.cpu().numpy()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("V,k,T,p", [(4097, 30, 0.7, 0.7), (1024, 30, 1.0, 0.9), (4097, 64, 1.2, 0.5),
                                     (4097, 1, 0.7, 0.7), (100, 100, 1.0, 2.0), (31, 7, 0.5, 0.9),
                                     (1, 1, 1.0, 0.5), (4097, 300, 1.0, 0.95), (5000, 256, 0.8, 0.99)])
def test_given_noise_diagnostics_bitwise(ctx, oracle, dtype, V, k, T, p):
    rng = np.random.default_rng(V * 7 + k)
    N = 48
    x = (rng.standard_normal((N, V)) * 3).astype(np.float32)
    xt = dev(x, torch.bfloat16 if dtype == "bf16" else torch.float32)
    xh = host_logits(xt)
    u = rng.random((N, k), dtype=np.float32)
    u[0, 0] = 0.0
    ids, status, kept, probs, topk = run_given(ctx, xt, dev(u), T, p)
    xf = xh.astype(np.uint32).__lshift__(16).view(np.float32) if dtype == "bf16" else xh
    for r in range(N):
        rid, tids, oprobs, d = oracle.sample_row(xf[r], T, p, k, u[r])
        assert ids[r] == rid and status[r] == 0 and kept[r] == d.kept, r
        assert topk[r].tolist() == tids.tolist(), r
        assert probs[r].view(np.uint32).tolist() == oprobs.view(np.uint32).tolist(), r


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("V,top_k", [(4097, 30), (1024, 30), (4097, 64), (4097, 4097), (20000, 30),
                                     (8192, 256), (8193, 40), (2, 5), (256, 30), (257, 64),
                                     (511, 128), (3072, 129), (4096, 200), (6000, 17), (300, 300)])
def test_key_mode_matches_oracle(ctx, oracle, dtype, V, top_k):
    """sample_top_k_top_p: one split of the state, u = uniform(sub, [N, k])."""
    import d3s
    rng = np.random.default_rng(V + top_k)
    N = 40
    x = (rng.standard_normal((N, V)) * 2.5).astype(np.float32)
    xt = dev(x, torch.bfloat16 if dtype == "bf16" else torch.float32)
    xh = host_logits(xt)
    state = d3s.key_from_seed(V)
    ostate = oracle.key_from_seed(V)
    for _ in range(2):
        ids = ctx.sample_top_k_top_p(xt, 0.8, top_k, 0.9, state)
        want = oracle.sample_top_k_top_p(ostate, xh, 0.8, top_k, 0.9)
        assert ids.cpu().numpy().tolist() == want.tolist()


def test_rows_config2_bf16(ctx, oracle, synth):
    x = synth.c2_logits(256, seed=3)
    seeds = torch.arange(5000, 5256, device="cuda", dtype=torch.int64)
    ids = torch.empty(256, dtype=torch.int32, device="cuda")
    ctx.sample_rows(x, ids, temperature=0.7, top_p=0.7, top_k=30, seeds=seeds)
    want = oracle.sample_rows(host_logits(x), 0.7, 0.7, 30, seeds.cpu().numpy().astype(np.uint64))
    assert ids.cpu().numpy().tolist() == want.tolist()


def test_rows_config4_heads(ctx, oracle, synth):
    x = synth.c4_logits(512 * 9, seed=4)
    seeds = torch.arange(512 * 9, device="cuda", dtype=torch.int64) * 7 + 1
    ids = torch.empty(512 * 9, dtype=torch.int32, device="cuda")
    ctx.sample_rows(x, ids, temperature=1.0, top_p=0.9, top_k=30, seeds=seeds)
    want = oracle.sample_rows(host_logits(x), 1.0, 0.9, 30, seeds.cpu().numpy().astype(np.uint64))
    assert ids.cpu().numpy().tolist() == want.tolist()


def test_rows_config5_per_row_params(ctx, oracle, synth):
    x, T, p, k, seeds = synth.c5_batch(4096, seed=5)
    ids = torch.empty(4096, dtype=torch.int32, device="cuda")
    kept = torch.empty_like(ids)
    ctx.sample_rows(x, ids, temperature=T, top_p=p, top_k=k, seeds=seeds, kept=kept)
    want = oracle.sample_rows(host_logits(x), T.cpu().numpy(), p.cpu().numpy(), k.cpu().numpy(),
                              seeds.cpu().numpy().astype(np.uint64))
    assert ids.cpu().numpy().tolist() == want.tolist()


@pytest.mark.parametrize("dtype,V,N", [("f32", 2049, 2500), ("f32", 6000, 2500), ("bf16", 4097, 2500),
                                        ("f32", 4097, 2048), ("bf16", 1024, 3000)])
def test_rows_both_kernel_paths(ctx, oracle, dtype, V, N):
    """Large batches of long rows run the stats + select kernels, batches of at
    most 2048 rows and short rows the one-warp-per-row kernel: both against
    the oracle on per-row parameters."""
    rng = np.random.default_rng(V + N)
    x = (rng.standard_normal((N, V)) * 3.0).astype(np.float32)
    T = rng.uniform(0.5, 1.2, N).astype(np.float32)
    p = rng.uniform(0.5, 1.0, N).astype(np.float32)
    k = rng.integers(1, 65, N).astype(np.int32)
    seeds = np.arange(N, dtype=np.int64) * 3 + V
    xt = dev(x, torch.bfloat16 if dtype == "bf16" else torch.float32)
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    ctx.sample_rows(xt, ids, temperature=dev(T), top_p=dev(p), top_k=dev(k), seeds=dev(seeds))
    want = oracle.sample_rows(host_logits(xt), T, p, k, seeds.astype(np.uint64))
    assert ids.cpu().numpy().tolist() == want.tolist()
    ctx.check()


def test_per_row_k_above_fast_limit_is_deferred(ctx, oracle):
    """Rows with k > 256 go through the wide kernel's hand-off list; a second
    launch checks the list counters were re-zeroed."""
    rng = np.random.default_rng(8)
    N, V = 300, 4097
    x = (rng.standard_normal((N, V)) * 2).astype(np.float32)
    k = rng.integers(1, 65, N).astype(np.int32)
    k[::7] = rng.integers(257, 5000, len(k[::7]))
    seeds = np.arange(N, dtype=np.int64) + 17
    for rep in range(2):
        ids = torch.empty(N, dtype=torch.int32, device="cuda")
        ctx.sample_rows(dev(x), ids, temperature=0.9, top_p=0.97, top_k=dev(k), seeds=dev(seeds))
        want = oracle.sample_rows(x, 0.9, 0.97, k, seeds.astype(np.uint64))
        assert ids.cpu().numpy().tolist() == want.tolist(), rep


def test_exact_selection_path_for_massive_ties(ctx, oracle):
    """All-equal and few-valued rows put more than the candidate buffer at the
    threshold: the kernel falls back to the exact 64-bit key bisection."""
    import d3s
    N, V = 16, 4097
    x = np.zeros((N, V), np.float32)
    x[1] = np.tile([1.0, 0.0], V)[:V]
    x[2, 100:3000] = 5.0
    x[3] = np.arange(V) % 3
    x[4, :] = -0.0
    x[5, ::2] = 0.0
    x[5, 1::2] = -0.0
    u = np.random.default_rng(2).random((N, 64), dtype=np.float32)
    ids, status, kept, probs, topk = run_given(ctx, dev(x), dev(u), 1.0, 0.8)
    for r in range(N):
        rid, tids, oprobs, d = oracle.sample_row(x[r], 1.0, 0.8, 64, u[r])
        assert ids[r] == rid and topk[r].tolist() == tids.tolist(), r
        assert probs[r].view(np.uint32).tolist() == oprobs.view(np.uint32).tolist()


def test_nonfinite_rows_are_flagged(ctx, oracle):
    import d3s
    rng = np.random.default_rng(3)
    N, V = 8, 4097
    x = (rng.standard_normal((N, V)) * 3).astype(np.float32)
    x[1, 5] = np.nan
    x[2, 7] = np.inf
    x[3] = -np.inf
    x[4, ::2] = -np.inf  # masked tokens are fine
    x[5, 9] = -np.nan
    u = rng.random((N, 30), dtype=np.float32)
    ids, status, kept, probs, topk = run_given(ctx, dev(x), dev(u), 0.7, 0.9)
    assert status.tolist() == [0, 1, 1, 1, 0, 1, 0, 0]
    assert ids[[1, 2, 3, 5]].tolist() == [-1] * 4
    for r in (0, 4, 6, 7):
        assert ids[r] == oracle.sample_row(x[r], 0.7, 0.9, 30, u[r])[0]
    out = np.zeros(N, np.int32)
    ids_sync = d3s.sample(x, 0.7, 30, 0.9, 1)
    assert d3s.last_status() == d3s.D3S_ERR_NONFINITE and ids_sync[1] == -1


def test_bad_params(ctx):
    import d3s
    x = torch.zeros(4, 64, device="cuda")
    with pytest.raises(d3s.D3SError):
        ctx.sample_top_k_top_p(x, 1.0, 0, 0.9)
    with pytest.raises(d3s.D3SError):
        ctx.sample_top_k_top_p(x, float("nan"), 5, 0.9)
    k = torch.tensor([5, 0, 3, -1], dtype=torch.int32, device="cuda")
    T = torch.tensor([1.0, 1.0, float("nan"), 1.0], device="cuda")
    ids = torch.empty(4, dtype=torch.int32, device="cuda")
    status = torch.empty_like(ids)
    req = ctx.request(x, ids, temperature_rows=T, top_p=0.9, top_k_rows=k, noise=d3s.NOISE_SEEDS,
                      seeds=torch.arange(4, device="cuda"), status=status)
    ctx.sample(req)
    assert status.cpu().tolist() == [0, 2, 2, 2] and ids.cpu().tolist()[1:] == [-1, -1, -1]


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("off", [100, 3, 1])
def test_strided_and_unaligned_rows(ctx, oracle, dtype, off):
    """ld > V and row starts off any 16-byte boundary (the bulk copy fetches
    the aligned span around each row)."""
    rng = np.random.default_rng(4 + off)
    big = (rng.standard_normal((10, 5000)) * 2).astype(np.float32)
    bt = dev(big, torch.bfloat16 if dtype == "bf16" else torch.float32)
    xt = bt[:, off:off + 4097]  # ld = 5000 > V = 4097
    xh = host_logits(xt)
    xf = (xh.astype(np.uint32) << 16).view(np.float32) if dtype == "bf16" else xh
    u = rng.random((10, 30), dtype=np.float32)
    ids = run_given(ctx, xt, dev(u), 0.7, 0.8)[0]
    for r in range(10):
        assert ids[r] == oracle.sample_row(xf[r], 0.7, 0.8, 30, u[r])[0]


def test_empty_batch_and_ctx_check(ctx):
    empty = torch.zeros(0, 4097, device="cuda")
    assert ctx.sample_top_k_top_p(empty, 1.0, 30, 0.9).numel() == 0
    ctx.check()


def test_full_size_config5(ctx, oracle, synth):
    """65536 x 4097 f32 with per-row parameters: deterministic, in range, and
    every one of the 65536 ids equal to the oracle's."""
    x, T, p, k, seeds = synth.c5_batch(65536, seed=11)
    ids = torch.empty(65536, dtype=torch.int32, device="cuda")
    ids2 = torch.empty_like(ids)
    ctx.sample_rows(x, ids, temperature=T, top_p=p, top_k=k, seeds=seeds)
    ctx.sample_rows(x, ids2, temperature=T, top_p=p, top_k=k, seeds=seeds)
    assert torch.equal(ids, ids2)
    assert int(ids.min()) >= 0 and int(ids.max()) < 4097
    want = oracle.sample_rows(host_logits(x), T.cpu().numpy(), p.cpu().numpy(), k.cpu().numpy(),
                              seeds.cpu().numpy().astype(np.uint64))
    got = ids.cpu().numpy()
    assert (got == want).all(), f"{int((got != want).sum())} of 65536 rows differ"
    ctx.check()


# ---- the approximate full-row sum of large batches and its certified cut ----

def test_ex2_approx_error_bound(ctx):
    """Large batches sum each row with the SFU's exp2; the error bound carried
    into the top-p cut assumes its relative error is below 2^-22.5 wherever the
    result is normal. Checked over every float input in [-127, 2^-8]."""
    worst = 0.0
    for lo, hi in [(0x80000000, 0xC2FE0001), (0x00000000, 0x3B800001)]:
        for s in range(lo, hi, 1 << 26):
            e = min(s + (1 << 26), hi)
            x = torch.arange(s, e, dtype=torch.int64, device="cuda").to(torch.int32).view(torch.float32)
            y = ctx.debug_math(4, x).double()
            ref = torch.exp2(x.double())
            normal = ref >= 2.0 ** -126
            worst = max(worst, float(((y - ref).abs() / ref)[normal].max()))
            del x, y, ref, normal
    assert worst < 2.0 ** -22.5, worst


def test_top_p_on_a_cumsum_takes_the_exact_sum(ctx, oracle):
    """Rows whose top_p sits exactly on one of their cumsums, or one float
    below it, leave the cut uncertain under the approximate sum's error bound:
    the kernel recomputes those rows' exact sums. Ids, kept counts and
    probabilities must equal the oracle's on every row of a large batch."""
    import d3s
    rng = np.random.default_rng(21)
    N, V, k = 2600, 4097, 48
    x = (rng.standard_normal((N, V)) * 3).astype(np.float32)
    T = rng.uniform(0.5, 1.2, N).astype(np.float32)
    p = rng.uniform(0.5, 1.0, N).astype(np.float32)
    special = rng.choice(N, 400, replace=False)
    for i, r in enumerate(special):
        cums = oracle.row_cums(x[r], float(T[r]), k)
        c = np.float32(cums[int(rng.integers(1, k))])
        p[r] = c if i % 2 == 0 else np.nextafter(c, np.float32(0.0))
    u = rng.random((N, k), dtype=np.float32)
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    kept, status = torch.empty_like(ids), torch.empty_like(ids)
    probs = torch.zeros(N, k, dtype=torch.float32, device="cuda")
    req = ctx.request(dev(x), ids, temperature_rows=dev(T), top_p_rows=dev(p), top_k=k,
                      noise=d3s.NOISE_GIVEN, u=dev(u), status=status, kept=kept, probs=probs)
    ctx.sample(req)
    got_ids, got_kept, got_probs = ids.cpu().numpy(), kept.cpu().numpy(), probs.cpu().numpy()
    for r in range(N):
        rid, _, oprobs, d = oracle.sample_row(x[r], float(T[r]), float(p[r]), k, u[r])
        assert got_ids[r] == rid and got_kept[r] == d.kept, r
        assert got_probs[r].view(np.uint32).tolist() == oprobs.view(np.uint32).tolist(), r
    ctx.check()


def test_rows_outside_the_approximate_path(ctx, oracle):
    """In a large batch, rows the approximate sum does not take (k > 128, T
    above 2^20, |x| above 2^60) run the exact per-element path in the same
    kernel; every row must equal the oracle."""
    rng = np.random.default_rng(22)
    N, V = 2600, 4097
    x = (rng.standard_normal((N, V)) * 3).astype(np.float32)
    T = rng.uniform(0.5, 1.2, N).astype(np.float32)
    p = rng.uniform(0.5, 1.0, N).astype(np.float32)
    k = rng.integers(1, 65, N).astype(np.int32)
    k[::5] = rng.integers(129, 257, len(k[::5]))
    T[1::7] = 2.0 ** 21
    x[3::11] *= np.float32(2.0 ** 61)
    seeds = np.arange(N, dtype=np.int64) * 5 + 1
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    ctx.sample_rows(dev(x), ids, temperature=dev(T), top_p=dev(p), top_k=dev(k), seeds=dev(seeds))
    want = oracle.sample_rows(x, T, p, k, seeds.astype(np.uint64))
    assert ids.cpu().numpy().tolist() == want.tolist()
    ctx.check()
