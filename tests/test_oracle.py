"""The CPU oracle against published known answers and the reference's own test
definitions (no GPU). The oracle is the checker for every GPU parity test, so
it is pinned here first."""

import json
import math
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
KNOWN = json.loads((GOLDEN / "known_answers.json").read_text())
M32 = 0xFFFFFFFF


# ---- an independent pure-Python threefry, to check the oracle's C restatement ----

def py_threefry(key, ctr):
    R = [13, 15, 26, 6, 17, 29, 16, 24]
    ks = [key[0], key[1], key[0] ^ key[1] ^ 0x1BD11BDA]
    x0, x1 = (ctr[0] + ks[0]) & M32, (ctr[1] + ks[1]) & M32
    for rnd in range(20):
        x0 = (x0 + x1) & M32
        r = R[rnd % 8]
        x1 = ((x1 << r) | (x1 >> (32 - r))) & M32
        x1 ^= x0
        if rnd % 4 == 3:
            g = rnd // 4
            x0 = (x0 + ks[(g + 1) % 3]) & M32
            x1 = (x1 + ks[(g + 2) % 3] + g + 1) & M32
    return x0, x1


def py_bits(key, n):
    """MLX RandomBits for one key and n words, written from its description."""
    h, o = n // 2, n % 2
    out = [0] * n
    for i in range(h):
        a, b = py_threefry(key, (i, h + o + i))
        out[i], out[h + o + i] = a, b
    if o:
        out[h] = py_threefry(key, (h, 0))[0]
    return out


def test_threefry_known_answers(oracle):
    for kat in KNOWN["threefry2x32_20"]:
        assert oracle.threefry(kat["key"], kat["ctr"]) == tuple(kat["out"])
        assert py_threefry(kat["key"], kat["ctr"]) == tuple(kat["out"])


def test_split_of_key_zero_matches_jax(oracle):
    k0, k1 = oracle.split(oracle.key_from_seed(0))
    assert k0.tolist() == KNOWN["split_key0"]["k0"]
    assert k1.tolist() == KNOWN["split_key0"]["k1"]


def test_key_from_seed_word_order(oracle):
    assert oracle.key_from_seed(0x0123456789ABCDEF).tolist() == [0x01234567, 0x89ABCDEF]


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 29, 30, 31, 64, 255])
def test_bits_layout_even_and_odd(oracle, n):
    key = oracle.split(oracle.key_from_seed(n))[1]
    assert oracle.bits(key, n).tolist() == py_bits(key.tolist(), n)
    for f in (0, n // 2, n - 1):
        assert int(oracle.lib().d3o_bits_word(np.ascontiguousarray(key).ctypes.data_as(
            oracle._u32p), n, f)) == py_bits(key.tolist(), n)[f]


def test_next_key_keeps_first_half(oracle):
    state = oracle.key_from_seed(42)
    k0, k1 = oracle.split(state.copy())
    sub = oracle.next_key(state)
    assert sub.tolist() == k1.tolist() and state.tolist() == k0.tolist()


def test_uniform_mapping_edges(oracle):
    b = np.array([0, 1, 0xFFFFFF7F, 0xFFFFFF80, 0xFFFFFFFF, 1 << 31], np.uint32)
    u = oracle.bits_to_uniform(b)
    assert u[0] == 0.0
    assert u[1] == np.float32(2.0 ** -32)
    upper = np.nextafter(np.float32(1), np.float32(0))
    assert u[2] == upper and u[3] == upper and u[4] == upper  # float(b) rounds up to 2^32
    assert u[5] == np.float32(0.5)
    assert (u < 1).all()


def test_uniform_is_bits_over_2_32(oracle):
    key = oracle.split(oracle.key_from_seed(3))[1]
    b = oracle.bits(key, 1001).astype(np.float64)
    u = oracle.uniform(key, 1001)
    ref = np.minimum((b.astype(np.float32).astype(np.float64) / 2.0 ** 32).astype(np.float32),
                     np.nextafter(np.float32(1), np.float32(0)))
    assert np.array_equal(u, ref)


def test_golden_regression(oracle):
    g = np.load(GOLDEN / "oracle_cases.npz")
    for pi, (T, k, p) in enumerate(g["d3_params"]):
        for s in range(4):
            ids = oracle.d3_sample(g["d3_logits"], float(T), int(k), float(p), s)
            assert ids.tolist() == g["d3_ids"][pi, s].tolist()
    ids = oracle.sample_rows(g["rows_bf16"], 0.7, 0.7, 30, g["rows_seeds"])
    assert ids.tolist() == g["rows_ids"].tolist()
    key = g["uniform_key"]
    assert np.array_equal(oracle.uniform(key, 5), g["uniform_5"])
    assert np.array_equal(oracle.uniform(key, 30), g["uniform_30"])
    assert np.array_equal(oracle.bits(key, 7), g["bits_7"])


# ---- exp / log ----

def ulp_err(y, ref):
    y = y.astype(np.float64)
    sp = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    return np.abs(y - ref) / sp


def test_exp_accuracy(oracle):
    x = np.linspace(-87.0, 88.5, 3_000_001).astype(np.float32)
    ulp = ulp_err(oracle.exp(x), np.exp(x.astype(np.float64)))
    assert ulp.max() < 1.0, ulp.max()
    assert oracle.exp(np.array([0.0], np.float32))[0] == 1.0
    sub = oracle.exp(np.array([-100.0, -103.9, -104.5, -np.inf], np.float32))
    assert sub[0] > 0 and sub[1] > 0 and sub[2] == 0 and sub[3] == 0
    assert np.isinf(oracle.exp(np.array([89.5], np.float32))[0])


def test_log_accuracy(oracle):
    x = np.exp(np.linspace(-100.0, 88.0, 3_000_001)).astype(np.float32)
    x = x[(x > 0) & np.isfinite(x) & (x != 1)]
    ulp = ulp_err(oracle.log(x), np.log(x.astype(np.float64)))
    assert ulp.max() < 2.0, ulp.max()
    one_minus_u = (1.0 - np.arange(1, 100_000, dtype=np.float32) * np.float32(2.0 ** -24)).astype(np.float32)
    ulp = ulp_err(oracle.log(one_minus_u), np.log(one_minus_u.astype(np.float64)))
    assert ulp.max() < 2.0
    sp = oracle.log(np.array([1.0, 0.0, -1.0, np.inf, 1e-45], np.float32))
    assert sp[0] == 0.0 and not np.signbit(sp[0])
    assert sp[1] == -np.inf and np.isnan(sp[2]) and sp[3] == np.inf
    assert abs(sp[4] - math.log(float(np.float32(1e-45)))) < 1e-4  # smallest subnormal


def test_exp_and_log_facts_the_certified_cut_uses(oracle):
    """The large-batch kernels sum a row with the SFU's exp2 and carry the error
    bound into the top-p cut. That bound assumes exp's relative error is below
    2^-23.5 over every float of [-86, 0] (the full-row-sum terms and the cumsum
    terms), and it brackets lse through log, which must never decrease over
    [1, 16384) (the normalised sum S / 2^46 of rows up to 8192 long)."""
    assert oracle.exp_max_relerr(-86.0, 0.0) < 2.0 ** -23.5
    assert oracle.log_nonmonotone(1.0, 16384.0) == 0


# ---- the sampler ----

def kept_set_definition(x, T, k, p):
    """The exact kept set and probabilities from the reference's test definition
    (tests/test_decode.py:100-109), in float64."""
    q = (x / np.float32(max(T, 1e-5))).astype(np.float32)
    order = np.argsort(-q, kind="stable")
    values = q[order].astype(np.float64)
    pr = np.exp(values - values.max())
    pr /= pr.sum()
    keep = ~((np.cumsum(pr) > p) | (np.arange(len(pr)) >= k))
    keep[0] = True
    probs = np.where(keep, pr, 0)
    probs /= probs.sum()
    return order[keep], probs[keep], np.cumsum(pr)


@pytest.mark.parametrize("T,k,p", [(0.7, 30, 0.7), (1.0, 30, 0.9), (1.0, 5, 1.0), (0.3, 30, 0.95),
                                   (0.5, 64, 0.5), (1.2, 1, 0.7)])
def test_kept_set_matches_definition(oracle, T, k, p):
    rng = np.random.default_rng(11)
    u = np.full(max(k, 1), 0.5, np.float32)
    near = 0
    for _ in range(60):
        x = (rng.standard_normal(4097) * 3).astype(np.float32)
        ids_def, probs_def, cum = kept_set_definition(x, T, k, p)
        _, topk_ids, probs, d = oracle.sample_row(x, T, p, min(k, 4097), u)
        kept = d.kept
        if np.min(np.abs(cum[:min(k, 4097)] - p)) < 1e-6:
            near += 1  # the float32 and float64 cuts may differ by a rank here
            continue
        assert topk_ids[:kept].tolist() == ids_def.tolist()
        np.testing.assert_allclose(probs[:kept], probs_def, rtol=1e-5)
        assert (probs[kept:] == 0).all()
    assert near < 3


@pytest.mark.parametrize("V,top_k", [(4097, 30), (1024, 30), (4097, 5)])
def test_ties_metal_order_equals_stable_order(oracle, V, top_k):
    """The reference's tests/test_decode.py:73-86 inputs (logits tied across the
    k-th place): the Metal kernel's selection keeps the same candidates, in the
    same order, as the op graph's stable sort (the lowest ids)."""
    rng = np.random.default_rng(1)
    logits = np.round(rng.standard_normal((8, V)) * 2).astype(np.float32)
    for row in logits:
        v1, i1 = oracle.topk_stable(row, top_k)
        v2, i2 = oracle.topk_metal_order(row, top_k)
        assert i1.tolist() == i2.tolist() and np.array_equal(v1, v2)
    for seed in range(40):
        a = oracle.d3_sample(logits, 1.0, top_k, 2.0, seed)
        b = oracle.d3_sample(logits, 1.0, top_k, 2.0, seed)
        assert a.tolist() == b.tolist()


@pytest.mark.parametrize("T,top_k,top_p", [(0.7, 30, 0.7), (1.0, 30, 0.9), (1.0, 5, 1.0),
                                           (0.3, 30, 0.95)])
def test_sampler_distribution(oracle, T, top_k, top_p):
    """tests/test_decode.py:89-114 restated: 4000 seeds, empirical frequencies
    within 4 sigma + 1e-3 of the exact kept-set probabilities."""
    rng = np.random.default_rng(0)
    logits = (rng.standard_normal((1, 4097)) * 3).astype(np.float32)
    n = 4000
    ours = np.array([oracle.d3_sample(logits, T, top_k, top_p, s)[0] for s in range(n)])
    ids, probs, _ = kept_set_definition(logits[0], T, top_k, top_p)
    expected = dict(zip(ids.tolist(), probs.tolist()))
    for token, prob in expected.items():
        freq = np.mean(ours == token)
        tol = 4 * np.sqrt(prob * (1 - prob) / n) + 1e-3
        assert abs(freq - prob) < tol, (token, freq, prob)
    assert set(np.unique(ours).tolist()) <= set(expected)


def test_edge_rows(oracle):
    V = 300
    u = np.full(64, 0.3, np.float32)
    x = np.zeros(V, np.float32)
    # all equal: top-k are the lowest ids, softmax uniform over survivors
    r, ids, probs, d = oracle.sample_row(x, 1.0, 2.0, 10, u)
    assert ids.tolist() == list(range(10)) and d.kept == 10
    np.testing.assert_allclose(probs, 0.1, rtol=1e-6)
    # NaN / +inf / all -inf rows are flagged
    for bad in (np.nan, np.inf):
        y = x.copy()
        y[7] = bad
        assert oracle.sample_row(y, 1.0, 0.9, 10, u)[0] == -1
    assert oracle.sample_row(np.full(V, -np.inf, np.float32), 1.0, 0.9, 10, u)[0] == -1
    # -inf entries are masked tokens
    y = np.full(V, -np.inf, np.float32)
    y[[5, 9]] = [1.0, 2.0]
    r, ids, probs, d = oracle.sample_row(y, 1.0, 2.0, 4, u)
    assert ids.tolist() == [9, 5, 0, 1] and r in (5, 9) and probs[2] == 0 and probs[3] == 0
    # top_p <= 0 keeps rank 0 only; NaN top_p drops nothing
    y = np.arange(V, dtype=np.float32) * 0.01
    assert oracle.sample_row(y, 1.0, 0.0, 10, u)[0] == V - 1
    assert oracle.sample_row(y, 1.0, np.nan, 10, u)[3].kept == 10
    # temperature 0 clamps to 1e-5: greedy
    assert oracle.sample_row(y, 0.0, 0.9, 10, u)[0] == V - 1
    # k = 1 is greedy, ties to the lowest id
    y = np.zeros(V, np.float32)
    y[[17, 40]] = 3.0
    assert oracle.sample_row(y, 1.0, 0.9, 1, u)[0] == 17
    # k >= V: the full sort
    assert oracle.d3_sample(y[None], 1.0, 10 ** 6, 0.9, 5)[0] in range(V)


def test_u_near_zero_gives_minus_inf_score(oracle):
    """-log(1 - u) is -0 when 1 - u rounds to 1, so p / noise is -inf and that
    rank cannot win (src/sampling.c:46-47, :135-137): restated as is."""
    x = np.array([5.0, 4.9, 0.0], np.float32)
    u = np.array([1e-9, 0.5, 0.5], np.float32)
    r, ids, probs, d = oracle.sample_row(x, 1.0, 2.0, 3, u)
    assert r != 0


def test_sample_rows_equals_per_row_d3_sample(oracle):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((12, 1024)) * 2.5).astype(np.float32)
    T = rng.uniform(0.5, 1.2, 12).astype(np.float32)
    p = rng.uniform(0.5, 1.0, 12).astype(np.float32)
    k = rng.integers(1, 65, 12).astype(np.int32)
    seeds = np.arange(77, 89, dtype=np.uint64)
    ids = oracle.sample_rows(x, T, p, k, seeds)
    for r in range(12):
        assert ids[r] == oracle.d3_sample(x[r:r + 1], float(T[r]), int(k[r]), float(p[r]), int(seeds[r]))[0]


def test_sample_top_k_top_p_key_sequence(oracle):
    """Two calls after one seed use two successive splits of the global key."""
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((3, 512)) * 2).astype(np.float32)
    state = oracle.key_from_seed(123)
    a = oracle.sample_top_k_top_p(state, x, 0.8, 20, 0.9)
    b = oracle.sample_top_k_top_p(state, x, 0.8, 20, 0.9)
    s2 = oracle.key_from_seed(123)
    sub1 = oracle.next_key(s2)
    sub2 = oracle.next_key(s2)
    assert a.tolist() == oracle.sample_with_noise(x, oracle.uniform(sub1, 60).reshape(3, 20), 0.8, 0.9).tolist()
    assert b.tolist() == oracle.sample_with_noise(x, oracle.uniform(sub2, 60).reshape(3, 20), 0.8, 0.9).tolist()
