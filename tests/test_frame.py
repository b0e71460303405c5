"""One decode frame of tower_decode_step (src/tower.c:405-452): the key order,
the RAS repetition check, candidate_token and c0, and the history window.

CPU tests pin the oracle's frame step against the reference's definitions;
the gpu tests compare the C ABI (d3s_keys_next, d3s_frame_main, d3s_sample
with per-row keys) with the oracle on the same inputs, bit for bit."""

import ctypes

import numpy as np
import pytest

SEM0, VOCAB, EOS = 1000, 4096, 7  # a config with eos below the semantic band (src/model.c:119-124)


def tok_of(idx):
    """candidate_token (src/tower.c:405-409)."""
    return EOS if idx == 0 else idx + SEM0 - 1


def peaked(V, idx, rng, height=60.0):
    x = rng.standard_normal(V).astype(np.float32)
    x[idx] += height
    return x


# ---- oracle (CPU) ----

def test_frame_main_maps_indices_and_clips_c0(oracle):
    rng = np.random.default_rng(1)
    k0, k1 = oracle.next_key(np.array([0, 5], np.uint32)), np.array([3, 4], np.uint32)
    for idx in (0, 1, 2, 4096):
        x = peaked(1 + VOCAB, idx, rng)
        main, c0, flags = oracle.frame_main(x, 0.7, 0.7, 30, k0, k1, [], SEM0, VOCAB, EOS)
        assert main == tok_of(idx)
        assert c0 == min(max(main - SEM0, 0), VOCAB - 1)
        assert flags == (oracle.FRAME_EOS if idx == 0 else 0)


def test_frame_main_retries_only_repeated_semantic_tokens(oracle):
    rng = np.random.default_rng(2)
    km, kr = np.array([11, 12], np.uint32), np.array([13, 14], np.uint32)
    x = peaked(1 + VOCAB, 77, rng)
    first = tok_of(77)
    # not in the history: the first draw stands
    assert oracle.frame_main(x, 0.7, 0.7, 30, km, kr, [SEM0 + 5, SEM0 + 9], SEM0, VOCAB, EOS)[0] == first
    # repeated: the retry draw (T 1.0, top_p 0.95, top_k 30, its own key) replaces it
    u = oracle.uniform(kr, 30)
    retry_idx, _, _, _ = oracle.sample_row(x, 1.0, 0.95, 30, u)
    main, c0, flags = oracle.frame_main(x, 0.7, 0.7, 30, km, kr, [SEM0, first], SEM0, VOCAB, EOS)
    assert main == tok_of(retry_idx) and flags & oracle.FRAME_RETRY
    # eos is never redrawn, even when it is in the history
    xe = peaked(1 + VOCAB, 0, rng)
    main, c0, flags = oracle.frame_main(xe, 0.7, 0.7, 30, km, kr, [EOS, EOS], SEM0, VOCAB, EOS)
    assert main == EOS and c0 == 0 and flags == oracle.FRAME_EOS


def test_frame_main_uses_the_main_draw_definition(oracle):
    """main draw == sample_row with u = uniform(key_main, min(top_k, V))."""
    rng = np.random.default_rng(3)
    km, kr = np.array([21, 22], np.uint32), np.array([23, 24], np.uint32)
    for t in range(20):
        x = (rng.standard_normal(1 + VOCAB) * 2).astype(np.float32)
        u = oracle.uniform(km, 50)
        idx, _, _, _ = oracle.sample_row(x, 0.9, 0.8, 50, u)
        assert oracle.frame_main(x, 0.9, 0.8, 50, km, kr, [], SEM0, VOCAB, EOS)[0] == tok_of(idx)


def test_frame_main_flags_non_finite_rows(oracle):
    rng = np.random.default_rng(4)
    km, kr = np.array([1, 2], np.uint32), np.array([3, 4], np.uint32)
    x = peaked(1 + VOCAB, 5, rng)
    x[100] = -np.inf  # samples, but the row is not finite (src/generate.c:92)
    main, c0, flags = oracle.frame_main(x, 0.7, 0.7, 30, km, kr, [], SEM0, VOCAB, EOS)
    assert main == tok_of(5) and flags == oracle.FRAME_NONFINITE
    x[200] = np.nan
    main, c0, flags = oracle.frame_main(x, 0.7, 0.7, 30, km, kr, [], SEM0, VOCAB, EOS)
    assert main == -1 and c0 == 0 and flags & oracle.FRAME_NONFINITE


def test_history_window(oracle):
    h = []
    for t in range(40):
        h = oracle.history_push(h, t)
        assert h == list(range(max(0, t + 1 - oracle.RAS_WINDOW), t + 1))
    # the C restatement agrees
    hist = np.zeros(oracle.RAS_WINDOW, np.int32)
    n = ctypes.c_int(0)
    L = oracle.lib()
    for t in range(40):
        L.d3o_history_push(hist.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ctypes.byref(n), t)
        assert list(hist[:n.value]) == list(range(max(0, t + 1 - 16), t + 1))


def test_stream_key_order_is_the_frame_noise_order(oracle):
    """Frame subkeys from streams_next_keys draw the same uniforms as the
    frame's sample_noise calls in order (src/tower.c:417-424)."""
    ks = [30, 30] + [30] * 9
    st = oracle.key_from_seed(99)
    u_frame = oracle.frame_noise(st.copy(), ks)
    _, subs = oracle.streams_next_keys(st.reshape(1, 2), len(ks))
    u_keys = np.concatenate([oracle.uniform(subs[0, i], k) for i, k in enumerate(ks)])
    np.testing.assert_array_equal(u_frame, u_keys)


def test_rows_keys_equals_per_row_uniforms(oracle):
    rng = np.random.default_rng(5)
    N, V = 40, 1024
    x = (rng.standard_normal((N, V)) * 2.5).astype(np.float32)
    keys = rng.integers(0, 2**32, (N, 3, 2), dtype=np.uint64).astype(np.uint32)
    ids = oracle.sample_rows_keys(x, 1.0, 0.9, 30, keys)
    for r in range(N):
        u = oracle.uniform(keys[r, 0], 30)
        assert ids[r] == oracle.sample_row(x[r], 1.0, 0.9, 30, u)[0]


def test_frame_request_layout_matches_header(tmp_path):
    import subprocess
    from pathlib import Path

    import d3s
    root = Path(__file__).resolve().parent.parent
    fields = [f[0] for f in d3s.FrameRequest._fields_]
    body = "".join(f'printf("{f} %zu\\n", offsetof(d3s_frame_request, {f}));' for f in fields)
    src = tmp_path / "probe.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "d3s.h"\n'
                   f'int main(void){{{body} printf("size %zu\\n", sizeof(d3s_frame_request)); return 0;}}\n')
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", f"-I{root / 'include'}", str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                      check=True).stdout.splitlines())
    for f in fields:
        assert getattr(d3s.FrameRequest, f).offset == int(out[f]), f
    assert ctypes.sizeof(d3s.FrameRequest) == int(out["size"])


# ---- CUDA vs oracle ----

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    import d3s
    c = d3s.Context(0)
    yield c
    c.close()


def _keys_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).cuda()


def _keys_host(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.gpu
def test_keys_next_matches_oracle(ctx, oracle):
    rng = np.random.default_rng(6)
    S, n = 513, 11
    st = rng.integers(0, 2**32, (S, 2), dtype=np.uint64).astype(np.uint32)
    st_dev = _keys_dev(st)
    sub = ctx.keys_next(st_dev, n)
    torch.cuda.synchronize()
    st2, subs = oracle.streams_next_keys(st, n)
    np.testing.assert_array_equal(_keys_host(sub), subs)
    np.testing.assert_array_equal(_keys_host(st_dev), st2)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_rows_keys_c4_heads(ctx, oracle, dtype):
    """Config C4's head rows: 512 streams, V = 1024, Zipf-biased, per-row keys
    taken with a stride from a [S, 11] subkey table (head j uses column 2 + j)."""
    import synth
    S, V = 512, 1024
    x = synth.c4_logits(S, seed=7, V=V) if hasattr(synth, "c4_logits") else None
    if x is None:
        pytest.skip("synth.c4_logits missing")
    x = x.to(torch.bfloat16 if dtype == "bf16" else torch.float32).cuda()
    rng = np.random.default_rng(8)
    table = rng.integers(0, 2**32, (S, 11, 2), dtype=np.uint64).astype(np.uint32)
    tdev = _keys_dev(table)
    ids = torch.empty(S, dtype=torch.int32, device="cuda")
    fin = torch.empty(S, dtype=torch.int32, device="cuda")
    for j in (0, 8):
        ctx.sample_rows_keys(x, ids, tdev[:, 2 + j], temperature=1.0, top_p=0.9, top_k=30,
                             finite=fin)
        want = oracle.sample_rows_keys(synth.to_host_logits(x), 1.0, 0.9, 30,
                                       np.ascontiguousarray(table[:, 2 + j:]))
        np.testing.assert_array_equal(ids.cpu().numpy(), want)
        assert fin.cpu().numpy().all()


@pytest.mark.gpu
def test_finite_flags(ctx):
    rng = np.random.default_rng(9)
    N, V = 64, 4097
    x = rng.standard_normal((N, V)).astype(np.float32)
    x[3, 10] = np.inf
    x[5, 0] = -np.inf
    x[7, 4096] = np.nan
    x[9, :] = -np.inf
    xd = torch.from_numpy(x).cuda()
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    fin = torch.full((N,), 7, dtype=torch.int32, device="cuda")
    seeds = torch.arange(N, dtype=torch.int64, device="cuda")
    import d3s
    req = ctx.request(xd, ids, temperature=0.8, top_p=0.9, top_k=30, noise=d3s.NOISE_SEEDS,
                      seeds=seeds, finite=fin)
    ctx.sample(req)
    want = np.isfinite(x).all(axis=1).astype(np.int32)
    np.testing.assert_array_equal(fin.cpu().numpy(), want)
    # the wide path (k > 256) writes them too
    fin.fill_(7)
    req = ctx.request(xd, ids, temperature=0.8, top_p=0.9, top_k=300, noise=d3s.NOISE_SEEDS,
                      seeds=seeds, finite=fin)
    ctx.sample(req)
    np.testing.assert_array_equal(fin.cpu().numpy(), want)


def _frame_logits(S, V, rng, with_bad=False):
    x = (rng.standard_normal((S, V)) * 2.0).astype(np.float32)
    x[:, 0] -= 4.0
    peaks = rng.integers(1, V, S)
    x[np.arange(S), peaks] += rng.uniform(4, 10, S).astype(np.float32)
    x[::17, 0] += 30.0  # some streams stop
    if with_bad:
        x[5, 9] = -np.inf
        x[6, 9] = np.nan
    return x, peaks


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_frame_main_matches_oracle(ctx, oracle, dtype):
    rng = np.random.default_rng(10)
    S, V = 300, 1 + VOCAB
    x, peaks = _frame_logits(S, V, rng, with_bad=True)
    xt = torch.from_numpy(x).to(torch.bfloat16 if dtype == "bf16" else torch.float32).cuda()
    xh = __import__("synth").to_host_logits(xt)
    # histories: some hold the likely first token, so the retry path runs
    hist = np.full((S, 16), -5, np.int32)
    hl = rng.integers(0, 17, S).astype(np.int32)
    for s in range(S):
        if s % 3 == 0 and hl[s] > 0:
            hist[s, rng.integers(0, hl[s])] = tok_of(int(peaks[s]))
    st = rng.integers(0, 2**32, (S, 2), dtype=np.uint64).astype(np.uint32)
    sub = ctx.keys_next(_keys_dev(st), 11)
    subs = _keys_host(sub)
    hd, hld = torch.from_numpy(hist).cuda(), torch.from_numpy(hl).cuda()
    main, c0, flags = ctx.frame_main(xt, sub, hd, hld, temperature=0.7, top_p=0.7, top_k=30,
                                     semantic_start=SEM0, code_vocab=VOCAB, eos_id=EOS)
    main, c0, flags = main.cpu().numpy(), c0.cpu().numpy(), flags.cpu().numpy()
    n_retry = 0
    for s in range(S):
        h = list(hist[s, :hl[s]])
        want = oracle.frame_main(xh[s], 0.7, 0.7, 30, subs[s, 0], subs[s, 1], h, SEM0, VOCAB, EOS)
        assert (main[s], c0[s], flags[s]) == want, s
        n_retry += bool(want[2] & oracle.FRAME_RETRY)
        # the history window was updated in place
        h2 = oracle.history_push(h, want[0])
        assert list(hd[s, :hld[s]].cpu().numpy()) == h2, s
    assert n_retry >= 20


@pytest.mark.gpu
def test_c4_frames_end_to_end(ctx, oracle):
    """Several frames of 64 streams: keys advance per frame, main + retry on
    the backbone row, then 9 head draws on V = 1024 rows, all against the
    oracle's per-stream loop."""
    rng = np.random.default_rng(11)
    S, Vb, Vh, H = 64, 1 + VOCAB, 1024, 9
    st = rng.integers(0, 2**32, (S, 2), dtype=np.uint64).astype(np.uint32)
    st_dev = _keys_dev(st)
    hist = np.zeros((S, 16), np.int32)
    hl = np.zeros(S, np.int32)
    hd, hld = torch.from_numpy(hist).cuda(), torch.from_numpy(hl).cuda()
    o_state = st.copy()
    o_hist = [[] for _ in range(S)]
    ids = torch.empty(S, dtype=torch.int32, device="cuda")
    for frame in range(4):
        xb, _ = _frame_logits(S, Vb, rng)
        heads = (rng.standard_normal((H, S, Vh)) * 2.5).astype(np.float32)
        sub = ctx.keys_next(st_dev, 2 + H)
        main, c0, flags = ctx.frame_main(torch.from_numpy(xb).cuda(), sub, hd, hld,
                                         temperature=0.8, top_p=0.9, top_k=30,
                                         semantic_start=SEM0, code_vocab=VOCAB, eos_id=EOS)
        codes = [main.cpu().numpy(), c0.cpu().numpy()]
        for j in range(H):
            ctx.sample_rows_keys(torch.from_numpy(heads[j]).cuda(), ids, sub[:, 2 + j],
                                 temperature=0.8, top_p=0.9, top_k=30)
            codes.append(ids.cpu().numpy().copy())
        # oracle: each stream's own key sequence, in tower_decode_step order
        o_state, o_subs = oracle.streams_next_keys(o_state, 2 + H)
        for s in range(S):
            m, c, f = oracle.frame_main(xb[s], 0.8, 0.9, 30, o_subs[s, 0], o_subs[s, 1],
                                        o_hist[s], SEM0, VOCAB, EOS)
            assert (codes[0][s], codes[1][s]) == (m, c), (frame, s)
            o_hist[s] = oracle.history_push(o_hist[s], m)
            for j in range(H):
                u = oracle.uniform(o_subs[s, 2 + j], 30)
                assert codes[2 + j][s] == oracle.sample_row(heads[j, s], 0.8, 0.9, 30, u)[0]
    np.testing.assert_array_equal(_keys_host(st_dev), o_state)


@pytest.mark.gpu
def test_frame_step_replays_from_a_cuda_graph(ctx, oracle):
    """One decode frame (key advance, main + retry, 9 head draws) captured once in
    a CUDA graph and replayed frame after frame gives the same codes as the same
    calls made one by one (scratch reserved and every kernel prepared before the
    capture, so nothing in the step allocates or queries the device)."""
    rng = np.random.default_rng(12)
    S, Vb, Vh, H = 64, 1 + VOCAB, 1024, 9
    xb = torch.from_numpy(_frame_logits(S, Vb, rng)[0]).to(torch.bfloat16).cuda()
    heads = torch.from_numpy((rng.standard_normal((H, S, Vh)) * 2.5).astype(np.float32)).to(
        torch.bfloat16).cuda()
    st0 = rng.integers(0, 2**32, (S, 2), dtype=np.uint64).astype(np.uint32)
    ctx.reserve(2 * S)

    def make_state():
        return (_keys_dev(st0), torch.zeros(S, 16, dtype=torch.int32, device="cuda"),
                torch.zeros(S, dtype=torch.int32, device="cuda"),
                torch.empty(S, 2 + H, 2, dtype=torch.int32, device="cuda"),
                torch.empty(H + 2, S, dtype=torch.int32, device="cuda"))

    def step(state, stream=None):
        states, hist, hl, sub, codes = state
        ctx.keys_next(states, 2 + H, sub=sub, stream=stream)
        m, c, _ = ctx.frame_main(xb, sub, hist, hl, temperature=0.8, top_p=0.9, top_k=30,
                                 semantic_start=SEM0, code_vocab=VOCAB, eos_id=EOS, stream=stream)
        codes[0].copy_(m)
        codes[1].copy_(c)
        for j in range(H):
            ctx.sample_rows_keys(heads[j], codes[2 + j], sub[:, 2 + j], temperature=0.8,
                                 top_p=0.9, top_k=30, stream=stream)

    eager, graphed = make_state(), make_state()
    step(make_state())  # warm-up: scratch, frame arrays and kernel attributes exist
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            step(graphed, stream=s)
    torch.cuda.synchronize()
    # the capture ran nothing: replay from the initial state
    graphed[0].copy_(_keys_dev(st0))
    graphed[1].zero_()
    graphed[2].zero_()
    for frame in range(3):
        step(eager)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(eager[4], graphed[4]), frame
        assert torch.equal(eager[0], graphed[0]) and torch.equal(eager[1], graphed[1])
