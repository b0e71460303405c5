"""ctypes loader for the CPU oracle (d3s_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the
checker and by bench.py's CPU-baseline / reference arm. The product path never
imports this module.

The library is built in-tree into oracle/_build/ (gcc, OpenMP, no FP
contraction). A build for x86-64-v3 (AVX2 + FMA) is used when the host CPU has
those features, otherwise a baseline x86-64 build; both give identical results
because every float operation is written out and rounds once.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "d3s_oracle.c"
HDR = HERE / "d3s_oracle.h"
BUILD = HERE / "_build"

F32 = 0
BF16 = 1


def _cpu_has_v3() -> bool:
    try:
        flags = Path("/proc/cpuinfo").read_text()
    except OSError:
        return False
    return all(f" {f}" in flags for f in ("avx2", "fma", "bmi2"))


def lib_path() -> Path:
    return BUILD / ("libd3s_oracle_v3.so" if _cpu_has_v3() else "libd3s_oracle_base.so")


def _src_hash() -> str:
    return hashlib.sha256(SRC.read_bytes() + HDR.read_bytes() + Path(__file__).read_bytes()).hexdigest()


def build(force: bool = False) -> Path:
    """Compile the oracle if its .so is missing or was built from other sources."""
    out = lib_path()
    stamp = out.with_name(out.name + ".srchash")
    if not force and out.exists() and stamp.exists() and stamp.read_text().strip() == _src_hash():
        return out
    BUILD.mkdir(exist_ok=True)
    march = "-march=x86-64-v3" if "v3" in out.name else "-march=x86-64"
    tmp = out.with_suffix(f".so.tmp{os.getpid()}")
    cmd = ["gcc", "-O3", "-std=c11", march, "-ffp-contract=off", "-fno-fast-math", "-fopenmp",
           "-fPIC", "-shared", "-Wall", "-Wno-unknown-pragmas", str(SRC), "-o", str(tmp), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    stamp.write_text(_src_hash() + "\n")
    return out


_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_u64p = ctypes.POINTER(ctypes.c_uint64)


class Diag(ctypes.Structure):
    _fields_ = [("gmax", ctypes.c_float), ("lse", ctypes.c_float), ("sum_fixed", ctypes.c_uint64),
                ("kept", ctypes.c_int), ("choice", ctypes.c_int), ("cum_margin", ctypes.c_float),
                ("race_gap", ctypes.c_float), ("bad", ctypes.c_int)]


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(build()))
        L.d3o_threefry2x32.argtypes = [_u32p, _u32p, _u32p]
        L.d3o_key_from_seed.argtypes = [ctypes.c_uint64, _u32p]
        L.d3o_split.argtypes = [_u32p, _u32p, _u32p]
        L.d3o_next_key.argtypes = [_u32p, _u32p]
        L.d3o_bits_word.restype = ctypes.c_uint32
        L.d3o_bits_word.argtypes = [_u32p, ctypes.c_uint64, ctypes.c_uint64]
        L.d3o_bits.argtypes = [_u32p, ctypes.c_uint64, _u32p]
        L.d3o_bits_to_uniform.restype = ctypes.c_float
        L.d3o_bits_to_uniform.argtypes = [ctypes.c_uint32]
        L.d3o_uniform.argtypes = [_u32p, ctypes.c_uint64, _f32p]
        L.d3o_exp.restype = ctypes.c_float
        L.d3o_exp.argtypes = [ctypes.c_float]
        L.d3o_log.restype = ctypes.c_float
        L.d3o_log.argtypes = [ctypes.c_float]
        L.d3o_exp_array.argtypes = [_f32p, _f32p, ctypes.c_int64]
        L.d3o_log_array.argtypes = [_f32p, _f32p, ctypes.c_int64]
        L.d3o_term_array.argtypes = [_f32p, _f32p, ctypes.c_int64]
        L.d3o_sample_row.restype = ctypes.c_int
        L.d3o_sample_row.argtypes = [_f32p, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                     ctypes.c_int, _f32p, _i32p, _f32p, ctypes.POINTER(Diag)]
        L.d3o_topk_metal_order.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, _i32p]
        L.d3o_topk_stable.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, _i32p]
        L.d3o_sample_with_noise.restype = ctypes.c_int
        L.d3o_sample_with_noise.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int64, _f32p, ctypes.c_int, ctypes.c_float,
                                            ctypes.c_float, _i32p, ctypes.c_int]
        L.d3o_sample_top_k_top_p.restype = ctypes.c_int
        L.d3o_sample_top_k_top_p.argtypes = [_u32p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                                             ctypes.c_int, ctypes.c_float, _i32p, ctypes.c_int]
        L.d3o_d3_sample.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                    ctypes.c_float, ctypes.c_uint64, _i32p]
        L.d3o_sample_rows.restype = ctypes.c_int
        L.d3o_sample_rows.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int64, _f32p, _f32p, _i32p, _u64p, ctypes.c_float,
                                      ctypes.c_float, ctypes.c_int, ctypes.c_uint64, _i32p,
                                      ctypes.c_int]
        L.d3o_frame_noise.argtypes = [_u32p, ctypes.c_int, _i32p, _f32p]
        L.d3o_sample_rows_keys.restype = ctypes.c_int
        L.d3o_sample_rows_keys.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int64, _f32p, _f32p, _i32p, ctypes.c_float,
                                           ctypes.c_float, ctypes.c_int, _u32p, ctypes.c_int64,
                                           _i32p, ctypes.c_int]
        L.d3o_frame_main.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                     ctypes.c_float, ctypes.c_int, _u32p, _u32p, _i32p,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     _i32p, _i32p, _i32p]
        L.d3o_row_cums.restype = ctypes.c_int
        L.d3o_row_cums.argtypes = [_f32p, ctypes.c_int, ctypes.c_float, ctypes.c_int, _f32p]
        L.d3o_exp_max_relerr.restype = ctypes.c_double
        L.d3o_exp_max_relerr.argtypes = [ctypes.c_float, ctypes.c_float]
        L.d3o_log_nonmonotone.restype = ctypes.c_int64
        L.d3o_log_nonmonotone.argtypes = [ctypes.c_float, ctypes.c_float]
        L.d3o_history_push.argtypes = [_i32p, ctypes.POINTER(ctypes.c_int), ctypes.c_int32]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


def _key(key) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(key, dtype=np.uint32).reshape(2))


# ---- random numbers ----

def threefry(key, ctr) -> tuple[int, int]:
    k, c, o = _key(key), _key(ctr), np.zeros(2, np.uint32)
    lib().d3o_threefry2x32(_p(k, _u32p), _p(c, _u32p), _p(o, _u32p))
    return int(o[0]), int(o[1])


def key_from_seed(seed: int) -> np.ndarray:
    k = np.zeros(2, np.uint32)
    lib().d3o_key_from_seed(seed, _p(k, _u32p))
    return k


def split(key) -> tuple[np.ndarray, np.ndarray]:
    k = _key(key)
    k0, k1 = np.zeros(2, np.uint32), np.zeros(2, np.uint32)
    lib().d3o_split(_p(k, _u32p), _p(k0, _u32p), _p(k1, _u32p))
    return k0, k1


def next_key(state: np.ndarray) -> np.ndarray:
    """Advance state (uint32[2], in place) and return the subkey."""
    assert state.dtype == np.uint32 and state.flags.c_contiguous
    sub = np.zeros(2, np.uint32)
    lib().d3o_next_key(_p(state, _u32p), _p(sub, _u32p))
    return sub


def bits(key, n: int) -> np.ndarray:
    k = _key(key)
    out = np.zeros(n, np.uint32)
    lib().d3o_bits(_p(k, _u32p), n, _p(out, _u32p))
    return out


def uniform(key, n: int) -> np.ndarray:
    k = _key(key)
    out = np.zeros(n, np.float32)
    lib().d3o_uniform(_p(k, _u32p), n, _p(out, _f32p))
    return out


def bits_to_uniform(b: np.ndarray) -> np.ndarray:
    L = lib()
    return np.array([L.d3o_bits_to_uniform(int(x)) for x in np.asarray(b).ravel()], np.float32)


# ---- math ----

def exp(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().d3o_exp_array(_p(x, _f32p), _p(y, _f32p), x.size)
    return y


def log(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().d3o_log_array(_p(x, _f32p), _p(y, _f32p), x.size)
    return y


def exp_term(x: np.ndarray) -> np.ndarray:
    """The full-row-sum term exp(max(d, -86))."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().d3o_term_array(_p(x, _f32p), _p(y, _f32p), x.size)
    return y


# ---- sampler ----

def _logits(logits: np.ndarray):
    if logits.dtype == np.float32:
        return np.ascontiguousarray(logits), F32
    if logits.dtype == np.uint16:  # raw bfloat16 bits
        return np.ascontiguousarray(logits), BF16
    raise TypeError("logits must be float32 or uint16 (bfloat16 bits)")


def sample_row(x: np.ndarray, temperature: float, top_p: float, k: int, u: np.ndarray):
    """One row: returns (id, topk_ids [k], probs [k], Diag)."""
    x = np.ascontiguousarray(x, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    assert u.size >= k
    ids = np.zeros(k, np.int32)
    probs = np.zeros(k, np.float32)
    d = Diag()
    r = lib().d3o_sample_row(_p(x, _f32p), x.size, temperature, top_p, k, _p(u, _f32p),
                             _p(ids, _i32p), _p(probs, _f32p), ctypes.byref(d))
    return r, ids, probs, d


def row_cums(x: np.ndarray, temperature: float, k: int) -> np.ndarray:
    """The inclusive cumsums [k] the top-p rule compares with top_p (no cut)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(k, np.float32)
    rc = lib().d3o_row_cums(_p(x, _f32p), x.size, temperature, k, _p(out, _f32p))
    assert rc == 0, "non-finite row"
    return out


def exp_max_relerr(lo: float, hi: float) -> float:
    """Largest relative error of the oracle's exp over every float in [lo, hi] (<= 0)."""
    return float(lib().d3o_exp_max_relerr(lo, hi))


def log_nonmonotone(lo: float, hi: float) -> int:
    """Adjacent float pairs in [lo, hi) where the oracle's log decreases."""
    return int(lib().d3o_log_nonmonotone(lo, hi))


def topk_stable(q: np.ndarray, k: int):
    q = np.ascontiguousarray(q, np.float32)
    v, i = np.zeros(k, np.float32), np.zeros(k, np.int32)
    lib().d3o_topk_stable(_p(q, _f32p), q.size, k, _p(v, _f32p), _p(i, _i32p))
    return v, i


def topk_metal_order(q: np.ndarray, k: int):
    q = np.ascontiguousarray(q, np.float32)
    v, i = np.zeros(k, np.float32), np.zeros(k, np.int32)
    lib().d3o_topk_metal_order(_p(q, _f32p), q.size, k, _p(v, _f32p), _p(i, _i32p))
    return v, i


def sample_with_noise(logits: np.ndarray, u: np.ndarray, temperature: float, top_p: float,
                      nthreads: int = 0) -> np.ndarray:
    lg, dt = _logits(logits)
    N, V = lg.shape
    u = np.ascontiguousarray(u, np.float32)
    assert u.shape[0] == N
    ids = np.zeros(N, np.int32)
    lib().d3o_sample_with_noise(lg.ctypes.data, dt, N, V, V, _p(u, _f32p), u.shape[1],
                                temperature, top_p, _p(ids, _i32p), nthreads)
    return ids


def sample_top_k_top_p(state: np.ndarray, logits: np.ndarray, temperature: float, top_k: int,
                       top_p: float, nthreads: int = 0) -> np.ndarray:
    lg, dt = _logits(logits)
    N, V = lg.shape
    ids = np.zeros(N, np.int32)
    lib().d3o_sample_top_k_top_p(_p(state, _u32p), lg.ctypes.data, dt, N, V, V, temperature,
                                 top_k, top_p, _p(ids, _i32p), nthreads)
    return ids


def d3_sample(logits: np.ndarray, temperature, top_k, top_p, seed) -> np.ndarray:
    """Mirror of the reference's tests/d3.py sample(): d3_sample on host arrays."""
    logits = np.ascontiguousarray(logits, np.float32)
    out = np.zeros(len(logits), np.int32)
    lib().d3o_d3_sample(_p(logits, _f32p), logits.shape[0], logits.shape[1], temperature, top_k,
                        top_p, seed, _p(out, _i32p))
    return out


def sample_rows(logits: np.ndarray, temperature, top_p, top_k, seeds, nthreads: int = 0,
                rows: int | None = None) -> np.ndarray:
    """Per-row parameters (arrays, or scalars for every row) and per-row seeds.
    `rows` limits the call to the first rows (a bounded sample)."""
    lg, dt = _logits(logits)
    N, V = lg.shape
    if rows is not None:
        N = min(N, rows)

    def arr(x, dtype):
        if np.isscalar(x):
            return None, x
        return np.ascontiguousarray(np.asarray(x, dtype)[:N]), 0

    T, T0 = arr(temperature, np.float32)
    P, P0 = arr(top_p, np.float32)
    K, K0 = arr(top_k, np.int32)
    S, S0 = arr(seeds, np.uint64)
    ids = np.zeros(N, np.int32)
    lib().d3o_sample_rows(lg.ctypes.data, dt, N, V, V, _p(T, _f32p), _p(P, _f32p), _p(K, _i32p),
                          _p(S, _u64p), float(T0), float(P0), int(K0), int(S0), _p(ids, _i32p),
                          nthreads)
    return ids


def frame_noise(state: np.ndarray, ks) -> np.ndarray:
    ks = np.ascontiguousarray(ks, np.int32)
    u = np.zeros(int(ks.sum()), np.float32)
    lib().d3o_frame_noise(_p(state, _u32p), len(ks), _p(ks, _i32p), _p(u, _f32p))
    return u


def sample_rows_keys(logits: np.ndarray, temperature, top_p, top_k, keys: np.ndarray,
                     nthreads: int = 0) -> np.ndarray:
    """Per-row keys: keys uint32 [N, 2] (or [N, m, 2]: column 0 of each row is
    used, as a key array with ld_keys = m). Parameters are arrays or scalars."""
    lg, dt = _logits(logits)
    N, V = lg.shape
    keys = np.ascontiguousarray(keys, np.uint32)
    ld_keys = 1 if keys.ndim == 2 else keys.shape[1]

    def arr(x, dtype):
        if np.isscalar(x):
            return None, x
        return np.ascontiguousarray(np.asarray(x, dtype)[:N]), 0

    T, T0 = arr(temperature, np.float32)
    P, P0 = arr(top_p, np.float32)
    K, K0 = arr(top_k, np.int32)
    ids = np.zeros(N, np.int32)
    lib().d3o_sample_rows_keys(lg.ctypes.data, dt, N, V, V, _p(T, _f32p), _p(P, _f32p),
                               _p(K, _i32p), float(T0), float(P0), int(K0), _p(keys, _u32p),
                               ld_keys, _p(ids, _i32p), nthreads)
    return ids


RAS_WINDOW = 16
FRAME_EOS, FRAME_NONFINITE, FRAME_RETRY = 1, 2, 4


def frame_main(logits_row: np.ndarray, temperature: float, top_p: float, top_k: int, key_main,
               key_retry, history, semantic_start: int, code_vocab: int, eos_id: int):
    """tower_decode_step's sampling of one stream: (main_tok, c0, flags)."""
    lg, dt = _logits(np.asarray(logits_row).reshape(1, -1))
    V = lg.shape[1]
    h = np.ascontiguousarray(np.asarray(history, np.int32).reshape(-1))
    out = np.zeros(3, np.int32)
    lib().d3o_frame_main(lg.ctypes.data, dt, V, temperature, top_p, top_k, _p(_key(key_main), _u32p),
                         _p(_key(key_retry), _u32p), _p(h, _i32p), len(h), semantic_start,
                         code_vocab, eos_id, _p(out[0:1], _i32p), _p(out[1:2], _i32p),
                         _p(out[2:3], _i32p))
    return int(out[0]), int(out[1]), int(out[2])


def history_push(history: list, tok: int) -> list:
    """The decode loop's history window step (drop the oldest when full)."""
    h = list(history) + [int(tok)]
    return h[-RAS_WINDOW:]


def streams_next_keys(states: np.ndarray, n: int):
    """Advance each stream's key n times: (new states [S, 2], subkeys [S, n, 2])."""
    states = np.array(states, np.uint32).reshape(-1, 2)
    subs = np.zeros((states.shape[0], n, 2), np.uint32)
    for s in range(states.shape[0]):
        st = np.ascontiguousarray(states[s])
        for i in range(n):
            sub = np.zeros(2, np.uint32)
            lib().d3o_next_key(_p(st, _u32p), _p(sub, _u32p))
            subs[s, i] = sub
        states[s] = st
    return states, subs
