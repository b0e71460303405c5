"""ctypes binding of libd3s.so, the B200 sampler's C ABI (include/d3s.h).

The host-side mirror of drama3-mlx's sampling interface:
  - sample(logits, temperature, top_k, top_p, seed)   -> d3_sample (src/testapi.c:155-166),
    the call the reference's tests make through tests/d3.py:211-217;
  - Context.sample_top_k_top_p / sample_with_noise / sample_noise
    -> src/sampling.c:179-209 on CUDA tensors;
  - Context.sample_rows -> the batched engine (per-row parameters and seeds).

There is no CPU fallback: without the library or a CUDA device every call
raises. torch is used only to hold device memory and streams.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("D3S_LIB", PKG / "lib" / "libd3s.so"))

D3S_OK = 0
D3S_ERR_ARG = -1
D3S_ERR_CUDA = -2
D3S_ERR_NONFINITE = -3
D3S_ERR_UNSUPPORTED = -4
D3S_ERR_NOMEM = -5
F32 = 0
BF16 = 1
ROW_OK, ROW_NONFINITE, ROW_BADPARAM = 0, 1, 2
NOISE_KEY, NOISE_SEEDS, NOISE_GIVEN, NOISE_KEYS = 0, 1, 2, 3
MAX_V = 131072
MAX_K = 16384

# every symbol include/d3s.h declares
EXPORTS = ("d3s_version", "d3s_last_error", "d3s_key_from_seed", "d3s_key_split", "d3s_seed",
           "d3s_next_key", "d3s_ctx_create", "d3s_ctx_destroy", "d3s_ctx_reserve",
           "d3s_sample_noise", "d3s_sample_with_noise", "d3s_sample_top_k_top_p", "d3s_sample",
           "d3s_debug_math", "d3s_debug_div_check", "d3s_ctx_check", "d3s_sample_rows_static",
           "d3_sample", "d3s_last_status", "d3s_keys_next", "d3s_frame_main", "d3s_lmhead",
           "d3s_lmhead_sample", "d3s_codes_write_npy", "d3s_static_check",
           "d3s_static_debug_set_error", "d3s_gather_create", "d3s_gather_export",
           "d3s_gather_attach", "d3s_gather_begin", "d3s_gather_end", "d3s_gather_release",
           "d3s_gather_check", "d3s_gather_destroy", "d3s_gather_copy_result", "d3s_gather_line_up",
           "d3s_debug_force_path")
RAS_WINDOW = 16
FRAME_EOS, FRAME_NONFINITE, FRAME_RETRY = 1, 2, 4
STATIC_MAX_ROWS = 4096
GATHER_HANDLE_BYTES = 64


class D3SError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"d3s error {code}: {msg}")
        self.code = code


class Key(ctypes.Structure):
    _fields_ = [("k", ctypes.c_uint32 * 2)]

    def tolist(self):
        return [int(self.k[0]), int(self.k[1])]


class Request(ctypes.Structure):
    _fields_ = [
        ("logits", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("N", ctypes.c_int32),
        ("V", ctypes.c_int32), ("ld", ctypes.c_int64), ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float), ("top_k", ctypes.c_int32),
        ("temperature_rows", ctypes.c_void_p), ("top_p_rows", ctypes.c_void_p),
        ("top_k_rows", ctypes.c_void_p), ("noise", ctypes.c_int32), ("key", Key),
        ("seeds", ctypes.c_void_p), ("u", ctypes.c_void_p), ("ld_u", ctypes.c_int64),
        ("ids", ctypes.c_void_p), ("status", ctypes.c_void_p), ("kept", ctypes.c_void_p),
        ("probs", ctypes.c_void_p), ("topk_ids", ctypes.c_void_p), ("ld_out", ctypes.c_int64),
        ("keys", ctypes.c_void_p), ("ld_keys", ctypes.c_int64), ("finite", ctypes.c_void_p),
    ]


class FrameRequest(ctypes.Structure):
    _fields_ = [
        ("logits", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("S", ctypes.c_int32),
        ("V", ctypes.c_int32), ("ld", ctypes.c_int64), ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float), ("top_k", ctypes.c_int32), ("keys", ctypes.c_void_p),
        ("ld_keys", ctypes.c_int64), ("history", ctypes.c_void_p), ("hist_len", ctypes.c_void_p),
        ("semantic_start", ctypes.c_int32), ("code_vocab", ctypes.c_int32),
        ("eos_id", ctypes.c_int32), ("update_history", ctypes.c_int32),
        ("main_tok", ctypes.c_void_p), ("c0", ctypes.c_void_p), ("flags", ctypes.c_void_p),
    ]


_lib = None


def build() -> Path:
    import importlib.util
    spec = importlib.util.spec_from_file_location("d3s_build", PKG / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build()


def lib() -> ctypes.CDLL:
    """Load libd3s.so (building it first if the sources are newer)."""
    global _lib
    if _lib is None:
        if "D3S_LIB" not in os.environ:
            build()
        if not LIB_PATH.exists():
            raise D3SError(D3S_ERR_UNSUPPORTED, f"{LIB_PATH} is missing; run drama3-mlx_b200/build.py")
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i32, i64, f32, u64 = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                                  ctypes.c_uint64)
        kp = ctypes.POINTER(Key)
        L.d3s_version.restype = i32
        L.d3s_last_error.restype = ctypes.c_char_p
        L.d3s_key_from_seed.argtypes = [u64, kp]
        L.d3s_key_split.argtypes = [kp, kp, kp]
        L.d3s_seed.argtypes = [kp, u64]
        L.d3s_next_key.argtypes = [kp, kp]
        L.d3s_ctx_create.argtypes = [i32, ctypes.POINTER(vp)]
        L.d3s_ctx_destroy.argtypes = [vp]
        L.d3s_ctx_destroy.restype = None
        L.d3s_ctx_reserve.argtypes = [vp, i64]
        L.d3s_sample_noise.argtypes = [vp, kp, i32, i32, i32, vp, vp]
        L.d3s_sample_with_noise.argtypes = [vp, vp, i32, i32, i32, i64, vp, i32, i64, f32, f32, vp,
                                            vp]
        L.d3s_sample_top_k_top_p.argtypes = [vp, vp, i32, i32, i32, i64, f32, i32, f32, kp, vp, vp]
        L.d3s_sample.argtypes = [vp, ctypes.POINTER(Request), vp]
        L.d3s_debug_math.argtypes = [vp, i32, vp, vp, i64, f32, vp]
        L.d3s_debug_div_check.argtypes = [vp, vp, i32, u64, u64, u64, vp, vp, vp]
        L.d3s_ctx_check.argtypes = [vp]
        L.d3s_debug_force_path.argtypes = [i32]
        L.d3s_sample_rows_static.argtypes = [vp, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp]
        L.d3s_static_check.argtypes = [vp]
        L.d3s_gather_create.argtypes = [i32, i32, i32, i64, i32, ctypes.POINTER(vp)]
        L.d3s_gather_export.argtypes = [vp, vp]
        L.d3s_gather_attach.argtypes = [vp, vp]
        L.d3s_gather_begin.argtypes = [vp, i64, ctypes.POINTER(vp), vp]
        L.d3s_gather_end.argtypes = [vp, i64, ctypes.POINTER(vp), vp]
        L.d3s_gather_release.argtypes = [vp, i64, vp]
        L.d3s_gather_check.argtypes = [vp, vp]
        L.d3s_gather_copy_result.argtypes = [vp, i64, vp, vp]
        L.d3s_gather_line_up.argtypes = [vp, i64, vp]
        L.d3s_gather_destroy.argtypes = [vp]
        L.d3s_gather_destroy.restype = None
        L.d3s_static_debug_set_error.argtypes = [ctypes.c_int32, vp]
        L.d3_sample.argtypes = [ctypes.POINTER(ctypes.c_float), i32, i32, f32, i32, f32,
                                ctypes.c_ulonglong, ctypes.POINTER(ctypes.c_int32)]
        L.d3_sample.restype = None
        L.d3s_last_status.restype = i32
        L.d3s_keys_next.argtypes = [vp, vp, i32, i32, vp, i64, vp]
        L.d3s_frame_main.argtypes = [vp, ctypes.POINTER(FrameRequest), vp]
        L.d3s_lmhead.argtypes = [vp, vp, i64, vp, i64, i32, i32, i32, vp, i64, vp]
        L.d3s_codes_write_npy.argtypes = [ctypes.c_char_p, vp, i32, i32, i32]
        L.d3s_lmhead_sample.argtypes = [vp, vp, i64, vp, i64, i32, ctypes.POINTER(Request), vp]
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != D3S_OK:
        raise D3SError(rc, lib().d3s_last_error().decode())


# ---- keys (host) ----

def key_from_seed(seed: int) -> Key:
    k = Key()
    _check(lib().d3s_key_from_seed(seed, ctypes.byref(k)))
    return k


def key_split(key: Key) -> tuple[Key, Key]:
    a, b = Key(), Key()
    _check(lib().d3s_key_split(ctypes.byref(key), ctypes.byref(a), ctypes.byref(b)))
    return a, b


def seed(s: int, state: Key | None = None) -> None:
    """m_seed: seeds `state`, or the library's global key when None."""
    _check(lib().d3s_seed(ctypes.byref(state) if state is not None else None, s))


def next_key(state: Key | None = None) -> Key:
    sub = Key()
    _check(lib().d3s_next_key(ctypes.byref(state) if state is not None else None, ctypes.byref(sub)))
    return sub


def codes_write_npy(path, frames, n_codebooks: int) -> None:
    """Write the codes of a take (frames: int32 array [n_frames, 1 + n_codebooks
    or wider], column 0 the main token) as the reference's codes .npy."""
    import numpy as np
    fr = np.ascontiguousarray(frames, dtype=np.int32)
    _check(lib().d3s_codes_write_npy(str(path).encode(), fr.ctypes.data, fr.shape[0], fr.shape[1],
                                     n_codebooks))


def sample_rows_static(logits, ids, temperature, top_p, top_k, seeds, stream=None) -> None:
    """d3s_sample_rows_static on CUDA tensors: logits [N, V] (float32 or
    bfloat16, unit stride along V), and the per-row arrays, all required and
    contiguous on the logits' device: temperature and top_p float32 [N], top_k
    int32 [N], seeds int64 or uint64 [N], ids int32 [N] (written)."""
    import torch
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a [N, V] tensor with unit stride along V")
    N, V = logits.shape
    want = [("temperature", temperature, (torch.float32,)), ("top_p", top_p, (torch.float32,)),
            ("top_k", top_k, (torch.int32,)), ("seeds", seeds, (torch.int64, torch.uint64)),
            ("ids", ids, (torch.int32,))]
    for name, t, dtypes in want:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a tensor")
        if t.dtype not in dtypes:
            raise TypeError(f"{name} must be {' or '.join(map(str, dtypes))}, got {t.dtype}")
        if t.numel() != N or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous tensor of {N} elements")
        if t.device != logits.device:
            raise ValueError(f"{name} is on {t.device}, the logits on {logits.device}")
    _check(lib().d3s_sample_rows_static(_ptr(logits), _dtype_code(logits), N, V, logits.stride(0),
                                        _ptr(temperature), _ptr(top_p), _ptr(top_k), _ptr(seeds),
                                        _ptr(ids), _stream_ptr(stream)))


def static_check(stream=None) -> None:
    """d3s_static_check: waits for `stream`, raises D3SError if a
    d3s_sample_rows_static call since the last check recorded a failure."""
    _check(lib().d3s_static_check(_stream_ptr(stream)))


def static_debug_set_error(value: int, stream=None) -> None:
    """Test hook: set the static scratch's error word (no failure is caused)."""
    _check(lib().d3s_static_debug_set_error(value, _stream_ptr(stream)))


# ---- the reference's test entry point ----

def sample(logits: np.ndarray, temperature, top_k, top_p, seed) -> np.ndarray:
    """d3_sample on host arrays, as the reference's tests/d3.py sample() calls it."""
    L = lib()
    logits = np.ascontiguousarray(logits, np.float32)
    out = np.zeros(len(logits), np.int32)
    L.d3_sample(logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), logits.shape[0],
                logits.shape[1], temperature, top_k, top_p, seed,
                out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    rc = L.d3s_last_status()
    if rc not in (D3S_OK, D3S_ERR_NONFINITE):
        _check(rc)
    return out


PATH_AUTO, PATH_PAIR, PATH_ROWWARP, PATH_PAIR1W = 0, 1, 3, 4


def force_path(path: int) -> None:
    """Test hook: the kernel for batches above the small-batch path (PATH_*)."""
    _check(lib().d3s_debug_force_path(path))


def last_status() -> int:
    return lib().d3s_last_status()


# ---- device API on torch tensors ----

def _ptr(t) -> int | None:
    if t is None or isinstance(t, int):
        return t
    return t.data_ptr()


def _stream_ptr(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _dtype_code(t) -> int:
    import torch
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError(f"logits must be float32 or bfloat16, got {t.dtype}")


class Context:
    """A d3s_ctx on one CUDA device (scratch + staging)."""

    def __init__(self, device: int = 0):
        import torch
        if not torch.cuda.is_available():
            raise D3SError(D3S_ERR_CUDA, "no CUDA device: the sampler has no CPU path")
        self.device = device
        self._h = ctypes.c_void_p()
        _check(lib().d3s_ctx_create(device, ctypes.byref(self._h)))

    def close(self) -> None:
        if self._h:
            lib().d3s_ctx_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reserve(self, max_rows: int) -> None:
        _check(lib().d3s_ctx_reserve(self._h, max_rows))

    def sample(self, req: Request, stream=None) -> None:
        _check(lib().d3s_sample(self._h, ctypes.byref(req), _stream_ptr(stream)))

    def request(self, logits, ids, *, temperature=1.0, top_p=1.0, top_k=1, temperature_rows=None,
                top_p_rows=None, top_k_rows=None, noise=NOISE_KEY, key: Key | None = None,
                seeds=None, u=None, status=None, kept=None, probs=None, topk_ids=None,
                keys=None, finite=None) -> Request:
        """keys: int32/uint32 device tensor [N, 2] (or [N, m, 2]: column 0 of
        each row is used) for NOISE_KEYS."""
        N, V = logits.shape
        r = Request()
        r.logits = _ptr(logits)
        r.dtype = _dtype_code(logits)
        r.N, r.V, r.ld = N, V, logits.stride(0)
        r.temperature, r.top_p, r.top_k = float(temperature), float(top_p), int(top_k)
        r.temperature_rows = _ptr(temperature_rows)
        r.top_p_rows = _ptr(top_p_rows)
        r.top_k_rows = _ptr(top_k_rows)
        r.noise = noise
        if key is not None:
            r.key = key
        r.seeds = _ptr(seeds)
        r.u = _ptr(u)
        r.ld_u = u.stride(0) if u is not None else 0
        r.ids = _ptr(ids)
        r.status = _ptr(status)
        r.kept = _ptr(kept)
        r.probs = _ptr(probs)
        r.topk_ids = _ptr(topk_ids)
        out = probs if probs is not None else topk_ids
        r.ld_out = out.stride(0) if out is not None else 0
        r.keys = _ptr(keys)
        r.ld_keys = (keys.stride(0) // 2) if keys is not None else 0
        r.finite = _ptr(finite)
        return r

    def sample_top_k_top_p(self, logits, temperature: float, top_k: int, top_p: float,
                           state: Key | None = None, ids=None, stream=None):
        import torch
        N, V = logits.shape
        if ids is None:
            ids = torch.empty(N, dtype=torch.int32, device=logits.device)
        _check(lib().d3s_sample_top_k_top_p(self._h, _ptr(logits), _dtype_code(logits), N, V,
                                            logits.stride(0), temperature, top_k, top_p,
                                            ctypes.byref(state) if state is not None else None,
                                            _ptr(ids), _stream_ptr(stream)))
        return ids

    def sample_with_noise(self, logits, u, temperature: float, top_p: float, ids=None,
                          stream=None):
        import torch
        N, V = logits.shape
        if ids is None:
            ids = torch.empty(N, dtype=torch.int32, device=logits.device)
        _check(lib().d3s_sample_with_noise(self._h, _ptr(logits), _dtype_code(logits), N, V,
                                           logits.stride(0), _ptr(u), u.shape[1], u.stride(0),
                                           temperature, top_p, _ptr(ids), _stream_ptr(stream)))
        return ids

    def sample_noise(self, rows: int, V: int, top_k: int, state: Key | None = None, stream=None):
        import torch
        k = min(top_k, V)
        u = torch.empty(rows, k, dtype=torch.float32, device=f"cuda:{self.device}")
        _check(lib().d3s_sample_noise(self._h, ctypes.byref(state) if state is not None else None,
                                      rows, V, top_k, _ptr(u), _stream_ptr(stream)))
        return u

    def sample_rows(self, logits, ids, *, temperature, top_p, top_k, seeds, status=None,
                    kept=None, stream=None) -> None:
        """Per-row parameters (tensors or scalars) and per-row seeds (int64 tensor).
        ids: an int32 tensor of N, or a raw device address of N int32 (the
        slot a Gather gives, which may be another GPU's memory)."""
        import torch

        def split(x):
            return (x, 0) if isinstance(x, torch.Tensor) else (None, x)

        T, T0 = split(temperature)
        P, P0 = split(top_p)
        K, K0 = split(top_k)
        req = self.request(logits, ids, temperature=T0, top_p=P0, top_k=K0 or 1,
                           temperature_rows=T, top_p_rows=P, top_k_rows=K, noise=NOISE_SEEDS,
                           seeds=seeds, status=status, kept=kept)
        self.sample(req, stream)

    def sample_rows_keys(self, logits, ids, keys, *, temperature, top_p, top_k, status=None,
                         finite=None, stream=None) -> None:
        """Per-row keys (a stream's subkey per row: int32 tensor [N, 2] or
        [N, m, 2]) and per-row or scalar parameters."""
        import torch

        def split(x):
            return (x, 0) if isinstance(x, torch.Tensor) else (None, x)

        T, T0 = split(temperature)
        P, P0 = split(top_p)
        K, K0 = split(top_k)
        req = self.request(logits, ids, temperature=T0, top_p=P0, top_k=K0 or 1,
                           temperature_rows=T, top_p_rows=P, top_k_rows=K, noise=NOISE_KEYS,
                           keys=keys, status=status, finite=finite)
        self.sample(req, stream)

    def keys_next(self, states, n: int, sub=None, stream=None):
        """Advance each stream's key (int32 device tensor [S, 2], in place) n
        times; returns the subkeys [S, n, 2] in draw order."""
        import torch
        S = states.shape[0]
        if sub is None:
            sub = torch.empty(S, n, 2, dtype=torch.int32, device=states.device)
        _check(lib().d3s_keys_next(self._h, _ptr(states), S, n, _ptr(sub), sub.stride(0) // 2,
                                   _stream_ptr(stream)))
        return sub

    def frame_main(self, logits, sub, history, hist_len, *, temperature: float, top_p: float,
                   top_k: int, semantic_start: int, code_vocab: int, eos_id: int,
                   update_history: bool = True, stream=None):
        """tower_decode_step's main + retry draws for S streams: logits [S, V]
        device, sub [S, n, 2] (the frame's subkeys: 0 main, 1 retry), history
        int32 [S, RAS_WINDOW], hist_len int32 [S]. Returns (main_tok, c0, flags)."""
        import torch
        S, V = logits.shape
        dev = logits.device
        main_tok = torch.empty(S, dtype=torch.int32, device=dev)
        c0 = torch.empty(S, dtype=torch.int32, device=dev)
        flags = torch.empty(S, dtype=torch.int32, device=dev)
        f = FrameRequest()
        f.logits = _ptr(logits)
        f.dtype = _dtype_code(logits)
        f.S, f.V, f.ld = S, V, logits.stride(0)
        f.temperature, f.top_p, f.top_k = float(temperature), float(top_p), int(top_k)
        f.keys = _ptr(sub)
        f.ld_keys = sub.stride(0) // 2
        f.history = _ptr(history)
        f.hist_len = _ptr(hist_len)
        f.semantic_start, f.code_vocab, f.eos_id = semantic_start, code_vocab, eos_id
        f.update_history = 1 if update_history else 0
        f.main_tok, f.c0, f.flags = _ptr(main_tok), _ptr(c0), _ptr(flags)
        _check(lib().d3s_frame_main(self._h, ctypes.byref(f), _stream_ptr(stream)))
        return main_tok, c0, flags

    def lmhead(self, h, W, out=None, stream=None):
        """logits [B, V] bf16 = bf16(h [B, D] @ W [V, D]^T), fp32 accumulation."""
        import torch
        B, D = h.shape
        V = W.shape[0]
        if out is None:
            out = torch.empty(B, V, dtype=torch.bfloat16, device=h.device)
        _check(lib().d3s_lmhead(self._h, _ptr(h), h.stride(0), _ptr(W), W.stride(0), B, V, D,
                                _ptr(out), out.stride(0), _stream_ptr(stream)))
        return out

    def lmhead_sample(self, h, W, logits, ids, stream=None, **request):
        """d3s_lmhead into `logits` (bf16 [B, V]) then d3s_sample; keyword
        arguments as for request()."""
        req = self.request(logits, ids, **request)
        _check(lib().d3s_lmhead_sample(self._h, _ptr(h), h.stride(0), _ptr(W), W.stride(0),
                                       h.shape[1], ctypes.byref(req), _stream_ptr(stream)))

    def check(self) -> None:
        """Synchronise and raise if a kernel recorded a failure (a bounded wait)."""
        _check(lib().d3s_ctx_check(self._h))

    def debug_math(self, op: int, x, param: float = 1.0, stream=None):
        import torch
        y = torch.empty_like(x)
        _check(lib().d3s_debug_math(self._h, op, _ptr(x), _ptr(y), x.numel(), param,
                                    _stream_ptr(stream)))
        return y

    def debug_div_check(self, Ts, lo: int = 0, hi: int = 1 << 32, step: int = 1, stream=None):
        """(mismatch count, example (x, T)) of the reciprocal-path division."""
        import torch
        bad = torch.zeros(1, dtype=torch.int64, device=Ts.device)
        ex = torch.zeros(2, dtype=torch.float32, device=Ts.device)
        _check(lib().d3s_debug_div_check(self._h, _ptr(Ts), Ts.numel(), lo, hi, step, _ptr(bad),
                                         _ptr(ex), _stream_ptr(stream)))
        torch.cuda.synchronize()
        return int(bad.item()), ex.cpu().tolist()


class Gather:
    """d3s_gather: the ids of rows sharded over the ranks of one node written
    straight into rank 0's result by each rank's sampler (NVLink peer stores),
    with a completion counter in rank 0's memory. `exchange(handle or None)`
    is the caller's channel for rank 0's 64-byte IPC handle: it is called once
    on every rank with rank 0's handle (bytes) on rank 0 and None elsewhere,
    and returns rank 0's handle on every rank."""

    def __init__(self, device: int, world: int, rank: int, rows: int, exchange, slots: int = 2):
        self.rank, self.world, self.rows, self.slots = rank, world, rows, slots
        self._h = ctypes.c_void_p()
        _check(lib().d3s_gather_create(device, world, rank, rows, slots, ctypes.byref(self._h)))
        try:
            mine = None
            if rank == 0:
                buf = ctypes.create_string_buffer(GATHER_HANDLE_BYTES)
                _check(lib().d3s_gather_export(self._h, buf))
                mine = buf.raw
            handle = exchange(mine)
            if rank != 0:
                buf = ctypes.create_string_buffer(bytes(handle), GATHER_HANDLE_BYTES)
                _check(lib().d3s_gather_attach(self._h, buf))
        except Exception:
            self.close()
            raise

    def begin(self, step: int, stream=None) -> int:
        """Device address where this rank's sampler writes the ids of its rows at `step`."""
        p = ctypes.c_void_p()
        _check(lib().d3s_gather_begin(self._h, step, ctypes.byref(p), _stream_ptr(stream)))
        return int(p.value)

    def end(self, step: int, stream=None) -> int | None:
        """After the sampler: signal (ranks > 0) or wait for every rank (rank 0).
        Rank 0 gets the device address of the step's N ids."""
        p = ctypes.c_void_p()
        _check(lib().d3s_gather_end(self._h, step, ctypes.byref(p), _stream_ptr(stream)))
        return int(p.value) if p.value else None

    def release(self, step: int, stream=None) -> None:
        _check(lib().d3s_gather_release(self._h, step, _stream_ptr(stream)))

    def line_up(self, line: int, stream=None) -> None:
        """d3s_gather_line_up: the stream waits until every rank's stream has
        reached its line-th start line (line counts from 1 on every rank)."""
        _check(lib().d3s_gather_line_up(self._h, line, _stream_ptr(stream)))

    def copy_result(self, step: int, out, stream=None):
        """Rank 0: the N ids of `step` into `out` (int32 CUDA tensor of N), on the stream."""
        if out.dtype.itemsize != 4 or out.numel() != self.rows or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous int32 tensor of {self.rows} ids")
        _check(lib().d3s_gather_copy_result(self._h, step, _ptr(out), _stream_ptr(stream)))
        return out

    def check(self, stream=None) -> None:
        _check(lib().d3s_gather_check(self._h, _stream_ptr(stream)))

    def close(self) -> None:
        if self._h:
            lib().d3s_gather_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
