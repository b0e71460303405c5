"""The C-ABI library without a GPU: it loads, exports every symbol
include/d3s.h declares, its host-side key functions equal the oracle's, and
with no CUDA device it fails loudly instead of computing on the CPU."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "d3s.h").read_text()
    return sorted(set(re.findall(r"D3S_API\s+[\w\s\*]*?\b((?:d3s|d3)_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import d3s
    L = d3s.lib()
    names = declared_symbols()
    assert len(names) >= 15
    for name in names:
        assert hasattr(L, name), name
    assert sorted(d3s.EXPORTS) == names
    assert L.d3s_version() == 1


def test_request_struct_layout_matches_header(tmp_path):
    """ctypes' Request must match d3s_request's C layout: a C probe compiled
    against the header prints every field offset."""
    import subprocess

    import d3s
    fields = [f[0] for f in d3s.Request._fields_]
    src = tmp_path / "probe.c"
    body = "".join(f'printf("{f} %zu\\n", offsetof(d3s_request, {f}));' for f in fields)
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "d3s.h"\n'
                   f'int main(void){{{body} printf("size %zu\\n", sizeof(d3s_request)); return 0;}}\n')
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                      check=True).stdout.splitlines())
    for f in fields:
        assert getattr(d3s.Request, f).offset == int(out[f]), f
    assert ctypes.sizeof(d3s.Request) == int(out["size"])


@pytest.mark.parametrize("seed", [0, 1, 42, 2 ** 32 + 5, 2 ** 64 - 1])
def test_keys_equal_oracle(oracle, seed):
    import d3s
    k = d3s.key_from_seed(seed)
    assert k.tolist() == oracle.key_from_seed(seed).tolist()
    a, b = d3s.key_split(k)
    o0, o1 = oracle.split(oracle.key_from_seed(seed))
    assert a.tolist() == o0.tolist() and b.tolist() == o1.tolist()
    state = d3s.Key()
    d3s.seed(seed, state)
    ostate = oracle.key_from_seed(seed)
    for _ in range(5):
        assert d3s.next_key(state).tolist() == oracle.next_key(ostate).tolist()
        assert state.tolist() == ostate.tolist()


def test_global_key_sequence():
    import d3s
    d3s.seed(99)
    a = d3s.next_key()
    b = d3s.next_key()
    s = d3s.key_from_seed(99)
    assert a.tolist() == d3s.next_key(s).tolist() and b.tolist() == d3s.next_key(s).tolist()


def test_no_cpu_fallback_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import d3s
    x = np.zeros((2, 64), np.float32)
    out = d3s.lib()
    ids = np.full(2, 7, np.int32)
    out.d3_sample(x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 2, 64, 1.0, 5, 0.9, 1,
                  ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    assert out.d3s_last_status() != d3s.D3S_OK
    assert (ids == -1).all()
    with pytest.raises(d3s.D3SError):
        d3s.Context(0)


def test_new_entry_points_check_their_arguments_before_any_device_work():
    """Argument errors come back as codes without touching a device: the
    allocation-free entry point's row limit, the gather's world / rank / slots,
    and the kernel-path test hook's range."""
    import d3s
    L = d3s.lib()
    vp = ctypes.c_void_p
    rc = L.d3s_sample_rows_static(vp(16), d3s.F32, d3s.STATIC_MAX_ROWS + 1, 8, 8, vp(16), vp(16),
                                  vp(16), vp(16), vp(16), None)
    assert rc == d3s.D3S_ERR_UNSUPPORTED
    assert L.d3s_sample_rows_static(None, d3s.F32, -1, 8, 8, None, None, None, None, None,
                                    None) == d3s.D3S_ERR_ARG
    assert L.d3s_sample_rows_static(None, 7, 1, 8, 8, None, None, None, None, None,
                                    None) == d3s.D3S_ERR_ARG
    assert L.d3s_sample_rows_static(None, d3s.F32, 0, 8, 8, None, None, None, None, None,
                                    None) == d3s.D3S_OK
    g = vp()
    for world, rank, rows, slots in [(0, 0, 8, 2), (2, 2, 8, 2), (2, -1, 8, 2), (2, 0, -1, 2),
                                     (2, 0, 8, 1), (2, 0, 8, 65)]:
        assert L.d3s_gather_create(0, world, rank, rows, slots, ctypes.byref(g)) == d3s.D3S_ERR_ARG
        assert not g.value
    for bad in (-1, 2, 5, 100):
        with pytest.raises(d3s.D3SError):
            d3s.force_path(bad)
    d3s.force_path(d3s.PATH_AUTO)
