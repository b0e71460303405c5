"""The codes .npy output (d3s_codes_write_npy) on the host: the file is
byte-identical to numpy's own .npy of the int64 codes array, i.e. the format
npy_write_codes writes (src/npy.c:98-129), and the codes are the codebook
columns of the frame rows (src/generate.c:162-168)."""

import numpy as np
import pytest


@pytest.mark.parametrize("n_frames,n_codebooks,width", [(0, 10, 11), (1, 10, 11), (37, 10, 11),
                                                        (500, 4, 6), (3, 1, 2)])
def test_codes_npy_matches_numpy(tmp_path, n_frames, n_codebooks, width):
    import d3s
    rng = np.random.default_rng(n_frames + width)
    frames = rng.integers(-5, 5000, (n_frames, width)).astype(np.int32)
    path = tmp_path / "codes.npy"
    d3s.codes_write_npy(path, frames, n_codebooks)
    codes = frames[:, 1:1 + n_codebooks].T.astype(np.int64)  # codes[k][t] = frames[t][1 + k]
    ref = tmp_path / "ref.npy"
    np.save(ref, np.ascontiguousarray(codes))
    assert path.read_bytes() == ref.read_bytes()
    assert (len(path.read_bytes()) - 8 * codes.size) % 64 == 0
    np.testing.assert_array_equal(np.load(path), codes)


def test_codes_npy_rejects_bad_arguments(tmp_path):
    import d3s
    with pytest.raises(d3s.D3SError):
        d3s.codes_write_npy(tmp_path / "x.npy", np.zeros((2, 3), np.int32), 5)  # width < 1 + 5
    with pytest.raises(d3s.D3SError):
        d3s.codes_write_npy(tmp_path / "no_such_dir" / "x.npy", np.zeros((2, 11), np.int32), 10)
