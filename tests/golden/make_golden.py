"""Writes the golden fixtures under tests/golden/.

    python tests/golden/make_golden.py

known_answers.json - published known-answer vectors (not generated):
  * Threefry-2x32 with 20 rounds: the Random123 distribution's kat_vectors
    file (Salmon et al., SC'11), lines "threefry2x32 20 <ctr0> <ctr1> <key0>
    <key1> <out0> <out1>".
  * The split of key 0 as JAX documents it (jax.random.split(PRNGKey(0))
    -> [[4146024105, 967050713], [2718843009, 1272950319]]); MLX's
    random::split uses the same threefry counter layout.

oracle_cases.npz - regression fixtures of the CPU oracle on small seeded inputs
(the reference's own tests hold no golden ids, so these freeze the restatement
against accidental change; the oracle is itself checked against the published
vectors above and against the definitions in the reference's tests).
"""

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))

KNOWN = {
    "threefry2x32_20": [
        # ctr, key, out
        {"ctr": [0x00000000, 0x00000000], "key": [0x00000000, 0x00000000], "out": [0x6b200159, 0x99ba4efe]},
        {"ctr": [0xffffffff, 0xffffffff], "key": [0xffffffff, 0xffffffff], "out": [0x1cb996fc, 0xbb002be7]},
        {"ctr": [0x243f6a88, 0x85a308d3], "key": [0x13198a2e, 0x03707344], "out": [0xc4923a9c, 0x483df7a0]},
    ],
    "split_key0": {"key": [0, 0], "k0": [4146024105, 967050713], "k1": [2718843009, 1272950319]},
}


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest even) and return the raw uint16 bits."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return b.astype(np.uint16)


def cases():
    import oracle as o
    out = {}
    rng = np.random.default_rng(20261201)
    # d3_sample on f32 rows (configs 1 and 5 shapes, small N)
    x = (rng.standard_normal((8, 4097)) * 3).astype(np.float32)
    x[np.arange(8), rng.integers(1, 4097, 8)] += 6.0
    out["d3_logits"] = x
    params = [(0.7, 30, 0.7), (1.0, 30, 0.9), (1.0, 5, 1.0), (0.3, 30, 0.95), (1.2, 64, 0.5)]
    out["d3_params"] = np.array(params, np.float64)
    out["d3_ids"] = np.stack([np.stack([o.d3_sample(x, T, k, p, s) for s in range(4)])
                              for (T, k, p) in params])
    # bf16 rows, per-row seeds (config 2 shape, small N)
    xb = (rng.standard_normal((16, 4097)) * 2).astype(np.float32)
    xb[:, 0] = rng.normal(-4, 1, 16)
    out["rows_bf16"] = bf16_bits(xb)
    out["rows_seeds"] = np.arange(1000, 1016, dtype=np.uint64)
    out["rows_ids"] = o.sample_rows(out["rows_bf16"], 0.7, 0.7, 30, out["rows_seeds"])
    # uniform words: even and odd counts
    key = o.split(o.key_from_seed(7))[1]
    out["uniform_key"] = key
    out["uniform_5"] = o.uniform(key, 5)
    out["uniform_30"] = o.uniform(key, 30)
    out["bits_7"] = o.bits(key, 7)
    return out


def main():
    (HERE / "known_answers.json").write_text(json.dumps(KNOWN, indent=1) + "\n")
    np.savez_compressed(HERE / "oracle_cases.npz", **cases())
    print("wrote", HERE / "known_answers.json", HERE / "oracle_cases.npz")


if __name__ == "__main__":
    main()
