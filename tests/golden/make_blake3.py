"""Writes blake3_vectors.json: BLAKE3 digests of seeded byte strings, computed with the
`blake3` Python package (bindings to the BLAKE3 team's Rust crate, the implementation the
reference's SMT code calls: model-lab Cargo.lock pins blake3 1.8.7). The lengths cover the
block (64 B) and chunk (1 KiB) boundaries, uneven trees and inputs past 1 MiB, where the
library hashes subtrees on several threads.

Run from the repository root: python -m tests.golden.make_blake3
"""
from __future__ import annotations

import json
import os

import numpy as np

LENGTHS = [0, 1, 2, 63, 64, 65, 127, 128, 129, 1023, 1024, 1025, 2047, 2048, 2049, 3072, 3073,
           4096, 4097, 5120, 7168, 8191, 8192, 8193, 16384, 31744, 65537, 102400,
           (1 << 20) - 1, 1 << 20, (1 << 20) + 1, (3 << 20) + 4321, 1 << 23]


def data(seed: int, n: int) -> bytes:
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8).tobytes()


def main():
    import blake3
    out = [{"seed": i, "len": n, "digest": blake3.blake3(data(i, n)).hexdigest()} for i, n in enumerate(LENGTHS)]
    path = os.path.join(os.path.dirname(__file__), "blake3_vectors.json")
    with open(path, "w") as f:
        json.dump({"generator": "blake3 (Python bindings) " + getattr(blake3, "__version__", "?"),
                   "vectors": out}, f, indent=1)
    print(path, len(out))


if __name__ == "__main__":
    main()
