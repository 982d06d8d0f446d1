"""Writes tests/golden/block_select_threshold.npz: score grids with the decisions the reference's own block_select_host
(dflash/src/flashprefill_select.cpp:27-84, compiled by oracle/build_oracle.py into oracle/_ref/) takes on them.

Run where the reference checkout is present:  python tests/golden/make_block_select_threshold.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import block_sparse as BS, build_oracle   # noqa: E402

CASES = [  # (H, M, seed, sink, window, last_n_full, alpha, kind)
    (8, 37, 0, 2, 4, 2, 0.12, "normal"),
    (4, 33, 1, 0, 1, 0, 0.9, "normal"),
    (2, 40, 2, 1, 4, 0, 1.0, "ties"),
    (2, 24, 3, 2, 2, 3, 0.5, "negative"),
    (3, 20, 4, 1, 3, 1, 0.0, "positive"),
]


def make_scores(H, M, seed, kind):
    rng = np.random.default_rng(seed)
    if kind == "ties":
        sc = rng.integers(0, 4, size=(H, M, M)).astype(np.float32)
    elif kind == "negative":
        sc = -np.abs(rng.standard_normal((H, M, M))).astype(np.float32) - 0.1
    elif kind == "positive":
        sc = np.abs(rng.standard_normal((H, M, M))).astype(np.float32)
    else:
        sc = rng.standard_normal((H, M, M)).astype(np.float32)
    return sc


def main():
    assert build_oracle.build_ref_block_select() is not None, "reference checkout missing"
    out = {}
    for i, (H, M, seed, sink, window, last_full, alpha, kind) in enumerate(CASES):
        sc = make_scores(H, M, seed, kind)
        keep = BS.reference_block_select(sc, sink, window, last_full, alpha)
        out[f"scores{i}"] = sc
        out[f"keep{i}"] = np.packbits(keep, axis=-1)
        out[f"params{i}"] = np.array([sink, window, last_full], dtype=np.int32)
        out[f"alpha{i}"] = np.float32(alpha)
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "block_select_threshold.npz"), **out)
    print("written", len(CASES), "cases")


if __name__ == "__main__":
    main()
