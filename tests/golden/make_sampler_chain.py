"""Writes tests/golden/sampler_chain.npz: logits, sampler settings and the draws the reference's own CPU sampler chain
(SamplerCfg + sample_logits of dflash/test/test_dflash.cpp, compiled by oracle/build_oracle.py into oracle/_ref/)
makes on them from a std::mt19937_64 seeded per case.

Run where the reference checkout is present:  python tests/golden/make_sampler_chain.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import build_oracle, sampling as S   # noqa: E402

CASES = [  # (vocab, logits seed, scale, temp, top_k, top_p, rep_pen, n_history, rng seed)
    (1000, 0, 2.0, 1.0, 0, 1.0, 1.0, 0, 42),
    (1000, 1, 2.0, 0.7, 50, 1.0, 1.0, 0, 7),
    (1000, 2, 3.0, 0.9, 0, 0.9, 1.0, 0, 8),
    (1000, 3, 2.0, 0.8, 40, 0.5, 1.3, 12, 9),
    (300, 4, 1.0, 1.5, 10, 0.95, 1.1, 400, 10),
    (300, 5, 4.0, 0.0005, 0, 1.0, 1.0, 0, 11),
]
N_DRAWS = 300


def case_inputs(vocab, lseed, scale, n_hist):
    rng = np.random.default_rng(lseed)
    logits = (rng.standard_normal(vocab) * scale).astype(np.float32)
    hist = rng.integers(0, vocab, size=n_hist).astype(np.int32)
    if n_hist:
        hist[-1] = int(np.argmax(logits))              # the penalty must hit the most likely token too
    return logits, hist


def main():
    assert build_oracle.build_ref_sampler() is not None, "reference checkout missing"
    lib = S.compiled_reference_sampler()
    out = {}
    for i, (vocab, lseed, scale, temp, top_k, top_p, rep, n_hist, seed) in enumerate(CASES):
        logits, hist = case_inputs(vocab, lseed, scale, n_hist)
        out[f"logits{i}"] = logits
        out[f"history{i}"] = hist
        out[f"cfg{i}"] = np.array([temp, top_k, top_p, rep, seed], dtype=np.float64)
        out[f"draws{i}"] = S.compiled_reference_draws(lib, logits, temp, top_k, top_p, rep, hist, seed, N_DRAWS)
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampler_chain.npz"), **out)
    print("written", len(CASES), "cases")


if __name__ == "__main__":
    main()
