"""CPU restatement of the prompt compressor's chunk selection (TEST INFRASTRUCTURE: only tests may use it).

Follows steps 2-4 of drafter_score_and_compress (dflash/src/qwen3_drafter.cpp:112-175): mean over the lookahead rows
(:113-120), average-pool smoothing over [j - pool/2, j + pool/2] clipped to the prompt (:122-132), chunk means
(:134-145), the max(1, int(n_chunks * keep_ratio)) best chunks (:135,146-152; equal means: lower chunk index first --
the reference's partial_sort leaves that order open), kept positions ascending (:154-172; merging adjacent spans does
not change the sequence).  All sums in float32 in the reference's order.

Pinned: oracle/build_oracle.py cuts those lines out of the checkout into oracle/_ref/libref_drafter_select.so and
tests/test_drafter.py holds this restatement and the library's mk_drafter_select to it on random score arrays.
The tail-attention scores themselves come from oracle/qwen35_oracle.py (Oracle.tail_lookahead).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "libref_drafter_select.so")


def select_positions(running_max, keep_ratio, chunk_size, pool_kernel):
    rm = np.asarray(running_max, dtype=np.float32)
    n, S = rm.shape
    score = np.zeros(S, np.float32)
    for j in range(S):
        s = np.float32(0)
        for t in range(n):
            s = np.float32(s + rm[t, j])
        score[j] = s / np.float32(n)
    half = pool_kernel // 2
    smooth = np.zeros(S, np.float32)
    for j in range(S):
        lo, hi = max(0, j - half), min(S - 1, j + half)
        s = np.float32(0)
        for k in range(lo, hi + 1):
            s = np.float32(s + score[k])
        smooth[j] = s / np.float32(hi - lo + 1)
    n_chunks = (S + chunk_size - 1) // chunk_size
    n_keep = min(n_chunks, max(1, int(np.float32(n_chunks) * np.float32(keep_ratio))))
    means = []
    for c in range(n_chunks):
        s0, e0 = c * chunk_size, min(S, (c + 1) * chunk_size)
        m = np.float32(0)
        for j in range(s0, e0):
            m = np.float32(m + smooth[j])
        means.append((-float(m / np.float32(max(1, e0 - s0))), c))
    sel = sorted(c for _, c in sorted(means)[:n_keep])
    return np.array([j for c in sel for j in range(c * chunk_size, min(S, (c + 1) * chunk_size))], dtype=np.int32)


def reference_select_ids(running_max, ids, keep_ratio, chunk_size, pool_kernel):
    """The reference's own lines (built into oracle/_ref): returns the kept ids, or None when the library is absent."""
    if not os.path.exists(REF_LIB):
        return None
    lib = ctypes.CDLL(REF_LIB)
    rm = np.ascontiguousarray(np.asarray(running_max, dtype=np.float32))
    n, S = rm.shape
    ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
    out = np.empty(S, np.int32)
    k = lib.ref_drafter_select(rm.ctypes.data_as(ctypes.c_void_p), n, S, ctypes.c_float(keep_ratio), chunk_size, pool_kernel,
                               ids.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p))
    return out[:k].copy()
