"""CPU restatement of the block-sparse prefill attention: block selection and masked attention.

TEST INFRASTRUCTURE ONLY (checker for tests/; the product path never imports it).

Rule (the benchmark configuration for long prompts): attention is computed over 128 x 128 blocks of
(query positions x key positions).  For every query head h and query block i the kept key blocks are

    block 0 (attention sink)  |  the local window j in [i-3, i]  |  the top ceil(0.10 * (i+1)) causal
    key blocks j <= i ranked by score(i, j) = mean_pool(q)[h, i] . mean_pool(k)[h // 4, j]

with mean_pool the average over the (up to) 128 positions of a block of the post-norm, post-RoPE bf16
query / key vectors, and ties broken towards the lower block index.  Structure after the reference's
host-side selection (dflash/src/flashprefill_select.cpp:27-84: sink + window + score threshold against
the row maximum); the ranking rule and the 10 % budget are the benchmark's.

parity unpinned for the ranking rule: the reference holds no vectors for it (its own selection rule differs and
belongs to another model); the CUDA kernels are held to this restatement bit for bit, which is why
every floating-point step below fixes its summation order.  The reference's own keep rule (select_threshold below)
IS pinned: against the reference function compiled from its source file, and through a committed fixture made by it.

  * block sums run sequentially over positions 0..127 in f32, then one multiply by 1/count;
  * a score is a 256-term dot product taken as 32 lane partials (lane l sums dims 8l..8l+7 in order,
    products rounded before each add: no fused multiply-add), then a butterfly over lane distances
    16, 8, 4, 2, 1.
"""
import math

import numpy as np

BLOCK = 128


def pool_means(x):
    """x: [P, D] float32 (bf16-representable values).  Returns [ceil(P/128), D] block means."""
    P, D = x.shape
    nb = (P + BLOCK - 1) // BLOCK
    out = np.zeros((nb, D), dtype=np.float32)
    for b in range(nb):
        acc = np.zeros(D, dtype=np.float32)
        lo, hi = b * BLOCK, min(P, (b + 1) * BLOCK)
        for p in range(lo, hi):
            acc = (acc + x[p]).astype(np.float32)
        out[b] = acc * np.float32(1.0 / (hi - lo))
    return out


def _dot_lanes(a, b):
    """[..., 256] x [..., 256] -> [...] with the summation order of the kernel."""
    prod = (a.astype(np.float32) * b.astype(np.float32)).astype(np.float32)
    prod = prod.reshape(prod.shape[:-1] + (32, 8))
    part = prod[..., 0]
    for e in range(1, 8):
        part = (part + prod[..., e]).astype(np.float32)
    for o in (16, 8, 4, 2, 1):
        idx = np.arange(32) ^ o
        part = (part + part[..., idx]).astype(np.float32)
    return part[..., 0]


def block_scores(qmean, kmean):
    """qmean [M, D], kmean [N, D] -> [M, N] float32."""
    return _dot_lanes(qmean[:, None, :], kmean[None, :, :])


def select_blocks(scores, top_frac=0.10, window=4, sink=1):
    """scores [M, N] -> bool [M, N], causal in blocks (j <= i)."""
    M, N = scores.shape
    keep = np.zeros((M, N), dtype=bool)
    for i in range(M):
        n = min(i + 1, N)
        keep[i, :min(sink, n)] = True
        keep[i, max(0, i - window + 1):n] = True
        k = int(math.ceil(top_frac * n))
        order = sorted(range(n), key=lambda j: (-float(scores[i, j]), j))
        for j in order[:k]:
            keep[i, j] = True
    return keep


def select_threshold(scores, sink=2, window=4, last_n_full=2, alpha=0.12):
    """The reference's own keep rule on a score grid (dflash/src/flashprefill_select.cpp:27-84, block_select_host):
    scores [M, N] f32 -> bool [M, N].  Per query block m, over the causal key blocks n <= m: n < sink, m - n < window,
    every block when m >= M - last_n_full, and score >= max_score * alpha with the product taken in f32.
    Pinned against the compiled reference function (tests/test_block_select_threshold.py)."""
    M, N = scores.shape
    keep = np.zeros((M, N), dtype=bool)
    a = np.float32(alpha)
    for m in range(M):
        row = scores[m, :m + 1].astype(np.float32)
        mx = np.float32(-np.inf)
        for v in row:
            if v > mx:
                mx = v
        with np.errstate(invalid="ignore"):
            thresh = np.float32(mx * a)
        full = m >= M - last_n_full
        for n in range(m + 1):
            keep[m, n] = (n < sink) or (m - n < window) or full or bool(row[n] >= thresh)
    return keep


def reference_block_select(scores_hmn, sink, window, last_n_full, alpha):
    """Runs the compiled reference function (oracle/_ref/libref_block_select.so) on scores [H, M, N] f32 and
    returns bool [H, M, N], or None when the library is not there."""
    import ctypes
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref_block_select.so")
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    H, M, N = scores_hmn.shape
    sc = np.ascontiguousarray(np.transpose(scores_hmn.astype(np.float32), (1, 2, 0)))[None]      # [1, M, N, H]
    idx = np.full((1, M, N, H), -7, dtype=np.int32)
    cnt = np.zeros((1, M, H), dtype=np.int32)
    lib.ref_block_select_host(sc.ctypes.data_as(ctypes.c_void_p), 1, M, N, H, int(sink), int(window), int(last_n_full),
                              ctypes.c_float(alpha), idx.ctypes.data_as(ctypes.c_void_p), cnt.ctypes.data_as(ctypes.c_void_p))
    keep = np.zeros((H, M, N), dtype=bool)
    for h in range(H):
        for m in range(M):
            c = int(cnt[0, m, h])
            ks = idx[0, m, :c, h]
            assert np.all(ks[1:] > ks[:-1]) and np.all(idx[0, m, c:, h] == -1)
            keep[h, m, ks] = True
    return keep


def select_for_heads(q, k, gqa=4, **kw):
    """q [Hq, S, D], k [Hk, S, D] float32 -> bool [Hq, M, N]."""
    kmeans = [pool_means(k[g]) for g in range(k.shape[0])]
    return np.stack([select_blocks(block_scores(pool_means(q[h]), kmeans[h // gqa]), **kw) for h in range(q.shape[0])])


def select_threshold_for_heads(q, k, gqa=4, **kw):
    """The reference's keep rule on the mean-pooled scores: q [Hq, S, D], k [Hk, S, D] float32 -> bool [Hq, M, N]."""
    kmeans = [pool_means(k[g]) for g in range(k.shape[0])]
    return np.stack([select_threshold(block_scores(pool_means(q[h]), kmeans[h // gqa]), **kw) for h in range(q.shape[0])])


def token_mask(keep, S):
    """Block mask [M, N] -> causal position mask [S, S]."""
    m = np.repeat(np.repeat(keep, BLOCK, axis=0), BLOCK, axis=1)[:S, :S]
    return m & np.tril(np.ones((S, S), dtype=bool))
