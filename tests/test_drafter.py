"""Prompt compressor (speculative prefill with this model as its own drafter).

CPU: the chunk selection (mk_drafter_select in the library, oracle/drafter.py) against the reference's own lines of
dflash/src/qwen3_drafter.cpp, cut out at build time into oracle/_ref (skipped where that library is absent).
GPU: the tail-attention scores the prefill leaves against the oracle's attention, dense and block-sparse, and the
compressed prompt end to end."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import drafter as OD


def _lib():
    import luce_megakernel_b200 as L
    return L.lib()


def _scores(n, S, seed, ties=False):
    g = np.random.default_rng(seed)
    rm = g.random((n, S), dtype=np.float32) ** 4          # a few large values, like attention mass
    if ties:
        rm[:] = np.float32(0.25)                           # every chunk mean equal: the tie rule decides
    return rm


@pytest.mark.parametrize("n,S,keep,chunk,pool", [(8, 1000, 0.25, 32, 13), (8, 4096, 0.05, 32, 13), (4, 97, 0.5, 16, 5),
                                                 (1, 33, 0.01, 32, 1), (8, 640, 1.0, 64, 31), (2, 50, 0.3, 7, 4)])
def test_selection_matches_the_reference_lines_and_the_restatement(n, S, keep, chunk, pool):
    from luce_megakernel_b200 import drafter as D
    rm = _scores(n, S, 3 * S + n)
    got = D.select_positions(_lib(), rm, keep, chunk, pool)
    assert np.array_equal(got, OD.select_positions(rm, keep, chunk, pool))
    ids = np.arange(1000, 1000 + S, dtype=np.int32)
    ref = OD.reference_select_ids(rm, ids, keep, chunk, pool)
    if ref is None:
        pytest.skip("oracle/_ref/libref_drafter_select.so not built (no reference checkout at build time)")
    assert np.array_equal(ids[got], ref)                    # same tokens, same order as the reference returns
    n_chunks = (S + chunk - 1) // chunk
    assert len(got) <= max(1, int(n_chunks * keep)) * chunk and np.all(np.diff(got) > 0)


def test_selection_edge_cases():
    from luce_megakernel_b200 import drafter as D
    lib = _lib()
    rm = _scores(8, 320, 1, ties=True)
    got = D.select_positions(lib, rm, 0.3, 32, 13)
    # interior chunks see a full smoothing window of equal values; so do the border chunks: all means equal, lowest chunks win
    assert np.array_equal(got, np.arange(0, 3 * 32))
    assert np.array_equal(got, OD.select_positions(rm, 0.3, 32, 13))
    # keep_ratio 0 still keeps one chunk; a ratio above 1 keeps everything
    assert len(D.select_positions(lib, _scores(8, 100, 2), 0.0, 32, 13)) in (32, 4)
    assert np.array_equal(D.select_positions(lib, _scores(8, 100, 2), 3.0, 32, 13), np.arange(100))
    out = np.empty(8, np.int32)
    lib.mk_drafter_select.restype = ctypes.c_int
    assert lib.mk_drafter_select(None, 8, 8, ctypes.c_float(0.5), 4, 3, out.ctypes.data_as(ctypes.c_void_p)) == -1
    assert lib.mk_drafter_select(out.ctypes.data_as(ctypes.c_void_p), 0, 8, ctypes.c_float(0.5), 4, 3,
                                 out.ctypes.data_as(ctypes.c_void_p)) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("S,sparse", [(300, None), (1500, None), (1500, (0.10, 4, 1))])
def test_tail_scores_match_the_oracle(small_model, S, sparse):
    """running_max of the last 8 positions over a prompt, against the oracle's attention probabilities (bf16 q and k on
    both sides; the prefill's other rounding points move a probability by a few 1e-3 at most)."""
    from luce_megakernel_b200 import model as M, drafter as D
    from oracle import qwen35_oracle as O
    sd, _ = small_model("unit", "decode")
    dec = M.Decoder(weights=M.weights_from_state_dict(sd), max_seq_len=2048, api="cabi")
    g = torch.Generator().manual_seed(S)
    ids = torch.randint(0, 2048, (S,), generator=g).tolist()
    rm = D.tail_scores(dec, ids, 8, block_sparse=sparse)
    bs = None if sparse is None else {"top_frac": sparse[0], "window": sparse[1], "sink": sparse[2]}
    orc = O.Oracle(sd, rounding="decode", block_sparse=bs)
    orc.tail_lookahead = 8
    orc.forward(ids, O.State.new(8, 2048, 2048))
    ref = orc.tail_running_max
    assert rm.shape == ref.shape == (8, S)
    assert float(rm.min()) >= 0.0 and float(rm.max()) <= 1.0 + 1e-6
    # keys beyond a tail query's position are masked: exactly zero
    for t in range(8):
        assert not rm[t, S - 8 + t + 1:].any()
    err = float((rm - ref).abs().max())
    assert err <= 2e-2, err
    # and the selection built on them agrees with the selection built on the oracle's scores up to near-ties
    a = set(D.select_positions(dec._lib, rm.numpy(), 0.25, 32, 13).tolist())
    b = set(D.select_positions(dec._lib, ref.numpy(), 0.25, 32, 13).tolist())
    assert len(a ^ b) <= 2 * 32


@pytest.mark.gpu
def test_score_and_compress_end_to_end(small_model):
    from luce_megakernel_b200 import model as M, drafter as D
    sd, _ = small_model("unit", "decode")
    dec = M.Decoder(weights=M.weights_from_state_dict(sd), max_seq_len=4096, api="cabi")
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, 2048, (3000,), generator=g).tolist()
    out = D.score_and_compress(dec, ids, keep_ratio=0.2, chunk_size=32, n_lookahead=8, pool_kernel=13, block_sparse=(0.10, 4, 1))
    n_chunks = (3000 + 31) // 32
    assert len(out) <= int(n_chunks * 0.2) * 32 and len(out) >= (int(n_chunks * 0.2) - 1) * 32
    it = iter(ids)                                           # a subsequence of the prompt, in order
    assert all(any(t == x for x in it) for t in out)
    assert D.score_and_compress(dec, ids[:5], 0.2) == ids[:5]        # too short to score: returned as is
    # the compressed prompt prefills and decodes like any other
    dec.reset()
    first = dec.prefill(torch.tensor(out, dtype=torch.int32).cuda())
    assert 0 <= first < 2048
