"""The reference's own block keep rule (dflash/src/flashprefill_select.cpp:27-84): sink blocks, local window, every
causal block for the last query blocks, and score >= alpha * row maximum.

CPU: the restatement (oracle/block_sparse.select_threshold) against decisions taken by the reference function itself
-- the committed fixture (made by tests/golden/make_block_select_threshold.py) and, where the compiled function is
present (oracle/_ref/libref_block_select.so), fresh random grids.  GPU: mk_block_select_threshold must take exactly the
reference function's decisions on the scores it reports (bit-exact: the decisions are integer work).
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import block_sparse as BS

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "block_select_threshold.npz")


def _restated(sc, sink, window, last_full, alpha):
    return np.stack([BS.select_threshold(sc[h], sink, window, last_full, alpha) for h in range(sc.shape[0])])


def test_restatement_matches_reference_fixture():
    z = np.load(GOLD)
    n = len([k for k in z.files if k.startswith("scores")])
    assert n >= 5
    for i in range(n):
        sc = z[f"scores{i}"]
        sink, window, last_full = (int(v) for v in z[f"params{i}"])
        alpha = float(z[f"alpha{i}"])
        M = sc.shape[1]
        want = np.unpackbits(z[f"keep{i}"], axis=-1)[..., :M].astype(bool)
        got = _restated(sc, sink, window, last_full, alpha)
        assert (got == want).all(), f"case {i}: {int((got != want).sum())} decisions differ"
        assert not np.triu(got, 1).any()                     # causal in blocks


def test_restatement_matches_compiled_reference():
    rng = np.random.default_rng(11)
    ran = 0
    for trial in range(6):
        H, M = int(rng.integers(1, 5)), int(rng.integers(1, 50))
        sc = rng.standard_normal((H, M, M)).astype(np.float32)
        if trial % 2:
            sc = np.round(sc * 2) / 2                         # many exact ties with the threshold
        sink, window, last_full = int(rng.integers(0, 3)), int(rng.integers(1, 6)), int(rng.integers(0, 4))
        alpha = float(rng.choice([0.0, 0.12, 0.5, 1.0, 1.5]))
        want = BS.reference_block_select(sc, sink, window, last_full, alpha)
        if want is None:
            pytest.skip("compiled reference function not present (the fixture test covers the pin)")
        assert (_restated(sc, sink, window, last_full, alpha) == want).all()
        ran += 1
    assert ran == 6


# ---- GPU ---------------------------------------------------------------------------------------------

def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _make(S, seed):
    g = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(S, 5120, generator=g) * 0.7).to(torch.bfloat16)
    drift = torch.randn((S + 127) // 128, 512, generator=g).repeat_interleave(128, 0)[:S] * 0.5
    qkv[:, 4096:4608] = (qkv[:, 4096:4608].float() + drift).to(torch.bfloat16)
    kc = torch.zeros(2, S, 256, dtype=torch.bfloat16)
    kc[:, :S] = qkv[:, 4096:4608].reshape(S, 2, 256).transpose(0, 1)
    return qkv, kc


@pytest.mark.gpu
@pytest.mark.parametrize("S,alpha,window,sink,last_full", [(1000, 0.12, 4, 2, 2), (4100, 0.5, 2, 0, 0), (4100, 1.0, 1, 1, 3),
                                                           (16384, 0.12, 4, 2, 2), (65536, 0.12, 4, 2, 2)])
def test_gpu_decisions_are_the_reference_functions(S, alpha, window, sink, last_full):
    import luce_megakernel_b200 as L
    lib = L.lib()
    qkv, kc = _make(S, 7 + S)
    dq, dk = qkv.cuda(), kc.cuda()
    nblk = (S + 127) // 128
    nwords = (nblk + 31) // 32
    lib.mk_block_select_scratch_bytes.restype = ctypes.c_size_t
    scratch = torch.empty(lib.mk_block_select_scratch_bytes(S), dtype=torch.uint8, device="cuda")
    mask = torch.zeros(8, nblk, nwords, dtype=torch.int32, device="cuda")
    scores = torch.zeros(8, nblk, nblk, dtype=torch.float32, device="cuda")
    rc = lib.mk_block_select_threshold(_ptr(dq), _ptr(dk), S, S, ctypes.c_float(alpha), window, sink, last_full, _ptr(mask),
                                       _ptr(scores), _ptr(scratch), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    words = mask.cpu().numpy().astype(np.uint32)
    bits = ((words[..., None] >> np.arange(32, dtype=np.uint32)) & 1).astype(bool).reshape(8, nblk, nwords * 32)[..., :nblk]
    sc = scores.cpu().numpy()
    # the reported scores are the ranking rule's scores (restated with the kernel's summation order)
    q = qkv[:, :4096].reshape(S, 8, 512)[:, :, :256].permute(1, 0, 2).float().numpy()
    k = kc.float().numpy()
    if S <= 4100:
        km = [BS.pool_means(k[g]) for g in range(2)]
        for h in (0, 5):
            ref_sc = BS.block_scores(BS.pool_means(q[h]), km[h // 4])
            tri = np.tril(np.ones((nblk, nblk), dtype=bool))
            assert (sc[h][tri] == ref_sc[tri]).all()
    want = BS.reference_block_select(sc, sink, window, last_full, alpha)
    if want is None:
        want = _restated(sc, sink, window, last_full, alpha)
    assert (bits == want).all(), f"{int((bits != want).sum())} block decisions differ"
    tri = np.tril(np.ones((nblk, nblk), dtype=bool))
    if nblk >= 16:
        assert (~bits[:, tri]).any()                          # something is actually dropped
