"""Sampling at the LM-head boundary (temperature / top-k / top-p).

Pin: the CPU sampler chain of the reference's speculative-decoding driver (dflash/test/test_dflash.cpp:113-188) is
restated in oracle/sampling.py and must reproduce, draw for draw, what that function itself drew -- the committed
fixture (tests/golden/sampler_chain.npz, made by tests/golden/make_sampler_chain.py) and, where the compiled function
is present, fresh cases.  The kernel's definition (sample / kept_mask / nucleus_mask) must then have exactly the
chain's support and probabilities.

CPU: the restatement (oracle/sampling.py) draws from the distribution it claims -- softmax(logits / T) over the top-k
set -- and its top-k rule breaks ties towards the lower index.  GPU: mk_sample_top_k equals the restatement token for
token on the same logits (it is a deterministic function of logits, seed and counter), including ties at the top-k
boundary and NaN logits; through the decoder, temperature 0 reproduces the greedy token and the stored logits are
the ones the argmax was taken over.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import sampling as S


def test_uniforms_are_in_the_open_interval_and_reproducible():
    u = S.uniforms(7, 3, 100000)
    assert u.min() > 0.0 and u.max() < 1.0
    assert np.array_equal(u, S.uniforms(7, 3, 100000))
    assert not np.array_equal(u, S.uniforms(7, 4, 100000))
    assert abs(u.mean() - 0.5) < 0.01 and abs(u.var() - 1 / 12) < 0.01


def test_top_k_rule_breaks_ties_towards_the_lower_index():
    l = np.array([1.0, 3.0, 2.0, 3.0, 2.0, 2.0, -1.0, np.nan], dtype=np.float32)
    assert S.kept_mask(l, 2).nonzero()[0].tolist() == [1, 3]
    assert S.kept_mask(l, 4).nonzero()[0].tolist() == [1, 2, 3, 4]          # two of the three 2.0s: the lowest indices
    assert S.kept_mask(l, 0).nonzero()[0].tolist() == [0, 1, 2, 3, 4, 5, 6]  # everything but the NaN
    assert S.sample(l, 0.0, 0, 1, 1) == 1 and S.sample(l, 1.0, 1, 1, 1) == 1


def test_restatement_draws_from_the_softmax_over_the_kept_set():
    rng = np.random.default_rng(0)
    l = (rng.standard_normal(50) * 2).astype(np.float32)
    for T, k in ((1.0, 0), (0.7, 8), (1.5, 20)):
        p = S.distribution(l, T, k)
        n = 20000
        counts = np.bincount([S.sample(l, T, k, 11, c) for c in range(n)], minlength=50)
        assert counts[p == 0].sum() == 0                         # nothing outside the kept set
        sel = p > 0
        chi2 = (((counts[sel] - n * p[sel]) ** 2) / (n * p[sel])).sum()
        assert chi2 < 3 * sel.sum() + 30, (T, k, chi2)            # far inside for a correct sampler, far outside for a wrong one


GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sampler_chain.npz")


def test_restated_chain_reproduces_the_reference_draws_of_the_fixture():
    z = np.load(GOLD)
    n = len([k for k in z.files if k.startswith("logits")])
    assert n >= 6
    for i in range(n):
        temp, top_k, top_p, rep, seed = z[f"cfg{i}"]
        rng = S.MT19937_64(int(seed))
        hist = z[f"history{i}"].tolist()
        got = [S.reference_chain_draw(z[f"logits{i}"], float(temp), int(top_k), float(top_p), rng, float(rep), hist)
               for _ in range(len(z[f"draws{i}"]))]
        assert got == z[f"draws{i}"].tolist(), f"case {i}"


def test_restated_chain_reproduces_the_compiled_reference():
    lib = S.compiled_reference_sampler()
    if lib is None:
        pytest.skip("compiled reference sampler not present (the fixture test covers the pin)")
    rng = np.random.default_rng(5)
    for trial in range(5):
        vocab = int(rng.integers(20, 600))
        l = (rng.standard_normal(vocab) * rng.uniform(0.5, 4)).astype(np.float32)
        temp, top_k = float(rng.choice([0.3, 0.8, 1.0, 1.7])), int(rng.choice([0, 5, 40]))
        top_p, rep = float(rng.choice([1.0, 0.95, 0.6])), float(rng.choice([1.0, 1.2]))
        hist = rng.integers(0, vocab, size=int(rng.integers(0, 30))).astype(np.int32)
        want = S.compiled_reference_draws(lib, l, temp, top_k, top_p, rep, hist, 100 + trial, 100)
        g = S.MT19937_64(100 + trial)
        got = [S.reference_chain_draw(l, temp, top_k, top_p, g, rep, hist.tolist()) for _ in range(100)]
        assert got == want.tolist(), (trial, temp, top_k, top_p, rep)


def test_kernel_definition_has_the_support_and_probabilities_of_the_reference_chain():
    rng = np.random.default_rng(9)
    for vocab, T, k, p in ((200, 1.0, 0, 1.0), (200, 0.7, 30, 1.0), (500, 0.9, 0, 0.9), (500, 0.8, 40, 0.5), (64, 1.4, 10, 0.8)):
        l = (rng.standard_normal(vocab) * 2).astype(np.float32)
        assert len(np.unique(l)) == vocab                        # no ties: the chain leaves their order open
        cand, probs = S.reference_chain(l, T, k, p)
        keep = S.nucleus_mask(l, S.kept_mask(l, k), T, p)
        assert sorted(cand.tolist()) == np.nonzero(keep)[0].tolist(), (vocab, T, k, p)
        ours = S.distribution(l, T, k, p)
        assert np.allclose(ours[cand], probs, rtol=2e-5, atol=1e-7)
        assert ours[~keep].sum() == 0.0


def test_restatement_with_nucleus_draws_from_its_distribution():
    rng = np.random.default_rng(2)
    l = (rng.standard_normal(50) * 2).astype(np.float32)
    p = S.distribution(l, 0.9, 20, 0.8)
    n = 20000
    counts = np.bincount([S.sample(l, 0.9, 20, 3, c, top_p=0.8) for c in range(n)], minlength=50)
    sel = p > 0
    assert 1 < sel.sum() < 20 and counts[~sel].sum() == 0
    chi2 = (((counts[sel] - n * p[sel]) ** 2) / (n * p[sel])).sum()
    assert chi2 < 3 * sel.sum() + 30


# ---- GPU -----------------------------------------------------------------------------------------------------

def _gpu_sample(lib, logits, T, k, seed, counter):
    out = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    rc = lib.mk_sample_top_k(ctypes.c_void_p(logits.data_ptr()), ctypes.c_int(logits.numel()), ctypes.c_float(T), ctypes.c_int(k),
                             ctypes.c_ulonglong(seed), ctypes.c_ulonglong(counter), ctypes.c_void_p(out.data_ptr()),
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    return int(out.item())


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1000, 248320])
def test_kernel_equals_restatement(n):
    import luce_megakernel_b200 as L
    lib = L.lib()
    g = torch.Generator().manual_seed(n)
    l = (torch.randn(n, generator=g) * 3).float()
    l[5] = l[17] = l[n - 1] = l.topk(40).values[-1]              # ties exactly at a top-40 boundary, among others
    l[n // 2] = float("nan")
    ld, ln = l.cuda(), l.numpy()
    for T, k in ((0.0, 0), (1.0, 1), (1.0, 0), (0.8, 40), (0.8, 39), (0.8, 41), (1.3, 500), (0.5, n), (2.0, n + 5)):
        for c in range(6):
            assert _gpu_sample(lib, ld, T, k, 1234, c) == S.sample(ln, T, k, 1234, c), (T, k, c)
    assert lib.mk_sample_top_k(None, 10, ctypes.c_float(1.0), 0, ctypes.c_ulonglong(0), ctypes.c_ulonglong(0), None, None) == 1


def _gpu_sample_p(lib, logits, T, k, p, seed, counter):
    out = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    rc = lib.mk_sample_top_k_top_p(ctypes.c_void_p(logits.data_ptr()), ctypes.c_int(logits.numel()), ctypes.c_float(T), ctypes.c_int(k),
                                   ctypes.c_float(p), ctypes.c_ulonglong(seed), ctypes.c_ulonglong(counter),
                                   ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    return int(out.item())


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1000, 248320])
def test_kernel_with_nucleus_equals_restatement(n):
    import luce_megakernel_b200 as L
    lib = L.lib()
    g = torch.Generator().manual_seed(n + 1)
    l = (torch.randn(n, generator=g) * 3).float()
    l[n // 3] = float("nan")
    ld, ln = l.cuda(), l.numpy()
    for T, k, p in ((1.0, 0, 0.9), (0.8, 40, 0.5), (0.8, 40, 0.999), (1.3, 500, 0.3), (0.6, 0, 0.05), (1.0, 0, 1.0), (1.0, 7, 0.0)):
        keep = S.nucleus_mask(ln, S.kept_mask(ln, k), T, p)
        for c in range(8):
            got = _gpu_sample_p(lib, ld, T, k, p, 77, c)
            assert got == S.sample(ln, T, k, 77, c, top_p=p), (T, k, p, c)
            assert keep[got]


@pytest.mark.gpu
def test_kernel_draws_what_the_reference_chain_draws_in_distribution():
    """Same logits and settings through the kernel (Gumbel-max, counter-based generator) and through the reference's
    chain (inverse CDF, Mersenne twister): the tokens that can come out are the same set and their frequencies follow
    the chain's probabilities."""
    import luce_megakernel_b200 as L
    lib = L.lib()
    rng = np.random.default_rng(4)
    l = (rng.standard_normal(64) * 2).astype(np.float32)
    ld = torch.from_numpy(l).cuda()
    T, k, p = 0.9, 12, 0.8
    cand, probs = S.reference_chain(l, T, k, p)
    n = 4000
    out = torch.empty(n, dtype=torch.int32, device="cuda")
    for c in range(n):
        lib.mk_sample_top_k_top_p(ctypes.c_void_p(ld.data_ptr()), 64, ctypes.c_float(T), k, ctypes.c_float(p), ctypes.c_ulonglong(5),
                                  ctypes.c_ulonglong(c), ctypes.c_void_p(out[c:c + 1].data_ptr()),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    counts = np.bincount(out.cpu().numpy(), minlength=64)
    assert set(np.nonzero(counts)[0].tolist()) <= set(cand.tolist()) and 1 < len(cand) < k
    chi2 = (((counts[cand] - n * probs) ** 2) / (n * probs)).sum()
    assert chi2 < 3 * len(cand) + 30
    lib_ref = S.compiled_reference_sampler()
    if lib_ref is not None:                                      # and the chain's own draws, side by side
        ref_counts = np.bincount(S.compiled_reference_draws(lib_ref, l, T, k, p, 1.0, np.zeros(0, np.int32), 1, n), minlength=64)
        assert set(np.nonzero(ref_counts)[0].tolist()) <= set(cand.tolist())
        tot = counts[cand] + ref_counts[cand]
        chi2 = (((counts[cand] - tot / 2) ** 2) / (tot / 2 + 1e-9)).sum() * 2
        assert chi2 < 3 * len(cand) + 30


@pytest.mark.gpu
def test_kernel_follows_the_distribution():
    import luce_megakernel_b200 as L
    lib = L.lib()
    rng = np.random.default_rng(1)
    l = (rng.standard_normal(64) * 2).astype(np.float32)
    ld = torch.from_numpy(l).cuda()
    p = S.distribution(l, 0.9, 10)
    n = 4000
    out = torch.empty(n, dtype=torch.int32, device="cuda")
    for c in range(n):
        lib.mk_sample_top_k(ctypes.c_void_p(ld.data_ptr()), 64, ctypes.c_float(0.9), 10, ctypes.c_ulonglong(5), ctypes.c_ulonglong(c),
                            ctypes.c_void_p(out[c:c + 1].data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    counts = np.bincount(out.cpu().numpy(), minlength=64)
    sel = p > 0
    assert counts[~sel].sum() == 0
    chi2 = (((counts[sel] - n * p[sel]) ** 2) / (n * p[sel])).sum()
    assert chi2 < 3 * sel.sum() + 30


@pytest.mark.gpu
def test_decoder_sampling_step(small_model):
    from luce_megakernel_b200 import model as M
    from oracle import qwen35_oracle as O
    sd, orc = small_model("unit", "decode")
    dec = M.Decoder(weights=M.weights_from_state_dict(sd), max_seq_len=64, api="cabi")
    g = torch.Generator().manual_seed(3)
    toks = torch.randint(0, 2048, (6,), generator=g).tolist()
    st = O.State.new(8, 64, 2048)
    for i, t in enumerate(toks):
        got = dec.step_sampled(t, 0.8, 20, seed=99)
        tr = orc.forward([t], st)
        logits = dec._logits.cpu()
        assert float((logits - tr.logits).abs().max()) <= 5e-2            # the stored logits are the step's logits
        assert got == S.sample(logits.numpy(), 0.8, 20, 99, i + 1)        # counter = position of the sampled token
        assert S.kept_mask(logits.numpy(), 20)[got]
    # temperature 0 = the greedy step
    dec.reset()
    a = [dec.step_sampled(t, 0.0) for t in toks]
    dec.reset()
    b = [dec.step(t) for t in toks]
    assert a == b
