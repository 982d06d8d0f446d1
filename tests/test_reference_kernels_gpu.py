"""Second pin, on the GPU: the reference's own kernels on identical weights.

oracle/build_oracle.py compiles megakernel/kernel.cu and megakernel/prefill.cu of the reference
checkout, unmodified, for sm_100a into oracle/_ref/libref_megakernel.so (test infrastructure, built
where the checkout exists; these tests skip without it).  The full-size model (24 layers, vocabulary
248320, seeded random weights) runs through the reference's `launch_decode` / `launch_prefill_bf16`.

What the runs show, and what is asserted:

* Everything before the first attention layer agrees with this library to the last bit or two, at
  every position: conv windows and DeltaNet states of the first three layers (decode and prefill).
* The reference kernels rotate the query in place (kernel.cu:487-497, prefill.cu:1057-1064): rotary
  dims 32..63 are computed from partner values that were already rotated (and are normalised a
  second time).  Position 0 is unaffected; from position 1 on the reference kernels deviate from
  the reference's own PyTorch baseline (transformers' rotate_half), which is what the CPU oracle
  restates and this library implements.  The oracle can reproduce the in-place form
  (`ref_q_rope_in_place=True`); with it the oracle matches the reference decode kernel over a whole
  teacher-forced run to within bf16 noise, which pins every other part of the restatement (DeltaNet
  recurrence, conv, gates, attention, MLP, norms, LM head argmax) to the reference kernels.
* This library, the oracle without the flag and the reference kernels agree at position 0.

The reference kernels' throughput on the same GPU is measured by `bench.py --impl reference_gpu`.
"""
import ctypes
import math
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle.ref_kernels import REF_LIB, RefDecoder  # noqa: E402

MAXSEQ = 1024


def bf16_ulp(x):
    return 2.0 ** (math.floor(math.log2(max(x, 1e-30))) - 7)


@pytest.fixture(scope="module")
def pair():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libref_megakernel.so not built (needs the reference checkout at build time)")
    from luce_megakernel_b200 import model as M
    from oracle import qwen35_oracle as O
    lib = ctypes.CDLL(REF_LIB)
    sd = O.init_weights(0, 24, O.VOCAB, norm_init="unit")
    mine = M.Decoder(weights=M.weights_from_state_dict(sd), max_seq_len=MAXSEQ, api="cabi")
    mine._sd = sd
    return mine, RefDecoder(lib, mine, MAXSEQ)


def seeded(n, seed, vocab):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g).tolist()


def _oracles(mine_weights_sd):
    from oracle import qwen35_oracle as O
    return O, O.Oracle(mine_weights_sd, rounding="decode", ref_q_rope_in_place=True), O.Oracle(mine_weights_sd, rounding="decode")


@pytest.fixture(scope="module")
def state_dict(pair):
    return pair[0]._sd


def test_layers_before_first_attention_agree_bitwise(pair):
    mine, ref = pair
    mine.reset(); ref.reset()
    for t in seeded(12, 0, mine.vocab):
        mine.step_async(t); ref.step_async(t)
    torch.cuda.synchronize()
    for l in range(3):
        dc = float((mine._conv_bufs[l] - ref.conv[l]).abs().max())
        ds = float((mine._dn_states[l] - ref.dn[l]).abs().max())
        print(f"\ndecode, 12 tokens, DeltaNet layer {l}: conv diff {dc:.2e}, state diff {ds:.2e}")
        # layer 0 sees the embedding rows only; layers 1 and 2 see a bf16 residual stream in which a sum
        # taken in another order flips an occasional last bit
        assert (dc <= 2e-5 and ds <= 1e-6) if l == 0 else (dc <= 0.05 and ds <= 2e-4), f"DeltaNet layer {l}: conv {dc}, state {ds}"
    # keys and values of the first attention layer: bf16 roundings of sums taken in another order
    assert float((mine._fa_k_cache[0].float() - ref.k[0].float()).abs().max()) <= 2 * 0.0078125 * 4
    assert float((mine._fa_v_cache[0].float() - ref.v[0].float()).abs().max()) <= 2 * 0.0078125 * 4


def test_position0_all_three_agree(pair, state_dict):
    mine, ref = pair
    O, _, orc = _oracles(state_dict)
    mine.reset(); ref.reset()
    t = seeded(1, 5, mine.vocab)[0]
    a, b = mine.step(t), ref.step(t)
    tr = orc.forward([t], O.State.new(24, 8, mine.vocab))
    h = tr.hidden[-1][0]
    tol = max(2e-2, 4 * bf16_ulp(float(h.abs().max())))
    assert float((ref.hidden.float().cpu() - h).abs().max()) <= tol
    assert float((mine._hidden.float().cpu() - h).abs().max()) <= tol
    top = torch.topk(tr.logits, 2)
    near_tie = float(top.values[0] - top.values[1]) <= 0.1
    assert (a == b == tr.token) or near_tie


def test_reference_decode_kernel_matches_oracle_with_in_place_rotation(pair, state_dict):
    """Pins the restatement to the reference kernel itself; the plain oracle (and this library) must
    be measurably further from the reference kernel than the in-place variant is.  The reference kernel
    is not deterministic from run to run at positions >= 1 (its attention phase lets the blocks of
    different heads share one scratch area, kernel.cu:537), so no tight bound holds for it and the
    comparison is repeated up to three times."""
    mine, ref = pair
    O, orc_q, orc = _oracles(state_dict)
    toks = seeded(10, 7, mine.vocab)
    ok = False
    for attempt in range(3):
        ref.reset(); mine.reset()
        st_q, st = O.State.new(24, 64, mine.vocab), O.State.new(24, 64, mine.vocab)
        worst_q, worst_plain, worst_mine = 0.0, 0.0, 0.0
        for t in toks:
            ref.step(t)
            mine.step(t)
            hq = orc_q.forward([t], st_q, want_logits=False).hidden[-1][0]
            hp = orc.forward([t], st, want_logits=False).hidden[-1][0]
            hr = ref.hidden.float().cpu()
            ulp = bf16_ulp(float(hr.abs().max()))
            worst_q = max(worst_q, float((hr - hq).abs().max()) / ulp)
            worst_plain = max(worst_plain, float((hr - hp).abs().max()) / ulp)
            worst_mine = max(worst_mine, float((mine._hidden.float().cpu() - hp).abs().max()) / ulp)
        print(f"\nattempt {attempt}: reference decode kernel vs oracle with in-place rotation: {worst_q:.1f} bf16 ulps; "
              f"vs plain oracle: {worst_plain:.1f}; this library vs plain oracle: {worst_mine:.1f}")
        assert worst_mine <= 6.0
        if worst_q < 0.8 * worst_plain:
            ok = True
            break
    assert ok, "the in-place form did not explain the reference kernel's distance to its baseline"


def test_reference_prefill_layers_before_first_attention(pair):
    mine, ref = pair
    S = 200
    ids = torch.tensor(seeded(S, 2, mine.vocab), dtype=torch.int32, device="cuda")
    mine.reset(); ref.reset()
    mine.prefill(ids)
    ref.prefill(ids)
    torch.cuda.synchronize()
    for l in range(3):
        es = float((mine._dn_states[l] - ref.dn[l]).abs().max())
        ec = float((mine._conv_bufs[l] - ref.conv[l]).abs().max())
        rms = float(ref.dn[l].pow(2).mean().sqrt())
        print(f"\nprefill S={S}, DeltaNet layer {l}: state diff {es:.6f} (rms {rms:.5f}), conv diff {ec:.5f}")
        assert (es <= 5e-5 and ec <= 1e-5) if l == 0 else (es <= 2e-3 and ec <= 0.1)
    assert float((mine._fa_v_cache[0].float()[:, :S] - ref.v[0].float()[:, :S]).abs().max()) <= 0.07
