"""Prefill with NVFP4 weights and NVFP4 activations on the block-scaled tensor cores (mk_prefill_nvfp4_mma) against the
CPU oracle run on the dequantised weights AND with every projection input passed through the same activation
quantiser (oracle/nvfp4.py quantize_b -> dequantize_b, the plain-C restatement of the reference's 16-block E4M3
quantiser).  The library is switched to the restatement's IEEE arithmetic for these tests, so device and oracle
quantise identically up to inputs that differ by earlier rounding.

What can and cannot be bounded.  The quantiser (bit-exact, test_nvfp4.py) and the block-scaled GEMM (exact product of
the dequantised operands, test_gemm_nvfp4_gpu.py) are pinned on their own; this file checks that the prefill wires
them correctly.  A 4-bit activation turns a one-ulp difference of its bf16 input (a different summation order
upstream) into a jump of a whole e2m1 step, so from the second quantisation point of a layer on, device and oracle
take different rounding decisions and drift apart by a sizeable fraction of the quantisation effect itself: on the
CPU, perturbing 5 % of the oracle's projection inputs by one bf16 ulp moves its output by 0.7-0.9 of the distance
between the oracle with and without activation quantisation.  Bounds are therefore relative to that distance n
(rms over the compared tensor):
  * up to the first re-quantisation the paths agree tightly: the DeltaNet state of a one-layer model (quantised
    input -> qkv / z GEMMs -> convolution -> recurrence) matches the quantised oracle to 0.1 n;
  * everything else must be closer to the quantised oracle than to the unquantised one, and within 0.95 n of it
    (measured 0.57-0.83 n); wrong wiring (another matrix, scale tiles of another layout, a wrong row stride) lands at
    several n;
  * the first generated token is the quantised oracle's, or its logit is within the stated margin.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import nvfp4, qwen35_oracle as O  # noqa: E402
from test_nvfp4_ts_decode_gpu import dequantised_state_dict  # noqa: E402

V = 2048


def act_quant(x):
    """[T, K] f32 -> values of the NVFP4 activation the device multiplies (bf16 input, 16-blocks, E4M3 scales)."""
    T, K = x.shape
    pad = (-T) % 128
    xb = torch.cat([x, x.new_zeros(pad, K)]).to(torch.bfloat16)
    out = nvfp4.dequantize_b(*nvfp4.quantize_b(xb))
    return torch.from_numpy(out[:T].copy())


@pytest.fixture(scope="module")
def ieee_quantiser():
    import luce_megakernel_b200 as L
    lib = L.lib()
    lib.mk_set_quantize_arithmetic(0)
    yield lib
    lib.mk_set_quantize_arithmetic(1)


def _rms(x):
    return float(x.float().pow(2).mean().sqrt())


@pytest.mark.parametrize("layers,S", [(1, 40), (2, 64), (4, 200), (8, 520)])
def test_prefill_nvfp4_mma_matches_quantised_oracle(ieee_quantiser, layers, S):
    from luce_megakernel_b200 import model as M, model_nvfp4 as MQ
    sd = O.init_weights(3, layers, V, norm_init="unit")
    dec = MQ.DecoderTS(M.weights_from_state_dict(sd), max_seq_len=1024)
    dq = dequantised_state_dict(sd)
    g = torch.Generator().manual_seed(17 + S)
    prompt = torch.randint(0, V, (S,), generator=g).tolist()
    tok = dec.prefill(prompt)
    assert ieee_quantiser.mk_prefill_status() == 0 and ieee_quantiser.mk_gemm_nvfp4_status() == 0
    st_q, st = O.State.new(layers, 1024, V), O.State.new(layers, 1024, V)
    tr_q = O.Oracle(dq, rounding="decode", act_quant=act_quant).forward(prompt, st_q)
    tr = O.Oracle(dq, rounding="decode").forward(prompt, st)

    def check(name, got, ref_q, ref_n, frac=0.95):
        n, e_q, e_n = _rms(ref_q - ref_n), _rms(got - ref_q), _rms(got - ref_n)
        assert n > 0, name
        assert e_q <= frac * n, f"{name}: {e_q} from the quantised oracle, quantisation effect {n}"
        assert e_q < e_n, f"{name}: closer to the unquantised oracle ({e_n}) than to the quantised one ({e_q})"

    check("last hidden state", dec._hidden.float().cpu(), tr_q.hidden[-1][-1], tr.hidden[-1][-1])
    check("DeltaNet state", dec._dn_states.cpu(), st_q.dn_states, st.dn_states, 0.1 if layers == 1 else 0.95)
    check("conv window", dec._conv_bufs.cpu(), st_q.conv_bufs, st.conv_bufs, 0.1 if layers == 1 else 0.95)
    if layers >= 4:
        check("K cache", dec._fa_k_cache[:, :, :S].float().cpu(), st_q.k_cache[:, :, :S], st.k_cache[:, :, :S])
        check("V cache", dec._fa_v_cache[:, :, :S].float().cpu(), st_q.v_cache[:, :, :S], st.v_cache[:, :, :S])
    n_l = float((tr_q.logits - tr.logits).abs().max())
    assert tok == tr_q.token or float(tr_q.logits[tr_q.token] - tr_q.logits[tok]) <= n_l, (tok, tr_q.token)


def test_decode_continues_from_the_nvfp4_prefill(ieee_quantiser):
    """The state mk_prefill_nvfp4_mma leaves is the one the NVFP4 decode kernels continue from: 8 greedy steps run and
    agree with the oracle's greedy continuation wherever the oracle's own top-2 margin is clear."""
    from luce_megakernel_b200 import model as M, model_nvfp4 as MQ
    sd = O.init_weights(3, 4, V, norm_init="unit")
    dec = MQ.DecoderTS(M.weights_from_state_dict(sd), max_seq_len=256)
    orc_q = O.Oracle(dequantised_state_dict(sd), rounding="decode", act_quant=act_quant)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, V, (96,), generator=g).tolist()
    t = dec.prefill(prompt)
    out = dec.step_many(t, 8).cpu().tolist()
    assert all(0 <= x < V for x in out)
    assert ieee_quantiser.mk_device_status() == 0
