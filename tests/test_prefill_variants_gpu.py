"""The reference's other prefill entry points (prefill_bf16_mega, prefill_megakernel_nvfp4,
prefill_bf16_nvfp4_lm) on the 8-layer test model.

* per-matrix GEMMs (no fused weight tensors) must reproduce the fused path bit for bit;
* the NVFP4 prefill must agree with feeding the same prompt through the NVFP4 decode kernel (both
  use the same quantised weights; the prefill rounds the dequantised matrices to bf16, the decode
  kernel does not, so the bound is the bf16-noise bound of the other prefill tests);
* bf16 layers + NVFP4 LM head: the hidden state is the bf16 prefill's, the token is the argmax of the
  dequantised LM head applied to the final-normed vector.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

NL, V, MAXSEQ = 8, 2048, 512


def bf16_ulp(x):
    return 2.0 ** (math.floor(math.log2(max(x, 1e-30))) - 7)


def prompt(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, V, (n,), generator=g).tolist()


@pytest.fixture(scope="module")
def weights(small_model):
    from luce_megakernel_b200 import model as M
    sd, _ = small_model("unit", "decode")
    return M.weights_from_state_dict(sd)


def test_per_matrix_gemms_equal_fused(weights):
    from luce_megakernel_b200 import model as M
    dec = M.Decoder(weights=weights, max_seq_len=MAXSEQ, api="cabi")
    toks = prompt(150, 3)
    dec.reset()
    a = dec.prefill(toks)
    ha, sa, ka = dec._hidden_bf16_out.clone(), dec._dn_states.clone(), dec._fa_k_cache.clone()
    # the same call without the fused tensors
    ids = torch.tensor(toks, dtype=torch.int32, device="cuda")
    dec.reset()
    L = dec._lib
    p = lambda t: ctypes.c_void_p(t.data_ptr() if t is not None else 0)
    rc = L.mk_prefill_bf16(p(ids), len(toks), p(dec._out_token), p(dec._embed_weight), p(dec._layer_weights_packed),
                           p(dec._final_norm_weight), p(dec._lm_head_weight), p(dec._fa_k_cache), p(dec._fa_v_cache),
                           p(dec._dn_states), p(dec._conv_bufs), p(None), p(None), p(dec._final_normed), p(dec._hidden_bf16_out),
                           MAXSEQ, NL, V, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    assert int(dec._out_token.item()) == a
    assert torch.equal(dec._hidden_bf16_out, ha) and torch.equal(dec._dn_states, sa) and torch.equal(dec._fa_k_cache, ka)


def test_prefill_bf16_mega_op(weights):
    import luce_megakernel_b200 as L
    from luce_megakernel_b200 import model as M
    ops = L.load_ops()
    dec = M.Decoder(weights=weights, max_seq_len=MAXSEQ, api="cabi")
    toks = prompt(70, 4)
    dec.reset()
    want = dec.prefill(toks)
    hw = dec._hidden_bf16_out.clone()
    dec.reset()
    e = torch.empty(1, dtype=torch.bfloat16, device="cuda")
    f = torch.empty(1, dtype=torch.float32, device="cuda")
    i = torch.empty(1, dtype=torch.int32, device="cuda")
    ids = torch.tensor(toks, dtype=torch.int32, device="cuda")
    ops.prefill_bf16_mega(dec._out_token, ids, dec._embed_weight, dec._layer_weights_packed, dec._final_norm_weight,
                          dec._lm_head_weight, dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs,
                          e, e, e, e, e, e, e, e, f, f, dec._final_normed, dec._hidden_bf16_out, f, i)
    assert int(dec._out_token.item()) == want
    assert torch.equal(dec._hidden_bf16_out, hw)


@pytest.mark.parametrize("S", [5, 130])
def test_nvfp4_prefill_matches_nvfp4_decode(weights, S):
    from luce_megakernel_b200 import model_nvfp4 as MQ
    dec = MQ.Decoder(weights, max_seq_len=MAXSEQ)
    toks = prompt(S, 20 + S)
    dec.reset()
    for t in toks[:-1]:
        dec.step_async(t)
    tok_d = dec.step(toks[-1])
    h_d = dec._hidden.float().clone()
    s_d, k_d = dec._dn_states.clone(), dec._fa_k_cache.float().clone()
    logits_margin = None
    tok_p = dec.prefill_tokens(toks, mode="raw")
    h_p = dec._hidden.float()
    ulp = bf16_ulp(float(h_d.abs().max()))
    eh = float((h_p - h_d).abs().max())
    print(f"\nNVFP4 prefill vs NVFP4 decode, S={S}: hidden diff {eh / ulp:.1f} ulps, state diff {float((dec._dn_states - s_d).abs().max()):.5f}")
    assert eh <= 8 * ulp
    assert float((dec._dn_states - s_d).abs().max()) <= 2e-2
    assert float((dec._fa_k_cache.float()[:, :, :S] - k_d[:, :, :S]).abs().max()) <= 0.13
    # continue decoding from the prefilled state: the decode kernel accepts it
    nxt = dec.step_many(tok_p, 4).cpu().tolist()
    assert len(nxt) == 4
    if tok_p != tok_d:
        print(f"first token differs ({tok_p} vs {tok_d}): near-tie between two bf16 pipelines")


def test_bf16_layers_with_nvfp4_lm_head(weights):
    import numpy as np
    from luce_megakernel_b200 import model as M, model_nvfp4 as MQ, lib
    dec = M.Decoder(weights=weights, max_seq_len=MAXSEQ, api="cabi")
    q = MQ.Decoder(weights, max_seq_len=MAXSEQ)
    toks = prompt(90, 8)
    dec.reset()
    dec.prefill(toks)
    tok = q.prefill_tokens(toks, mode="bf16")
    assert torch.equal(q._hidden, dec._hidden_bf16_out)
    # reference logits: dequantised LM head (bit-exact dequantiser) times the final-normed vector
    Wd = torch.empty(V, 1024, dtype=torch.float32, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    assert lib().mk_dequantize_nvfp4(1, p(q._lm_packed), p(q._lm_scales), p(Wd), V, 1024, 16,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    h = dec._hidden_bf16_out.float()
    w = weights["final_norm_weight"].float()
    n = h * torch.rsqrt(h.pow(2).mean() + 1e-6) * (1.0 + w)
    logits = Wd @ n
    top = torch.topk(logits, 2)
    assert tok == int(top.indices[0]) or (float(top.values[0] - top.values[1]) < 1e-3 and tok in top.indices.tolist())
