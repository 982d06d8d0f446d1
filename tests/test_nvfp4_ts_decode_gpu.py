"""Decode on the NVFP4 format with a per-tensor scale (16-element blocks, E4M3 block scales, fp32 scale per matrix,
every linear layer and the LM head) against the CPU oracle run on the dequantised weights -- the plain-C
restatement's quantise -> dequantise of the same bf16 weights (oracle/nvfp4_oracle.c, mk_oracle_quantize_ts /
mk_oracle_dequantize_ts) -- token by token, teacher forced.  Bounds are those of the bf16 decode tests."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import nvfp4, qwen35_oracle as O  # noqa: E402

NL, V, MAXSEQ = 8, 2048, 256
_QUANT = ("in_proj_qkv", "in_proj_z", "out_proj", "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def dequantised_state_dict(sd):
    out = {}
    for k, w in sd.items():
        if w.dim() == 2 and any(q in k for q in _QUANT):
            out[k] = torch.from_numpy(nvfp4.dequantize_ts(*nvfp4.quantize_ts(w)))
        else:
            out[k] = w.float()
    out["lm_head.weight"] = torch.from_numpy(nvfp4.dequantize_ts(*nvfp4.quantize_ts(sd["model.embed_tokens.weight"])))
    return out


def bf16_ulp(x):
    return 2.0 ** (math.floor(math.log2(max(x, 1e-30))) - 7)


def _make_decoder(kind, weights, max_seq_len):
    """kind: "ts" = mma.sync kernel (mk_decode_nvfp4_ts); "mma8" / "mma4" = block-scaled tcgen05 kernel
    (mk_decode_nvfp4_mma) with the activation expanded into 8 / 4 NVFP4 residual terms."""
    from luce_megakernel_b200 import model_nvfp4 as MQ
    if kind == "ts":
        return MQ.DecoderTS(weights, max_seq_len=max_seq_len)
    return MQ.DecoderMMA(weights, max_seq_len=max_seq_len, act_terms=int(kind[3:]))


@pytest.fixture(scope="module", params=["ts", "mma8", "mma4"])
def setup(request, small_model):
    from luce_megakernel_b200 import model as M
    sd, _ = small_model("unit", "decode")
    dec = _make_decoder(request.param, M.weights_from_state_dict(sd), MAXSEQ)
    orc = O.Oracle(dequantised_state_dict(sd), rounding="decode")
    return dec, orc


def test_packed_weights_equal_the_restatement(setup, small_model):
    """What the decode kernel streams is what the C restatement produces: codes, block scales (as plain rows) and the
    tensor scale of one matrix of each shape."""
    dec, _ = setup
    sd, _ = small_model("unit", "decode")
    nv = dec._weights["nvfp4_ts"]
    for key, slot in (("model.layers.0.linear_attn.in_proj_qkv.weight", 1), ("model.layers.0.linear_attn.out_proj.weight", 13),
                      ("model.layers.0.mlp.down_proj.weight", 23)):
        w = sd[key]
        rp, rs_tiled, rts = nvfp4.quantize_ts(w)
        rows, cols = w.shape
        packed, srows, ts = nv["layer_data"][0]["ptrs"][slot:slot + 3]
        assert np.array_equal(packed.cpu().numpy(), rp)
        assert float(ts[0].item()) == float(np.asarray(rts).reshape(-1)[0])
        r = np.arange(rows)[:, None]
        c = np.arange(cols // 16)[None, :]
        idx = ((r >> 7) * (cols // 64) + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3)
        assert np.array_equal(srows.cpu().numpy(), np.asarray(rs_tiled).reshape(-1)[idx])


def test_ts_decode_matches_oracle(setup):
    dec, orc = setup
    dec.reset()
    st = O.State.new(NL, MAXSEQ, V)
    g = torch.Generator().manual_seed(31)
    toks = torch.randint(0, V, (72,), generator=g).tolist()      # crosses one 64-position attention chunk
    for i, t in enumerate(toks):
        tok = dec.step(t)
        tr = orc.forward([t], st)
        ref_h = tr.hidden[-1][0]
        eh = float((dec._hidden.float().cpu() - ref_h).abs().max())
        assert eh <= max(2e-2, 4 * bf16_ulp(float(ref_h.abs().max()))), f"pos {i}: hidden error {eh}"
        logits = orc.lm_head @ dec._normalized.cpu()
        assert float((logits - tr.logits).abs().max()) <= 5e-2
        top = torch.topk(tr.logits, 2)
        margin = float(top.values[0] - top.values[1])
        assert tok == tr.token or (margin <= 0.1 and tok in top.indices.tolist()), f"pos {i}: {tok} vs {tr.token}"
    assert float((dec._dn_states.cpu() - st.dn_states).abs().max()) < 5e-3


def test_ts_one_launch_equals_single_steps(setup):
    dec, _ = setup
    g = torch.Generator().manual_seed(32)
    toks = torch.randint(0, V, (12,), generator=g).tolist()
    runs = []
    for mode in ("single", "many", "many"):
        dec.reset()
        for t in toks[:-1]:
            dec.step_many(t, 1)
        if mode == "single":
            out, t = [], toks[-1]
            for _ in range(24):
                t = dec.step(t)
                out.append(t)
        else:
            out = dec.step_many(toks[-1], 24).cpu().tolist()
        runs.append((out, dec._dn_states.clone(), dec._fa_k_cache.clone()))
    assert runs[0][0] == runs[1][0] == runs[2][0]
    assert torch.equal(runs[0][1], runs[1][1]) and torch.equal(runs[1][1], runs[2][1])
    assert torch.equal(runs[0][2], runs[1][2])


@pytest.mark.parametrize("kind", ["ts", "mma8", "mma4"])
def test_ts_full_size_model_short_run(kind):
    """24 layers, vocabulary 248320: 8 prompt tokens and 8 teacher-forced steps against the oracle on dequantised weights."""
    from luce_megakernel_b200 import model as M
    sd = O.init_weights(0, 24, O.VOCAB, norm_init="unit")
    dec = _make_decoder(kind, M.weights_from_state_dict(sd), 64)
    dq = dequantised_state_dict(sd)
    orc, o32 = O.Oracle(dq, rounding="decode"), O.Oracle(dq, rounding="none")
    g = torch.Generator().manual_seed(33)
    toks = torch.randint(0, O.VOCAB, (16,), generator=g).tolist()
    st, st32 = O.State.new(24, 64, O.VOCAB), O.State.new(24, 64, O.VOCAB)
    for i, t in enumerate(toks):
        tok = dec.step(t)
        tr, tr32 = orc.forward([t], st), o32.forward([t], st32)
        ref_h = tr.hidden[-1][0]
        eh = float((dec._hidden.float().cpu() - ref_h).abs().max())
        h_tol = max(2e-2, 4 * bf16_ulp(float(ref_h.abs().max())), 2.0 * float((tr32.hidden[-1][0] - ref_h).abs().max()))
        assert eh <= h_tol, f"pos {i}: hidden error {eh} (bound {h_tol})"
        logit_tol = max(5e-2, 2.0 * float((tr32.logits - tr.logits).abs().max()))
        el = float((orc.lm_head @ dec._normalized.cpu() - tr.logits).abs().max())
        assert el <= logit_tol, f"pos {i}: logit error {el} (bound {logit_tol})"
        assert tok == tr.token or float(tr.logits[tr.token] - tr.logits[tok]) <= 2 * logit_tol
