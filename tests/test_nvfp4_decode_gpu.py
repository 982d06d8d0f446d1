"""NVFP4 decode against the CPU oracle run on the dequantised weights (the C oracle's
quantise -> dequantise of the same bf16 weights), token by token, teacher forced."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import nvfp4, qwen35_oracle as O  # noqa: E402

NL, V, MAXSEQ = 8, 2048, 128
_QUANT = ("in_proj_qkv", "in_proj_z", "out_proj", "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def dequantised_state_dict(sd):
    out = {}
    for k, w in sd.items():
        if w.dim() == 2 and any(q in k for q in _QUANT):
            p, s = nvfp4.quantize_a(w, 32)
            out[k] = torch.from_numpy(nvfp4.dequantize_a(p, s, 32))
        else:
            out[k] = w.float()
    p, s = nvfp4.quantize_b(sd["model.embed_tokens.weight"])
    out["lm_head.weight"] = torch.from_numpy(nvfp4.dequantize_b(p, s))
    return out


def bf16_ulp(x):
    import math
    return 2.0 ** (math.floor(math.log2(max(x, 1e-30))) - 7)


@pytest.fixture(scope="module")
def setup(small_model):
    from luce_megakernel_b200 import model as M, model_nvfp4 as MQ
    sd, _ = small_model("unit", "decode")
    import luce_megakernel_b200 as L
    L.lib().mk_set_quantize_arithmetic(0)      # the oracle's weights come from the C restatement (IEEE divides)
    try:
        dec = MQ.Decoder(M.weights_from_state_dict(sd), max_seq_len=MAXSEQ)
        torch.cuda.synchronize()
    finally:
        L.lib().mk_set_quantize_arithmetic(1)
    orc = O.Oracle(dequantised_state_dict(sd), rounding="decode")
    return dec, orc


def test_nvfp4_decode_matches_oracle(setup):
    dec, orc = setup
    dec.reset()
    st = O.State.new(NL, MAXSEQ, V)
    g = torch.Generator().manual_seed(21)
    toks = torch.randint(0, V, (40,), generator=g).tolist()
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


def test_nvfp4_step_many_equals_steps_and_repeats(setup):
    dec, _ = setup
    g = torch.Generator().manual_seed(22)
    toks = torch.randint(0, V, (12,), generator=g).tolist()
    runs = []
    for mode in ("single", "many", "many"):
        dec.reset()
        for t in toks[:-1]:
            dec.step_async(t)
        if mode == "single":
            out, t = [], toks[-1]
            for _ in range(16):
                t = dec.step(t)
                out.append(t)
        else:
            out = dec.step_many(toks[-1], 16).cpu().tolist()
        runs.append((out, dec._dn_states.clone()))
    assert runs[0][0] == runs[1][0] == runs[2][0]
    assert torch.equal(runs[1][1], runs[2][1])


def test_nvfp4_rejects_other_group_sizes(setup):
    import ctypes
    dec, _ = setup
    from luce_megakernel_b200.model import _ptr
    rc = dec._lib.launch_decode_nvfp4(_ptr(dec._out_token), _ptr(dec._out_token), *dec._common_args(), ctypes.c_int(0),
                                      ctypes.c_int(MAXSEQ), ctypes.c_int(64), dec._stream())
    assert rc == 1


def test_nvfp4_ops_surface(setup):
    """torch.ops.qwen35_megakernel_bf16_C.decode_nvfp4 / decode_many_nvfp4 with the reference's schemas."""
    import luce_megakernel_b200 as L
    ops = L.load_ops()
    dec, _ = setup
    e = torch.empty(1, dtype=torch.bfloat16, device="cuda")
    f = torch.empty(1, dtype=torch.float32, device="cuda")
    u = torch.empty(1, dtype=torch.uint8, device="cuda")
    h = torch.empty(1, dtype=torch.float16, device="cuda")
    i = torch.empty(1, dtype=torch.int32, device="cuda")

    def common():
        return (dec._embed_weight, dec._layer_weights_packed, dec._final_norm_weight, dec._lm_packed, dec._lm_scales,
                e, u, u, h, dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs, dec._hidden, f, e, f, f, f,
                f, f, f, f, dec._normalized, i, i, f, i, i)
    g = torch.Generator().manual_seed(23)
    toks = torch.randint(0, V, (6,), generator=g).tolist()
    dec.reset()
    ref = [dec.step(t) for t in toks]
    ref_many = dec.step_many(ref[-1], 5).cpu().tolist()
    dec.reset()
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    got = []
    for p_, t in enumerate(toks):
        ops.decode_nvfp4(out, t, *common(), p_, MAXSEQ, 32)
        got.append(int(out.item()))
    assert got == ref
    many = torch.empty(5, dtype=torch.int32, device="cuda")
    buf = torch.empty(1, dtype=torch.int32, device="cuda")
    ops.decode_many_nvfp4(many, buf, got[-1], *common(), len(toks), MAXSEQ, 32)
    assert many.cpu().tolist() == ref_many
