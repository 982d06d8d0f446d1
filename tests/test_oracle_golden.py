"""The CPU oracle against the vectors recorded from the reference's PyTorch path
(transformers Qwen3_5ForCausalLM, fp32; see tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from oracle import qwen35_oracle as O


@pytest.mark.parametrize("norm_init", ["literal", "unit"])
def test_oracle_matches_hf_golden(golden, norm_init):
    NL, V, PL, ND, SEED = (int(x) for x in golden["meta"])
    w = O.init_weights(SEED, NL, V, norm_init=norm_init)
    orc = O.Oracle(w, rounding="none")
    st = O.State.new(NL, 64, V)
    pre = norm_init + "_"
    prompt = golden[pre + "prompt"]
    # the committed prompt is what the seeded generator yields
    g = torch.Generator().manual_seed(SEED)
    assert torch.randint(0, V, (PL,), generator=g).tolist() == prompt.tolist()

    tr = orc.forward(prompt, st)
    tokens = [tr.token]
    hid = torch.tensor(golden[pre + "hidden_last"])
    logits = torch.tensor(golden[pre + "logits"])
    scale = float(hid.abs().max())
    tol_h = 2e-5 * max(1.0, scale)
    for l in range(NL):
        assert (tr.hidden[l][-1] - hid[0, l]).abs().max() < tol_h
    assert (tr.hidden[-1] - torch.tensor(golden[pre + "prefill_rows_last_layer"])).abs().max() < tol_h
    assert (tr.logits - logits[0]).abs().max() < 1e-4
    for s in range(ND):
        tr = orc.forward([int(golden[pre + "tokens"][s])], st)
        tokens.append(tr.token)
        for l in range(NL):
            assert (tr.hidden[l][-1] - hid[s + 1, l]).abs().max() < tol_h
        assert (tr.logits - logits[s + 1]).abs().max() < 1e-4
    assert tokens == golden[pre + "tokens"].tolist()
    # session state in the op layouts: dn_states [value][key], conv window, post-RoPE keys
    L = PL + ND
    assert (st.dn_states[0, 0] - torch.tensor(golden[pre + "dn_state_l0_h0"])).abs().max() < 1e-6
    assert (st.dn_states[0].sum(dim=(-1, -2)) - torch.tensor(golden[pre + "dn_state_l0_sum"])).abs().max() < 1e-4
    assert (st.conv_bufs[0, :64] - torch.tensor(golden[pre + "conv_l0_first64"])).abs().max() < 1e-6
    assert (st.k_cache[0, 0, :L] - torch.tensor(golden[pre + "k_l3_h0"])).abs().max() < 1e-4
    assert (st.v_cache[0, 1, L - 1] - torch.tensor(golden[pre + "v_l3_h1_last"])).abs().max() < 1e-5


def test_prefill_equals_token_by_token(small_model):
    """One multi-token forward and the same tokens fed one at a time leave the same state
    (the reference's own structural check, megakernel/bench_pp_tg.py:80-131)."""
    sd, orc = small_model("unit", "none")
    g = torch.Generator().manual_seed(3)
    toks = torch.randint(0, 2048, (12,), generator=g).tolist()
    a, b = O.State.new(8, 32, 2048), O.State.new(8, 32, 2048)
    ta = orc.forward(toks, a)
    for t in toks:
        tb = orc.forward([t], b)
    assert (ta.logits - tb.logits).abs().max() < 1e-4
    assert ta.token == tb.token
    assert (a.dn_states - b.dn_states).abs().max() < 1e-5
    assert (a.k_cache - b.k_cache).abs().max() < 1e-5
    assert (a.conv_bufs - b.conv_bufs).abs().max() < 1e-5


def test_decode_rounding_stays_close_to_fp32(small_model):
    """The bf16 rounding points of the decode path move the logits by far less than the
    5e-2 budget on this model."""
    sd, o32 = small_model("unit", "none")
    _, obf = small_model("unit", "decode")
    toks = [5, 900, 77, 1500]
    a, b = O.State.new(8, 16, 2048), O.State.new(8, 16, 2048)
    la, lb = o32.forward(toks, a).logits, obf.forward(toks, b).logits
    assert (la - lb).abs().max() < 5e-2


def test_repetition_penalty_rule(small_model):
    sd, orc = small_model("unit", "none")
    st = O.State.new(8, 16, 2048)
    base = orc.forward([7, 8, 9], st.clone()).logits
    pen = orc.forward([7, 8, 9], st.clone(), repetition_penalty=1.5).logits
    for t in (7, 8, 9):
        exp = base[t] / 1.5 if base[t] > 0 else base[t] * 1.5
        assert abs(float(pen[t] - exp)) < 1e-6
    mask = torch.ones(2048, dtype=torch.bool)
    mask[[7, 8, 9]] = False
    assert torch.equal(pen[mask], base[mask])
