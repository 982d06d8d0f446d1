"""The batched step on the NVFP4 format with a per-tensor scale (BASELINE's NVFP4 batch-8 case) against per-sequence
oracle runs: prompts go through the bf16 prefill (oracle: bf16 weights), the steps read the 4-bit weights (oracle:
the plain-C restatement's dequantised weights), teacher-forced, with the bounds of the bf16 batched test."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import qwen35_oracle as O  # noqa: E402
from test_nvfp4_ts_decode_gpu import dequantised_state_dict  # noqa: E402
from test_prefill_gpu import bf16_ulp  # noqa: E402

NL, V, MAXSEQ = 8, 2048, 256


def prompt(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, V, (n,), generator=g).tolist()


@pytest.fixture(scope="module")
def setup(small_model):
    from luce_megakernel_b200 import model as M
    sd, orc = small_model("unit", "decode")
    dec = M.Decoder(weights=M.weights_from_state_dict(sd), max_seq_len=MAXSEQ, api="cabi")
    dq = dequantised_state_dict(sd)
    return dec, orc, O.Oracle(dq, rounding="decode"), O.Oracle(dq, rounding="none")


@pytest.mark.parametrize("lengths", [[3, 17, 40, 64, 9, 21, 5, 33], [12] * 11])
def test_nvfp4_batch_follows_oracle_per_sequence(setup, lengths):
    from luce_megakernel_b200 import model as M
    dec, orc_bf16, orc, o32 = setup
    B, steps = len(lengths), 8
    prompts = [prompt(n, 300 + 5 * i + n) for i, n in enumerate(lengths)]
    bd = M.BatchDecoder(dec, B, nvfp4_ts=True)
    bd.prefill(prompts)
    refs = []
    for p in prompts:
        st, st32 = O.State.new(NL, MAXSEQ, V), O.State.new(NL, MAXSEQ, V)
        tr = orc_bf16.forward(p, st)
        o_bf32 = O.Oracle(orc_bf16.w, rounding="none")
        o_bf32.forward(p, st32, want_logits=False)
        toks, hid, hid32, logits = [tr.token], [], [], []
        for _ in range(steps):
            t = orc.forward([toks[-1]], st)
            t32 = o32.forward([toks[-1]], st32, want_logits=False)
            toks.append(t.token); hid.append(t.hidden[-1][-1]); hid32.append(t32.hidden[-1][-1]); logits.append(t.logits)
        refs.append((toks, hid, hid32, logits, st))
    worst = 0.0
    for s in range(steps):
        got = bd.step([refs[b][0][s] for b in range(B)])
        hidden = bd._hidden_bf16_out.float().cpu()
        for b in range(B):
            toks, hid, hid32, logits, _ = refs[b]
            eh = float((hidden[b] - hid[s]).abs().max())
            tol = max(2e-2, 6 * bf16_ulp(float(hid[s].abs().max())), 3.0 * float((hid32[s] - hid[s]).abs().max()))
            worst = max(worst, eh / tol)
            assert eh <= tol, f"sequence {b} step {s}: hidden error {eh} (bound {tol})"
            short = float(logits[s][toks[s + 1]] - logits[s][got[b]])
            assert got[b] == toks[s + 1] or short <= 0.1, f"sequence {b} step {s}: token {got[b]} vs {toks[s + 1]} (gap {short})"
    print(f"\nNVFP4 batch {B}: worst hidden error / bound = {worst:.2f}")
    for b in range(B):
        st = refs[b][4]
        assert float((bd._dn_states[b].cpu() - st.dn_states).abs().max()) < 2e-2


def test_nvfp4_batch_many_equals_single_steps_and_batch1_kernel(setup):
    """Device token feedback equals host-fed steps; and the free-running tokens agree with the batch-1 NVFP4 megakernel
    on most sequences (two kernels with different rounding points: they part at the first near-tie)."""
    from luce_megakernel_b200 import model as M, model_nvfp4 as MQ
    dec = setup[0]
    prompts = [prompt(10 + 3 * i, 50 + i) for i in range(8)]
    a = M.BatchDecoder(dec, 8, nvfp4_ts=True)
    first = a.prefill(prompts)
    many = a.step_many(12).cpu().tolist()
    b = M.BatchDecoder(dec, 8, nvfp4_ts=True)
    b.prefill(prompts)
    single, t = [], first
    for _ in range(12):
        t = b.step(t)
        single.append(t)
    assert many == single
    q = MQ.DecoderTS(dec._weights, max_seq_len=MAXSEQ)
    agree = 0
    for i, p in enumerate(prompts):
        dec.reset()
        f = dec.prefill(p)
        q.adopt_state(dec)
        solo = q.step_many(f, 12).cpu().tolist()
        agree += solo[:6] == [row[i] for row in many][:6]
    assert agree >= 5, f"only {agree} of 8 sequences agree with the batch-1 kernel over 6 steps"
