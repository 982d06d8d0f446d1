"""Oracle parity on the shapes the benchmark reports, at full size.

  * the headline workload itself: 24 layers, vocabulary 248320, seed 0, a 520-token prompt through the
    prefill op, then 128 decode steps (teacher-forced against the oracle with the decode kernel's rounding
    points, plus the free-running token stream and its first divergence);
  * the whole prefill at 8192 tokens on a 4-layer model (3 DeltaNet + 1 attention layer): persistent GEMM
    tiles wrapping around, more than 32 chunk blocks per head in the chunk scan, 128 key tiles per query tile;
  * the prefill attention kernel at 32768 tokens on sampled query rows (first and last tile, rows 127-129
    around a block boundary, the middle), dense and with a block mask;
  * block selection at 65536 tokens (512 blocks per head) with the benchmark's rule, bit for bit.

The comparison is always with the CPU oracle (oracle/), never with another CUDA path.  Bounds are the ones
of tests/test_decode_gpu.py and tests/test_prefill_gpu.py.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import block_sparse as BS  # noqa: E402
from oracle import qwen35_oracle as O  # noqa: E402


def bf16_ulp(x):
    return 2.0 ** (math.floor(math.log2(max(x, 1e-30))) - 7)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


@pytest.mark.parametrize("norm_init", ["literal", "unit"])
def test_headline_workload_pp520_then_tg128(norm_init):
    """BASELINE configs[1] literally.  "literal": every norm tensor is 1.0, as in the benchmark (each (1+w) norm then
    doubles its input, |hidden| reaches ~20 and the bf16 noise of any implementation is large: the bounds below widen
    with the distance between the two oracles); "unit": effective norm weight 1, where the fixed bounds apply."""
    from luce_megakernel_b200 import model as M
    NL, V, S, STEPS, MAXSEQ = 24, O.VOCAB, 520, 128, 2048
    sd = O.init_weights(0, NL, V, norm_init=norm_init)
    orc, o32 = O.Oracle(sd, rounding="decode"), O.Oracle(sd, rounding="none")
    dec = M.Decoder(weights=M.weights_from_state_dict(sd), max_seq_len=MAXSEQ, api="cabi")
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, V, (S,), generator=g).tolist()
    lm = sd["model.embed_tokens.weight"].float()

    first = dec.prefill(prompt)
    st, st32 = O.State.new(NL, S + STEPS + 8, V), O.State.new(NL, S + STEPS + 8, V)
    tr, tr32 = orc.forward(prompt, st), o32.forward(prompt, st32)
    prefill_token = tr.token
    ref_h = tr.hidden[-1][-1]
    eh = float((dec._hidden_bf16_out.float().cpu() - ref_h).abs().max())
    tol = max(2e-2, 4 * bf16_ulp(float(ref_h.abs().max())), 2.0 * float((tr32.hidden[-1][-1] - ref_h).abs().max()))
    assert eh <= tol, f"prefill: last-row hidden error {eh} (bound {tol})"
    logit_tol = max(6e-2, 2.0 * float((tr32.logits - tr.logits).abs().max()))
    el = float((lm @ dec._final_normed.float().cpu() - tr.logits).abs().max())
    assert el <= logit_tol, f"prefill: logit error {el} (bound {logit_tol})"
    # token rule: the chosen token's oracle logit lies within twice the logit bound of the oracle's best
    assert first == tr.token or float(tr.logits[tr.token] - tr.logits[first]) <= 2 * logit_tol
    # the caches the decode steps will read: every prompt position of every attention layer.  Keys reach ~10 here
    # (every (1+w) norm doubles), one bf16 step is 0.06; the bound per layer is the larger of 0.13 and twice the
    # distance between the two oracles' caches (what the bf16 rounding points alone move a cache entry by)
    for name, got, a, b in (("K", dec._fa_k_cache, st.k_cache, st32.k_cache), ("V", dec._fa_v_cache, st.v_cache, st32.v_cache)):
        for l in range(got.shape[0]):
            bound = max(0.13, 2.0 * float((a[l, :, :S] - b[l, :, :S]).abs().max()))
            err = float((got[l].float().cpu()[:, :S] - a[l, :, :S]).abs().max())
            assert err <= bound, f"{name} cache of attention layer {l}: error {err} (bound {bound})"
    assert float((dec._dn_states.cpu() - st.dn_states).abs().max()) < 2e-2

    # 128 decode steps from the prefill's state, teacher-forced with the oracle's tokens
    ck = dec.state_dict()
    oracle_tokens, feed, worst_h, worst_l = [], tr.token, 0.0, 0.0
    for i in range(STEPS):
        got = dec.step(feed)
        tr, tr32 = orc.forward([feed], st), o32.forward([feed], st32)
        ref_h = tr.hidden[-1][0]
        eh = float((dec._hidden.float().cpu() - ref_h).abs().max())
        h_tol = max(2e-2, 4 * bf16_ulp(float(ref_h.abs().max())), 2.0 * float((tr32.hidden[-1][0] - ref_h).abs().max()))
        assert eh <= h_tol, f"step {i} (position {S + i}): hidden error {eh} (bound {h_tol})"
        logit_tol = max(5e-2, 2.0 * float((tr32.logits - tr.logits).abs().max()))
        el = float((lm @ dec._normalized.cpu() - tr.logits).abs().max())
        assert el <= logit_tol, f"step {i}: logit error {el} (bound {logit_tol})"
        top = torch.topk(tr.logits, 2)
        margin = float(top.values[0] - top.values[1])
        assert got == tr.token or float(tr.logits[tr.token] - tr.logits[got]) <= 2 * logit_tol, \
            f"step {i}: token {got} vs {tr.token} (top-2 margin {margin}, bound {2 * logit_tol})"
        worst_h, worst_l = max(worst_h, eh), max(worst_l, el)
        oracle_tokens.append((tr.token, margin, logit_tol))
        feed = tr.token
    print(f"\npp520+tg128 teacher-forced: worst hidden error {worst_h:.4g}, worst logit error {worst_l:.4g}")

    # the benchmark's own loop: free-running greedy decode with device token feedback from the same state
    dec.load_state_dict(ck)
    free = dec.step_many(first, STEPS).cpu().tolist()
    # the oracle stream above is the oracle's own greedy continuation (it was fed its own tokens)
    want = [t for t, _, _ in oracle_tokens]
    if first != prefill_token:
        print("free-running: the prefill's first token already differs from the oracle's (accepted above at low margin)")
        return
    k = next((i for i, (a, b) in enumerate(zip(free, want)) if a != b), STEPS)
    if k < STEPS:
        _, margin, lt = oracle_tokens[k]
        print(f"free-running: first divergence at step {k} of {STEPS}, oracle margin {margin:.4g} (logit bound {lt:.4g})")
        assert margin <= 2 * lt, "free-running tokens diverged at a step where the oracle's margin is not small"
    else:
        print(f"free-running: all {STEPS} greedy tokens identical to the oracle")


def test_prefill_8192_tokens_four_layers():
    from luce_megakernel_b200 import model as M, lib
    NL, V, S = 4, 2048, 8192
    sd = O.init_weights(0, NL, V, norm_init="unit")
    orc, o32 = O.Oracle(sd, rounding="decode"), O.Oracle(sd, rounding="none")
    dec = M.Decoder(weights=M.weights_from_state_dict(sd), max_seq_len=S + 8, api="cabi")
    g = torch.Generator().manual_seed(8192)
    toks = torch.randint(0, V, (S,), generator=g).tolist()
    tok = dec.prefill(toks)
    assert lib().mk_prefill_status() == 0
    st = O.State.new(NL, S + 8, V)
    tr = orc.forward(toks, st)
    st32 = O.State.new(NL, S + 8, V)
    tr32 = o32.forward(toks, st32)
    ref_h = tr.hidden[-1][-1]
    eh = float((dec._hidden_bf16_out.float().cpu() - ref_h).abs().max())
    tol = max(2e-2, 4 * bf16_ulp(float(ref_h.abs().max())), 2.0 * float((tr32.hidden[-1][-1] - ref_h).abs().max()))
    assert eh <= tol, f"hidden error {eh} (bound {tol})"
    lm = sd["model.embed_tokens.weight"].float()
    logit_tol = max(6e-2, 2.0 * float((tr32.logits - tr.logits).abs().max()))
    assert float((lm @ dec._final_normed.float().cpu() - tr.logits).abs().max()) <= logit_tol
    top = torch.topk(tr.logits, 2)
    assert tok == tr.token or (float(top.values[0] - top.values[1]) <= 0.1 and tok in top.indices.tolist())
    # keys and values of the attention layer at every one of the 8192 positions: each is a function of the three
    # DeltaNet layers' outputs at that position, so this checks every row of the chunked scan, not only the last
    kerr = (dec._fa_k_cache.float().cpu()[:, :, :S] - st.k_cache[:, :, :S]).abs()
    verr = (dec._fa_v_cache.float().cpu()[:, :, :S] - st.v_cache[:, :, :S]).abs()
    kb = max(0.13, 2.0 * float((st.k_cache[:, :, :S] - st32.k_cache[:, :, :S]).abs().max()))
    vb = max(0.13, 2.0 * float((st.v_cache[:, :, :S] - st32.v_cache[:, :, :S]).abs().max()))
    assert float(kerr.max()) <= kb and float(verr.max()) <= vb, (float(kerr.max()), kb, float(verr.max()), vb)
    assert float(dec._fa_k_cache[:, :, S:].abs().max()) == 0.0
    assert float((dec._dn_states.cpu() - st.dn_states).abs().max()) < 2e-2
    assert float((dec._conv_bufs.cpu() - st.conv_bufs).abs().max()) < 0.1
    print(f"\nprefill 8192: hidden error {eh:.4g} (bound {tol:.4g}), K error {float(kerr.max()):.4g}, "
          f"state error {float((dec._dn_states.cpu() - st.dn_states).abs().max()):.4g}")


def _make_qkv(S, seed):
    """qkv [S, 5120] bf16 = 8 x [q | gate], k, v with some block structure in the keys; caches filled from it."""
    g = torch.Generator().manual_seed(seed)
    qkv = torch.empty(S, 5120, dtype=torch.bfloat16)
    for r0 in range(0, S, 8192):
        r1 = min(S, r0 + 8192)
        qkv[r0:r1] = (torch.randn(r1 - r0, 5120, generator=g) * 0.7).to(torch.bfloat16)
    drift = torch.randn((S + 127) // 128, 512, generator=g).repeat_interleave(128, 0)[:S] * 0.5
    qkv[:, 4096:4608] = (qkv[:, 4096:4608].float() + drift).to(torch.bfloat16)
    kc = qkv[:, 4096:4608].reshape(S, 2, 256).transpose(0, 1).contiguous()
    vc = qkv[:, 4608:5120].reshape(S, 2, 256).transpose(0, 1).contiguous()
    return qkv, kc, vc


def _select(lib, dq, dk, S, top_frac, window, sink):
    nblk = (S + 127) // 128
    nwords = (nblk + 31) // 32
    lib.mk_block_select_scratch_bytes.restype = ctypes.c_size_t
    scratch = torch.empty(lib.mk_block_select_scratch_bytes(S), dtype=torch.uint8, device="cuda")
    mask = torch.zeros(8, nblk, nwords, dtype=torch.int32, device="cuda")
    rc = lib.mk_block_select(_ptr(dq), _ptr(dk), S, S, ctypes.c_double(top_frac), window, sink, _ptr(mask), _ptr(scratch),
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    words = mask.cpu().numpy().astype(np.uint32)
    bits = ((words[..., None] >> np.arange(32, dtype=np.uint32)) & 1).astype(bool).reshape(8, nblk, nwords * 32)[..., :nblk]
    return mask, bits


def _attention_rows(qkv, kc, vc, rows, keep=None):
    """softmax(q k^T / 16) v * sigmoid(gate) for the given query positions, fp32 on the CPU:
    the oracle's attention arithmetic (oracle/qwen35_oracle.py, Oracle._attention) on the rows asked for."""
    out = torch.empty(len(rows), 8, 256)
    for i, r in enumerate(rows):
        q = qkv[r, :4096].reshape(8, 512).float()
        for h in range(8):
            K, Vv = kc[h // 4, :r + 1].float(), vc[h // 4, :r + 1].float()
            s = (K @ q[h, :256]) / 16.0
            if keep is not None:
                kept = torch.from_numpy(keep[h, r // 128])[torch.arange(r + 1) // 128]
                s = s.masked_fill(~kept, float("-inf"))
            out[i, h] = (torch.softmax(s, 0) @ Vv) * torch.sigmoid(q[h, 256:])
    return out.reshape(len(rows), 2048)


@pytest.mark.parametrize("sparse", [False, True])
def test_attention_32768_sampled_rows(sparse):
    import luce_megakernel_b200 as L
    lib = L.lib()
    S = 32768
    qkv, kc, vc = _make_qkv(S, 32768)
    dq, dk, dv = qkv.cuda(), kc.cuda(), vc.cuda()
    keep, mask = None, None
    if sparse:
        mask, keep = _select(lib, dq, dk, S, 0.10, 4, 1)
        assert not keep.reshape(8, -1).all(axis=1).any()
    out = torch.empty(S, 2048, dtype=torch.bfloat16, device="cuda")
    rc = lib.mk_attention_prefill(_ptr(dq), _ptr(dk), _ptr(dv), _ptr(out), S, S, _ptr(mask),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert lib.mk_prefill_status() == 0
    rows = [0, 1, 31, 32, 63, 127, 128, 129, 255, 4095, 4096, 16383, 16384, 16511, 16512, 32639, 32640, 32641,
            32735, 32736, 32766, 32767]
    ref = _attention_rows(qkv, kc, vc, rows, keep)
    got = out[torch.tensor(rows, device="cuda")].float().cpu()
    err = (got - ref).abs().max(dim=1).values
    worst = int(err.argmax())
    assert float(err.max()) <= 2e-2, f"attention error {float(err.max())} at row {rows[worst]}"


def test_block_selection_65536_bit_exact():
    """The long-prompt configuration: 512 key blocks per head, sink 1 + window 4 + top 10 % (up to 52 ranked blocks)."""
    import luce_megakernel_b200 as L
    lib = L.lib()
    S = 65536
    qkv, kc, _ = _make_qkv(S, 65536)
    _, bits = _select(lib, qkv.cuda(), kc.cuda(), S, 0.10, 4, 1)
    q = qkv[:, :4096].reshape(S, 8, 512)[:, :, :256].permute(1, 0, 2).float().numpy()
    ref = BS.select_for_heads(q, kc.float().numpy(), top_frac=0.10, window=4, sink=1)
    assert ref.shape == bits.shape == (8, 512, 512)
    assert (bits == ref).all(), f"{int((bits != ref).sum())} block decisions differ"
    assert int(ref[0, 511].sum()) >= 52
