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

Reference throughput on this GPU is printed next to this library's (pytest -s).
"""
import ctypes
import math
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libref_megakernel.so")
MAXSEQ = 1024


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def bf16_ulp(x):
    return 2.0 ** (math.floor(math.log2(max(x, 1e-30))) - 7)


class RefDecoder:
    """The reference kernels behind their C entry points, with buffers sized as megakernel/model.py:208-240."""

    def __init__(self, lib, mine):
        self.lib, self.m = lib, mine
        dev = "cuda"
        bf, f32, i32 = torch.bfloat16, torch.float32, torch.int32
        self.k = torch.zeros_like(mine._fa_k_cache)
        self.v = torch.zeros_like(mine._fa_v_cache)
        self.dn = torch.zeros_like(mine._dn_states)
        self.conv = torch.zeros_like(mine._conv_bufs)
        self.hidden = torch.zeros(1024, dtype=bf, device=dev)
        self.act = torch.empty(1024 * 8 + 3584, dtype=f32, device=dev)
        self.residual = torch.empty(1024, dtype=bf, device=dev)
        self.qkv = torch.empty(6144, dtype=f32, device=dev)
        self.kv = torch.empty(1024, dtype=f32, device=dev)
        self.attn = torch.empty(2048, dtype=f32, device=dev)
        self.mlp = torch.empty(3584, dtype=f32, device=dev)
        self.z = torch.empty(2048, dtype=f32, device=dev)
        self.beta = torch.empty(16, dtype=f32, device=dev)
        self.alpha = torch.empty(16, dtype=f32, device=dev)
        self.normalized = torch.empty(1024, dtype=f32, device=dev)
        self.bar_c = torch.zeros(1, dtype=i32, device=dev)
        self.bar_g = torch.zeros(1, dtype=i32, device=dev)
        self.bmv = torch.empty(1024, dtype=f32, device=dev)
        self.bmi = torch.empty(1024, dtype=i32, device=dev)
        self.lm_sync = torch.zeros(1, dtype=i32, device=dev)
        self.seen = torch.zeros(mine.vocab, dtype=f32, device=dev)
        self.out = torch.zeros(1, dtype=i32, device=dev)
        self.pos = 0

    def reset(self):
        for t in (self.k, self.v, self.dn, self.conv):
            t.zero_()
        self.pos = 0

    def step_async(self, tok):
        m = self.m
        self.lib.launch_decode(
            ctypes.c_int(int(tok)), _p(self.out), _p(m._embed_weight), _p(m._layer_weights_packed), _p(m._final_norm_weight),
            _p(m._lm_head_weight), _p(self.k), _p(self.v), _p(self.dn), _p(self.conv), _p(self.hidden), _p(self.act),
            _p(self.residual), _p(self.qkv), _p(self.kv), _p(self.attn), _p(self.mlp), _p(self.z), _p(self.beta),
            _p(self.alpha), _p(self.normalized), _p(self.bar_c), _p(self.bar_g), _p(self.bmv), _p(self.bmi),
            _p(self.lm_sync), _p(self.seen), ctypes.c_float(1.0), ctypes.c_int(self.pos), ctypes.c_int(MAXSEQ),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        self.pos += 1

    def step(self, tok):
        self.step_async(tok)
        return int(self.out.item())

    def prefill(self, ids):
        """Scratch sizes: megakernel/final_bench.py:52-63 and megakernel/model.py:262-272, except the two
        projection buffers: the reference writes the fused gate/up output ([S, 7168], prefill.cu:1269) into a
        buffer its callers size for 6144 columns, so they are made 7168 wide here."""
        m, S = self.m, int(ids.numel())
        bf, f32, i32, dev = torch.bfloat16, torch.float32, torch.int32, "cuda"
        mx, spad = 7168, ((S + 31) // 32) * 32
        b = dict(hidden=torch.empty(S * 1024, dtype=bf, device=dev), residual=torch.empty(S * 1024, dtype=bf, device=dev),
                 normalized=torch.empty(S * 1024, dtype=bf, device=dev), proj=torch.empty(S * mx, dtype=bf, device=dev),
                 proj2=torch.empty(S * mx, dtype=bf, device=dev), attn=torch.empty(S * 2048, dtype=bf, device=dev),
                 mlp=torch.empty(S * 3584, dtype=bf, device=dev), dn_out=torch.empty(S * 2048, dtype=bf, device=dev),
                 beta=torch.empty(S * 16, dtype=f32, device=dev), alpha=torch.empty(S * 16, dtype=f32, device=dev),
                 pre=torch.empty(S * 6144, dtype=f32, device=dev), u=torch.empty(spad * 16 * 128, dtype=f32, device=dev),
                 w=torch.empty(spad * 16 * 128, dtype=f32, device=dev), cs=torch.empty(spad * 16, dtype=f32, device=dev),
                 fn=torch.empty(1024, dtype=bf, device=dev), hout=torch.empty(1024, dtype=bf, device=dev))
        self._pf = b
        self.lib.launch_prefill_bf16(
            _p(ids), ctypes.c_int(S), _p(self.out), _p(m._embed_weight), _p(m._layer_weights_packed), _p(m._final_norm_weight),
            _p(m._lm_head_weight), _p(self.k), _p(self.v), _p(self.dn), _p(self.conv), _p(b["hidden"]), _p(b["residual"]),
            _p(b["normalized"]), _p(b["proj"]), _p(b["proj2"]), _p(b["attn"]), _p(b["mlp"]), _p(b["dn_out"]), _p(b["beta"]),
            _p(b["alpha"]), _p(b["pre"]), _p(b["u"]), _p(b["w"]), _p(b["cs"]), _p(m._fused_fa_qkv), _p(m._fused_gate_up),
            _p(b["fn"]), _p(b["hout"]), _p(self.bmv), _p(self.bmi), ctypes.c_int(MAXSEQ),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        self.pos = S
        return int(self.out.item())


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
    return mine, RefDecoder(lib, mine)


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


def test_reference_throughput_beside_ours(pair):
    """Not a parity check: prints the reference kernels' speed on this GPU next to this library's."""
    mine, ref = pair
    S = 520
    ids = torch.tensor(seeded(S, 3, mine.vocab), dtype=torch.int32, device="cuda")
    res = {}
    for name, d in (("reference", ref), ("this library", mine)):
        d.reset(); d.prefill(ids)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            if d is mine:
                d._position = 0
            d.prefill(ids)
        e1.record(); torch.cuda.synchronize()
        pp = S / (e0.elapsed_time(e1) / 3e3)
        t = 11
        e0.record()
        for _ in range(128):
            t = d.step(t)
        e1.record(); torch.cuda.synchronize()
        tg = 128 / (e0.elapsed_time(e1) / 1e3)
        res[name] = (pp, tg)
        print(f"\n{name}: pp520 {pp:.0f} tok/s, tg128 (host token loop) {tg:.0f} tok/s")
    assert res["this library"][1] > 0
