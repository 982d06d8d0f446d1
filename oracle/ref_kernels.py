"""The reference's own decode / prefill kernels behind their C entry points.

TEST INFRASTRUCTURE ONLY: used by tests/ (second parity pin) and by `bench.py --impl reference_gpu` (the
reference's kernels timed on the same GPU), never by the product path.

oracle/build_oracle.py compiles megakernel/kernel.cu and megakernel/prefill.cu of the reference checkout,
unmodified and where they lie, for sm_100a into oracle/_ref/libref_megakernel.so.  RefDecoder drives that
library's launch_decode / launch_prefill_bf16 with buffers sized as megakernel/model.py:208-240 and
megakernel/final_bench.py:52-63 size them, on the weights and pointer table of a luce_megakernel_b200.model.Decoder.
"""
import ctypes
import os

import torch

REF_LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref_megakernel.so")


def load_ref_lib():
    """ctypes handle of the compiled reference kernels, or None when they were not built."""
    return ctypes.CDLL(REF_LIB) if os.path.exists(REF_LIB) else None


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


class RefDecoder:
    def __init__(self, lib, mine, max_seq_len=None):
        self.lib, self.m = lib, mine
        self.max_seq_len = int(max_seq_len or mine.max_seq_len)
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
            _p(self.lm_sync), _p(self.seen), ctypes.c_float(1.0), ctypes.c_int(self.pos), ctypes.c_int(self.max_seq_len),
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
        bf, f32, dev = torch.bfloat16, torch.float32, "cuda"
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
            _p(b["fn"]), _p(b["hout"]), _p(self.bmv), _p(self.bmi), ctypes.c_int(self.max_seq_len),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        self.pos = S
        return int(self.out.item())
