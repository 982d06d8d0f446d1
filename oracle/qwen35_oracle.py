"""CPU fp32 oracle for the Qwen3.5-0.8B-architecture hybrid decode / prefill path.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA path: it may be
imported by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline legs and
by nothing else.  The product path never routes through it.

It restates, in plain PyTorch on the CPU, the arithmetic of the reference decode
megakernel (reference: megakernel/kernel.cu) for one or more consecutive tokens:

  * residual stream and (1+w) RMSNorm ........ kernel.cu:189-231, 905-920
  * Gated DeltaNet mixer ..................... kernel.cu:594-757
      conv1d(k=4)+SiLU  kernel.cu:633-648,   gates  kernel.cu:651-658,
      L2 norms          kernel.cu:662-672,   delta rule on S[value][key]  kernel.cu:686-713,
      gated RMSNorm (plain w) * SiLU(z)      kernel.cu:715-728
  * gated GQA attention mixer ................ kernel.cu:425-588
      per-head RMSNorm(1+w) + partial RoPE (first 64 of 256 dims, rotate-half, theta 1e7)
      kernel.cu:456-503, online softmax over the bf16 KV cache kernel.cu:506-560,
      sigmoid output gate kernel.cu:551-556
  * SwiGLU MLP ............................... kernel.cu:313-384
  * LM head + greedy argmax (+ repetition penalty) kernel.cu:763-826

The reference has no CPU implementation of its own; its PyTorch path is the
third-party `transformers` model `Qwen3_5ForCausalLM` (megakernel/final_bench.py:117).
Parity pin: with `rounding="none"` this oracle is checked against that model
(transformers 5.5.0) on seeded random weights; the vectors are committed under
tests/golden/ together with the script that generated them.

`rounding="decode"` additionally applies the bf16 rounding points of the reference
decode kernel (normed activations, residual stream and the KV cache are bf16; everything
else is f32) so that a bf16 GPU path can be compared at tight tolerance.

Tensor layouts are the ones the reference's Python driver allocates
(megakernel/model.py:208-240):
  fa_k_cache / fa_v_cache : [n_fa, 2, max_seq, 256]        (K stored post-norm, post-RoPE)
  dn_states               : [n_dn, 16, 128(value), 128(key)]
  conv_bufs               : [n_dn, 6144, 4]  last 4 pre-activation conv inputs, oldest first
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

HIDDEN = 1024
INTER = 3584
VOCAB = 248320
NUM_LAYERS = 24
RMS_EPS = 1e-6

FA_Q_HEADS = 8
FA_KV_HEADS = 2
FA_HEAD_DIM = 256
FA_Q_SIZE = FA_Q_HEADS * FA_HEAD_DIM          # 2048
FA_QPROJ = 2 * FA_Q_SIZE                      # 4096  per head [q(256) | gate(256)]
FA_KV_SIZE = FA_KV_HEADS * FA_HEAD_DIM        # 512
FA_ROT = 64
ROPE_THETA = 1.0e7

DN_HEADS = 16
DN_KEY = 128
DN_VAL = 128
DN_QK = DN_HEADS * DN_KEY                     # 2048
DN_V = DN_HEADS * DN_VAL                      # 2048
DN_CONV_CH = 2 * DN_QK + DN_V                 # 6144
DN_CONV_K = 4


def layer_types(num_layers: int = NUM_LAYERS) -> List[int]:
    """0 = Gated DeltaNet, 1 = full attention; pattern [DN,DN,DN,FA] (kernel.cu:65-67)."""
    return [1 if (i % 4) == 3 else 0 for i in range(num_layers)]


# ----------------------------------------------------------------------------------------
# Seeded random-init weights
# ----------------------------------------------------------------------------------------

def weight_names(num_layers: int = NUM_LAYERS) -> List[str]:
    """Tensor names in `transformers` state-dict order for this architecture."""
    names = ["model.embed_tokens.weight"]
    for i, lt in enumerate(layer_types(num_layers)):
        p = f"model.layers.{i}."
        if lt == 0:
            names += [p + "linear_attn." + s for s in (
                "dt_bias", "A_log", "conv1d.weight", "norm.weight", "out_proj.weight",
                "in_proj_qkv.weight", "in_proj_z.weight", "in_proj_b.weight", "in_proj_a.weight")]
        else:
            names += [p + "self_attn." + s for s in (
                "q_proj.weight", "k_proj.weight", "v_proj.weight", "o_proj.weight",
                "q_norm.weight", "k_norm.weight")]
        names += [p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight", p + "mlp.down_proj.weight",
                  p + "input_layernorm.weight", p + "post_attention_layernorm.weight"]
    names.append("model.norm.weight")
    return names


def _shape_of(name: str, vocab: int):
    tail = name.split(".", 3)[-1] if name.startswith("model.layers.") else name
    table = {
        "model.embed_tokens.weight": (vocab, HIDDEN),
        "model.norm.weight": (HIDDEN,),
        "linear_attn.dt_bias": (DN_HEADS,),
        "linear_attn.A_log": (DN_HEADS,),
        "linear_attn.conv1d.weight": (DN_CONV_CH, 1, DN_CONV_K),
        "linear_attn.norm.weight": (DN_VAL,),
        "linear_attn.out_proj.weight": (HIDDEN, DN_V),
        "linear_attn.in_proj_qkv.weight": (DN_CONV_CH, HIDDEN),
        "linear_attn.in_proj_z.weight": (DN_V, HIDDEN),
        "linear_attn.in_proj_b.weight": (DN_HEADS, HIDDEN),
        "linear_attn.in_proj_a.weight": (DN_HEADS, HIDDEN),
        "self_attn.q_proj.weight": (FA_QPROJ, HIDDEN),
        "self_attn.k_proj.weight": (FA_KV_SIZE, HIDDEN),
        "self_attn.v_proj.weight": (FA_KV_SIZE, HIDDEN),
        "self_attn.o_proj.weight": (HIDDEN, FA_Q_SIZE),
        "self_attn.q_norm.weight": (FA_HEAD_DIM,),
        "self_attn.k_norm.weight": (FA_HEAD_DIM,),
        "mlp.gate_proj.weight": (INTER, HIDDEN),
        "mlp.up_proj.weight": (INTER, HIDDEN),
        "mlp.down_proj.weight": (HIDDEN, INTER),
        "input_layernorm.weight": (HIDDEN,),
        "post_attention_layernorm.weight": (HIDDEN,),
    }
    return table[tail]


def init_weights(seed: int = 0, num_layers: int = NUM_LAYERS, vocab: int = VOCAB,
                 norm_init: str = "literal") -> Dict[str, torch.Tensor]:
    """Seeded random-init weights as bf16 tensors (CPU), drawn in state-dict order from one
    torch.Generator(seed): every >=2-D weight ~N(0, 0.02); A_log ~U(ln 1, ln 16);
    dt_bias ~U(-4, -1); norm weight tensors are constants:
      norm_init="literal": every norm tensor = 1.0 (so the (1+w) norms scale by 2)
      norm_init="unit"   : (1+w) norm tensors = 0.0 and the gated norm = 1.0 (effective weight 1)
    The CPU generator stream is identical on every machine with the same torch build, so the
    GPU side and the oracle side regenerate identical values from the seed.
    """
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    out: Dict[str, torch.Tensor] = {}
    for name in weight_names(num_layers):
        shape = _shape_of(name, vocab)
        if name.endswith("A_log"):
            t = torch.empty(shape).uniform_(math.log(1.0), math.log(16.0), generator=g)
        elif name.endswith("dt_bias"):
            t = torch.empty(shape).uniform_(-4.0, -1.0, generator=g)
        elif len(shape) >= 2:
            t = torch.empty(shape).normal_(0.0, 0.02, generator=g)
        else:  # norm weights
            if norm_init == "literal" or name.endswith("linear_attn.norm.weight"):
                t = torch.ones(shape)
            elif norm_init == "unit":
                t = torch.zeros(shape)
            else:
                raise ValueError(norm_init)
        out[name] = t.to(torch.bfloat16)
    return out


# ----------------------------------------------------------------------------------------
# Session state
# ----------------------------------------------------------------------------------------

@dataclass
class State:
    num_layers: int
    max_seq: int
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    dn_states: torch.Tensor
    conv_bufs: torch.Tensor
    position: int = 0
    seen: Optional[torch.Tensor] = None

    @staticmethod
    def new(num_layers: int = NUM_LAYERS, max_seq: int = 2048, vocab: int = VOCAB) -> "State":
        lt = layer_types(num_layers)
        n_fa, n_dn = sum(lt), len(lt) - sum(lt)
        return State(
            num_layers=num_layers, max_seq=max_seq,
            k_cache=torch.zeros(n_fa, FA_KV_HEADS, max_seq, FA_HEAD_DIM),
            v_cache=torch.zeros(n_fa, FA_KV_HEADS, max_seq, FA_HEAD_DIM),
            dn_states=torch.zeros(n_dn, DN_HEADS, DN_VAL, DN_KEY),
            conv_bufs=torch.zeros(n_dn, DN_CONV_CH, DN_CONV_K),
            position=0, seen=torch.zeros(vocab))

    def clone(self) -> "State":
        return State(self.num_layers, self.max_seq, self.k_cache.clone(), self.v_cache.clone(),
                     self.dn_states.clone(), self.conv_bufs.clone(), self.position,
                     None if self.seen is None else self.seen.clone())


@dataclass
class Trace:
    """What one forward over T tokens leaves behind for comparison."""
    hidden: List[torch.Tensor] = field(default_factory=list)   # per layer, [T, 1024] (layer output)
    final_normed: Optional[torch.Tensor] = None                # [1024] last row, f32
    logits: Optional[torch.Tensor] = None                      # [vocab] last row, f32
    token: int = -1


def _bf(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def _rms(x: torch.Tensor, w1p: torch.Tensor) -> torch.Tensor:
    """x * rsqrt(mean x^2 + eps) * w1p   with w1p already (1+w).  kernel.cu:220-228"""
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + RMS_EPS) * w1p


class Oracle:
    """fp32 restatement of the reference decode arithmetic, usable for T>=1 consecutive tokens."""

    def __init__(self, weights: Dict[str, torch.Tensor], rounding: str = "decode", ref_q_rope_in_place: bool = False,
                 block_sparse: Optional[dict] = None, act_quant=None):
        """ref_q_rope_in_place reproduces what the reference decode kernel actually computes for the
        query's rotary dims 32..63: it rotates q in place (kernel.cu:487-497), so by the time a lane
        reaches dim i+32 its partner dim i already holds the rotated value, which is then normalised
        a second time.  At position 0 the rotation is the identity and nothing changes; from position
        1 on the result differs from the reference's own PyTorch baseline (transformers' rotate_half).
        This library follows the baseline; the flag exists only so that the tests can pin this
        restatement against the reference kernels themselves, run on a GPU."""
        assert rounding in ("decode", "none")
        self.rounding = rounding
        # act_quant: optional callable [T, K] f32 -> [T, K] f32 applied to the input of every quantised projection
        # (qkv / z / out, q / k / v / o, gate / up / down; not beta / alpha, not the LM head): models a path that
        # multiplies quantised activations, e.g. NVFP4 x NVFP4 on the block-scaled tensor cores
        self.act_quant = act_quant
        # tail_lookahead = n > 0: a prompt processed from position 0 also leaves tail_running_max [n, T], the maximum
        # over attention layers and query heads of the causal softmax of the last n queries over every key
        # (what the reference's prompt compressor scores with, dflash/src/qwen3_0p6b_graph.cpp:430-496)
        self.tail_lookahead = 0
        self.tail_running_max = None
        self.ref_q_rope_in_place = ref_q_rope_in_place
        # block_sparse = {"top_frac": .., "window": .., "sink": ..} (ranking rule) or {"alpha": .., "window": .., "sink": ..,
        # "last_n_full": ..} (the reference's threshold rule): prompts processed from position 0 attend only to the
        # key blocks oracle/block_sparse.py selects (bf16-rounded q and k feed the selection)
        self.block_sparse = block_sparse
        self.w = {k: v.to(torch.float32) for k, v in weights.items()}
        self.num_layers = 1 + max(int(k.split(".")[2]) for k in weights if k.startswith("model.layers."))
        self.types = layer_types(self.num_layers)
        self.vocab = self.w["model.embed_tokens.weight"].shape[0]
        self.lm_head = self.w.get("lm_head.weight", self.w["model.embed_tokens.weight"])
        # inv_freq_p = theta^(-2p/64), p = 0..31  (kernel.cu:468-469)
        self.inv_freq = 1.0 / (ROPE_THETA ** (torch.arange(0, FA_ROT, 2, dtype=torch.float32) / FA_ROT))

    def _r(self, x):
        return _bf(x) if self.rounding == "decode" else x

    def _q(self, x):
        return self.act_quant(x) if self.act_quant is not None else x

    # -- token mixers ----------------------------------------------------------------

    def _deltanet(self, p: str, x: torch.Tensor, st: State, idx: int) -> torch.Tensor:
        w = self.w
        T = x.shape[0]
        xq = self._q(x)
        c = xq @ w[p + "in_proj_qkv.weight"].T                   # [T, 6144]  kernel.cu:621
        z = xq @ w[p + "in_proj_z.weight"].T                     # [T, 2048]
        b = x @ w[p + "in_proj_b.weight"].T                      # [T, 16]
        a = x @ w[p + "in_proj_a.weight"].T                      # [T, 16]
        # causal depthwise conv over [state(4) | new(T)], SiLU        kernel.cu:633-648
        seq = torch.cat([st.conv_bufs[idx], c.T], dim=1)          # [6144, 4+T]
        cw = w[p + "conv1d.weight"].reshape(DN_CONV_CH, DN_CONV_K)
        win = seq.unfold(1, DN_CONV_K, 1)[:, 1:, :]                # [6144, T, 4] windows ending at each new t
        u = F.silu((win * cw[:, None, :]).sum(-1)).T               # [T, 6144]
        st.conv_bufs[idx] = seq[:, -DN_CONV_K:].clone()
        q = u[:, :DN_QK].reshape(T, DN_HEADS, DN_KEY)
        k = u[:, DN_QK:2 * DN_QK].reshape(T, DN_HEADS, DN_KEY)
        v = u[:, 2 * DN_QK:].reshape(T, DN_HEADS, DN_VAL)
        q = q * torch.rsqrt(q.pow(2).sum(-1, keepdim=True) + 1e-6) / math.sqrt(DN_KEY)   # kernel.cu:662-667
        k = k * torch.rsqrt(k.pow(2).sum(-1, keepdim=True) + 1e-6)                        # kernel.cu:668-672
        beta = torch.sigmoid(b)                                                           # kernel.cu:652
        gamma = torch.exp(-torch.exp(w[p + "A_log"]) * F.softplus(a + w[p + "dt_bias"], threshold=20.0))
        S = st.dn_states[idx]                                     # [16, value, key]
        o = torch.empty(T, DN_HEADS, DN_VAL)
        for t in range(T):                                        # kernel.cu:694-713
            kt, qt, vt = k[t], q[t], v[t]                         # [16,128]
            gt, bt = gamma[t][:, None], beta[t][:, None]
            pj = torch.einsum("hji,hi->hj", S, kt)
            delta = (vt - gt * pj) * bt
            S = gt[:, :, None] * S + delta[:, :, None] * kt[:, None, :]
            o[t] = torch.einsum("hji,hi->hj", S, qt)
        st.dn_states[idx] = S
        # gated RMSNorm with plain weight, then SiLU(z)              kernel.cu:715-728
        y = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + RMS_EPS) * w[p + "norm.weight"]
        y = y * F.silu(z.reshape(T, DN_HEADS, DN_VAL))
        return y.reshape(T, DN_V)

    def _attention(self, p: str, x: torch.Tensor, st: State, idx: int, pos0: int) -> torch.Tensor:
        w = self.w
        T = x.shape[0]
        x = self._q(x)
        qg = (x @ w[p + "q_proj.weight"].T).reshape(T, FA_Q_HEADS, 2 * FA_HEAD_DIM)     # kernel.cu:450
        q, gate = qg[..., :FA_HEAD_DIM], qg[..., FA_HEAD_DIM:]
        k = (x @ w[p + "k_proj.weight"].T).reshape(T, FA_KV_HEADS, FA_HEAD_DIM)
        v = (x @ w[p + "v_proj.weight"].T).reshape(T, FA_KV_HEADS, FA_HEAD_DIM)
        q_scale = torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + RMS_EPS)
        q = _rms(q, 1.0 + w[p + "q_norm.weight"])                                       # kernel.cu:487-491
        k = _rms(k, 1.0 + w[p + "k_norm.weight"])                                       # kernel.cu:462-466
        pos = torch.arange(pos0, pos0 + T, dtype=torch.float32)
        ang = pos[:, None] * self.inv_freq[None, :]                                     # [T, 32]
        cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]

        def rope(t):                                                                    # kernel.cu:467-475
            lo, hi, rest = t[..., :32], t[..., 32:64], t[..., 64:]
            return torch.cat([lo * cos - hi * sin, hi * cos + lo * sin, rest], dim=-1)

        if self.ref_q_rope_in_place:
            w1p = 1.0 + w[p + "q_norm.weight"]
            lo, hi, rest = q[..., :32], q[..., 32:64], q[..., 64:]
            lo_out = lo * cos - hi * sin
            partner = lo_out * q_scale * w1p[:32]          # the already rotated value, normalised again
            q = torch.cat([lo_out, partner * sin + hi * cos, rest], dim=-1)
        else:
            q = rope(q)
        k = rope(k)
        st.k_cache[idx, :, pos0:pos0 + T] = self._r(k).transpose(0, 1)                   # kernel.cu:474-476
        st.v_cache[idx, :, pos0:pos0 + T] = self._r(v).transpose(0, 1)
        L = pos0 + T
        K = st.k_cache[idx, :, :L].repeat_interleave(FA_Q_HEADS // FA_KV_HEADS, dim=0)   # [8, L, 256]
        V = st.v_cache[idx, :, :L].repeat_interleave(FA_Q_HEADS // FA_KV_HEADS, dim=0)
        if self.tail_lookahead and pos0 == 0 and T > self.tail_lookahead:
            n = self.tail_lookahead
            s = torch.einsum("thd,hld->htl", _bf(q[T - n:]), K[:, :T]) / math.sqrt(FA_HEAD_DIM)       # [8, n, T]
            causal = torch.arange(T)[None, :] <= torch.arange(T - n, T)[:, None]
            pm = torch.softmax(s.masked_fill(~causal[None], float("-inf")), dim=-1).amax(dim=0)     # [n, T]
            self.tail_running_max = pm if self.tail_running_max is None else torch.maximum(self.tail_running_max, pm)
        keep = None
        if self.block_sparse is not None and pos0 == 0 and T > 1:
            from . import block_sparse as BS
            pick = BS.select_threshold_for_heads if "alpha" in self.block_sparse else BS.select_for_heads
            keep = pick(_bf(q).permute(1, 0, 2).numpy(), st.k_cache[idx, :, :L].numpy(), **self.block_sparse)
        # query rows in slabs of 1024 (every row's softmax is independent; the slabs only bound the size of the
        # score matrix for prompts of many thousand tokens)
        o = torch.empty(T, FA_Q_HEADS, FA_HEAD_DIM)
        for r0 in range(0, T, 1024):
            r1 = min(T, r0 + 1024)
            Lr = pos0 + r1                                                               # keys a row of this slab can see
            s = torch.einsum("thd,hld->htl", q[r0:r1], K[:, :Lr]) / math.sqrt(FA_HEAD_DIM)   # kernel.cu:509,528-529
            causal = torch.arange(Lr)[None, :] <= (pos0 + torch.arange(r0, r1))[:, None]
            s = s.masked_fill(~causal[None], float("-inf"))
            if keep is not None:
                blk_q = torch.arange(r0, r1) // BS.BLOCK
                blk_k = torch.arange(Lr) // BS.BLOCK
                for hh in range(FA_Q_HEADS):
                    kept = torch.from_numpy(keep[hh])[blk_q][:, blk_k]                   # [rows, Lr] bool
                    s[hh] = s[hh].masked_fill(~kept, float("-inf"))
            o[r0:r1] = torch.einsum("htl,hld->thd", torch.softmax(s, dim=-1), V[:, :Lr])
        o = o * torch.sigmoid(gate)                                                      # kernel.cu:551-556
        return o.reshape(T, FA_Q_SIZE)

    # -- full forward ----------------------------------------------------------------

    def forward(self, tokens, st: State, want_logits: bool = True,
                repetition_penalty: float = 1.0) -> Trace:
        """Advance `st` over `tokens` (consecutive positions from st.position).  Returns the
        per-layer outputs for all T rows and, for the last row, the final-normed vector, the
        logits and the greedy token."""
        w = self.w
        tokens = torch.as_tensor(tokens, dtype=torch.long).reshape(-1)
        T = tokens.numel()
        pos0 = st.position
        assert pos0 + T <= st.max_seq
        if repetition_penalty > 1.0 and st.seen is not None:
            st.seen[tokens] = 1.0                                                        # kernel.cu:862-866
        h = w["model.embed_tokens.weight"][tokens]                                       # kernel.cu:874
        tr = Trace()
        dn_i = fa_i = 0
        for li, lt in enumerate(self.types):
            p = f"model.layers.{li}."
            x = self._r(_rms(h, 1.0 + w[p + "input_layernorm.weight"]))                  # kernel.cu:228
            if lt == 0:
                a = self._deltanet(p + "linear_attn.", x, st, dn_i)
                h = self._r(self._q(a) @ w[p + "linear_attn.out_proj.weight"].T + h)     # kernel.cu:739
                dn_i += 1
            else:
                a = self._attention(p + "self_attn.", x, st, fa_i, pos0)
                h = self._r(self._q(a) @ w[p + "self_attn.o_proj.weight"].T + h)         # kernel.cu:568
                fa_i += 1
            x = self._r(_rms(h, 1.0 + w[p + "post_attention_layernorm.weight"]))         # kernel.cu:574
            xq = self._q(x)
            m = F.silu(xq @ w[p + "mlp.gate_proj.weight"].T) * (xq @ w[p + "mlp.up_proj.weight"].T)
            h = self._r(self._q(m) @ w[p + "mlp.down_proj.weight"].T + h)                # kernel.cu:585
            tr.hidden.append(h.clone())
        st.position = pos0 + T
        n = _rms(h[-1], 1.0 + w["model.norm.weight"])                                    # kernel.cu:916-919 (f32)
        tr.final_normed = n
        if want_logits:
            logits = self.lm_head @ n                                                    # kernel.cu:783-792
            if repetition_penalty > 1.0 and st.seen is not None:                         # kernel.cu:793-795
                adj = torch.where(logits > 0, logits / repetition_penalty, logits * repetition_penalty)
                logits = torch.where(st.seen > 0, adj, logits)
            tr.logits = logits
            tr.token = int(torch.argmax(logits))     # lowest index wins on exact ties
        return tr

    def generate(self, prompt, n_new: int, st: State) -> List[int]:
        """Prefill the prompt, then n_new greedy tokens (the first comes from the prefill)."""
        tr = self.forward(prompt, st)
        out = [tr.token]
        for _ in range(n_new - 1):
            tr = self.forward([out[-1]], st)
            out.append(tr.token)
        return out
