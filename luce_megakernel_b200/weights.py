"""Seeded random-init weights of the Qwen3.5-0.8B architecture (no checkpoint is needed).

Tensors are drawn on the CPU, in `transformers` state-dict order, from one
torch.Generator(seed): every >=2-D weight ~N(0, 0.02); A_log ~U(ln 1, ln 16);
dt_bias ~U(-4, -1); norm weight tensors constant ("literal": all 1.0; "unit": the (1+w)
norms 0.0 and the gated DeltaNet norm 1.0).  Values are rounded to bf16.
"""
import math

import torch

from .model import (DN_CONV_CHANNELS, DN_CONV_KERNEL, DN_NUM_HEADS, DN_V_SIZE, DN_VALUE_DIM, FA_HEAD_DIM,
                    FA_KV_SIZE, FA_Q_SIZE, FA_QPROJ_SIZE, HIDDEN_SIZE, INTERMEDIATE_SIZE, NUM_LAYERS, VOCAB_SIZE,
                    layer_types)


def _names_and_shapes(num_layers, vocab):
    out = [("model.embed_tokens.weight", (vocab, HIDDEN_SIZE))]
    for i, lt in enumerate(layer_types(num_layers)):
        p = f"model.layers.{i}."
        if lt == 0:
            q = p + "linear_attn."
            out += [(q + "dt_bias", (DN_NUM_HEADS,)), (q + "A_log", (DN_NUM_HEADS,)),
                    (q + "conv1d.weight", (DN_CONV_CHANNELS, 1, DN_CONV_KERNEL)), (q + "norm.weight", (DN_VALUE_DIM,)),
                    (q + "out_proj.weight", (HIDDEN_SIZE, DN_V_SIZE)), (q + "in_proj_qkv.weight", (DN_CONV_CHANNELS, HIDDEN_SIZE)),
                    (q + "in_proj_z.weight", (DN_V_SIZE, HIDDEN_SIZE)), (q + "in_proj_b.weight", (DN_NUM_HEADS, HIDDEN_SIZE)),
                    (q + "in_proj_a.weight", (DN_NUM_HEADS, HIDDEN_SIZE))]
        else:
            q = p + "self_attn."
            out += [(q + "q_proj.weight", (FA_QPROJ_SIZE, HIDDEN_SIZE)), (q + "k_proj.weight", (FA_KV_SIZE, HIDDEN_SIZE)),
                    (q + "v_proj.weight", (FA_KV_SIZE, HIDDEN_SIZE)), (q + "o_proj.weight", (HIDDEN_SIZE, FA_Q_SIZE)),
                    (q + "q_norm.weight", (FA_HEAD_DIM,)), (q + "k_norm.weight", (FA_HEAD_DIM,))]
        out += [(p + "mlp.gate_proj.weight", (INTERMEDIATE_SIZE, HIDDEN_SIZE)), (p + "mlp.up_proj.weight", (INTERMEDIATE_SIZE, HIDDEN_SIZE)),
                (p + "mlp.down_proj.weight", (HIDDEN_SIZE, INTERMEDIATE_SIZE)), (p + "input_layernorm.weight", (HIDDEN_SIZE,)),
                (p + "post_attention_layernorm.weight", (HIDDEN_SIZE,))]
    out.append(("model.norm.weight", (HIDDEN_SIZE,)))
    return out


def random_state_dict(seed=0, num_layers=NUM_LAYERS, vocab=VOCAB_SIZE, norm_init="literal", device="cpu"):
    """`device="cpu"` gives the machine-independent stream the parity tests rely on; a CUDA
    device draws the same distributions from the device generator (much faster, different
    values), which is what the benchmarks use."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    sd = {}
    for name, shape in _names_and_shapes(num_layers, vocab):
        if name.endswith("A_log"):
            t = torch.empty(shape, device=device).uniform_(math.log(1.0), math.log(16.0), generator=g)
        elif name.endswith("dt_bias"):
            t = torch.empty(shape, device=device).uniform_(-4.0, -1.0, generator=g)
        elif len(shape) >= 2:
            t = torch.empty(shape, device=device).normal_(0.0, 0.02, generator=g)
        elif norm_init == "literal" or name.endswith("linear_attn.norm.weight"):
            t = torch.ones(shape, device=device)
        elif norm_init == "unit":
            t = torch.zeros(shape, device=device)
        else:
            raise ValueError(norm_init)
        sd[name] = t.to(torch.bfloat16)
    return sd
