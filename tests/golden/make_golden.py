"""Generate tests/golden/hf_qwen35_small.npz from the reference's PyTorch path.

The reference's only PyTorch implementation of this model is the third-party
`transformers` class it loads with AutoModelForCausalLM (reference:
megakernel/final_bench.py:117-149).  This script builds that class
(transformers 5.5.0, Qwen3_5ForCausalLM, its pure-torch gated-delta-rule fallback) in
fp32 on the CPU for a reduced depth / vocabulary of the same architecture, loads the
seeded weights of oracle.qwen35_oracle.init_weights into it, and records what a
prefill of a seeded prompt plus greedy decode steps produce.  The fixture is small and
travels with the repo; the test-suite compares the oracle against it.

Run from the repo root (needs `transformers`; no GPU, no network):
    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import qwen35_oracle as O  # noqa: E402

NUM_LAYERS = 8
VOCAB = 2048
PROMPT_LEN = 24
N_DECODE = 8
SEED = 0


def build_hf(weights):
    from transformers import AutoModelForCausalLM, Qwen3_5TextConfig
    cfg = Qwen3_5TextConfig(
        vocab_size=VOCAB, hidden_size=O.HIDDEN, intermediate_size=O.INTER, num_hidden_layers=NUM_LAYERS,
        num_attention_heads=O.FA_Q_HEADS, num_key_value_heads=O.FA_KV_HEADS, head_dim=O.FA_HEAD_DIM,
        linear_num_key_heads=O.DN_HEADS, linear_num_value_heads=O.DN_HEADS,
        linear_key_head_dim=O.DN_KEY, linear_value_head_dim=O.DN_VAL, linear_conv_kernel_dim=O.DN_CONV_K,
        tie_word_embeddings=True, max_position_embeddings=4096, rms_norm_eps=O.RMS_EPS,
        rope_parameters={"rope_theta": O.ROPE_THETA, "partial_rotary_factor": 0.25, "rope_type": "default"},
    )
    assert cfg.layer_types == ["linear_attention"] * 3 + ["full_attention"] + ["linear_attention"] * 3 + ["full_attention"]
    model = AutoModelForCausalLM.from_config(cfg, dtype=torch.float32)
    sd = {k: v.to(torch.float32) for k, v in weights.items()}
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, unexpected = model.load_state_dict(sd, strict=True)
    model.eval()
    return model


def main():
    out = {}
    for norm_init in ("literal", "unit"):
        weights = O.init_weights(SEED, NUM_LAYERS, VOCAB, norm_init=norm_init)
        model = build_hf(weights)
        g = torch.Generator().manual_seed(SEED)
        prompt = torch.randint(0, VOCAB, (PROMPT_LEN,), generator=g)
        layer_out = []
        hooks = [l.register_forward_hook(lambda m, i, o: layer_out.append((o[0] if isinstance(o, tuple) else o).detach()))
                 for l in model.model.layers]
        hid, logits, tokens = [], [], []
        with torch.no_grad():
            r = model(input_ids=prompt[None], use_cache=True)
            cache = r.past_key_values
            hid.append(torch.stack([h[0, -1] for h in layer_out]))
            logits.append(r.logits[0, -1])
            prefill_all_rows_last_layer = layer_out[-1][0].clone()
            tokens.append(int(r.logits[0, -1].argmax()))
            for _ in range(N_DECODE):
                layer_out.clear()
                r = model(input_ids=torch.tensor([[tokens[-1]]]), past_key_values=cache, use_cache=True)
                cache = r.past_key_values
                hid.append(torch.stack([h[0, -1] for h in layer_out]))
                logits.append(r.logits[0, -1])
                tokens.append(int(r.logits[0, -1].argmax()))
        for h in hooks:
            h.remove()
        # final session state in the op layout (dn_states transposed to [value][key])
        L = PROMPT_LEN + N_DECODE
        rec = cache.layers[0].recurrent_states[0].transpose(-1, -2).contiguous()   # [16, value, key]
        conv = cache.layers[0].conv_states[0].contiguous()                          # [6144, 4]
        keys = cache.layers[3].keys[0, :, :L].contiguous()                          # [2, L, 256]
        vals = cache.layers[3].values[0, :, :L].contiguous()
        pre = norm_init + "_"
        out[pre + "prompt"] = prompt.numpy().astype(np.int32)
        out[pre + "tokens"] = np.asarray(tokens, dtype=np.int32)
        out[pre + "hidden_last"] = torch.stack(hid).numpy()                         # [1+N_DECODE, layers, 1024]
        out[pre + "logits"] = torch.stack(logits).numpy()                           # [1+N_DECODE, vocab]
        out[pre + "prefill_rows_last_layer"] = prefill_all_rows_last_layer.numpy()  # [PROMPT_LEN, 1024]
        out[pre + "dn_state_l0_h0"] = rec[0].numpy()                                # [128,128]
        out[pre + "dn_state_l0_sum"] = rec.sum(dim=(-1, -2)).numpy()                # [16]
        out[pre + "conv_l0_first64"] = conv[:64].numpy()
        out[pre + "k_l3_h0"] = keys[0].numpy()                                      # [L,256]
        out[pre + "v_l3_h1_last"] = vals[1, -1].numpy()
    out["meta"] = np.asarray([NUM_LAYERS, VOCAB, PROMPT_LEN, N_DECODE, SEED], dtype=np.int32)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "hf_qwen35_small.npz")
    np.savez_compressed(path, **out)
    import transformers
    print("wrote", path, os.path.getsize(path), "bytes; transformers", transformers.__version__, "torch", torch.__version__)


if __name__ == "__main__":
    main()
