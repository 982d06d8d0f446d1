"""Checkpoint ingestion (safetensors directory -> pointer-table order) and the packed-weights file."""
import json
import os

import pytest
import torch

from luce_megakernel_b200 import checkpoint as C, model as M, weights as W

NL, V = 4, 512


def _write_checkpoint(tmp_path, sd, prefix="model.", shards=2, extra=None):
    """A Hugging Face style directory: sharded safetensors + index, keys under `prefix`."""
    from safetensors.torch import save_file
    items = [((prefix + k[len("model."):]) if k.startswith("model.") else k, v.contiguous()) for k, v in sd.items()]
    items += list((extra or {}).items())
    weight_map = {}
    for s in range(shards):
        part = dict(items[s::shards])
        name = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        save_file(part, os.path.join(tmp_path, name))
        weight_map.update({k: name for k in part})
    json.dump({"metadata": {}, "weight_map": weight_map}, open(os.path.join(tmp_path, "model.safetensors.index.json"), "w"))


@pytest.mark.parametrize("prefix", ["model.", "model.language_model."])
def test_checkpoint_dir_round_trip(tmp_path, prefix):
    sd = W.random_state_dict(3, NL, V)
    extra = {"model.visual.patch_embed.weight": torch.zeros(4, 4), "mtp.fc.weight": torch.zeros(2, 2)} if prefix != "model." else None
    _write_checkpoint(str(tmp_path), sd, prefix=prefix, extra=extra)
    got = C.load_checkpoint_dir(str(tmp_path))
    assert set(got) == set(sd)
    for k in sd:
        assert torch.equal(got[k], sd[k]), k
    assert C.check_architecture(got) == NL
    w = C.weights_from_checkpoint(str(tmp_path), device="cpu")
    ref = M.weights_from_state_dict(sd, device="cpu")
    assert [ld["type"] for ld in w["layer_data"]] == [0, 0, 0, 1]
    for a, b in zip(w["layer_data"], ref["layer_data"]):
        assert all(torch.equal(x, y) for x, y in zip(a["ptrs"], b["ptrs"]))
    assert w["lm_head_weight"] is w["embed_weight"]


def test_checkpoint_of_another_architecture_is_refused(tmp_path):
    sd = W.random_state_dict(3, NL, V)
    sd["model.layers.0.mlp.gate_proj.weight"] = torch.zeros(100, 1024, dtype=torch.bfloat16)
    _write_checkpoint(str(tmp_path), sd)
    with pytest.raises(ValueError, match="gate_proj"):
        C.weights_from_checkpoint(str(tmp_path), device="cpu")
    with pytest.raises(FileNotFoundError):
        C.load_checkpoint_dir(str(tmp_path / "nowhere"))


def test_packed_file_round_trip_bf16(tmp_path):
    w = M.weights_from_state_dict(W.random_state_dict(5, NL, V), device="cpu")
    path = C.save_packed(w, str(tmp_path / "w.safetensors"))
    r = C.load_packed(path, device="cpu")
    assert r["lm_head_weight"] is r["embed_weight"] and torch.equal(r["embed_weight"], w["embed_weight"])
    for a, b in zip(w["layer_data"], r["layer_data"]):
        assert a["type"] == b["type"] and len(a["ptrs"]) == len(b["ptrs"])
        assert all(torch.equal(x, y) for x, y in zip(a["ptrs"], b["ptrs"]))
    with pytest.raises(ValueError):
        from safetensors.torch import save_file
        save_file({"x": torch.zeros(1)}, str(tmp_path / "other.safetensors"))
        C.load_packed(str(tmp_path / "other.safetensors"), device="cpu")


@pytest.mark.gpu
def test_packed_file_carries_both_nvfp4_packings(tmp_path):
    """Quantise once, save, load in place of quantising: identical tensors, identical decode tokens."""
    from luce_megakernel_b200 import model_nvfp4 as MQ
    NLg, Vg = 4, 1024
    w = M.weights_from_state_dict(W.random_state_dict(6, NLg, Vg, "unit"))
    MQ.attach_nvfp4_weights(w)
    MQ.attach_nvfp4_ts_weights(w)
    torch.cuda.synchronize()
    path = C.save_packed(w, str(tmp_path / "packed.safetensors"))
    r = C.load_packed(path)
    assert set(r) == set(w)
    for key in ("nvfp4", "nvfp4_ts"):
        for a, b in zip(w[key]["layer_data"], r[key]["layer_data"]):
            assert len(a["ptrs"]) == len(b["ptrs"]) and all(torch.equal(x, y) for x, y in zip(a["ptrs"], b["ptrs"]))
    assert torch.equal(w["nvfp4_ts"]["lm"]["scales"], r["nvfp4_ts"]["lm"]["scales"])
    size = os.path.getsize(path)
    bf16_bytes = sum(x.numel() * 2 for ld in w["layer_data"] for x in ld["ptrs"]) + w["embed_weight"].numel() * 2
    assert size < 1.75 * bf16_bytes                 # both 4-bit packings add ~0.56 of the bf16 bytes; shared tensors stored once
    toks = [3, 77, 500, 9, 1001]
    a, b = MQ.DecoderTS(w, max_seq_len=32), MQ.DecoderTS(r, max_seq_len=32)
    assert [a.step(t) for t in toks] == [b.step(t) for t in toks]
    a1, b1 = MQ.Decoder(w, max_seq_len=32), MQ.Decoder(r, max_seq_len=32)
    assert [a1.step(t) for t in toks] == [b1.step(t) for t in toks]
