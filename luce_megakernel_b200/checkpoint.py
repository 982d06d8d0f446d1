"""Checkpoint ingestion and the packed-weights file.

Two on-disk sides of the decode / prefill path:

* `load_checkpoint_dir(path)` reads a Hugging Face checkpoint directory of the Qwen3.5-0.8B architecture
  (`*.safetensors`, optionally sharded with `model.safetensors.index.json`) straight into the state dict the
  weight packer consumes -- no model object is built and nothing is downloaded.  The reference goes through
  `AutoModelForCausalLM.from_pretrained` for the same tensors (megakernel/model.py:66-157); the tensor names it reads
  from the state dict are the ones kept here.  Key prefixes of wrapped checkpoints (`model.language_model.`,
  `language_model.model.`) are normalised to `model.`; tensors the path does not use (vision tower, multi-token
  prediction heads) are skipped.

* `save_packed(weights, path)` / `load_packed(path)`: one safetensors file holding every device-ready tensor of a
  `weights` dict -- the bf16 tensors and, when attached, both NVFP4 packings (the reference's 32-group / fp16-scale
  layer format with its 16-block LM head, megakernel/model_nvfp4.py:249-337, and the 16-block / E4M3 / fp32
  tensor-scale format) -- so that a serving process maps the file instead of re-quantising 0.75 B parameters at
  start-up.  Layout: tensor names `bf16.embed`, `bf16.final_norm`, `bf16.lm_head` (absent when tied),
  `bf16.layers.<i>.<slot>`, `nvfp4.layers.<i>.<slot>`, `nvfp4.lm.packed|scales`, `nvfp4_ts.layers.<i>.<slot>`,
  `nvfp4_ts.lm.packed|scales|tensor_scale`; slots are the positions of the kernels' pointer tables.  The header
  metadata carries `format = luce_megakernel_b200.packed`, `version`, the layer types and the NVFP4 group size.
"""
import glob
import json
import os

import torch

PACKED_FORMAT = "luce_megakernel_b200.packed"
PACKED_VERSION = 1

_PREFIXES = ("model.language_model.", "language_model.model.", "model.text_model.")
_SKIP = ("visual.", "vision_tower.", "mtp.", "model.visual.", "model.mtp.")


def _normalise_key(k):
    for s in _SKIP:
        if k.startswith(s):
            return None
    for p in _PREFIXES:
        if k.startswith(p):
            return "model." + k[len(p):]
    if k.startswith("language_model.lm_head."):
        return k[len("language_model."):]
    return k


def load_checkpoint_dir(path, device="cpu"):
    """State dict (transformers names, e.g. `model.layers.3.self_attn.q_proj.weight`) of the checkpoint in `path`."""
    from safetensors import safe_open
    if not os.path.isdir(path):
        raise FileNotFoundError(f"{path} is not a directory")
    index = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(index):
        files = sorted(set(json.load(open(index))["weight_map"].values()))
        files = [os.path.join(path, f) for f in files]
    else:
        files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no .safetensors file in {path}")
    sd = {}
    for f in files:
        with safe_open(f, framework="pt", device=str(device)) as h:
            for k in h.keys():
                nk = _normalise_key(k)
                if nk is not None and (nk.startswith("model.") or nk.startswith("lm_head.")):
                    sd[nk] = h.get_tensor(k)
    if "model.embed_tokens.weight" not in sd:
        raise KeyError("model.embed_tokens.weight not found: not a checkpoint of this architecture")
    return sd


def check_architecture(sd):
    """Raises ValueError unless the state dict has the dimensions the kernels are built for."""
    from . import model as M
    n = 1 + max(int(k.split(".")[2]) for k in sd if k.startswith("model.layers."))
    if n > M.NUM_LAYERS:
        raise ValueError(f"{n} layers; the kernels are built for at most {M.NUM_LAYERS}")
    want = {"model.embed_tokens.weight": (None, M.HIDDEN_SIZE), "model.norm.weight": (M.HIDDEN_SIZE,)}
    for i, lt in enumerate(M.layer_types(n)):
        p = f"model.layers.{i}."
        want[p + "mlp.gate_proj.weight"] = (M.INTERMEDIATE_SIZE, M.HIDDEN_SIZE)
        want[p + "mlp.down_proj.weight"] = (M.HIDDEN_SIZE, M.INTERMEDIATE_SIZE)
        if lt == 1:
            want[p + "self_attn.q_proj.weight"] = (M.FA_QPROJ_SIZE, M.HIDDEN_SIZE)
            want[p + "self_attn.k_proj.weight"] = (M.FA_KV_SIZE, M.HIDDEN_SIZE)
        else:
            want[p + "linear_attn.in_proj_qkv.weight"] = (M.DN_CONV_CHANNELS, M.HIDDEN_SIZE)
            want[p + "linear_attn.conv1d.weight"] = (M.DN_CONV_CHANNELS, 1, M.DN_CONV_KERNEL)
    for k, shape in want.items():
        if k not in sd:
            raise ValueError(f"missing tensor {k}")
        got = tuple(sd[k].shape)
        if len(got) != len(shape) or any(s is not None and s != g for s, g in zip(shape, got)):
            raise ValueError(f"{k} has shape {got}, expected {shape}")
    return n


def weights_from_checkpoint(path, device="cuda"):
    """Checkpoint directory -> the `weights` dict of model.Decoder (bf16 on `device`)."""
    from .model import weights_from_state_dict
    sd = load_checkpoint_dir(path)
    n = check_architecture(sd)
    return weights_from_state_dict(sd, device=device, num_layers=n)


# ---- packed file -----------------------------------------------------------------------------------------------

def save_packed(weights, path):
    """Writes every tensor of `weights` (and of its attached NVFP4 packings) to one safetensors file."""
    from safetensors.torch import save_file
    t = {"bf16.embed": weights["embed_weight"], "bf16.final_norm": weights["final_norm_weight"]}
    tied = weights["lm_head_weight"] is weights["embed_weight"] or \
        weights["lm_head_weight"].data_ptr() == weights["embed_weight"].data_ptr()
    if not tied:
        t["bf16.lm_head"] = weights["lm_head_weight"]
    for i, ld in enumerate(weights["layer_data"]):
        for s, x in enumerate(ld["ptrs"]):
            t[f"bf16.layers.{i}.{s}"] = x
    meta = {"format": PACKED_FORMAT, "version": str(PACKED_VERSION), "tied_lm_head": "1" if tied else "0",
            "layer_types": ",".join(str(ld["type"]) for ld in weights["layer_data"]), "packings": "bf16"}
    if "nvfp4" in weights:
        nv = weights["nvfp4"]
        for i, ld in enumerate(nv["layer_data"]):
            for s, x in enumerate(ld["ptrs"]):
                t[f"nvfp4.layers.{i}.{s}"] = x
        t["nvfp4.lm.packed"], t["nvfp4.lm.scales"] = nv["lm_head_weight_packed"], nv["lm_head_scales"]
        meta["nvfp4_group_size"] = str(nv["group_size"])
        meta["packings"] += ",nvfp4"
    if "nvfp4_ts" in weights:
        nv = weights["nvfp4_ts"]
        for i, ld in enumerate(nv["layer_data"]):
            for s, x in enumerate(ld["ptrs"]):
                t[f"nvfp4_ts.layers.{i}.{s}"] = x
        for k in ("packed", "scales", "tensor_scale"):
            t[f"nvfp4_ts.lm.{k}"] = nv["lm"][k]
        meta["packings"] += ",nvfp4_ts"
    # the NVFP4 tables repeat the bf16 norm / conv tensors of a layer: store each storage once
    seen, out, alias = {}, {}, {}
    for k, x in t.items():
        key = (x.data_ptr(), tuple(x.shape), x.dtype)
        if key in seen:
            alias[k] = seen[key]
        else:
            seen[key] = k
            out[k] = x.detach().contiguous().cpu()
    meta["aliases"] = json.dumps(alias)
    save_file(out, path, metadata=meta)
    return path


def load_packed(path, device="cuda"):
    """The `weights` dict saved by save_packed, tensors on `device`; nothing is re-quantised."""
    from safetensors import safe_open
    with safe_open(path, framework="pt", device=str(device)) as h:
        meta = h.metadata() or {}
        if meta.get("format") != PACKED_FORMAT:
            raise ValueError(f"{path} is not a {PACKED_FORMAT} file")
        if int(meta.get("version", "0")) != PACKED_VERSION:
            raise ValueError(f"{path}: version {meta.get('version')} (this library reads version {PACKED_VERSION})")
        t = {k: h.get_tensor(k) for k in h.keys()}
    for k, src in json.loads(meta.get("aliases", "{}")).items():
        t[k] = t[src]
    types = [int(x) for x in meta["layer_types"].split(",")]

    def layers(prefix):
        out = []
        for i, lt in enumerate(types):
            slots = sorted(int(k.rsplit(".", 1)[1]) for k in t if k.startswith(f"{prefix}.layers.{i}."))
            out.append({"type": lt, "ptrs": [t[f"{prefix}.layers.{i}.{s}"] for s in slots]})
        return out

    embed = t["bf16.embed"]
    w = {"embed_weight": embed, "final_norm_weight": t["bf16.final_norm"],
         "lm_head_weight": embed if meta.get("tied_lm_head") == "1" else t["bf16.lm_head"], "layer_data": layers("bf16")}
    packings = meta.get("packings", "bf16").split(",")
    if "nvfp4" in packings:
        w["nvfp4"] = {"group_size": int(meta["nvfp4_group_size"]), "lm_group_size": 16, "layer_data": layers("nvfp4"),
                      "lm_head_weight_packed": t["nvfp4.lm.packed"], "lm_head_scales": t["nvfp4.lm.scales"]}
    if "nvfp4_ts" in packings:
        w["nvfp4_ts"] = {"layer_data": layers("nvfp4_ts"),
                         "lm": {k: t[f"nvfp4_ts.lm.{k}"] for k in ("packed", "scales", "tensor_scale")}}
    return w
