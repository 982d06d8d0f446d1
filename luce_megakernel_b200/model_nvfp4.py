"""NVFP4 decode driver: quantises the bf16 weights with the library's quantisers, packs the
24 x 208-byte pointer table and drives launch_decode_nvfp4 / launch_decode_many_nvfp4.

Host-side mirror of the reference's NVFP4 driver (reference: megakernel/model_nvfp4.py:126-160,
249-337, 456-473, 704-769): layer matrices in the 32-group / fp16-scale format, the LM head as its
own packed copy in the 16-block / E4M3 format (even when it is tied to the embedding), norms, conv,
beta / alpha projections and the embedding gather table in bf16.
"""
import ctypes
import struct

import torch

from .model import (DN_CONV_CHANNELS, DN_CONV_KERNEL, DN_KEY_DIM, DN_NUM_HEADS, DN_VALUE_DIM, FA_HEAD_DIM,
                    FA_NUM_KV_HEADS, HIDDEN_SIZE, _ptr)

NVFP4_GROUP_SIZE = 32
NVFP4_LM_GROUP_SIZE = 16


def _quantize_matrix_nvfp4(lib, w, group_size=NVFP4_GROUP_SIZE):
    rows, cols = w.shape
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(rows, cols // group_size, dtype=torch.float16, device=w.device)
    rc = lib.launch_quantize_nvfp4_out(_ptr(w), rows, cols, group_size, _ptr(packed), _ptr(scales),
                                       ctypes.c_void_p(torch.cuda.current_stream(w.device).cuda_stream))
    if rc != 0:
        raise RuntimeError("quantize_nvfp4_out failed")
    return {"packed": packed, "scales": scales}


def _quantize_matrix_nvfp4_lm(lib, w):
    rows, cols = w.shape
    if rows % 128 or cols % 64:
        raise ValueError("LM head needs rows % 128 == 0 and cols % 64 == 0")
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8, device=w.device)
    scales = torch.zeros((rows // 128) * (cols // 64) * 512, dtype=torch.uint8, device=w.device)
    rc = lib.launch_quantize_nvfp4_lm_out(_ptr(w), rows, cols, _ptr(packed), _ptr(scales),
                                          ctypes.c_void_p(torch.cuda.current_stream(w.device).cuda_stream))
    if rc != 0:
        raise RuntimeError("quantize_nvfp4_lm_out failed")
    return {"packed": packed, "scales": scales}


def attach_nvfp4_weights(weights, group_size=NVFP4_GROUP_SIZE):
    """Adds weights["nvfp4"] (reference: megakernel/model_nvfp4.py:249-337)."""
    from . import lib as _lib
    lib = _lib()
    if "nvfp4" in weights and weights["nvfp4"]["group_size"] == group_size:
        return weights
    layers = []
    for ld in weights["layer_data"]:
        p = ld["ptrs"]
        q = lambda i: _quantize_matrix_nvfp4(lib, p[i], group_size)
        if ld["type"] == 1:
            qq, kk, vv, oo, gg, uu, dd = q(1), q(2), q(3), q(6), q(8), q(9), q(10)
            ptrs = [p[0], qq["packed"], qq["scales"], kk["packed"], kk["scales"], vv["packed"], vv["scales"], p[4], p[5],
                    oo["packed"], oo["scales"], p[7], gg["packed"], gg["scales"], uu["packed"], uu["scales"],
                    dd["packed"], dd["scales"]]
        else:
            qkv, zz, oo, gg, uu, dd = q(1), q(2), q(9), q(11), q(12), q(13)
            ptrs = [p[0], qkv["packed"], qkv["scales"], zz["packed"], zz["scales"], p[3], p[4], p[5], p[6], p[7], p[8],
                    oo["packed"], oo["scales"], p[10], gg["packed"], gg["scales"], uu["packed"], uu["scales"],
                    dd["packed"], dd["scales"]]
        layers.append({"type": ld["type"], "ptrs": ptrs})
    lm = _quantize_matrix_nvfp4_lm(lib, weights["lm_head_weight"])
    weights["nvfp4"] = {"group_size": group_size, "lm_group_size": NVFP4_LM_GROUP_SIZE, "layer_data": layers,
                        "lm_head_weight_packed": lm["packed"], "lm_head_scales": lm["scales"]}
    return weights


def _pack_layer_weights_nvfp4(layer_data, group_size):
    """Device blob of 208-byte entries {int type; int group_size; int pad[2]; void* ptrs[24]}
    (reference: megakernel/model_nvfp4.py:456-473)."""
    entry = struct.Struct("<4i24Q")
    assert entry.size == 208
    blob = bytearray()
    for ld in layer_data:
        ptrs = [t.data_ptr() for t in ld["ptrs"]]
        blob += entry.pack(ld["type"], group_size, 0, 0, *(ptrs + [0] * (24 - len(ptrs))))
    return torch.frombuffer(blob, dtype=torch.uint8).cuda()


class Decoder:
    """Stateful greedy decoder over the NVFP4 weights (reference: megakernel/model_nvfp4.py:499-769)."""

    def __init__(self, weights, max_seq_len=2048, group_size=NVFP4_GROUP_SIZE):
        from . import lib as _lib
        self._lib = _lib()
        self._weights = attach_nvfp4_weights(weights, group_size)
        nv = self._weights["nvfp4"]
        self.group_size = group_size
        self.max_seq_len = int(max_seq_len)
        self._embed_weight = weights["embed_weight"]
        self._final_norm_weight = weights["final_norm_weight"]
        self._lm_packed, self._lm_scales = nv["lm_head_weight_packed"], nv["lm_head_scales"]
        self.num_layers = len(nv["layer_data"])
        self.vocab = int(self._embed_weight.shape[0])
        self._layer_weights_packed = _pack_layer_weights_nvfp4(nv["layer_data"], group_size)
        dev = self._embed_weight.device
        types = [ld["type"] for ld in nv["layer_data"]]
        n_fa, n_dn = sum(types), len(types) - sum(types)
        self._fa_k_cache = torch.zeros(max(n_fa, 1), FA_NUM_KV_HEADS, self.max_seq_len, FA_HEAD_DIM, dtype=torch.bfloat16, device=dev)
        self._fa_v_cache = torch.zeros_like(self._fa_k_cache)
        self._dn_states = torch.zeros(max(n_dn, 1), DN_NUM_HEADS, DN_KEY_DIM, DN_VALUE_DIM, dtype=torch.float32, device=dev)
        self._conv_bufs = torch.zeros(max(n_dn, 1), DN_CONV_CHANNELS, DN_CONV_KERNEL, dtype=torch.float32, device=dev)
        self._hidden = torch.empty(HIDDEN_SIZE, dtype=torch.bfloat16, device=dev)
        self._normalized = torch.empty(HIDDEN_SIZE, dtype=torch.float32, device=dev)
        self._out_token = torch.empty(1, dtype=torch.int32, device=dev)
        self._token_buffer = torch.empty(1, dtype=torch.int32, device=dev)
        self._position = 0

    def _common_args(self):
        z = ctypes.c_void_p(0)
        return [_ptr(self._embed_weight), _ptr(self._layer_weights_packed), _ptr(self._final_norm_weight),
                _ptr(self._lm_packed), _ptr(self._lm_scales), z, z, z, z, _ptr(self._fa_k_cache), _ptr(self._fa_v_cache),
                _ptr(self._dn_states), _ptr(self._conv_bufs), _ptr(self._hidden), z, z, z, z, z, z, z, z, z,
                _ptr(self._normalized), z, z, z, z, z]

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(f"luce_megakernel_b200 error {rc}: {self._lib.mk_last_error_string().decode()}")

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self._embed_weight.device).cuda_stream)

    def step_async(self, token_id: int):
        if self._position >= self.max_seq_len:
            raise ValueError("position exceeds max_seq_len")
        self._check(self._lib.mk_set_model_dims(self.num_layers, self.vocab))
        self._out_token.fill_(int(token_id))       # the token travels through device memory, as in the reference op
        self._check(self._lib.launch_decode_nvfp4(
            _ptr(self._out_token), _ptr(self._out_token), *self._common_args(), ctypes.c_int(self._position),
            ctypes.c_int(self.max_seq_len), ctypes.c_int(self.group_size), self._stream()))
        self._position += 1

    def step(self, token_id: int) -> int:
        self.step_async(token_id)
        return int(self._out_token.item())

    def step_many(self, token_id: int, steps: int) -> torch.Tensor:
        if self._position + steps > self.max_seq_len:
            raise ValueError("position + steps exceeds max_seq_len")
        self._check(self._lib.mk_set_model_dims(self.num_layers, self.vocab))
        out = torch.empty(steps, dtype=torch.int32, device=self._out_token.device)
        self._token_buffer.fill_(int(token_id))
        self._check(self._lib.launch_decode_many_nvfp4(
            _ptr(self._token_buffer), _ptr(out), ctypes.c_int(steps), *self._common_args(),
            ctypes.c_int(self._position), ctypes.c_int(self.max_seq_len), ctypes.c_int(self.group_size), self._stream()))
        self._position += steps
        return out

    def prefill_tokens(self, token_ids, mode: str = "raw") -> int:
        """Run prompt prefill from position 0 and return the first generated token id
        (reference: megakernel/model_nvfp4.py:771-825).  mode "raw": NVFP4 layer weights
        (launch_prefill_megakernel_nvfp4); mode "bf16": bf16 layer weights with the NVFP4 LM head
        (launch_prefill_bf16_nvfp4_lm's arithmetic)."""
        ids = torch.as_tensor(token_ids, dtype=torch.int32).to(self._embed_weight.device).contiguous()
        S = int(ids.numel())
        if S < 1 or S > self.max_seq_len:
            raise ValueError("prompt length must be in [1, max_seq_len]")
        self.reset()
        self._check(self._lib.mk_set_model_dims(self.num_layers, self.vocab))
        z = ctypes.c_void_p(0)
        if mode == "raw":
            rc = self._lib.mk_prefill_nvfp4(
                _ptr(ids), ctypes.c_int(S), _ptr(self._out_token), _ptr(self._embed_weight), _ptr(self._layer_weights_packed),
                _ptr(self._final_norm_weight), _ptr(self._lm_packed), _ptr(self._lm_scales), _ptr(self._fa_k_cache),
                _ptr(self._fa_v_cache), _ptr(self._dn_states), _ptr(self._conv_bufs), z, _ptr(self._hidden),
                ctypes.c_int(self.max_seq_len), ctypes.c_int(self.group_size), ctypes.c_int(self.num_layers),
                ctypes.c_int(self.vocab), self._stream())
        elif mode == "bf16":
            if not hasattr(self, "_bf16_table"):
                from .model import _pack_layer_weights
                self._bf16_table = _pack_layer_weights(self._weights["layer_data"])
            rc = self._lib.mk_prefill_bf16_nvfp4_lm(
                _ptr(ids), ctypes.c_int(S), _ptr(self._out_token), _ptr(self._embed_weight), _ptr(self._bf16_table),
                _ptr(self._final_norm_weight), _ptr(self._lm_packed), _ptr(self._lm_scales), _ptr(self._fa_k_cache),
                _ptr(self._fa_v_cache), _ptr(self._dn_states), _ptr(self._conv_bufs), z, _ptr(self._hidden),
                ctypes.c_int(self.max_seq_len), ctypes.c_int(self.num_layers), ctypes.c_int(self.vocab), self._stream())
        else:
            raise ValueError("mode must be 'raw' or 'bf16'")
        if rc != 0:
            self._lib.mk_prefill_error.restype = ctypes.c_char_p
            raise RuntimeError(f"prefill failed ({rc}): {self._lib.mk_prefill_error().decode()}")
        self._position = S
        return int(self._out_token.item())

    def reset(self):
        self._position = 0
        for t in (self._fa_k_cache, self._fa_v_cache, self._dn_states, self._conv_bufs):
            t.zero_()


# ---------------------------------------------------------------------------------------------------------------
# NVFP4 with a per-tensor scale: e2m1 values in 16-element blocks, E4M3 block scales, one fp32 scale per matrix, for
# every linear layer and the LM head.  The reference's NVFP4 decode has no such format (megakernel/model_nvfp4.py:
# 249-337 packs 32-groups with fp16 scales for the layers); this is the additional format next to it.
# ---------------------------------------------------------------------------------------------------------------

def _quantize_matrix_nvfp4_ts(lib, w):
    """bf16 [rows, cols] -> packed codes, block scales as plain rows [rows, cols/16], device float[1] tensor scale."""
    rows, cols = w.shape
    if rows % 128 or cols % 64:
        raise ValueError("the tensor-scale NVFP4 format needs rows % 128 == 0 and cols % 64 == 0")
    stream = ctypes.c_void_p(torch.cuda.current_stream(w.device).cuda_stream)
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8, device=w.device)
    tiled = torch.zeros((rows // 128) * (cols // 64) * 512, dtype=torch.uint8, device=w.device)
    ts = torch.zeros(4, dtype=torch.float32, device=w.device)        # 16 bytes: keeps later allocations aligned
    if lib.mk_quantize_nvfp4_tensor_scale(_ptr(w), rows, cols, _ptr(packed), _ptr(tiled), _ptr(ts), stream) != 0:
        raise RuntimeError("mk_quantize_nvfp4_tensor_scale failed")
    srows = torch.empty(rows, cols // 16, dtype=torch.uint8, device=w.device)
    if lib.mk_nvfp4_scales_to_rows(_ptr(tiled), rows, cols, _ptr(srows), stream) != 0:
        raise RuntimeError("mk_nvfp4_scales_to_rows failed")
    return {"packed": packed, "scales_tiled": tiled, "scales": srows, "tensor_scale": ts}


def attach_nvfp4_ts_weights(weights):
    """Adds weights["nvfp4_ts"]: per layer the slot list of the 224-byte table (a quantised matrix takes three
    slots: packed, row-major block scales, tensor scale), plus the LM head's own packed copy."""
    from . import lib as _lib
    lib = _lib()
    if "nvfp4_ts" in weights:
        return weights
    layers = []
    for ld in weights["layer_data"]:
        p = ld["ptrs"]

        tiled = {}

        def q(i):
            m = _quantize_matrix_nvfp4_ts(lib, p[i])
            tiled[id(m["scales"])] = m["scales_tiled"]
            return [m["packed"], m["scales"], m["tensor_scale"]]
        if ld["type"] == 1:
            ptrs = [p[0]] + q(1) + q(2) + q(3) + [p[4], p[5]] + q(6) + [p[7]] + q(8) + q(9) + q(10)
        else:
            ptrs = [p[0]] + q(1) + q(2) + [p[3], p[4], p[5], p[6], p[7], p[8]] + q(9) + [p[10]] + q(11) + q(12) + q(13)
        # the same slot list with every scale slot pointing at the quantiser's 128 x 4 tiles (block-scaled GEMM operand)
        ptrs_tiled = [tiled.get(id(t), t) for t in ptrs]
        layers.append({"type": ld["type"], "ptrs": ptrs, "ptrs_tiled": ptrs_tiled})
    lm = _quantize_matrix_nvfp4_ts(lib, weights["lm_head_weight"])
    weights["nvfp4_ts"] = {"layer_data": layers, "lm": lm}
    return weights


def _pack_layer_weights_nvfp4_ts(layer_data):
    """Device blob of 224-byte entries {int type; int pad[3]; void* ptrs[26]}."""
    entry = struct.Struct("<4i26Q")
    assert entry.size == 224
    blob = bytearray()
    for ld in layer_data:
        ptrs = [t.data_ptr() for t in ld["ptrs"]]
        assert len(ptrs) == (25 if ld["type"] == 1 else 26)
        blob += entry.pack(ld["type"], 0, 0, 0, *(ptrs + [0] * (26 - len(ptrs))))
    return torch.frombuffer(blob, dtype=torch.uint8).cuda()


class DecoderTS:
    """Stateful greedy decoder over the tensor-scale NVFP4 weights (mk_decode_nvfp4_ts); same session interface as
    Decoder above.  The prompt is fed token by token or prefilled in bf16 by a model.Decoder sharing the state."""

    def __init__(self, weights, max_seq_len=2048):
        from . import lib as _lib
        self._lib = _lib()
        self._weights = attach_nvfp4_ts_weights(weights)
        nv = self._weights["nvfp4_ts"]
        self.max_seq_len = int(max_seq_len)
        self._embed_weight = weights["embed_weight"]
        self._final_norm_weight = weights["final_norm_weight"]
        self._lm = nv["lm"]
        self.num_layers = len(nv["layer_data"])
        self.vocab = int(self._embed_weight.shape[0])
        self._layer_weights_packed = _pack_layer_weights_nvfp4_ts(nv["layer_data"])
        dev = self._embed_weight.device
        types = [ld["type"] for ld in nv["layer_data"]]
        n_fa, n_dn = sum(types), len(types) - sum(types)
        self._fa_k_cache = torch.zeros(max(n_fa, 1), FA_NUM_KV_HEADS, self.max_seq_len, FA_HEAD_DIM, dtype=torch.bfloat16, device=dev)
        self._fa_v_cache = torch.zeros_like(self._fa_k_cache)
        self._dn_states = torch.zeros(max(n_dn, 1), DN_NUM_HEADS, DN_KEY_DIM, DN_VALUE_DIM, dtype=torch.float32, device=dev)
        self._conv_bufs = torch.zeros(max(n_dn, 1), DN_CONV_CHANNELS, DN_CONV_KERNEL, dtype=torch.float32, device=dev)
        self._hidden = torch.empty(HIDDEN_SIZE, dtype=torch.bfloat16, device=dev)
        self._normalized = torch.empty(HIDDEN_SIZE, dtype=torch.float32, device=dev)
        self._token_buffer = torch.empty(1, dtype=torch.int32, device=dev)
        self._position = 0

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(f"luce_megakernel_b200 error {rc}: {self._lib.mk_last_error_string().decode()}")

    def step_many(self, token_id: int, steps: int) -> torch.Tensor:
        """`steps` greedy steps in one launch; returns the int32 device tensor of tokens without synchronising."""
        if steps < 1 or self._position + steps > self.max_seq_len:
            raise ValueError("steps must be positive and position + steps within max_seq_len")
        self._check(self._lib.mk_set_model_dims(self.num_layers, self.vocab))
        out = torch.empty(steps, dtype=torch.int32, device=self._token_buffer.device)
        self._token_buffer.fill_(int(token_id))
        self._check(self._lib.mk_decode_nvfp4_ts(
            _ptr(self._token_buffer), _ptr(out), ctypes.c_int(steps), _ptr(self._embed_weight),
            _ptr(self._layer_weights_packed), _ptr(self._final_norm_weight), _ptr(self._lm["packed"]),
            _ptr(self._lm["scales"]), _ptr(self._lm["tensor_scale"]), _ptr(self._fa_k_cache), _ptr(self._fa_v_cache),
            _ptr(self._dn_states), _ptr(self._conv_bufs), _ptr(self._hidden), _ptr(self._normalized),
            ctypes.c_int(self._position), ctypes.c_int(self.max_seq_len),
            ctypes.c_void_p(torch.cuda.current_stream(self._embed_weight.device).cuda_stream)))
        self._position += steps
        return out

    def step(self, token_id: int) -> int:
        tok = int(self.step_many(token_id, 1).item())
        if tok < 0:     # the launch gave up on a bounded wait and drained
            self._lib.mk_device_status_detail.restype = ctypes.c_uint
            raise RuntimeError("decode launch gave up on a device-side wait: status word 0x%08x"
                               % self._lib.mk_device_status_detail())
        return tok

    def prefill(self, token_ids) -> int:
        """Prompt from position 0 with NVFP4 weights and NVFP4 activations on the block-scaled tensor cores
        (mk_prefill_nvfp4_mma); returns the first generated token."""
        ids = torch.as_tensor(token_ids, dtype=torch.int32).to(self._embed_weight.device).contiguous()
        S = int(ids.numel())
        if S < 1 or S > self.max_seq_len:
            raise ValueError("prompt length must be in [1, max_seq_len]")
        if not hasattr(self, "_table_tiled"):
            nv = self._weights["nvfp4_ts"]
            self._table_tiled = _pack_layer_weights_nvfp4_ts([{"type": ld["type"], "ptrs": ld["ptrs_tiled"]} for ld in nv["layer_data"]])
            self._final_normed_bf16 = torch.empty(HIDDEN_SIZE, dtype=torch.bfloat16, device=self._embed_weight.device)
        self._check(self._lib.mk_set_model_dims(self.num_layers, self.vocab))
        out = torch.empty(1, dtype=torch.int32, device=self._embed_weight.device)
        self._check(self._lib.mk_prefill_nvfp4_mma(
            _ptr(ids), ctypes.c_int(S), _ptr(out), _ptr(self._embed_weight), _ptr(self._table_tiled),
            _ptr(self._final_norm_weight), _ptr(self._lm["packed"]), _ptr(self._lm["scales_tiled"]), _ptr(self._fa_k_cache),
            _ptr(self._fa_v_cache), _ptr(self._dn_states), _ptr(self._conv_bufs), _ptr(self._final_normed_bf16), _ptr(self._hidden),
            ctypes.c_int(self.max_seq_len), ctypes.c_int(self.num_layers), ctypes.c_int(self.vocab),
            ctypes.c_void_p(torch.cuda.current_stream(self._embed_weight.device).cuda_stream)))
        self._position = S
        return int(out.item())

    def adopt_state(self, other):
        """Take over the session state (caches, DeltaNet state, conv window, position) of another decoder over the
        same model, e.g. a bf16 model.Decoder that has just prefilled the prompt."""
        self._fa_k_cache, self._fa_v_cache = other._fa_k_cache, other._fa_v_cache
        self._dn_states, self._conv_bufs = other._dn_states, other._conv_bufs
        self.max_seq_len, self._position = other.max_seq_len, other._position

    def reset(self):
        self._position = 0
        for t in (self._fa_k_cache, self._fa_v_cache, self._dn_states, self._conv_bufs):
            t.zero_()


# ---------------------------------------------------------------------------------------------------------------
# The same tensor-scale NVFP4 values as per-CTA chunk images for the tcgen05 decode kernel (mk_decode_nvfp4_mma).
# ---------------------------------------------------------------------------------------------------------------

def attach_nvfp4_mma_weights(weights):
    """Adds weights["nvfp4_mma"]: the slot lists of weights["nvfp4_ts"] with the first slot of every phase's matrix
    group replaced by that phase's chunk images, and the LM-head images."""
    from . import nvfp4_images as I
    if "nvfp4_mma" in weights:
        return weights
    attach_nvfp4_ts_weights(weights)
    ts = weights["nvfp4_ts"]
    layers = []
    for ld in ts["layer_data"]:
        p = list(ld["ptrs"])
        if ld["type"] == 1:       # attention: q(1) k(4) v(7) o(12) gate(16) up(19) down(22)
            groups, o, g, u, d = (1, 4, 7), 12, 16, 19, 22
            in_phase = "fa_in"
        else:                     # DeltaNet: qkv(1) z(4) out(13) gate(17) up(20) down(23)
            groups, o, g, u, d = (1, 4), 13, 17, 20, 23
            in_phase = "dn_in"
        img_in = I.build_phase_images(in_phase, torch.cat([p[i] for i in groups]), torch.cat([p[i + 1] for i in groups]))
        img_o = I.build_phase_images("out", p[o], p[o + 1])
        img_g = I.build_gateup_images(p[g], p[g + 1], p[u], p[u + 1])
        img_d = I.build_phase_images("down", p[d], p[d + 1])
        q = list(p)
        q[groups[0]], q[o], q[g], q[d] = img_in, img_o, img_g, img_d
        layers.append({"type": ld["type"], "ptrs": q})
    lm_img, chunks = I.build_lm_images(ts["lm"]["packed"], ts["lm"]["scales"])
    weights["nvfp4_mma"] = {"layer_data": layers, "lm_images": lm_img, "lm_chunks": chunks,
                            "lm_tensor_scale": ts["lm"]["tensor_scale"]}
    return weights


class DecoderMMA(DecoderTS):
    """DecoderTS on the block-scaled tensor-core kernel (mk_decode_nvfp4_mma).  act_terms: NVFP4 residual terms the
    activation vector of every projection is expanded into (1..8)."""

    def __init__(self, weights, max_seq_len=2048, act_terms=4):
        super().__init__(weights, max_seq_len)
        attach_nvfp4_mma_weights(self._weights)
        mm = self._weights["nvfp4_mma"]
        self._mma = mm
        self._layer_weights_packed = _pack_layer_weights_nvfp4_ts(mm["layer_data"])
        self.act_terms = int(act_terms)

    def step_many(self, token_id: int, steps: int) -> torch.Tensor:
        if steps < 1 or self._position + steps > self.max_seq_len:
            raise ValueError("steps must be positive and position + steps within max_seq_len")
        self._check(self._lib.mk_set_model_dims(self.num_layers, self.vocab))
        out = torch.empty(steps, dtype=torch.int32, device=self._token_buffer.device)
        self._token_buffer.fill_(int(token_id))
        self._check(self._lib.mk_decode_nvfp4_mma(
            _ptr(self._token_buffer), _ptr(out), ctypes.c_int(steps), _ptr(self._embed_weight),
            _ptr(self._layer_weights_packed), _ptr(self._final_norm_weight), _ptr(self._mma["lm_images"]),
            ctypes.c_int(self._mma["lm_chunks"]), _ptr(self._mma["lm_tensor_scale"]), _ptr(self._fa_k_cache),
            _ptr(self._fa_v_cache), _ptr(self._dn_states), _ptr(self._conv_bufs), _ptr(self._hidden), _ptr(self._normalized),
            ctypes.c_int(self._position), ctypes.c_int(self.max_seq_len), ctypes.c_int(self.act_terms),
            ctypes.c_void_p(torch.cuda.current_stream(self._embed_weight.device).cuda_stream)))
        self._position += steps
        return out
