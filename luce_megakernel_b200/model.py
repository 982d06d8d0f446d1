"""Weight packing and the stateful decoder over the sm_100a ops.

Host-side mirror of the reference's Python driver (reference: megakernel/model.py): the same
constants, the same 24 x 128-byte layer pointer table, the same state / scratch tensors and
the same `Decoder.step / reset / generate / alloc_prefill_scratch` interface, so code written
against the reference driver runs against this one.  The arithmetic lives in the native
library; nothing here computes on the CPU.
"""
import ctypes
import struct

import torch

NUM_LAYERS = 24
HIDDEN_SIZE = 1024
INTERMEDIATE_SIZE = 3584
VOCAB_SIZE = 248320
MAX_SEQ_LEN = 2048

FA_NUM_Q_HEADS = 8
FA_NUM_KV_HEADS = 2
FA_HEAD_DIM = 256
FA_Q_SIZE = FA_NUM_Q_HEADS * FA_HEAD_DIM
FA_QPROJ_SIZE = FA_Q_SIZE * 2
FA_KV_SIZE = FA_NUM_KV_HEADS * FA_HEAD_DIM

DN_NUM_HEADS = 16
DN_KEY_DIM = 128
DN_VALUE_DIM = 128
DN_QK_SIZE = DN_NUM_HEADS * DN_KEY_DIM
DN_V_SIZE = DN_NUM_HEADS * DN_VALUE_DIM
DN_CONV_CHANNELS = DN_QK_SIZE * 2 + DN_V_SIZE
DN_CONV_KERNEL = 4


def layer_types(num_layers=NUM_LAYERS):
    """0 = Gated DeltaNet, 1 = full attention, pattern [DN, DN, DN, FA]."""
    return [1 if i % 4 == 3 else 0 for i in range(num_layers)]


LAYER_TYPE = layer_types()

_FA_KEYS = ("input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
            "self_attn.v_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
            "self_attn.o_proj.weight", "post_attention_layernorm.weight",
            "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")
_DN_KEYS = ("input_layernorm.weight", "linear_attn.in_proj_qkv.weight", "linear_attn.in_proj_z.weight",
            "linear_attn.in_proj_b.weight", "linear_attn.in_proj_a.weight", "linear_attn.conv1d.weight",
            "linear_attn.A_log", "linear_attn.dt_bias", "linear_attn.norm.weight",
            "linear_attn.out_proj.weight", "post_attention_layernorm.weight",
            "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")


def weights_from_state_dict(state, device="cuda", num_layers=None):
    """Orders a `transformers`-style state dict into the per-layer pointer lists the kernels
    read: 11 tensors for an attention layer, 14 for a DeltaNet layer
    (reference: megakernel/model.py:90-148).  Tensors become contiguous bf16 on `device`."""
    if num_layers is None:
        num_layers = 1 + max(int(k.split(".")[2]) for k in state if k.startswith("model.layers."))

    def w(key):
        return state[key].to(device=device, dtype=torch.bfloat16).contiguous()

    layer_data = []
    for i, lt in enumerate(layer_types(num_layers)):
        keys = _FA_KEYS if lt == 1 else _DN_KEYS
        layer_data.append({"type": lt, "ptrs": [w(f"model.layers.{i}.{k}") for k in keys]})
    embed = w("model.embed_tokens.weight")
    lm_head = w("lm_head.weight") if "lm_head.weight" in state else embed
    return {"embed_weight": embed, "final_norm_weight": w("model.norm.weight"),
            "lm_head_weight": lm_head, "layer_data": layer_data}


def load_weights(model_name="Qwen/Qwen3.5-0.8B", verbose=True, seed=None, num_layers=NUM_LAYERS,
                 vocab=VOCAB_SIZE, norm_init="literal", device_init=False):
    """Returns (weights, tokenizer).  With `seed` set, seeded random-init weights of the
    architecture are produced (tokenizer None; drawn on the CPU unless device_init, see
    weights.random_state_dict); otherwise `model_name` is a local checkpoint directory (its safetensors
    shards are read directly, see checkpoint.py) or a hub name loaded through transformers, like the
    reference does (megakernel/model.py:66-157)."""
    if seed is not None:
        from .weights import random_state_dict
        dev = torch.device("cuda", torch.cuda.current_device()) if device_init else "cpu"
        sd = random_state_dict(seed, num_layers, vocab, norm_init, device=dev)
        return weights_from_state_dict(sd, device=torch.device("cuda", torch.cuda.current_device()),
                                       num_layers=num_layers), None
    import os
    if os.path.isdir(model_name):
        # a local checkpoint directory: read the safetensors shards directly (no model object, no network)
        from .checkpoint import weights_from_checkpoint
        if verbose:
            print(f"Reading checkpoint {model_name} (bf16)...")
        weights = weights_from_checkpoint(model_name, device=torch.device("cuda", torch.cuda.current_device()))
        tokenizer = None
        if os.path.exists(os.path.join(model_name, "tokenizer_config.json")):
            from transformers import AutoTokenizer
            tokenizer = AutoTokenizer.from_pretrained(model_name)
        return weights, tokenizer
    from transformers import AutoModelForCausalLM, AutoTokenizer
    if verbose:
        print(f"Loading {model_name} (bf16)...")
    model = AutoModelForCausalLM.from_pretrained(model_name, dtype=torch.bfloat16, device_map="cuda")
    tokenizer = AutoTokenizer.from_pretrained(model_name)
    weights = weights_from_state_dict(model.state_dict())
    del model
    torch.cuda.empty_cache()
    return weights, tokenizer


def _pack_layer_weights(layer_data):
    """Device blob of len(layer_data) entries {int type; int pad[3]; void* ptrs[14]} (128 B each),
    the layout of MkLayerWeights (reference: megakernel/model.py:160-177)."""
    entry = struct.Struct("<4i14Q")
    assert entry.size == 128
    blob = bytearray()
    for ld in layer_data:
        ptrs = [t.data_ptr() for t in ld["ptrs"]]
        blob += entry.pack(ld["type"], 0, 0, 0, *(ptrs + [0] * (14 - len(ptrs))))
    from . import lib
    lib().mk_prefill_forget_tables()      # a new table may reuse the address of a freed one
    return torch.frombuffer(blob, dtype=torch.uint8).cuda()


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


class Decoder:
    """Stateful greedy decoder (reference: megakernel/model.py:180-318).

    `api="ops"` calls torch.ops.qwen35_megakernel_bf16_C.* exactly like the reference
    driver; `api="cabi"` calls the C ABI of libluce_megakernel_b200.so through ctypes."""

    def __init__(self, weights=None, tokenizer=None, model_name="Qwen/Qwen3.5-0.8B", verbose=True,
                 max_seq_len=MAX_SEQ_LEN, repetition_penalty=1.0, decode_blocks=None, api="ops"):
        if max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if repetition_penalty < 1.0:
            raise ValueError("repetition_penalty must be >= 1.0")
        if decode_blocks is not None and decode_blocks < 0:
            raise ValueError("decode_blocks must be non-negative")
        if api not in ("ops", "cabi"):
            raise ValueError("api must be 'ops' or 'cabi'")
        from . import lib, load_ops
        self._lib = lib()
        self._ops = load_ops() if api == "ops" else None
        self.api = api
        self._step_args = None          # ctypes argument tuple of step(), built on first use
        if weights is None:
            weights, tokenizer = load_weights(model_name, verbose=verbose)
        self.tokenizer = tokenizer
        self._position = 0
        self.max_seq_len = int(max_seq_len)
        self.repetition_penalty = float(repetition_penalty)
        self._weights = weights
        self._embed_weight = weights["embed_weight"]
        self._final_norm_weight = weights["final_norm_weight"]
        self._lm_head_weight = weights["lm_head_weight"]
        layer_data = weights["layer_data"]
        self.num_layers = len(layer_data)
        self.vocab = int(self._embed_weight.shape[0])
        self._layer_weights_packed = _pack_layer_weights(layer_data)
        self._bind_dims()
        self._lib.set_decode_blocks_override(0 if decode_blocks is None else int(decode_blocks))

        dev = self._embed_weight.device
        bf16 = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        u32 = dict(dtype=torch.uint32, device=dev)
        types = [ld["type"] for ld in layer_data]
        n_fa, n_dn = sum(types), len(types) - sum(types)
        self._fa_k_cache = torch.zeros(max(n_fa, 1), FA_NUM_KV_HEADS, self.max_seq_len, FA_HEAD_DIM, **bf16)
        self._fa_v_cache = torch.zeros_like(self._fa_k_cache)
        self._dn_states = torch.zeros(max(n_dn, 1), DN_NUM_HEADS, DN_KEY_DIM, DN_VALUE_DIM, **f32)
        self._conv_bufs = torch.zeros(max(n_dn, 1), DN_CONV_CHANNELS, DN_CONV_KERNEL, **f32)
        self._hidden = torch.empty(HIDDEN_SIZE, **bf16)
        self._activations = torch.empty(HIDDEN_SIZE * 8 + INTERMEDIATE_SIZE, **f32)
        self._residual = torch.empty(HIDDEN_SIZE, **bf16)
        self._qkv_scratch = torch.empty(max(FA_QPROJ_SIZE, DN_CONV_CHANNELS), **f32)
        self._kv_scratch = torch.empty(FA_KV_SIZE * 2, **f32)
        self._attn_out = torch.empty(max(FA_Q_SIZE, DN_V_SIZE), **f32)
        self._mlp_inter = torch.empty(INTERMEDIATE_SIZE, **f32)
        self._z_scratch = torch.empty(DN_V_SIZE, **f32)
        self._beta_scratch = torch.empty(DN_NUM_HEADS, **f32)
        self._alpha_scratch = torch.empty(DN_NUM_HEADS, **f32)
        self._normalized = torch.empty(HIDDEN_SIZE, **f32)
        self._barrier_counter = torch.zeros(1, **u32)
        self._barrier_generation = torch.zeros(1, **u32)
        self._block_max_vals = torch.empty(1024, **f32)
        self._block_max_idxs = torch.empty(1024, **i32)
        self._lm_sync_counter = torch.zeros(1, **u32)
        self._seen_token_mask = torch.zeros(self.vocab, **f32)
        self._out_token = torch.empty(1, **i32)
        self._token_buffer = torch.empty(1, **i32)
        self._final_normed = torch.empty(HIDDEN_SIZE, **bf16)
        self._hidden_bf16_out = torch.empty(HIDDEN_SIZE, **bf16)

        # fused weights for the prefill GEMMs: q|k|v rows of every attention layer and gate|up rows
        # of every layer (reference: megakernel/model.py:242-260)
        fa = [torch.cat([ld["ptrs"][1], ld["ptrs"][2], ld["ptrs"][3]], dim=0) for ld in layer_data if ld["type"] == 1]
        self._fused_fa_qkv = (torch.stack(fa, dim=0).contiguous() if fa
                              else torch.zeros(1, FA_QPROJ_SIZE + 2 * FA_KV_SIZE, HIDDEN_SIZE, **bf16))
        gu = [torch.cat([ld["ptrs"][11], ld["ptrs"][12]] if ld["type"] == 0 else [ld["ptrs"][8], ld["ptrs"][9]], dim=0)
              for ld in layer_data]
        self._fused_gate_up = torch.stack(gu, dim=0).contiguous()

    # ------------------------------------------------------------------------------------
    def _bind_dims(self):
        rc = self._lib.mk_set_model_dims(self.num_layers, self.vocab)
        if rc != 0:
            raise RuntimeError(self._lib.mk_last_error_string().decode())

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(f"luce_megakernel_b200 error {rc}: {self._lib.mk_last_error_string().decode()}")

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self._embed_weight.device).cuda_stream)

    def step_async(self, token_id: int):
        """Enqueue one decode step; the next token lands in self._out_token (no host sync)."""
        if self._position >= self.max_seq_len:
            raise ValueError(f"position {self._position} exceeds max_seq_len={self.max_seq_len}")
        self._bind_dims()
        if self.api == "ops":
            self._ops.decode(
                self._out_token, token_id, self._embed_weight, self._layer_weights_packed,
                self._final_norm_weight, self._lm_head_weight, self._fa_k_cache, self._fa_v_cache,
                self._dn_states, self._conv_bufs, self._hidden, self._activations, self._residual,
                self._qkv_scratch, self._kv_scratch, self._attn_out, self._mlp_inter, self._z_scratch,
                self._beta_scratch, self._alpha_scratch, self._normalized, self._barrier_counter,
                self._barrier_generation, self._block_max_vals, self._block_max_idxs, self._lm_sync_counter,
                self._seen_token_mask, self.repetition_penalty, self._position, self.max_seq_len)
        else:
            self._check(self._lib.launch_decode(
                ctypes.c_int(int(token_id)), _ptr(self._out_token), _ptr(self._embed_weight),
                _ptr(self._layer_weights_packed), _ptr(self._final_norm_weight), _ptr(self._lm_head_weight),
                _ptr(self._fa_k_cache), _ptr(self._fa_v_cache), _ptr(self._dn_states), _ptr(self._conv_bufs),
                _ptr(self._hidden), _ptr(self._activations), _ptr(self._residual), _ptr(self._qkv_scratch),
                _ptr(self._kv_scratch), _ptr(self._attn_out), _ptr(self._mlp_inter), _ptr(self._z_scratch),
                _ptr(self._beta_scratch), _ptr(self._alpha_scratch), _ptr(self._normalized),
                _ptr(self._barrier_counter), _ptr(self._barrier_generation), _ptr(self._block_max_vals),
                _ptr(self._block_max_idxs), _ptr(self._lm_sync_counter), _ptr(self._seen_token_mask),
                ctypes.c_float(self.repetition_penalty), ctypes.c_int(self._position),
                ctypes.c_int(self.max_seq_len), self._stream()))
        self._position += 1

    def step(self, token_id: int) -> int:
        """Decode one token.  Returns the next token id (synchronises with the device)."""
        if self.api != "cabi":
            self.step_async(token_id)
            return int(self._out_token.item())
        # C ABI: mk_decode_step_host returns the token through mapped pinned memory (no device-to-host copy, no stream
        # synchronisation); the pointer arguments of a session never change, so they are converted once
        if self._position >= self.max_seq_len:
            raise ValueError(f"position {self._position} exceeds max_seq_len={self.max_seq_len}")
        if self._step_args is None:
            self._step_host_tok = ctypes.c_int(0)
            self._step_args = (
                _ptr(self._out_token), ctypes.byref(self._step_host_tok), _ptr(self._embed_weight),
                _ptr(self._layer_weights_packed), _ptr(self._final_norm_weight), _ptr(self._lm_head_weight),
                _ptr(self._fa_k_cache), _ptr(self._fa_v_cache), _ptr(self._dn_states), _ptr(self._conv_bufs),
                _ptr(self._hidden), _ptr(self._qkv_scratch), _ptr(self._kv_scratch), _ptr(self._attn_out),
                _ptr(self._mlp_inter), _ptr(self._z_scratch), _ptr(self._beta_scratch), _ptr(self._alpha_scratch),
                _ptr(self._normalized), _ptr(self._seen_token_mask))
        self._bind_dims()
        self._check(self._lib.mk_decode_step_host(
            ctypes.c_int(int(token_id)), *self._step_args, ctypes.c_float(self.repetition_penalty),
            ctypes.c_int(self._position), ctypes.c_int(self.max_seq_len), self._stream()))
        self._position += 1
        return int(self._step_host_tok.value)

    def step_sampled(self, token_id: int, temperature: float, top_k: int = 0, seed: int = 0, top_p: float = 1.0) -> int:
        """One decode step whose next token is drawn from softmax(logits / temperature) over the top_k largest
        logits, cut to the nucleus of mass top_p, instead of the argmax (the repetition penalty, if any, is applied to
        the logits first, as in the greedy path; reference hook: megakernel/kernel.cu:793-795; order of the stages as
        in the sampler chain of dflash/test/test_dflash.cpp:127-188).  Reproducible: the draw depends on
        (seed, position) only.  The step's logits stay in self._logits (f32 [vocab])."""
        if not hasattr(self, "_logits"):
            self._logits = torch.empty(self.vocab, dtype=torch.float32, device=self._embed_weight.device)
        self._lib.mk_set_logits_buffer(_ptr(self._logits))
        try:
            self.step_async(token_id)
        finally:
            self._lib.mk_set_logits_buffer(ctypes.c_void_p(0))
        rc = self._lib.mk_sample_top_k_top_p(_ptr(self._logits), ctypes.c_int(self.vocab), ctypes.c_float(float(temperature)),
                                             ctypes.c_int(int(top_k)), ctypes.c_float(float(top_p)), ctypes.c_ulonglong(int(seed)),
                                             ctypes.c_ulonglong(self._position), _ptr(self._out_token), self._stream())
        if rc != 0:
            self._lib.mk_sample_error.restype = ctypes.c_char_p
            raise RuntimeError(f"sampling failed ({rc}): {self._lib.mk_sample_error().decode()}")
        return int(self._out_token.item())

    def step_many(self, token_id: int, steps: int) -> torch.Tensor:
        """`steps` greedy steps with the token fed back on the device; returns the int32 device
        tensor of generated tokens without synchronising (bf16 counterpart of the reference's
        NVFP4 step_many, megakernel/model_nvfp4.py:742-769)."""
        if steps <= 0:
            return torch.empty(0, dtype=torch.int32, device=self._out_token.device)
        if self._position + steps > self.max_seq_len:
            raise ValueError("position + steps exceeds max_seq_len")
        self._bind_dims()
        out = torch.empty(steps, dtype=torch.int32, device=self._out_token.device)
        self._token_buffer.fill_(int(token_id))
        self._check(self._lib.mk_decode_many_bf16(
            _ptr(self._token_buffer), _ptr(out), ctypes.c_int(steps), _ptr(self._embed_weight),
            _ptr(self._layer_weights_packed), _ptr(self._final_norm_weight), _ptr(self._lm_head_weight),
            _ptr(self._fa_k_cache), _ptr(self._fa_v_cache), _ptr(self._dn_states), _ptr(self._conv_bufs),
            _ptr(self._hidden), _ptr(self._qkv_scratch), _ptr(self._kv_scratch), _ptr(self._attn_out),
            _ptr(self._mlp_inter), _ptr(self._z_scratch), _ptr(self._beta_scratch), _ptr(self._alpha_scratch),
            _ptr(self._normalized), _ptr(self._seen_token_mask), ctypes.c_float(self.repetition_penalty),
            ctypes.c_int(self._position), ctypes.c_int(self.max_seq_len), self._stream()))
        self._position += steps
        return out

    def alloc_prefill_scratch(self, S: int):
        """Scratch tensors of the reference's prefill signature (reference: megakernel/model.py:262-272).
        The sm_100a prefill keeps its own workspace, so these are minimal placeholders."""
        f32 = dict(dtype=torch.float32, device=self._embed_weight.device)
        return dict(dn_pre_qkv=torch.empty(1, **f32), dn_u_scratch=torch.empty(1, **f32),
                    dn_w_scratch=torch.empty(1, **f32), dn_cs_scratch=torch.empty(1, **f32))

    def prefill(self, token_ids) -> int:
        """Process a whole prompt from position 0 (state must be reset); returns the first generated
        token.  Afterwards step()/step_many() continue from position len(token_ids)."""
        tok = int(self.prefill_async(token_ids).item())
        st = self._lib.mk_prefill_status()
        if st != 0:
            raise RuntimeError(f"a bounded wait ran out inside a prefill kernel (status {st})")
        return tok

    def prefill_async(self, token_ids):
        """prefill() without the device-to-host read: returns the int32[1] device tensor that will hold
        the first generated token.  After the first call for a given weight table this only enqueues
        work, so it can be captured into a CUDA graph (pass a device int32 tensor of ids)."""
        ids = torch.as_tensor(token_ids, dtype=torch.int32).to(self._embed_weight.device).contiguous()
        S = int(ids.numel())
        if S < 1 or S > self.max_seq_len:
            raise ValueError("prompt length must be in [1, max_seq_len]")
        if self._position != 0:
            raise ValueError("prefill starts at position 0: call reset() first")
        self._bind_dims()
        if self.api == "ops":
            e = torch.empty(1, dtype=torch.bfloat16, device=ids.device)
            f = torch.empty(1, dtype=torch.float32, device=ids.device)
            i = torch.empty(1, dtype=torch.int32, device=ids.device)
            self._ops.prefill_bf16(
                self._out_token, ids, self._embed_weight, self._layer_weights_packed, self._final_norm_weight,
                self._lm_head_weight, self._fa_k_cache, self._fa_v_cache, self._dn_states, self._conv_bufs,
                e, e, e, e, e, e, e, e, f, f, f, f, f, f, self._fused_fa_qkv, self._fused_gate_up,
                self._final_normed, self._hidden_bf16_out, f, i, self.max_seq_len)
        else:
            self._lib.mk_prefill_error.restype = ctypes.c_char_p
            rc = self._lib.mk_prefill_bf16(
                _ptr(ids), ctypes.c_int(S), _ptr(self._out_token), _ptr(self._embed_weight),
                _ptr(self._layer_weights_packed), _ptr(self._final_norm_weight), _ptr(self._lm_head_weight),
                _ptr(self._fa_k_cache), _ptr(self._fa_v_cache), _ptr(self._dn_states), _ptr(self._conv_bufs),
                _ptr(self._fused_fa_qkv), _ptr(self._fused_gate_up), _ptr(self._final_normed),
                _ptr(self._hidden_bf16_out), ctypes.c_int(self.max_seq_len), ctypes.c_int(self.num_layers),
                ctypes.c_int(self.vocab), self._stream())
            if rc != 0:
                raise RuntimeError(f"prefill failed ({rc}): {self._lib.mk_prefill_error().decode()}")
        self._position = S
        return self._out_token

    def prefill_graphed(self, token_ids) -> int:
        """reset() + prefill() replayed from a CUDA graph kept per prompt length, the ids going through a static device
        buffer (the reference's NVFP4 driver does the same: megakernel/model_nvfp4.py:676-702, _build_prefill_graph /
        _prefill_graph_state).  The graph bakes in the library workspace's addresses: the workspace is reserved for
        the length before the capture, and a graph taken before a later growth is captured again."""
        ids = torch.as_tensor(token_ids, dtype=torch.int32).to(self._embed_weight.device).contiguous()
        S = int(ids.numel())
        if S < 1 or S > self.max_seq_len:
            raise ValueError("prompt length must be in [1, max_seq_len]")
        lib = self._lib
        lib.mk_prefill_workspace_generation.restype = ctypes.c_uint
        cache = self.__dict__.setdefault("_prefill_graphs", {})
        st = cache.get(S)
        if st is None or st["generation"] != lib.mk_prefill_workspace_generation():
            if lib.mk_prefill_reserve(ctypes.c_int(S)) != 0:
                raise RuntimeError("mk_prefill_reserve failed")
            static_ids = torch.zeros(S, dtype=torch.int32, device=ids.device)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):            # eager once: host-side caches filled, nothing left to allocate
                self.reset()
                self.prefill_async(static_ids)
            side.synchronize()
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self.reset()
                self.prefill_async(static_ids)
            st = {"graph": graph, "ids": static_ids, "generation": lib.mk_prefill_workspace_generation()}
            cache[S] = st
        st["ids"].copy_(ids)
        st["graph"].replay()
        self._position = S
        tok = int(self._out_token.item())
        status = lib.mk_prefill_status()
        if status != 0:
            raise RuntimeError(f"a bounded wait ran out inside a prefill kernel (status {status})")
        return tok

    def reset(self):
        self._position = 0
        self._fa_k_cache.zero_()
        self._fa_v_cache.zero_()
        self._dn_states.zero_()
        self._conv_bufs.zero_()
        self._seen_token_mask.zero_()

    def state_dict(self):
        """The whole session state (a checkpoint of a generation in flight)."""
        return {"position": self._position, "fa_k_cache": self._fa_k_cache.clone(),
                "fa_v_cache": self._fa_v_cache.clone(), "dn_states": self._dn_states.clone(),
                "conv_bufs": self._conv_bufs.clone(), "seen_token_mask": self._seen_token_mask.clone()}

    def load_state_dict(self, sd):
        self._position = int(sd["position"])
        self._fa_k_cache.copy_(sd["fa_k_cache"])
        self._fa_v_cache.copy_(sd["fa_v_cache"])
        self._dn_states.copy_(sd["dn_states"])
        self._conv_bufs.copy_(sd["conv_bufs"])
        self._seen_token_mask.copy_(sd["seen_token_mask"])

    def generate_ids(self, prompt_ids, max_tokens=100, eos=None, temperature=0.0, top_k=0, seed=0):
        """Token-level generate: feeds the prompt token by token, then decodes greedily (temperature 0) or samples."""
        self.reset()
        for tid in prompt_ids[:-1]:
            self.step_async(int(tid))
        out, nxt = [], int(prompt_ids[-1])
        for _ in range(max_tokens):
            nxt = self.step(nxt) if not temperature > 0 else self.step_sampled(nxt, temperature, top_k, seed)
            if eos is not None and nxt == eos:
                break
            out.append(nxt)
        return out

    def generate(self, prompt: str, max_tokens: int = 100) -> str:
        ids = self.tokenizer.encode(prompt, add_special_tokens=True)
        out = self.generate_ids(ids, max_tokens, self.tokenizer.eos_token_id)
        return self.tokenizer.decode(out, skip_special_tokens=True)


class BatchDecoder:
    """`batch` independent greedy sequences decoded together: every step reads each weight matrix once for all of
    them.  The reference has no batched op (megakernel/torch_bindings.cpp:569-675 are all batch 1); the state
    tensors are the reference's per-sequence layouts (megakernel/model.py:200-214) with a leading batch
    dimension, so slice b is exactly the state of a batch-1 Decoder.  Weights are shared with `decoder`.

    Sequences may have different lengths: prefill() takes one prompt per sequence and runs the prompt path on
    each slice; step()/step_many() then advance all sequences by one token per step."""

    MAX_BATCH = 16

    def __init__(self, decoder: Decoder, batch: int, nvfp4_ts: bool = False):
        """nvfp4_ts: the steps read the NVFP4 packing with a per-tensor scale (model_nvfp4.attach_nvfp4_ts_weights) instead
        of the bf16 weights; prompts are still prefilled in bf16."""
        if not 1 <= batch <= self.MAX_BATCH:
            raise ValueError(f"batch must be in [1, {self.MAX_BATCH}]")
        self._d = decoder
        self._ts = None
        if nvfp4_ts:
            from . import model_nvfp4 as MQ
            nv = MQ.attach_nvfp4_ts_weights(decoder._weights)["nvfp4_ts"]
            self._ts = {"table": MQ._pack_layer_weights_nvfp4_ts(nv["layer_data"]), "lm": nv["lm"]}
        self._lib = decoder._lib
        self.batch = int(batch)
        self.max_seq_len = decoder.max_seq_len
        dev = decoder._embed_weight.device
        types = [ld["type"] for ld in decoder._weights["layer_data"]]
        n_fa, n_dn = sum(types), len(types) - sum(types)
        B = self.batch
        self._fa_k_cache = torch.zeros(B, max(n_fa, 1), FA_NUM_KV_HEADS, self.max_seq_len, FA_HEAD_DIM,
                                       dtype=torch.bfloat16, device=dev)
        self._fa_v_cache = torch.zeros_like(self._fa_k_cache)
        self._dn_states = torch.zeros(B, max(n_dn, 1), DN_NUM_HEADS, DN_KEY_DIM, DN_VALUE_DIM, dtype=torch.float32, device=dev)
        self._conv_bufs = torch.zeros(B, max(n_dn, 1), DN_CONV_CHANNELS, DN_CONV_KERNEL, dtype=torch.float32, device=dev)
        self._tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self._positions = torch.zeros(B, dtype=torch.int32, device=dev)
        self._out_tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self._final_normed = torch.empty(B, HIDDEN_SIZE, dtype=torch.bfloat16, device=dev)
        self._hidden_bf16_out = torch.empty(B, HIDDEN_SIZE, dtype=torch.bfloat16, device=dev)
        self._host_positions = [0] * B

    def reset(self):
        for t in (self._fa_k_cache, self._fa_v_cache, self._dn_states, self._conv_bufs, self._tokens, self._positions):
            t.zero_()
        self._host_positions = [0] * self.batch

    def _fail(self, rc, what):
        self._lib.mk_prefill_error.restype = ctypes.c_char_p
        raise RuntimeError(f"{what} failed ({rc}): {self._lib.mk_prefill_error().decode()}")

    def _status(self):
        st = self._lib.mk_prefill_status()
        if st != 0:
            raise RuntimeError(f"a bounded wait ran out inside a kernel (status {st})")

    def prefill(self, prompts):
        """One prompt (list of ids) per sequence, from position 0.  Returns the first generated token of each;
        they are also the inputs of the next step()."""
        d = self._d
        if len(prompts) != self.batch:
            raise ValueError("one prompt per sequence")
        if any(p != 0 for p in self._host_positions):
            raise ValueError("prefill starts at position 0: call reset() first")
        d._bind_dims()
        for b, prompt in enumerate(prompts):
            ids = torch.as_tensor(prompt, dtype=torch.int32).to(self._tokens.device).contiguous()
            S = int(ids.numel())
            if S < 1 or S >= self.max_seq_len:
                raise ValueError("prompt length must be in [1, max_seq_len)")
            rc = self._lib.mk_prefill_bf16(
                _ptr(ids), ctypes.c_int(S), _ptr(self._tokens[b:b + 1]), _ptr(d._embed_weight), _ptr(d._layer_weights_packed),
                _ptr(d._final_norm_weight), _ptr(d._lm_head_weight), _ptr(self._fa_k_cache[b]), _ptr(self._fa_v_cache[b]),
                _ptr(self._dn_states[b]), _ptr(self._conv_bufs[b]), _ptr(d._fused_fa_qkv), _ptr(d._fused_gate_up),
                _ptr(self._final_normed[b]), _ptr(self._hidden_bf16_out[b]), ctypes.c_int(self.max_seq_len),
                ctypes.c_int(d.num_layers), ctypes.c_int(d.vocab), d._stream())
            if rc != 0:
                self._fail(rc, "prefill")
            self._host_positions[b] = S
        self._positions.copy_(torch.tensor(self._host_positions, dtype=torch.int32))
        first = self._tokens.cpu().tolist()
        self._status()
        return first

    def _args(self):
        d = self._d
        return (_ptr(d._embed_weight), _ptr(d._layer_weights_packed), _ptr(d._final_norm_weight), _ptr(d._lm_head_weight),
                _ptr(self._fa_k_cache), _ptr(self._fa_v_cache), _ptr(self._dn_states), _ptr(self._conv_bufs),
                _ptr(d._fused_fa_qkv), _ptr(d._fused_gate_up))

    def _args_ts(self):
        d, t = self._d, self._ts
        return (_ptr(d._embed_weight), _ptr(t["table"]), _ptr(d._final_norm_weight), _ptr(t["lm"]["packed"]),
                _ptr(t["lm"]["scales"]), _ptr(t["lm"]["tensor_scale"]), _ptr(self._fa_k_cache), _ptr(self._fa_v_cache),
                _ptr(self._dn_states), _ptr(self._conv_bufs))

    def step_async(self, tokens=None):
        """Enqueue one step for all sequences (inputs: `tokens`, or the tokens of the previous step / prefill).
        Returns the device int32[batch] tensor that will hold the chosen tokens.  Capturable into a CUDA graph
        when `tokens` is None or a device tensor."""
        d = self._d
        if max(self._host_positions) >= self.max_seq_len:
            raise ValueError("a sequence has reached max_seq_len")
        if tokens is not None:
            self._tokens.copy_(torch.as_tensor(tokens, dtype=torch.int32), non_blocking=True)
        if self._ts is not None:
            rc = self._lib.mk_decode_batch_nvfp4_ts(
                ctypes.c_int(1), _ptr(self._tokens), _ptr(self._positions), _ptr(self._out_tokens), ctypes.c_void_p(0),
                ctypes.c_int(self.batch), *self._args_ts(), _ptr(self._final_normed), _ptr(self._hidden_bf16_out),
                ctypes.c_int(self.max_seq_len), ctypes.c_int(d.num_layers), ctypes.c_int(d.vocab), d._stream())
        else:
            rc = self._lib.mk_decode_batch(
                _ptr(self._tokens), _ptr(self._positions), _ptr(self._out_tokens), ctypes.c_int(self.batch), *self._args(),
                _ptr(self._final_normed), _ptr(self._hidden_bf16_out), ctypes.c_int(self.max_seq_len),
                ctypes.c_int(d.num_layers), ctypes.c_int(d.vocab), d._stream())
        if rc != 0:
            self._fail(rc, "batched step")
        self._positions += 1
        self._tokens.copy_(self._out_tokens)
        self._host_positions = [p + 1 for p in self._host_positions]
        return self._out_tokens

    def step(self, tokens=None):
        out = self.step_async(tokens).cpu().tolist()
        self._status()
        return out

    def step_many(self, steps: int) -> torch.Tensor:
        """`steps` greedy steps with the chosen tokens fed back on the device; returns int32 [steps][batch]."""
        d = self._d
        if steps < 1 or max(self._host_positions) + steps > self.max_seq_len:
            raise ValueError("steps must be positive and stay within max_seq_len")
        log = torch.empty(steps, self.batch, dtype=torch.int32, device=self._tokens.device)
        if self._ts is not None:
            rc = self._lib.mk_decode_batch_nvfp4_ts(
                ctypes.c_int(steps), _ptr(self._tokens), _ptr(self._positions), ctypes.c_void_p(0), _ptr(log),
                ctypes.c_int(self.batch), *self._args_ts(), ctypes.c_void_p(0), ctypes.c_void_p(0),
                ctypes.c_int(self.max_seq_len), ctypes.c_int(d.num_layers), ctypes.c_int(d.vocab), d._stream())
        else:
            rc = self._lib.mk_decode_batch_many(
                ctypes.c_int(steps), _ptr(self._tokens), _ptr(self._positions), _ptr(log), ctypes.c_int(self.batch), *self._args(),
                ctypes.c_int(self.max_seq_len), ctypes.c_int(d.num_layers), ctypes.c_int(d.vocab), d._stream())
        if rc != 0:
            self._fail(rc, "batched steps")
        self._host_positions = [p + steps for p in self._host_positions]
        return log
