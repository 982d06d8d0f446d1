"""Host-side logic that needs no GPU: pointer-table packing, weight provider, C-ABI exports."""
import ctypes
import os
import re
import struct

import pytest
import torch

from luce_megakernel_b200 import CORE_LIB_PATH, model as M, weights as W
from oracle import qwen35_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_constants_match_oracle():
    assert (M.HIDDEN_SIZE, M.INTERMEDIATE_SIZE, M.VOCAB_SIZE, M.NUM_LAYERS) == (O.HIDDEN, O.INTER, O.VOCAB, O.NUM_LAYERS)
    assert M.LAYER_TYPE == O.layer_types()
    assert M.DN_CONV_CHANNELS == O.DN_CONV_CH and M.FA_QPROJ_SIZE == O.FA_QPROJ


def test_weight_provider_equals_oracle_init():
    a = W.random_state_dict(0, 4, 512, "literal")
    b = O.init_weights(0, 4, 512, "literal")
    assert list(a) == list(b)
    for k in a:
        assert torch.equal(a[k], b[k]), k
    c = W.random_state_dict(0, 4, 512, "unit")
    assert float(c["model.layers.0.input_layernorm.weight"].abs().max()) == 0.0
    assert float(c["model.layers.0.linear_attn.norm.weight"].min()) == 1.0


def test_layer_pointer_order():
    sd = W.random_state_dict(1, 4, 64)
    w = M.weights_from_state_dict(sd, device="cpu")
    assert [ld["type"] for ld in w["layer_data"]] == [0, 0, 0, 1]
    dn, fa = w["layer_data"][0]["ptrs"], w["layer_data"][3]["ptrs"]
    assert len(dn) == 14 and len(fa) == 11
    assert tuple(dn[1].shape) == (6144, 1024) and tuple(dn[5].shape) == (6144, 1, 4) and tuple(dn[9].shape) == (1024, 2048)
    assert tuple(fa[1].shape) == (4096, 1024) and tuple(fa[6].shape) == (1024, 2048) and tuple(fa[10].shape) == (1024, 3584)
    assert w["lm_head_weight"] is w["embed_weight"]      # tied


def test_pack_layout_is_128_bytes_per_layer():
    entry = struct.Struct("<4i14Q")
    assert entry.size == 128
    blob = entry.pack(1, 0, 0, 0, *range(100, 114))
    t, _, _, _, *ptrs = entry.unpack(blob)
    assert t == 1 and ptrs == list(range(100, 114))


def _declared_symbols():
    txt = open(os.path.join(ROOT, "include", "luce_megakernel_b200.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(launch_\w+|mk_\w+|set_decode_blocks_override|query_max_safe_decode_blocks)\s*\(", txt)))


def test_cabi_library_exports_every_declared_symbol():
    assert os.path.exists(CORE_LIB_PATH), "native library missing: run python -m luce_megakernel_b200._build"
    lib = ctypes.CDLL(CORE_LIB_PATH)
    names = _declared_symbols()
    assert "launch_decode" in names and "mk_decode_many_bf16" in names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"


def test_bad_arguments_are_rejected_without_a_gpu():
    lib = ctypes.CDLL(CORE_LIB_PATH)
    lib.mk_last_error_string.restype = ctypes.c_char_p
    assert lib.mk_set_model_dims(0, 10) == 1
    assert lib.mk_set_model_dims(25, 10) == 1
    assert lib.mk_set_model_dims(24, 0) == 1
    assert b"num_layers" in lib.mk_last_error_string() or b"vocab" in lib.mk_last_error_string()
    assert lib.mk_set_model_dims(24, 248320) == 0
    # null pointers are refused before any CUDA call
    nul = ctypes.c_void_p(0)
    rc = lib.launch_decode(ctypes.c_int(1), nul, *([nul] * 25), ctypes.c_float(1.0), ctypes.c_int(0), ctypes.c_int(16), nul)
    assert rc == 1


def test_static_scratch_entry_rejects_misaligned_pointers_without_a_gpu():
    """A pointer that is 4-byte but not 16-byte aligned (a sliced cache or embedding tensor) would make the kernel's
    bulk copies and vector loads fault on the device: it must be refused on the host, before any CUDA call."""
    lib = ctypes.CDLL(CORE_LIB_PATH)
    lib.mk_decode_bf16_static_scratch_error.restype = ctypes.c_char_p
    base = 0x7f0000000000                      # never dereferenced: validation fails first

    def call(bad_index):
        ptrs = [ctypes.c_void_p(base + 4096 * i + (4 if i == bad_index else 0)) for i in range(19)]
        return lib.mk_decode_bf16_static_scratch(
            ctypes.c_int(1), *ptrs, ctypes.c_float(1.0), ctypes.c_int(0), ctypes.c_int(16), ctypes.c_int(4),
            ctypes.c_int(1024), ctypes.c_void_p(0))

    # 1 embed, 2 layer table, 3 final norm, 4 lm head, 5/6 caches, 7 states, 8 conv, 9 hidden, 10-14 vector scratch, 17 normalized
    for i in (1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 17):
        assert call(i) == 1, f"argument {i} misaligned by 4 bytes was accepted"
        assert b"16-byte" in lib.mk_decode_bf16_static_scratch_error()
    ptrs = [ctypes.c_void_p(base + 4096 * i + (2 if i == 0 else 0)) for i in range(19)]
    assert lib.mk_decode_bf16_static_scratch(ctypes.c_int(1), *ptrs, ctypes.c_float(1.0), ctypes.c_int(0), ctypes.c_int(16),
                                             ctypes.c_int(4), ctypes.c_int(1024), ctypes.c_void_p(0)) == 1


def test_missing_library_fails_loudly(monkeypatch):
    import luce_megakernel_b200 as L
    monkeypatch.setattr(L, "_lib", None)
    monkeypatch.setattr(L, "CORE_LIB_PATH", "/nonexistent/libluce.so")
    with pytest.raises(L.NativeLibraryMissing):
        L.lib()
