"""The allocation-free decode entry point against the regular one.

Some hosts cannot let this library allocate device memory (a server that reserved all HBM for
its own pool, a loop that cannot take cudaMalloc's device-wide synchronisation).  For them
mk_decode_bf16_static_scratch() runs the decode kernel with its scratch in a static device
array.  This test drives both entry points through the C ABI on identical weights, state and
tokens, twice in a row (the second call finds the first call's leftovers in the shared array),
and requires identical tokens and bit-identical state, which is the bound the other tests use
for two runs of the same kernel.  It builds its own small model, so it passes alone in a fresh
process as well as after the rest of the suite (it is collected last on purpose).
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

NL, V, MAXSEQ = 4, 1024, 64


def _decoder():
    from luce_megakernel_b200 import model as M
    from luce_megakernel_b200.weights import random_state_dict
    sd = random_state_dict(11, NL, V, "unit")
    return M.Decoder(weights=M.weights_from_state_dict(sd), max_seq_len=MAXSEQ, api="cabi")


def _static_step(dec, token):
    """One step through mk_decode_bf16_static_scratch on the decoder's own tensors."""
    from luce_megakernel_b200.model import _ptr
    lib = dec._lib
    lib.mk_decode_bf16_static_scratch_error.restype = ctypes.c_char_p
    rc = lib.mk_decode_bf16_static_scratch(
        ctypes.c_int(int(token)), _ptr(dec._out_token), _ptr(dec._embed_weight), _ptr(dec._layer_weights_packed),
        _ptr(dec._final_norm_weight), _ptr(dec._lm_head_weight), _ptr(dec._fa_k_cache), _ptr(dec._fa_v_cache),
        _ptr(dec._dn_states), _ptr(dec._conv_bufs), _ptr(dec._hidden), _ptr(dec._qkv_scratch), _ptr(dec._kv_scratch),
        _ptr(dec._attn_out), _ptr(dec._mlp_inter), _ptr(dec._z_scratch), _ptr(dec._beta_scratch),
        _ptr(dec._alpha_scratch), _ptr(dec._normalized), _ptr(dec._seen_token_mask), ctypes.c_float(1.0),
        ctypes.c_int(dec._position), ctypes.c_int(dec.max_seq_len), ctypes.c_int(dec.num_layers),
        ctypes.c_int(dec.vocab), dec._stream())
    assert rc == 0, lib.mk_decode_bf16_static_scratch_error().decode()
    dec._position += 1
    return int(dec._out_token.item())


def test_static_scratch_entry_matches_launch_decode():
    a, b = _decoder(), _decoder()
    tokens = [17, 901]                       # two calls in a row on each entry point
    for t in tokens:
        ta = a.step(t)                       # launch_decode (library-allocated workspace)
        tb = _static_step(b, t)              # static scratch, nothing allocated
        assert ta == tb
        assert torch.equal(a._hidden, b._hidden)
        assert torch.equal(a._normalized, b._normalized)
    assert torch.equal(a._dn_states, b._dn_states)
    assert torch.equal(a._conv_bufs, b._conv_bufs)
    assert torch.equal(a._fa_k_cache, b._fa_k_cache) and torch.equal(a._fa_v_cache, b._fa_v_cache)


def test_static_scratch_entry_rejects_sizes_beyond_its_maximum():
    dec = _decoder()
    from luce_megakernel_b200.model import _ptr
    lib = dec._lib
    lib.mk_decode_bf16_static_scratch_error.restype = ctypes.c_char_p

    def call(num_layers, position):
        return lib.mk_decode_bf16_static_scratch(
            ctypes.c_int(1), _ptr(dec._out_token), _ptr(dec._embed_weight), _ptr(dec._layer_weights_packed),
            _ptr(dec._final_norm_weight), _ptr(dec._lm_head_weight), _ptr(dec._fa_k_cache), _ptr(dec._fa_v_cache),
            _ptr(dec._dn_states), _ptr(dec._conv_bufs), _ptr(dec._hidden), _ptr(dec._qkv_scratch),
            _ptr(dec._kv_scratch), _ptr(dec._attn_out), _ptr(dec._mlp_inter), _ptr(dec._z_scratch),
            _ptr(dec._beta_scratch), _ptr(dec._alpha_scratch), _ptr(dec._normalized), _ptr(dec._seen_token_mask),
            ctypes.c_float(1.0), ctypes.c_int(position), ctypes.c_int(MAXSEQ), ctypes.c_int(num_layers),
            ctypes.c_int(V), dec._stream())

    assert call(25, 0) == 1
    assert b"maximum" in lib.mk_decode_bf16_static_scratch_error()
    assert call(NL, MAXSEQ) == 1
    torch.cuda.synchronize()


def test_static_scratch_entry_allocates_nothing_and_reports_its_status():
    """The property the entry point exists for: free device memory is the same before and after further calls
    (the first call only resolves the array's address; nothing here calls launch_decode on this decoder), and the
    status word of a normal launch reads 0 through the allocation-free status query."""
    dec = _decoder()
    status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    _static_step(dec, 5)                                      # first call: one-time set-up for this device
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    toks = []
    for t in (9, 33, 2):
        toks.append(_static_step(dec, t))
        rc = dec._lib.mk_decode_bf16_static_scratch_status(ctypes.c_void_p(status.data_ptr()), dec._stream())
        assert rc == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes across static-scratch calls"
    assert int(status.item()) == 0
    assert all(0 <= t < V for t in toks)
