"""CUDA-graph capture of the prefill and of the batched step, and the workspace rules that make it safe.

The prefill entry points and the batched decode step share one grow-only library workspace per device.  A
graph bakes the workspace's device pointers in, so: the workspace is sized once with mk_prefill_reserve()
before capturing, growth during a capture is refused instead of invalidating it, and a growth after a capture is
visible through mk_prefill_workspace_generation() (the graph must then be captured again).
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

NL, V, MAXSEQ = 4, 1024, 512


@pytest.fixture(scope="module")
def dec():
    from luce_megakernel_b200 import model as M
    from luce_megakernel_b200.weights import random_state_dict
    sd = random_state_dict(21, NL, V, "unit")
    return M.Decoder(weights=M.weights_from_state_dict(sd), max_seq_len=MAXSEQ, api="cabi")


def _ids(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, V, (n,), generator=g).to(torch.int32).cuda()


def test_prefill_and_batched_step_replay_from_a_graph(dec):
    from luce_megakernel_b200 import model as M, lib
    L = lib()
    L.mk_prefill_workspace_generation.restype = ctypes.c_uint
    assert L.mk_prefill_reserve(300) == 0
    ids = _ids(40, 1)
    dec.reset()
    want = dec.prefill(ids)                          # eager run (also caches the pointer table on the host)
    want_state = dec._dn_states.clone()
    gen = L.mk_prefill_workspace_generation()

    dec.reset()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dec.prefill_async(ids)
    dec.reset()
    dec._out_token.fill_(-5)
    g.replay()
    torch.cuda.synchronize()
    assert int(dec._out_token.item()) == want
    assert torch.equal(dec._dn_states, want_state)
    assert L.mk_prefill_workspace_generation() == gen and L.mk_prefill_status() == 0

    # batched step: eager, then the same step from a graph
    bd = M.BatchDecoder(dec, 2)
    prompts = [ids.tolist(), ids[:17].tolist()]
    bd.prefill(prompts)
    ck = [t.clone() for t in (bd._fa_k_cache, bd._fa_v_cache, bd._dn_states, bd._conv_bufs, bd._tokens, bd._positions)]
    eager = bd.step()
    for t, c in zip((bd._fa_k_cache, bd._fa_v_cache, bd._dn_states, bd._conv_bufs, bd._tokens, bd._positions), ck):
        t.copy_(c)
    bd._host_positions = [40, 17]
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        bd.step_async()
    for t, c in zip((bd._fa_k_cache, bd._fa_v_cache, bd._dn_states, bd._conv_bufs, bd._tokens, bd._positions), ck):
        t.copy_(c)
    g2.replay()
    torch.cuda.synchronize()
    assert bd._out_tokens.cpu().tolist() == eager


def test_growth_is_refused_during_capture_and_visible_afterwards(dec):
    from luce_megakernel_b200 import model as M, lib
    L = lib()
    L.mk_prefill_workspace_generation.restype = ctypes.c_uint
    assert L.mk_prefill_reserve(300) == 0
    cap = L.mk_prefill_workspace_tokens()            # the workspace is per process: other tests may have grown it
    assert cap >= 300
    gen = L.mk_prefill_workspace_generation()
    big = M.Decoder(weights=dec._weights, max_seq_len=cap + 80, api="cabi")
    long_ids = _ids(cap + 64, 2)                     # needs more workspace than there is
    big.prefill(_ids(8, 3))                          # pointer table cached, nothing left to do on the host
    big.reset()
    refused = None
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        try:
            big.prefill_async(long_ids)
            refused = False
        except RuntimeError as e:
            refused = "mk_prefill_reserve" in str(e)
    assert refused is True
    assert L.mk_prefill_workspace_generation() == gen        # nothing was reallocated under the capture
    big.reset()
    big.prefill(long_ids)                            # outside a capture the workspace grows ...
    assert L.mk_prefill_workspace_generation() != gen        # ... and says so: earlier graphs must be captured again
    assert L.mk_prefill_workspace_tokens() >= cap + 64 and L.mk_prefill_status() == 0


def test_prefill_graphed_keeps_one_graph_per_length_and_recaptures_after_growth(dec):
    """Decoder.prefill_graphed (the reference's per-length prefill graph cache, megakernel/model_nvfp4.py:676-702)."""
    from luce_megakernel_b200 import model as M, lib
    L = lib()
    a, b = _ids(33, 5), _ids(33, 6)
    dec.reset(); want_a = dec.prefill(a); state_a = dec._dn_states.clone()
    dec.reset(); want_b = dec.prefill(b)
    assert dec.prefill_graphed(a) == want_a and torch.equal(dec._dn_states, state_a) and dec._position == 33
    g33 = dec._prefill_graphs[33]["graph"]
    assert dec.prefill_graphed(b) == want_b                   # same length: the cached graph, new ids, state reset inside
    assert dec._prefill_graphs[33]["graph"] is g33
    assert dec.step(int(want_b)) >= 0                          # decoding continues from the graph's state
    c = _ids(57, 7)
    dec.reset(); want_c = dec.prefill(c)
    assert dec.prefill_graphed(c) == want_c and set(dec._prefill_graphs) >= {33, 57}
    # a growth of the library workspace invalidates the baked-in addresses: the next call captures again
    L.mk_prefill_workspace_generation.restype = ctypes.c_uint
    cap = L.mk_prefill_workspace_tokens()
    big = M.Decoder(weights=dec._weights, max_seq_len=cap + 80, api="cabi")
    big.prefill(_ids(cap + 64, 8))
    assert L.mk_prefill_workspace_generation() != dec._prefill_graphs[33]["generation"]
    assert dec.prefill_graphed(a) == want_a and dec._prefill_graphs[33]["graph"] is not g33
    assert L.mk_prefill_status() == 0
