"""Prompt compression for speculative prefill with the decoder's own model as the drafter.

Mirrors the reference's `drafter_score_and_compress(ctx, ids, keep_ratio, chunk_size, n_lookahead, pool_kernel)`
(dflash/src/qwen3_drafter.cpp:86-183): one forward pass over the whole prompt (here: this library's prefill, block-sparse
for long prompts), tail-attention scores of the last `n_lookahead` positions over every key, then chunk selection.
The reference hosts a separate 0.6 B drafter model; here the model that will answer scores its own prompt.
"""
import ctypes

import numpy as np
import torch


def tail_scores(decoder, ids, n_lookahead=8, block_sparse=None):
    """running_max [n_lookahead, S] (torch f32, CPU) of a prefill of `ids` from position 0.  `block_sparse`:
    None = dense attention, or (top_frac, window, sink) for the block-sparse prefill.  The decoder's session state is
    overwritten by the prefill (reset it afterwards if the prompt is not the one to continue from)."""
    lib = decoder._lib
    ids = torch.as_tensor(ids, dtype=torch.int32)
    S = int(ids.numel())
    if S <= n_lookahead:
        raise ValueError("the prompt must be longer than the lookahead")
    buf = torch.zeros(n_lookahead, S, dtype=torch.float32, device=decoder._embed_weight.device)
    lib.mk_prefill_set_tail_scoring(ctypes.c_int(n_lookahead), ctypes.c_void_p(buf.data_ptr()))
    if block_sparse is not None:
        lib.mk_prefill_set_block_sparse(1, ctypes.c_double(block_sparse[0]), int(block_sparse[1]), int(block_sparse[2]))
    try:
        decoder.reset()
        decoder.prefill(ids.to(decoder._embed_weight.device))
        torch.cuda.synchronize()
    finally:
        lib.mk_prefill_set_tail_scoring(0, ctypes.c_void_p(0))
        if block_sparse is not None:
            lib.mk_prefill_set_block_sparse(0, ctypes.c_double(0.10), 4, 1)
    return buf.cpu()


def select_positions(lib, running_max, keep_ratio, chunk_size=32, pool_kernel=13):
    """Kept token positions (ascending numpy int32) for a running_max [n_lookahead, S] array (mk_drafter_select)."""
    rm = np.ascontiguousarray(np.asarray(running_max, dtype=np.float32))
    n, S = rm.shape
    out = np.empty(S, dtype=np.int32)
    lib.mk_drafter_select.restype = ctypes.c_int
    k = lib.mk_drafter_select(rm.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(n), ctypes.c_int(S), ctypes.c_float(keep_ratio),
                              ctypes.c_int(chunk_size), ctypes.c_int(pool_kernel), out.ctypes.data_as(ctypes.c_void_p))
    if k < 0:
        raise ValueError("mk_drafter_select: bad argument")
    return out[:k].copy()


def score_and_compress(decoder, ids, keep_ratio, chunk_size=32, n_lookahead=8, pool_kernel=13, block_sparse=None):
    """The compressed prompt: ids of the kept chunks in their original order (the reference returns the prompt unchanged
    when it is too short to score; so does this)."""
    ids = [int(t) for t in ids]
    if len(ids) < n_lookahead + 1:
        return ids
    rm = tail_scores(decoder, ids, n_lookahead, block_sparse)
    keep = select_positions(decoder._lib, rm.numpy(), keep_ratio, chunk_size, pool_kernel)
    return [ids[j] for j in keep]
