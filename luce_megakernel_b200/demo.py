"""Minimal end-to-end example: a random-init model of the architecture decodes a few tokens.

    python -m luce_megakernel_b200.demo [--steps 8] [--context 520] [--layers 24] [--vocab 248320] [--batch 8]

Also the small, bounded workload used for profiler captures of the decode kernel (few launches,
about 1.6 GB on the device).
"""
import argparse
import time

import torch

from . import lib
from . import model as M


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--context", type=int, default=520)
    ap.add_argument("--layers", type=int, default=M.NUM_LAYERS)
    ap.add_argument("--vocab", type=int, default=M.VOCAB_SIZE)
    ap.add_argument("--prefill", type=int, default=0, help="prompt length processed by the prefill op instead of the decode kernel")
    ap.add_argument("--batch", type=int, default=0, help="decode this many sequences together (batched step) at --context")
    args = ap.parse_args()
    weights, _ = M.load_weights(seed=0, num_layers=args.layers, vocab=args.vocab, device_init=True)
    dec = M.Decoder(weights=weights, max_seq_len=max(2048, args.context + args.steps + 8, args.prefill + args.steps + 8), api="cabi")
    if args.batch > 0:
        # batched step at the requested context (caches are zero: same traffic as real ones), tokens fed back on the device
        bd = M.BatchDecoder(dec, args.batch)
        bd._host_positions = [args.context] * args.batch
        bd._positions.fill_(args.context)
        bd._tokens.copy_(torch.arange(11, 11 + args.batch, dtype=torch.int32))
        bd.step_many(1)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = bd.step_many(args.steps)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        if lib().mk_prefill_status() != 0:
            raise SystemExit("device-side wait timed out")
        print(f"batch {args.batch}: {args.steps} steps in {dt * 1e3:.2f} ms ({args.batch * args.steps / dt:.0f} tok/s): {out[-1].tolist()[:8]}")
        return
    if args.prefill > 0:
        g = torch.Generator().manual_seed(0)
        ids = torch.randint(0, args.vocab, (args.prefill,), generator=g)
        dec.prefill(ids)                    # warm-up (sizes the workspace)
        dec.reset()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        tok = dec.prefill(ids)
        dt = time.perf_counter() - t0
        print(f"prefill of {args.prefill} tokens in {dt * 1e3:.2f} ms ({args.prefill / dt:.0f} tok/s)")
    else:
        tok = 11
        for _ in range(4):                  # a short prompt through the decode kernel
            tok = dec.step(tok)
        dec._position = args.context        # continue at the requested context length
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = dec.step_many(tok, args.steps)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    status = lib().mk_device_status()
    if status != 0:
        raise SystemExit(f"device-side wait timed out (status {status})")
    print(f"{args.steps} tokens in {dt * 1e3:.2f} ms ({args.steps / dt:.0f} tok/s): {out.tolist()[:8]}")


if __name__ == "__main__":
    main()
