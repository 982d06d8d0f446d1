"""Minimal end-to-end example: a random-init model of the architecture decodes a few tokens.

    python -m luce_megakernel_b200.demo [--steps 8] [--context 520] [--layers 24] [--vocab 248320] [--batch 8]
                                        [--nvfp4 ts|mma] [--gemm M,N,K]

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
    ap.add_argument("--nvfp4", default="", choices=["", "ts", "mma"],
                    help="decode the steps with NVFP4 weights: ts = mma.sync kernel, mma = block-scaled tcgen05 kernel")
    ap.add_argument("--gemm", default="", help="M,N,K: run the NVFP4 and the bf16 projection GEMM on random operands and exit")
    args = ap.parse_args()
    if args.gemm:
        return gemm_demo(*[int(x) for x in args.gemm.split(",")])
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
    if args.nvfp4:
        from . import model_nvfp4 as MQ
        q = MQ.DecoderTS(weights, max_seq_len=dec.max_seq_len) if args.nvfp4 == "ts" else MQ.DecoderMMA(weights, max_seq_len=dec.max_seq_len)
        q.adopt_state(dec)
        dec = q
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = dec.step_many(tok, args.steps)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    status = lib().mk_device_status()
    if status != 0:
        raise SystemExit(f"device-side wait timed out (status {status})")
    print(f"{args.steps} tokens in {dt * 1e3:.2f} ms ({args.steps / dt:.0f} tok/s): {out.tolist()[:8]}")


def gemm_demo(m, n, k):
    """Three calls each of the NVFP4 x NVFP4 and the bf16 GEMM on [m, k] x [n, k]^T (m % 128 == 0)."""
    import ctypes
    L = lib()
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda") * 0.05).to(torch.bfloat16)
    c = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    q = []
    for x in (a, w):
        r, cols = x.shape
        pk = torch.zeros(r, cols // 2, dtype=torch.uint8, device="cuda")
        sc = torch.zeros((r // 128) * (cols // 64) * 512, dtype=torch.uint8, device="cuda")
        ts = torch.zeros(4, dtype=torch.float32, device="cuda")
        if L.mk_quantize_nvfp4_tensor_scale(P(x), r, cols, P(pk), P(sc), P(ts), st) != 0:
            raise SystemExit("quantiser failed")
        q.append((pk, sc, ts))
    for _ in range(3):
        if L.mk_gemm_nvfp4_tn(P(q[0][0]), P(q[0][1]), P(q[0][2]), P(q[1][0]), P(q[1][1]), P(q[1][2]), P(c), None, m, n, k, st) != 0:
            raise SystemExit("NVFP4 GEMM failed")
    for _ in range(3):
        if L.mk_gemm_bf16_tn(P(a), P(w), P(c), None, m, n, k, st) != 0:
            raise SystemExit("bf16 GEMM failed")
    torch.cuda.synchronize()
    if L.mk_gemm_nvfp4_status() != 0:
        raise SystemExit("a bounded wait ran out in the NVFP4 GEMM")
    print(f"gemm {m}x{n}x{k}: done, c[0,0]={float(c[0, 0]):.4f}")


if __name__ == "__main__":
    main()
