#!/usr/bin/env python
"""Headline benchmark: batch-1 greedy decode (tg128 after a 520-token prompt) of the 24-layer
Qwen3.5-0.8B-architecture hybrid in bf16 on B200, random-init weights, synthetic token ids.

    python bench.py --gpus N --steps K --warmup W                # this repo's kernels
    python bench.py --impl reference --gpus N --steps K ...      # CPU baseline arm (rank 0 only)
    python bench.py --impl reference_gpu --steps K ...           # the reference's own CUDA kernels, same GPU (rank 0 only)

One "step" is one tg128 pass: 128 greedy decode steps with the token fed back on the device.
Multi-GPU runs are independent replicas (one process per GPU, no data-path collective); the
reported value is the aggregate over all ranks divided by the slowest rank's time.
Prints ONE JSON line on rank 0.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_LEN = 520
GEN_LEN = 128
MAX_SEQ = 2048
WEIGHT_BYTES_PER_TOKEN = 1_546_073_728      # bf16 weights + DeltaNet state r/w + conv state r/w
NVFP4_BYTES_PER_TOKEN = 466_073_216         # the same with every linear layer and the LM head at 0.5625 bytes per weight
KV_BYTES_PER_POS = 12_288                   # K and V rows read per cached position, 6 layers
STATE_BYTES_PER_SEQ = 41_287_680            # DeltaNet state and conv window, read + written once per token
# dram__bytes_read.sum + dram__bytes_write.sum of one bf16 decode step: ncu capture of a 4-step launch at context 520
# (6.0436 GB read + 7.2 MB written), divided by 4
TRAFFIC_BYTES_PER_LAUNCH = 1_512_704_000


def algorithmic_bytes_per_token(context_len: float, nvfp4: bool = False) -> float:
    return (NVFP4_BYTES_PER_TOKEN if nvfp4 else WEIGHT_BYTES_PER_TOKEN) + KV_BYTES_PER_POS * context_len


def batch_step_bytes(batch: int, context_len: float) -> float:
    """Algorithmic HBM bytes of one batched step: the weights once, state and cache rows once per sequence."""
    return (WEIGHT_BYTES_PER_TOKEN - STATE_BYTES_PER_SEQ) + batch * (STATE_BYTES_PER_SEQ + KV_BYTES_PER_POS * context_len)


def kept_block_fraction(S: int, top_frac=0.10, window=4, sink=1) -> float:
    """Upper bound on the fraction of causal 128 x 128 blocks the sparse rule keeps (overlaps not subtracted)."""
    import math
    nb = (S + 127) // 128
    kept = sum(min(i + 1, sink + window + math.ceil(top_frac * (i + 1))) for i in range(nb))
    return kept / (nb * (nb + 1) / 2.0)


def prefill_tflop(S: int, sparse: bool = False) -> float:
    """Algorithmic FLOPs of a prefill of S tokens, in TFLOP: all per-token linear layers, causal attention
    (6 layers, 8 heads, head_dim 256; only the kept blocks when sparse), the gated delta rule in its
    recurrent-form count, one LM-head pass."""
    gemm = 2.0 * 497_614_848 * S
    attn = 6 * 8 * (4 * 256) * S * (S + 1) / 2.0 * (kept_block_fraction(S) if sparse else 1.0)
    scan = 18 * 16 * (6 * 128 * 128) * S
    return (gemm + attn + scan + 2.0 * 254_279_680) / 1e12


PREFILL_TFLOP_PP520 = prefill_tflop(520)        # 0.539


def measured_bf16_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(path))["bf16_tflops"])
    except Exception:
        return 1590.0


def measured_hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        try:
            return float(json.load(open(path))["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""
    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc = index, None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 6:
                continue
            try:
                sm.append(float(f[0])); mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[2:6]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        res = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons)}
        if not sm:
            # nvidia-smi had not produced a line yet: one query right after the timed region (clocks are still up)
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits"],
                                     capture_output=True, text=True, timeout=20).stdout
                f = [x.strip() for x in out.strip().splitlines()[0].split(",")]
                res = {"sm_mhz": float(f[0]), "sm_max_mhz": float(f[1]),
                       "reasons": sorted(n for n, v in zip(names, f[2:6]) if v.lower().startswith("active")),
                       "sampled": "once, right after the timed region"}
            except Exception:
                pass
        return res


# ---- CPU baselines ---------------------------------------------------------------------------------------------

class HfCpuBaseline:
    """The reference's PyTorch path on the host cores: `transformers`' Qwen3_5ForCausalLM (the class the reference
    loads in megakernel/final_bench.py:117-149), fp32, eager, with the benchmark's seeded weights: an untimed
    `context`-token prefill, then timed greedy decode steps on all host threads."""
    kind = "hf"

    def __init__(self, state_dict, context, threads):
        from transformers import AutoModelForCausalLM, Qwen3_5TextConfig
        torch.set_num_threads(threads)
        vocab = state_dict["model.embed_tokens.weight"].shape[0]
        n_layers = 1 + max(int(k.split(".")[2]) for k in state_dict if k.startswith("model.layers."))
        cfg = Qwen3_5TextConfig(
            vocab_size=vocab, hidden_size=1024, intermediate_size=3584, num_hidden_layers=n_layers,
            num_attention_heads=8, num_key_value_heads=2, head_dim=256, linear_num_key_heads=16, linear_num_value_heads=16,
            linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4, tie_word_embeddings=True,
            max_position_embeddings=max(4096, context + 4096), rms_norm_eps=1e-6,
            rope_parameters={"rope_theta": 1.0e7, "partial_rotary_factor": 0.25, "rope_type": "default"})
        with torch.device("meta"):                      # no random init of 0.75 B parameters that are overwritten anyway
            model = AutoModelForCausalLM.from_config(cfg, dtype=torch.float32)
        model = model.to_empty(device="cpu")
        model.model.rotary_emb = type(model.model.rotary_emb)(config=cfg)       # its buffers are not in the state dict
        sd = {k: v.to(torch.float32) for k, v in state_dict.items()}
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
        model.load_state_dict(sd, strict=True, assign=True)
        self.model = model.eval()
        g = torch.Generator().manual_seed(0)
        prompt = torch.randint(0, vocab, (context,), generator=g)
        with torch.no_grad():
            r = self.model(input_ids=prompt[None], use_cache=True)
        self.cache, self.tok = r.past_key_values, int(r.logits[0, -1].argmax())

    def tokens_per_s(self, n_tokens):
        t0 = time.perf_counter()
        with torch.no_grad():
            for _ in range(n_tokens):
                r = self.model(input_ids=torch.tensor([[self.tok]]), past_key_values=self.cache, use_cache=True)
                self.cache, self.tok = r.past_key_values, int(r.logits[0, -1].argmax())
        return n_tokens / (time.perf_counter() - t0)


class PortCpuBaseline:
    """Fallback when `transformers` cannot be imported: the CPU oracle (fp32 port of the reference decode arithmetic)."""
    kind = "port"

    def __init__(self, state_dict, context, threads):
        from oracle import qwen35_oracle as O      # the checker, timed here only as the CPU baseline
        torch.set_num_threads(threads)
        self.orc = O.Oracle(state_dict, rounding="none")
        self.st = O.State.new(self.orc.num_layers, context + 4096, self.orc.vocab)
        g = torch.Generator().manual_seed(0)
        prompt = torch.randint(0, self.orc.vocab, (context,), generator=g)
        self.tok = self.orc.forward(prompt, self.st).token

    def tokens_per_s(self, n_tokens):
        t0 = time.perf_counter()
        for _ in range(n_tokens):
            self.tok = self.orc.forward([self.tok], self.st).token
        return n_tokens / (time.perf_counter() - t0)


def make_cpu_baseline(state_dict, context, threads):
    try:
        return HfCpuBaseline(state_dict, context, threads)
    except Exception as e:                      # transformers missing or without this model class
        sys.stderr.write(f"transformers path unavailable ({e!r}); timing the oracle port instead\n")
        return PortCpuBaseline(state_dict, context, threads)


def cpu_baseline_in_child():
    """The CPU baseline of the GPU arm: the reference arm of this file (`--impl reference`, 2 timed steps of 4 tokens) in
    a child process that does not see the GPU -- this process has CUDA initialised, and transformers then picks
    kernels that cannot run on host tensors.  Returns the child's cpu_baseline object, or None if it failed."""
    import subprocess
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE"):
        env.pop(k, None)
    try:
        r = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "reference", "--steps", "2", "--warmup", "1"],
                           env=env, capture_output=True, text=True, timeout=900)
        line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1]
        cb = json.loads(line)["cpu_baseline"]
        cb["sample"] += " (2 timed steps, child process without the GPU)"
        return cb
    except Exception as e:
        sys.stderr.write(f"CPU baseline child failed ({e!r}); timing the oracle port in this process\n")
        return None


def cpu_baseline_in_process(weights):
    threads = os.cpu_count() or 1
    n_tok = 8
    base = PortCpuBaseline(cpu_state_dict(weights), PROMPT_LEN, threads)
    return {"value": base.tokens_per_s(n_tok), "unit": "tok/s", "cores": threads, "kind": base.kind,
            "sample": cpu_sample_text(base, n_tok, PROMPT_LEN)}


def cpu_sample_text(base, n_tokens, context):
    what = ("transformers Qwen3_5ForCausalLM, fp32 eager (the reference's PyTorch path)" if base.kind == "hf"
            else "fp32 oracle port of the reference decode arithmetic")
    return f"{n_tokens} greedy decode tokens after a {context}-token prompt; {what}; all host threads"


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    return rank, local, world


def workload_config(n_gpus):
    return {"workload": "configs[1]: 24-layer bf16 hybrid decode, batch 1, 520-token prompt then tg128 greedy",
            "prompt_len": PROMPT_LEN, "gen_len": GEN_LEN, "weights": "random-init seed 0 (drawn on the device)",
            "replicas": n_gpus, "l2": "inputs larger than L2 (1.5 GB of weights streamed per token)"}


def run_reference(args):
    """CPU arm: the reference's PyTorch path on this box's host cores, same model, same context, bounded sample."""
    rank, _, _ = dist_env()
    if rank != 0:
        return
    # this arm never touches the GPU; with a GPU visible, transformers routes parts of the model through Triton kernels
    # that cannot take host tensors, so hide it before anything initialises CUDA
    os.environ["CUDA_VISIBLE_DEVICES"] = ""
    from luce_megakernel_b200.weights import random_state_dict
    threads = os.cpu_count() or 1
    per_step = 4
    base = make_cpu_baseline(random_state_dict(0), PROMPT_LEN, threads)
    rates = []
    for i in range(args.warmup + args.steps):
        r = base.tokens_per_s(per_step)
        if i >= args.warmup:
            rates.append(r)
    value = statistics.mean(rates)
    cfg = workload_config(args.gpus)
    cfg.update({"weights": "random-init seed 0 (drawn on the host)", "replicas": 1,
                "sample_per_step": f"{per_step} decode tokens per step (of the 128 of a tg128 pass), context {PROMPT_LEN}+",
                "l2": "n/a (host memory)"})
    emit({
        "impl": "reference", "metric": "decode_tokens_per_s_tg128", "value": value, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * per_step / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": cfg,
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": base.kind,
                         "sample": cpu_sample_text(base, per_step, PROMPT_LEN) + ", per step"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


def run_reference_gpu(args):
    """The reference's own decode / prefill kernels (megakernel/kernel.cu, prefill.cu, compiled unmodified for sm_100a by
    oracle/build_oracle.py) through their stock launch_decode / launch_prefill_bf16 entry points on this GPU: pp520, then
    tg128 with the host token loop the reference's driver uses (megakernel/model.py:278-293)."""
    rank, local, _ = dist_env()
    if rank != 0:
        return
    from oracle.ref_kernels import RefDecoder, load_ref_lib      # test infrastructure, executed only by this arm
    lib = load_ref_lib()
    if lib is None or not torch.cuda.is_available():
        emit({"impl": "reference_gpu", "unavailable": "oracle/_ref/libref_megakernel.so was not built (needs the reference checkout at build time) or no GPU"})
        return
    torch.cuda.set_device(local)
    from luce_megakernel_b200 import model as M
    weights, _ = M.load_weights(seed=0, device_init=True)
    mine = M.Decoder(weights=weights, max_seq_len=MAX_SEQ, api="cabi")     # holds the weights and the pointer table only
    ref = RefDecoder(lib, mine, MAX_SEQ)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, M.VOCAB_SIZE, (PROMPT_LEN,), generator=g).to(torch.int32).cuda()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def tg128():
        ref.pos = PROMPT_LEN
        t = first
        for _ in range(GEN_LEN):
            t = ref.step(t)

    ref.reset()
    first = ref.prefill(ids)
    for _ in range(max(args.warmup, 1)):
        tg128()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        tg128()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    ref.reset(); ref.prefill(ids)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(5):
        ref.reset(); ref.prefill(ids)
    e1.record()
    torch.cuda.synchronize()
    pp_ms = e0.elapsed_time(e1) / 5
    value = GEN_LEN * args.steps / (ms * 1e-3)
    emit({
        "impl": "reference_gpu", "metric": "decode_tokens_per_s_tg128", "value": value, "unit": "tok/s", "n_gpus": 1,
        "steps": args.steps, "warmup": max(args.warmup, 1), "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": workload_config(1),
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 4 * GEN_LEN, "d2h_bytes_per_step": 4 * GEN_LEN,
                "api": "launch_decode per token with a host round trip, as the reference's Decoder.step() does"},
        "prefill": {"prompt_len": PROMPT_LEN, "ms": pp_ms, "tok_s": PROMPT_LEN / (pp_ms * 1e-3)},
        "gpu_launches": 2 * GEN_LEN * args.steps,
        "note": "reference kernels compiled from the checkout for sm_100a with NUM_BLOCKS=148 (megakernel/setup.py flags)",
    })


_RESULT_FD = None


NVFP4_NOMINAL_TFLOPS = 9000.0      # dense fp4 tensor peak of a B200 (nominal: the measured-peaks file has bf16 only)


def nvfp4_extras(MQ, M, weights, dec, q, prompt_dev, tg128_device, timed, g, args):
    """Single-GPU figures of the block-scaled tensor-core path (tcgen05.mma kind::mxf4nvf4): the GEMM on its own,
    the prefill with NVFP4 weights and activations, the decode variant that multiplies chunk images, and the batched
    step on NVFP4 weights.  `q` is the DecoderTS sharing dec's session state."""
    import ctypes
    from luce_megakernel_b200 import lib
    L = lib()
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = {}

    def quant(x):
        rows, cols = x.shape
        pk = torch.zeros(rows, cols // 2, dtype=torch.uint8, device="cuda")
        sc = torch.zeros((rows // 128) * (cols // 64) * 512, dtype=torch.uint8, device="cuda")
        ts = torch.zeros(4, dtype=torch.float32, device="cuda")
        if L.mk_quantize_nvfp4_tensor_scale(P(x), rows, cols, P(pk), P(sc), P(ts), stream()) != 0:
            raise SystemExit("quantiser failed")
        return pk, sc, ts

    gemms = []
    for (m, n, k) in ((8192, 7168, 1024), (8192, 1024, 3584), (8192, 8192, 8192)):
        a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        w = (torch.randn(n, k, device="cuda") * 0.05).to(torch.bfloat16)
        (apk, asc, ats), (wpk, wsc, wts) = quant(a), quant(w)
        c = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        f4 = lambda: L.mk_gemm_nvfp4_tn(P(apk), P(asc), P(ats), P(wpk), P(wsc), P(wts), P(c), None, m, n, k, stream())
        f16 = lambda: L.mk_gemm_bf16_tn(P(a), P(w), P(c), None, m, n, k, stream())
        for f in (f4, f16):
            for _ in range(3):
                f()
        us4 = timed(lambda: [f4() for _ in range(10)], 1) * 100.0
        us16 = timed(lambda: [f16() for _ in range(10)], 1) * 100.0
        tf4 = 2.0 * m * n * k / us4 / 1e6
        gemms.append({"m": m, "n": n, "k": k, "us": us4, "tflops": tf4, "frac_of_nominal_fp4_peak": tf4 / NVFP4_NOMINAL_TFLOPS,
                      "vs_measured_bf16_peak": tf4 / measured_bf16_peak(), "bf16_kernel_us": us16, "speedup_vs_bf16_kernel": us16 / us4})
        del a, w, apk, asc, wpk, wsc, c
    if L.mk_gemm_nvfp4_status() != 0:
        raise SystemExit("a bounded wait ran out in the NVFP4 GEMM")
    out["gemm"] = {"kernel": "gemm_nvfp4_tn_kernel: NVFP4 x NVFP4 -> bf16, 128 x 128 tiles, block scales in tensor memory",
                   "peak_note": f"fraction of the NOMINAL dense fp4 peak ({NVFP4_NOMINAL_TFLOPS:.0f} TFLOP/s); no fp4 peak was measured on this pool",
                   "shapes": gemms}

    # prefill with NVFP4 weights and NVFP4 activations, pp520 (into the shared session state) and 8192 tokens
    pf = []
    for S_ in (PROMPT_LEN, 8192):
        d4 = q if S_ == PROMPT_LEN else MQ.DecoderTS(weights, max_seq_len=S_ + 8)
        ids = prompt_dev if S_ == PROMPT_LEN else torch.randint(0, M.VOCAB_SIZE, (S_,), generator=g).to(torch.int32).cuda()

        def run(d=d4, x=ids):
            d._dn_states.zero_(); d._conv_bufs.zero_()
            return d.prefill(x)
        run(); run()
        ms_ = timed(lambda: [run() for _ in range(3)], 1) / 3
        pf.append({"prompt_len": S_, "ms": ms_, "tok_s": S_ / (ms_ * 1e-3)})
    if L.mk_prefill_status() != 0 or L.mk_gemm_nvfp4_status() != 0:
        raise SystemExit("a bounded wait ran out in the NVFP4 prefill")
    out["prefill"] = {"op": "mk_prefill_nvfp4_mma: every projection input quantised to NVFP4, block-scaled GEMMs; "
                            "attention, DeltaNet scan and norms as in the bf16 prefill", "runs": pf}

    # restore the bf16 prompt state, then the decode variant on the block-scaled tensor cores
    dec._position = 0
    dec._dn_states.zero_(); dec._conv_bufs.zero_()
    dec.prefill(prompt_dev)
    qm = MQ.DecoderMMA(weights, max_seq_len=MAX_SEQ, act_terms=4)
    qm.adopt_state(dec)
    for _ in range(3):
        tg128_device(qm)
    mm_ms = timed(lambda: tg128_device(qm), args.steps)
    if L.mk_device_status() != 0:
        raise SystemExit("device-side wait timed out during the tcgen05 NVFP4 decode")
    out["decode"] = {"op": "mk_decode_nvfp4_mma, activation expanded into 4 NVFP4 terms", "us_per_token": mm_ms * 1e3 / (GEN_LEN * args.steps),
                     "tok_s": GEN_LEN * args.steps / (mm_ms * 1e-3),
                     "note": "issue-bound: one tcgen05.cp / tcgen05.mma costs about 42 ns and a projection of K inputs needs K/32 of "
                             "them after the activation is known; the mma.sync variant (nvfp4_decode) is the faster NVFP4 decode"}
    del qm

    # batched step on NVFP4 weights (batch 8)
    bd = M.BatchDecoder(dec, 8, nvfp4_ts=True)
    prompts = [torch.randint(0, M.VOCAB_SIZE, (PROMPT_LEN,), generator=g).tolist() for _ in range(8)]
    runs = []
    for r in range(3):
        bd.reset()
        bd.prefill(prompts)
        runs.append(timed(lambda: bd.step_many(GEN_LEN), 1))
    t_ = sum(runs[1:]) / 2 / GEN_LEN
    out["decode_batch"] = {"batch_per_gpu": 8, "ms_per_step": t_, "tok_s": 8 / (t_ * 1e-3),
                           "note": "mk_decode_batch_nvfp4_ts: NVFP4 weights dequantised in registers for mma.sync; launch-bound like the bf16 step"}
    del bd
    return out


def protect_stdout():
    """Libraries print to stdout from native code (NCCL's version banner): keep fd 1 for the one JSON line and send
    everything else to stderr."""
    global _RESULT_FD
    if _RESULT_FD is None:
        sys.stdout.flush()
        _RESULT_FD = os.dup(1)
        os.dup2(2, 1)


def emit(obj):
    line = (json.dumps(obj) + "\n").encode()
    sys.stdout.flush()
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, line)


def cpu_state_dict(weights):
    """Rebuilds a transformers-style state dict (CPU tensors) from the packed device weights."""
    from luce_megakernel_b200.model import _DN_KEYS, _FA_KEYS
    sd = {"model.embed_tokens.weight": weights["embed_weight"].cpu(), "model.norm.weight": weights["final_norm_weight"].cpu()}
    for i, ld in enumerate(weights["layer_data"]):
        keys = _FA_KEYS if ld["type"] == 1 else _DN_KEYS
        for k, t in zip(keys, ld["ptrs"]):
            sd[f"model.layers.{i}.{k}"] = t.cpu()
    return sd


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference_gpu"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-long-prefill", action="store_true")
    ap.add_argument("--no-batch", action="store_true", help="skip the batch 8 / batch 16 decode figures")
    ap.add_argument("--no-nvfp4", action="store_true", help="skip the NVFP4 decode figure")
    ap.add_argument("--barrier", default="gloo", choices=["nccl", "gloo"],
                    help="process group for the timing barriers and the final reduction (N > 1); the data path has no "
                         "collective.  gloo by default: with an NCCL communicator alive in the process the persistent "
                         "decode kernel ran 0.7 % (rank 0) and 5.7 % (rank 1) slower on 2 GPUs, with gloo every rank runs "
                         "at its single-GPU speed")
    ap.add_argument("--no-sampler", action="store_true", help="do not run the nvidia-smi clock sampler beside the timed region")
    args = ap.parse_args()
    protect_stdout()
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "reference_gpu":
        return run_reference_gpu(args)

    rank, local, world = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device: the hot path has no CPU fallback")
    torch.cuda.set_device(local)
    use_dist = world > 1
    if use_dist:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if args.barrier == "gloo":
            dist.init_process_group("gloo")
        else:
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))

    from luce_megakernel_b200 import lib, model as M, replicas as R
    weights, _ = M.load_weights(seed=rank, device_init=True)
    dec = M.Decoder(weights=weights, max_seq_len=MAX_SEQ, api="cabi")
    g = torch.Generator().manual_seed(rank)
    prompt = torch.randint(0, M.VOCAB_SIZE, (PROMPT_LEN,), generator=g).tolist()
    pinned_tok = torch.empty(1, dtype=torch.int32).pin_memory()

    # prompt through the prefill op (not part of the timed tg128 region; timed separately below)
    prompt_dev = torch.tensor(prompt, dtype=torch.int32, device="cuda")
    first = dec.prefill(prompt_dev)

    def tg128_device(d=dec):
        d._position = PROMPT_LEN
        return d.step_many(first, GEN_LEN)          # ONE persistent launch: 128 steps, token fed back on the device

    def tg128_e2e():
        # reference-style public API: one call per token, token id from the host, result read back
        dec._position = PROMPT_LEN
        t = first
        for _ in range(GEN_LEN):
            pinned_tok[0] = t
            t = dec.step(int(pinned_tok[0]))
        return t

    def barrier():
        R.timing_barrier(torch.cuda.synchronize)

    def timed(fn, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        barrier()
        return e0.elapsed_time(e1)

    # the sampler starts with the warm-up (the same workload as the timed region) so that short runs, and runs where
    # eight ranks start nvidia-smi at once, still collect samples under load
    sampler = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ else 0)
    if not args.no_sampler:
        sampler.start()
    for _ in range(max(args.warmup, 3)):
        tg128_device()
    ms = timed(tg128_device, args.steps)
    clocks = sampler.stop() if not args.no_sampler else {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["not sampled"]}
    status = lib().mk_device_status()
    if status != 0:
        raise SystemExit(f"device-side wait timed out (status {status})")

    # end-to-end: host token in, host token out, per token (at most 3 steps to bound the run)
    e2e_steps = min(args.steps, 3)
    tg128_e2e()
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        tg128_e2e()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0

    # NVFP4 decode: every linear layer and the LM head as e2m1 in 16-element blocks with E4M3
    # block scales and an fp32 tensor scale, bf16 KV cache; same prompt state (bf16 prefill), then tg128
    nv_ms = 0.0
    nv_extra = None
    if not args.no_nvfp4:
        from luce_megakernel_b200 import model_nvfp4 as MQ
        q = MQ.DecoderTS(weights, max_seq_len=MAX_SEQ)
        q.adopt_state(dec)
        for _ in range(3):
            tg128_device(q)
        nv_ms = timed(lambda: tg128_device(q), args.steps)
        if lib().mk_device_status() != 0:
            raise SystemExit("device-side wait timed out during the NVFP4 decode")
        if world == 1:
            nv_extra = nvfp4_extras(MQ, M, weights, dec, q, prompt_dev, tg128_device, timed, g, args)
        del q
        weights.pop("nvfp4_mma", None)
        weights.pop("nvfp4_ts", None)

    # prefill pp520 (secondary figure): 3 warm-ups, then 10 timed calls of the prefill op
    def pp():
        dec._position = 0
        dec._dn_states.zero_(); dec._conv_bufs.zero_()
        return dec.prefill(prompt_dev)
    for _ in range(3):
        pp()
    pp_ms = timed(pp, 10) / 10
    # the same prompt replayed from the CUDA graph Decoder.prefill_graphed keeps per prompt length (reset included)
    dec._position = 0
    dec.prefill_graphed(prompt_dev)
    pp_graph = dec._prefill_graphs[PROMPT_LEN]["graph"]
    for _ in range(3):
        pp_graph.replay()
    pp_graph_ms = timed(pp_graph.replay, 10) / 10

    # dense prefill at 8192 and 32768 tokens, single GPU only: 1 warm-up + 2 timed calls
    long_pp = []
    if world == 1 and not args.no_long_prefill:
        import ctypes
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for S_, sparse in ((8192, False), (32768, False), (65536, True)):
            d2 = M.Decoder(weights=weights, max_seq_len=S_ + 8, api="cabi")
            ids = torch.randint(0, M.VOCAB_SIZE, (S_,), generator=g).to(torch.int32).cuda()
            # 128 x 128 blocks, sink block 0, 4-block window, top 10 % by pooled q.k
            lib().mk_prefill_set_block_sparse(1 if sparse else 0, ctypes.c_double(0.10), 4, 1)
            try:
                d2.prefill(ids)
                torch.cuda.synchronize()
                p0.record()
                for _ in range(2):
                    d2._position = 0
                    d2.prefill_async(ids)
                p1.record()
                torch.cuda.synchronize()
            finally:
                lib().mk_prefill_set_block_sparse(0, ctypes.c_double(0.10), 4, 1)
            long_pp.append((S_, p0.elapsed_time(p1) / 2, sparse))
            del d2
        if lib().mk_device_status() != 0 or lib().mk_prefill_status() != 0:
            raise SystemExit("device-side wait timed out during the long prefill")

    # batched decode (BASELINE.json configs[3] and [4]): batch 8 and 16 per GPU, a pp520 prompt per sequence, then tg128
    # with the tokens fed back on the device; 1 warm-up run + 2 timed runs of 128 steps
    batch_ms = []
    if not args.no_batch:
        for B_ in (8, 16):
            bd = M.BatchDecoder(dec, B_)
            prompts = [torch.randint(0, M.VOCAB_SIZE, (PROMPT_LEN,), generator=g).tolist() for _ in range(B_)]
            runs = []
            for r in range(3):
                bd.reset()
                bd.prefill(prompts)
                runs.append(timed(lambda: bd.step_many(GEN_LEN), 1))
            batch_ms.append(sum(runs[1:]) / 2 / GEN_LEN)
            del bd
        if lib().mk_prefill_status() != 0:
            raise SystemExit("device-side wait timed out during the batched decode")

    # every rank's device time for the timed tg128 region (the whole-job figure uses the slowest), plus the other timings
    tokens = GEN_LEN * args.steps
    per_rank = R.gather_results(R.ReplicaResult(tokens=tokens, seconds=ms * 1e-3))
    agg = R.aggregate(per_rank)
    t_all = torch.tensor([e2e_s, pp_ms, nv_ms] + (batch_ms or [0.0, 0.0]), dtype=torch.float64, device="cuda")
    if use_dist:
        if args.barrier == "gloo":
            t_all = t_all.cpu()
        dist.all_reduce(t_all, op=dist.ReduceOp.MAX)
    e2e_max, pp_max, nv_max = float(t_all[0]), float(t_all[1]), float(t_all[2])
    batch_max = [float(t_all[3]), float(t_all[4])]

    if rank == 0:
        ms_max = agg["seconds"] * 1e3
        value = agg["tokens_per_s"]
        us_per_launch_step = ms_max * 1e3 / tokens
        avg_ctx = PROMPT_LEN + 1 + (GEN_LEN - 1) / 2.0
        peak, peak_kind = measured_hbm_peak()
        # one launch of the persistent kernel runs GEN_LEN steps: bytes and duration per launch are per 128 tokens
        bytes_per_launch = GEN_LEN * algorithmic_bytes_per_token(avg_ctx)
        achieved = bytes_per_launch / (GEN_LEN * us_per_launch_step * 1e-6) / 1e9
        out = {
            "metric": "decode_tokens_per_s_tg128", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": f"of {peak_kind}", "traffic": GEN_LEN * TRAFFIC_BYTES_PER_LAUNCH,
                         "algorithmic_bytes_per_launch": bytes_per_launch,
                         "algorithmic_bytes_per_token": algorithmic_bytes_per_token(avg_ctx),
                         "us_per_launch": GEN_LEN * us_per_launch_step, "us_per_token": us_per_launch_step,
                         "tokens_per_launch": GEN_LEN, "kernel": "decode_megakernel_bf16",
                         "traffic_note": "ncu capture of a 4-step launch at context 520: bytes per step times the 128 steps of a launch"},
            "per_rank_us_per_token": [r.seconds * 1e6 / r.tokens for r in per_rank],
            "e2e": {"value": world * GEN_LEN * e2e_steps / e2e_max, "unit": "tok/s",
                    "h2d_bytes_per_step": 4 * GEN_LEN, "d2h_bytes_per_step": 4 * GEN_LEN,
                    "api": "Decoder.step(): one mk_decode_step_host call per token (launch_decode + the token returned through mapped pinned memory), host token in, host token out"},
            "prefill": {"prompt_len": PROMPT_LEN, "ms": pp_max, "tok_s": world * PROMPT_LEN / (pp_max * 1e-3),
                        "tflops_algorithmic": PREFILL_TFLOP_PP520 / (pp_max * 1e-3),
                        "frac_of_bf16_peak": PREFILL_TFLOP_PP520 / (pp_max * 1e-3) / measured_bf16_peak(),
                        "graph_replay_ms": pp_graph_ms,
                        "note": "prefill_bf16 op: persistent tcgen05/TMEM GEMMs fed by TMA, chunk-64 DeltaNet scan on "
                                "mma.sync, causal GQA flash attention on tcgen05/TMEM"},
            "gpu_launches": world * args.steps,
            "clocks": clocks,
        }
        if nv_max > 0:
            nv_us = nv_max * 1e3 / tokens
            nv_bytes = algorithmic_bytes_per_token(avg_ctx, nvfp4=True)
            out["nvfp4_decode"] = {
                "format": "e2m1 in 16-element blocks, E4M3 block scales, fp32 scale per matrix; all linear layers and the LM head; bf16 KV cache",
                "tok_s": world * 1e6 / nv_us, "us_per_token": nv_us, "vs_bf16": us_per_launch_step / nv_us,
                "roofline": {"bound": "hbm", "achieved": nv_bytes / (nv_us * 1e-6) / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": nv_bytes / (nv_us * 1e-6) / 1e9 / peak, "algorithmic_bytes_per_token": nv_bytes},
                "note": "mk_decode_nvfp4_ts: 128 steps per launch; one dependent phase is one ring chunk per CTA, so the "
                        "step is bound by the 120 activation exchanges, not by bytes"}
            if nv_extra:
                out["nvfp4_tensor_core"] = nv_extra
        if batch_ms:
            hbm, _ = measured_hbm_peak()
            out["decode_batch"] = [
                {"batch_per_gpu": B_, "ms_per_step": t_, "tok_s": world * B_ / (t_ * 1e-3),
                 "hbm_gbs_algorithmic": batch_step_bytes(B_, avg_ctx) / (t_ * 1e-3) / 1e9,
                 "frac_of_hbm_peak": batch_step_bytes(B_, avg_ctx) / (t_ * 1e-3) / 1e9 / hbm,
                 "note": "mk_decode_batch_many: every sequence has its own pp520 prompt and state; 131 kernels per step"}
                for B_, t_ in zip((8, 16), batch_max)]
        if world == 1 and long_pp:
            out["prefill_long"] = [
                {"prompt_len": S_, "attention": "block-sparse 128x128: sink 1 + window 4 + top 10%" if sp_ else "dense causal",
                 "ms": ms_, "tok_s": S_ / (ms_ * 1e-3),
                 "tflops_algorithmic": prefill_tflop(S_, sp_) / (ms_ * 1e-3),
                 "frac_of_bf16_peak": prefill_tflop(S_, sp_) / (ms_ * 1e-3) / measured_bf16_peak(),
                 "tflops_dense_equivalent": prefill_tflop(S_) / (ms_ * 1e-3)} for S_, ms_, sp_ in long_pp]
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline_in_child() or cpu_baseline_in_process(weights)
        emit(out)
    if use_dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
