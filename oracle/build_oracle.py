"""Builds the checker libraries under oracle/ (test infrastructure, never part of the product).

  oracle/libnvfp4_oracle.so        plain-C restatement of the reference's NVFP4 quantisers (gcc)
  oracle/_ref/libref_nvfp4_quant.so the reference's two NVFP4 weight quantiser kernels with their launchers
                                   (megakernel/kernel_gb10_nvfp4.cu: quantize_fp4_code, quantize_nvfp4_kernel,
                                   quantize_nvfp4_lm_kernel, launch_quantize_nvfp4_out, launch_quantize_nvfp4_lm_out),
                                   cut out of the checkout at build time into a generated translation unit under
                                   oracle/_ref/ (the file as a whole refuses to compile below sm_120) and compiled
                                   for sm_100a with the reference's own flags, --use_fast_math included.
  oracle/_ref/libref_drafter_select.so steps 2-4 of the reference's prompt compressor (dflash/src/qwen3_drafter.cpp),
                                   cut out at build time and wrapped in one C function (g++, host only).
  oracle/_ref/libref_sampler.so    the CPU sampler chain of the reference's speculative-decoding driver (SamplerCfg and
                                   sample_logits, dflash/test/test_dflash.cpp), cut out at build time and wrapped
                                   in one C function (g++, host only).
  oracle/_ref/libref_block_select.so the reference's host-side block selection (dflash/src/flashprefill_select.cpp),
                                   compiled where it lies together with oracle/ref_block_select_wrap.cpp (g++).
  oracle/_ref/libref_megakernel.so the reference's own decode and prefill kernels (megakernel/kernel.cu,
                                   megakernel/prefill.cu), compiled for sm_100a from the sources where they lie
                                   in the reference checkout, with the flags of megakernel/setup.py and
                                   NUM_BLOCKS=148.  Built only where the checkout is present; the GPU tests use
                                   it as a second pin (token identity against the reference kernels) and skip
                                   when it is absent.  No reference source is copied.
"""
import json
import os
import re
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
NVFP4_LIB = os.path.join(HERE, "libnvfp4_oracle.so")


def _newer(target, src):
    return not os.path.exists(target) or os.path.getmtime(src) > os.path.getmtime(target)


def build_nvfp4(force=False):
    src = os.path.join(HERE, "nvfp4_oracle.c")
    if force or _newer(NVFP4_LIB, src):
        # -ffp-contract=off: every multiply and divide must round on its own, like the reference kernels
        subprocess.check_call(["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
                               "-o", NVFP4_LIB, src, "-lm"])
    return NVFP4_LIB


def _reference_dir():
    """The reference checkout: $LUCE_REFERENCE_DIR, else `reference_path` of the BASELINE.json next to this
    package; None when neither names an existing directory (the prebuilt files are then used as they are)."""
    cand = os.environ.get("LUCE_REFERENCE_DIR")
    if not cand:
        try:
            cand = json.load(open(os.path.join(HERE, "..", "BASELINE.json"))).get("reference_path")
        except (OSError, ValueError):
            cand = None
    return cand if cand and os.path.isdir(cand) else None


REF_DIR = _reference_dir() or ""
REF_LIB = os.path.join(HERE, "_ref", "libref_megakernel.so")
REF_QUANT_LIB = os.path.join(HERE, "_ref", "libref_nvfp4_quant.so")
# flags of megakernel/setup.py:49-59 (the arch is this build's)
REF_NVCC_FLAGS = ["-O3", "-gencode", "arch=compute_100a,code=sm_100a", "--use_fast_math", "-std=c++17",
                  "-DNUM_BLOCKS=148", "-DBLOCK_SIZE=512", "-DLM_NUM_BLOCKS=512", "-DLM_BLOCK_SIZE=256",
                  "-DMEGAKERNEL_DN_PHASE2_WMMA=0", "-DTARGET_SM=100"]


def build_ref(force=False):
    """nvcc on the reference's two source files (flags: megakernel/setup.py:40-60).  Returns the path or
    None when the reference checkout or nvcc is missing."""
    srcs = [os.path.join(REF_DIR, "megakernel", f) for f in ("kernel.cu", "prefill.cu")]
    if not all(os.path.exists(s) for s in srcs):
        return REF_LIB if os.path.exists(REF_LIB) else None
    if not force and os.path.exists(REF_LIB) and all(os.path.getmtime(s) <= os.path.getmtime(REF_LIB) for s in srcs):
        return REF_LIB
    os.makedirs(os.path.dirname(REF_LIB), exist_ok=True)
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    cmd = [nvcc, *REF_NVCC_FLAGS, "-shared", "-Xcompiler", "-fPIC", *srcs, "-lcublas", "-o", REF_LIB]
    subprocess.check_call(cmd)
    return REF_LIB


def _cut_definition(text, start_pattern):
    """The definition that starts at the first match of start_pattern, up to its closing brace."""
    m = re.search(start_pattern, text, re.M)
    if not m:
        raise RuntimeError("not found in the reference source: " + start_pattern)
    i = text.index("{", m.end())
    depth, j = 0, i
    while True:
        depth += {"{": 1, "}": -1}.get(text[j], 0)
        j += 1
        if depth == 0:
            return text[m.start():j]


def build_ref_quant(force=False):
    """The reference's NVFP4 quantisers as the reference builds them.  Returns the library path, or None when
    neither the checkout nor a prebuilt library is there."""
    src = os.path.join(REF_DIR, "megakernel", "kernel_gb10_nvfp4.cu")
    if not os.path.exists(src):
        return REF_QUANT_LIB if os.path.exists(REF_QUANT_LIB) else None
    if not force and os.path.exists(REF_QUANT_LIB) and os.path.getmtime(src) <= os.path.getmtime(REF_QUANT_LIB) \
            and os.path.getmtime(__file__) <= os.path.getmtime(REF_QUANT_LIB):
        return REF_QUANT_LIB
    os.makedirs(os.path.dirname(REF_QUANT_LIB), exist_ok=True)
    text = open(src).read()
    parts = ["// GENERATED at build time from the reference checkout (never committed): the two NVFP4 weight\n"
             "// quantisers of megakernel/kernel_gb10_nvfp4.cu with their launchers, nothing else of that file.\n"
             "#include <cuda_bf16.h>\n#include <cuda_fp8.h>\n#include <cuda_fp4.h>\n#include <cuda_fp16.h>\n"
             "#include <cuda_runtime.h>\n#include <stdint.h>\n"]
    parts += re.findall(r"^constexpr int LM_SCALE_(?:ROWS_PER_TILE|COLS_PER_TILE|BLOCK_K|K_PER_TILE|THREADS) = [^;]*;", text, re.M)
    parts.append(_cut_definition(text, r"^__device__ __forceinline__ unsigned int quantize_fp4_code\("))
    parts.append(_cut_definition(text, r"^__global__ void quantize_nvfp4_kernel\("))
    parts.append(_cut_definition(text, r"^__global__ void __launch_bounds__\(LM_SCALE_THREADS\)\s*quantize_nvfp4_lm_kernel\("))
    parts.append(_cut_definition(text, r'^extern "C" void launch_quantize_nvfp4_out\('))
    parts.append(_cut_definition(text, r'^extern "C" void launch_quantize_nvfp4_lm_out\('))
    gen = os.path.join(HERE, "_ref", "ref_nvfp4_quant_gen.cu")
    with open(gen, "w") as f:
        f.write("\n\n".join(parts) + "\n")
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    subprocess.check_call([nvcc, *REF_NVCC_FLAGS, "-shared", "-Xcompiler", "-fPIC", gen, "-o", REF_QUANT_LIB])
    return REF_QUANT_LIB


REF_DRAFTER_LIB = os.path.join(HERE, "_ref", "libref_drafter_select.so")


def build_ref_drafter(force=False):
    """Steps 2-4 of the reference's drafter_score_and_compress (dflash/src/qwen3_drafter.cpp: mean over the lookahead,
    average-pool smoothing, chunk top-K, span merge) -- plain C++ on std::vector, cut out of the checkout at build time
    between its own section comments into a generated translation unit under oracle/_ref/ and wrapped in one C
    function.  (Step 1, the forward pass, needs ggml and another model.)  Returns the library path or None."""
    src = os.path.join(REF_DIR, "dflash", "src", "qwen3_drafter.cpp")
    if not os.path.exists(src):
        return REF_DRAFTER_LIB if os.path.exists(REF_DRAFTER_LIB) else None
    if not force and os.path.exists(REF_DRAFTER_LIB) and os.path.getmtime(src) <= os.path.getmtime(REF_DRAFTER_LIB) \
            and os.path.getmtime(__file__) <= os.path.getmtime(REF_DRAFTER_LIB):
        return REF_DRAFTER_LIB
    os.makedirs(os.path.dirname(REF_DRAFTER_LIB), exist_ok=True)
    text = open(src).read()
    a = text.index("2. Mean over lookahead")
    a = text.rindex("\n", 0, a) + 1
    b = text.index("auto t2 = std::chrono", a)
    body = text[a:b]
    gen = os.path.join(HERE, "_ref", "ref_drafter_select_gen.cpp")
    with open(gen, "w") as f:
        f.write("// GENERATED at build time from the reference checkout (never committed): steps 2-4 of\n"
                "// drafter_score_and_compress in dflash/src/qwen3_drafter.cpp, wrapped in one C function.\n"
                "#include <algorithm>\n#include <cstdint>\n#include <utility>\n#include <vector>\n"
                'extern "C" int ref_drafter_select(const float* rm, int n_lookahead, int S, float keep_ratio, int chunk_size,\n'
                "                                  int pool_kernel, const int32_t* ids_in, int32_t* out_ids) {\n"
                "    std::vector<float> running_max(rm, rm + (size_t)n_lookahead * S);\n"
                "    std::vector<int32_t> ids(ids_in, ids_in + S);\n"
                + body +
                "    for (size_t i = 0; i < out.size(); ++i) out_ids[i] = out[i];\n"
                "    return (int)out.size();\n}\n")
    subprocess.check_call(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", gen, "-o", REF_DRAFTER_LIB])
    return REF_DRAFTER_LIB


REF_SAMPLER_LIB = os.path.join(HERE, "_ref", "libref_sampler.so")


def build_ref_sampler(force=False):
    """SamplerCfg + sample_logits of the reference's driver (dflash/test/test_dflash.cpp: plain C++ on std containers
    inside a 3 700-line program that needs ggml): the two definitions are cut out of the checkout at build time into a
    generated translation unit under oracle/_ref/ and wrapped in one C function that seeds a std::mt19937_64 and
    draws n times.  Returns the library path or None."""
    src = os.path.join(REF_DIR, "dflash", "test", "test_dflash.cpp")
    if not os.path.exists(src):
        return REF_SAMPLER_LIB if os.path.exists(REF_SAMPLER_LIB) else None
    if not force and os.path.exists(REF_SAMPLER_LIB) and not _newer(REF_SAMPLER_LIB, src) and not _newer(REF_SAMPLER_LIB, __file__):
        return REF_SAMPLER_LIB
    os.makedirs(os.path.dirname(REF_SAMPLER_LIB), exist_ok=True)
    text = open(src).read()
    a = text.index("struct SamplerCfg {")
    b = text.index("static bool parse_sampler_token", a)
    body = text[a:b]
    gen = os.path.join(HERE, "_ref", "ref_sampler_gen.cpp")
    with open(gen, "w") as f:
        f.write("// GENERATED at build time from the reference checkout (never committed): SamplerCfg and sample_logits of\n"
                "// dflash/test/test_dflash.cpp, wrapped in one C function.\n"
                "#include <algorithm>\n#include <cmath>\n#include <cstdint>\n#include <random>\n#include <unordered_set>\n"
                "#include <utility>\n#include <vector>\n"
                + body +
                'extern "C" int ref_sample_logits(const float* logits, int vocab, float temp, float top_p, int top_k, float rep_pen,\n'
                "                                 const int32_t* history, int n_history, unsigned long long seed, int n_draws,\n"
                "                                 int32_t* out) {\n"
                "    SamplerCfg cfg; cfg.temp = temp; cfg.top_p = top_p; cfg.top_k = top_k; cfg.rep_pen = rep_pen; cfg.seed = seed;\n"
                "    std::vector<int32_t> hist(history, history + n_history);\n"
                "    std::mt19937_64 rng; rng.seed(seed);\n"
                "    for (int i = 0; i < n_draws; ++i) out[i] = sample_logits(logits, vocab, cfg, hist, rng);\n"
                "    return n_draws;\n}\n")
    subprocess.check_call(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", gen, "-o", REF_SAMPLER_LIB])
    return REF_SAMPLER_LIB


REF_BLOCK_SELECT_LIB = os.path.join(HERE, "_ref", "libref_block_select.so")


def build_ref_block_select(force=False):
    """The reference's block_select_host (dflash/src/flashprefill_select.cpp:27-84): plain C++ with no dependency,
    compiled from the checkout together with the C wrapper of this folder.  Returns the library path or None."""
    src = os.path.join(REF_DIR, "dflash", "src", "flashprefill_select.cpp")
    wrap = os.path.join(HERE, "ref_block_select_wrap.cpp")
    if not os.path.exists(src):
        return REF_BLOCK_SELECT_LIB if os.path.exists(REF_BLOCK_SELECT_LIB) else None
    if not force and os.path.exists(REF_BLOCK_SELECT_LIB) and not _newer(REF_BLOCK_SELECT_LIB, src) \
            and not _newer(REF_BLOCK_SELECT_LIB, wrap):
        return REF_BLOCK_SELECT_LIB
    os.makedirs(os.path.dirname(REF_BLOCK_SELECT_LIB), exist_ok=True)
    subprocess.check_call(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", wrap, src, "-o", REF_BLOCK_SELECT_LIB])
    return REF_BLOCK_SELECT_LIB


def build_all(force=False):
    build_nvfp4(force)
    build_ref(force)
    build_ref_quant(force)
    build_ref_drafter(force)
    build_ref_block_select(force)
    build_ref_sampler(force)


if __name__ == "__main__":
    build_all(True)
    print("built", NVFP4_LIB, REF_LIB if os.path.exists(REF_LIB) else "(no reference checkout: _ref skipped)")
