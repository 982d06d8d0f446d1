"""Builds the checker libraries under oracle/ (test infrastructure, never part of the product).

  oracle/libnvfp4_oracle.so        plain-C restatement of the reference's NVFP4 quantisers (gcc)
  oracle/_ref/libref_megakernel.so the reference's own decode and prefill kernels (megakernel/kernel.cu,
                                   megakernel/prefill.cu), compiled for sm_100a from the sources where they lie
                                   in the reference checkout, with the flags of megakernel/setup.py and
                                   NUM_BLOCKS=148.  Built only where the checkout is present; the GPU tests use
                                   it as a second pin (token identity against the reference kernels) and skip
                                   when it is absent.  No reference source is copied.
"""
import os
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


REF_DIR = os.environ.get("LUCE_REFERENCE_DIR", "/root/reference")
REF_LIB = os.path.join(HERE, "_ref", "libref_megakernel.so")


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
    cmd = [nvcc, "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "--use_fast_math", "-std=c++17",
           "-DNUM_BLOCKS=148", "-DBLOCK_SIZE=512", "-DLM_NUM_BLOCKS=512", "-DLM_BLOCK_SIZE=256",
           "-DMEGAKERNEL_DN_PHASE2_WMMA=0", "-DTARGET_SM=100", "-shared", "-Xcompiler", "-fPIC",
           *srcs, "-lcublas", "-o", REF_LIB]
    subprocess.check_call(cmd)
    return REF_LIB


def build_all(force=False):
    build_nvfp4(force)
    build_ref(force)


if __name__ == "__main__":
    build_all(True)
    print("built", NVFP4_LIB, REF_LIB if os.path.exists(REF_LIB) else "(no reference checkout: _ref skipped)")
