"""Builds the checker libraries under oracle/ (test infrastructure, never part of the product).

  oracle/libnvfp4_oracle.so   plain-C restatement of the reference's NVFP4 quantisers (gcc)
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


def build_all(force=False):
    build_nvfp4(force)


if __name__ == "__main__":
    build_all(True)
    print("built", NVFP4_LIB)
