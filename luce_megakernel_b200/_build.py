"""In-tree build of the native libraries (sm_100a only).

  libluce_megakernel_b200.so   C-ABI core: CUDA kernels + launchers (no torch types)
  qwen35_megakernel_bf16_C.so  PyTorch op surface over the C ABI (same op schemas as the
                               reference extension, megakernel/torch_bindings.cpp:568-677)

Both are built next to this file so that they travel with the source tree.
"""
import glob
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
CORE_LIB = os.path.join(HERE, "libluce_megakernel_b200.so")
TORCH_EXT = os.path.join(HERE, "qwen35_megakernel_bf16_C.so")

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
              "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"] + os.environ.get("MK_NVCC_EXTRA", "").split()


def _newer(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: %s\n%s" % (" ".join(cmd), r.stdout))
    return r.stdout


def build_core(force=False, verbose=False):
    cus = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = cus + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(HERE, "..", "include", "*.h")) + [os.path.abspath(__file__)]
    if not force and not _newer(CORE_LIB, deps):
        return CORE_LIB
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    objs = []
    for cu in cus:
        obj = os.path.join(CSRC, os.path.basename(cu)[:-3] + ".o")
        if force or _newer(obj, deps):
            # *_fastmath.cu restate reference code that the reference compiles with --use_fast_math
            extra = ["--use_fast_math"] if cu.endswith("_fastmath.cu") else []
            out = _run([nvcc] + NVCC_FLAGS + extra + (["-Xptxas", "-v"] if verbose else []) + ["-c", cu, "-o", obj])
            if verbose:
                print(out)
        objs.append(obj)
    _run([nvcc, "-shared", "-o", CORE_LIB] + objs + ["-lcuda"])
    return CORE_LIB


def build_torch_ext(force=False):
    src = os.path.join(CSRC, "torch_ops.cpp")
    if not force and not _newer(TORCH_EXT, [src, CORE_LIB]):
        return TORCH_EXT
    import torch
    from torch.utils import cpp_extension as ce
    inc = ce.include_paths(device_type="cuda") if "device_type" in ce.include_paths.__code__.co_varnames else ce.include_paths(cuda=True)
    tlib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-DTORCH_EXTENSION_NAME=qwen35_megakernel_bf16_C",
           "-D_GLIBCXX_USE_CXX11_ABI=%d" % int(torch._C._GLIBCXX_USE_CXX11_ABI),
           "-I" + sysconfig.get_paths()["include"], "-I/usr/local/cuda/include"]
    cmd += ["-I" + i for i in inc]
    cmd += [src, "-o", TORCH_EXT, "-L" + tlib, "-L" + HERE, "-lluce_megakernel_b200",
            "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
            "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + tlib]
    _run(cmd)
    return TORCH_EXT


def build_all(force=False, verbose=False):
    build_core(force=force, verbose=verbose)
    build_torch_ext(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built", CORE_LIB, TORCH_EXT)
