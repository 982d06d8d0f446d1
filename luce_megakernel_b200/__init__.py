"""B200-native (sm_100a) decode / prefill hot path of the Qwen3.5-0.8B hybrid model.

The product is the C-ABI library `libluce_megakernel_b200.so` (declared in
include/luce_megakernel_b200.h) and the PyTorch op surface built over it.  This package
only loads them; it has no CPU fallback and raises when the native library is missing.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
CORE_LIB_PATH = os.path.join(_HERE, "libluce_megakernel_b200.so")
TORCH_EXT_PATH = os.path.join(_HERE, "qwen35_megakernel_bf16_C.so")

_lib = None
_ops_loaded = False


class NativeLibraryMissing(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """The C-ABI core library.  Raises NativeLibraryMissing if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(CORE_LIB_PATH):
            raise NativeLibraryMissing(
                f"{CORE_LIB_PATH} is missing: run `python -m luce_megakernel_b200._build` "
                "(there is no CPU or PyTorch fallback for the hot path)")
        _lib = ctypes.CDLL(CORE_LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        _lib.mk_last_error_string.restype = ctypes.c_char_p
    return _lib


def load_ops():
    """Registers torch.ops.qwen35_megakernel_bf16_C.* (the reference's op namespace)."""
    global _ops_loaded
    if not _ops_loaded:
        import torch
        lib()
        if not os.path.exists(TORCH_EXT_PATH):
            raise NativeLibraryMissing(f"{TORCH_EXT_PATH} is missing: run `python -m luce_megakernel_b200._build`")
        torch.ops.load_library(TORCH_EXT_PATH)
        _ops_loaded = True
    import torch
    return torch.ops.qwen35_megakernel_bf16_C


def last_error() -> str:
    return lib().mk_last_error_string().decode()
