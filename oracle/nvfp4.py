"""ctypes front end of oracle/nvfp4_oracle.c (the CPU restatement of the reference's NVFP4
quantisers).  TEST INFRASTRUCTURE ONLY."""
import ctypes

import numpy as np

from . import build_oracle

_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build_oracle.build_nvfp4())
        _lib.mk_oracle_e4m3_to_f32.restype = ctypes.c_float
        _lib.mk_oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        _lib.mk_oracle_f32_to_e4m3.restype = ctypes.c_uint8
        _lib.mk_oracle_f32_to_e4m3.argtypes = [ctypes.c_float]
        _lib.mk_oracle_f32_to_e2m1.restype = ctypes.c_uint8
        _lib.mk_oracle_f32_to_e2m1.argtypes = [ctypes.c_float]
        _lib.mk_oracle_scale_index_b.restype = ctypes.c_size_t
        _lib.mk_oracle_scale_index_b.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
        _lib.mk_oracle_f32_to_f16.restype = ctypes.c_uint16
        _lib.mk_oracle_f32_to_f16.argtypes = [ctypes.c_float]
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _bf16_bits(w):
    """torch bf16 tensor or uint16 array -> contiguous uint16 numpy array of bf16 bit patterns."""
    if isinstance(w, np.ndarray):
        return np.ascontiguousarray(w.astype(np.uint16))
    import torch
    return np.ascontiguousarray(w.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16))


def quantize_a(w, group_size=32):
    bits = _bf16_bits(w)
    rows, cols = bits.shape
    packed = np.zeros((rows, cols // 2), np.uint8)
    scales = np.zeros((rows, cols // group_size), np.uint16)      # fp16 bit patterns
    lib().mk_oracle_quantize_a(_p(bits), rows, cols, group_size, _p(packed), _p(scales))
    return packed, scales


def quantize_b(w):
    bits = _bf16_bits(w)
    rows, cols = bits.shape
    assert rows % 128 == 0 and cols % 64 == 0
    packed = np.zeros((rows, cols // 2), np.uint8)
    scales = np.zeros((rows // 128) * (cols // 64) * 512, np.uint8)
    lib().mk_oracle_quantize_b(_p(bits), rows, cols, _p(packed), _p(scales))
    return packed, scales


def dequantize_a(packed, scales, group_size=32):
    rows, half = packed.shape
    out = np.zeros((rows, half * 2), np.float32)
    lib().mk_oracle_dequantize_a(_p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scales)), rows, half * 2,
                                 group_size, _p(out))
    return out


def dequantize_b(packed, scales):
    rows, half = packed.shape
    out = np.zeros((rows, half * 2), np.float32)
    lib().mk_oracle_dequantize_b(_p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scales)), rows, half * 2, _p(out))
    return out


def quantize_ts(w):
    """16-blocks, E4M3 block scales (layout of format B), f32 per-tensor scale.  Returns packed, scales, scale."""
    bits = _bf16_bits(w)
    rows, cols = bits.shape
    assert rows % 128 == 0 and cols % 64 == 0
    packed = np.zeros((rows, cols // 2), np.uint8)
    scales = np.zeros((rows // 128) * (cols // 64) * 512, np.uint8)
    ts = np.zeros(1, np.float32)
    lib().mk_oracle_quantize_ts(_p(bits), rows, cols, _p(packed), _p(scales), _p(ts))
    return packed, scales, ts


def dequantize_ts(packed, scales, tensor_scale):
    rows, half = packed.shape
    out = np.zeros((rows, half * 2), np.float32)
    lib().mk_oracle_dequantize_ts(_p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scales)),
                                  ctypes.c_float(float(np.asarray(tensor_scale).reshape(-1)[0])), rows, half * 2, _p(out))
    return out
