"""NVFP4 x NVFP4 GEMM on the block-scaled tensor-core path against the CPU restatement of the format.

Both operands are quantised by the library (bit-exact to oracle/nvfp4.py, see test_nvfp4.py), dequantised on the
CPU by the oracle, and multiplied in float64: the kernel's result must be that product rounded to bf16.  The
products code x scale x code x scale are exact in f32 and the block sums short, so the only rounding that matters is
the final bf16 one (2^-8 relative) plus f32 accumulation order (bounded by K * 2^-24 of the absolute row sums).
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import nvfp4

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _quantize(lib, x):
    """bf16 [rows, cols] (rows % 128 == 0) -> packed, tiled scales, tensor scale (device)."""
    rows, cols = x.shape
    pk = torch.zeros(rows, cols // 2, dtype=torch.uint8, device="cuda")
    sc = torch.zeros((rows // 128) * (cols // 64) * 512, dtype=torch.uint8, device="cuda")
    ts = torch.zeros(4, dtype=torch.float32, device="cuda")
    assert lib.mk_quantize_nvfp4_tensor_scale(_p(x), rows, cols, _p(pk), _p(sc), _p(ts), _stream()) == 0
    return pk, sc, ts


def _dequant_cpu(pk, sc, ts):
    return nvfp4.dequantize_ts(pk.cpu().numpy(), sc.cpu().numpy(), ts[:1].cpu().numpy()).astype(np.float64)


def _rand(rows, cols, seed, gain=1.0, outliers=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g) * gain
    if outliers:                                   # a few large entries: block scales then span the E4M3 range
        idx = torch.randint(0, rows * cols, (rows * cols // 97,), generator=g)
        x.view(-1)[idx] *= 40.0
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K,gain,outliers,residual", [
    (128, 128, 256, 1.0, False, False),            # one tile, one ring stage
    (128, 128, 1024, 1.0, False, False),           # one tile, four stages
    (256, 1024, 1024, 0.05, True, False),
    (200, 512, 2048, 1.0, True, True),             # ragged M: rows 200..255 are not stored
    (520, 3584, 1024, 3.0, False, True),           # the gate / up projection of a 520-token prompt
    (640, 1024, 3584, 1.0, True, False),           # the down projection: 14 stages, ring wraps
    (4096, 6144, 1024, 1.0, False, False),         # more tiles than SMs: persistent loop, both accumulator buffers
])
def test_gemm_nvfp4_matches_dequantised_product(M, N, K, gain, outliers, residual):
    import luce_megakernel_b200 as L
    lib = L.lib()
    lib.mk_last_error_string.restype = ctypes.c_char_p
    mp = (M + 127) // 128 * 128
    a = torch.zeros(mp, K, dtype=torch.bfloat16)
    a[:M] = _rand(M, K, 11 + M, gain, outliers)
    w = _rand(N, K, 13 + N, 0.03, outliers)
    a, w = a.cuda(), w.cuda()
    apk, asc, ats = _quantize(lib, a)
    wpk, wsc, wts = _quantize(lib, w)
    r = _rand(M, N, 5, 2.0).cuda() if residual else None
    c = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = lib.mk_gemm_nvfp4_tn(_p(apk), _p(asc), _p(ats), _p(wpk), _p(wsc), _p(wts), _p(c),
                              _p(r) if residual else None, M, N, K, _stream())
    assert rc == 0, lib.mk_last_error_string().decode()
    torch.cuda.synchronize()
    assert lib.mk_gemm_nvfp4_status() == 0
    ad, wd = _dequant_cpu(apk, asc, ats)[:M], _dequant_cpu(wpk, wsc, wts)
    ref = ad @ wd.T
    mag = np.abs(ad) @ np.abs(wd).T
    if residual:
        ref = ref + r.cpu().double().numpy()
        mag = mag + np.abs(r.cpu().double().numpy())
    got = c.cpu().double().numpy()
    assert np.isfinite(got).all()
    tol = np.abs(ref) * 2.0 ** -8 + mag * (K * 2.0 ** -23) + 1e-30
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} entries off; worst {np.abs(got - ref).max()} vs tol {tol[bad].min()}"


def test_gemm_nvfp4_rejects_bad_shapes():
    import luce_megakernel_b200 as L
    lib = L.lib()
    x = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    f = torch.ones(4, dtype=torch.float32, device="cuda")
    c = torch.zeros(128 * 128, dtype=torch.bfloat16, device="cuda")
    for (M, N, K) in ((128, 64, 256), (128, 128, 128), (0, 128, 256)):
        assert lib.mk_gemm_nvfp4_tn(_p(x), _p(x), _p(f), _p(x), _p(x), _p(f), _p(c), None, M, N, K, _stream()) != 0
    assert lib.mk_gemm_nvfp4_tn(None, _p(x), _p(f), _p(x), _p(x), _p(f), _p(c), None, 128, 128, 256, _stream()) != 0
