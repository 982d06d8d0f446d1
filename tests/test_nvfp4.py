"""NVFP4: the C oracle against the recorded CUDA conversion intrinsics (CPU), and the CUDA
quantisers against the C oracle, bit for bit (GPU)."""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import nvfp4

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(autouse=True)
def _ieee_quantiser_arithmetic(request):
    """The C restatement computes with correctly rounded divides; the library's default is the arithmetic of the
    reference's binary (built with --use_fast_math), which tests/test_nvfp4_reference_pin_gpu.py holds to that binary.
    The comparisons with the C restatement in this file therefore switch the library to IEEE arithmetic."""
    if request.node.get_closest_marker("gpu") is None:
        yield
        return
    import luce_megakernel_b200 as L
    L.lib().mk_set_quantize_arithmetic(0)
    yield
    L.lib().mk_set_quantize_arithmetic(1)


@pytest.fixture(scope="module")
def intr():
    return np.load(os.path.join(ROOT, "tests", "golden", "nvfp4_intrinsics.npz"))


def test_e4m3_tables_match_cuda_intrinsics(intr):
    L = nvfp4.lib()
    dec = np.array([L.mk_oracle_e4m3_to_f32(c) for c in range(256)], np.float32)
    assert np.array_equal(np.nan_to_num(dec, nan=-999.0), np.nan_to_num(intr["e4m3_decode"], nan=-999.0))
    x = intr["e4m3_in_bits"].view(np.float32)
    mine = np.array([L.mk_oracle_f32_to_e4m3(float(v)) for v in x], np.uint8)
    assert np.array_equal(mine, intr["e4m3_code"])


def test_e2m1_rounding_matches_cuda_intrinsics(intr):
    L = nvfp4.lib()
    mine = np.array([L.mk_oracle_f32_to_e2m1(float(a)) | (L.mk_oracle_f32_to_e2m1(float(b)) << 4)
                     for a, b in zip(intr["fp4_a"], intr["fp4_b"])], np.uint8)
    assert np.array_equal(mine, intr["fp4_byte"])       # low nibble = first element, ties to even code


def _rand_bf16(rows, cols, seed, scale=0.02):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(rows, cols, generator=g) * scale).to(torch.bfloat16)
    w[0, :32] = 0                       # an all-zero group
    w[1, 5] = 3.0                       # an outlier that sets its group's scale
    w[2, :16] = torch.tensor([6, -6, 4, 3, 2, 1.5, 1, .5, 5, 3.5, 2.5, 1.75, 1.25, .75, .25, 0]).to(torch.bfloat16)
    return w


def test_format_a_properties():
    w = _rand_bf16(64, 256, 0)
    packed, scales = nvfp4.quantize_a(w, 32)
    deq = nvfp4.dequantize_a(packed, scales, 32)
    wf = w.float().numpy()
    # dequantised values are within half a step of the group's largest element
    amax = np.abs(wf.reshape(64, 8, 32)).max(-1).repeat(32, -1).reshape(64, 256)
    assert np.all(np.abs(deq - wf) <= amax / 6.0 * 1.0 + 1e-3 * amax + 1e-12)
    assert np.all(packed[0, :16] == 0)                              # zero group -> zero bytes, scale 1
    assert scales[0, 0] == nvfp4.lib().mk_oracle_f32_to_f16(1.0)
    # the tie row: codes by the thresholds, half-way cases up in magnitude
    codes = [(packed[2, i // 2] >> (4 * (i & 1))) & 15 for i in range(16)]
    assert codes == [7, 15, 6, 5, 4, 3, 2, 1, 7, 6, 5, 4, 3, 2, 1, 0]


def test_format_b_properties():
    w = _rand_bf16(128, 128, 1)
    packed, scales = nvfp4.quantize_b(w)
    deq = nvfp4.dequantize_b(packed, scales)
    wf = w.float().numpy()
    amax = np.abs(wf.reshape(128, 8, 16)).max(-1).repeat(16, -1).reshape(128, 128)
    # weights of ~0.02 put amax/6 in the E4M3 subnormal range (steps of 2^-9), where the scale can
    # round down by up to a third and the largest element saturates: the bound is loose on purpose
    assert np.all(np.abs(deq - wf) <= amax * 0.5 + 1e-9)
    # swizzle: scale of (row, block) sits at tile*512 + (row%32)*16 + ((row%128)//32)*4 + block%4
    L = nvfp4.lib()
    seen = set()
    for r in range(128):
        for b in range(8):
            seen.add(L.mk_oracle_scale_index_b(r, b, 128))
    assert seen == set(range(128 * 8))          # a bijection onto the tile storage
    # round-to-nearest-even codes on the tie row (scale is 1.0 there: amax 6)
    codes = [(packed[2, i // 2] >> (4 * (i & 1))) & 15 for i in range(16)]
    assert codes == [7, 15, 6, 5, 4, 3, 2, 1, 6, 6, 4, 4, 2, 2, 0, 0]


def _gpu_quant(fn, w, outs):
    import luce_megakernel_b200 as L
    lib = L.lib()
    lib.mk_quantize_error.restype = ctypes.c_char_p
    rc = fn(lib, w, outs)
    assert rc == 0, lib.mk_quantize_error().decode()
    torch.cuda.synchronize()


@pytest.mark.gpu
@pytest.mark.parametrize("shape,group", [((64, 256), 32), ((6144, 1024), 32), ((1024, 3584), 32), ((48, 96), 16), ((16, 1024), 64)])
def test_gpu_quantizer_a_bit_exact(shape, group):
    w = _rand_bf16(shape[0], shape[1], 3)
    wd = w.cuda()
    packed = torch.empty(shape[0], shape[1] // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(shape[0], shape[1] // group, dtype=torch.float16, device="cuda")
    _gpu_quant(lambda lib, w_, o: lib.launch_quantize_nvfp4_out(
        ctypes.c_void_p(w_.data_ptr()), shape[0], shape[1], group, ctypes.c_void_p(o[0].data_ptr()),
        ctypes.c_void_p(o[1].data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), wd, (packed, scales))
    rp, rs = nvfp4.quantize_a(w, group)
    assert np.array_equal(packed.cpu().numpy(), rp)
    assert np.array_equal(scales.cpu().view(torch.int16).numpy().view(np.uint16), rs)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(128, 64), (256, 1024), (2048, 1024)])
def test_gpu_quantizer_b_bit_exact(shape):
    w = _rand_bf16(shape[0], shape[1], 4)
    wd = w.cuda()
    packed = torch.empty(shape[0], shape[1] // 2, dtype=torch.uint8, device="cuda")
    scales = torch.zeros((shape[0] // 128) * (shape[1] // 64) * 512, dtype=torch.uint8, device="cuda")
    _gpu_quant(lambda lib, w_, o: lib.launch_quantize_nvfp4_lm_out(
        ctypes.c_void_p(w_.data_ptr()), shape[0], shape[1], ctypes.c_void_p(o[0].data_ptr()),
        ctypes.c_void_p(o[1].data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), wd, (packed, scales))
    rp, rs = nvfp4.quantize_b(w)
    assert np.array_equal(packed.cpu().numpy(), rp)
    assert np.array_equal(scales.cpu().numpy(), rs)


@pytest.mark.gpu
def test_gpu_quantizer_rejects_bad_shapes():
    import luce_megakernel_b200 as L
    lib = L.lib()
    p = ctypes.c_void_p(16)
    assert lib.launch_quantize_nvfp4_out(p, 4, 100, 32, p, p, None) == 1
    assert lib.launch_quantize_nvfp4_lm_out(p, 100, 64, p, p, None) == 1
    assert lib.launch_quantize_nvfp4_lm_out(p, 128, 100, p, p, None) == 1


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,shape", [(0, (256, 1024)), (0, (1024, 3584)), (1, (256, 1024)), (1, (2048, 1024))])
def test_gpu_dequant_bit_exact_and_matvec(fmt, shape):
    """Dequantised weights are bit-identical to the C oracle; the in-register dequantising row
    product agrees with a float64 product of those weights to f32 rounding."""
    import luce_megakernel_b200 as L
    lib = L.lib()
    lib.mk_nvfp4_error.restype = ctypes.c_char_p
    rows, cols = shape
    w = _rand_bf16(rows, cols, 7 + fmt)
    if fmt == 0:
        packed, scales = nvfp4.quantize_a(w, 32)
        ref = nvfp4.dequantize_a(packed, scales, 32)
        sc_t = torch.from_numpy(scales.view(np.int16)).cuda()
    else:
        packed, scales = nvfp4.quantize_b(w)
        ref = nvfp4.dequantize_b(packed, scales)
        sc_t = torch.from_numpy(scales).cuda()
    pk_t = torch.from_numpy(packed).cuda()
    out = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
    rc = lib.mk_dequantize_nvfp4(fmt, ctypes.c_void_p(pk_t.data_ptr()), ctypes.c_void_p(sc_t.data_ptr()),
                                 ctypes.c_void_p(out.data_ptr()), rows, cols, 32, _stream())
    assert rc == 0, lib.mk_nvfp4_error().decode()
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))      # bit-exact
    g = torch.Generator().manual_seed(1)
    x = torch.randn(cols, generator=g)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    xd = x.cuda()
    rc = lib.mk_matvec_nvfp4(fmt, ctypes.c_void_p(pk_t.data_ptr()), ctypes.c_void_p(sc_t.data_ptr()),
                             ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(y.data_ptr()), rows, cols, 32, _stream())
    assert rc == 0, lib.mk_nvfp4_error().decode()
    torch.cuda.synchronize()
    yref = ref.astype(np.float64) @ x.numpy().astype(np.float64)
    err = np.abs(y.cpu().numpy() - yref).max()
    assert err <= 1e-5 * max(1.0, np.abs(yref).max()) + 1e-6, err


@pytest.mark.gpu
def test_quantize_ops_surface():
    """The torch ops of the reference's names and schemas give the oracle's bytes."""
    import luce_megakernel_b200 as L
    ops = L.load_ops()
    w = _rand_bf16(256, 1024, 9)
    wd = w.cuda()
    packed = torch.empty(256, 512, dtype=torch.uint8, device="cuda")
    scales = torch.empty(256, 32, dtype=torch.float16, device="cuda")
    ops.quantize_nvfp4_out(packed, scales, wd, 32)
    rp, rs = nvfp4.quantize_a(w, 32)
    assert np.array_equal(packed.cpu().numpy(), rp)
    assert np.array_equal(scales.cpu().view(torch.int16).numpy().view(np.uint16), rs)
    packed_b = torch.empty(256, 512, dtype=torch.uint8, device="cuda")
    scales_b = torch.zeros(2 * 16 * 512, dtype=torch.uint8, device="cuda")
    ops.quantize_nvfp4_lm_out(packed_b, scales_b, wd)
    bp, bs = nvfp4.quantize_b(w)
    assert np.array_equal(packed_b.cpu().numpy(), bp) and np.array_equal(scales_b.cpu().numpy(), bs)
    with pytest.raises(RuntimeError):
        ops.quantize_nvfp4_out(packed, scales, wd, 48)


def test_tensor_scale_format_properties():
    """CPU: the largest block scale is E4M3's 448, dequantised values stay within half an e2m1 step of the block
    scale, an all-zero tensor quantises to zeros with scale 1."""
    w = _rand_bf16(256, 512, 21) * 3.0
    packed, scales, ts = nvfp4.quantize_ts(w.to(torch.bfloat16))
    amax = float(w.to(torch.bfloat16).float().abs().max())
    assert np.float32(ts[0]) == np.float32(amax) / np.float32(2688.0)
    dec = np.array([nvfp4.lib().mk_oracle_e4m3_to_f32(int(c)) for c in np.unique(scales)])
    assert dec.max() == 448.0
    deq = nvfp4.dequantize_ts(packed, scales, ts)
    ref = w.to(torch.bfloat16).float().numpy()
    blk_amax = np.abs(ref).reshape(256, -1, 16).max(-1, keepdims=True)
    # e2m1 steps are at most 2 (between 4 and 6) in units of the block scale ~ amax / 6, E4M3 adds up to 1/16
    assert (np.abs(deq - ref).reshape(256, -1, 16) <= blk_amax * (1.0 / 6.0 + 1.0 / 16.0) + 1e-12).all()
    z = torch.zeros(128, 64, dtype=torch.bfloat16)
    zp, zs, zt = nvfp4.quantize_ts(z)
    assert zt[0] == 1.0 and not zp.any()
    assert not nvfp4.dequantize_ts(zp, zs, zt).any()


@pytest.mark.gpu
@pytest.mark.parametrize("shape,gain", [((256, 1024), 1.0), ((1024, 3584), 0.02), ((128, 64), 300.0)])
def test_gpu_tensor_scale_format_bit_exact(shape, gain):
    """Quantiser (codes, block scales, tensor scale) and dequantised weights bit-identical to the C restatement."""
    import luce_megakernel_b200 as L
    lib = L.lib()
    lib.mk_quantize_error.restype = ctypes.c_char_p
    rows, cols = shape
    w = (_rand_bf16(rows, cols, 5).float() * gain).to(torch.bfloat16)
    rp, rs, rt = nvfp4.quantize_ts(w)
    wd = w.cuda()
    pk = torch.zeros(rows, cols // 2, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(rs.size, dtype=torch.uint8, device="cuda")
    ts = torch.zeros(1, dtype=torch.float32, device="cuda")
    rc = lib.mk_quantize_nvfp4_tensor_scale(ctypes.c_void_p(wd.data_ptr()), rows, cols, ctypes.c_void_p(pk.data_ptr()),
                                            ctypes.c_void_p(sc.data_ptr()), ctypes.c_void_p(ts.data_ptr()), _stream())
    assert rc == 0, lib.mk_quantize_error().decode()
    torch.cuda.synchronize()
    assert np.array_equal(ts.cpu().numpy().view(np.uint32), rt.view(np.uint32))
    assert np.array_equal(sc.cpu().numpy(), rs)
    assert np.array_equal(pk.cpu().numpy(), rp)
    out = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
    rc = lib.mk_dequantize_nvfp4_tensor_scale(ctypes.c_void_p(pk.data_ptr()), ctypes.c_void_p(sc.data_ptr()),
                                              ctypes.c_void_p(ts.data_ptr()), ctypes.c_void_p(out.data_ptr()), 0, rows, cols, _stream())
    assert rc == 0
    ob = torch.empty(rows, cols, dtype=torch.bfloat16, device="cuda")
    rc = lib.mk_dequantize_nvfp4_tensor_scale(ctypes.c_void_p(pk.data_ptr()), ctypes.c_void_p(sc.data_ptr()),
                                              ctypes.c_void_p(ts.data_ptr()), ctypes.c_void_p(ob.data_ptr()), 1, rows, cols, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    ref = nvfp4.dequantize_ts(rp, rs, rt)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))       # bit-exact
    assert torch.equal(ob.cpu(), torch.from_numpy(ref).to(torch.bfloat16))
    # and close to the original weights: relative error of a 4-bit format
    err = np.abs(ref - w.float().numpy()).max() / float(w.float().abs().max())
    assert err <= 0.2
