"""The NVFP4 quantisers against the reference's own quantiser kernels, as the reference builds them.

oracle/build_oracle.py cuts quantize_nvfp4_kernel (layer format: groups of 32, fp16 scales; reference:
megakernel/kernel_gb10_nvfp4.cu:1764-1817) and quantize_nvfp4_lm_kernel (16-blocks, E4M3 scales; :1373-1437) out
of the reference checkout and compiles them for sm_100a with the reference's flags, --use_fast_math included
(megakernel/setup.py:49-59), into oracle/_ref/libref_nvfp4_quant.so.  Under that flag `amax / 6.0f` and
`1.0f / scale` are approximate operations, so this is the comparison that decides whether "bit-exact to the
reference" holds for the binary a user of the reference actually runs.

Compared: packed codes and scales of launch_quantize_nvfp4_out / launch_quantize_nvfp4_lm_out on the real
layer shapes with the benchmark's weight distribution, and on adversarial inputs (values placed on the seven
code thresholds of their group, group maxima swept over every bf16 mantissa and a range of exponents).
"""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_QUANT = os.path.join(ROOT, "oracle", "_ref", "libref_nvfp4_quant.so")


@pytest.fixture(scope="module")
def libs():
    if not os.path.exists(REF_QUANT):
        pytest.skip("oracle/_ref/libref_nvfp4_quant.so was not built (no reference checkout at build time)")
    import luce_megakernel_b200 as L
    return L.lib(), ctypes.CDLL(REF_QUANT)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _quant_a(fn, w, group):
    rows, cols = w.shape
    packed = torch.zeros(rows, cols // 2, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(rows, cols // group, dtype=torch.float16, device="cuda")
    fn(_p(w), rows, cols, group, _p(packed), _p(scales), _stream())
    torch.cuda.synchronize()
    return packed.cpu(), scales.cpu().view(torch.int16)


def _quant_b(fn, w):
    rows, cols = w.shape
    packed = torch.zeros(rows, cols // 2, dtype=torch.uint8, device="cuda")
    scales = torch.zeros((rows // 128) * (cols // 64) * 512, dtype=torch.uint8, device="cuda")
    fn(_p(w), rows, cols, _p(packed), _p(scales), _stream())
    torch.cuda.synchronize()
    return packed.cpu(), scales.cpu()


def _weights(rows, cols, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(rows, cols, device="cuda", generator=g) * 0.02).to(torch.bfloat16).contiguous()


def _adversarial(group):
    """Rows of `group`-element groups.  Every group has one element that sets amax (all 128 bf16 mantissas x
    exponents 2^-12 .. 2^3, both signs) and elements at amax/6 * {0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5} -- the
    seven thresholds of the code table -- rounded to bf16, one bf16 step below and one above."""
    mant = torch.arange(128, dtype=torch.float32) / 128.0 + 1.0
    exps = torch.arange(-12, 4, dtype=torch.float32)
    amax = (mant[None, :] * torch.exp2(exps)[:, None]).reshape(-1)                  # 2048 group maxima
    thr = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    base = (amax[:, None] / 6.0 * thr[None, :]).to(torch.bfloat16)                  # [2048, 7]
    bits = base.view(torch.int16).to(torch.int32)
    below = (bits - 1).to(torch.int16).view(torch.bfloat16)
    above = (bits + 1).to(torch.int16).view(torch.bfloat16)
    vals = torch.cat([base, below, above], dim=1).float()                          # [2048, 21]
    vals = torch.minimum(vals, amax[:, None])
    n = vals.shape[1]
    reps = (group - 1 + n - 1) // n
    fill = vals.repeat(1, reps)[:, :group - 1]
    sign = torch.where(torch.arange(group - 1) % 2 == 0, 1.0, -1.0)
    grp = torch.cat([amax[:, None], fill * sign[None, :]], dim=1)                  # [2048, group]
    grp = torch.cat([grp, -grp], dim=0)                                            # both signs of amax
    return grp


def _report(name, a, b):
    diff = int((a != b).sum())
    return f"{name}: {diff} of {a.numel()} differ"


@pytest.mark.parametrize("shape", [(6144, 1024), (2048, 1024), (1024, 2048), (3584, 1024), (1024, 3584), (4096, 1024)])
def test_layer_format_matches_reference_binary_on_layer_shapes(libs, shape):
    mine, ref = libs
    w = _weights(*shape, seed=shape[0] + shape[1])
    pm, sm = _quant_a(mine.launch_quantize_nvfp4_out, w, 32)
    pr, sr = _quant_a(ref.launch_quantize_nvfp4_out, w, 32)
    assert torch.equal(sm, sr), _report("fp16 group scales", sm, sr)
    assert torch.equal(pm, pr), _report("packed codes", pm, pr)


def test_layer_format_matches_reference_binary_on_thresholds(libs):
    mine, ref = libs
    grp = _adversarial(32)                                           # [4096, 32]
    w = grp.reshape(128, 1024).to(torch.bfloat16).cuda().contiguous()
    pm, sm = _quant_a(mine.launch_quantize_nvfp4_out, w, 32)
    pr, sr = _quant_a(ref.launch_quantize_nvfp4_out, w, 32)
    assert torch.equal(sm, sr), _report("fp16 group scales", sm, sr)
    assert torch.equal(pm, pr), _report("packed codes", pm, pr)


@pytest.mark.parametrize("shape", [(248320, 1024), (6144, 1024), (1024, 3584)])
def test_lm_format_matches_reference_binary(libs, shape):
    mine, ref = libs
    w = _weights(*shape, seed=7 + shape[0])
    pm, sm = _quant_b(mine.launch_quantize_nvfp4_lm_out, w)
    pr, sr = _quant_b(ref.launch_quantize_nvfp4_lm_out, w)
    assert torch.equal(sm, sr), _report("E4M3 block scales", sm, sr)
    assert torch.equal(pm, pr), _report("packed codes", pm, pr)


def test_lm_format_matches_reference_binary_on_thresholds(libs):
    """16-element blocks; the e2m1 conversion rounds to nearest even, so the half-way points between codes
    (0.25, 0.75, ... times the decoded block scale) are the inputs on which an approximate reciprocal could
    tip a code."""
    mine, ref = libs
    grp = _adversarial(16)                                           # [4096, 16]
    w = grp.reshape(128, 512).to(torch.bfloat16).cuda().contiguous()
    pm, sm = _quant_b(mine.launch_quantize_nvfp4_lm_out, w)
    pr, sr = _quant_b(ref.launch_quantize_nvfp4_lm_out, w)
    assert torch.equal(sm, sr), _report("E4M3 block scales", sm, sr)
    assert torch.equal(pm, pr), _report("packed codes", pm, pr)
