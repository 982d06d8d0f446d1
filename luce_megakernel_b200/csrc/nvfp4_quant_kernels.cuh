// The two reference-format quantiser kernels, included by nvfp4_quant.cu (IEEE arithmetic: every divide and
// multiply correctly rounded, the arithmetic of the plain-C restatement) and by nvfp4_quant_fastmath.cu (plain
// operators, compiled with --use_fast_math like the reference extension, megakernel/setup.py:49-59: `amax / 6.0f`
// and `1.0f / scale` are then the approximate divide / reciprocal the reference's binary executes).
// The includer defines MK_QK(name), MK_Q_DIV(a, b) and MK_Q_MUL(a, b).
//  format A (layer weights; reference: megakernel/kernel_gb10_nvfp4.cu:1764-1817)
//  format B (LM head / tensor-core layout; reference: megakernel/kernel_gb10_nvfp4.cu:1373-1437)
#pragma once

__device__ __forceinline__ float bf_at(const uint4& v, int i) {
    const uint32_t w = (i < 2) ? v.x : (i < 4) ? v.y : (i < 6) ? v.z : v.w;
    return __uint_as_float((i & 1) ? (w & 0xffff0000u) : (w << 16));
}

__device__ __forceinline__ unsigned code_thresholds(float x) {
    const float ax = fabsf(x);
    const unsigned mag = ax < 0.25f ? 0u : ax < 0.75f ? 1u : ax < 1.25f ? 2u : ax < 1.75f ? 3u
                       : ax < 2.5f ? 4u : ax < 3.5f ? 5u : ax < 5.0f ? 6u : 7u;
    return (x < 0.0f) ? (mag | 8u) : mag;
}

__global__ void MK_QK(quantize_a_kernel)(const __nv_bfloat16* __restrict__ w, uint8_t* __restrict__ packed,
                                  __half* __restrict__ scales, long long total_groups, int groups_per_row, int group) {
    const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= total_groups) return;
    const long long row = gid / groups_per_row;
    const int g = (int)(gid - row * groups_per_row);
    const size_t cols = (size_t)groups_per_row * group;
    const __nv_bfloat16* src = w + row * cols + (size_t)g * group;
    uint8_t* dst = packed + row * (cols / 2) + (size_t)g * (group / 2);
    float amax = 0.0f;
    const bool vec = (group % 8 == 0) && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
    if (vec) {
        for (int i = 0; i < group; i += 8) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + i));
#pragma unroll
            for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(bf_at(v, e)));
        }
    } else {
        for (int i = 0; i < group; ++i) amax = fmaxf(amax, fabsf(__bfloat162float(src[i])));
    }
    const float scale = (amax > 0.0f) ? MK_Q_DIV(amax, 6.0f) : 1.0f;
    scales[gid] = __float2half_rn(scale);
    if (amax == 0.0f) {
        for (int i = 0; i < group / 2; ++i) dst[i] = 0;
        return;
    }
    const float inv = MK_Q_DIV(1.0f, scale);
    if (vec) {
        for (int i = 0; i < group; i += 8) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + i));
            uint32_t out = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) out |= code_thresholds(MK_Q_MUL(bf_at(v, e), inv)) << (4 * e);
            if ((reinterpret_cast<uintptr_t>(dst + i / 2) & 3u) == 0) *reinterpret_cast<uint32_t*>(dst + i / 2) = out;
            else for (int b = 0; b < 4; ++b) dst[i / 2 + b] = (uint8_t)(out >> (8 * b));
        }
    } else {
        for (int i = 0; i < group; i += 2) {
            const unsigned lo = code_thresholds(MK_Q_MUL(__bfloat162float(src[i]), inv));
            const unsigned hi = code_thresholds(MK_Q_MUL(__bfloat162float(src[i + 1]), inv));
            dst[i / 2] = (uint8_t)(lo | (hi << 4));
        }
    }
}

__global__ void MK_QK(quantize_b_kernel)(const __nv_bfloat16* __restrict__ w, uint8_t* __restrict__ packed,
                                  uint8_t* __restrict__ scales, int rows, int cols) {
    const int blocks_per_row = cols / 16;
    const long long bid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (bid >= (long long)rows * blocks_per_row) return;
    const int row = (int)(bid / blocks_per_row), sc = (int)(bid % blocks_per_row);
    const uint4* src = reinterpret_cast<const uint4*>(w + (size_t)row * cols + (size_t)sc * 16);
    const uint4 v0 = __ldg(src), v1 = __ldg(src + 1);
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fmaxf(fabsf(bf_at(v0, e)), fabsf(bf_at(v1, e))));
    const float scale_f = fmaxf(MK_Q_MUL(amax, (1.0f / 6.0f)), 1.0f / (float)(1 << 28));
    const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(scale_f, __NV_SATFINITE, __NV_E4M3);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(s8, __NV_E4M3);
    const float dec = __half2float(*reinterpret_cast<const __half*>(&hr));
    const float inv = (dec > 0.0f) ? MK_Q_DIV(1.0f, dec) : 0.0f;
    unsigned long long out = 0;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const uint4& v = (p < 4) ? v0 : v1;
        const float2 f = make_float2(MK_Q_MUL(bf_at(v, (2 * p) & 7), inv), MK_Q_MUL(bf_at(v, (2 * p + 1) & 7), inv));
        const __nv_fp4x2_storage_t q = __nv_cvt_float2_to_fp4x2(f, __NV_E2M1, cudaRoundNearest);
        out |= (unsigned long long)(uint8_t)q << (8 * p);
    }
    *reinterpret_cast<unsigned long long*>(packed + (size_t)row * (cols / 2) + (size_t)sc * 8) = out;
    const size_t tile = (size_t)(row >> 7) * (cols / 64) + (sc >> 2);
    scales[tile * 512 + (size_t)(row & 31) * 16 + (size_t)((row & 127) >> 5) * 4 + (sc & 3)] = (uint8_t)s8;
}

