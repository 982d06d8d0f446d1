// NVFP4 weight quantisers for sm_100a, bit-exact to the reference's two formats.  Two arithmetics: the
// reference binary's (its extension is built with --use_fast_math; kernels in nvfp4_quant_fastmath.cu, the
// default) and IEEE (what the plain-C restatement computes); mk_set_quantize_arithmetic() selects.
//
//  format A (layer weights; reference: megakernel/kernel_gb10_nvfp4.cu:1764-1817)
//    groups of `group_size` along K, scale = amax/6 as fp16 (1 for an all-zero group), code by the
//    thresholds .25/.75/1.25/1.75/2.5/3.5/5 on x * (1/scale) with the unrounded f32 scale.
//  format B (LM head / tensor-core layout; reference: megakernel/kernel_gb10_nvfp4.cu:1373-1437)
//    blocks of 16, scale = max(amax/6, 2^-28) in E4M3, values rounded to e2m1 (nearest even),
//    scales in 128-row x 4-column tiles of 512 bytes.
//
// Both are HBM-bound byte work: one thread per group/block, 128-bit loads of the bf16 row,
// 64/128-bit stores of the packed nibbles; consecutive threads take consecutive groups of a row.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/luce_megakernel_b200.h"

namespace {

#define MK_QK(name) name
#define MK_Q_DIV(a, b) __fdiv_rn((a), (b))
#define MK_Q_MUL(a, b) __fmul_rn((a), (b))
#include "nvfp4_quant_kernels.cuh"

// ---- format B with a per-tensor scale ------------------------------------------------------------------------
// s_t = amax(tensor) / (6 * 448) (1 for an all-zero tensor); block scale = E4M3(max((amax(block) / 6) / s_t, 2^-28));
// code = e2m1_rne(x / (dec * s_t)).  The reference stores block scales without a tensor scale
// (megakernel/kernel_gb10_nvfp4.cu:1373-1437, alpha = 1 at :451); this is the format of the NVFP4 recipe with an
// fp32 per-tensor scale, same packing and scale tiling as format B.
__global__ void tensor_amax_kernel(const __nv_bfloat16* __restrict__ w, size_t n8, unsigned* __restrict__ amax_bits) {
    float amax = 0.0f;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(w) + i);
#pragma unroll
        for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(bf_at(v, e)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(amax));     // non-negative floats order like their bits
}

__global__ void tensor_scale_kernel(unsigned* __restrict__ amax_bits_to_scale) {
    const float amax = __uint_as_float(*amax_bits_to_scale);
    *reinterpret_cast<float*>(amax_bits_to_scale) = amax > 0.0f ? __fdiv_rn(amax, 2688.0f) : 1.0f;
}

__global__ void quantize_ts_kernel(const __nv_bfloat16* __restrict__ w, uint8_t* __restrict__ packed,
                                   uint8_t* __restrict__ scales, const float* __restrict__ tensor_scale, int rows, int cols) {
    const int blocks_per_row = cols / 16;
    const long long bid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (bid >= (long long)rows * blocks_per_row) return;
    const float st = *tensor_scale;
    const int row = (int)(bid / blocks_per_row), sc = (int)(bid % blocks_per_row);
    const uint4* src = reinterpret_cast<const uint4*>(w + (size_t)row * cols + (size_t)sc * 16);
    const uint4 v0 = __ldg(src), v1 = __ldg(src + 1);
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fmaxf(fabsf(bf_at(v0, e)), fabsf(bf_at(v1, e))));
    const float rel = __fdiv_rn(__fmul_rn(amax, 1.0f / 6.0f), st);
    const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(fmaxf(rel, 1.0f / (float)(1 << 28)), __NV_SATFINITE, __NV_E4M3);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(s8, __NV_E4M3);
    const float eff = __fmul_rn(__half2float(*reinterpret_cast<const __half*>(&hr)), st);
    const float inv = (eff > 0.0f) ? __fdiv_rn(1.0f, eff) : 0.0f;
    unsigned long long out = 0;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const uint4& v = (p < 4) ? v0 : v1;
        const float2 f = make_float2(__fmul_rn(bf_at(v, (2 * p) & 7), inv), __fmul_rn(bf_at(v, (2 * p + 1) & 7), inv));
        const __nv_fp4x2_storage_t q = __nv_cvt_float2_to_fp4x2(f, __NV_E2M1, cudaRoundNearest);
        out |= (unsigned long long)(uint8_t)q << (8 * p);
    }
    *reinterpret_cast<unsigned long long*>(packed + (size_t)row * (cols / 2) + (size_t)sc * 8) = out;
    const size_t tile = (size_t)(row >> 7) * (cols / 64) + (sc >> 2);
    scales[tile * 512 + (size_t)(row & 31) * 16 + (size_t)((row & 127) >> 5) * 4 + (sc & 3)] = (uint8_t)s8;
}

// E4M3 block scales from the 128-row x 4-column tiles of the tensor-core layout to plain rows [rows][cols / 16]
__global__ void scales_to_rows_kernel(const uint8_t* __restrict__ tiled, uint8_t* __restrict__ rows_out, int rows, int cols) {
    const int spr = cols / 16;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * spr) return;
    const int row = (int)(i / spr), sc = (int)(i % spr);
    const size_t tile = (size_t)(row >> 7) * (cols / 64) + (sc >> 2);
    rows_out[i] = tiled[tile * 512 + (size_t)(row & 31) * 16 + (size_t)((row & 127) >> 5) * 4 + (sc & 3)];
}

thread_local char g_qerr[160] = "";
int g_quant_arith = 1;      // 1 = the reference binary's arithmetic (fast-math divide / reciprocal), 0 = IEEE
int qfail(const char* m) { snprintf(g_qerr, sizeof(g_qerr), "%s", m); return MK_ERR_BAD_ARG; }

}  // namespace

namespace mk {
// nvfp4_quant_fastmath.cu: the same two kernels compiled with --use_fast_math
void launch_quantize_a_fastmath(const __nv_bfloat16* w, uint8_t* packed, __half* scales, long long total, int gpr, int group,
                                unsigned blocks, int threads, cudaStream_t stream);
void launch_quantize_b_fastmath(const __nv_bfloat16* w, uint8_t* packed, uint8_t* scales, int rows, int cols, unsigned blocks,
                                int threads, cudaStream_t stream);
}  // namespace mk

extern "C" const char* mk_quantize_error(void) { return g_qerr; }
extern "C" void mk_set_quantize_arithmetic(int reference_binary) { g_quant_arith = reference_binary ? 1 : 0; }

extern "C" int launch_quantize_nvfp4_out(const void* weight, int rows, int cols, int group_size, void* packed_out,
                                         void* scales_out, cudaStream_t stream) {
    if (!weight || !packed_out || !scales_out) return qfail("null pointer argument");
    if (rows <= 0 || cols <= 0) return qfail("rows and cols must be positive");
    if (group_size <= 0 || (group_size & 1) || cols % group_size) return qfail("group_size must be even and divide cols");
    const int gpr = cols / group_size;
    const long long total = (long long)rows * gpr;
    const int threads = 256;
    const unsigned blocks = (unsigned)((total + threads - 1) / threads);
    if (g_quant_arith)
        mk::launch_quantize_a_fastmath((const __nv_bfloat16*)weight, (uint8_t*)packed_out, (__half*)scales_out, total, gpr,
                                       group_size, blocks, threads, stream);
    else
        quantize_a_kernel<<<blocks, threads, 0, stream>>>((const __nv_bfloat16*)weight, (uint8_t*)packed_out,
                                                          (__half*)scales_out, total, gpr, group_size);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_qerr, sizeof(g_qerr), "quantize launch: %s", cudaGetErrorString(e)); return MK_ERR_CUDA; }
    return MK_OK;
}

extern "C" int launch_quantize_nvfp4_lm_out(const void* weight, int rows, int cols, void* packed_out, void* scales_out,
                                            cudaStream_t stream) {
    if (!weight || !packed_out || !scales_out) return qfail("null pointer argument");
    if (rows <= 0 || rows % 128) return qfail("rows must be a positive multiple of 128");
    if (cols <= 0 || cols % 64) return qfail("cols must be a positive multiple of 64");
    if ((reinterpret_cast<uintptr_t>(weight) & 15u) || (reinterpret_cast<uintptr_t>(packed_out) & 7u))
        return qfail("weight must be 16-byte aligned and packed_out 8-byte aligned");
    const long long total = (long long)rows * (cols / 16);
    const int threads = 256;
    const unsigned blocks = (unsigned)((total + threads - 1) / threads);
    if (g_quant_arith)
        mk::launch_quantize_b_fastmath((const __nv_bfloat16*)weight, (uint8_t*)packed_out, (uint8_t*)scales_out, rows, cols,
                                       blocks, threads, stream);
    else
        quantize_b_kernel<<<blocks, threads, 0, stream>>>((const __nv_bfloat16*)weight, (uint8_t*)packed_out,
                                                          (uint8_t*)scales_out, rows, cols);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_qerr, sizeof(g_qerr), "quantize launch: %s", cudaGetErrorString(e)); return MK_ERR_CUDA; }
    return MK_OK;
}

// 16-block / E4M3 / fp32 per-tensor scale.  tensor_scale_out: device float[1].
extern "C" int mk_quantize_nvfp4_tensor_scale(const void* weight, int rows, int cols, void* packed_out, void* scales_out,
                                              float* tensor_scale_out, cudaStream_t stream) {
    if (!weight || !packed_out || !scales_out || !tensor_scale_out) return qfail("null pointer argument");
    if (rows <= 0 || rows % 128) return qfail("rows must be a positive multiple of 128");
    if (cols <= 0 || cols % 64) return qfail("cols must be a positive multiple of 64");
    if ((reinterpret_cast<uintptr_t>(weight) & 15u) || (reinterpret_cast<uintptr_t>(packed_out) & 7u))
        return qfail("weight must be 16-byte aligned and packed_out 8-byte aligned");
    cudaError_t e = cudaMemsetAsync(tensor_scale_out, 0, 4, stream);
    if (e == cudaSuccess) {
        const size_t n8 = (size_t)rows * cols / 8;
        tensor_amax_kernel<<<592, 256, 0, stream>>>((const __nv_bfloat16*)weight, n8, reinterpret_cast<unsigned*>(tensor_scale_out));
        tensor_scale_kernel<<<1, 1, 0, stream>>>(reinterpret_cast<unsigned*>(tensor_scale_out));
        const long long total = (long long)rows * (cols / 16);
        quantize_ts_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>((const __nv_bfloat16*)weight, (uint8_t*)packed_out,
                                                                             (uint8_t*)scales_out, tensor_scale_out, rows, cols);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) { snprintf(g_qerr, sizeof(g_qerr), "quantize launch: %s", cudaGetErrorString(e)); return MK_ERR_CUDA; }
    return MK_OK;
}

// Block scales of the tiled layout as plain rows: what the decode kernel streams (a row's scales contiguous).
extern "C" int mk_nvfp4_scales_to_rows(const void* tiled_scales, int rows, int cols, void* rows_out, cudaStream_t stream) {
    if (!tiled_scales || !rows_out) return qfail("null pointer argument");
    if (rows <= 0 || rows % 128) return qfail("rows must be a positive multiple of 128");
    if (cols <= 0 || cols % 64) return qfail("cols must be a positive multiple of 64");
    const long long total = (long long)rows * (cols / 16);
    scales_to_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>((const uint8_t*)tiled_scales, (uint8_t*)rows_out, rows, cols);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_qerr, sizeof(g_qerr), "scale re-layout launch: %s", cudaGetErrorString(e)); return MK_ERR_CUDA; }
    return MK_OK;
}
