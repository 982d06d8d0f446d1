// NVFP4 weights dequantised in registers: y = dequant(W) . x for both reference formats, and a
// plain dequantiser for bit-exact checks.
//
//  format A: packed uint8 [N, K/2], fp16 scales [N, K/32]            (layer weights)
//  format B: packed uint8 [N, K/2], E4M3 scales in 128 x 4 tiles      (LM head)
// value = e2m1(code) * scale (reference: megakernel/kernel_gb10_nvfp4.cu:80-83, 528-552, 1439-1456).
//
// HBM-bound streaming kernel: one warp per row, a lane takes 16 packed bytes (32 weights) per
// step with one 128-bit load, converts nibble pairs with the e2m1x2 -> f16x2 hardware conversion
// and accumulates in f32 against the activation kept in shared memory; 4 rows per warp are in
// flight.  Grid = 8 resident CTAs of 256 threads per SM.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/luce_megakernel_b200.h"
#include "mk_common.cuh"

namespace {

__device__ __forceinline__ float2 e2m1x2_to_float2(uint8_t byte) {
    const __half2_raw h = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)byte, __NV_E2M1);
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
__device__ __forceinline__ float e4m3_to_float(uint8_t c) {
    const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)c, __NV_E4M3);
    return __half2float(*reinterpret_cast<const __half*>(&h));
}
__device__ __forceinline__ size_t scale_index_b(int row, int blk, int cols) {
    return ((size_t)(row >> 7) * (cols >> 6) + (blk >> 2)) * 512 + (size_t)(row & 31) * 16 + (size_t)((row & 127) >> 5) * 4 + (blk & 3);
}

// dot of 32 weights (16 packed bytes) with 32 activations; FMT 0: one scale, FMT 1: two scales (16 + 16)
template <int FMT>
__device__ __forceinline__ float dot32(const uint4& p, const float* x, float s0, float s1) {
    const uint32_t w[4] = {p.x, p.y, p.z, p.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float part = 0.f;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const float2 v = e2m1x2_to_float2((uint8_t)(w[i] >> (8 * b)));
            part = fmaf(v.x, x[8 * i + 2 * b], part);
            part = fmaf(v.y, x[8 * i + 2 * b + 1], part);
        }
        if (i < 2) a0 += part; else a1 += part;
    }
    return FMT == 0 ? (a0 + a1) * s0 : a0 * s0 + a1 * s1;
}

template <int FMT>
__global__ void __launch_bounds__(256) matvec_nvfp4_kernel(const uint8_t* __restrict__ packed, const void* __restrict__ scales,
                                                           const float* __restrict__ x, float* __restrict__ y, int N, int K) {
    extern __shared__ float xs[];
    for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = K >> 5;                         // 32-weight steps per row
    for (int row = blockIdx.x * 8 + warp; row < N; row += gridDim.x * 8) {
        const uint4* prow = reinterpret_cast<const uint4*>(packed + (size_t)row * (K >> 1));
        float acc = 0.f;
        for (int g = lane; g < groups; g += 32) {
            const uint4 p = __ldg(prow + g);
            float s0, s1 = 0.f;
            if (FMT == 0) {
                s0 = __half2float(__ldg(reinterpret_cast<const __half*>(scales) + (size_t)row * groups + g));
            } else {
                const uint8_t* sp = reinterpret_cast<const uint8_t*>(scales) + scale_index_b(row, 2 * g, K);
                const unsigned short two = __ldg(reinterpret_cast<const unsigned short*>(sp));   // blocks 2g, 2g+1 are adjacent
                s0 = e4m3_to_float((uint8_t)(two & 0xff));
                s1 = e4m3_to_float((uint8_t)(two >> 8));
            }
            acc += dot32<FMT>(p, xs + 32 * g, s0, s1);
        }
        acc = mk::warp_sum(acc);
        if (lane == 0) y[row] = acc;
    }
}

template <int FMT>
__global__ void dequant_nvfp4_kernel(const uint8_t* __restrict__ packed, const void* __restrict__ scales,
                                     float* __restrict__ out, int N, int K, int group) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;      // one thread per packed byte
    if (i >= (size_t)N * (K >> 1)) return;
    const int row = (int)(i / (K >> 1)), c = (int)(i % (K >> 1)) * 2;
    const float2 v = e2m1x2_to_float2(packed[i]);
    float s;
    if (FMT == 0) s = __half2float(reinterpret_cast<const __half*>(scales)[(size_t)row * (K / group) + c / group]);
    else s = e4m3_to_float(reinterpret_cast<const uint8_t*>(scales)[scale_index_b(row, c >> 4, K)]);
    out[(size_t)row * K + c] = v.x * s;
    out[(size_t)row * K + c + 1] = v.y * s;
}

// format B with a per-tensor scale: value = e2m1(code) * (E4M3 block scale * tensor scale); f32 or bf16 output
template <typename OUT>
__global__ void dequant_nvfp4_ts_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                                        const float* __restrict__ tensor_scale, OUT* __restrict__ out, int N, int K) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;      // one thread per packed byte
    if (i >= (size_t)N * (K >> 1)) return;
    const int row = (int)(i / (K >> 1)), c = (int)(i % (K >> 1)) * 2;
    const float2 v = e2m1x2_to_float2(packed[i]);
    const float s = __fmul_rn(e4m3_to_float(scales[scale_index_b(row, c >> 4, K)]), *tensor_scale);
    out[(size_t)row * K + c] = (OUT)__fmul_rn(v.x, s);
    out[(size_t)row * K + c + 1] = (OUT)__fmul_rn(v.y, s);
}

thread_local char g_merr[160] = "";
int mfail(const char* m) { snprintf(g_merr, sizeof(g_merr), "%s", m); return MK_ERR_BAD_ARG; }

}  // namespace

extern "C" const char* mk_nvfp4_error(void) { return g_merr; }

extern "C" int mk_matvec_nvfp4(int format, const void* packed, const void* scales, const float* x, float* y, int rows,
                               int cols, int group_size, cudaStream_t stream) {
    if (!packed || !scales || !x || !y) return mfail("null pointer argument");
    if (rows <= 0 || cols <= 0 || cols % 64) return mfail("cols must be a positive multiple of 64");
    if (format == 0 && group_size != 32) return mfail("format A matvec supports group_size 32");
    if (format == 1 && rows % 128) return mfail("format B needs rows % 128 == 0");
    if (format != 0 && format != 1) return mfail("format must be 0 (A) or 1 (B)");
    if (reinterpret_cast<uintptr_t>(packed) & 15u) return mfail("packed must be 16-byte aligned");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int blocks = sms * 8;
    const size_t smem = (size_t)cols * 4;
    if (format == 0) matvec_nvfp4_kernel<0><<<blocks, 256, smem, stream>>>((const uint8_t*)packed, scales, x, y, rows, cols);
    else matvec_nvfp4_kernel<1><<<blocks, 256, smem, stream>>>((const uint8_t*)packed, scales, x, y, rows, cols);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_merr, sizeof(g_merr), "matvec launch: %s", cudaGetErrorString(e)); return MK_ERR_CUDA; }
    return MK_OK;
}

extern "C" int mk_dequantize_nvfp4(int format, const void* packed, const void* scales, float* out, int rows, int cols,
                                   int group_size, cudaStream_t stream) {
    if (!packed || !scales || !out) return mfail("null pointer argument");
    if (rows <= 0 || cols <= 0 || (cols & 1)) return mfail("bad shape");
    if (format == 0 && (group_size <= 0 || cols % group_size)) return mfail("group_size must divide cols");
    if (format == 1 && (rows % 128 || cols % 64)) return mfail("format B needs rows % 128 == 0 and cols % 64 == 0");
    if (format != 0 && format != 1) return mfail("format must be 0 (A) or 1 (B)");
    const size_t n = (size_t)rows * (cols / 2);
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (format == 0) dequant_nvfp4_kernel<0><<<blocks, 256, 0, stream>>>((const uint8_t*)packed, scales, out, rows, cols, group_size);
    else dequant_nvfp4_kernel<1><<<blocks, 256, 0, stream>>>((const uint8_t*)packed, scales, out, rows, cols, 16);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_merr, sizeof(g_merr), "dequantize launch: %s", cudaGetErrorString(e)); return MK_ERR_CUDA; }
    return MK_OK;
}

// 16-block / E4M3 / fp32 per-tensor scale (mk_quantize_nvfp4_tensor_scale).  out_is_bf16: 0 = f32 [rows][cols] (exact
// values), 1 = bf16 (what a bf16 GEMM consumes; e2m1 x E4M3 has at most 5 significant bits, the tensor scale adds
// up to 24, so this rounds).
extern "C" int mk_dequantize_nvfp4_tensor_scale(const void* packed, const void* scales, const float* tensor_scale, void* out,
                                                int out_is_bf16, int rows, int cols, cudaStream_t stream) {
    if (!packed || !scales || !tensor_scale || !out) return mfail("null pointer argument");
    if (rows <= 0 || cols <= 0 || rows % 128 || cols % 64) return mfail("needs rows % 128 == 0 and cols % 64 == 0");
    const size_t n = (size_t)rows * (cols / 2);
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (out_is_bf16) dequant_nvfp4_ts_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>((const uint8_t*)packed, (const uint8_t*)scales, tensor_scale, (__nv_bfloat16*)out, rows, cols);
    else dequant_nvfp4_ts_kernel<float><<<blocks, 256, 0, stream>>>((const uint8_t*)packed, (const uint8_t*)scales, tensor_scale, (float*)out, rows, cols);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_merr, sizeof(g_merr), "dequantize launch: %s", cudaGetErrorString(e)); return MK_ERR_CUDA; }
    return MK_OK;
}
