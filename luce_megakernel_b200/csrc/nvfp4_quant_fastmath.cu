// The reference-format NVFP4 quantiser kernels with the arithmetic of the reference's binary.
//
// The reference builds its extension with --use_fast_math (megakernel/setup.py:49-59), so `amax / 6.0f` and
// `1.0f / scale` in its quantisers (megakernel/kernel_gb10_nvfp4.cu:1801,1811,1412) execute as an approximate
// divide and an approximate reciprocal, and denormals are flushed.  About one packed byte in 1700 then differs
// from correctly rounded arithmetic on N(0, 0.02) weights (a value within an ulp of a code threshold lands on the
// other side).  THIS FILE IS COMPILED WITH --use_fast_math (see _build.py) and writes the same expressions with
// plain operators, so that the compiler emits for them what it emits for the reference.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace {
#define MK_QK(name) name##_fastmath
#define MK_Q_DIV(a, b) ((a) / (b))
#define MK_Q_MUL(a, b) ((a) * (b))
#include "nvfp4_quant_kernels.cuh"
}  // namespace

namespace mk {
void launch_quantize_a_fastmath(const __nv_bfloat16* w, uint8_t* packed, __half* scales, long long total, int gpr, int group,
                                unsigned blocks, int threads, cudaStream_t stream) {
    quantize_a_kernel_fastmath<<<blocks, threads, 0, stream>>>(w, packed, scales, total, gpr, group);
}
void launch_quantize_b_fastmath(const __nv_bfloat16* w, uint8_t* packed, uint8_t* scales, int rows, int cols, unsigned blocks,
                                int threads, cudaStream_t stream) {
    quantize_b_kernel_fastmath<<<blocks, threads, 0, stream>>>(w, packed, scales, rows, cols);
}
}  // namespace mk
