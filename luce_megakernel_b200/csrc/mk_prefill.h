// Prefill building blocks (host-callable launchers).
#pragma once

#include <cuda_runtime.h>

namespace mk {

// C[M,N] = A[M,K] . W[N,K]^T (+ R[M,N]); bf16 row-major, f32 accumulate; tcgen05 / TMEM / TMA.
// N % 128 == 0, K % 64 == 0, lda and ldc multiples of 8 elements, pointers 16-byte aligned.
// err_flag: device int, set to 1 if a bounded wait ran out inside the kernel.
cudaError_t gemm_bf16_tn(const void* A, const void* W, void* C, const void* R, int M, int N, int K, int lda, int ldc,
                         int* err_flag, cudaStream_t stream);

}  // namespace mk
