// Prefill building blocks (host-callable launchers).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mk {

// Launch with programmatic stream serialisation (the kernels call pdl_enter() first): launch latency and the
// next kernel's set-up overlap the tail of the previous kernel.  A prompt of 520 tokens is ~310 short kernels.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid; cfg.blockDim = block; cfg.dynamicSmemBytes = smem; cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr; cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// C[M,N] = A[M,K] . W[N,K]^T (+ R[M,N]); bf16 row-major, f32 accumulate; tcgen05 / TMEM / TMA.
// N % 128 == 0, K % 64 == 0, lda and ldc multiples of 8 elements, pointers 16-byte aligned.
// err_flag: device int, set to 1 if a bounded wait ran out inside the kernel.
// splitk_ws / splitk_bytes: caller-owned f32 scratch for the partial products of a K-split (small M, K >= 2048);
// the split uses as many parts as fit (none when null).  The call allocates nothing.
// norm_w / norm_out (optional, N = 1024): when the product is split along K, the kernel that adds the parts also
// writes norm_out = RMSNorm(C) * (1 + norm_w) (the bits of the separate RMSNorm kernel) and sets *norm_done;
// otherwise *norm_done stays false and the caller normalises C itself.
cudaError_t gemm_bf16_tn(const void* A, const void* W, void* C, const void* R, int M, int N, int K, int lda, int ldc,
                         int* err_flag, float* splitk_ws, size_t splitk_bytes, cudaStream_t stream,
                         const void* norm_w = nullptr, void* norm_out = nullptr, bool* norm_done = nullptr);
// C1[M, N1] = A . W1^T and C2[M, N2] = A . W2^T in one launch (same tiles, same bits as two calls).  N1, N2 % 256 == 0.
cudaError_t gemm_bf16_tn_dual(const void* A, const void* W1, void* C1, int N1, int ldc1, const void* W2, void* C2, int N2, int ldc2,
                              int M, int K, int lda, int* err_flag, cudaStream_t stream);
// C[M, N] = silu(A . Wg^T) * (A . Wu^T), Wg = rows [0, N) and Wu = rows [glu_off, glu_off + N) of W [*, K]: the SwiGLU
// of the MLP inside the gate|up product's epilogue (both products rounded to bf16 first, as the separate kernel saw
// them).  N % 128 == 0, K % 64 == 0.
cudaError_t gemm_bf16_glu(const void* A, const void* W, void* C, int M, int N, int K, int lda, int ldc, int glu_off, int* err_flag,
                          cudaStream_t stream);

// C[M,N] = (ta[0] * tw[0]) * (A[M,K] . W[N,K]^T) (+ R[M,N]); A and W NVFP4 (packed e2m1 rows of K/2 bytes, E4M3 block
// scales in 128-row x 4-block tiles of 512 bytes, one fp32 tensor scale each), C and R bf16 row-major; block-scaled
// tcgen05 (kind::mxf4nvf4) with the scale tiles copied into tensor memory.  N % 128 == 0, K % 256 == 0, ldc % 8 == 0,
// pointers 16-byte aligned; the scale arrays cover whole 128-row blocks (rows rounded up).  Allocates nothing.
cudaError_t gemm_nvfp4_tn(const void* a_packed, const void* a_scales, const float* a_tensor_scale, const void* w_packed,
                          const void* w_scales, const float* w_tensor_scale, void* C, const void* R, int M, int N, int K, int ldc,
                          int* err_flag, cudaStream_t stream);

// Tail attention of one attention layer for the prompt compressor: for each of the last n_look prompt positions and each
// query head, the causal softmax over all keys, folded into running_max [n_look][S] (f32, >= 0) with a maximum.
// qkv: [S][5120] bf16 with q normalised and rotated in place; kc: that layer's K cache [2][max_seq][256].
cudaError_t tail_attention_scores(const void* qkv, const void* kc, int S, int max_seq, int n_look, float* running_max,
                                  cudaStream_t stream);

// Gated delta rule over a prompt in chunks of 64 tokens (all 16 heads of one layer).
// qkv: bf16 [S][6144] projection outputs q | k | v (the causal conv1d + SiLU and the L2 norms are applied inside);
// conv_w: bf16 [6144][4]; conv_state: f32 [6144][4], the four inputs before the prompt (read only);
// gates: f32 [S][16][4] = beta, decay, -, log decay; state: f32 [16][128 value][128 key], updated in place;
// o: f32 [S][2048]; scratch: dn_chunked_scratch_bytes(S).
size_t dn_chunked_scratch_bytes(int S);
cudaError_t dn_chunked(const void* qkv, const void* conv_w, const float* conv_state, const float* gates, float* state, float* o,
                       int S, void* scratch, int* err, cudaStream_t stream);

// Causal GQA attention over a prompt (one layer): qkv bf16 [S][5120] = 8 x [q | gate] | k | v with q normalised
// and rotated; kc, vc: bf16 [2][max_seq][256] (already holding the prompt's keys / values); out bf16 [S][2048]
// = softmax(q k^T / 16) v * sigmoid(gate).
// mask: null = dense; else the block mask written by block_select (one bit per 128-key block, per head and
// 128-query block).
cudaError_t fa_prefill(const void* qkv, const void* kc, const void* vc, void* out, int S, int max_seq, const uint32_t* mask,
                       cudaStream_t stream);

// The same attention (dense, or block-sparse with a mask) on tcgen05 / TMEM (TMA-fed, scores and P.V as tcgen05.mma, softmax one thread per row).
// err: device int, set to 3 if a bounded wait ran out.
cudaError_t fa_prefill_tcgen05(const void* qkv, const void* kc, const void* vc, void* out, int S, int max_seq, int* err,
                               const uint32_t* mask, cudaStream_t stream);

// Block selection for sparse attention over 128 x 128 blocks: keep the first `sink` key blocks, the `window`
// most recent ones and the ceil(top_frac * causal blocks) best by mean-pooled q . mean-pooled k, per query head.
// scratch: block_select_scratch_bytes(S); *mask_out points into it: uint32 [8][blocks][ceil(blocks / 32)].
size_t block_select_scratch_bytes(int S);
// rule 1 replaces the ranking by the reference's threshold rule (score >= alpha * row maximum, and every causal block
// for the last `last_full` query blocks); scores_out (optional) receives the f32 scores [8][blocks][blocks], j <= i.
cudaError_t block_select(const void* qkv, const void* kc, int S, int max_seq, double top_frac, int window, int sink,
                         void* scratch, uint32_t** mask_out, cudaStream_t stream, int rule = 0, float alpha = 0.f,
                         int last_full = 0, float* scores_out = nullptr);

}  // namespace mk
