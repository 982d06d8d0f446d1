// Speculative-prefill scoring with this model as its own drafter: which parts of a long prompt do the LAST few
// positions attend to?  The reference's pflash drafter (dflash/src/qwen3_drafter.cpp:86-183, forward in
// dflash/src/qwen3_0p6b_graph.cpp:430-496) runs a small model over the whole prompt with block-sparse attention,
// takes, per attention layer, the softmax of the last n_lookahead queries over every key ("tail attention"),
// reduces it to running_max[t][j] = max over layers and heads, and then keeps the top chunks of the prompt by the
// smoothed mean score.  Here the block-sparse prefill of this library plays the forward pass:
//   * tail_attention_scores (device): called by the prefill after the q / k norm + RoPE of every attention layer
//     (queries rewritten in place, keys already in the cache); one block per (tail query, query head) computes the
//     causal softmax over all keys in two passes and folds it into running_max with an atomic max (probabilities
//     are non-negative, so their bit patterns order like unsigned integers);
//   * mk_drafter_select (host): mean over the lookahead, average-pool smoothing, chunk means, top chunks, kept
//     positions in ascending order -- steps 2-4 of the reference function, restated.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>

#include <algorithm>
#include <vector>

#include "../../include/luce_megakernel_b200.h"
#include "mk_common.cuh"
#include "mk_prefill.h"

namespace mk {

namespace {

constexpr int TS_WARPS = 8;

// qkv: [S][5120] bf16 rows of 8 x [q(256) | gate(256)], k(512), v(512), q already normalised and rotated;
// kc: K cache of this layer [2][max_seq][256] bf16; running_max: [n_look][S] f32, >= 0
__global__ void __launch_bounds__(TS_WARPS * 32) k_tail_scores(const __nv_bfloat16* __restrict__ qkv,
                                                                const __nv_bfloat16* __restrict__ kc, int S, int max_seq,
                                                                int n_look, float* __restrict__ running_max) {
    pdl_enter();
    __shared__ float s_m[TS_WARPS], s_z[TS_WARPS];
    const int ti = blockIdx.x, h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = S - n_look + ti;                                  // position of this tail query
    const __nv_bfloat16* q = qkv + (size_t)t * FA_QKV_ROWS + (size_t)h * 2 * FA_HEAD_DIM;
    const __nv_bfloat16* kbase = kc + (size_t)(h / FA_GQA) * max_seq * FA_HEAD_DIM;
    float qf[8];
    {
        const uint4 v = reinterpret_cast<const uint4*>(q)[lane];
        qf[0] = bf_lo(v.x); qf[1] = bf_hi(v.x); qf[2] = bf_lo(v.y); qf[3] = bf_hi(v.y);
        qf[4] = bf_lo(v.z); qf[5] = bf_hi(v.z); qf[6] = bf_lo(v.w); qf[7] = bf_hi(v.w);
    }
    auto logit = [&](int j) {
        const uint4 v = reinterpret_cast<const uint4*>(kbase + (size_t)j * FA_HEAD_DIM)[lane];
        float d = qf[0] * bf_lo(v.x) + qf[1] * bf_hi(v.x) + qf[2] * bf_lo(v.y) + qf[3] * bf_hi(v.y) +
                  qf[4] * bf_lo(v.z) + qf[5] * bf_hi(v.z) + qf[6] * bf_lo(v.w) + qf[7] * bf_hi(v.w);
        return warp_sum(d) * 0.0625f;                               // 1 / sqrt(256)
    };
    // pass 1: running maximum and normaliser of this warp's keys (j <= t: causal)
    float m = -INFINITY, z = 0.f;
    for (int j = warp; j <= t; j += TS_WARPS) {
        const float l = logit(j);
        const float mn = fmaxf(m, l);
        z = z * expf(m - mn) + expf(l - mn);
        m = mn;
    }
    if (lane == 0) { s_m[warp] = m; s_z[warp] = z; }
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < TS_WARPS; ++w) M = fmaxf(M, s_m[w]);
    float Z = 0.f;
#pragma unroll
    for (int w = 0; w < TS_WARPS; ++w) Z += (s_m[w] == -INFINITY) ? 0.f : s_z[w] * expf(s_m[w] - M);
    const float inv = 1.0f / Z;
    // pass 2: probabilities into the running maximum over heads and layers
    unsigned int* out = reinterpret_cast<unsigned int*>(running_max + (size_t)ti * S);
    for (int j = warp; j <= t; j += TS_WARPS) {
        const float p = expf(logit(j) - M) * inv;
        if (lane == 0) atomicMax(out + j, __float_as_uint(p));
    }
}

}  // namespace

cudaError_t tail_attention_scores(const void* qkv, const void* kc, int S, int max_seq, int n_look, float* running_max,
                                  cudaStream_t stream) {
    if (n_look < 1 || n_look > S) return cudaErrorInvalidValue;
    return launch_pdl(k_tail_scores, dim3(n_look, FA_Q_HEADS), TS_WARPS * 32, 0, stream, (const __nv_bfloat16*)qkv,
                      (const __nv_bfloat16*)kc, S, max_seq, n_look, running_max);
}

}  // namespace mk

// Steps 2-4 of drafter_score_and_compress (dflash/src/qwen3_drafter.cpp:112-175) on a host copy of running_max:
// per-token score = mean over the lookahead rows; smoothed = mean over the window [j - pool/2, j + pool/2] clipped
// to the prompt; chunk mean of the smoothed scores; the n_keep = max(1, int(n_chunks * keep_ratio)) chunks with the
// largest means are kept (the reference's partial_sort leaves the order of equal means open: here the lower chunk
// index wins).  Writes the kept token POSITIONS in ascending order (the reference returns ids[position] for exactly
// these positions, spans of adjacent chunks merged) and returns their count, or -1 on a bad argument.
extern "C" int mk_drafter_select(const float* running_max, int n_lookahead, int seq_len, float keep_ratio, int chunk_size,
                                 int pool_kernel, int* kept_positions_out) {
    if (!running_max || !kept_positions_out || n_lookahead < 1 || seq_len < 1 || chunk_size < 1 || pool_kernel < 1 ||
        !(keep_ratio >= 0.0f))
        return -1;
    const int S = seq_len;
    std::vector<float> score((size_t)S), smooth((size_t)S);
    for (int j = 0; j < S; ++j) {
        float s = 0.0f;
        for (int t = 0; t < n_lookahead; ++t) s += running_max[(size_t)t * S + j];
        score[j] = s / (float)n_lookahead;
    }
    const int half = pool_kernel / 2;
    for (int j = 0; j < S; ++j) {
        const int lo = std::max(0, j - half), hi = std::min(S - 1, j + half);
        float s = 0.0f;
        for (int k = lo; k <= hi; ++k) s += score[k];
        smooth[j] = s / (float)(hi - lo + 1);
    }
    const int n_chunks = (S + chunk_size - 1) / chunk_size;
    const int n_keep = std::min(n_chunks, std::max(1, (int)((float)n_chunks * keep_ratio)));
    std::vector<std::pair<float, int>> means((size_t)n_chunks);
    for (int c = 0; c < n_chunks; ++c) {
        const int s0 = c * chunk_size, e0 = std::min(S, (c + 1) * chunk_size);
        float m = 0.0f;
        for (int j = s0; j < e0; ++j) m += smooth[j];
        means[c] = {m / (float)std::max(1, e0 - s0), c};
    }
    std::partial_sort(means.begin(), means.begin() + n_keep, means.end(), [](const std::pair<float, int>& a, const std::pair<float, int>& b) {
        return a.first > b.first || (a.first == b.first && a.second < b.second);
    });
    std::vector<int> sel((size_t)n_keep);
    for (int i = 0; i < n_keep; ++i) sel[i] = means[i].second;
    std::sort(sel.begin(), sel.end());
    int n = 0;
    for (int c : sel)
        for (int j = c * chunk_size; j < std::min(S, (c + 1) * chunk_size); ++j) kept_positions_out[n++] = j;
    return n;
}
