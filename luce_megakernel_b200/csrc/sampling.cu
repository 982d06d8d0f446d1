// Sampling at the LM-head boundary: temperature and top-k over the logits of one decode step.
//
// The reference decodes greedily; its only hook at this boundary is the repetition penalty applied to the logits
// before the argmax (megakernel/kernel.cu:793-795).  This is the next step after it: the decode kernel can store the
// step's logits (mk_set_logits_buffer), and the kernel below draws a token from softmax(logits / temperature)
// restricted to the top_k largest logits.
//
// Definition (restated on the CPU in oracle/sampling.py, which the tests hold this kernel to, token for token):
//   kept set  = the top_k logits, ordered by (value descending, index ascending); everything when top_k <= 0 or >= n
//   u_i       = uniform in (0, 1) from splitmix64(seed + counter * 0x9E3779B97F4A7C15 + (i + 1) * 0xD1B54A32D192ED03)
//   token     = argmax over the kept set of  logit_i / temperature - log(-log(u_i))     (ties: lowest index)
// i.e. the Gumbel-max form of categorical sampling: exact, and an argmax like the greedy path -- no normalisation, no
// prefix sums whose rounding would depend on the summation order.  temperature <= 0 or top_k == 1 is the greedy argmax.
// NaN logits are never chosen.  One block of 1024 threads; n <= 2^24.
//
// Nucleus (top_p) cut, after the sampler chain of the reference's speculative-decoding driver (repetition penalty ->
// top_k -> softmax(logit / temperature) -> top_p -> draw; dflash/test/test_dflash.cpp:127-188): over the set kept by
// top_k, in descending logit order, keep the shortest prefix whose probability mass reaches top_p (the element that
// crosses it included).  Here the cut is found without sorting, by a second radix descent over the order-preserving
// keys with the probability mass of each bin in place of its count; logits equal to the cut value are all kept.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/luce_megakernel_b200.h"

namespace {

constexpr int SAMPLE_THREADS = 1024;

__device__ __forceinline__ uint32_t order_key(float f) {
    if (f != f) return 0u;                                   // NaN sorts below everything
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);       // monotone: larger float -> larger key (-0 < +0)
}

__device__ __forceinline__ double uniform01(unsigned long long seed, unsigned long long counter, int i) {
    unsigned long long z = seed + counter * 0x9E3779B97F4A7C15ull + (unsigned long long)(i + 1) * 0xD1B54A32D192ED03ull;
    z ^= z >> 30; z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27; z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return ((double)(z >> 11) + 0.5) * (1.0 / 9007199254740992.0);       // (0, 1), 53 bits
}

struct Best { double v; int i; };
__device__ __forceinline__ bool better(double v, int i, const Best& b) { return v > b.v || (v == b.v && i < b.i); }

__global__ void __launch_bounds__(SAMPLE_THREADS) sample_kernel(const float* __restrict__ logits, int n, float temperature,
                                                                 int top_k, float top_p, unsigned long long seed,
                                                                 unsigned long long counter, int* __restrict__ token_out) {
    __shared__ unsigned hist[256];
    __shared__ double mass[256];
    __shared__ double s_red[SAMPLE_THREADS / 32];
    __shared__ double s_above, s_total;
    __shared__ float s_max;
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_need, s_equal;
    __shared__ double s_bv[SAMPLE_THREADS / 32];
    __shared__ int s_bi[SAMPLE_THREADS / 32];
    __shared__ int s_scan[SAMPLE_THREADS / 32];
    const int tid = threadIdx.x;
    const bool greedy = !(temperature > 0.0f) || top_k == 1;
    const bool keep_all = greedy || top_k <= 0 || top_k >= n;

    // ---- threshold: the key of the top_k-th largest logit (4 passes of an 8-bit radix select) ----
    uint32_t thr = 0u;
    int need = 0, equal = 0;
    if (!keep_all) {
        if (tid == 0) { s_prefix = 0u; s_mask = 0u; s_need = top_k; }
        __syncthreads();
        for (int pass = 3; pass >= 0; --pass) {
            const int shift = pass * 8;
            if (tid < 256) hist[tid] = 0u;
            __syncthreads();
            const uint32_t prefix = s_prefix, mask = s_mask;
            for (int i = tid; i < n; i += SAMPLE_THREADS) {
                const uint32_t key = order_key(logits[i]);
                if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                int rest = s_need, b = 255;
                while (b > 0 && (int)hist[b] < rest) { rest -= (int)hist[b]; --b; }
                s_need = rest;                       // how many of bin b's elements are still wanted
                s_equal = (int)hist[b];
                s_prefix = prefix | ((uint32_t)b << shift);
                s_mask = mask | (0xffu << shift);
            }
            __syncthreads();
        }
        thr = s_prefix; need = s_need; equal = s_equal;
    }

    const double inv_t = greedy ? 1.0 : 1.0 / (double)temperature;

    // ---- nucleus cut: the largest key t such that the mass of {key >= t} within the top_k set reaches top_p ----
    // Logits equal to the top_k threshold all carry the same mass, so when only `need` of the `equal` of them are kept
    // each counts need / equal: the totals are exact without ranking them here.
    uint32_t cut = 0u;                                   // keys below it are dropped
    if (!greedy && top_p > 0.0f && top_p < 1.0f) {
        const double tie_w = (!keep_all && need < equal) ? (double)need / (double)equal : 1.0;
        float mx = -INFINITY;
        for (int i = tid; i < n; i += SAMPLE_THREADS) {
            const float l = logits[i];
            if (l == l && (keep_all || order_key(l) >= thr)) mx = fmaxf(mx, l);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((tid & 31) == 0) s_red[tid >> 5] = (double)mx;
        __syncthreads();
        if (tid == 0) {
            double m = s_red[0];
            for (int w = 1; w < SAMPLE_THREADS / 32; ++w) m = fmax(m, s_red[w]);
            s_max = (float)m; s_above = 0.0; s_prefix = 0u; s_mask = 0u;
        }
        __syncthreads();
        const double shift_v = (double)s_max * inv_t;
        auto weight = [&](float l, uint32_t key) -> double {
            if (!(l == l) || (!keep_all && key < thr)) return 0.0;
            const double w = exp((double)l * inv_t - shift_v);
            return (!keep_all && key == thr) ? w * tie_w : w;
        };
        // total mass of the kept set (fixed order per thread, then a fixed-order tree: the same bits every run)
        double part = 0.0;
        for (int i = tid; i < n; i += SAMPLE_THREADS) { const float l = logits[i]; part += weight(l, order_key(l)); }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if ((tid & 31) == 0) s_red[tid >> 5] = part;
        __syncthreads();
        if (tid == 0) { double z = 0.0; for (int w = 0; w < SAMPLE_THREADS / 32; ++w) z += s_red[w]; s_total = z; }
        __syncthreads();
        const double target = (double)top_p * s_total;
        for (int pass = 3; pass >= 0; --pass) {
            const int shift = pass * 8;
            if (tid < 256) mass[tid] = 0.0;
            __syncthreads();
            const uint32_t prefix = s_prefix, mask = s_mask;
            for (int i = tid; i < n; i += SAMPLE_THREADS) {
                const float l = logits[i];
                const uint32_t key = order_key(l);
                if ((key & mask) == prefix) { const double w = weight(l, key); if (w > 0.0) atomicAdd(&mass[(key >> shift) & 255u], w); }
            }
            __syncthreads();
            if (tid == 0) {
                double acc = s_above;
                int b = 255;
                while (b > 0 && acc + mass[b] < target) { acc += mass[b]; --b; }
                s_above = acc;                           // mass of the keys above the chosen bin
                s_prefix = prefix | ((uint32_t)b << shift);
                s_mask = mask | (0xffu << shift);
            }
            __syncthreads();
        }
        cut = s_prefix;
    }

    // ---- Gumbel-max over the kept set ----
    Best best; best.v = -INFINITY; best.i = 0x7fffffff;
    const bool ranked = !keep_all && need < equal;      // only some of the logits equal to the threshold are kept: the lowest indices
    int taken_before = 0;                               // threshold-equal elements seen in earlier rounds (ranked mode)
    for (int base = 0; base < n; base += SAMPLE_THREADS) {
        const int i = base + tid;
        const float l = (i < n) ? logits[i] : 0.0f;
        const uint32_t key = (i < n) ? order_key(l) : 0u;
        bool kept = (i < n) && (l == l) && key >= cut && (keep_all || key > thr || (key == thr && !ranked));
        if (ranked) {                                    // uniform branch: rank the threshold-equal elements by index
            const bool eq = (i < n) && key == thr;
            const unsigned m = __ballot_sync(0xffffffffu, eq);
            if ((tid & 31) == 0) s_scan[tid >> 5] = __popc(m);
            __syncthreads();
            int before = taken_before;
            for (int w = 0; w < (tid >> 5); ++w) before += s_scan[w];
            int total = 0;
            for (int w = 0; w < SAMPLE_THREADS / 32; ++w) total += s_scan[w];
            before += __popc(m & ((1u << (tid & 31)) - 1u));
            if (eq && before < need && key >= cut) kept = true;
            taken_before += total;
            __syncthreads();
        }
        if (kept) {
            const double v = greedy ? (double)l : (double)l * inv_t - log(-log(uniform01(seed, counter, i)));
            if (better(v, i, best)) { best.v = v; best.i = i; }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const double ov = __shfl_xor_sync(0xffffffffu, best.v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best.i, o);
        if (better(ov, oi, best)) { best.v = ov; best.i = oi; }
    }
    if ((tid & 31) == 0) { s_bv[tid >> 5] = best.v; s_bi[tid >> 5] = best.i; }
    __syncthreads();
    if (tid < 32) {
        best.v = s_bv[tid]; best.i = s_bi[tid];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, best.v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best.i, o);
            if (better(ov, oi, best)) { best.v = ov; best.i = oi; }
        }
        if (tid == 0) *token_out = (best.i == 0x7fffffff) ? 0 : best.i;
    }
}

thread_local char g_serr[160] = "";

}  // namespace

extern "C" const char* mk_sample_error(void) { return g_serr; }

extern "C" int mk_sample_top_k(const float* logits, int n, float temperature, int top_k, unsigned long long seed,
                               unsigned long long counter, int* token_out, cudaStream_t stream) {
    return mk_sample_top_k_top_p(logits, n, temperature, top_k, 1.0f, seed, counter, token_out, stream);
}

extern "C" int mk_sample_top_k_top_p(const float* logits, int n, float temperature, int top_k, float top_p, unsigned long long seed,
                                     unsigned long long counter, int* token_out, cudaStream_t stream) {
    if (!logits || !token_out) { snprintf(g_serr, sizeof(g_serr), "null pointer argument"); return MK_ERR_BAD_ARG; }
    if (n < 1 || n > (1 << 24)) { snprintf(g_serr, sizeof(g_serr), "n must be in [1, 2^24]"); return MK_ERR_BAD_ARG; }
    if (temperature != temperature) { snprintf(g_serr, sizeof(g_serr), "temperature is NaN"); return MK_ERR_BAD_ARG; }
    if (top_p != top_p) { snprintf(g_serr, sizeof(g_serr), "top_p is NaN"); return MK_ERR_BAD_ARG; }
    sample_kernel<<<1, SAMPLE_THREADS, 0, stream>>>(logits, n, temperature, top_k, top_p, seed, counter, token_out);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_serr, sizeof(g_serr), "sampling launch: %s", cudaGetErrorString(e)); return MK_ERR_CUDA; }
    return MK_OK;
}
