// bf16 prefill of the Qwen3.5-0.8B hybrid for sm_100a: prompt of S tokens from position 0.
//
// The dense projections and the MLP run as tcgen05 / TMEM GEMMs fed by TMA (gemm_tcgen05.cu); the
// kernels in this file are the pieces between them.  Arithmetic follows the reference prefill
// (megakernel/prefill.cu:1559-1793) and, token by token, the decode kernel: bf16 activations
// between GEMMs, f32 inside every kernel, f32 DeltaNet state.
//
// First version of this path: the DeltaNet scan is token-serial per (head, 16 value rows) and the
// causal attention is a scalar online-softmax warp per (query, head).  Both are correct for any S
// and are the parts a later version replaces with the chunked scan / tensor-core flash attention.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/luce_megakernel_b200.h"
#include "mk_common.cuh"
#include "mk_prefill.h"

namespace mk {
namespace {

__constant__ float c_pf_inv_freq[FA_ROT / 2];

__device__ __forceinline__ float ld_bf(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// ---- embedding + RMSNorm -------------------------------------------------------------------

__global__ void k_embed(const int* __restrict__ tok, const __nv_bfloat16* __restrict__ embed,
                        __nv_bfloat16* __restrict__ hidden, int S, int vocab) {
    pdl_enter();
    const int t = blockIdx.x;
    int id = tok[t];
    id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
    const uint4* src = reinterpret_cast<const uint4*>(embed + (size_t)id * HIDDEN);
    uint4* dst = reinterpret_cast<uint4*>(hidden + (size_t)t * HIDDEN);
    for (int i = threadIdx.x; i < HIDDEN / 8; i += blockDim.x) dst[i] = __ldg(src + i);
}

// one warp per row: out = bf16( x * rsqrt(mean x^2 + eps) * (1 + w) )   (reference: prefill.cu:72-88)
// dst may be global or shared memory (the batched step normalises while it stages its activations).
__device__ __forceinline__ void rmsnorm_row(const uint4* __restrict__ src, const __nv_bfloat16* __restrict__ w, uint4* dst, int lane) {
    float v[32];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 u = src[i * 32 + lane];
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) { v[i * 8 + 2 * e] = bf_lo(q[e]); v[i * 8 + 2 * e + 1] = bf_hi(q[e]); }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss * (1.0f / HIDDEN) + RMS_EPS);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 wu = __ldg(reinterpret_cast<const uint4*>(w) + i * 32 + lane);
        const uint32_t wq[4] = {wu.x, wu.y, wu.z, wu.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 p = __floats2bfloat162_rn(v[i * 8 + 2 * e] * rstd * (1.0f + bf_lo(wq[e])),
                                                           v[i * 8 + 2 * e + 1] * rstd * (1.0f + bf_hi(wq[e])));
            o[e] = *reinterpret_cast<const uint32_t*>(&p);
        }
        dst[i * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

__global__ void k_rmsnorm(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                          __nv_bfloat16* __restrict__ out, int S) {
    pdl_enter();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= S) return;
    rmsnorm_row(reinterpret_cast<const uint4*>(x + (size_t)row * HIDDEN), w, reinterpret_cast<uint4*>(out + (size_t)row * HIDDEN), lane);
}

// ---- DeltaNet pieces ---------------------------------------------------------------------------

// beta = sigmoid(Wb x), decay = exp(g), g = -exp(A_log) softplus(Wa x + dt_bias)  (reference: prefill.cu:91-99, 400-412)
// gates: [t][head][4] = beta, decay, (q.k, written by the recurrent path's conv kernel), g.
// One CTA per 16 tokens: [16 x 1024] x [1024 x 32] with mma.sync (columns 0-15 = beta rows of Wb, 16-31 = alpha
// rows of Wa), eight warps split K and each requests its whole eighth of both operands before the first product
// (the kernel is one memory round trip long, not one per k-step); operands straight from global memory (the 64 KB
// of gate weights stay in L1 / L2), partial sums meet in shared memory.
__global__ void __launch_bounds__(256) k_dn_gates_mma(const __nv_bfloat16* __restrict__ xn, const __nv_bfloat16* __restrict__ Wb,
                                                      const __nv_bfloat16* __restrict__ Wa, const __nv_bfloat16* __restrict__ a_log,
                                                      const __nv_bfloat16* __restrict__ dt_bias, float* __restrict__ gates, int S) {
    pdl_enter();
    __shared__ float part[8][16][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g8 = lane >> 2, t4 = lane & 3;
    const int t0 = blockIdx.x * 16;
    const int r0 = min(t0 + g8, S - 1), r1 = min(t0 + g8 + 8, S - 1);        // rows past the prompt repeat the last one
    const uint32_t* x0 = reinterpret_cast<const uint32_t*>(xn + (size_t)r0 * HIDDEN) + warp * 64 + t4;
    const uint32_t* x1 = reinterpret_cast<const uint32_t*>(xn + (size_t)r1 * HIDDEN) + warp * 64 + t4;
    // B fragment of n-tile n: column g8 = output row 8 n + g8 of [Wb ; Wa]
    const uint32_t* wrow[4];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
        const int o = n * 8 + g8;
        wrow[n] = reinterpret_cast<const uint32_t*>((o < 16 ? Wb + (size_t)o * HIDDEN : Wa + (size_t)(o - 16) * HIDDEN)) + warp * 64 + t4;
    }
    float acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) { acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f; }
    uint32_t a[8][4], b[8][4][2];                           // this warp's eighth of K: 128 elements = 8 k-steps
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
        a[ks][0] = x0[ks * 8]; a[ks][1] = x1[ks * 8]; a[ks][2] = x0[ks * 8 + 4]; a[ks][3] = x1[ks * 8 + 4];
#pragma unroll
        for (int n = 0; n < 4; ++n) { b[ks][n][0] = __ldg(wrow[n] + ks * 8); b[ks][n][1] = __ldg(wrow[n] + ks * 8 + 4); }
    }
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                         : "+f"(acc[n][0]), "+f"(acc[n][1]), "+f"(acc[n][2]), "+f"(acc[n][3])
                         : "r"(a[ks][0]), "r"(a[ks][1]), "r"(a[ks][2]), "r"(a[ks][3]), "r"(b[ks][n][0]), "r"(b[ks][n][1]));
        }
    }
#pragma unroll
    for (int n = 0; n < 4; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) part[warp][g8 + (e >> 1) * 8][n * 8 + 2 * t4 + (e & 1)] = acc[n][e];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 16 * 32; i += 256) {
        const int tt = i >> 5, o = i & 31, t = t0 + tt;
        if (t >= S) continue;
        const float v = ((part[0][tt][o] + part[1][tt][o]) + (part[2][tt][o] + part[3][tt][o])) +
                        ((part[4][tt][o] + part[5][tt][o]) + (part[6][tt][o] + part[7][tt][o]));
        if (o < 16) gates[((size_t)t * 16 + o) * 4] = 1.0f / (1.0f + expf(-v));
        else {
            const int h = o - 16;
            const float x = v + ld_bf(dt_bias + h);
            const float sp = (x > 20.0f) ? x : log1pf(expf(x));
            const float g = -expf(ld_bf(a_log + h)) * sp;
            gates[((size_t)t * 16 + h) * 4 + 1] = expf(g);
            gates[((size_t)t * 16 + h) * 4 + 3] = g;
        }
    }
}

// causal depthwise conv (k=4) + SiLU over all t in parallel, then per-head L2 norm of q (x 1/sqrt(128))
// and k; block = (t, head), thread c = channel c of q, k and v of that head.  Inputs for t < 3 come
// from the stored conv window.  Also leaves q.k per (t, head).  (reference: prefill.cu:1281-1368)
__global__ void k_dn_preproject(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ conv_w,
                                const float* __restrict__ conv_state, float* __restrict__ pre, float* __restrict__ kq, int S) {
    pdl_enter();
    const int t = blockIdx.x, h = blockIdx.y, c = threadIdx.x;
    __shared__ float red[3][4];
    float val[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        const int ch = r * DN_QK + h * DN_KEY + c;
        const uint2 wr = __ldg(reinterpret_cast<const uint2*>(conv_w) + ch);
        const float w4[4] = {bf_lo(wr.x), bf_hi(wr.x), bf_lo(wr.y), bf_hi(wr.y)};
        float co = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int tt = t - 3 + k;
            const float x = (tt >= 0) ? ld_bf(qkv + (size_t)tt * DN_CONV_CH + ch) : conv_state[ch * 4 + 4 + tt];
            co += x * w4[k];
        }
        val[r] = silu_f(co);
    }
    float sq = warp_sum(val[0] * val[0]), sk = warp_sum(val[1] * val[1]), sqk = warp_sum(val[0] * val[1]);
    if ((c & 31) == 0) { red[0][c >> 5] = sq; red[1][c >> 5] = sk; red[2][c >> 5] = sqk; }
    __syncthreads();
    sq = red[0][0] + red[0][1] + red[0][2] + red[0][3];
    sk = red[1][0] + red[1][1] + red[1][2] + red[1][3];
    sqk = red[2][0] + red[2][1] + red[2][2] + red[2][3];
    const float qn = rsqrtf(sq + 1e-6f) * 0.08838834764831845f, kn = rsqrtf(sk + 1e-6f);
    float* dst = pre + (size_t)t * DN_CONV_CH + h * DN_KEY + c;
    dst[0] = val[0] * qn;
    dst[DN_QK] = val[1] * kn;
    dst[2 * DN_QK] = val[2];
    if (c == 0) kq[(t * 16 + h) * 4 + 2] = sqk * qn * kn;
}

// conv window after the prompt: the last four pre-activation inputs (reference: prefill.cu:1373-1395)
__global__ void k_dn_conv_state(const __nv_bfloat16* __restrict__ qkv, float* __restrict__ conv_state, int S) {
    pdl_enter();
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= DN_CONV_CH) return;
    float old[4], nw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) old[k] = conv_state[ch * 4 + k];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int tt = S - 4 + k;
        nw[k] = (tt >= 0) ? ld_bf(qkv + (size_t)tt * DN_CONV_CH + ch) : old[4 + tt];
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) conv_state[ch * 4 + k] = nw[k];
}

// Gated delta rule, token-serial.  Block = (head, 16 value rows), 16 warps; warp = one value row,
// lane = 4 keys, the state row stays in registers for the whole prompt.  The per-token inputs
// (q and k of the head, the 16 v values, beta / decay / q.k) are staged through shared memory in
// tiles of 32 tokens with cp.async double buffering, so a step costs shared-memory latency plus
// the two warp reductions instead of an L2 round trip.  (reference: prefill.cu:114-221)
constexpr int SCAN_TT = 32;                       // tokens per staged tile
constexpr int SCAN_TOK_FLOATS = 256 + 16 + 4;     // q[128] | k[128] | v[16 rows of this block] | beta, decay, q.k, pad
constexpr int SCAN_TILE_FLOATS = SCAN_TT * SCAN_TOK_FLOATS;
constexpr int SCAN_SMEM = 2 * SCAN_TILE_FLOATS * 4;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// gates: [t][head][4] = beta, decay, q.k, log decay
__global__ void __launch_bounds__(512) k_dn_scan(const float* __restrict__ pre, const float* __restrict__ gates,
                                                 float* __restrict__ state, float* __restrict__ o, int S) {
    pdl_enter();
    extern __shared__ __align__(16) float scan_sm[];
    const int h = blockIdx.x >> 3, slice = blockIdx.x & 7;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = slice * 16 + warp;
    float* srow = state + ((size_t)h * DN_VAL + row) * DN_KEY;
    float4 s = reinterpret_cast<const float4*>(srow)[lane];
    const int ntiles = (S + SCAN_TT - 1) / SCAN_TT;
    auto stage = [&](int tile, int buf) {
        // per token 69 16-byte pieces: 32 of q, 32 of k, 4 of v, 1 of gates
        float* dst = scan_sm + buf * SCAN_TILE_FLOATS;
        for (int i = threadIdx.x; i < SCAN_TT * 69; i += 512) {
            const int tt = i / 69, piece = i - tt * 69;
            const int t = tile * SCAN_TT + tt;
            if (t < S) {
                const float* src;
                if (piece < 32) src = pre + (size_t)t * DN_CONV_CH + h * DN_KEY + piece * 4;
                else if (piece < 64) src = pre + (size_t)t * DN_CONV_CH + DN_QK + h * DN_KEY + (piece - 32) * 4;
                else if (piece < 68) src = pre + (size_t)t * DN_CONV_CH + 2 * DN_QK + h * DN_VAL + slice * 16 + (piece - 64) * 4;
                else src = gates + ((size_t)t * 16 + h) * 4;
                cp_async16(dst + tt * SCAN_TOK_FLOATS + piece * 4, src);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    stage(0, 0);
    for (int tile = 0; tile < ntiles; ++tile) {
        const int buf = tile & 1;
        if (tile + 1 < ntiles) stage(tile + 1, buf ^ 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();
        const float* tb = scan_sm + buf * SCAN_TILE_FLOATS;
        const int t0 = tile * SCAN_TT, tn = min(SCAN_TT, S - t0);
#pragma unroll 2
        for (int tt = 0; tt < tn; ++tt) {
            const float* tok = tb + tt * SCAN_TOK_FLOATS;
            const float4 q4 = reinterpret_cast<const float4*>(tok)[lane];
            const float4 k4 = reinterpret_cast<const float4*>(tok + 128)[lane];
            const float vj = tok[256 + warp];
            const float4 gt = *reinterpret_cast<const float4*>(tok + 272);     // beta, decay, q.k
            float stk = s.x * k4.x + s.y * k4.y + s.z * k4.z + s.w * k4.w;
            float sqv = s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w;
#pragma unroll
            for (int of = 16; of > 0; of >>= 1) {
                stk += __shfl_xor_sync(0xffffffffu, stk, of);
                sqv += __shfl_xor_sync(0xffffffffu, sqv, of);
            }
            const float err = (vj - gt.y * stk) * gt.x;
            s.x = fmaf(s.x, gt.y, k4.x * err); s.y = fmaf(s.y, gt.y, k4.y * err);
            s.z = fmaf(s.z, gt.y, k4.z * err); s.w = fmaf(s.w, gt.y, k4.w * err);
            if (lane == 0) o[(size_t)(t0 + tt) * DN_V + h * DN_VAL + row] = gt.y * sqv + err * gt.z;
        }
        __syncthreads();
    }
    reinterpret_cast<float4*>(srow)[lane] = s;
}

// y = o * rsqrt(mean o^2 + eps) * w * silu(z), one warp per (t, head) (reference: prefill.cu:1493-1523)
__global__ void k_dn_gated_norm(const float* __restrict__ o, const __nv_bfloat16* __restrict__ z,
                                const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int S) {
    pdl_enter();
    const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (wid >= S * DN_HEADS) return;
    const float4 o4 = reinterpret_cast<const float4*>(o + (size_t)wid * DN_VAL)[lane];
    const uint2 z2 = reinterpret_cast<const uint2*>(z + (size_t)wid * DN_VAL)[lane];
    const uint2 w2 = __ldg(reinterpret_cast<const uint2*>(w) + lane);
    const float ss = warp_sum(o4.x * o4.x + o4.y * o4.y + o4.z * o4.z + o4.w * o4.w);
    const float rstd = rsqrtf(ss * (1.0f / DN_VAL) + RMS_EPS);
    const __nv_bfloat162 p0 = __floats2bfloat162_rn(o4.x * rstd * bf_lo(w2.x) * silu_f(bf_lo(z2.x)),
                                                    o4.y * rstd * bf_hi(w2.x) * silu_f(bf_hi(z2.x)));
    const __nv_bfloat162 p1 = __floats2bfloat162_rn(o4.z * rstd * bf_lo(w2.y) * silu_f(bf_lo(z2.y)),
                                                    o4.w * rstd * bf_hi(w2.y) * silu_f(bf_hi(z2.y)));
    uint2 r;
    r.x = *reinterpret_cast<const uint32_t*>(&p0); r.y = *reinterpret_cast<const uint32_t*>(&p1);
    reinterpret_cast<uint2*>(out + (size_t)wid * DN_VAL)[lane] = r;
}

// ---- attention pieces ------------------------------------------------------------------------------

// per-head RMSNorm(1+w) + partial RoPE; q rewritten in place (bf16), K and V appended to the caches.
// warp per (t, slot): slots 0-7 = q heads, 8-9 = k heads, 10-11 = v heads.  Row layout of the fused
// projection: 8 x [q(256) | gate(256)], k(512), v(512).  (reference: prefill.cu:1041-1087)
__global__ void k_fa_norm_rope(__nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ q_norm,
                               const __nv_bfloat16* __restrict__ k_norm, __nv_bfloat16* __restrict__ kc,
                               __nv_bfloat16* __restrict__ vc, int S, int max_seq,
                               const int* __restrict__ row_pos, size_t row_cache_stride) {
    pdl_enter();
    const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (wid >= S * 12) return;
    const int r = wid / 12, slot = wid % 12;
    __nv_bfloat16* row = qkv + (size_t)r * FA_QKV_ROWS;
    // prompt: row r is position r of one sequence; batched step: row r is sequence r at position row_pos[r]
    int t = r;
    if (row_pos) {
        t = min(max(row_pos[r], 0), max_seq - 1);
        kc += (size_t)r * row_cache_stride;
        vc += (size_t)r * row_cache_stride;
    }
    if (slot >= 10) {
        const int g = slot - 10;
        const uint4* src = reinterpret_cast<const uint4*>(row + FA_QPROJ + FA_KV_SIZE + g * FA_HEAD_DIM);
        reinterpret_cast<uint4*>(vc + ((size_t)g * max_seq + t) * FA_HEAD_DIM)[lane] = src[lane];
        return;
    }
    const bool isq = slot < 8;
    __nv_bfloat16* src = isq ? row + slot * 2 * FA_HEAD_DIM : row + FA_QPROJ + (slot - 8) * FA_HEAD_DIM;
    const __nv_bfloat16* wn = isq ? q_norm : k_norm;
    float n[8], ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) { n[e] = ld_bf(src + lane + 32 * e); ss += n[e] * n[e]; }
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss * (1.0f / FA_HEAD_DIM) + RMS_EPS);
#pragma unroll
    for (int e = 0; e < 8; ++e) n[e] = n[e] * rstd * (1.0f + ld_bf(wn + lane + 32 * e));
    float sn, cs;
    sincosf((float)t * c_pf_inv_freq[lane], &sn, &cs);
    const float a = n[0], b = n[1];
    n[0] = a * cs - b * sn;
    n[1] = b * cs + a * sn;
    __nv_bfloat16* dst = isq ? src : kc + ((size_t)(slot - 8) * max_seq + t) * FA_HEAD_DIM;
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[lane + 32 * e] = __float2bfloat16_rn(n[e]);
}

// ---- MLP glue, final norm, LM head -------------------------------------------------------------------

// act[t, i] = silu(gu[t, i]) * gu[t, 3584 + i]   (reference: prefill.cu:1239-1247)
__global__ void k_silu_mul(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ act, int S) {
    pdl_enter();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;     // one thread per 8 outputs
    if (i >= (size_t)S * (INTER / 8)) return;
    const size_t t = i / (INTER / 8), c = (i % (INTER / 8)) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + t * (2 * INTER) + c);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + t * (2 * INTER) + INTER + c);
    const uint32_t ga[4] = {gv.x, gv.y, gv.z, gv.w}, ua[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 p = __floats2bfloat162_rn(silu_f(bf_lo(ga[e])) * bf_lo(ua[e]), silu_f(bf_hi(ga[e])) * bf_hi(ua[e]));
        o[e] = *reinterpret_cast<const uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(act + t * INTER + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

// last row: final norm (f32 for the LM head, bf16 copy for the caller) (reference: prefill.cu:297-311)
__global__ void k_final_norm(const __nv_bfloat16* __restrict__ hidden_last, const __nv_bfloat16* __restrict__ w,
                             float* __restrict__ normed_f32, __nv_bfloat16* __restrict__ normed_bf16,
                             __nv_bfloat16* __restrict__ hidden_out) {
    pdl_enter();
    __shared__ float red[32];
    const size_t off = (size_t)blockIdx.x * HIDDEN;            // one block per row (the prompt's last row: one block)
    hidden_last += off; normed_f32 += off;
    if (normed_bf16) normed_bf16 += off;
    if (hidden_out) hidden_out += off;
    float v[2], ss = 0.f;
    for (int i = 0; i < 2; ++i) { v[i] = ld_bf(hidden_last + threadIdx.x + 512 * i); ss += v[i] * v[i]; }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < 16; ++i) tot += red[i];
    const float rstd = rsqrtf(tot * (1.0f / HIDDEN) + RMS_EPS);
    for (int i = 0; i < 2; ++i) {
        const int c = threadIdx.x + 512 * i;
        const float x = v[i] * rstd * (1.0f + ld_bf(w + c));
        normed_f32[c] = x;
        if (normed_bf16) normed_bf16[c] = __float2bfloat16_rn(x);
        if (hidden_out) hidden_out[c] = hidden_last[c];
    }
}

// logits = W x, per-block argmax (lowest index on ties) (reference: prefill.cu:314-339)
__global__ void __launch_bounds__(256) k_lm_head(const float* __restrict__ x, const __nv_bfloat16* __restrict__ W, int vocab,
                                                 float* __restrict__ bval, int* __restrict__ bidx) {
    pdl_enter();
    __shared__ float sv[8];
    __shared__ int si[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float xr[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int e = 0; e < 8; ++e) xr[i * 8 + e] = x[i * 256 + lane * 8 + e];
    }
    float best = -INFINITY;
    int besti = 0x7fffffff;
    for (int row = blockIdx.x * 8 + warp; row < vocab; row += gridDim.x * 8) {
        const uint4* wp = reinterpret_cast<const uint4*>(W + (size_t)row * HIDDEN) + lane;
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) acc = dot8(__ldg(wp + i * 32), xr + i * 8, acc);
        acc = warp_sum(acc);
        if (acc > best) { best = acc; besti = row; }
    }
    if (lane == 0) { sv[warp] = best; si[warp] = besti; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < besti)) { best = sv[w]; besti = si[w]; }
        bval[blockIdx.x] = best;
        bidx[blockIdx.x] = besti;
    }
}

__global__ void k_lm_reduce(const float* __restrict__ bval, const int* __restrict__ bidx, int n, int* __restrict__ out) {
    pdl_enter();
    bval += (size_t)blockIdx.x * n; bidx += (size_t)blockIdx.x * n; out += blockIdx.x;     // one block per row of logits
    float best = -INFINITY;
    int besti = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += 32) {
        const float v = bval[i];
        const int ix = bidx[i];
        if (v > best || (v == best && ix < besti)) { best = v; besti = ix; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
    }
    if (threadIdx.x == 0) *out = besti;
}

// ---- workspace -----------------------------------------------------------------------------------------

struct PrefillWs {
    int cap = 0;                    // tokens the buffers are sized for
    __nv_bfloat16 *hidden = nullptr, *normed = nullptr, *wide = nullptr, *z = nullptr, *act = nullptr;
    float *pre = nullptr, *o = nullptr, *beta = nullptr, *decay = nullptr, *kq = nullptr, *normed_f32 = nullptr, *bval = nullptr;
    int *bidx = nullptr, *err = nullptr;
    void* chunk_scratch = nullptr;
    void* select_scratch = nullptr;
    float* splitk = nullptr;        // f32 partial products of the K-split projections of short prompts
    size_t splitk_bytes = 0;
    // NVFP4 x NVFP4 prefill: the current GEMM input quantised to NVFP4 (codes, 128 x 4 scale tiles) and the constant 1
    // that stands in for an activation tensor scale
    uint8_t *q_packed = nullptr, *q_scales = nullptr;
    float* one = nullptr;
};
PrefillWs g_pws[64];
constexpr int SPLITK_MAX_TOKENS = 2048;     // longer prompts fill the SMs without a K-split
constexpr int LM_BLOCKS = 1184;     // 8 resident blocks of 256 threads on each of 148 SMs

// Grow-only.  Growing frees and reallocates every buffer, which (a) is illegal while `stream` is being captured
// into a CUDA graph and (b) invalidates the device pointers baked into graphs captured earlier: the first is
// refused here, the second is made visible through g_ws_generation (mk_prefill_workspace_generation()).
// Callers that capture graphs size the workspace once with mk_prefill_reserve() and never grow it afterwards.
unsigned g_ws_generation[64] = {0};
cudaError_t ensure_ws(PrefillWs& w, int S, cudaStream_t stream = nullptr, bool check_capture = false) {
    S = (S + 127) & ~127;           // whole 128-row blocks: the NVFP4 activation quantiser and its scale tiles work on those
    if (S <= w.cap) return cudaSuccess;
    if (check_capture) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
            return cudaErrorStreamCaptureUnsupported;
    }
    // work enqueued earlier (on any stream) may still use the buffers about to be freed
    cudaError_t es = cudaDeviceSynchronize();
    if (es != cudaSuccess) return es;
    ++g_ws_generation[&w - g_pws];
    void** ptrs[] = {(void**)&w.hidden, (void**)&w.normed, (void**)&w.wide, (void**)&w.z, (void**)&w.act, (void**)&w.pre,
                     (void**)&w.o, (void**)&w.beta, (void**)&w.decay, (void**)&w.kq, &w.chunk_scratch, &w.select_scratch,
                     (void**)&w.splitk, (void**)&w.q_packed, (void**)&w.q_scales};
    w.splitk_bytes = 0;
    for (void** p : ptrs) { if (*p) cudaFree(*p); *p = nullptr; }
    const size_t s = (size_t)S;
    const size_t sizes[] = {s * HIDDEN * 2, s * HIDDEN * 2, s * 2 * INTER * 2, s * DN_V * 2, s * INTER * 2,
                            s * DN_CONV_CH * 4, s * DN_V * 4, s * 16 * 16, 16, 16, dn_chunked_scratch_bytes(S), block_select_scratch_bytes(S),
                            (size_t)(S < SPLITK_MAX_TOKENS ? S : SPLITK_MAX_TOKENS) * 4 * HIDDEN * sizeof(float),
                            s * (INTER / 2), (s / 128) * (INTER / 64) * 512};
    for (int i = 0; i < 15; ++i) {
        cudaError_t e = cudaMalloc(ptrs[i], sizes[i]);
        if (e != cudaSuccess) { w.cap = 0; return e; }
    }
    if (!w.normed_f32) {
        cudaError_t e = cudaMalloc((void**)&w.normed_f32, HIDDEN * 4);
        if (e == cudaSuccess) e = cudaMalloc((void**)&w.bval, LM_BLOCKS * 4);
        if (e == cudaSuccess) e = cudaMalloc((void**)&w.bidx, LM_BLOCKS * 4);
        if (e == cudaSuccess) e = cudaMalloc((void**)&w.err, 4);
        if (e == cudaSuccess) e = cudaMemset(w.err, 0, 4);
        if (e == cudaSuccess) e = cudaMalloc((void**)&w.one, 16);
        const float one = 1.0f;
        if (e == cudaSuccess) e = cudaMemcpy(w.one, &one, 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return e;
        float tab[FA_ROT / 2];
        for (int i = 0; i < FA_ROT / 2; ++i) tab[i] = (float)(1.0 / pow(ROPE_THETA, (2.0 * i) / FA_ROT));
        e = cudaMemcpyToSymbol(c_pf_inv_freq, tab, sizeof(tab));
        if (e != cudaSuccess) return e;
    }
    w.cap = S;
    w.splitk_bytes = sizes[12];
    return cudaSuccess;
}

struct HostTable { const void* src = nullptr; int n = 0; size_t entry = 0; unsigned char rows[MAX_LAYERS * sizeof(LayerWeightsNVFP4)]; };
HostTable g_tables[64];
// host copy of a 224-byte-per-entry table (tensor-scale NVFP4), cached like the others
struct HostTableTS { const void* src = nullptr; int n = 0; LayerWeightsNVFP4TS rows[MAX_LAYERS]; };
HostTableTS g_tables_ts[64];
thread_local char g_perr[200] = "";
struct SparseCfg { bool enabled = false; double top_frac = 0.10; int window = 4, sink = 1; int rule = 0; float alpha = 0.f; int last_full = 0; };
SparseCfg g_sparse;
struct TailCfg { int n = 0; float* running_max = nullptr; };   // tail-attention scoring for the prompt compressor (drafter.cu)
TailCfg g_tail;
int g_attn_impl = 1;              // attention kernel: 1 = tcgen05 / TMEM (default), 0 = mma.sync
int g_fuse_glu = 1;               // 1 = SwiGLU in the gate|up product's epilogue (default), 0 = separate kernel
int g_fuse_norm = 1;              // 1 = RMSNorm in the kernel that adds the K parts of a split product (default), 0 = separate kernel
int g_scan_mode = 1;              // 1 = chunks of 64 on the tensor cores, 0 = token-serial recurrence
int pfail(int code, const char* what, cudaError_t e = cudaSuccess) {
    if (e != cudaSuccess) snprintf(g_perr, sizeof(g_perr), "%s: %s", what, cudaGetErrorString(e));
    else snprintf(g_perr, sizeof(g_perr), "%s", what);
    return code;
}

#define PF_CHECK(call, what)                                     \
    do {                                                         \
        cudaError_t e_ = (call);                                 \
        if (e_ != cudaSuccess) return pfail(MK_ERR_CUDA, what, e_); \
    } while (0)

}  // namespace
}  // namespace mk

extern "C" const char* mk_prefill_error(void) { return mk::g_perr; }
extern "C" int mk_prefill_reserve(int max_tokens) {
    using namespace mk;
    if (max_tokens < 1) return pfail(MK_ERR_BAD_ARG, "max_tokens must be positive");
    int dev = 0;
    PF_CHECK(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= 64) return pfail(MK_ERR_BAD_ARG, "device index out of range");
    PF_CHECK(ensure_ws(g_pws[dev], max_tokens < 64 ? 64 : max_tokens), "prefill workspace");
    return MK_OK;
}
extern "C" int mk_prefill_workspace_tokens(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    return mk::g_pws[dev].cap;
}
extern "C" unsigned int mk_prefill_workspace_generation(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    return mk::g_ws_generation[dev];
}
extern "C" void mk_prefill_forget_tables(void) {
    for (auto& t : mk::g_tables) { t.src = nullptr; t.n = 0; }
    for (auto& t : mk::g_tables_ts) { t.src = nullptr; t.n = 0; }
}
extern "C" int mk_prefill_set_block_sparse(int enable, double top_frac, int window, int sink) {
    if (enable && (!(top_frac >= 0.0 && top_frac <= 1.0) || window < 1 || sink < 0)) return MK_ERR_BAD_ARG;
    mk::g_sparse.enabled = enable != 0;
    if (enable) { mk::g_sparse.top_frac = top_frac; mk::g_sparse.window = window; mk::g_sparse.sink = sink; mk::g_sparse.rule = 0; }
    return MK_OK;
}
// The reference's keep rule instead of the ranking (dflash/src/flashprefill_select.cpp:27-84).
extern "C" int mk_prefill_set_block_sparse_threshold(int enable, float alpha, int window, int sink, int last_n_full) {
    if (enable && (!(alpha == alpha) || window < 1 || sink < 0 || last_n_full < 0)) return MK_ERR_BAD_ARG;
    mk::g_sparse.enabled = enable != 0;
    if (enable) {
        mk::g_sparse.rule = 1; mk::g_sparse.alpha = alpha; mk::g_sparse.window = window; mk::g_sparse.sink = sink;
        mk::g_sparse.last_full = last_n_full;
    }
    return MK_OK;
}
// Status word of the prefill kernels on the current device: 0 = no bounded wait has run out; 1 = a GEMM wait,
// 2 = a chunk-scan wait, 3 = an attention wait.  Synchronises the device (it reads device memory).
extern "C" int mk_prefill_status(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    mk::PrefillWs& w = mk::g_pws[dev];
    if (!w.err) return 0;
    int v = 0;
    if (cudaMemcpy(&v, w.err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return v;
}
extern "C" void mk_prefill_set_attention_impl(int tcgen05) { mk::g_attn_impl = tcgen05 ? 1 : 0; }
extern "C" void mk_prefill_set_fused_swiglu(int on) {     // 0 none, 1 both (default), 2 SwiGLU only, 3 RMSNorm only
    mk::g_fuse_glu = (on == 1 || on == 2) ? 1 : 0;
    mk::g_fuse_norm = (on == 1 || on == 3) ? 1 : 0;
}
extern "C" void mk_prefill_set_tail_scoring(int n_lookahead, float* running_max) {
    mk::g_tail.n = (n_lookahead > 0 && running_max) ? n_lookahead : 0;
    mk::g_tail.running_max = mk::g_tail.n ? running_max : nullptr;
}
extern "C" void mk_prefill_set_scan_mode(int chunked) { mk::g_scan_mode = chunked ? 1 : 0; }

namespace mk {
namespace {

// One layer's device pointers as the prefill uses them (bf16 unless noted).  Fused pointers ([q|k|v] rows and
// [gate|up] rows in one matrix) take precedence; otherwise the separate matrices are multiplied into column
// slices of the same activation buffers.
struct LayerView {
    int type = 0;
    const void *in_norm = nullptr, *post_norm = nullptr;
    const void *w_qkv = nullptr, *w_z = nullptr, *w_b = nullptr, *w_a = nullptr, *conv_w = nullptr, *a_log = nullptr,
               *dt_bias = nullptr, *dn_norm = nullptr, *w_out = nullptr;                       // DeltaNet
    const void *w_faqkv = nullptr, *w_q = nullptr, *w_k = nullptr, *w_v = nullptr, *q_norm = nullptr, *k_norm = nullptr,
               *w_o = nullptr;                                                                  // attention
    const void *w_gateup = nullptr, *w_gate = nullptr, *w_up = nullptr, *w_down = nullptr;      // MLP
    // NVFP4 x NVFP4 prefill: when fp4 is set, the projections above are these quantised matrices instead
    // (packed e2m1, E4M3 block scales in 128 x 4 tiles, device fp32 tensor scale); beta / alpha stay bf16
    struct W4 { const void* packed = nullptr; const void* scales = nullptr; const float* ts = nullptr; };
    bool fp4 = false;
    W4 x_qkv, x_z, x_out, x_q, x_k, x_v, x_o, x_gate, x_up, x_down;
};
struct LmView { const void* bf16 = nullptr; const void* packed = nullptr; const void* scales = nullptr; };

LayerView view_of(const LayerWeights& lw, const void* fused_faqkv, const void* fused_gateup) {
    LayerView v;
    v.type = lw.layer_type;
    v.in_norm = lw.ptrs[0];
    if (lw.layer_type == 0) {
        v.w_qkv = lw.ptrs[DN_W_QKV]; v.w_z = lw.ptrs[DN_W_Z]; v.w_b = lw.ptrs[DN_W_B]; v.w_a = lw.ptrs[DN_W_A];
        v.conv_w = lw.ptrs[DN_CONV_W]; v.a_log = lw.ptrs[DN_A_LOG]; v.dt_bias = lw.ptrs[DN_DT_BIAS];
        v.dn_norm = lw.ptrs[DN_NORM_W]; v.w_out = lw.ptrs[DN_W_OUT]; v.post_norm = lw.ptrs[DN_POST_NORM];
        v.w_gate = lw.ptrs[DN_W_GATE]; v.w_up = lw.ptrs[DN_W_UP]; v.w_down = lw.ptrs[DN_W_DOWN];
    } else {
        v.w_q = lw.ptrs[FA_W_Q]; v.w_k = lw.ptrs[FA_W_K]; v.w_v = lw.ptrs[FA_W_V]; v.q_norm = lw.ptrs[FA_Q_NORM];
        v.k_norm = lw.ptrs[FA_K_NORM]; v.w_o = lw.ptrs[FA_W_O]; v.post_norm = lw.ptrs[FA_POST_NORM];
        v.w_gate = lw.ptrs[FA_W_GATE]; v.w_up = lw.ptrs[FA_W_UP]; v.w_down = lw.ptrs[FA_W_DOWN];
        v.w_faqkv = fused_faqkv;
    }
    v.w_gateup = fused_gateup;
    return v;
}

// greedy argmax over a logit vector, lowest index on ties (one block)
__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ logits, int n, int* __restrict__ out) {
    pdl_enter();
    __shared__ float sv[32];
    __shared__ int si[32];
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += 1024) {
        const float v = logits[i];
        if (v > best) { best = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        best = sv[threadIdx.x]; bi = si[threadIdx.x];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
        }
        if (threadIdx.x == 0) *out = bi;
    }
}

// NVFP4 layer-weight format (groups of 32 along K, fp16 scales) -> bf16 matrix for the tensor-core GEMMs.
// One thread per 8 weights.  value = e2m1(code) * scale in f32, rounded to bf16 (the GEMM operand type):
// unlike the decode kernel, which multiplies the exact dequantised value, the prefill carries this rounding.
__global__ void k_dequant_a_bf16(const uint8_t* __restrict__ packed, const __half* __restrict__ scales,
                                 __nv_bfloat16* __restrict__ out, size_t n8, int cols) {
    pdl_enter();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    const size_t e0 = i * 8, row = e0 / cols;
    const int col = (int)(e0 - row * cols);
    const float sc = __half2float(scales[row * (cols / 32) + col / 32]);
    const uint32_t w = reinterpret_cast<const uint32_t*>(packed)[i];
    const float lut[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t b = (w >> (8 * k)) & 0xffu;
        const float lo = (b & 0x8u) ? -lut[b & 7u] : lut[b & 7u];
        const float hi = (b & 0x80u) ? -lut[(b >> 4) & 7u] : lut[(b >> 4) & 7u];
        const __nv_bfloat162 p2 = __floats2bfloat162_rn(lo * sc, hi * sc);
        o[k] = *reinterpret_cast<const uint32_t*>(&p2);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

struct NvScratch { __nv_bfloat16 *qkv = nullptr, *z = nullptr, *out = nullptr, *gateup = nullptr, *down = nullptr; float* logits = nullptr; };
NvScratch g_nvs[64];
float* g_logits[64] = {nullptr};

template <typename LayerSource>
int prefill_core(const int* token_ids, int seq_len, int* output_token, const void* embed_weight, LayerSource source,
                 int num_layers, const void* final_norm_w, LmView lm, void* fa_k_cache, void* fa_v_cache, void* dn_states,
                 void* conv_bufs, void* final_normed, void* hidden_bf16_out, int max_seq_len, int vocab, int dev,
                 cudaStream_t stream, bool source_ahead = false) {
    // source(li, view) is called once per layer, in order.  source_ahead: it may be called for layer li + 1 before the
    // last projection of layer li is enqueued (it only reads tables; a source that launches work of its own into
    // scratch shared between layers must not be)
    PrefillWs& w = g_pws[dev];
    PF_CHECK(ensure_ws(w, seq_len, stream, true), "prefill workspace (grow it with mk_prefill_reserve() before capturing a graph)");
    static bool scan_attr[64] = {false};
    if (!scan_attr[dev]) {
        PF_CHECK(cudaFuncSetAttribute(k_dn_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, SCAN_SMEM), "scan smem");
        scan_attr[dev] = true;
    }
    const int S = seq_len;
    typedef __nv_bfloat16 bf;
    auto gemm = [&](const void* A, const void* W, void* C, const void* R, int N, int K, int ldc) {
        return gemm_bf16_tn(A, W, C, R, S, N, K, K, ldc, w.err, w.splitk, w.splitk_bytes, stream);
    };
    // a projection into the residual stream followed by the RMSNorm of the result: for short prompts (K-split products)
    // the norm rides in the kernel that adds the K parts; `normed` says whether w.normed already holds it
    bool normed = false;
    auto gemm_norm = [&](const void* A, const void* W, int K, const void* norm_w) {
        return gemm_bf16_tn(A, W, w.hidden, w.hidden, S, HIDDEN, K, K, HIDDEN, w.err, w.splitk, w.splitk_bytes, stream,
                            g_fuse_norm ? norm_w : nullptr, w.normed, &normed);
    };
    // NVFP4 x NVFP4: quantise the [S, K] input of the coming projections once (16-element blocks along K, E4M3 block
    // scales, no tensor scale: the quantiser of the reference's LM-head format), then multiply on the block-scaled
    // tensor cores.  Rows S .. (S rounded up to 128) of the input are whatever the buffer holds: they are quantised
    // with the rest and never stored.
    const int S_pad = (S + 127) & ~127;
    auto quant = [&](const void* X, int K) {
        return launch_quantize_nvfp4_lm_out(X, S_pad, K, w.q_packed, w.q_scales, stream) == MK_OK ? cudaSuccess : cudaErrorInvalidValue;
    };
    auto gemm4 = [&](const LayerView::W4& W, void* C, const void* R, int N, int K, int ldc) {
        return gemm_nvfp4_tn(w.q_packed, w.q_scales, w.one, W.packed, W.scales, W.ts, C, R, S, N, K, ldc, w.err, stream);
    };
    const int wpb = 8;                                            // warps per 256-thread block
    auto blocks_for_warps = [&](long long nw) { return (unsigned)((nw + wpb - 1) / wpb); };

    const bool tail = g_tail.n > 0 && g_tail.running_max && S > g_tail.n;
    if (tail) PF_CHECK(cudaMemsetAsync(g_tail.running_max, 0, (size_t)g_tail.n * S * sizeof(float), stream), "tail score reset");
    launch_pdl(k_embed, S, 128, 0, stream, token_ids, (const bf*)embed_weight, w.hidden, S, vocab);
    int dn_idx = 0, fa_idx = 0;
    LayerView ahead;
    bool have_ahead = false;
    for (int li = 0; li < num_layers; ++li) {
        LayerView lv;
        if (have_ahead) {
            lv = ahead;
            have_ahead = false;
        } else {
            const int rc = source(li, lv);
            if (rc != MK_OK) return rc;
        }
        const bool dn = (lv.type == 0);
        if (!normed) launch_pdl(k_rmsnorm, blocks_for_warps(S), 256, 0, stream, w.hidden, (const bf*)lv.in_norm, w.normed, S);
        normed = false;
        if (dn) {
            float* state = (float*)dn_states + (size_t)dn_idx * DN_HEADS * DN_VAL * DN_KEY;
            float* cstate = (float*)conv_bufs + (size_t)dn_idx * DN_CONV_CH * DN_CONV_K;
            if (lv.fp4) {
                PF_CHECK(quant(w.normed, HIDDEN), "quantise activations");
                PF_CHECK(gemm4(lv.x_qkv, w.wide, nullptr, DN_CONV_CH, HIDDEN, DN_CONV_CH), "gemm qkv");
                PF_CHECK(gemm4(lv.x_z, w.z, nullptr, DN_V, HIDDEN, DN_V), "gemm z");
            } else {
                if (g_fuse_glu) {          // the qkv and the z projection as one launch over both weight matrices
                    PF_CHECK(gemm_bf16_tn_dual(w.normed, lv.w_qkv, w.wide, DN_CONV_CH, DN_CONV_CH, lv.w_z, w.z, DN_V, DN_V, S, HIDDEN, HIDDEN,
                                               w.err, stream), "gemm qkv + z");
                } else {
                    PF_CHECK(gemm(w.normed, lv.w_qkv, w.wide, nullptr, DN_CONV_CH, HIDDEN, DN_CONV_CH), "gemm qkv");
                    PF_CHECK(gemm(w.normed, lv.w_z, w.z, nullptr, DN_V, HIDDEN, DN_V), "gemm z");
                }
            }
            launch_pdl(k_dn_gates_mma, (unsigned)((S + 15) / 16), 256, 0, stream, w.normed, (const bf*)lv.w_b, (const bf*)lv.w_a,
                       (const bf*)lv.a_log, (const bf*)lv.dt_bias, w.beta, S);
            if (g_scan_mode == 0) {
                launch_pdl(k_dn_preproject, dim3(S, DN_HEADS), 128, 0, stream, w.wide, (const bf*)lv.conv_w, cstate, w.pre, w.beta, S);
                launch_pdl(k_dn_scan, 128, 512, SCAN_SMEM, stream, w.pre, w.beta, state, w.o, S);
            } else {
                PF_CHECK(dn_chunked(w.wide, lv.conv_w, cstate, w.beta, state, w.o, S, w.chunk_scratch, w.err, stream), "chunked scan");
            }
            launch_pdl(k_dn_conv_state, (DN_CONV_CH + 255) / 256, 256, 0, stream, w.wide, cstate, S);
            launch_pdl(k_dn_gated_norm, blocks_for_warps((long long)S * DN_HEADS), 256, 0, stream, w.o, w.z, (const bf*)lv.dn_norm, w.act, S);
            if (lv.fp4) {
                PF_CHECK(quant(w.act, DN_V), "quantise activations");
                PF_CHECK(gemm4(lv.x_out, w.hidden, w.hidden, HIDDEN, DN_V, HIDDEN), "gemm out");
            } else {
                PF_CHECK(gemm_norm(w.act, lv.w_out, DN_V, lv.post_norm), "gemm out");
            }
            ++dn_idx;
        } else {
            bf* kc = (bf*)fa_k_cache + (size_t)fa_idx * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;
            bf* vc = (bf*)fa_v_cache + (size_t)fa_idx * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;
            if (lv.fp4) {
                PF_CHECK(quant(w.normed, HIDDEN), "quantise activations");
                PF_CHECK(gemm4(lv.x_q, w.wide, nullptr, FA_QPROJ, HIDDEN, FA_QKV_ROWS), "gemm q");
                PF_CHECK(gemm4(lv.x_k, w.wide + FA_QPROJ, nullptr, FA_KV_SIZE, HIDDEN, FA_QKV_ROWS), "gemm k");
                PF_CHECK(gemm4(lv.x_v, w.wide + FA_QPROJ + FA_KV_SIZE, nullptr, FA_KV_SIZE, HIDDEN, FA_QKV_ROWS), "gemm v");
            } else if (lv.w_faqkv) {
                PF_CHECK(gemm(w.normed, lv.w_faqkv, w.wide, nullptr, FA_QKV_ROWS, HIDDEN, FA_QKV_ROWS), "gemm fa qkv");
            } else {
                PF_CHECK(gemm(w.normed, lv.w_q, w.wide, nullptr, FA_QPROJ, HIDDEN, FA_QKV_ROWS), "gemm q");
                PF_CHECK(gemm(w.normed, lv.w_k, w.wide + FA_QPROJ, nullptr, FA_KV_SIZE, HIDDEN, FA_QKV_ROWS), "gemm k");
                PF_CHECK(gemm(w.normed, lv.w_v, w.wide + FA_QPROJ + FA_KV_SIZE, nullptr, FA_KV_SIZE, HIDDEN, FA_QKV_ROWS), "gemm v");
            }
            launch_pdl(k_fa_norm_rope, blocks_for_warps((long long)S * 12), 256, 0, stream, w.wide, (const bf*)lv.q_norm, (const bf*)lv.k_norm, kc, vc, S, max_seq_len,
                       (const int*)nullptr, (size_t)0);
            if (tail) PF_CHECK(tail_attention_scores(w.wide, kc, S, max_seq_len, g_tail.n, g_tail.running_max, stream), "tail scores");
            const uint32_t* bmask = nullptr;
            if (g_sparse.enabled) {
                uint32_t* m = nullptr;
                PF_CHECK(block_select(w.wide, kc, S, max_seq_len, g_sparse.top_frac, g_sparse.window, g_sparse.sink,
                                      w.select_scratch, &m, stream, g_sparse.rule, g_sparse.alpha, g_sparse.last_full, nullptr),
                         "block selection");
                bmask = m;
            }
            if (g_attn_impl == 1) PF_CHECK(fa_prefill_tcgen05(w.wide, kc, vc, w.act, S, max_seq_len, w.err, bmask, stream), "attention");
            else PF_CHECK(fa_prefill(w.wide, kc, vc, w.act, S, max_seq_len, bmask, stream), "attention");
            if (lv.fp4) {
                PF_CHECK(quant(w.act, FA_Q_SIZE), "quantise activations");
                PF_CHECK(gemm4(lv.x_o, w.hidden, w.hidden, HIDDEN, FA_Q_SIZE, HIDDEN), "gemm o");
            } else {
                PF_CHECK(gemm_norm(w.act, lv.w_o, FA_Q_SIZE, lv.post_norm), "gemm o");
            }
            ++fa_idx;
        }
        if (!normed) launch_pdl(k_rmsnorm, blocks_for_warps(S), 256, 0, stream, w.hidden, (const bf*)lv.post_norm, w.normed, S);
        normed = false;
        if (lv.fp4) {
            PF_CHECK(quant(w.normed, HIDDEN), "quantise activations");
            PF_CHECK(gemm4(lv.x_gate, w.wide, nullptr, INTER, HIDDEN, 2 * INTER), "gemm gate");
            PF_CHECK(gemm4(lv.x_up, w.wide + INTER, nullptr, INTER, HIDDEN, 2 * INTER), "gemm up");
        } else if (lv.w_gateup && g_fuse_glu) {
            // gate | up product with the SwiGLU in its epilogue: straight to the down projection's input
            PF_CHECK(gemm_bf16_glu(w.normed, lv.w_gateup, w.act, S, INTER, HIDDEN, HIDDEN, INTER, INTER, w.err, stream), "gemm gate_up + SwiGLU");
        } else if (lv.w_gateup) {
            PF_CHECK(gemm(w.normed, lv.w_gateup, w.wide, nullptr, 2 * INTER, HIDDEN, 2 * INTER), "gemm gate_up");
        } else {
            PF_CHECK(gemm(w.normed, lv.w_gate, w.wide, nullptr, INTER, HIDDEN, 2 * INTER), "gemm gate");
            PF_CHECK(gemm(w.normed, lv.w_up, w.wide + INTER, nullptr, INTER, HIDDEN, 2 * INTER), "gemm up");
        }
        if (lv.fp4 || !lv.w_gateup || !g_fuse_glu)
            launch_pdl(k_silu_mul, (unsigned)(((size_t)S * (INTER / 8) + 255) / 256), 256, 0, stream, w.wide, w.act, S);
        if (lv.fp4) {
            PF_CHECK(quant(w.act, INTER), "quantise activations");
            PF_CHECK(gemm4(lv.x_down, w.hidden, w.hidden, HIDDEN, INTER, HIDDEN), "gemm down");
        } else {
            // the next layer's input norm, if there is a next layer
            const void* next_norm = nullptr;
            if (source_ahead && li + 1 < num_layers) {
                ahead = LayerView();
                const int rn = source(li + 1, ahead);
                if (rn != MK_OK) return rn;
                have_ahead = true;
                next_norm = ahead.in_norm;
            }
            PF_CHECK(gemm_norm(w.act, lv.w_down, INTER, next_norm), "gemm down");
        }
    }
    launch_pdl(k_final_norm, 1, 512, 0, stream, w.hidden + (size_t)(S - 1) * HIDDEN, (const bf*)final_norm_w, w.normed_f32,
                                        (bf*)final_normed, (bf*)hidden_bf16_out);
    if (lm.packed) {
        // NVFP4 LM head (16-block / E4M3 format): logits by the in-register dequantising row product, then argmax
        if (!g_logits[dev]) PF_CHECK(cudaMalloc((void**)&g_logits[dev], (size_t)DEFAULT_VOCAB * 4 * 2), "logits buffer");
        if (vocab > 2 * DEFAULT_VOCAB) return pfail(MK_ERR_BAD_ARG, "vocabulary too large for the logits buffer");
        if (mk_matvec_nvfp4(1, lm.packed, lm.scales, w.normed_f32, g_logits[dev], vocab, HIDDEN, 16, stream) != MK_OK)
            return pfail(MK_ERR_BAD_ARG, mk_nvfp4_error());
        launch_pdl(k_argmax, 1, 1024, 0, stream, g_logits[dev], vocab, output_token);
    } else {
        launch_pdl(k_lm_head, LM_BLOCKS, 256, 0, stream, w.normed_f32, (const bf*)lm.bf16, vocab, w.bval, w.bidx);
        launch_pdl(k_lm_reduce, 1, 32, 0, stream, w.bval, w.bidx, LM_BLOCKS, output_token);
    }
    PF_CHECK(cudaGetLastError(), "prefill launch");
    return MK_OK;
}

int check_common(const void* const* req, int nreq, int seq_len, int max_seq_len, int num_layers, int vocab, int& dev) {
    for (int i = 0; i < nreq; ++i) if (!req[i]) return pfail(MK_ERR_BAD_ARG, "null pointer argument");
    if (seq_len <= 0 || seq_len > max_seq_len) return pfail(MK_ERR_BAD_ARG, "seq_len must be in [1, max_seq_len]");
    if (num_layers < 1 || num_layers > MAX_LAYERS || vocab < 1) return pfail(MK_ERR_BAD_ARG, "bad model dimensions");
    PF_CHECK(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= 64) return pfail(MK_ERR_BAD_ARG, "device index out of range");
    return MK_OK;
}

// host copy of a pointer table (kept per device and table address, see mk_prefill_forget_tables)
int host_table(int dev, const void* layers, int num_layers, size_t entry, cudaStream_t stream, const unsigned char*& rows) {
    HostTable& ht = g_tables[dev];
    if (ht.src != layers || ht.n != num_layers || ht.entry != entry) {
        PF_CHECK(cudaMemcpyAsync(ht.rows, layers, (size_t)num_layers * entry, cudaMemcpyDeviceToHost, stream), "table copy");
        PF_CHECK(cudaStreamSynchronize(stream), "table copy sync");
        ht.src = layers; ht.n = num_layers; ht.entry = entry;
    }
    rows = ht.rows;
    return MK_OK;
}

#include "decode_batch.cuh"
#include "decode_batch_fp4.cuh"

}  // namespace
}  // namespace mk

// The host copy of the pointer table is kept per device and table address, as the reference keeps its own
// (megakernel/prefill.cu:1578-1584): a caller that rewrites a table in place must call
// mk_prefill_forget_tables() first.  With the copy cached a call enqueues work only (no synchronisation), so a
// whole prefill can be captured into a CUDA graph.
extern "C" int mk_prefill_bf16(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const MkLayerWeights* layers, const void* final_norm_w, const void* lm_head_w,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    const void* fused_fa_qkv_base, const void* fused_gate_up_base,
    void* final_normed, void* hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream) {
    using namespace mk;
    const void* req[] = {token_ids, output_token, embed_weight, layers, final_norm_w, lm_head_w, fa_k_cache, fa_v_cache, dn_states, conv_bufs};
    int dev = 0;
    int rc = check_common(req, 10, seq_len, max_seq_len, num_layers, vocab, dev);
    if (rc != MK_OK) return rc;
    const unsigned char* rows = nullptr;
    rc = host_table(dev, layers, num_layers, sizeof(LayerWeights), stream, rows);
    if (rc != MK_OK) return rc;
    const LayerWeights* hl = reinterpret_cast<const LayerWeights*>(rows);
    int fa_seen = 0;
    auto source = [&](int li, LayerView& lv) {
        const bool fa = hl[li].layer_type != 0;
        lv = view_of(hl[li],
                     (fa && fused_fa_qkv_base) ? (const __nv_bfloat16*)fused_fa_qkv_base + (size_t)fa_seen * FA_QKV_ROWS * HIDDEN : nullptr,
                     fused_gate_up_base ? (const __nv_bfloat16*)fused_gate_up_base + (size_t)li * 2 * INTER * HIDDEN : nullptr);
        if (fa) ++fa_seen;
        return (int)MK_OK;
    };
    LmView lm;
    lm.bf16 = lm_head_w;
    return prefill_core(token_ids, seq_len, output_token, embed_weight, source, num_layers, final_norm_w, lm, fa_k_cache,
                        fa_v_cache, dn_states, conv_bufs, final_normed, hidden_bf16_out, max_seq_len, vocab, dev, stream, true);
}

// bf16 layers, NVFP4 LM head (16-block / E4M3 format) for the first generated token
// (reference: launch_prefill_bf16_nvfp4_lm, megakernel/prefill_bw.cu:1486-1530).
extern "C" int mk_prefill_bf16_nvfp4_lm(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const MkLayerWeights* layers, const void* final_norm_w,
    const void* lm_head_weight_packed, const void* lm_head_scales,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* final_normed, void* hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream) {
    using namespace mk;
    const void* req[] = {token_ids, output_token, embed_weight, layers, final_norm_w, lm_head_weight_packed, lm_head_scales,
                         fa_k_cache, fa_v_cache, dn_states, conv_bufs};
    int dev = 0;
    int rc = check_common(req, 11, seq_len, max_seq_len, num_layers, vocab, dev);
    if (rc != MK_OK) return rc;
    if (vocab % 128) return pfail(MK_ERR_BAD_ARG, "the NVFP4 LM head needs a vocabulary that is a multiple of 128");
    const unsigned char* rows = nullptr;
    rc = host_table(dev, layers, num_layers, sizeof(LayerWeights), stream, rows);
    if (rc != MK_OK) return rc;
    const LayerWeights* hl = reinterpret_cast<const LayerWeights*>(rows);
    auto source = [&](int li, LayerView& lv) { lv = view_of(hl[li], nullptr, nullptr); return (int)MK_OK; };
    LmView lm;
    lm.packed = lm_head_weight_packed; lm.scales = lm_head_scales;
    return prefill_core(token_ids, seq_len, output_token, embed_weight, source, num_layers, final_norm_w, lm, fa_k_cache,
                        fa_v_cache, dn_states, conv_bufs, final_normed, hidden_bf16_out, max_seq_len, vocab, dev, stream, true);
}

// Prefill on NVFP4 weights (208-byte table): every quantised matrix of a layer is dequantised into bf16 scratch
// right before the layer runs, then the bf16 pipeline is used; NVFP4 LM head.
// (reference: launch_prefill_megakernel_nvfp4, megakernel/kernel_gb10_nvfp4.cu:2127-2190)
extern "C" int mk_prefill_nvfp4(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const void* layers, const void* final_norm_w,
    const void* lm_head_weight_packed, const void* lm_head_scales,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* final_normed, void* hidden_bf16_out,
    int max_seq_len, int group_size, int num_layers, int vocab, cudaStream_t stream) {
    using namespace mk;
    const void* req[] = {token_ids, output_token, embed_weight, layers, final_norm_w, lm_head_weight_packed, lm_head_scales,
                         fa_k_cache, fa_v_cache, dn_states, conv_bufs};
    int dev = 0;
    int rc = check_common(req, 11, seq_len, max_seq_len, num_layers, vocab, dev);
    if (rc != MK_OK) return rc;
    if (group_size != 32) return pfail(MK_ERR_BAD_ARG, "group_size must be 32");
    if (vocab % 128) return pfail(MK_ERR_BAD_ARG, "the NVFP4 LM head needs a vocabulary that is a multiple of 128");
    const unsigned char* rows = nullptr;
    rc = host_table(dev, layers, num_layers, sizeof(LayerWeightsNVFP4), stream, rows);
    if (rc != MK_OK) return rc;
    const LayerWeightsNVFP4* hl = reinterpret_cast<const LayerWeightsNVFP4*>(rows);
    NvScratch& ns = g_nvs[dev];
    if (!ns.qkv) {
        PF_CHECK(cudaMalloc((void**)&ns.qkv, (size_t)DN_CONV_CH * HIDDEN * 2), "dequant scratch");
        PF_CHECK(cudaMalloc((void**)&ns.z, (size_t)DN_V * HIDDEN * 2), "dequant scratch");
        PF_CHECK(cudaMalloc((void**)&ns.out, (size_t)HIDDEN * DN_V * 2), "dequant scratch");
        PF_CHECK(cudaMalloc((void**)&ns.gateup, (size_t)2 * INTER * HIDDEN * 2), "dequant scratch");
        PF_CHECK(cudaMalloc((void**)&ns.down, (size_t)HIDDEN * INTER * 2), "dequant scratch");
    }
    auto deq = [&](const void* packed, const void* scales, __nv_bfloat16* out, int rws, int cols) {
        const size_t n8 = (size_t)rws * cols / 8;
        launch_pdl(k_dequant_a_bf16, (unsigned)((n8 + 255) / 256), 256, 0, stream, (const uint8_t*)packed, (const __half*)scales, out, n8, cols);
    };
    // slots of the 208-byte table (reference: megakernel/model_nvfp4.py:274-311)
    auto source = [&](int li, LayerView& lv) {
        const LayerWeightsNVFP4& t = hl[li];
        lv.type = t.layer_type;
        lv.in_norm = t.ptrs[0];
        if (t.layer_type == 0) {
            deq(t.ptrs[1], t.ptrs[2], ns.qkv, DN_CONV_CH, HIDDEN);
            deq(t.ptrs[3], t.ptrs[4], ns.z, DN_V, HIDDEN);
            deq(t.ptrs[11], t.ptrs[12], ns.out, HIDDEN, DN_V);
            deq(t.ptrs[14], t.ptrs[15], ns.gateup, INTER, HIDDEN);
            deq(t.ptrs[16], t.ptrs[17], ns.gateup + (size_t)INTER * HIDDEN, INTER, HIDDEN);
            deq(t.ptrs[18], t.ptrs[19], ns.down, HIDDEN, INTER);
            lv.w_qkv = ns.qkv; lv.w_z = ns.z; lv.w_b = t.ptrs[5]; lv.w_a = t.ptrs[6]; lv.conv_w = t.ptrs[7];
            lv.a_log = t.ptrs[8]; lv.dt_bias = t.ptrs[9]; lv.dn_norm = t.ptrs[10]; lv.w_out = ns.out; lv.post_norm = t.ptrs[13];
        } else {
            deq(t.ptrs[1], t.ptrs[2], ns.qkv, FA_QPROJ, HIDDEN);
            deq(t.ptrs[3], t.ptrs[4], ns.qkv + (size_t)FA_QPROJ * HIDDEN, FA_KV_SIZE, HIDDEN);
            deq(t.ptrs[5], t.ptrs[6], ns.qkv + (size_t)(FA_QPROJ + FA_KV_SIZE) * HIDDEN, FA_KV_SIZE, HIDDEN);
            deq(t.ptrs[9], t.ptrs[10], ns.out, HIDDEN, FA_Q_SIZE);
            deq(t.ptrs[12], t.ptrs[13], ns.gateup, INTER, HIDDEN);
            deq(t.ptrs[14], t.ptrs[15], ns.gateup + (size_t)INTER * HIDDEN, INTER, HIDDEN);
            deq(t.ptrs[16], t.ptrs[17], ns.down, HIDDEN, INTER);
            lv.w_faqkv = ns.qkv; lv.q_norm = t.ptrs[7]; lv.k_norm = t.ptrs[8]; lv.w_o = ns.out; lv.post_norm = t.ptrs[11];
        }
        lv.w_gateup = ns.gateup; lv.w_down = ns.down;
        return cudaGetLastError() == cudaSuccess ? (int)MK_OK : pfail(MK_ERR_CUDA, "dequantise launch");
    };
    LmView lm;
    lm.packed = lm_head_weight_packed; lm.scales = lm_head_scales;
    return prefill_core(token_ids, seq_len, output_token, embed_weight, source, num_layers, final_norm_w, lm, fa_k_cache,
                        fa_v_cache, dn_states, conv_bufs, final_normed, hidden_bf16_out, max_seq_len, vocab, dev, stream);
}

extern "C" int launch_prefill_bf16(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const MkLayerWeights* layers,
    const void* final_norm_w, const void* lm_head_w,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden, void* residual, void* normalized,
    void* proj_buf, void* proj_buf2, void* attn_buf, void* mlp_buf,
    void* dn_out_buf, void* beta_buf, void* alpha_buf, void* dn_pre_qkv,
    void* dn_u_scratch, void* dn_w_scratch, void* dn_cs_scratch,
    const void* fused_fa_qkv_base, const void* fused_gate_up_base,
    void* final_normed, void* hidden_bf16_out,
    void* lm_bmv, void* lm_bmi,
    int max_seq_len, cudaStream_t stream) {
    (void)hidden; (void)residual; (void)normalized; (void)proj_buf; (void)proj_buf2; (void)attn_buf; (void)mlp_buf;
    (void)dn_out_buf; (void)beta_buf; (void)alpha_buf; (void)dn_pre_qkv; (void)dn_u_scratch; (void)dn_w_scratch;
    (void)dn_cs_scratch; (void)lm_bmv; (void)lm_bmi;
    int nl = 0, vocab = 0;
    mk_get_model_dims(&nl, &vocab);
    return mk_prefill_bf16(token_ids, seq_len, output_token, embed_weight, layers, final_norm_w, lm_head_w, fa_k_cache,
                           fa_v_cache, dn_states, conv_bufs, fused_fa_qkv_base, fused_gate_up_base, final_normed,
                           hidden_bf16_out, max_seq_len, nl, vocab, stream);
}

// ---- the reference's other prefill entry points, same argument lists ---------------------------------------
// Two of them carry no max_seq_len (the reference compiles the cache stride in): the stride is taken from
// mk_set_prefill_max_seq_len (default 2048, the reference's MAX_SEQ_LEN); the torch ops set it from the cache
// tensor's shape.
namespace mk { namespace { int g_default_max_seq = 2048; } }
extern "C" void mk_set_prefill_max_seq_len(int max_seq_len) { if (max_seq_len > 0) mk::g_default_max_seq = max_seq_len; }

extern "C" int launch_prefill_bf16_mega(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const MkLayerWeights* layers,
    const void* final_norm_w, const void* lm_head_w,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden, void* residual, void* normalized,
    void* proj_buf, void* proj_buf2, void* attn_buf, void* mlp_buf,
    void* dn_out_buf, void* beta_buf, void* alpha_buf,
    void* final_normed, void* hidden_bf16_out,
    void* lm_bmv, void* lm_bmi, cudaStream_t stream) {
    (void)hidden; (void)residual; (void)normalized; (void)proj_buf; (void)proj_buf2; (void)attn_buf; (void)mlp_buf;
    (void)dn_out_buf; (void)beta_buf; (void)alpha_buf; (void)lm_bmv; (void)lm_bmi;
    int nl = 0, vocab = 0;
    mk_get_model_dims(&nl, &vocab);
    return mk_prefill_bf16(token_ids, seq_len, output_token, embed_weight, layers, final_norm_w, lm_head_w, fa_k_cache,
                           fa_v_cache, dn_states, conv_bufs, nullptr, nullptr, final_normed, hidden_bf16_out,
                           mk::g_default_max_seq, nl, vocab, stream);
}

extern "C" int launch_prefill_bf16_nvfp4_lm(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const MkLayerWeights* layers, const void* fused_layers,
    const void* final_norm_w, const void* lm_head_w,
    const void* lm_head_weight_packed, const void* lm_head_scales,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden, void* residual, void* normalized,
    void* proj_buf, void* proj_buf2, void* proj_buf_half, void* proj_act_packed, void* proj_act_scales,
    void* attn_buf, void* mlp_buf, void* dn_out_buf, void* beta_buf, void* alpha_buf,
    void* final_normed, void* hidden_bf16_out, void* lm_bmv, void* lm_bmi,
    void* lm_hidden_bf16, void* lm_hidden_packed, void* lm_hidden_scales, void* lm_logits_f16, cudaStream_t stream) {
    (void)fused_layers; (void)lm_head_w; (void)hidden; (void)residual; (void)normalized; (void)proj_buf; (void)proj_buf2;
    (void)proj_buf_half; (void)proj_act_packed; (void)proj_act_scales; (void)attn_buf; (void)mlp_buf; (void)dn_out_buf;
    (void)beta_buf; (void)alpha_buf; (void)lm_bmv; (void)lm_bmi; (void)lm_hidden_bf16; (void)lm_hidden_packed;
    (void)lm_hidden_scales; (void)lm_logits_f16;
    int nl = 0, vocab = 0;
    mk_get_model_dims(&nl, &vocab);
    return mk_prefill_bf16_nvfp4_lm(token_ids, seq_len, output_token, embed_weight, layers, final_norm_w, lm_head_weight_packed,
                                    lm_head_scales, fa_k_cache, fa_v_cache, dn_states, conv_bufs, final_normed, hidden_bf16_out,
                                    mk::g_default_max_seq, nl, vocab, stream);
}

extern "C" int launch_prefill_megakernel_nvfp4(
    const int* token_ids, int seq_len, int* output_token_id,
    const void* embed_weight, const void* layer_weights, const void* final_norm_weight,
    const void* lm_head_weight_packed, const void* lm_head_scales,
    void* lm_hidden_bf16, void* lm_hidden_packed, void* lm_hidden_scales, void* lm_logits_f16,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer, void* g_activations, void* g_residual,
    void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch,
    void* g_alpha_scratch, void* g_normalized,
    unsigned int* barrier_counter, unsigned int* barrier_generation,
    float* block_max_vals, int* block_max_idxs, unsigned int* lm_sync_counter,
    int max_seq_len, int group_size, cudaStream_t stream) {
    (void)lm_hidden_bf16; (void)lm_hidden_packed; (void)lm_hidden_scales; (void)lm_logits_f16; (void)g_activations;
    (void)g_residual; (void)g_qkv_scratch; (void)g_kv_scratch; (void)g_attn_out; (void)g_mlp_inter; (void)g_z_scratch;
    (void)g_beta_scratch; (void)g_alpha_scratch; (void)g_normalized; (void)barrier_counter; (void)barrier_generation;
    (void)block_max_vals; (void)block_max_idxs; (void)lm_sync_counter;
    int nl = 0, vocab = 0;
    mk_get_model_dims(&nl, &vocab);
    // the reference leaves the last row of the residual stream in hidden_buffer for the decode steps that follow
    return mk_prefill_nvfp4(token_ids, seq_len, output_token_id, embed_weight, layer_weights, final_norm_weight,
                            lm_head_weight_packed, lm_head_scales, fa_k_cache, fa_v_cache, dn_states, conv_bufs, nullptr,
                            hidden_buffer, max_seq_len, group_size, nl, vocab, stream);
}

// Prefill with NVFP4 weights AND NVFP4 activations on the block-scaled tensor cores: every projection input is
// quantised per 16 values along K (E4M3 block scales) and multiplied with the quantised weights by
// tcgen05.mma kind::mxf4nvf4; nothing is dequantised to bf16.  layers: 224-byte entries as for mk_decode_nvfp4_ts, but
// the scale slot of each matrix points at the 128 x 4 scale TILES the quantiser writes (not at plain rows).
extern "C" int mk_prefill_nvfp4_mma(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const void* layers, const void* final_norm_w,
    const void* lm_head_packed, const void* lm_head_scales_tiled,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* final_normed, void* hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream) {
    using namespace mk;
    const void* req[] = {token_ids, output_token, embed_weight, layers, final_norm_w, lm_head_packed, lm_head_scales_tiled,
                         fa_k_cache, fa_v_cache, dn_states, conv_bufs};
    int dev = 0;
    int rc = check_common(req, 11, seq_len, max_seq_len, num_layers, vocab, dev);
    if (rc != MK_OK) return rc;
    if (vocab % 128) return pfail(MK_ERR_BAD_ARG, "the NVFP4 LM head needs a vocabulary that is a multiple of 128");
    HostTableTS& ht = g_tables_ts[dev];
    if (ht.src != layers || ht.n != num_layers) {
        PF_CHECK(cudaMemcpyAsync(ht.rows, layers, (size_t)num_layers * sizeof(LayerWeightsNVFP4TS), cudaMemcpyDeviceToHost, stream), "table copy");
        PF_CHECK(cudaStreamSynchronize(stream), "table copy sync");
        ht.src = layers; ht.n = num_layers;
    }
    const LayerWeightsNVFP4TS* hl = ht.rows;
    auto source = [&](int li, LayerView& lv) -> int {
        const LayerWeightsNVFP4TS& e = hl[li];
        auto m = [&](int slot) { return LayerView::W4{e.ptrs[slot], e.ptrs[slot + 1], (const float*)e.ptrs[slot + 2]}; };
        lv.type = e.layer_type;
        lv.fp4 = true;
        lv.in_norm = e.ptrs[0];
        if (e.layer_type == 0) {   // in_norm, qkv(3), z(3), w_beta, w_alpha, conv_w, A_log, dt_bias, norm_w, out(3), post_norm, gate(3), up(3), down(3)
            lv.x_qkv = m(1); lv.x_z = m(4); lv.w_b = e.ptrs[7]; lv.w_a = e.ptrs[8]; lv.conv_w = e.ptrs[9]; lv.a_log = e.ptrs[10];
            lv.dt_bias = e.ptrs[11]; lv.dn_norm = e.ptrs[12]; lv.x_out = m(13); lv.post_norm = e.ptrs[16];
            lv.x_gate = m(17); lv.x_up = m(20); lv.x_down = m(23);
        } else {                   // in_norm, q(3), k(3), v(3), q_norm, k_norm, o(3), post_norm, gate(3), up(3), down(3)
            lv.x_q = m(1); lv.x_k = m(4); lv.x_v = m(7); lv.q_norm = e.ptrs[10]; lv.k_norm = e.ptrs[11]; lv.x_o = m(12);
            lv.post_norm = e.ptrs[15]; lv.x_gate = m(16); lv.x_up = m(19); lv.x_down = m(22);
        }
        return MK_OK;
    };
    LmView lm;
    lm.packed = lm_head_packed; lm.scales = lm_head_scales_tiled;     // the LM head's tensor scale is positive: the argmax does not need it
    return prefill_core(token_ids, seq_len, output_token, embed_weight, source, num_layers, final_norm_w, lm, fa_k_cache, fa_v_cache,
                        dn_states, conv_bufs, final_normed, hidden_bf16_out, max_seq_len, vocab, dev, stream);
}

// The attention building blocks on their own (tests call these through the C ABI).
extern "C" int mk_block_select(const void* qkv, const void* k_cache, int seq_len, int max_seq_len, double top_frac, int window,
                               int sink, unsigned int* mask_out, void* scratch, cudaStream_t stream) {
    using namespace mk;
    if (!qkv || !k_cache || !mask_out || !scratch || seq_len < 1 || seq_len > max_seq_len || window < 1 || sink < 0)
        return pfail(MK_ERR_BAD_ARG, "bad argument");
    uint32_t* m = nullptr;
    PF_CHECK(block_select(qkv, k_cache, seq_len, max_seq_len, top_frac, window, sink, scratch, &m, stream), "block selection");
    const int nblk = (seq_len + 127) / 128, nwords = (nblk + 31) / 32;
    PF_CHECK(cudaMemcpyAsync(mask_out, m, (size_t)8 * nblk * nwords * 4, cudaMemcpyDeviceToDevice, stream), "mask copy");
    return MK_OK;
}
extern "C" int mk_block_select_threshold(const void* qkv, const void* k_cache, int seq_len, int max_seq_len, float alpha, int window,
                                         int sink, int last_n_full, unsigned int* mask_out, float* scores_out, void* scratch,
                                         cudaStream_t stream) {
    using namespace mk;
    if (!qkv || !k_cache || !mask_out || !scratch || seq_len < 1 || seq_len > max_seq_len || window < 1 || sink < 0 ||
        last_n_full < 0 || !(alpha == alpha))
        return pfail(MK_ERR_BAD_ARG, "bad argument");
    uint32_t* m = nullptr;
    PF_CHECK(block_select(qkv, k_cache, seq_len, max_seq_len, 0.0, window, sink, scratch, &m, stream, 1, alpha, last_n_full, scores_out),
             "block selection");
    const int nblk = (seq_len + 127) / 128, nwords = (nblk + 31) / 32;
    PF_CHECK(cudaMemcpyAsync(mask_out, m, (size_t)8 * nblk * nwords * 4, cudaMemcpyDeviceToDevice, stream), "mask copy");
    return MK_OK;
}
extern "C" size_t mk_block_select_scratch_bytes(int seq_len) { return mk::block_select_scratch_bytes(seq_len); }
extern "C" int mk_attention_prefill(const void* qkv, const void* k_cache, const void* v_cache, void* out, int seq_len, int max_seq_len,
                                    const unsigned int* mask, cudaStream_t stream) {
    using namespace mk;
    if (!qkv || !k_cache || !v_cache || !out || seq_len < 1 || seq_len > max_seq_len) return pfail(MK_ERR_BAD_ARG, "bad argument");
    if (g_attn_impl == 1) {
        int dev = 0;
        PF_CHECK(cudaGetDevice(&dev), "cudaGetDevice");
        PrefillWs& w = g_pws[dev < 0 || dev >= 64 ? 0 : dev];
        PF_CHECK(ensure_ws(w, 1), "prefill workspace");
        PF_CHECK(fa_prefill_tcgen05(qkv, k_cache, v_cache, out, seq_len, max_seq_len, w.err, mask, stream), "attention");
    } else {
        PF_CHECK(fa_prefill(qkv, k_cache, v_cache, out, seq_len, max_seq_len, mask, stream), "attention");
    }
    return MK_OK;
}

// ---- batched decode (no counterpart in the reference: every op of megakernel/torch_bindings.cpp:569-675 is batch 1) ----
namespace mk {
namespace {
int decode_batch_entry(int steps, int* tokens, int* positions, int* output_tokens, int* tokens_log, int batch,
                       const void* embed_weight, const MkLayerWeights* layers, const void* final_norm_w, const void* lm_head_w,
                       void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
                       const void* fused_fa_qkv_base, const void* fused_gate_up_base, void* final_normed,
                       void* hidden_bf16_out, int max_seq_len, int num_layers, int vocab, cudaStream_t stream) {
    const void* req[] = {tokens, positions, embed_weight, layers, final_norm_w, lm_head_w, fa_k_cache, fa_v_cache, dn_states, conv_bufs};
    int dev = 0;
    int rc = check_common(req, 10, 1, max_seq_len, num_layers, vocab, dev);
    if (rc != MK_OK) return rc;
    if (batch < 1 || batch > BATCH_MAX) return pfail(MK_ERR_BAD_ARG, "batch must be in [1, 16]");
    if (steps < 1 || (steps > 1 && !tokens_log) || (steps == 1 && !output_tokens && !tokens_log))
        return pfail(MK_ERR_BAD_ARG, "bad step count or missing output");
    const unsigned char* rows = nullptr;
    rc = host_table(dev, layers, num_layers, sizeof(LayerWeights), stream, rows);
    if (rc != MK_OK) return rc;
    const LayerWeights* hl = reinterpret_cast<const LayerWeights*>(rows);
    int n_fa = 0;
    for (int li = 0; li < num_layers; ++li) n_fa += hl[li].layer_type != 0;
    const int n_dn = num_layers - n_fa;
    int fa_seen = 0;
    auto source = [&](int li, LayerView& lv) {
        const bool fa = hl[li].layer_type != 0;
        lv = view_of(hl[li],
                     (fa && fused_fa_qkv_base) ? (const __nv_bfloat16*)fused_fa_qkv_base + (size_t)fa_seen * FA_QKV_ROWS * HIDDEN : nullptr,
                     fused_gate_up_base ? (const __nv_bfloat16*)fused_gate_up_base + (size_t)li * 2 * INTER * HIDDEN : nullptr);
        if (fa) ++fa_seen;
        return (int)MK_OK;
    };
    if (steps == 1 && output_tokens)
        return decode_batch_core(tokens, positions, output_tokens, batch, embed_weight, source, num_layers, n_fa, n_dn, final_norm_w,
                                 lm_head_w, fa_k_cache, fa_v_cache, dn_states, conv_bufs, final_normed, hidden_bf16_out,
                                 max_seq_len, vocab, dev, stream);
    PF_CHECK(ensure_batch_ws(g_bws[dev]), "batch workspace");
    for (int s = 0; s < steps; ++s) {
        fa_seen = 0;
        rc = decode_batch_core(tokens, positions, g_bws[dev].chosen, batch, embed_weight, source, num_layers, n_fa, n_dn,
                               final_norm_w, lm_head_w, fa_k_cache, fa_v_cache, dn_states, conv_bufs, final_normed,
                               hidden_bf16_out, max_seq_len, vocab, dev, stream);
        if (rc != MK_OK) return rc;
        launch_pdl(k_batch_advance, 1, 32, 0, stream, tokens, (const int*)g_bws[dev].chosen, positions, tokens_log + (size_t)s * batch, batch);
    }
    PF_CHECK(cudaGetLastError(), "batched steps launch");
    return MK_OK;
}
}  // namespace
}  // namespace mk

// Batched step(s) on the tensor-scale NVFP4 weights: the arguments of mk_decode_batch / mk_decode_batch_many with the
// 224-byte table and the LM head's three tensors in place of the bf16 ones.
extern "C" int mk_decode_batch_nvfp4_ts(
    int steps, int* tokens, int* positions, int* output_tokens, int* tokens_log, int batch,
    const void* embed_weight, const void* layers, const void* final_norm_w,
    const void* lm_head_packed, const void* lm_head_scales_rows, const float* lm_head_tensor_scale,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs, void* final_normed, void* hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream) {
    using namespace mk;
    const void* req[] = {tokens, positions, embed_weight, layers, final_norm_w, lm_head_packed, lm_head_scales_rows,
                         lm_head_tensor_scale, fa_k_cache, fa_v_cache, dn_states, conv_bufs};
    int dev = 0;
    int rc = check_common(req, 12, 1, max_seq_len, num_layers, vocab, dev);
    if (rc != MK_OK) return rc;
    if (batch < 1 || batch > BATCH_MAX) return pfail(MK_ERR_BAD_ARG, "batch must be in [1, 16]");
    if (steps < 1 || (steps > 1 && !tokens_log) || (steps == 1 && !output_tokens && !tokens_log))
        return pfail(MK_ERR_BAD_ARG, "bad step count or missing output");
    HostTableTS& ht = g_tables_ts[dev];
    if (ht.src != layers || ht.n != num_layers) {
        PF_CHECK(cudaMemcpyAsync(ht.rows, layers, (size_t)num_layers * sizeof(LayerWeightsNVFP4TS), cudaMemcpyDeviceToHost, stream), "table copy");
        PF_CHECK(cudaStreamSynchronize(stream), "table copy sync");
        ht.src = layers; ht.n = num_layers;
    }
    int n_fa = 0;
    for (int li = 0; li < num_layers; ++li) n_fa += ht.rows[li].layer_type != 0;
    const int n_dn = num_layers - n_fa;
    const Fp4Mat lm{(const uint8_t*)lm_head_packed, (const uint8_t*)lm_head_scales_rows, lm_head_tensor_scale};
    if (steps == 1 && output_tokens)
        return decode_batch_core_fp4(tokens, positions, output_tokens, batch, embed_weight, ht.rows, num_layers, n_fa, n_dn, final_norm_w,
                                     lm, fa_k_cache, fa_v_cache, dn_states, conv_bufs, final_normed, hidden_bf16_out, max_seq_len,
                                     vocab, dev, stream);
    PF_CHECK(ensure_batch_ws(g_bws[dev]), "batch workspace");
    for (int s = 0; s < steps; ++s) {
        rc = decode_batch_core_fp4(tokens, positions, g_bws[dev].chosen, batch, embed_weight, ht.rows, num_layers, n_fa, n_dn,
                                   final_norm_w, lm, fa_k_cache, fa_v_cache, dn_states, conv_bufs, final_normed, hidden_bf16_out,
                                   max_seq_len, vocab, dev, stream);
        if (rc != MK_OK) return rc;
        launch_pdl(k_batch_advance, 1, 32, 0, stream, tokens, (const int*)g_bws[dev].chosen, positions, tokens_log + (size_t)s * batch, batch);
    }
    PF_CHECK(cudaGetLastError(), "batched steps launch");
    return MK_OK;
}

extern "C" void mk_decode_batch_set_residual_kernel(int mode) { mk::g_batch_res_kernel = (mode >= 0 && mode <= 2) ? mode : 1; }
extern "C" void mk_decode_batch_set_lm_head(int tensor_cores) { mk::g_batch_lm_mma = tensor_cores ? 1 : 0; }

extern "C" int mk_decode_batch(
    const int* tokens, const int* positions, int* output_tokens, int batch,
    const void* embed_weight, const MkLayerWeights* layers, const void* final_norm_w, const void* lm_head_w,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    const void* fused_fa_qkv_base, const void* fused_gate_up_base, void* final_normed, void* hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream) {
    if (!output_tokens) return mk::pfail(MK_ERR_BAD_ARG, "null pointer argument");
    return mk::decode_batch_entry(1, const_cast<int*>(tokens), const_cast<int*>(positions), output_tokens, nullptr, batch,
                                  embed_weight, layers, final_norm_w, lm_head_w, fa_k_cache, fa_v_cache, dn_states, conv_bufs,
                                  fused_fa_qkv_base, fused_gate_up_base, final_normed, hidden_bf16_out, max_seq_len, num_layers,
                                  vocab, stream);
}

extern "C" int mk_decode_batch_many(
    int steps, int* tokens, int* positions, int* tokens_log, int batch,
    const void* embed_weight, const MkLayerWeights* layers, const void* final_norm_w, const void* lm_head_w,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    const void* fused_fa_qkv_base, const void* fused_gate_up_base,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream) {
    if (!tokens_log) return mk::pfail(MK_ERR_BAD_ARG, "null pointer argument");
    return mk::decode_batch_entry(steps, tokens, positions, nullptr, tokens_log, batch, embed_weight, layers, final_norm_w,
                                  lm_head_w, fa_k_cache, fa_v_cache, dn_states, conv_bufs, fused_fa_qkv_base,
                                  fused_gate_up_base, nullptr, nullptr, max_seq_len, num_layers, vocab, stream);
}
