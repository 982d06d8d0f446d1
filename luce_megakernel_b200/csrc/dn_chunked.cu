// Gated delta rule in chunked form (chunks of 64 tokens) for prefill.
//
// Per head, with state S[value j][key i], per-token log-decay g, write strength beta, and the
// normalised q, k and the value v (reference statements: megakernel/prefill.cu:355-490 for the
// chunk-parallel preparation and :507-680 for the chunk-serial pass; the reference uses chunks
// of 8, the formulas are those of its recurrent form prefill.cu:114-221 regrouped):
//
//   inside a chunk, G_r = sum_{s<=r} g_s, Gam_r = exp(G_r)
//   A[s][u] = beta_s exp(G_s - G_u) (k_s . k_u)   for u < s          (strictly lower)
//   T = (I + A)^-1
//   W = T (beta Gam k)     [64 x 128 keys]        U = T (beta v)      [64 x 128 values]
//   P[r][s] = exp(G_r - G_s) (q_r . k_s)          for s <= r
//   D = U - W S0^T                                  (the per-token write vectors)
//   O = (Gam q) S0^T + P D
//   S1 = Gam_last S0 + D^T (exp(G_last - G_s) k_s)
//
// k_dn_chunk_prepare computes everything that does not depend on S0 for all (chunk, head) pairs in
// parallel; k_dn_chunk_scan walks the chunks of one head serially, one CTA per (head, 16 value
// rows), state in f32 accumulator registers, every product on mma.sync (fp16 operands: all of them
// are bounded by construction and fp16 carries three more mantissa bits than bf16; f32 accumulate;
// T and the state enter as two fp16 terms hi + lo).  The serial pass computes D, O
// and S transposed (value rows as the MMA M dimension), so D goes from accumulator registers to
// the next MMA through 2 KB of shared memory and the state never leaves registers.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "mk_common.cuh"
#include "mk_prefill.h"

namespace mk {
namespace {

constexpr int CH = 64;                                    // tokens per chunk
// shared block written by the preparation and read whole by every CTA of the head
constexpr int OFF_W = 0;                                  // fp16 [64][128], 256-byte rows, 16-byte pieces xor (row & 7)
constexpr int OFF_QG = OFF_W + CH * 256;                  // fp16 [64][128], same layout: Gam_r q_r
constexpr int OFF_KD = OFF_QG + CH * 256;                 // fp16 [128 keys][64 tokens], 128-byte rows, swizzled
constexpr int OFF_P = OFF_KD + 128 * 128;                 // fp16 [64][64], 128-byte rows, swizzled
constexpr int OFF_GL = OFF_P + CH * 128;                  // f32 Gam_last (+ pad to 16 bytes)
constexpr int BLK_BYTES = OFF_GL + 16;                    // 57360
constexpr int SCAN_GROUPS = 1;                            // groups of 16 value rows per CTA of the serial pass
constexpr int SCAN_ROWS = 16 * SCAN_GROUPS;               // value rows per CTA: 128 / SCAN_ROWS CTAs per head
constexpr int U_BYTES = CH * 128 * 4;                     // f32 [slices][64][SCAN_ROWS]
constexpr int U_SLICE_BYTES = CH * SCAN_ROWS * 4;
constexpr int PAIR_BYTES = BLK_BYTES + U_BYTES;           // per (chunk, head)

__host__ __device__ inline size_t pair_offset(int chunk, int head) { return ((size_t)chunk * DN_HEADS + head) * PAIR_BYTES; }

__device__ __forceinline__ uint32_t swz256(int row, int col) {     // byte offset of 16-bit (row, col), 256-byte rows
    return (uint32_t)(row * 256 + ((((col >> 3) ^ (row & 7)) << 4) | ((col & 7) << 1)));
}
__device__ __forceinline__ uint32_t swz128(int row, int col) {     // 128-byte rows
    return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7)) << 4) | ((col & 7) << 1)));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma_h(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3]) : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h(float lo, float hi) {
    const __half2 p = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&p);
}
// two fp16 terms of a pair of floats: hi = fp16(x), lo = fp16(x - hi)
__device__ __forceinline__ void split_pair(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __half xh = __float2half_rn(x), yh = __float2half_rn(y);
    const __half2 h2 = __halves2half2(xh, yh);
    hi = *reinterpret_cast<const uint32_t*>(&h2);
    lo = pack_h(x - __half2float(xh), y - __half2float(yh));
}

// ---- preparation: one CTA per (chunk, head), 256 threads ------------------------------------------------

constexpr int PADROW = 136;                               // fp16 elements per padded row (272 bytes: rows shift 4 banks)
constexpr int TROW = 72;                                  // fp16 elements per row of T (144 bytes)
constexpr int AROW = 68;                                  // floats per row of A
constexpr int PREP_KB = 0;                                // fp16 k
constexpr int PREP_QB = PREP_KB + CH * PADROW * 2;        // fp16 q
constexpr int PREP_KG = PREP_QB + CH * PADROW * 2;        // fp16 beta Gam k
constexpr int PREP_VB = PREP_KG + CH * PADROW * 2;        // fp16 beta v
constexpr int PREP_A = PREP_VB + CH * PADROW * 2;         // f32 A
constexpr int PREP_TH = PREP_A + CH * AROW * 4;           // fp16 T hi
constexpr int PREP_TL = PREP_TH + CH * TROW * 2;          // fp16 T lo
constexpr int PREP_G = PREP_TL + CH * TROW * 2;           // f32 G[64], beta[64]
constexpr int PREP_SMEM = PREP_G + 2 * CH * 4 + 16 * 17 * 4;   // 107 072 bytes: two CTAs per SM
constexpr int PREP_KDT = PREP_A;                          // staging of the decayed, transposed keys (16 KB), flushed
                                                          // to global memory before A is written

// qkv: bf16 [t][6144] projection outputs (q | k | v before the convolution); conv_w: bf16 [6144][4];
// conv_state: f32 [6144][4], the four inputs before the prompt; gates: [t][head][4] = beta, decay, -, log decay.
// The causal depthwise convolution (k = 4), SiLU and the L2 norms of q (x 1/sqrt(128)) and k
// (reference: megakernel/prefill.cu:1281-1368) are computed here, one warp per 8 consecutive tokens with the
// convolution window sliding through registers.
__global__ void __launch_bounds__(256, 2) k_dn_chunk_prepare(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ conv_w,
                                                             const float* __restrict__ conv_state, const float* __restrict__ gates,
                                                             unsigned char* __restrict__ scratch, int S) {
    pdl_enter();
    extern __shared__ __align__(128) unsigned char sm[];
    const int chunk = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = chunk * CH;
    float* sG = reinterpret_cast<float*>(sm + PREP_G);
    float* sBeta = sG + CH;
    float* sA = reinterpret_cast<float*>(sm + PREP_A);
    unsigned char* outg = scratch + pair_offset(chunk, h);          // the shared block in global memory

    // cumulative log-decay of the chunk (tokens past the prompt: beta 0, g 0)
    if (warp < 2) {
        const int t = t0 + tid;
        float g = 0.f, b = 0.f;
        if (t < S) { const float4 gt = *reinterpret_cast<const float4*>(gates + ((size_t)t * DN_HEADS + h) * 4); b = gt.x; g = gt.w; }
        float acc = g;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) { const float n = __shfl_up_sync(0xffffffffu, acc, o); if (lane >= o) acc += n; }
        sG[tid] = acc;
        sBeta[tid] = b;
    }
    __syncthreads();
    if (warp == 1) sG[tid] += sG[31];
    __syncthreads();
    const float Glast = sG[CH - 1];

    {
        // convolution + SiLU + L2 norms, then the fp16 operand tiles and the two scaled copies of the shared block.
        // One warp = 8 consecutive tokens, lane = 4 channels; q, k and v are processed one after the other so that
        // all 11 input rows of a pass (8 tokens + 3 of history) can be in flight at once.
        const int c4 = lane * 4;
        const int tb = t0 + warp * 8;
        __half* kdt = reinterpret_cast<__half*>(sm + PREP_KDT);
#pragma unroll 1
        for (int m = 0; m < 3; ++m) {
            const int chan = m * DN_QK + h * DN_KEY + c4;
            float wq[4][4];                                 // [channel][tap]
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint2 wr = __ldg(reinterpret_cast<const uint2*>(conv_w) + chan + e);
                wq[e][0] = bf_lo(wr.x); wq[e][1] = bf_hi(wr.x); wq[e][2] = bf_lo(wr.y); wq[e][3] = bf_hi(wr.y);
            }
            uint2 raw[11];
#pragma unroll
            for (int i = 0; i < 11; ++i) {
                const int tt = tb - 3 + i;
                raw[i] = (tt >= 0 && tt < S) ? *reinterpret_cast<const uint2*>(qkv + (size_t)tt * DN_CONV_CH + chan) : make_uint2(0u, 0u);
            }
            float x[11][4];
#pragma unroll
            for (int i = 0; i < 11; ++i) { x[i][0] = bf_lo(raw[i].x); x[i][1] = bf_hi(raw[i].x); x[i][2] = bf_lo(raw[i].y); x[i][3] = bf_hi(raw[i].y); }
            if (tb < 3) {                                   // the first rows of the prompt: history from the stored window
#pragma unroll
                for (int i = 0; i < 3; ++i) {
                    const int tt = tb - 3 + i;
                    if (tt < 0) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) x[i][e] = conv_state[(chan + e) * 4 + 4 + tt];
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = warp * 8 + i, t = t0 + r;
                float val[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float co = x[i][e] * wq[e][0] + x[i + 1][e] * wq[e][1] + x[i + 2][e] * wq[e][2] + x[i + 3][e] * wq[e][3];
                    val[e] = (t < S) ? silu_f(co) : 0.f;
                }
                const float G = sG[r], bta = sBeta[r];
                if (m == 2) {                               // values: beta v
                    *reinterpret_cast<uint2*>(sm + PREP_VB + (r * PADROW + c4) * 2) =
                        make_uint2(pack_h(bta * val[0], bta * val[1]), pack_h(bta * val[2], bta * val[3]));
                } else {
                    const float ss = warp_sum(val[0] * val[0] + val[1] * val[1] + val[2] * val[2] + val[3] * val[3]);
                    const float nrm = rsqrtf(ss + 1e-6f) * (m == 0 ? 0.08838834764831845f : 1.0f);
                    const float v0 = val[0] * nrm, v1 = val[1] * nrm, v2 = val[2] * nrm, v3 = val[3] * nrm;
                    const float gam = __expf(G);
                    if (m == 0) {                           // queries: q and Gam q
                        *reinterpret_cast<uint2*>(sm + PREP_QB + (r * PADROW + c4) * 2) = make_uint2(pack_h(v0, v1), pack_h(v2, v3));
                        *reinterpret_cast<uint2*>(outg + OFF_QG + swz256(r, c4)) =
                            make_uint2(pack_h(gam * v0, gam * v1), pack_h(gam * v2, gam * v3));
                    } else {                                // keys: k, beta Gam k, and the decayed transposed copy
                        const float bg = bta * gam, kd = __expf(Glast - G);
                        *reinterpret_cast<uint2*>(sm + PREP_KB + (r * PADROW + c4) * 2) = make_uint2(pack_h(v0, v1), pack_h(v2, v3));
                        *reinterpret_cast<uint2*>(sm + PREP_KG + (r * PADROW + c4) * 2) =
                            make_uint2(pack_h(bg * v0, bg * v1), pack_h(bg * v2, bg * v3));
                        kdt[swz128(c4 + 0, r) >> 1] = __float2half_rn(kd * v0);
                        kdt[swz128(c4 + 1, r) >> 1] = __float2half_rn(kd * v1);
                        kdt[swz128(c4 + 2, r) >> 1] = __float2half_rn(kd * v2);
                        kdt[swz128(c4 + 3, r) >> 1] = __float2half_rn(kd * v3);
                    }
                }
            }
        }
    }
    if (tid == 0) *reinterpret_cast<float4*>(outg + OFF_GL) = make_float4(__expf(Glast), 0.f, 0.f, 0.f);
    __syncthreads();
    {   // flush the transposed keys (their staging area is reused for A below)
        const uint4* src = reinterpret_cast<const uint4*>(sm + PREP_KDT);
        uint4* dst = reinterpret_cast<uint4*>(outg + OFF_KD);
        for (int i = tid; i < 128 * 128 / 16; i += 256) dst[i] = src[i];
    }
    __syncthreads();

    const int g8 = lane >> 2, t4 = lane & 3;
    {
        // warps 0-3: K K^T (-> A), warps 4-7: Q K^T (-> P); each warp one 16-row tile, all 64 columns
        const int mt = warp & 3, isq = warp >> 2;
        const uint32_t abase = smem_u32(sm + (isq ? PREP_QB : PREP_KB));
        const uint32_t bbase = smem_u32(sm + PREP_KB);
        float acc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) { acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f; }
        const int arow = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, acol = (lane >> 4) * 8;
        const int brow = (lane & 7) + (lane >> 4) * 8, bcol = ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t a0, a1, a2, a3;
            ldsm4(abase + (arow * PADROW + ks * 16 + acol) * 2, a0, a1, a2, a3);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm4(bbase + ((np * 16 + brow) * PADROW + ks * 16 + bcol) * 2, b0, b1, b2, b3);
                mma_h(acc[2 * np], a0, a1, a2, a3, b0, b1);
                mma_h(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
            }
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = mt * 16 + g8 + (e >> 1) * 8, c = n * 8 + 2 * t4 + (e & 1);
                const float dec = __expf(sG[r] - sG[c]);
                if (!isq) sA[r * AROW + c] = (c < r) ? sBeta[r] * dec * acc[n][e] : 0.f;
                else acc[n][e] = (c <= r) ? dec * acc[n][e] : 0.f;
            }
            if (isq) {
                const int c = n * 8 + 2 * t4;
                *reinterpret_cast<uint32_t*>(outg + OFF_P + swz128(mt * 16 + g8, c)) = pack_h(acc[n][0], acc[n][1]);
                *reinterpret_cast<uint32_t*>(outg + OFF_P + swz128(mt * 16 + g8 + 8, c)) = pack_h(acc[n][2], acc[n][3]);
            }
        }
    }
    __syncthreads();

    // T = (I + A)^-1, A strictly lower triangular, in 16 x 16 blocks: the four diagonal blocks by forward
    // substitution (one thread per column), then each block row i from right to left,
    //   T_ij = -(sum_{k=j+1..i} T_ik A_kj) T_jj,
    // one thread per element.  T is written as fp16 head + remainder (the form the products below read).
    {
        __half* TH = reinterpret_cast<__half*>(sm + PREP_TH);
        __half* TL = reinterpret_cast<__half*>(sm + PREP_TL);
        // f32 working copy of T in the (now unused) q tile: the block products read it with one load per term
        float* Tf = reinterpret_cast<float*>(sm + PREP_QB);
        auto put = [&](int r, int c, float v) {
            const __half hi = __float2half_rn(v);
            TH[r * TROW + c] = hi;
            TL[r * TROW + c] = __float2half_rn(v - __half2float(hi));
            Tf[r * AROW + c] = v;
        };
        auto get = [&](int r, int c) { return Tf[r * AROW + c]; };
        if (tid < 64) {
            const int bb = (tid >> 4) * 16, c = tid & 15;
            float x[16];
#pragma unroll
            for (int s = 0; s < 16; ++s) {
                float acc = (s == c) ? 1.f : 0.f;
#pragma unroll
                for (int u = 0; u < s; ++u) acc = fmaf(-sA[(bb + s) * AROW + bb + u], x[u], acc);
                x[s] = acc;
                put(bb + s, bb + c, acc);
            }
        }
        // zero the blocks above the diagonal
        for (int i = tid; i < 6 * 256; i += 256) {
            const int blk = i >> 8, r = (i >> 4) & 15, c = i & 15;
            const int bi = (blk < 3) ? 0 : (blk < 5 ? 1 : 2), bj = (blk < 3) ? blk + 1 : (blk < 5 ? blk - 1 : 3);
            put(bi * 16 + r, bj * 16 + c, 0.f);
        }
        __syncthreads();
        float* Ms = sG + 2 * CH;                 // 16 x 17 floats of scratch after G and beta
        const int r = tid >> 4, c = tid & 15;
#pragma unroll 1
        for (int bi = 3; bi >= 1; --bi) {
#pragma unroll 1
            for (int bj = bi - 1; bj >= 0; --bj) {
                float m[4] = {0.f, 0.f, 0.f, 0.f};
                for (int k = bj + 1; k <= bi; ++k) {
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        m[e & 3] = fmaf(get(bi * 16 + r, k * 16 + e), sA[(k * 16 + e) * AROW + bj * 16 + c], m[e & 3]);
                }
                Ms[r * 17 + c] = (m[0] + m[1]) + (m[2] + m[3]);
                __syncthreads();
                float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e & 3] = fmaf(Ms[r * 17 + e], get(bj * 16 + e, bj * 16 + c), v[e & 3]);
                put(bi * 16 + r, bj * 16 + c, -((v[0] + v[1]) + (v[2] + v[3])));
                __syncthreads();
            }
        }
    }
    {
        // warps 0-3: W = T (beta Gam k), warps 4-7: U = T (beta v); each warp one 16-row tile, 128 columns
        const int mt = warp & 3, isu = warp >> 2;
        const uint32_t th = smem_u32(sm + PREP_TH), tl = smem_u32(sm + PREP_TL);
        const uint32_t bbase = smem_u32(sm + (isu ? PREP_VB : PREP_KG));
        const int arow = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, acol = (lane >> 4) * 8;
        uint32_t ah[4][4], al[4][4];
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            ldsm4(th + (arow * TROW + ks * 16 + acol) * 2, ah[ks][0], ah[ks][1], ah[ks][2], ah[ks][3]);
            ldsm4(tl + (arow * TROW + ks * 16 + acol) * 2, al[ks][0], al[ks][1], al[ks][2], al[ks][3]);
        }
        // block row mt of T is zero right of block column mt: k-steps beyond it are skipped
        float* Uout = reinterpret_cast<float*>(outg + BLK_BYTES);
#pragma unroll 2
        for (int np = 0; np < 8; ++np) {                 // pairs of 8-column tiles
            float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                if (ks > mt) continue;
                uint32_t b0, b1, b2, b3;                  // operand stored [k][n]: transposing load
                ldsm4t(bbase + ((ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * PADROW + np * 16 + (lane >> 4) * 8) * 2, b0, b1, b2, b3);
                mma_h(c0, ah[ks][0], ah[ks][1], ah[ks][2], ah[ks][3], b0, b1);
                mma_h(c0, al[ks][0], al[ks][1], al[ks][2], al[ks][3], b0, b1);
                mma_h(c1, ah[ks][0], ah[ks][1], ah[ks][2], ah[ks][3], b2, b3);
                mma_h(c1, al[ks][0], al[ks][1], al[ks][2], al[ks][3], b2, b3);
            }
            const int r = mt * 16 + g8, col = np * 16 + 2 * t4;
            if (!isu) {
                *reinterpret_cast<uint32_t*>(outg + OFF_W + swz256(r, col)) = pack_h(c0[0], c0[1]);
                *reinterpret_cast<uint32_t*>(outg + OFF_W + swz256(r + 8, col)) = pack_h(c0[2], c0[3]);
                *reinterpret_cast<uint32_t*>(outg + OFF_W + swz256(r, col + 8)) = pack_h(c1[0], c1[1]);
                *reinterpret_cast<uint32_t*>(outg + OFF_W + swz256(r + 8, col + 8)) = pack_h(c1[2], c1[3]);
            } else {
                // U[slice][token][SCAN_ROWS values]
                auto uaddr = [&](int row, int j) { return Uout + ((size_t)(j / SCAN_ROWS) * CH + row) * SCAN_ROWS + (j % SCAN_ROWS); };
                *reinterpret_cast<float2*>(uaddr(r, col)) = make_float2(c0[0], c0[1]);
                *reinterpret_cast<float2*>(uaddr(r + 8, col)) = make_float2(c0[2], c0[3]);
                *reinterpret_cast<float2*>(uaddr(r, col + 8)) = make_float2(c1[0], c1[1]);
                *reinterpret_cast<float2*>(uaddr(r + 8, col + 8)) = make_float2(c1[2], c1[3]);
            }
        }
    }
}

// ---- serial pass: one CTA per (head, SCAN_ROWS value rows), 128 threads per group of 16 rows ------------------------------------------

constexpr int STAGE_BYTES_DN = BLK_BYTES + U_SLICE_BYTES;         // 65552
constexpr int SC_STAGE0 = 0;
constexpr int SC_S_HI = 2 * STAGE_BYTES_DN;                       // fp16 [32 value rows][128 keys], swizzled 256-byte rows
constexpr int SC_S_LO = SC_S_HI + 32 * 256;
constexpr int DROW = 72;                                          // fp16 per row of D^T (144 bytes)
constexpr int SC_D = SC_S_LO + 32 * 256;                          // fp16 [32 value rows][64 tokens]
constexpr int SC_BAR = SC_D + 32 * DROW * 2;
constexpr int SCAN2_SMEM = SC_BAR + 16;

__global__ void __launch_bounds__(128 * SCAN_GROUPS, 1) k_dn_chunk_scan(const unsigned char* __restrict__ scratch, float* __restrict__ state,
                                                          float* __restrict__ o, int S, int nchunks, int* __restrict__ err) {
    pdl_enter();
    extern __shared__ __align__(128) unsigned char sm[];
    constexpr int SLICES = DN_VAL / SCAN_ROWS;
    const int h = blockIdx.x / SLICES, slice = blockIdx.x % SLICES;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = warp >> 2, wq = warp & 3;                     // grp: 16 value rows; wq: quarter of the columns
    const int g8 = lane >> 2, t4 = lane & 3;
    const uint32_t bar0 = smem_u32(sm + SC_BAR);
    if (tid == 0) { mbar_init(bar0, 1); mbar_init(bar0 + 8, 1); fence_mbar_init(); }
    __syncthreads();
    const uint64_t pol = l2_policy_evict_first();
    auto issue = [&](int c) {
        const uint32_t bar = bar0 + (c & 1) * 8, dst = smem_u32(sm + SC_STAGE0 + (c & 1) * STAGE_BYTES_DN);
        const unsigned char* src = scratch + pair_offset(c, h);
        mbar_expect_tx(bar, STAGE_BYTES_DN);
        bulk_g2s(dst, src, BLK_BYTES, bar, pol);
        bulk_g2s(dst + BLK_BYTES, src + BLK_BYTES + slice * U_SLICE_BYTES, U_SLICE_BYTES, bar, pol);
    };
    if (tid == 0) { issue(0); if (nchunks > 1) issue(1); }

    // state rows of this warp group: accumulator layout, this warp holds key columns [32 wq, 32 wq + 32)
    const int jrow = slice * SCAN_ROWS + grp * 16;                // first value row of the group within the head
    float sacc[4][4];
    float* sg = state + ((size_t)h * DN_VAL + jrow) * DN_KEY;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
        const int col = wq * 32 + n * 8 + 2 * t4;
        const float2 lo = *reinterpret_cast<const float2*>(sg + (size_t)g8 * DN_KEY + col);
        const float2 hi = *reinterpret_cast<const float2*>(sg + (size_t)(g8 + 8) * DN_KEY + col);
        sacc[n][0] = lo.x; sacc[n][1] = lo.y; sacc[n][2] = hi.x; sacc[n][3] = hi.y;
    }
    auto publish_state = [&]() {
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            const int col = wq * 32 + n * 8 + 2 * t4;
            uint32_t h0, l0, h1, l1;
            split_pair(sacc[n][0], sacc[n][1], h0, l0);
            split_pair(sacc[n][2], sacc[n][3], h1, l1);
            *reinterpret_cast<uint32_t*>(sm + SC_S_HI + swz256(grp * 16 + g8, col)) = h0;
            *reinterpret_cast<uint32_t*>(sm + SC_S_LO + swz256(grp * 16 + g8, col)) = l0;
            *reinterpret_cast<uint32_t*>(sm + SC_S_HI + swz256(grp * 16 + g8 + 8, col)) = h1;
            *reinterpret_cast<uint32_t*>(sm + SC_S_LO + swz256(grp * 16 + g8 + 8, col)) = l1;
        }
    };
    publish_state();
    __syncthreads();

    const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, acol8 = (lane >> 4);          // A-operand lane pattern (16 x 16)
    const int brow = (lane & 7) + (lane >> 4) * 8, bcol8 = ((lane >> 3) & 1);          // B-operand pattern, two 8-column tiles
    bool dead = false;
    for (int c = 0; c < nchunks; ++c) {
        const unsigned char* st = sm + SC_STAGE0 + (c & 1) * STAGE_BYTES_DN;
        const uint32_t stb = smem_u32(st);
        if (!mbar_wait(bar0 + (c & 1) * 8, (c >> 1) & 1)) { dead = true; }
        if (__syncthreads_or(dead)) { if (tid == 0) atomicExch(err, 2); break; }
        const float gam_last = *reinterpret_cast<const float*>(st + OFF_GL);

        // state operand fragments (hi, lo) for the 16 value rows of the group, all 128 keys
        uint32_t sh[8][4], sl[8][4];
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const uint32_t off = swz256(grp * 16 + arow, (2 * ks + acol8) * 8);
            ldsm4(smem_u32(sm + SC_S_HI) + off, sh[ks][0], sh[ks][1], sh[ks][2], sh[ks][3]);
            ldsm4(smem_u32(sm + SC_S_LO) + off, sl[ks][0], sl[ks][1], sl[ks][2], sl[ks][3]);
        }
        // D^T[value][token] for tokens [16 wq, 16 wq + 16): U^T - S W^T
        float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        float oi[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t b0, b1, b2, b3;
            ldsm4(stb + OFF_W + swz256(wq * 16 + brow, (2 * ks + bcol8) * 8), b0, b1, b2, b3);
            mma_h(d[0], sh[ks][0], sh[ks][1], sh[ks][2], sh[ks][3], b0, b1);
            mma_h(d[0], sl[ks][0], sl[ks][1], sl[ks][2], sl[ks][3], b0, b1);
            mma_h(d[1], sh[ks][0], sh[ks][1], sh[ks][2], sh[ks][3], b2, b3);
            mma_h(d[1], sl[ks][0], sl[ks][1], sl[ks][2], sl[ks][3], b2, b3);
            // the state-dependent part of the output for the same tokens: S (Gam q)^T
            ldsm4(stb + OFF_QG + swz256(wq * 16 + brow, (2 * ks + bcol8) * 8), b0, b1, b2, b3);
            mma_h(oi[0], sh[ks][0], sh[ks][1], sh[ks][2], sh[ks][3], b0, b1);
            mma_h(oi[0], sl[ks][0], sl[ks][1], sl[ks][2], sl[ks][3], b0, b1);
            mma_h(oi[1], sh[ks][0], sh[ks][1], sh[ks][2], sh[ks][3], b2, b3);
            mma_h(oi[1], sl[ks][0], sl[ks][1], sl[ks][2], sl[ks][3], b2, b3);
        }
        {
            const float* U = reinterpret_cast<const float*>(st + BLK_BYTES);       // [token][SCAN_ROWS values of this slice]
            __half* D = reinterpret_cast<__half*>(sm + SC_D);
#pragma unroll
            for (int n = 0; n < 2; ++n) {
                const int tok = wq * 16 + n * 8 + 2 * t4, j = grp * 16 + g8;
                const float d0 = U[tok * SCAN_ROWS + j] - d[n][0], d1 = U[(tok + 1) * SCAN_ROWS + j] - d[n][1];
                const float d2 = U[tok * SCAN_ROWS + j + 8] - d[n][2], d3 = U[(tok + 1) * SCAN_ROWS + j + 8] - d[n][3];
                *reinterpret_cast<uint32_t*>(D + j * DROW + tok) = pack_h(d0, d1);
                *reinterpret_cast<uint32_t*>(D + (j + 8) * DROW + tok) = pack_h(d2, d3);
            }
        }
        named_bar_sync(1 + grp, 128);
        // D^T as the A operand, all 64 tokens
        uint32_t da[4][4];
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
            ldsm4(smem_u32(sm + SC_D) + ((grp * 16 + arow) * DROW + (2 * ks + acol8) * 8) * 2, da[ks][0], da[ks][1], da[ks][2], da[ks][3]);
        // outputs for tokens [16 wq, +16): add D^T P^T
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            uint32_t b0, b1, b2, b3;
            ldsm4(stb + OFF_P + swz128(wq * 16 + brow, (2 * ks + bcol8) * 8), b0, b1, b2, b3);
            mma_h(oi[0], da[ks][0], da[ks][1], da[ks][2], da[ks][3], b0, b1);
            mma_h(oi[1], da[ks][0], da[ks][1], da[ks][2], da[ks][3], b2, b3);
        }
#pragma unroll
        for (int n = 0; n < 2; ++n) {
            const int tok = c * CH + wq * 16 + n * 8 + 2 * t4;
            float* orow = o + (size_t)tok * DN_V + h * DN_VAL + jrow + g8;
            if (tok < S) { orow[0] = oi[n][0]; orow[8] = oi[n][2]; }
            if (tok + 1 < S) { orow[DN_V] = oi[n][1]; orow[DN_V + 8] = oi[n][3]; }
        }
        // state: Gam_last S + D^T Kd, key columns [32 wq, +32)
#pragma unroll
        for (int n = 0; n < 4; ++n) { sacc[n][0] *= gam_last; sacc[n][1] *= gam_last; sacc[n][2] *= gam_last; sacc[n][3] *= gam_last; }
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
            for (int np = 0; np < 2; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm4(stb + OFF_KD + swz128(wq * 32 + np * 16 + brow, (2 * ks + bcol8) * 8), b0, b1, b2, b3);
                mma_h(sacc[2 * np], da[ks][0], da[ks][1], da[ks][2], da[ks][3], b0, b1);
                mma_h(sacc[2 * np + 1], da[ks][0], da[ks][1], da[ks][2], da[ks][3], b2, b3);
            }
        }
        publish_state();
        __syncthreads();                                           // stage consumed, new state visible
        if (tid == 0 && c + 2 < nchunks) issue(c + 2);
    }
#pragma unroll
    for (int n = 0; n < 4; ++n) {
        const int col = wq * 32 + n * 8 + 2 * t4;
        *reinterpret_cast<float2*>(sg + (size_t)g8 * DN_KEY + col) = make_float2(sacc[n][0], sacc[n][1]);
        *reinterpret_cast<float2*>(sg + (size_t)(g8 + 8) * DN_KEY + col) = make_float2(sacc[n][2], sacc[n][3]);
    }
}

}  // namespace

size_t dn_chunked_scratch_bytes(int S) { return (size_t)((S + CH - 1) / CH) * DN_HEADS * PAIR_BYTES; }

cudaError_t dn_chunked(const void* qkv, const void* conv_w, const float* conv_state, const float* gates, float* state, float* o,
                       int S, void* scratch, int* err, cudaStream_t stream) {
    static bool attr[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        e = cudaFuncSetAttribute(k_dn_chunk_prepare, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(k_dn_chunk_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, SCAN2_SMEM);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    const int nchunks = (S + CH - 1) / CH;
    launch_pdl(k_dn_chunk_prepare, dim3(nchunks, DN_HEADS), 256, PREP_SMEM, stream, (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)conv_w, conv_state,
                                                                         gates, (unsigned char*)scratch, S);
    launch_pdl(k_dn_chunk_scan, DN_HEADS * (DN_VAL / SCAN_ROWS), 128 * SCAN_GROUPS, SCAN2_SMEM, stream, (const unsigned char*)scratch, state, o, S, nchunks, err);
    return cudaGetLastError();
}

}  // namespace mk
