// Causal GQA attention for prefill (8 query heads, 2 KV heads, head_dim 256) with online softmax,
// scores and P.V on mma.sync (bf16 operands, f32 accumulate), output times sigmoid(gate).
// (reference: the cuBLAS score / softmax / value path megakernel/prefill.cu:1202-1236 and its
// scalar fallback :270-294; the arithmetic is softmax(q k^T / 16) v over keys <= query.)
//
// One CTA = 32 consecutive query positions x the 4 query heads of one KV head: 8 warps, each one
// 16-row MMA tile (head = warp / 2), so a K/V tile of 64 keys staged in shared memory serves all four
// heads.  K/V tiles are double-buffered with cp.async; Q stays in shared memory and is re-read per
// tile (with head_dim 256 the output accumulator alone takes 128 registers).
#include <cuda_bf16.h>
#include <stdint.h>

#include "mk_common.cuh"
#include "mk_prefill.h"

namespace mk {
namespace {

constexpr int QB = 32;                       // query positions per CTA
constexpr int KB = 64;                       // keys per tile
constexpr int ROWB = FA_HEAD_DIM * 2;        // 512 bytes per row
constexpr int FA_Q_BYTES = 4 * QB * ROWB;    // 65536
constexpr int FA_KV_BYTES = KB * ROWB;       // 32768
constexpr int FA_SMEM = FA_Q_BYTES + 4 * FA_KV_BYTES;   // Q | K0 | K1 | V0 | V1

__device__ __forceinline__ uint32_t swz512(int row, int chunk) { return (uint32_t)(row * ROWB + ((chunk ^ (row & 7)) << 4)); }
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3]) : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&p);
}
// 16-byte async copy; bytes = 0 writes zeros
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}

constexpr int MAX_KEY_BLOCKS = 1024;          // block-sparse mode: prompts of up to 131072 tokens
constexpr int FA_SMEM_SPARSE = FA_SMEM + MAX_KEY_BLOCKS * 4 + 16;   // + list of up to 2048 tile ids + count

// qkv: [S][5120] = 8 x [q(256) | gate(256)] | k(512) | v(512), q already normalised and rotated;
// kc, vc: [2][max_seq][256]; out: [S][2048].
// SPARSE: mask[head][query block of 128][word] holds one bit per key block of 128; a CTA walks the union
// of the kept key blocks of its four heads and each warp skips the blocks its own head dropped.
template <bool SPARSE>
__global__ void __launch_bounds__(256, 1) k_fa_prefill(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ kc,
                                                       const __nv_bfloat16* __restrict__ vc, __nv_bfloat16* __restrict__ out,
                                                       int S, int max_seq, const uint32_t* __restrict__ mask, int nblk, int nwords) {
    pdl_enter();
    extern __shared__ __align__(128) unsigned char sm[];
    const int qblk = gridDim.x - 1 - blockIdx.x;          // longest rows first
    const int g = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
    const int q0 = qblk * QB;
    const uint32_t sQ = smem_u32(sm), sK = sQ + FA_Q_BYTES, sV = sK + 2 * FA_KV_BYTES;
    const __nv_bfloat16* K = kc + (size_t)g * max_seq * FA_HEAD_DIM;
    const __nv_bfloat16* V = vc + (size_t)g * max_seq * FA_HEAD_DIM;

    // Q tile: row = head_in_group * 32 + query
    for (int i = tid; i < 4 * QB * 32; i += 256) {
        const int row = i >> 5, chunk = i & 31, hh = row >> 5, qi = row & 31, t = q0 + qi;
        const __nv_bfloat16* src = qkv + (size_t)min(t, S - 1) * FA_QKV_ROWS + (g * FA_GQA + hh) * 2 * FA_HEAD_DIM + chunk * 8;
        cp16(sQ + swz512(row, chunk), src, t < S ? 16 : 0);
    }
    const int last_q = min(q0 + QB, S) - 1;
    int ntiles = last_q / KB + 1;
    // tile list (sparse): 64-key tiles of the kept 128-key blocks, in ascending order
    unsigned short* tlist = reinterpret_cast<unsigned short*>(sm + FA_SMEM);
    const uint32_t* hmask = nullptr;         // mask row of this warp's head
    if (SPARSE) {
        const int qb = q0 >> 7;
        const uint32_t* m0 = mask + ((size_t)(g * FA_GQA) * nblk + qb) * nwords;
        const size_t hstride = (size_t)nblk * nwords;
        hmask = m0 + (size_t)(warp >> 1) * hstride;
        if (tid == 0) {
            int n = 0;
            for (int w = 0; w < nwords; ++w) {
                uint32_t u = m0[w] | m0[w + hstride] | m0[w + 2 * hstride] | m0[w + 3 * hstride];
                while (u) {
                    const int b = __ffs(u) - 1;
                    u &= u - 1;
                    const int t0 = (w * 32 + b) * 2;
                    if (t0 * KB <= last_q) tlist[n++] = (unsigned short)t0;
                    if ((t0 + 1) * KB <= last_q) tlist[n++] = (unsigned short)(t0 + 1);
                }
            }
            *reinterpret_cast<int*>(sm + FA_SMEM + MAX_KEY_BLOCKS * 4) = n;
        }
        __syncthreads();
        ntiles = *reinterpret_cast<const int*>(sm + FA_SMEM + MAX_KEY_BLOCKS * 4);
    }
    auto tile_of = [&](int it) { return SPARSE ? (int)tlist[it] : it; };
    auto load_kv = [&](int it, int buf) {
        const int j = tile_of(it);
        for (int i = tid; i < KB * 32; i += 256) {
            const int row = i >> 5, chunk = i & 31, key = j * KB + row;
            const int ok = key <= last_q ? 16 : 0;
            const size_t off = (size_t)min(key, last_q) * FA_HEAD_DIM + chunk * 8;
            cp16(sK + buf * FA_KV_BYTES + swz512(row, chunk), K + off, ok);
            cp16(sV + buf * FA_KV_BYTES + swz512(row, chunk), V + off, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load_kv(0, 0);

    const int mrow = warp * 16;                            // first row of this warp in the Q tile
    const int qpos0 = q0 + (warp & 1) * 16;                // query position of row 0 of this warp
    float oacc[32][4];
#pragma unroll
    for (int n = 0; n < 32; ++n) { oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f; }
    float mx[2] = {-1e30f, -1e30f}, lsum[2] = {0.f, 0.f};
    const float sc = 0.0625f * 1.4426950408889634f;        // 1/sqrt(256) * log2(e)
    const int arow = mrow + (lane & 7) + ((lane >> 3) & 1) * 8, achunk = lane >> 4;
    const int brow = (lane & 7) + (lane >> 4) * 8, bchunk = (lane >> 3) & 1;
    const int trow = (lane & 7) + ((lane >> 3) & 1) * 8, tchunk = lane >> 4;

    for (int it = 0; it < ntiles; ++it) {
        const int buf = it & 1;
        const int j = tile_of(it);
        if (it + 1 < ntiles) load_kv(it + 1, buf ^ 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();
        if (SPARSE && !((hmask[j >> 6] >> ((j >> 1) & 31)) & 1u)) { __syncthreads(); continue; }   // this head dropped the block
        const uint32_t kb = sK + buf * FA_KV_BYTES, vb = sV + buf * FA_KV_BYTES;
        float s[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) { s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f; }
#pragma unroll 4
        for (int ks = 0; ks < 16; ++ks) {
            uint32_t a0, a1, a2, a3;
            ldsm4(sQ + swz512(arow, 2 * ks + achunk), a0, a1, a2, a3);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm4(kb + swz512(np * 16 + brow, 2 * ks + bchunk), b0, b1, b2, b3);
                mma_bf16(s[2 * np], a0, a1, a2, a3, b0, b1);
                mma_bf16(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
            }
        }
        // causal mask (only tiles that reach past the first query of the warp), scale, online softmax
        const int key0 = j * KB;
        const bool diag = key0 + KB - 1 > qpos0;
        float tmax[2] = {-1e30f, -1e30f};
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float v = s[n][e] * sc;
                if (diag) {
                    const int key = key0 + n * 8 + 2 * t4 + (e & 1), qp = qpos0 + g8 + (e >> 1) * 8;
                    if (key > qp) v = -1e30f;
                }
                s[n][e] = v;
                tmax[e >> 1] = fmaxf(tmax[e >> 1], v);
            }
        }
        float corr[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
            tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
            const float mn = fmaxf(mx[r], tmax[r]);
            corr[r] = exp2f(mx[r] - mn);
            mx[r] = mn;
        }
        float rs[2] = {0.f, 0.f};
        uint32_t pa[4][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const float p0 = exp2f(s[n][0] - mx[0]), p1 = exp2f(s[n][1] - mx[0]);
            const float p2 = exp2f(s[n][2] - mx[1]), p3 = exp2f(s[n][3] - mx[1]);
            // the reference rounds P to bf16 before P.V; the row sum uses the rounded values too
            const uint32_t lo = pack_bf16(p0, p1), hi = pack_bf16(p2, p3);
            rs[0] += bf_lo(lo) + bf_hi(lo);
            rs[1] += bf_lo(hi) + bf_hi(hi);
            pa[n >> 1][(n & 1) * 2] = lo;
            pa[n >> 1][(n & 1) * 2 + 1] = hi;
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) lsum[r] = lsum[r] * corr[r] + rs[r];
#pragma unroll
        for (int n = 0; n < 32; ++n) { oacc[n][0] *= corr[0]; oacc[n][1] *= corr[0]; oacc[n][2] *= corr[1]; oacc[n][3] *= corr[1]; }
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
            for (int np = 0; np < 16; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm4t(vb + swz512(ks * 16 + trow, 2 * np + tchunk), b0, b1, b2, b3);
                mma_bf16(oacc[2 * np], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b0, b1);
                mma_bf16(oacc[2 * np + 1], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b2, b3);
            }
        }
        __syncthreads();
    }
    // finish: row sums across the 4 lanes of a row, normalise, gate, store
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], 1);
        lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], 2);
    }
    const int head = g * FA_GQA + (warp >> 1);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int t = qpos0 + g8 + r * 8;
        if (t >= S) continue;
        const float inv = 1.0f / lsum[r];
        const __nv_bfloat16* gate = qkv + (size_t)t * FA_QKV_ROWS + head * 2 * FA_HEAD_DIM + FA_HEAD_DIM;
        __nv_bfloat16* dst = out + (size_t)t * FA_Q_SIZE + head * FA_HEAD_DIM;
#pragma unroll
        for (int n = 0; n < 32; ++n) {
            const int col = n * 8 + 2 * t4;
            const uint32_t gu = *reinterpret_cast<const uint32_t*>(gate + col);
            *reinterpret_cast<uint32_t*>(dst + col) =
                pack_bf16(oacc[n][2 * r] * inv * sigmoid_f(bf_lo(gu)), oacc[n][2 * r + 1] * inv * sigmoid_f(bf_hi(gu)));
        }
    }
}

}  // namespace

namespace {

// ---- block selection ----------------------------------------------------------------------------------
// Mean over the (up to) 128 positions of a block, sequentially in f32; slots 0-7 = query heads, 8-9 = key heads.
__global__ void __launch_bounds__(256) k_bs_pool(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ kc,
                                                 float* __restrict__ means, int S, int max_seq, int nblk) {
    pdl_enter();
    const int b = blockIdx.x, slot = blockIdx.y, d = threadIdx.x;
    const int lo = b * 128, hi = min(S, lo + 128);
    float acc = 0.f;
    if (slot < 8) {
        const __nv_bfloat16* src = qkv + (size_t)lo * FA_QKV_ROWS + slot * 2 * FA_HEAD_DIM + d;
        for (int p = lo; p < hi; ++p, src += FA_QKV_ROWS) acc = __fadd_rn(acc, bf2f(*src));
    } else {
        const __nv_bfloat16* src = kc + ((size_t)(slot - 8) * max_seq + lo) * FA_HEAD_DIM + d;
        for (int p = lo; p < hi; ++p, src += FA_HEAD_DIM) acc = __fadd_rn(acc, bf2f(*src));
    }
    means[((size_t)slot * nblk + b) * FA_HEAD_DIM + d] = __fmul_rn(acc, 1.0f / (float)(hi - lo));
}

// One CTA per (query block i, head): scores against all causal key blocks, then keep the sink blocks, the
// local window and the `topk` best by score (ties to the lower index).  Every add and multiply is rounded
// on its own and in a fixed order, so the scores can be reproduced bit for bit on a CPU.
// rule 1 is the reference's own keep rule (dflash/src/flashprefill_select.cpp:27-84) on the same scores: sink blocks,
// the local window, every causal block for the last `last_full` query blocks, and the blocks whose score reaches
// alpha times the row maximum (one f32 multiply, `>=`).  scores_out (optional): f32 [8][nblk][nblk], entries j <= i.
__global__ void __launch_bounds__(256) k_bs_select(const float* __restrict__ means, uint32_t* __restrict__ mask, int nblk, int nwords,
                                                   double top_frac, int window, int sink, int rule, float alpha, int last_full,
                                                   float* __restrict__ scores_out) {
    pdl_enter();
    extern __shared__ float sc[];                           // nblk scores, then nwords mask words
    uint32_t* words = reinterpret_cast<uint32_t*>(sc + nblk);
    const int i = blockIdx.x, h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = i + 1;
    const float* qm = means + ((size_t)h * nblk + i) * FA_HEAD_DIM + lane * 8;
    float q[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) q[e] = qm[e];
    for (int j = warp; j < n; j += 8) {
        const float* km = means + ((size_t)(8 + h / FA_GQA) * nblk + j) * FA_HEAD_DIM + lane * 8;
        float part = __fmul_rn(q[0], km[0]);
#pragma unroll
        for (int e = 1; e < 8; ++e) part = __fadd_rn(part, __fmul_rn(q[e], km[e]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
        if (lane == 0) sc[j] = part;
    }
    for (int w = threadIdx.x; w < nwords; w += 256) words[w] = 0u;
    __syncthreads();
    if (scores_out)
        for (int j = threadIdx.x; j < n; j += 256) scores_out[((size_t)h * nblk + i) * nblk + j] = sc[j];
    if (rule == 1) {
        float mx = -INFINITY;                               // every thread scans the row: max is order-independent
        for (int o = 0; o < n; ++o) mx = fmaxf(mx, sc[o]);
        const float thresh = __fmul_rn(mx, alpha);
        const bool all = i >= nblk - last_full;
        for (int j = threadIdx.x; j < n; j += 256)
            if (j < sink || i - j < window || all || sc[j] >= thresh) atomicOr(&words[j >> 5], 1u << (j & 31));
    }
    const int topk = (int)ceil(top_frac * (double)n);
    for (int j = threadIdx.x; rule == 0 && j < n; j += 256) {
        bool keep = j < sink || j > i - window;
        if (!keep) {
            const float s = sc[j];
            int rank = 0;
            for (int o = 0; o < n; ++o) { const float t = sc[o]; rank += (t > s) || (t == s && o < j); }
            keep = rank < topk;
        }
        if (keep) atomicOr(&words[j >> 5], 1u << (j & 31));
    }
    __syncthreads();
    for (int w = threadIdx.x; w < nwords; w += 256) mask[((size_t)h * nblk + i) * nwords + w] = words[w];
}

}  // namespace

size_t block_select_scratch_bytes(int S) {
    const int nblk = (S + 127) / 128, nwords = (nblk + 31) / 32;
    return (size_t)10 * nblk * FA_HEAD_DIM * 4 + (size_t)8 * nblk * nwords * 4;
}

cudaError_t block_select(const void* qkv, const void* kc, int S, int max_seq, double top_frac, int window, int sink,
                         void* scratch, uint32_t** mask_out, cudaStream_t stream, int rule, float alpha, int last_full,
                         float* scores_out) {
    const int nblk = (S + 127) / 128, nwords = (nblk + 31) / 32;
    if (nblk > MAX_KEY_BLOCKS) return cudaErrorInvalidValue;
    float* means = (float*)scratch;
    uint32_t* mask = (uint32_t*)((char*)scratch + (size_t)10 * nblk * FA_HEAD_DIM * 4);
    launch_pdl(k_bs_pool, dim3(nblk, 10), 256, 0, stream, (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)kc, means, S, max_seq, nblk);
    launch_pdl(k_bs_select, dim3(nblk, 8), 256, (nblk + nwords) * 4, stream, means, mask, nblk, nwords, top_frac, window, sink, rule, alpha,
               last_full, scores_out);
    *mask_out = mask;
    return cudaGetLastError();
}

cudaError_t fa_prefill(const void* qkv, const void* kc, const void* vc, void* out, int S, int max_seq, const uint32_t* mask,
                       cudaStream_t stream) {
    static bool attr[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        e = cudaFuncSetAttribute(k_fa_prefill<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_fa_prefill<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM_SPARSE);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    const dim3 grid((S + QB - 1) / QB, FA_KV_HEADS);
    if (mask) {
        const int nblk = (S + 127) / 128, nwords = (nblk + 31) / 32;
        if (nblk > MAX_KEY_BLOCKS) return cudaErrorInvalidValue;
        launch_pdl(k_fa_prefill<true>, grid, 256, FA_SMEM_SPARSE, stream, (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)kc,
                                                                   (const __nv_bfloat16*)vc, (__nv_bfloat16*)out, S, max_seq, mask, nblk, nwords);
    } else {
        launch_pdl(k_fa_prefill<false>, grid, 256, FA_SMEM, stream, (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)kc, (const __nv_bfloat16*)vc,
                                                            (__nv_bfloat16*)out, S, max_seq, nullptr, 0, 0);
    }
    return cudaGetLastError();
}

}  // namespace mk
