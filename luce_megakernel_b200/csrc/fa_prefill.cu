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

// qkv: [S][5120] = 8 x [q(256) | gate(256)] | k(512) | v(512), q already normalised and rotated;
// kc, vc: [2][max_seq][256]; out: [S][2048]
__global__ void __launch_bounds__(256, 1) k_fa_prefill(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ kc,
                                                       const __nv_bfloat16* __restrict__ vc, __nv_bfloat16* __restrict__ out,
                                                       int S, int max_seq) {
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
    const int ntiles = last_q / KB + 1;
    auto load_kv = [&](int j, int buf) {
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

    for (int j = 0; j < ntiles; ++j) {
        const int buf = j & 1;
        if (j + 1 < ntiles) load_kv(j + 1, buf ^ 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();
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

cudaError_t fa_prefill(const void* qkv, const void* kc, const void* vc, void* out, int S, int max_seq, cudaStream_t stream) {
    static bool attr[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        e = cudaFuncSetAttribute(k_fa_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    k_fa_prefill<<<dim3((S + QB - 1) / QB, FA_KV_HEADS), 256, FA_SMEM, stream>>>(
        (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)kc, (const __nv_bfloat16*)vc, (__nv_bfloat16*)out, S, max_seq);
    return cudaGetLastError();
}

}  // namespace mk
