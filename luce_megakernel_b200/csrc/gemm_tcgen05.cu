// bf16 GEMM for the prefill projections on the 5th-generation tensor cores (sm_100a):
//   C[M, N] = A[M, K] . W[N, K]^T     A, W, C bf16 row-major (both operands K-major), f32 accumulate
// optionally C += R (residual, bf16 [M, N]) before the bf16 rounding.
//
// Persistent kernel, one CTA per SM, each walking 128 x BN output tiles (BN = 256, or 128 for small
// problems).  Warp 0 streams A and W tiles (rows x 64 k, 128-byte swizzle) with TMA into a
// shared-memory ring; one thread of warp 1 issues tcgen05.mma (M128 x BN x K16, cta_group::1) into one
// of two accumulator buffers in tensor memory; warps 2-5 read a finished accumulator back with
// tcgen05.ld (each warp its own 32-lane quadrant), add the residual and store bf16 while the MMA
// thread is already working on the next tile.  With BN = 256 an MMA reads 12 KB of shared memory per
// 128 tensor-core cycles, which stays under the shared-memory bandwidth; 128-wide tiles sit at it.
// M is the token dimension: rows beyond M are zero-filled by TMA and not stored.
// Variants of the same kernel: a K split for products with far fewer tiles than SMs (f32 partial tiles, added up by
// gemm_splitk_reduce, or by gemm_splitk_reduce_norm which also writes the RMSNorm of the finished row); GLU (gate and up
// rows of the same outputs stacked in one B tile, silu(gate) * up in the epilogue); two products sharing A in one
// launch (the tiles of both, two weight maps, two outputs).
// Every wait is bounded; on expiry the kernel sets *err and leaves.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "mk_common.cuh"
#include "mk_prefill.h"

namespace mk {

namespace {

constexpr int BM = 128, BK = 64;
constexpr int TILE_A_BYTES = BM * BK * 2;                 // 16 KB
constexpr int GEMM_THREADS = 192;
template <int BN> struct Cfg {
    static constexpr int STAGES = (BN == 256) ? 4 : 6;
    static constexpr int TILE_B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = TILE_A_BYTES + TILE_B_BYTES;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256;
    static constexpr uint32_t TMEM_COLS = 2 * BN;         // two accumulator buffers
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar) : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of 128 bytes,
// 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3ffffu) >> 4);             // start address, 16-byte units
    d |= (uint64_t)1 << 16;                               // leading-dimension byte offset (unused with swizzle)
    d |= (uint64_t)(1024 >> 4) << 32;                     // stride-dimension byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;                               // descriptor version of sm_100
    d |= (uint64_t)2 << 61;                               // layout: 128-byte swizzle
    return d;
}

// Instruction descriptor of tcgen05.mma.kind::f16: bf16 x bf16 -> f32, both operands K-major.
__device__ __forceinline__ uint32_t idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, int* err) {
    for (uint32_t n = 0; n < (1u << 24); ++n)
        if (mbar_try_wait(bar, parity)) return true;
    atomicExch(err, 1);
    return false;
}

// SPLIT: the K range is cut into `ks` parts, a work item is (tile, part) and leaves its f32 partial tile in
// `partial` ([part][M][N]); gemm_splitk_reduce adds the parts (and the residual) and rounds to bf16.  Used when
// a problem has far fewer tiles than the machine has SMs (the K = 2048 / 3584 projections of a short prompt).
// GLU: the weight matrix holds two blocks of rows, gate rows [0, N) and up rows [glu_off, glu_off + N); a tile's B
// operand is BN/2 gate rows stacked on the BN/2 up rows of the same outputs (two tensor copies per stage), so the
// accumulator holds gate and up of BN/2 output columns side by side and the epilogue stores
// silu(bf16(gate)) * bf16(up) -- bit for bit what the separate SwiGLU kernel makes of the two rounded products
// (reference: megakernel/prefill.cu:1239-1247) -- without the [M, 2 N] intermediate ever reaching memory.
template <int BN, bool SPLIT, bool GLU = false>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                    __nv_bfloat16* __restrict__ C, const __nv_bfloat16* __restrict__ R, int M, int N, int K, int ldc,
                    int* err, float* __restrict__ partial, int ks, int glu_off,
                    const __grid_constant__ CUtensorMap map_w2, __nv_bfloat16* __restrict__ C2, int n_split, int ldc2) {
    // n_split > 0: two products that share A in one launch -- output columns [0, n_split) come from map_w into C,
    // columns [n_split, N) from map_w2 into C2 (row pitch ldc2); no residual, no K split
    constexpr int BNO = GLU ? BN / 2 : BN;                // output columns per tile
    // the next kernel may be scheduled now; this one sets up barriers and tensor memory while its predecessor
    // drains and waits for it (griddepcontrol.wait below) before the first operand is read
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    typedef Cfg<BN> G;
    constexpr int STAGES = G::STAGES;
    extern __shared__ char smem_raw[];
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t a0 = sbase, b0 = sbase + STAGES * TILE_A_BYTES;
    const uint32_t bars = sbase + STAGES * G::STAGE_BYTES;
    const uint32_t full0 = bars, empty0 = bars + 8 * STAGES, tfull0 = bars + 16 * STAGES, tempty0 = tfull0 + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + STAGES * G::STAGE_BYTES + 16 * STAGES + 32);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk_all = K / BK;
    const int mt = (M + BM - 1) / BM, ntiles = mt * (N / BNO) * (SPLIT ? ks : 1);
    // work item -> (tile, K part); part p covers k-steps [p nk / ks, (p + 1) nk / ks)
    auto item = [&](int it_, int& m0, int& n0, int& kb0, int& kb1, int& part) {
        const int tile = SPLIT ? it_ / ks : it_;
        part = SPLIT ? it_ - tile * ks : 0;
        m0 = (tile % mt) * BM; n0 = (tile / mt) * BNO;
        kb0 = SPLIT ? (part * nk_all) / ks : 0;
        kb1 = SPLIT ? ((part + 1) * nk_all) / ks : nk_all;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(full0 + 8 * s, 1); mbar_init(empty0 + 8 * s, 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(tfull0 + 8 * b, 1); mbar_init(tempty0 + 8 * b, 4); }
        fence_mbar_init();
    }
    if (warp == 1) {   // one warp allocates the accumulator columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(G::TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
    bool ok = true;
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                int m0, n0, kb0, kb1, part;
                item(tile, m0, n0, kb0, kb1, part);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const uint32_t s = it % STAGES, par = (it / STAGES) & 1u;
                    ok = wait_bounded(empty0 + 8 * s, par ^ 1u, err);
                    if (!ok) break;
                    mbar_expect_tx(full0 + 8 * s, G::STAGE_BYTES);
                    tma_load_2d(a0 + s * TILE_A_BYTES, &map_a, kb * BK, m0, full0 + 8 * s);
                    if (!GLU && !SPLIT && n_split > 0 && n0 >= n_split)
                        tma_load_2d(b0 + s * G::TILE_B_BYTES, &map_w2, kb * BK, n0 - n_split, full0 + 8 * s);
                    else
                        tma_load_2d(b0 + s * G::TILE_B_BYTES, &map_w, kb * BK, n0, full0 + 8 * s);
                    if (GLU) tma_load_2d(b0 + s * G::TILE_B_BYTES + BNO * BK * 2, &map_w, kb * BK, glu_off + n0, full0 + 8 * s);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16(BM, BN);
            uint32_t it = 0, local = 0;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++local) {
                const uint32_t buf = local & 1u, use = local >> 1;
                ok = wait_bounded(tempty0 + 8 * buf, (use & 1u) ^ 1u, err);     // epilogue has drained this buffer
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + buf * BN;
                int m0, n0, kb0, kb1, part;
                item(tile, m0, n0, kb0, kb1, part);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const uint32_t s = it % STAGES, par = (it / STAGES) & 1u;
                    ok = wait_bounded(full0 + 8 * s, par, err);
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t ad = smem_desc_sw128(a0 + s * TILE_A_BYTES), bd = smem_desc_sw128(b0 + s * G::TILE_B_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)   // 16 bf16 = 32 bytes = 2 descriptor units per step
                        umma(acc, ad + 2 * k, bd + 2 * k, idesc, ((kb - kb0) | k) ? 1u : 0u);
                    umma_commit(empty0 + 8 * s);        // frees the stage once these MMAs have read it
                }
                if (ok) umma_commit(tfull0 + 8 * buf);  // accumulator complete
            }
        }
    } else {
        // epilogue warps 2..5: warp w may touch TMEM lanes 32*(w%4) .. +31
        const int quad = warp & 3;
        uint32_t local = 0;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++local) {
            int m0, n0, kb0, kb1, part;
            item(tile, m0, n0, kb0, kb1, part);
            const uint32_t buf = local & 1u, use = local >> 1;
            ok = wait_bounded(tfull0 + 8 * buf, use & 1u, err);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int row = m0 + quad * 32 + lane;
#pragma unroll 1
            for (int c0 = 0; c0 < BNO; c0 += 32) {
                uint32_t v[32];
                const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + buf * BN + (uint32_t)c0;
                uint32_t u[32];
                if (GLU) {
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]),
                          "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
                          "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]),
                          "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15]),
                          "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]),
                          "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]),
                          "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]),
                          "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
                        : "r"(taddr + (uint32_t)BNO) : "memory");
                }
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                    "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
                      "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
                      "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                    : "r"(taddr) : "memory");
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (GLU) {
                    if (row < M) {
                        __nv_bfloat16* dst = C + (size_t)row * ldc + n0 + c0;
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            uint32_t o[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                // both products rounded to bf16 first, as when they were stored and read back
                                const __nv_bfloat162 gp = __floats2bfloat162_rn(__uint_as_float(v[j + 2 * e]), __uint_as_float(v[j + 2 * e + 1]));
                                const __nv_bfloat162 up = __floats2bfloat162_rn(__uint_as_float(u[j + 2 * e]),
                                                                                __uint_as_float(u[j + 2 * e + 1]));
                                const uint32_t gw = *reinterpret_cast<const uint32_t*>(&gp), uw = *reinterpret_cast<const uint32_t*>(&up);
                                const __nv_bfloat162 p = __floats2bfloat162_rn(silu_f(bf_lo(gw)) * bf_lo(uw), silu_f(bf_hi(gw)) * bf_hi(uw));
                                o[e] = *reinterpret_cast<const uint32_t*>(&p);
                            }
                            *reinterpret_cast<uint4*>(dst + j) = make_uint4(o[0], o[1], o[2], o[3]);
                        }
                    }
                } else if (SPLIT) {
                    if (row < M) {
                        float4* dst = reinterpret_cast<float4*>(partial + ((size_t)part * M + row) * N + n0 + c0);
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                 __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
                    }
                } else if (row < M) {
                    const bool second = n_split > 0 && n0 >= n_split;
                    __nv_bfloat16* dst = second ? C2 + (size_t)row * ldc2 + (n0 - n_split) + c0 : C + (size_t)row * ldc + n0 + c0;
                    const __nv_bfloat16* res = R ? R + (size_t)row * ldc + n0 + c0 : nullptr;
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[j + e]);
                        if (res) {
                            const uint4 r4 = *reinterpret_cast<const uint4*>(res + j);
                            f[0] += bf_lo(r4.x); f[1] += bf_hi(r4.x); f[2] += bf_lo(r4.y); f[3] += bf_hi(r4.y);
                            f[4] += bf_lo(r4.z); f[5] += bf_hi(r4.z); f[6] += bf_lo(r4.w); f[7] += bf_hi(r4.w);
                        }
                        uint4 o;
                        __nv_bfloat162 p0 = __floats2bfloat162_rn(f[0], f[1]), p1 = __floats2bfloat162_rn(f[2], f[3]);
                        __nv_bfloat162 p2 = __floats2bfloat162_rn(f[4], f[5]), p3 = __floats2bfloat162_rn(f[6], f[7]);
                        o.x = *reinterpret_cast<uint32_t*>(&p0); o.y = *reinterpret_cast<uint32_t*>(&p1);
                        o.z = *reinterpret_cast<uint32_t*>(&p2); o.w = *reinterpret_cast<uint32_t*>(&p3);
                        *reinterpret_cast<uint4*>(dst + j) = o;
                    }
                }
            }
            // hand the accumulator buffer back to the MMA thread
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8 * buf);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::TMEM_COLS) : "memory");
    }
}

// C[row][col] = bf16(sum over parts + residual), 8 columns per thread
__global__ void gemm_splitk_reduce(const float* __restrict__ partial, int ks, const __nv_bfloat16* __restrict__ R,
                                   __nv_bfloat16* __restrict__ C, int M, int N, int ldc) {
    pdl_enter();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int n8 = N / 8;
    if (i >= (size_t)M * n8) return;
    const int row = (int)(i / n8), col = (int)(i - (size_t)row * n8) * 8;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < ks; ++p) {
        const float4* src = reinterpret_cast<const float4*>(partial + ((size_t)p * M + row) * N + col);
        const float4 a = src[0], b = src[1];
        f[0] += a.x; f[1] += a.y; f[2] += a.z; f[3] += a.w; f[4] += b.x; f[5] += b.y; f[6] += b.z; f[7] += b.w;
    }
    if (R) {
        const uint4 r4 = *reinterpret_cast<const uint4*>(R + (size_t)row * ldc + col);
        f[0] += bf_lo(r4.x); f[1] += bf_hi(r4.x); f[2] += bf_lo(r4.y); f[3] += bf_hi(r4.y);
        f[4] += bf_lo(r4.z); f[5] += bf_hi(r4.z); f[6] += bf_lo(r4.w); f[7] += bf_hi(r4.w);
    }
    uint4 o;
    __nv_bfloat162 p0 = __floats2bfloat162_rn(f[0], f[1]), p1 = __floats2bfloat162_rn(f[2], f[3]);
    __nv_bfloat162 p2 = __floats2bfloat162_rn(f[4], f[5]), p3 = __floats2bfloat162_rn(f[6], f[7]);
    o.x = *reinterpret_cast<uint32_t*>(&p0); o.y = *reinterpret_cast<uint32_t*>(&p1);
    o.z = *reinterpret_cast<uint32_t*>(&p2); o.w = *reinterpret_cast<uint32_t*>(&p3);
    *reinterpret_cast<uint4*>(C + (size_t)row * ldc + col) = o;
}

// The same for N = 1024 with the RMSNorm of the finished row behind it (one block of four warps per row, warp i =
// columns [256 i, 256 i + 256), 8 per lane): the row is rounded to bf16 and stored, and
// out = bf16(x rsqrt(mean x^2 + eps) (1 + w)) is computed from the rounded values.  The sum of squares is taken in the
// order of the prefill's RMSNorm kernel (lane l adds its 32 values chunk after chunk, then a butterfly over the lanes),
// so the pair gives the bits of the two kernels it replaces (reference: megakernel/prefill.cu:72-88).
__global__ void __launch_bounds__(128) gemm_splitk_reduce_norm(const float* __restrict__ partial, int ks, const __nv_bfloat16* __restrict__ R,
                                                              __nv_bfloat16* __restrict__ C, int M, int ldc,
                                                              const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ normed) {
    pdl_enter();
    constexpr int N = 1024;
    __shared__ float sq[4][8][32];                        // [chunk][element][lane]
    __shared__ float s_rstd;
    const int row = blockIdx.x, i = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int col = (i * 32 + lane) * 8;
    const uint4 wu = __ldg(reinterpret_cast<const uint4*>(w) + i * 32 + lane);
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < ks; ++p) {
        const float4* src = reinterpret_cast<const float4*>(partial + ((size_t)p * M + row) * N + col);
        const float4 a = src[0], b = src[1];
        f[0] += a.x; f[1] += a.y; f[2] += a.z; f[3] += a.w; f[4] += b.x; f[5] += b.y; f[6] += b.z; f[7] += b.w;
    }
    if (R) {
        const uint4 r4 = *reinterpret_cast<const uint4*>(R + (size_t)row * ldc + col);
        f[0] += bf_lo(r4.x); f[1] += bf_hi(r4.x); f[2] += bf_lo(r4.y); f[3] += bf_hi(r4.y);
        f[4] += bf_lo(r4.z); f[5] += bf_hi(r4.z); f[6] += bf_lo(r4.w); f[7] += bf_hi(r4.w);
    }
    float v[8];
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 p2 = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
        o[e] = *reinterpret_cast<const uint32_t*>(&p2);
        v[2 * e] = bf_lo(o[e]); v[2 * e + 1] = bf_hi(o[e]);
    }
    *reinterpret_cast<uint4*>(C + (size_t)row * ldc + col) = make_uint4(o[0], o[1], o[2], o[3]);
#pragma unroll
    for (int e = 0; e < 8; ++e) sq[i][e][lane] = v[e] * v[e];
    __syncthreads();
    if (i == 0) {
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 8; ++e) ss += sq[c][e][lane];
        ss = warp_sum(ss);
        if (lane == 0) s_rstd = rsqrtf(ss * (1.0f / N) + RMS_EPS);
    }
    __syncthreads();
    const float rstd = s_rstd;
    const uint32_t wq[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 p2 = __floats2bfloat162_rn(v[2 * e] * rstd * (1.0f + bf_lo(wq[e])), v[2 * e + 1] * rstd * (1.0f + bf_hi(wq[e])));
        o[e] = *reinterpret_cast<const uint32_t*>(&p2);
    }
    reinterpret_cast<uint4*>(normed + (size_t)row * N)[i * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess) fn = (EncodeTiledFn)p;
    }
    return fn;
}

// rows x k bf16 matrix with row pitch `ld` elements; box = 64 k x box_rows rows, 128-byte swizzle
bool make_map(CUtensorMap* map, const void* base, int rows, int k, int ld, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
cudaError_t launch_gemm(const void* A, const void* W, void* C, const void* R, int M, int N, int K, int lda, int ldc, int* err_flag,
                        int sms, float* splitk_ws, size_t splitk_bytes, cudaStream_t stream, const void* norm_w = nullptr,
                        void* norm_out = nullptr, bool* norm_done = nullptr) {
    static bool attr_done = false;
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tn_kernel<BN, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_bf16_tn_kernel<BN, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    CUtensorMap ma, mw;
    if (!make_map(&ma, A, M, K, lda, BM) || !make_map(&mw, W, N, K, K, BN)) return cudaErrorInvalidValue;
    const int ntiles = ((M + BM - 1) / BM) * (N / BN);
    // split K when the tiles would leave most SMs idle and every part still has a few k-steps
    int ks = sms / ntiles;
    if (ks > 4) ks = 4;
    while (ks > 1 && (K / BK) / ks < 4) --ks;
    // the f32 partials live in the caller's workspace (nothing is allocated here: the call must stay capturable into
    // a CUDA graph); without room for them the product is not split
    while (ks > 1 && (size_t)ks * M * N * sizeof(float) > splitk_bytes) --ks;
    if (BN == 128 && ks >= 2 && K >= 2048) {      // only the long-K projections: K = 1024 products keep one summation order
        float* ws = splitk_ws;
        const int items = ntiles * ks;
        launch_pdl(gemm_bf16_tn_kernel<BN, true>, items < sms ? items : sms, GEMM_THREADS, Cfg<BN>::SMEM, stream, ma, mw, nullptr, nullptr, M, N, K, ldc, err_flag, ws, ks, 0, ma, nullptr, 0, 0);
        if (norm_w && norm_out && N == 1024) {
            launch_pdl(gemm_splitk_reduce_norm, (unsigned)M, 128, 0, stream, (const float*)ws, ks, (const __nv_bfloat16*)R,
                       (__nv_bfloat16*)C, M, ldc, (const __nv_bfloat16*)norm_w, (__nv_bfloat16*)norm_out);
            if (norm_done) *norm_done = true;
            return cudaGetLastError();
        }
        const size_t n = (size_t)M * (N / 8);
        launch_pdl(gemm_splitk_reduce, (unsigned)((n + 255) / 256), 256, 0, stream, ws, ks, (const __nv_bfloat16*)R, (__nv_bfloat16*)C, M, N, ldc);
        return cudaGetLastError();
    }
    launch_pdl(gemm_bf16_tn_kernel<BN, false>, ntiles < sms ? ntiles : sms, GEMM_THREADS, Cfg<BN>::SMEM, stream, ma, mw, (__nv_bfloat16*)C, (const __nv_bfloat16*)R, M, N, K, ldc, err_flag, nullptr, 1, 0, ma, nullptr, 0, 0);
    return cudaGetLastError();
}

template <int BN>
cudaError_t launch_gemm_glu(const void* A, const void* W, void* C, int M, int N, int K, int lda, int ldc, int glu_off, int* err_flag,
                            int sms, cudaStream_t stream) {
    static bool attr_done = false;
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tn_kernel<BN, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    CUtensorMap ma, mw;
    if (!make_map(&ma, A, M, K, lda, BM) || !make_map(&mw, W, glu_off + N, K, K, BN / 2)) return cudaErrorInvalidValue;
    const int ntiles = ((M + BM - 1) / BM) * (N / (BN / 2));
    launch_pdl(gemm_bf16_tn_kernel<BN, false, true>, ntiles < sms ? ntiles : sms, GEMM_THREADS, Cfg<BN>::SMEM, stream, ma, mw,
               (__nv_bfloat16*)C, (const __nv_bfloat16*)nullptr, M, N, K, ldc, err_flag, (float*)nullptr, 1, glu_off, ma, (__nv_bfloat16*)nullptr, 0, 0);
    return cudaGetLastError();
}

}  // namespace

template <int BN>
cudaError_t launch_gemm_dual(const void* A, const void* W1, void* C1, int N1, int ldc1, const void* W2, void* C2, int N2, int ldc2,
                             int M, int K, int lda, int* err_flag, int sms, cudaStream_t stream) {
    static bool attr_done = false;
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tn_kernel<BN, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    CUtensorMap ma, mw1, mw2;
    if (!make_map(&ma, A, M, K, lda, BM) || !make_map(&mw1, W1, N1, K, K, BN) || !make_map(&mw2, W2, N2, K, K, BN))
        return cudaErrorInvalidValue;
    const int ntiles = ((M + BM - 1) / BM) * ((N1 + N2) / BN);
    launch_pdl(gemm_bf16_tn_kernel<BN, false>, ntiles < sms ? ntiles : sms, GEMM_THREADS, Cfg<BN>::SMEM, stream, ma, mw1, (__nv_bfloat16*)C1,
               (const __nv_bfloat16*)nullptr, M, N1 + N2, K, ldc1, err_flag, (float*)nullptr, 1, 0, mw2, (__nv_bfloat16*)C2, N1, ldc2);
    return cudaGetLastError();
}

// Two products that share their left operand in one launch: C1[M, N1] = A . W1^T and C2[M, N2] = A . W2^T (the qkv and
// the z projection of a DeltaNet layer).  The tiles are the tiles of the two separate products, so are the bits.
cudaError_t gemm_bf16_tn_dual(const void* A, const void* W1, void* C1, int N1, int ldc1, const void* W2, void* C2, int N2, int ldc2,
                              int M, int K, int lda, int* err_flag, cudaStream_t stream) {
    if (M <= 0 || N1 <= 0 || N2 <= 0 || K <= 0 || N1 % 256 || N2 % 256 || K % BK) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W1) | reinterpret_cast<uintptr_t>(W2) |
         reinterpret_cast<uintptr_t>(C1) | reinterpret_cast<uintptr_t>(C2)) & 15u)
        return cudaErrorInvalidValue;
    if ((lda % 8) || (ldc1 % 8) || (ldc2 % 8)) return cudaErrorInvalidValue;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const int mt = (M + BM - 1) / BM;
    if (mt * ((N1 + N2) / 256) >= sms)
        return launch_gemm_dual<256>(A, W1, C1, N1, ldc1, W2, C2, N2, ldc2, M, K, lda, err_flag, sms, stream);
    return launch_gemm_dual<128>(A, W1, C1, N1, ldc1, W2, C2, N2, ldc2, M, K, lda, err_flag, sms, stream);
}

// C[M, N] = silu(A . Wg^T) * (A . Wu^T) with Wg = rows [0, N) and Wu = rows [glu_off, glu_off + N) of W, both
// products rounded to bf16 before the activation.  N % 128 == 0.
cudaError_t gemm_bf16_glu(const void* A, const void* W, void* C, int M, int N, int K, int lda, int ldc, int glu_off, int* err_flag,
                          cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0 || N % 128 || K % BK || glu_off < N) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(C)) & 15u)
        return cudaErrorInvalidValue;
    if ((lda % 8) || (ldc % 8)) return cudaErrorInvalidValue;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const int mt = (M + BM - 1) / BM;
    if (mt * (N / 128) >= sms) return launch_gemm_glu<256>(A, W, C, M, N, K, lda, ldc, glu_off, err_flag, sms, stream);
    return launch_gemm_glu<128>(A, W, C, M, N, K, lda, ldc, glu_off, err_flag, sms, stream);
}

cudaError_t gemm_bf16_tn(const void* A, const void* W, void* C, const void* R, int M, int N, int K, int lda, int ldc,
                         int* err_flag, float* splitk_ws, size_t splitk_bytes, cudaStream_t stream, const void* norm_w,
                         void* norm_out, bool* norm_done) {
    if (norm_done) *norm_done = false;
    if (M <= 0 || N <= 0 || K <= 0 || N % 128 || K % BK) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(C)) & 15u)
        return cudaErrorInvalidValue;
    if ((lda % 8) || (ldc % 8)) return cudaErrorInvalidValue;
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
    }
    // 256-wide tiles when they take fewer rounds of the machine than 128-wide ones at their cost: a 256-wide tile is
    // twice the work at about 1.5 x the time (a 128-wide MMA instruction costs ~2/3 of a 256-wide one: measured
    // 43 % against 61-68 % tensor-pipe activity on the same prompt).  128-wide tiles keep more SMs busy on small
    // problems and are the ones that can be split along K.
    const int mt = (M + BM - 1) / BM;
    if (N % 256 == 0) {
        const int t256 = mt * (N / 256), t128 = mt * (N / 128);
        const int rounds256 = (t256 + sms - 1) / sms, rounds128 = (t128 + sms - 1) / sms;
        if (t256 >= sms || (t128 > sms && 3 * rounds256 <= 2 * rounds128))
            return launch_gemm<256>(A, W, C, R, M, N, K, lda, ldc, err_flag, sms, splitk_ws, splitk_bytes, stream);
    }
    return launch_gemm<128>(A, W, C, R, M, N, K, lda, ldc, err_flag, sms, splitk_ws, splitk_bytes, stream, norm_w, norm_out, norm_done);
}

}  // namespace mk
