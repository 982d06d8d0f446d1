// NVFP4 x NVFP4 GEMM on the block-scaled 5th-generation tensor-core path (sm_100a):
//   C[M, N] = alpha * (A[M, K] . W[N, K]^T)  (+ R)      C, R bf16 row-major, f32 accumulate in tensor memory
// A and W are e2m1 codes, two per byte (element 2i in the low nibble), rows of K / 2 bytes, with one E4M3 scale per
// 16-element block stored in 128-row x 4-block tiles of 512 bytes:
//   byte offset = ((row / 128) * (K / 64) + block / 4) * 512 + (row % 32) * 16 + ((row % 128) / 32) * 4 + block % 4
// which is what launch_quantize_nvfp4_lm_out and mk_quantize_nvfp4_tensor_scale write, and is the order in which
// tcgen05.cp (32 lanes x 128 bits, replicated to the four lane quadrants) lays a tile into tensor memory for
// tcgen05.mma.kind::mxf4nvf4.block_scale: row r of a 128-row operand reads lane r % 32, column r / 32, one byte per
// block.  alpha carries the two per-tensor scales.  The reference has no such product: its NVFP4 prefill
// dequantises to bf16 and calls cuBLAS (megakernel/kernel_gb10_nvfp4.cu:2127-2145), and its decode multiplies on
// mma.sync after a LUT dequantisation (megakernel/kernel_gb10_nvfp4.cu:528-552).
//
// Persistent kernel, one CTA per SM over 128 x 128 output tiles.  A stage of the shared-memory ring holds 256 k
// (128 bytes per row, 128-byte swizzle) of both operands plus their scale tiles (2 KB each, plain bulk copies);
// warp 0 fills it, one thread of warp 1 copies the scale tiles into tensor memory and issues four K = 64 MMAs per
// stage, warps 2-5 drain finished accumulators (two buffers) while the next tile is being multiplied.
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

constexpr int BM = 128, BN = 128;
constexpr int BKB = 128;                                  // bytes of k per row and stage = 256 e2m1 values
constexpr int BK = 2 * BKB;
constexpr int TILE_BYTES = BM * BKB;                      // 16 KB per operand
constexpr int SF_BYTES = 4 * 512;                         // four 128 x 4 scale tiles per operand and stage
constexpr int STAGE_BYTES = 2 * TILE_BYTES + 2 * SF_BYTES;
constexpr int STAGES = 5;
constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int GEMM_THREADS = 192;
constexpr uint32_t ACC_COLS = 2 * BN;                     // two accumulator buffers
constexpr uint32_t SF_COLS = 2 * 32;                      // two slots of (4 k-steps x 4 columns) x (A, W)
constexpr uint32_t TMEM_COLS = 512;

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar) : "memory");
}

// K-major operand, 128-byte swizzle, rows of 128 bytes, 8-row groups 1024 bytes apart
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3ffffu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// a 512-byte scale tile: 32 rows of 16 bytes, no swizzle, 8-row groups 128 bytes apart
__device__ __forceinline__ uint64_t smem_desc_sf(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3ffffu) >> 4);
    d |= (uint64_t)(128 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// Instruction descriptor of kind::mxf4nvf4: e2m1 x e2m1 (format code 1), E4M3 block scales (scale format 0), both
// operands K-major, N at bit 17 in units of 8, M at bit 24 in units of 16, K = 64.
__device__ __forceinline__ uint32_t idesc_nvfp4(int m, int n) {
    return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_nvfp4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa,
                                           uint32_t sfb, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb) : "memory");
}

__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
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

__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_nvfp4_tn_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                     const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfw, const float* __restrict__ alpha_a,
                     const float* __restrict__ alpha_w, __nv_bfloat16* __restrict__ C, const __nv_bfloat16* __restrict__ R,
                     int M, int N, int K, int ldc, int* err) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ char smem_raw[];
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t a0 = sbase, b0 = a0 + STAGES * TILE_BYTES, fa0 = b0 + STAGES * TILE_BYTES, fb0 = fa0 + STAGES * SF_BYTES;
    const uint32_t bars = sbase + STAGES * STAGE_BYTES;
    const uint32_t full0 = bars, empty0 = bars + 8 * STAGES, tfull0 = bars + 16 * STAGES, tempty0 = tfull0 + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + STAGES * STAGE_BYTES + 16 * STAGES + 32);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = K / BK, kt = K / 64;                    // stages per tile; scale tiles per 128-row block
    const int mt = (M + BM - 1) / BM, ntiles = mt * (N / BN);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(full0 + 8 * s, 1); mbar_init(empty0 + 8 * s, 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(tfull0 + 8 * b, 1); mbar_init(tempty0 + 8 * b, 4); }
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS) : "memory");
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
            const uint64_t pol = l2_policy_evict_last();
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                const int mb = tile % mt, nb = tile / mt;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const uint32_t s = it % STAGES, par = (it / STAGES) & 1u;
                    ok = wait_bounded(empty0 + 8 * s, par ^ 1u, err);
                    if (!ok) break;
                    mbar_expect_tx(full0 + 8 * s, STAGE_BYTES);
                    tma_load_2d(a0 + s * TILE_BYTES, &map_a, kb * BKB, mb * BM, full0 + 8 * s);
                    tma_load_2d(b0 + s * TILE_BYTES, &map_w, kb * BKB, nb * BN, full0 + 8 * s);
                    bulk_g2s(fa0 + s * SF_BYTES, sfa + ((size_t)mb * kt + kb * 4) * 512, SF_BYTES, full0 + 8 * s, pol);
                    bulk_g2s(fb0 + s * SF_BYTES, sfw + ((size_t)nb * kt + kb * 4) * 512, SF_BYTES, full0 + 8 * s, pol);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_nvfp4(BM, BN);
            const uint32_t sf_t = tmem + ACC_COLS;
            uint32_t it = 0, local = 0;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++local) {
                const uint32_t buf = local & 1u, use = local >> 1;
                ok = wait_bounded(tempty0 + 8 * buf, (use & 1u) ^ 1u, err);
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + buf * BN;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const uint32_t s = it % STAGES, par = (it / STAGES) & 1u;
                    ok = wait_bounded(full0 + 8 * s, par, err);
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t ad = smem_desc_sw128(a0 + s * TILE_BYTES), bd = smem_desc_sw128(b0 + s * TILE_BYTES);
                    const uint32_t slot = sf_t + (it & 1u) * 32;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        tmem_cp_sf(slot + 4 * k, smem_desc_sf(fa0 + s * SF_BYTES + 512 * k));
                        tmem_cp_sf(slot + 16 + 4 * k, smem_desc_sf(fb0 + s * SF_BYTES + 512 * k));
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k)       // 64 e2m1 = 32 bytes = 2 descriptor units per step
                        umma_nvfp4(acc, ad + 2 * k, bd + 2 * k, idesc, slot + 4 * k, slot + 16 + 4 * k, (kb | k) ? 1u : 0u);
                    umma_commit(empty0 + 8 * s);
                }
                if (ok) umma_commit(tfull0 + 8 * buf);
            }
        }
    } else {
        const int quad = warp & 3;
        const float alpha = alpha_a[0] * alpha_w[0];
        uint32_t local = 0;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++local) {
            const int m0 = (tile % mt) * BM, n0 = (tile / mt) * BN;
            const uint32_t buf = local & 1u, use = local >> 1;
            ok = wait_bounded(tfull0 + 8 * buf, use & 1u, err);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int row = m0 + quad * 32 + lane;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t v[32];
                const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + buf * BN + (uint32_t)c0;
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
                if (row < M) {
                    __nv_bfloat16* dst = C + (size_t)row * ldc + n0 + c0;
                    const __nv_bfloat16* res = R ? R + (size_t)row * ldc + n0 + c0 : nullptr;
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[j + e]) * alpha;
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
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8 * buf);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
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

// rows x (k / 2) bytes of packed codes; box = 128 bytes x 128 rows, 128-byte swizzle; rows past the end read as zero
bool make_map_u8(CUtensorMap* map, const void* base, int rows, int k_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)k_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)k_bytes};
    cuuint32_t box[2] = {(cuuint32_t)BKB, (cuuint32_t)BM};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t gemm_nvfp4_tn(const void* a_packed, const void* a_scales, const float* a_tensor_scale, const void* w_packed,
                          const void* w_scales, const float* w_tensor_scale, void* C, const void* R, int M, int N, int K, int ldc,
                          int* err_flag, cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0 || N % BN || K % BK) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a_packed) | reinterpret_cast<uintptr_t>(w_packed) | reinterpret_cast<uintptr_t>(C) |
         reinterpret_cast<uintptr_t>(a_scales) | reinterpret_cast<uintptr_t>(w_scales) | reinterpret_cast<uintptr_t>(R)) & 15u)
        return cudaErrorInvalidValue;
    if (ldc % 8) return cudaErrorInvalidValue;
    static int sms = 0;
    static bool attr_done = false;
    if (!sms) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
    }
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(gemm_nvfp4_tn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    CUtensorMap ma, mw;
    if (!make_map_u8(&ma, a_packed, M, K / 2) || !make_map_u8(&mw, w_packed, N, K / 2)) return cudaErrorInvalidValue;
    const int ntiles = ((M + BM - 1) / BM) * (N / BN);
    launch_pdl(gemm_nvfp4_tn_kernel, ntiles < sms ? ntiles : sms, GEMM_THREADS, SMEM, stream, ma, mw, (const uint8_t*)a_scales,
               (const uint8_t*)w_scales, a_tensor_scale, w_tensor_scale, (__nv_bfloat16*)C, (const __nv_bfloat16*)R, M, N, K, ldc,
               err_flag);
    return cudaGetLastError();
}

}  // namespace mk
