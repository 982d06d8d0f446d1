// Persistent single-dispatch bf16 decode step for the Qwen3.5-0.8B hybrid, written for sm_100a.
//
// One CTA per SM (cooperative launch, so co-residency is guaranteed).  Each CTA has one
// producer warp and 16 consumer warps.
//
//  * Weight stream.  The producer warp walks the whole token's weight schedule for this CTA --
//    every layer, every phase, the rows this CTA owns -- and streams it with bulk async copies
//    (cp.async.bulk + mbarrier complete_tx, L2 evict_first) into a 6 x 32 KB shared-memory ring.
//    Weights do not depend on activations, so the producer never waits for another CTA: while
//    consumers wait for activations the next phases' weights keep landing in the ring.
//  * Activation exchange.  There is no grid barrier.  Every activation element travels through
//    global memory as one 64-bit word {f32 value, epoch}; the epoch is unique per launch and
//    layer.  A consumer spins on the words it needs until their epoch matches, so the cost of
//    a phase boundary is one store and one load through L2.
//  * Row products run on the tensor cores: a ring chunk is a 16 x K (or 8 x K, 4 x K) tile of
//    weight rows, each warp owns a K-slice of it and multiplies it with mma.sync m16n8k16
//    against the activation split into three bf16 terms (hi + mid + lo = the f32 value), which
//    occupy 3 of the 8 MMA columns.  Partial sums of the 16 warps meet in shared memory.
//
// Phases per DeltaNet layer: in-proj (+conv/gates) | recurrence | out-proj (+gated norm)
//                            | gate/up (+post norm, SwiGLU) | down (+residual)
// Phases per attention layer: qkv-proj | split-KV attention (+q/k norm, RoPE, KV append)
//                            | o-proj (+merge, sigmoid gate) | gate/up | down
// Last phase: final norm + LM head + grid-wide argmax.
//
// The arithmetic follows the reference decode kernel (megakernel/kernel.cu:425-826): bf16
// weights, bf16 normed activations and residual stream, f32 accumulation and f32 state.
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "mk_common.cuh"
#include "mk_decode.h"

namespace mk {

namespace {

constexpr int NCW = 16;                    // consumer warps
constexpr int NCT = NCW * 32;              // consumer threads
constexpr int NTHREADS = NCT + 32;         // + producer warp
constexpr int MAX_STAGES = 6;               // ring stages: 6 x 32 KB (bf16, NVFP4 layer format), 5 x 36 KB (tensor-scale NVFP4) or
                                            // 4 x 36 KB plus the tensor-core activation operand (tensor-scale NVFP4 on tcgen05)
constexpr int RING_BYTES = 196608;
constexpr int XK = 224;                    // largest K-slice of a warp (elements)
constexpr int XSW = 3 * XK / 2;            // 32-bit words of staging per warp: three bf16 planes of XK elements

constexpr int OFF_RING = 0;
constexpr int OFF_SCRATCH = RING_BYTES;          // activation staging (16 x 224 floats) / attention merge
constexpr int SCRATCH_BYTES = 21504;           // 16 x 1344 B of staging; attention uses 16640 B of merge slots + 4096 B of q
constexpr int OFF_PART = OFF_SCRATCH + SCRATCH_BYTES;      // 2 x (4 chunks x 16 warps x 16 rows) partial sums
constexpr int PART_HALF = 4 * NCW * 16;                    // floats; phases alternate between the halves
constexpr int PART_BYTES = 2 * PART_HALF * 4;
constexpr int OFF_RED = OFF_PART + PART_BYTES;             // 32 floats
constexpr int OFF_MISC = OFF_RED + 128;                    // 8 ints
constexpr int OFF_BAR = OFF_MISC + 32;                     // full[stages], empty[stages]
constexpr int OFF_ROPE = OFF_BAR + 2 * MAX_STAGES * 8;         // cos[32] | sin[32] of the step's position
constexpr int OFF_LAYERS = OFF_ROPE + 256;                 // copy of the layer pointer table
constexpr int OFF_DBG = OFF_LAYERS + MAX_LAYERS * (int)sizeof(LayerWeightsNVFP4TS);   // traced variants: 16 counters
constexpr int SMEM_BYTES = OFF_DBG + 64;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

enum { MISC_ABORT = 0, MISC_LAST = 1, MISC_TOKEN = 2, MISC_DETAIL = 3 };

// pause between failed polls of a flagged word: keeps the waiting threads of 148 CTAs from
// saturating the L2 slices that hold the words (and from delaying the stores they wait for)
#ifndef MK_POLL_SLEEP_NS
#define MK_POLL_SLEEP_NS 0
#endif
#define MK_POLL_BACKOFF() do { if (MK_POLL_SLEEP_NS > 0) __nanosleep(MK_POLL_SLEEP_NS); } while (0)

enum PhaseType { T_DN_IN = 0, T_DN_REC, T_DN_OUT, T_FA_IN, T_FA_ATT, T_FA_OUT, T_GATEUP, T_DOWN, T_LM };

}  // namespace

namespace plain {
namespace {
#define MK_TRACE 0
#define MK_WFMT 0
#include "decode_body.cuh"
#undef MK_WFMT
#undef MK_TRACE
}  // namespace
}  // namespace plain

namespace nvfp4 {
namespace {
#define MK_TRACE 0
#define MK_WFMT 1
#include "decode_body.cuh"
#undef MK_WFMT
#undef MK_TRACE
}  // namespace
}  // namespace nvfp4

namespace nvfp4ts {
namespace {
#define MK_TRACE 0
#define MK_WFMT 2
#include "decode_body.cuh"
#undef MK_WFMT
#undef MK_TRACE
}  // namespace
}  // namespace nvfp4ts

namespace traced {
namespace {
#define MK_TRACE 1
#define MK_WFMT 0
#include "decode_body.cuh"
#undef MK_WFMT
#undef MK_TRACE
}  // namespace
}  // namespace traced

namespace traced_ts {
namespace {
#define MK_TRACE 1
#define MK_WFMT 2
#include "decode_body.cuh"
#undef MK_WFMT
#undef MK_TRACE
}  // namespace
}  // namespace traced_ts

namespace nvfp4mma {
namespace {
#define MK_TRACE 0
#define MK_WFMT 3
#include "decode_body.cuh"
#undef MK_WFMT
#undef MK_TRACE
}  // namespace
}  // namespace nvfp4mma

namespace traced_mma {
namespace {
#define MK_TRACE 1
#define MK_WFMT 3
#include "decode_body.cuh"
#undef MK_WFMT
#undef MK_TRACE
}  // namespace
}  // namespace traced_mma

size_t decode_smem_bytes() { return SMEM_BYTES; }
int decode_image_ctas() { return nvfp4mma::U_CTAS; }

int decode_max_grid() {
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cudaFuncSetAttribute(plain::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, plain::decode_megakernel_bf16, NTHREADS, SMEM_BYTES) != cudaSuccess)
        return 0;
    int g = sms * per_sm;
    return g > MAX_GRID ? MAX_GRID : g;
}

// RoPE frequencies: inv_freq_i = theta^(-2i/64) evaluated in double; the kernel forms angle = position * inv_freq
// in f32 like the reference (megakernel/kernel.cu:468-470) and takes an accurate f32 sine and cosine of it.
void fill_rope(DecodeParams& p) {
    for (int i = 0; i < FA_ROT / 2; ++i) p.rope_inv_freq[i] = (float)(1.0 / pow(ROPE_THETA, (2.0 * i) / FA_ROT));
}

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [rows][256] bf16 cache, boxes of 64 elements x 32 rows, 128-byte swizzle; rows past the end read as zeros
bool make_kv_map(CUtensorMap* map, const void* base, unsigned long long rows) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* q = nullptr;
        cudaDriverEntryPointQueryResult r;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) != cudaSuccess || !q) return false;
        fn = (EncodeTiledFn)q;
    }
    cuuint64_t dims[2] = {(cuuint64_t)FA_HEAD_DIM, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)FA_HEAD_DIM * 2};
    cuuint32_t box[2] = {64, 32};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct KvMapCache { const void* k = nullptr; const void* v = nullptr; unsigned long long rows = 0; CUtensorMap mk, mv; };
thread_local KvMapCache g_kvmaps;

}  // namespace

cudaError_t launch_decode_kernel(const DecodeParams& p_in, int grid, cudaStream_t stream) {
    DecodeParams p = p_in;
    // every attention layer owns 2 * max_seq rows of each cache; n_fa_layers == 0 means the reference model's pattern
    // (every fourth layer)
    const int n_fa = p.n_fa_layers > 0 ? p.n_fa_layers : (p.num_layers / 4 > 0 ? p.num_layers / 4 : 1);
    const unsigned long long rows = (unsigned long long)n_fa * FA_KV_HEADS * (unsigned long long)p.max_seq_len;
    KvMapCache& kc = g_kvmaps;
    if (kc.k != p.k_cache || kc.v != p.v_cache || kc.rows != rows) {
        if (!make_kv_map(&kc.mk, p.k_cache, rows) || !make_kv_map(&kc.mv, p.v_cache, rows)) return cudaErrorInvalidValue;
        kc.k = p.k_cache; kc.v = p.v_cache; kc.rows = rows;
    }
    p.map_k = kc.mk; p.map_v = kc.mv;
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !attr_done[dev]) {
        e = cudaFuncSetAttribute(plain::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(traced::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(nvfp4::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(nvfp4ts::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(traced_ts::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(nvfp4mma::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(traced_mma::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_done[dev] = true;
    }
    if (grid < MIN_GRID || grid > MAX_GRID) return cudaErrorInvalidConfiguration;
    void* args[] = {(void*)&p};
    if (p.wfmt == 3 && (grid != nvfp4mma::U_CTAS || p.act_terms < 1 || p.act_terms > 8 || p.lm_image_chunks < 1))
        return cudaErrorInvalidConfiguration;
    const void* fn = (p.wfmt == 3 && p.trace) ? (const void*)traced_mma::decode_megakernel_bf16
                   : p.wfmt == 3 ? (const void*)nvfp4mma::decode_megakernel_bf16
                   : (p.wfmt == 2 && p.trace) ? (const void*)traced_ts::decode_megakernel_bf16
                   : p.wfmt == 2 ? (const void*)nvfp4ts::decode_megakernel_bf16
                   : p.wfmt == 1 ? (const void*)nvfp4::decode_megakernel_bf16
                   : p.trace   ? (const void*)traced::decode_megakernel_bf16
                               : (const void*)plain::decode_megakernel_bf16;
    return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(p.wfmt == 3 ? nvfp4mma::NTHR : NTHREADS), args, SMEM_BYTES, stream);
}

cudaError_t launch_wait_selftest(const DecodeParams& p, cudaStream_t stream) {
    plain::wait_selftest_kernel<<<2, 32, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace mk
