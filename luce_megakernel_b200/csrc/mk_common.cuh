// Shared definitions for the sm_100a kernels: model constants, the layer pointer-table
// layout, PTX wrappers (mbarrier, bulk async copy, acquire/release), small math helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mk {

// ---- model constants (reference: megakernel/kernel.cu:17-45, megakernel/model.py:6-36) ----
constexpr int HIDDEN = 1024;
constexpr int INTER = 3584;
constexpr int MAX_LAYERS = 24;
constexpr int DEFAULT_VOCAB = 248320;
constexpr float RMS_EPS = 1e-6f;

constexpr int FA_Q_HEADS = 8;
constexpr int FA_KV_HEADS = 2;
constexpr int FA_GQA = FA_Q_HEADS / FA_KV_HEADS;
constexpr int FA_HEAD_DIM = 256;
constexpr int FA_Q_SIZE = FA_Q_HEADS * FA_HEAD_DIM;      // 2048
constexpr int FA_QPROJ = 2 * FA_Q_SIZE;                  // 4096, per head [q | gate]
constexpr int FA_KV_SIZE = FA_KV_HEADS * FA_HEAD_DIM;    // 512
constexpr int FA_QKV_ROWS = FA_QPROJ + 2 * FA_KV_SIZE;   // 5120
constexpr int FA_ROT = 64;
constexpr double ROPE_THETA = 1.0e7;

constexpr int DN_HEADS = 16;
constexpr int DN_KEY = 128;
constexpr int DN_VAL = 128;
constexpr int DN_QK = DN_HEADS * DN_KEY;                 // 2048
constexpr int DN_V = DN_HEADS * DN_VAL;                  // 2048
constexpr int DN_CONV_CH = 2 * DN_QK + DN_V;             // 6144
constexpr int DN_CONV_K = 4;
constexpr int DN_IN_ROWS = DN_CONV_CH + DN_V + 2 * DN_HEADS;   // qkv | z | beta | alpha = 8224

// Device pointer table entry, 128 bytes, written by the caller
// (reference: megakernel/torch_bindings.cpp:30-34, megakernel/model.py:160-177).
struct LayerWeights {
    int layer_type;        // 0 = Gated DeltaNet, 1 = full attention
    int pad[3];
    const void* ptrs[14];
};
static_assert(sizeof(LayerWeights) == 128, "pointer table entry must be 128 bytes");

// Pointer table entry of the NVFP4 decode path, 208 bytes: quantised matrices take two slots
// (packed data, fp16 group scales) (reference: megakernel/torch_bindings.cpp:37-42,
// megakernel/kernel_gb10_nvfp4.cu:156-203, megakernel/model_nvfp4.py:274-311).
struct LayerWeightsNVFP4 {
    int layer_type;
    int group_size;
    int pad[2];
    const void* ptrs[24];
};
static_assert(sizeof(LayerWeightsNVFP4) == 208, "NVFP4 pointer table entry must be 208 bytes");

// Pointer table entry of the NVFP4 format with a per-tensor scale, 224 bytes: a quantised matrix takes three slots
// (packed e2m1 codes [rows][K/2], E4M3 block scales row-major [rows][K/16], device pointer to the fp32 tensor scale);
// norms, conv, beta / alpha projections, A_log, dt_bias stay bf16 (one slot each).  DeltaNet layers use 26 slots,
// attention layers 25.  No counterpart in the reference (its NVFP4 table has no tensor scale).
struct LayerWeightsNVFP4TS {
    int layer_type;
    int pad[3];
    const void* ptrs[26];
};
static_assert(sizeof(LayerWeightsNVFP4TS) == 224, "tensor-scale NVFP4 pointer table entry must be 224 bytes");

// pointer slots, DeltaNet layer (reference: megakernel/model.py:117-132)
enum { DN_IN_NORM = 0, DN_W_QKV, DN_W_Z, DN_W_B, DN_W_A, DN_CONV_W, DN_A_LOG, DN_DT_BIAS,
       DN_NORM_W, DN_W_OUT, DN_POST_NORM, DN_W_GATE, DN_W_UP, DN_W_DOWN };
// pointer slots, attention layer (reference: megakernel/model.py:99-111)
enum { FA_IN_NORM = 0, FA_W_Q, FA_W_K, FA_W_V, FA_Q_NORM, FA_K_NORM, FA_W_O, FA_POST_NORM,
       FA_W_GATE, FA_W_UP, FA_W_DOWN };

// status codes reported by the device through the status word
enum { ST_OK = 0, ST_GRID_TIMEOUT = 1, ST_MBAR_TIMEOUT = 2, ST_MISALIGNED = 3 };

// ---- PTX wrappers ------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait: returns false when the limit ran out (the caller records the status).
constexpr uint32_t MBAR_WAIT_TRIES = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t tries = MBAR_WAIT_TRIES) {
    for (uint32_t n = 0; n < tries; ++n)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// global -> shared bulk async copy; bytes % 16 == 0, both addresses 16-byte aligned
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Programmatic dependent launch: a kernel launched with the stream-serialisation attribute may start while
// its predecessor drains.  pdl_enter() is the first statement of every prefill kernel: it lets the next kernel
// in the stream be scheduled early and then waits until the predecessor has completed and its writes are
// visible, so no kernel touches its inputs before they exist.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// The two halves of pdl_enter(), for kernels that have something useful to do before their inputs exist: between
// them only memory that no kernel of the stream writes (weights) or that the predecessor does not write may be
// touched.  l2_prefetch asks for `bytes` (multiple of 16, 16-byte aligned start) to be brought into L2.
__device__ __forceinline__ void pdl_launch_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void l2_prefetch(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- math helpers ------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }

// 8 bf16 weights (one 16-byte word) times 8 f32 activations
__device__ __forceinline__ float dot8(const uint4& w, const float* x, float acc) {
    acc = fmaf(bf_lo(w.x), x[0], acc); acc = fmaf(bf_hi(w.x), x[1], acc);
    acc = fmaf(bf_lo(w.y), x[2], acc); acc = fmaf(bf_hi(w.y), x[3], acc);
    acc = fmaf(bf_lo(w.z), x[4], acc); acc = fmaf(bf_hi(w.z), x[5], acc);
    acc = fmaf(bf_lo(w.w), x[6], acc); acc = fmaf(bf_hi(w.w), x[7], acc);
    return acc;
}
__device__ __forceinline__ float dot4(const uint2& w, const float* x, float acc) {
    acc = fmaf(bf_lo(w.x), x[0], acc); acc = fmaf(bf_hi(w.x), x[1], acc);
    acc = fmaf(bf_lo(w.y), x[2], acc); acc = fmaf(bf_hi(w.y), x[3], acc);
    return acc;
}

// ---- NVFP4 decoding without conversion instructions -------------------------------------------------------

// Eight e2m1 codes (one 32-bit word, lowest nibble first) -> four f16x2 registers (codes 0|1, 2|3, 4|5, 6|7) with
// byte permutes instead of conversion instructions: the cvt from e2m1 issues at a small fraction of the integer
// rate on this GPU (a 64-row chunk spent ~2.3 us in conversions), and a row product converts every weight once.
// An e2m1 magnitude is one of 8 values whose f16 encodings differ in the high byte only (00 38 3C 3E 40 42 44 46):
// prmt looks four of them up at once, the packed nibbles being the selector; a second prmt spreads the bytes into
// f16 positions; the sign comes from prmt's sign-replicate mode (the msb of byte j of w is the sign of code 2j+1,
// that of w << 4 the sign of code 2j).
__device__ __forceinline__ void e2m1x8_to_f16x2x4(uint32_t w, uint32_t (&r)[4]) {
    const uint32_t mag = w & 0x77777777u;
    const uint32_t h_lo = __byte_perm(0x3E3C3800u, 0x46444240u, mag);          // f16 high bytes of codes 0..3
    const uint32_t h_hi = __byte_perm(0x3E3C3800u, 0x46444240u, mag >> 16);    // codes 4..7
    const uint32_t we = w << 4;
    r[0] = __byte_perm(h_lo, 0u, 0x1404u) | (__byte_perm(we, w, 0xC080u) & 0x80008000u);
    r[1] = __byte_perm(h_lo, 0u, 0x3424u) | (__byte_perm(we, w, 0xD090u) & 0x80008000u);
    r[2] = __byte_perm(h_hi, 0u, 0x1404u) | (__byte_perm(we, w, 0xE0A0u) & 0x80008000u);
    r[3] = __byte_perm(h_hi, 0u, 0x3424u) | (__byte_perm(we, w, 0xF0B0u) & 0x80008000u);
}
// E4M3 block scale (non-negative) as f16x2, without a conversion instruction: the f16 with bit pattern byte << 7
// is exactly scale * 2^-8, for normal and subnormal E4M3 alike (same exponent / mantissa split, exponent bias 15
// instead of 7; E4M3 subnormals land on f16 subnormals).  The factor 2^8 is applied with the tensor scale.
// A code times such a scale has at most 6 significant bits and lies in [2^-18, 10.5]: exact in f16.
constexpr float TS_SCALE_FOLD = 256.0f;
__device__ __forceinline__ __half2 e4m3_to_h2_div256(uint32_t byte) {
    const uint32_t v = (byte & 0xffu) * 0x00800080u;
    return *reinterpret_cast<const __half2*>(&v);
}
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, __half2 s) {
    const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), s);
    return *reinterpret_cast<const uint32_t*>(&r);
}

}  // namespace mk
