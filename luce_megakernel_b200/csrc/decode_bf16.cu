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
#include "mk_common.cuh"
#include "mk_decode.h"

namespace mk {

namespace {

constexpr int NCW = 16;                    // consumer warps
constexpr int NCT = NCW * 32;              // consumer threads
constexpr int NTHREADS = NCT + 32;         // + producer warp
constexpr int NSTAGE = 6;
constexpr int STAGE_BYTES = 32768;
constexpr int XK = 224;                    // largest K-slice of a warp (elements)
constexpr int XSW = 3 * XK / 2;            // 32-bit words of staging per warp: three bf16 planes of XK elements

constexpr int OFF_RING = 0;
constexpr int OFF_SCRATCH = NSTAGE * STAGE_BYTES;          // activation staging (16 x 224 floats) / attention merge
constexpr int SCRATCH_BYTES = 21504;           // 16 x 1344 B of staging; attention uses 16640 B of merge slots + 4096 B of q
constexpr int OFF_PART = OFF_SCRATCH + SCRATCH_BYTES;      // 2 x (4 chunks x 16 warps x 16 rows) partial sums
constexpr int PART_HALF = 4 * NCW * 16;                    // floats; phases alternate between the halves
constexpr int PART_BYTES = 2 * PART_HALF * 4;
constexpr int OFF_RED = OFF_PART + PART_BYTES;             // 32 floats
constexpr int OFF_MISC = OFF_RED + 128;                    // 8 ints
constexpr int OFF_BAR = OFF_MISC + 32;                     // full[NSTAGE], empty[NSTAGE]
constexpr int OFF_LAYERS = OFF_BAR + 2 * NSTAGE * 8;       // copy of the layer pointer table
constexpr int SMEM_BYTES = OFF_LAYERS + MAX_LAYERS * (int)sizeof(LayerWeights);
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

enum { MISC_ABORT = 0, MISC_LAST = 1 };

// pause between failed polls of a flagged word: keeps the waiting threads of 148 CTAs from
// saturating the L2 slices that hold the words (and from delaying the stores they wait for)
#ifndef MK_POLL_SLEEP_NS
#define MK_POLL_SLEEP_NS 0
#endif
#define MK_POLL_BACKOFF() do { if (MK_POLL_SLEEP_NS > 0) __nanosleep(MK_POLL_SLEEP_NS); } while (0)

enum PhaseType { T_DN_IN = 0, T_DN_REC, T_DN_OUT, T_FA_IN, T_FA_ATT, T_FA_OUT, T_GATEUP, T_DOWN, T_LM };

struct Geo {
    int r0, r1;       // rows (or outputs for gate/up, first unit for the recurrence)
    int nchunks;
};

__device__ __forceinline__ void split_rows(int n, int G, int c, int& a, int& b) {
    // n <= 248320 rows (or whatever the vocabulary is) times at most 256 CTAs fits 32 bits
    a = (int)(((unsigned)n * (unsigned)c) / (unsigned)G);
    b = (int)(((unsigned)n * (unsigned)(c + 1)) / (unsigned)G);
}

__device__ __forceinline__ Geo phase_geo(int type, int cta, int G, int vocab) {
    Geo g;
    g.r0 = g.r1 = 0;
    g.nchunks = 0;
    switch (type) {
        case T_DN_IN:  split_rows(DN_IN_ROWS, G, cta, g.r0, g.r1);  g.nchunks = (g.r1 - g.r0 + 15) >> 4; break;
        case T_FA_IN:  split_rows(FA_QKV_ROWS, G, cta, g.r0, g.r1); g.nchunks = (g.r1 - g.r0 + 15) >> 4; break;
        case T_DN_OUT:
        case T_FA_OUT: split_rows(HIDDEN, G, cta, g.r0, g.r1);      g.nchunks = (g.r1 - g.r0 + 7) >> 3; break;
        case T_GATEUP: split_rows(INTER, G, cta, g.r0, g.r1);       g.nchunks = (g.r1 - g.r0 + 7) >> 3; break;
        case T_DOWN:   split_rows(HIDDEN, G, cta, g.r0, g.r1);      g.nchunks = (g.r1 - g.r0 + 3) >> 2; break;
        case T_LM:     split_rows(vocab, G, cta, g.r0, g.r1);       g.nchunks = (g.r1 - g.r0 + 15) >> 4; break;
        case T_DN_REC: g.r0 = cta; g.nchunks = (cta < 128) ? (128 - cta + G - 1) / G : 0; break;
        default: break;
    }
    return g;
}

// Source of ring slot `slot` of chunk q; returns bytes (0 = slot unused) and the slot's ring offset.
__device__ __forceinline__ uint32_t chunk_slot_src(int type, const LayerWeights& lw, const DecodeParams& P,
                                                   const Geo& g, int q, int slot, int G, int dn_idx,
                                                   const char*& src, uint32_t& dst_off) {
    switch (type) {
        case T_DN_IN: {
            int r = g.r0 + q * 16 + slot;
            if (slot >= 16 || r >= g.r1) return 0;
            const char* base; int rr;
            if (r < DN_CONV_CH) { base = (const char*)lw.ptrs[DN_W_QKV]; rr = r; }
            else if (r < DN_CONV_CH + DN_V) { base = (const char*)lw.ptrs[DN_W_Z]; rr = r - DN_CONV_CH; }
            else if (r < DN_CONV_CH + DN_V + DN_HEADS) { base = (const char*)lw.ptrs[DN_W_B]; rr = r - DN_CONV_CH - DN_V; }
            else { base = (const char*)lw.ptrs[DN_W_A]; rr = r - DN_CONV_CH - DN_V - DN_HEADS; }
            src = base + (size_t)rr * (HIDDEN * 2); dst_off = slot * (HIDDEN * 2);
            return HIDDEN * 2;
        }
        case T_FA_IN: {
            int r = g.r0 + q * 16 + slot;
            if (slot >= 16 || r >= g.r1) return 0;
            const char* base; int rr;
            if (r < FA_QPROJ) { base = (const char*)lw.ptrs[FA_W_Q]; rr = r; }
            else if (r < FA_QPROJ + FA_KV_SIZE) { base = (const char*)lw.ptrs[FA_W_K]; rr = r - FA_QPROJ; }
            else { base = (const char*)lw.ptrs[FA_W_V]; rr = r - FA_QPROJ - FA_KV_SIZE; }
            src = base + (size_t)rr * (HIDDEN * 2); dst_off = slot * (HIDDEN * 2);
            return HIDDEN * 2;
        }
        case T_DN_OUT:
        case T_FA_OUT: {
            int r = g.r0 + q * 8 + slot;
            if (slot >= 8 || r >= g.r1) return 0;
            const char* base = (const char*)lw.ptrs[type == T_DN_OUT ? (int)DN_W_OUT : (int)FA_W_O];
            src = base + (size_t)r * (2048 * 2); dst_off = slot * (2048 * 2);
            return 2048 * 2;
        }
        case T_GATEUP: {
            int o = g.r0 + q * 8 + (slot & 7);
            if (slot >= 16 || o >= g.r1) return 0;
            const bool dn = (lw.layer_type == 0);
            const char* base = (const char*)(slot < 8 ? lw.ptrs[dn ? (int)DN_W_GATE : (int)FA_W_GATE]
                                                      : lw.ptrs[dn ? (int)DN_W_UP : (int)FA_W_UP]);
            src = base + (size_t)o * (HIDDEN * 2); dst_off = slot * (HIDDEN * 2);
            return HIDDEN * 2;
        }
        case T_DOWN: {
            int r = g.r0 + q * 4 + slot;
            if (slot >= 4 || r >= g.r1) return 0;
            const char* base = (const char*)lw.ptrs[lw.layer_type == 0 ? (int)DN_W_DOWN : (int)FA_W_DOWN];
            src = base + (size_t)r * (INTER * 2); dst_off = slot * (INTER * 2);
            return INTER * 2;
        }
        case T_LM: {
            int r = g.r0 + q * 16 + slot;
            if (slot >= 16 || r >= g.r1) return 0;
            src = (const char*)P.lm_head + (size_t)r * (HIDDEN * 2); dst_off = slot * (HIDDEN * 2);
            return HIDDEN * 2;
        }
        case T_DN_REC: {
            if (slot != 0) return 0;
            int u = g.r0 + q * G;                 // unit = (head, 16-row value slice)
            int h = u >> 3, s = u & 7;
            src = (const char*)(P.dn_states + ((size_t)(dn_idx * DN_HEADS + h) * DN_VAL + s * 16) * DN_KEY);
            dst_off = 0;
            return 16 * DN_KEY * 4;
        }
        default: return 0;
    }
}

}  // namespace

namespace plain {
namespace {
#define MK_TRACE 0
#include "decode_body.cuh"
#undef MK_TRACE
}  // namespace
}  // namespace plain

namespace traced {
namespace {
#define MK_TRACE 1
#include "decode_body.cuh"
#undef MK_TRACE
}  // namespace
}  // namespace traced

size_t decode_smem_bytes() { return SMEM_BYTES; }

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

// RoPE angles of one position: inv_freq_i = theta^(-2i/64) in double, angle in f32 like the
// reference (megakernel/kernel.cu:468-470), sine and cosine evaluated in double.
void fill_rope(DecodeParams& p) {
    for (int i = 0; i < FA_ROT / 2; ++i) {
        const float inv_freq = (float)(1.0 / pow(ROPE_THETA, (2.0 * i) / FA_ROT));
        const float ang = (float)p.position * inv_freq;
        p.rope_cos[i] = (float)cos((double)ang);
        p.rope_sin[i] = (float)sin((double)ang);
    }
}

cudaError_t launch_decode_kernel(const DecodeParams& p, int grid, cudaStream_t stream) {
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !attr_done[dev]) {
        e = cudaFuncSetAttribute(plain::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(traced::decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_done[dev] = true;
    }
    if (grid < MIN_GRID || grid > MAX_GRID) return cudaErrorInvalidConfiguration;
    void* args[] = {(void*)&p};
    const void* fn = p.trace ? (const void*)traced::decode_megakernel_bf16 : (const void*)plain::decode_megakernel_bf16;
    return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(NTHREADS), args, SMEM_BYTES, stream);
}

}  // namespace mk
