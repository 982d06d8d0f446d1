// Persistent single-dispatch bf16 decode step for the Qwen3.5-0.8B hybrid, written for sm_100a.
//
// One CTA per SM (cooperative launch, so co-residency is guaranteed).  Each CTA has one
// producer warp and 16 consumer warps.
//
//  * The producer warp walks the whole token's weight schedule for this CTA -- every layer,
//    every phase, the rows this CTA owns -- and streams it with bulk async copies
//    (cp.async.bulk + mbarrier complete_tx) into a 6 x 32 KB shared-memory ring.  Weights do
//    not depend on activations, so the producer never waits on the grid barrier: while the
//    consumers sit at a barrier the next phases' weights keep landing in the ring.
//  * The consumer warps wait at the grid barrier for the previous phase's activation vector,
//    stage it into shared memory / registers (RMSNorm, gated norm, attention merge are fused
//    into the staging), run warp-per-row dot products out of the ring, and write the phase
//    result with its epilogue (conv1d+SiLU, gates, residual add, SwiGLU, argmax) fused.
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

constexpr int OFF_RING = 0;
constexpr int OFF_SCRATCH = NSTAGE * STAGE_BYTES;          // 24 KB: activation vector / attention merge
constexpr int SCRATCH_BYTES = 24576;
constexpr int OFF_RES = OFF_SCRATCH + SCRATCH_BYTES;       // 256 floats of per-row results
constexpr int OFF_RED = OFF_RES + 1024;                    // 32 floats
constexpr int OFF_MISC = OFF_RED + 128;                    // 8 ints
constexpr int OFF_BAR = OFF_MISC + 32;                     // full[NSTAGE], empty[NSTAGE]
constexpr int OFF_LAYERS = OFF_BAR + 2 * NSTAGE * 8;        // copy of the layer pointer table
constexpr int SMEM_BYTES = OFF_LAYERS + MAX_LAYERS * (int)sizeof(LayerWeights);
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

enum { MISC_ABORT = 0, MISC_LAST = 1 };

enum PhaseType { T_DN_IN = 0, T_DN_REC, T_DN_OUT, T_FA_IN, T_FA_ATT, T_FA_OUT, T_GATEUP, T_DOWN, T_LM };

__constant__ float c_inv_freq[FA_ROT / 2];

struct Geo {
    int r0, r1;       // rows (or outputs for gate/up, first unit for the recurrence)
    int nchunks;
};

__device__ __forceinline__ void split_rows(int n, int G, int c, int& a, int& b) {
    a = (int)(((long long)n * c) / G);
    b = (int)(((long long)n * (c + 1)) / G);
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

struct Ctx {
    char* smem;
    float* xs;            // scratch as floats
    float* res;
    float* red;
    volatile int* misc;
    uint32_t full0, empty0, ring0;
    int tid, warp, lane, cta, G;
    uint32_t it;          // ring chunk counter (producer and consumers advance it identically)
    uint32_t epoch;       // grid barriers passed
    uint32_t trace_slot;
};

__device__ __noinline__ void fail(const DecodeParams& P, Ctx& c, uint32_t code) {
    c.misc[MISC_ABORT] = 1;
    atomicExch(&P.ws->abort_flag, 1u);
    if (P.host_status) { *((volatile uint32_t*)P.host_status) = code; __threadfence_system(); }
}

// Optional timeline: thread 0 of each CTA appends the global timer at fixed points of every phase.
__device__ __forceinline__ void trace_point(const DecodeParams& P, Ctx& c) {
    if (P.trace) {
        if (c.tid == 0 && c.trace_slot < (uint32_t)P.trace_slots) P.trace[(size_t)c.cta * P.trace_slots + c.trace_slot] = globaltimer_ns();
        c.trace_slot++;
    }
}

__device__ __forceinline__ void wait_full(const DecodeParams& P, Ctx& c, uint32_t stage, uint32_t parity) {
    if (c.misc[MISC_ABORT]) return;
    if (!mbar_wait(c.full0 + stage * 8, parity)) fail(P, c, ST_MBAR_TIMEOUT);
#ifdef MK_TRACE_CHUNKS
    if (P.trace && c.tid == 0 && c.it < 256 && P.trace_slots >= 1024) P.trace[(size_t)c.cta * P.trace_slots + 768 + c.it] = globaltimer_ns();
#endif
}

__device__ __forceinline__ void release_stage(Ctx& c, uint32_t stage) {
    __syncwarp();
    if (c.lane == 0 && !c.misc[MISC_ABORT]) mbar_arrive(c.empty0 + stage * 8);
}

// Grid-wide barrier over the consumer threads of all CTAs.  Bounded: gives up after 2 s.
__device__ __forceinline__ void grid_sync(const DecodeParams& P, Ctx& c) {
    trace_point(P, c);
    named_bar_sync(1, NCT);
    c.epoch++;
    if (c.tid == 0) {
        red_release_gpu_add(&P.ws->bar, 1u);
        const uint32_t target = c.epoch * (uint32_t)c.G;
        if (!c.misc[MISC_ABORT]) {
            uint64_t t0 = 0;
            uint32_t n = 0;
            while (ld_acquire_gpu(&P.ws->bar) < target) {
                if ((++n & 1023u) == 0) {
                    uint64_t now = globaltimer_ns();
                    if (t0 == 0) t0 = now;
                    if (now - t0 > 2000000000ull || ld_acquire_gpu(&P.ws->abort_flag) != 0u) {
                        fail(P, c, ST_GRID_TIMEOUT);
                        break;
                    }
                }
            }
        }
    }
    named_bar_sync(1, NCT);
    trace_point(P, c);
}

// ---- producer ---------------------------------------------------------------------------

__device__ void producer_phase(const DecodeParams& P, Ctx& c, int type, const LayerWeights& lw, int dn_idx,
                               uint64_t pol_stream, uint64_t pol_keep) {
    const Geo g = phase_geo(type, c.cta, c.G, P.vocab);
    for (int q = 0; q < g.nchunks; ++q, ++c.it) {
        if (c.misc[MISC_ABORT]) continue;
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        if (c.lane == 0 && !mbar_wait(c.empty0 + stage * 8, parity ^ 1u)) fail(P, c, ST_MBAR_TIMEOUT);
        __syncwarp();
        const char* src = nullptr;
        uint32_t dst_off = 0;
        uint32_t bytes = chunk_slot_src(type, lw, P, g, q, c.lane, c.G, dn_idx, src, dst_off);
        if (bytes && (((uintptr_t)src) & 15u)) { fail(P, c, ST_MISALIGNED); bytes = 0; }
        const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
        if (c.misc[MISC_ABORT]) continue;
        // Consecutive slots whose sources and destinations are contiguous (consecutive rows of one
        // matrix) travel as ONE bulk copy: the copy issue rate, not its size, limits a CTA.
        const unsigned long long prev_src = __shfl_up_sync(0xffffffffu, (unsigned long long)(uintptr_t)src, 1);
        const uint32_t prev_bytes = __shfl_up_sync(0xffffffffu, bytes, 1);
        const uint32_t prev_dst = __shfl_up_sync(0xffffffffu, dst_off, 1);
#ifdef MK_NO_MERGE
        const bool head = bytes != 0;
#else
        const bool head = bytes && (c.lane == 0 || prev_bytes == 0 ||
                                    prev_src + prev_bytes != (unsigned long long)(uintptr_t)src ||
                                    prev_dst + prev_bytes != dst_off);
#endif
        const uint32_t heads = __ballot_sync(0xffffffffu, head);
        const uint32_t valid = __ballot_sync(0xffffffffu, bytes != 0);
        const uint32_t above = (c.lane == 31) ? 0u : ~((2u << c.lane) - 1u);
        const uint32_t stop = (heads | ~valid) & above;
        const int end = stop ? (__ffs(stop) - 1) : 32;
        if (c.lane == 0) mbar_expect_tx(c.full0 + stage * 8, total);
#ifdef MK_TRACE_CHUNKS
        if (P.trace && c.lane == 0 && c.it < 256 && P.trace_slots >= 1024) P.trace[(size_t)c.cta * P.trace_slots + 512 + c.it] = globaltimer_ns();
#endif
        __syncwarp();
        if (head)
            bulk_g2s(c.ring0 + stage * STAGE_BYTES + dst_off, src, bytes * (uint32_t)(end - c.lane), c.full0 + stage * 8,
                     type == T_DN_REC ? pol_keep : pol_stream);
    }
}

// ---- activation staging -----------------------------------------------------------------

// xs[0..1024) = rms(src) * w1p, optionally rounded to bf16 (reference: megakernel/kernel.cu:189-231)
__device__ __forceinline__ void stage_rmsnorm(Ctx& c, const __nv_bfloat16* src, float w0, float w1, bool round_to_bf16,
                                              float* also_global) {
    const uint32_t raw = __ldcg(reinterpret_cast<const uint32_t*>(src) + c.tid);
    const float v0 = bf_lo(raw), v1 = bf_hi(raw);
    const float ss = warp_sum(v0 * v0 + v1 * v1);
    if (c.lane == 0) c.red[c.warp] = ss;
    named_bar_sync(1, NCT);
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < NCW; ++i) tot += c.red[i];
    const float rstd = rsqrtf(tot * (1.0f / HIDDEN) + RMS_EPS);
    float x0 = v0 * rstd * w0, x1 = v1 * rstd * w1;
    if (round_to_bf16) { x0 = round_bf16(x0); x1 = round_bf16(x1); }
    reinterpret_cast<float2*>(c.xs)[c.tid] = make_float2(x0, x1);
    if (also_global) reinterpret_cast<float2*>(also_global)[c.tid] = make_float2(x0, x1);
    named_bar_sync(1, NCT);
}

__device__ __forceinline__ void load_norm_w(const void* w, int tid, float& w0, float& w1) {
    const uint32_t raw = __ldg(reinterpret_cast<const uint32_t*>(w) + tid);
    w0 = 1.0f + bf_lo(raw);
    w1 = 1.0f + bf_hi(raw);
}

// ---- K = 1024 streaming matvec (one warp per ring slot) ------------------------------------

__device__ __forceinline__ void load_x1024(const Ctx& c, float* xr) {
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const float4 a = *reinterpret_cast<const float4*>(c.xs + it * 256 + c.lane * 8);
        const float4 b = *reinterpret_cast<const float4*>(c.xs + it * 256 + c.lane * 8 + 4);
        xr[it * 8 + 0] = a.x; xr[it * 8 + 1] = a.y; xr[it * 8 + 2] = a.z; xr[it * 8 + 3] = a.w;
        xr[it * 8 + 4] = b.x; xr[it * 8 + 5] = b.y; xr[it * 8 + 6] = b.z; xr[it * 8 + 7] = b.w;
    }
}

__device__ __forceinline__ float dot_row1024(const char* row, int lane, const float* xr) {
    const uint4* wp = reinterpret_cast<const uint4*>(row) + lane;
    const uint4 w0 = wp[0], w1 = wp[32], w2 = wp[64], w3 = wp[96];
    float a0 = dot8(w0, xr, 0.f), a1 = dot8(w1, xr + 8, 0.f);
    a0 = dot8(w2, xr + 16, a0); a1 = dot8(w3, xr + 24, a1);
    return a0 + a1;
}

// Runs the chunks of a K=1024 phase; results land in res[q*16 + slot].
__device__ __forceinline__ void matvec1024(const DecodeParams& P, Ctx& c, const Geo& g, int nvalid_total, bool gateup) {
    float xr[32];
    load_x1024(c, xr);
    for (int q = 0; q < g.nchunks; ++q, ++c.it) {
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        bool valid;
        if (gateup) valid = (q * 8 + (c.warp & 7)) < nvalid_total;
        else valid = (q * 16 + c.warp) < nvalid_total;
#ifdef MK_TRACE_CYCLES
        long long ta = clock64();
#endif
        wait_full(P, c, stage, parity);
#ifdef MK_TRACE_CYCLES
        long long tb = clock64();
#endif
        float acc = 0.f;
        if (valid) acc = dot_row1024(c.smem + OFF_RING + stage * STAGE_BYTES + c.warp * 2048, c.lane, xr);
#ifdef MK_TRACE_CYCLES
        long long tc = clock64();
#endif
        acc = warp_sum(acc);
        if (c.lane == 0 && valid) c.res[q * 16 + c.warp] = acc;
#ifdef MK_TRACE_CYCLES
        long long td = clock64();
#endif
        release_stage(c, stage);
#ifdef MK_TRACE_CYCLES
        long long te = clock64();
        if (P.trace && c.tid == 0 && c.it < 60 && P.trace_slots >= 1024) {
            unsigned long long* d = P.trace + (size_t)c.cta * P.trace_slots + 512 + c.it * 4;
            d[0] = tb - ta; d[1] = tc - tb; d[2] = td - tc; d[3] = te - td;
        }
#endif
    }
}

// ---- phases -----------------------------------------------------------------------------

__device__ void phase_dn_in(const DecodeParams& P, Ctx& c, const LayerWeights& lw, int dn_idx, const __nv_bfloat16* h_in,
                            bool first) {
    const Geo g = phase_geo(T_DN_IN, c.cta, c.G, P.vocab);
    const int nloc = g.r1 - g.r0;
    float w0, w1;
    load_norm_w(lw.ptrs[DN_IN_NORM], c.tid, w0, w1);
    // epilogue inputs that do not depend on this token: conv state and taps of the row this thread finishes
    const int r = g.r0 + c.tid;
    float4 cs = make_float4(0, 0, 0, 0);
    uint2 cw = make_uint2(0, 0);
    float a_log = 0.f, dt_b = 0.f;
    float* conv_row = nullptr;
    if (c.tid < nloc) {
        if (r < DN_CONV_CH) {
            conv_row = P.conv_bufs + ((size_t)dn_idx * DN_CONV_CH + r) * DN_CONV_K;
            cs = __ldcg(reinterpret_cast<const float4*>(conv_row));
            cw = __ldg(reinterpret_cast<const uint2*>(lw.ptrs[DN_CONV_W]) + r);
        } else if (r >= DN_CONV_CH + DN_V + DN_HEADS) {
            const int h = r - (DN_CONV_CH + DN_V + DN_HEADS);
            a_log = bf2f(reinterpret_cast<const __nv_bfloat16*>(lw.ptrs[DN_A_LOG])[h]);
            dt_b = bf2f(reinterpret_cast<const __nv_bfloat16*>(lw.ptrs[DN_DT_BIAS])[h]);
        }
    }
    if (!first) grid_sync(P, c);   // the first phase of a launch depends on nothing from this launch
    else { trace_point(P, c); trace_point(P, c); }
    stage_rmsnorm(c, h_in, w0, w1, true, nullptr);
    trace_point(P, c);
    matvec1024(P, c, g, nloc, false);
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nloc) {
        const float val = c.res[c.tid];
        if (r < DN_CONV_CH) {
            // shift the 4-tap window, append, dot with the taps, SiLU (reference: megakernel/kernel.cu:640-646)
            const float4 ns = make_float4(cs.y, cs.z, cs.w, val);
            *reinterpret_cast<float4*>(conv_row) = ns;
            const float co = ns.x * bf_lo(cw.x) + ns.y * bf_hi(cw.x) + ns.z * bf_lo(cw.y) + ns.w * bf_hi(cw.y);
            P.qkv[r] = silu_f(co);
        } else if (r < DN_CONV_CH + DN_V) {
            P.z[r - DN_CONV_CH] = val;
        } else if (r < DN_CONV_CH + DN_V + DN_HEADS) {
            P.beta[r - DN_CONV_CH - DN_V] = 1.0f / (1.0f + expf(-val));
        } else {
            // decay = exp(-exp(A_log) * softplus(a + dt_bias)) (reference: megakernel/kernel.cu:653-657)
            const float x = val + dt_b;
            const float sp = (x > 20.0f) ? x : log1pf(expf(x));
            P.alpha[r - DN_CONV_CH - DN_V - DN_HEADS] = expf(-expf(a_log) * sp);
        }
    }
}

// Gated delta rule for one token; unit = (head, 16 value rows), one warp per value row.
// State row j is contiguous over the key index (reference: megakernel/kernel.cu:686-713).
__device__ void phase_dn_rec(const DecodeParams& P, Ctx& c, int dn_idx) {
    const Geo g = phase_geo(T_DN_REC, c.cta, c.G, P.vocab);
    grid_sync(P, c);
    trace_point(P, c);
    for (int qi = 0; qi < g.nchunks; ++qi, ++c.it) {
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        const int u = g.r0 + qi * c.G;
        const int h = u >> 3, j = (u & 7) * 16 + c.warp;
        const float4 q4 = __ldcg(reinterpret_cast<const float4*>(P.qkv + h * DN_KEY) + c.lane);
        const float4 k4 = __ldcg(reinterpret_cast<const float4*>(P.qkv + DN_QK + h * DN_KEY) + c.lane);
        const float vj = __ldcg(P.qkv + 2 * DN_QK + h * DN_VAL + j);
        const float beta = __ldcg(P.beta + h), decay = __ldcg(P.alpha + h);
        float sq = q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w;
        float sk = k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w;
        float kq = q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w;
        sq = warp_sum(sq); sk = warp_sum(sk); kq = warp_sum(kq);
        const float qn = rsqrtf(sq + 1e-6f) * 0.08838834764831845f;   // 1/sqrt(128)
        const float kn = rsqrtf(sk + 1e-6f);
        kq *= qn * kn;
        wait_full(P, c, stage, parity);
        const float4 s4 = *reinterpret_cast<const float4*>(c.smem + OFF_RING + stage * STAGE_BYTES +
                                                           (c.warp * DN_KEY + c.lane * 4) * 4);
        float stk = (s4.x * k4.x + s4.y * k4.y + s4.z * k4.z + s4.w * k4.w) * kn;
        float sqv = (s4.x * q4.x + s4.y * q4.y + s4.z * q4.z + s4.w * q4.w) * qn;
        stk = warp_sum(stk); sqv = warp_sum(sqv);
        const float err = (vj - decay * stk) * beta;
        const float ek = err * kn;
        float4 sn;
        sn.x = s4.x * decay + k4.x * ek; sn.y = s4.y * decay + k4.y * ek;
        sn.z = s4.z * decay + k4.z * ek; sn.w = s4.w * decay + k4.w * ek;
        float* srow = P.dn_states + ((size_t)(dn_idx * DN_HEADS + h) * DN_VAL + j) * DN_KEY;
        reinterpret_cast<float4*>(srow)[c.lane] = sn;
        if (c.lane == 0) P.attn_out[h * DN_VAL + j] = decay * sqv + err * kq;
        release_stage(c, stage);
    }
    trace_point(P, c);
}

// K = 2048 matvec: 8 rows per chunk, two warps per row; adds the residual and writes bf16 hidden.
__device__ __forceinline__ void matvec2048_residual(const DecodeParams& P, Ctx& c, const Geo& g, const __nv_bfloat16* resid) {
    const int nloc = g.r1 - g.r0;
    float rs = 0.f;
    if (c.tid < nloc) rs = bf2f(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(resid) + g.r0 + c.tid)));
    const int slot = c.warp >> 1, part = c.warp & 1;
    float xr[32];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const float4 a = *reinterpret_cast<const float4*>(c.xs + part * 1024 + it * 256 + c.lane * 8);
        const float4 b = *reinterpret_cast<const float4*>(c.xs + part * 1024 + it * 256 + c.lane * 8 + 4);
        xr[it * 8 + 0] = a.x; xr[it * 8 + 1] = a.y; xr[it * 8 + 2] = a.z; xr[it * 8 + 3] = a.w;
        xr[it * 8 + 4] = b.x; xr[it * 8 + 5] = b.y; xr[it * 8 + 6] = b.z; xr[it * 8 + 7] = b.w;
    }
    for (int q = 0; q < g.nchunks; ++q, ++c.it) {
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        const bool valid = (q * 8 + slot) < nloc;
        wait_full(P, c, stage, parity);
        float acc = 0.f;
        if (valid) acc = dot_row1024(c.smem + OFF_RING + stage * STAGE_BYTES + slot * 4096 + part * 2048, c.lane, xr);
        acc = warp_sum(acc);
        if (c.lane == 0 && valid) c.res[(q * 8 + slot) * 2 + part] = acc;
        release_stage(c, stage);
    }
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nloc) {
        const float y = c.res[c.tid * 2] + c.res[c.tid * 2 + 1] + rs;
        reinterpret_cast<__nv_bfloat16*>(P.hidden)[g.r0 + c.tid] = __float2bfloat16_rn(y);
    }
}

// out-proj of a DeltaNet layer; staging fuses the gated RMSNorm (plain weight) * SiLU(z)
// (reference: megakernel/kernel.cu:715-741)
__device__ void phase_dn_out(const DecodeParams& P, Ctx& c, const LayerWeights& lw, const __nv_bfloat16* resid) {
    const Geo g = phase_geo(T_DN_OUT, c.cta, c.G, P.vocab);
    const uint2 nwr = __ldg(reinterpret_cast<const uint2*>(lw.ptrs[DN_NORM_W]) + c.lane);
    grid_sync(P, c);
    {
        const int h = c.warp;   // 16 warps = 16 heads
        const float4 o4 = __ldcg(reinterpret_cast<const float4*>(P.attn_out + h * DN_VAL) + c.lane);
        const float4 z4 = __ldcg(reinterpret_cast<const float4*>(P.z + h * DN_VAL) + c.lane);
        const float ss = warp_sum(o4.x * o4.x + o4.y * o4.y + o4.z * o4.z + o4.w * o4.w);
        const float rstd = rsqrtf(ss * (1.0f / DN_VAL) + RMS_EPS);
        float4 x;
        x.x = o4.x * rstd * bf_lo(nwr.x) * silu_f(z4.x);
        x.y = o4.y * rstd * bf_hi(nwr.x) * silu_f(z4.y);
        x.z = o4.z * rstd * bf_lo(nwr.y) * silu_f(z4.z);
        x.w = o4.w * rstd * bf_hi(nwr.y) * silu_f(z4.w);
        reinterpret_cast<float4*>(c.xs + h * DN_VAL)[c.lane] = x;
    }
    named_bar_sync(1, NCT);
    trace_point(P, c);
    matvec2048_residual(P, c, g, resid);
}

__device__ void phase_fa_in(const DecodeParams& P, Ctx& c, const LayerWeights& lw, const __nv_bfloat16* h_in, bool first) {
    const Geo g = phase_geo(T_FA_IN, c.cta, c.G, P.vocab);
    const int nloc = g.r1 - g.r0;
    float w0, w1;
    load_norm_w(lw.ptrs[FA_IN_NORM], c.tid, w0, w1);
    if (!first) grid_sync(P, c);
    else { trace_point(P, c); trace_point(P, c); }
    stage_rmsnorm(c, h_in, w0, w1, true, nullptr);
    trace_point(P, c);
    matvec1024(P, c, g, nloc, false);
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nloc) {
        const int r = g.r0 + c.tid;
        const float val = c.res[c.tid];
        if (r < FA_QPROJ) P.qkv[r] = val;          // per head [q(256) | gate(256)]
        else P.kv[r - FA_QPROJ] = val;             // k[512] then v[512]
    }
}

__device__ __forceinline__ int att_num_chunks(int L) {
    int nc = (L + ATT_CHUNK_POS - 1) / ATT_CHUNK_POS;
    return nc < 1 ? 1 : (nc > ATT_MAX_CHUNKS ? ATT_MAX_CHUNKS : nc);
}

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
    f[0] = bf_lo(u.x); f[1] = bf_hi(u.x); f[2] = bf_lo(u.y); f[3] = bf_hi(u.y);
    f[4] = bf_lo(u.z); f[5] = bf_hi(u.z); f[6] = bf_lo(u.w); f[7] = bf_hi(u.w);
}

// per-head RMSNorm(1+w) + partial RoPE on lane-strided dims d = lane + 32 e
// (dims i and i+32 of the rotary pair sit in the same lane).  reference: megakernel/kernel.cu:462-499
__device__ __forceinline__ void head_norm_rope(const float* src, const void* wn, int lane, int pos, float* n) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) { n[e] = __ldcg(src + lane + 32 * e); ss += n[e] * n[e]; }
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss * (1.0f / FA_HEAD_DIM) + RMS_EPS);
#pragma unroll
    for (int e = 0; e < 8; ++e)
        n[e] = n[e] * rstd * (1.0f + bf2f(reinterpret_cast<const __nv_bfloat16*>(wn)[lane + 32 * e]));
    float sn, cs;
    sincosf((float)pos * c_inv_freq[lane], &sn, &cs);
    const float a = n[0], b = n[1];
    n[0] = a * cs - b * sn;
    n[1] = b * cs + a * sn;
}

// Split-KV decode attention.  Unit = (KV head, position chunk); the 4 query heads of a KV head
// share every K/V load.  Each unit leaves (m, l, o[256]) per head in the workspace; the o-proj
// phase merges the chunks.  reference: megakernel/kernel.cu:506-560
__device__ void phase_fa_att(const DecodeParams& P, Ctx& c, const LayerWeights& lw, int fa_idx) {
    const int pos = P.position, L = pos + 1;
    const int NC = att_num_chunks(L);
    const int per = (L + NC - 1) / NC;
    float* slots = c.xs;                 // 4 slots x 4 heads x 260 floats
    float* qs = c.xs + 5120;             // 4 heads x 256 floats
    grid_sync(P, c);
    trace_point(P, c);
    for (int u = c.cta; u < FA_KV_HEADS * NC; u += c.G) {
        const int g = u / NC, ch = u % NC;
        const int p_lo = ch * per, p_hi = min(L, p_lo + per);
        const bool owner = (pos >= p_lo && pos < p_hi);
        __nv_bfloat16* Kb = reinterpret_cast<__nv_bfloat16*>(P.k_cache) + (size_t)(fa_idx * FA_KV_HEADS + g) * P.max_seq_len * FA_HEAD_DIM;
        __nv_bfloat16* Vb = reinterpret_cast<__nv_bfloat16*>(P.v_cache) + (size_t)(fa_idx * FA_KV_HEADS + g) * P.max_seq_len * FA_HEAD_DIM;
        if (c.warp < 4) {
            float n[8];
            head_norm_rope(P.qkv + (g * FA_GQA + c.warp) * 2 * FA_HEAD_DIM, lw.ptrs[FA_Q_NORM], c.lane, pos, n);
#pragma unroll
            for (int e = 0; e < 8; ++e) qs[c.warp * FA_HEAD_DIM + c.lane + 32 * e] = n[e];
        } else if (c.warp == 4 && owner) {
            float n[8];
            head_norm_rope(P.kv + g * FA_HEAD_DIM, lw.ptrs[FA_K_NORM], c.lane, pos, n);
#pragma unroll
            for (int e = 0; e < 8; ++e) Kb[(size_t)pos * FA_HEAD_DIM + c.lane + 32 * e] = __float2bfloat16_rn(n[e]);
        } else if (c.warp == 5 && owner) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
                Vb[(size_t)pos * FA_HEAD_DIM + c.lane + 32 * e] =
                    __float2bfloat16_rn(__ldcg(P.kv + FA_KV_SIZE + g * FA_HEAD_DIM + c.lane + 32 * e));
        }
        __threadfence_block();
        named_bar_sync(1, NCT);

        float qr[4][8], acc[4][8], m[4], l[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            m[h] = -1e30f; l[h] = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) { qr[h][e] = qs[h * FA_HEAD_DIM + c.lane * 8 + e] * 0.0625f; acc[h][e] = 0.f; }
        }
        int p = p_lo + c.warp;
        uint4 kk = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (p < p_hi) {
            kk = __ldcg(reinterpret_cast<const uint4*>(Kb + (size_t)p * FA_HEAD_DIM) + c.lane);
            vv = __ldcg(reinterpret_cast<const uint4*>(Vb + (size_t)p * FA_HEAD_DIM) + c.lane);
        }
        while (p < p_hi) {
            const int pn = p + NCW;
            uint4 kn = make_uint4(0, 0, 0, 0), vn = make_uint4(0, 0, 0, 0);
            if (pn < p_hi) {
                kn = __ldcg(reinterpret_cast<const uint4*>(Kb + (size_t)pn * FA_HEAD_DIM) + c.lane);
                vn = __ldcg(reinterpret_cast<const uint4*>(Vb + (size_t)pn * FA_HEAD_DIM) + c.lane);
            }
            float kf[8], vf[8], s[4];
            unpack8(kk, kf);
            unpack8(vv, vf);
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) d = fmaf(qr[h][e], kf[e], d);
                s[h] = d;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
                for (int h = 0; h < 4; ++h) s[h] += __shfl_xor_sync(0xffffffffu, s[h], o);
            }
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float mn = fmaxf(m[h], s[h]);
                const float corr = __expf(m[h] - mn), pe = __expf(s[h] - mn);
                l[h] = l[h] * corr + pe;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[h][e] = acc[h][e] * corr + pe * vf[e];
                m[h] = mn;
            }
            kk = kn; vv = vn; p = pn;
        }

        // merge the 16 warps' partial softmax states: three rounds into warps 0-3, then per head
        for (int r = 1; r <= 3; ++r) {
            if (c.warp >= 4 * r && c.warp < 4 * r + 4) {
                const int sl = c.warp - 4 * r;
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    float* d = slots + (sl * 4 + h) * ATT_PART_STRIDE;
                    if (c.lane == 0) { d[0] = m[h]; d[1] = l[h]; }
                    *reinterpret_cast<float4*>(d + 4 + c.lane * 8) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
                    *reinterpret_cast<float4*>(d + 8 + c.lane * 8) = make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
                }
            }
            named_bar_sync(1, NCT);
            if (c.warp < 4) {
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const float* d = slots + (c.warp * 4 + h) * ATT_PART_STRIDE;
                    const float m2 = d[0], l2 = d[1];
                    const float4 a = *reinterpret_cast<const float4*>(d + 4 + c.lane * 8);
                    const float4 b = *reinterpret_cast<const float4*>(d + 8 + c.lane * 8);
                    const float mn = fmaxf(m[h], m2);
                    const float f1 = __expf(m[h] - mn), f2 = __expf(m2 - mn);
                    l[h] = l[h] * f1 + l2 * f2;
                    acc[h][0] = acc[h][0] * f1 + a.x * f2; acc[h][1] = acc[h][1] * f1 + a.y * f2;
                    acc[h][2] = acc[h][2] * f1 + a.z * f2; acc[h][3] = acc[h][3] * f1 + a.w * f2;
                    acc[h][4] = acc[h][4] * f1 + b.x * f2; acc[h][5] = acc[h][5] * f1 + b.y * f2;
                    acc[h][6] = acc[h][6] * f1 + b.z * f2; acc[h][7] = acc[h][7] * f1 + b.w * f2;
                    m[h] = mn;
                }
            }
            named_bar_sync(1, NCT);
        }
        if (c.warp < 4) {
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                float* d = slots + (c.warp * 4 + h) * ATT_PART_STRIDE;
                if (c.lane == 0) { d[0] = m[h]; d[1] = l[h]; }
                *reinterpret_cast<float4*>(d + 4 + c.lane * 8) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
                *reinterpret_cast<float4*>(d + 8 + c.lane * 8) = make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
            }
        }
        named_bar_sync(1, NCT);
        if (c.warp < 4) {
            const int h = c.warp;
            float M = -1e30f;
#pragma unroll
            for (int s = 0; s < 4; ++s) M = fmaxf(M, slots[(s * 4 + h) * ATT_PART_STRIDE]);
            float lt = 0.f, o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const float* d = slots + (s * 4 + h) * ATT_PART_STRIDE;
                const float f = __expf(d[0] - M);
                lt += d[1] * f;
                const float4 a = *reinterpret_cast<const float4*>(d + 4 + c.lane * 8);
                const float4 b = *reinterpret_cast<const float4*>(d + 8 + c.lane * 8);
                o[0] += a.x * f; o[1] += a.y * f; o[2] += a.z * f; o[3] += a.w * f;
                o[4] += b.x * f; o[5] += b.y * f; o[6] += b.z * f; o[7] += b.w * f;
            }
            float* dst = P.ws->attn_part + ((size_t)(g * FA_GQA + h) * ATT_MAX_CHUNKS + ch) * ATT_PART_STRIDE;
            if (c.lane == 0) { dst[0] = M; dst[1] = lt; }
            *reinterpret_cast<float4*>(dst + 4 + c.lane * 8) = make_float4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<float4*>(dst + 8 + c.lane * 8) = make_float4(o[4], o[5], o[6], o[7]);
        }
        named_bar_sync(1, NCT);
    }
    trace_point(P, c);
}

// o-proj of an attention layer; staging merges the KV chunks and applies the sigmoid gate
// (reference: megakernel/kernel.cu:542-570)
__device__ void phase_fa_out(const DecodeParams& P, Ctx& c, const LayerWeights& lw, const __nv_bfloat16* resid) {
    const Geo g = phase_geo(T_FA_OUT, c.cta, c.G, P.vocab);
    const int NC = att_num_chunks(P.position + 1);
    grid_sync(P, c);
    {
        const int head = c.tid >> 6, d4 = (c.tid & 63) * 4;
        const float* part = P.ws->attn_part + (size_t)head * ATT_MAX_CHUNKS * ATT_PART_STRIDE;
        float mv[ATT_MAX_CHUNKS];
        float M = -1e30f;
#pragma unroll
        for (int ch = 0; ch < ATT_MAX_CHUNKS; ++ch) {
            mv[ch] = (ch < NC) ? __ldcg(part + ch * ATT_PART_STRIDE) : -1e30f;
            M = fmaxf(M, mv[ch]);
        }
        float den = 0.f;
        float4 o = make_float4(0, 0, 0, 0);
#pragma unroll
        for (int ch = 0; ch < ATT_MAX_CHUNKS; ++ch) {
            if (ch < NC) {
                const float f = __expf(mv[ch] - M);
                den += __ldcg(part + ch * ATT_PART_STRIDE + 1) * f;
                const float4 a = __ldcg(reinterpret_cast<const float4*>(part + ch * ATT_PART_STRIDE + 4 + d4));
                o.x += a.x * f; o.y += a.y * f; o.z += a.z * f; o.w += a.w * f;
            }
        }
        const float4 gt = __ldcg(reinterpret_cast<const float4*>(P.qkv + head * 2 * FA_HEAD_DIM + FA_HEAD_DIM + d4));
        const float inv = 1.0f / den;
        float4 x;
        x.x = o.x * inv * sigmoid_f(gt.x); x.y = o.y * inv * sigmoid_f(gt.y);
        x.z = o.z * inv * sigmoid_f(gt.z); x.w = o.w * inv * sigmoid_f(gt.w);
        *reinterpret_cast<float4*>(c.xs + head * FA_HEAD_DIM + d4) = x;
    }
    named_bar_sync(1, NCT);
    trace_point(P, c);
    matvec2048_residual(P, c, g, resid);
}

// post norm + SiLU(Wg x) * (Wu x)  (reference: megakernel/kernel.cu:313-347, 572-578)
__device__ void phase_gateup(const DecodeParams& P, Ctx& c, const LayerWeights& lw) {
    const Geo g = phase_geo(T_GATEUP, c.cta, c.G, P.vocab);
    const int nout = g.r1 - g.r0;
    float w0, w1;
    load_norm_w(lw.ptrs[lw.layer_type == 0 ? (int)DN_POST_NORM : (int)FA_POST_NORM], c.tid, w0, w1);
    grid_sync(P, c);
    stage_rmsnorm(c, reinterpret_cast<const __nv_bfloat16*>(P.hidden), w0, w1, true, nullptr);
    trace_point(P, c);
    matvec1024(P, c, g, nout, true);
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nout) {
        const float gv = c.res[(c.tid >> 3) * 16 + (c.tid & 7)];
        const float uv = c.res[(c.tid >> 3) * 16 + 8 + (c.tid & 7)];
        P.mlp_inter[g.r0 + c.tid] = silu_f(gv) * uv;
    }
}

// down projection + residual (reference: megakernel/kernel.cu:350-384)
__device__ void phase_down(const DecodeParams& P, Ctx& c) {
    const Geo g = phase_geo(T_DOWN, c.cta, c.G, P.vocab);
    const int nloc = g.r1 - g.r0;
    grid_sync(P, c);
    float rs = 0.f;
    if (c.tid < nloc)
        rs = bf2f(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(P.hidden) + g.r0 + c.tid)));
    for (int i = c.tid; i < INTER / 4; i += NCT)
        reinterpret_cast<float4*>(c.xs)[i] = __ldcg(reinterpret_cast<const float4*>(P.mlp_inter) + i);
    named_bar_sync(1, NCT);
    trace_point(P, c);
    const int slot = c.warp >> 2, part = c.warp & 3;
    float xr[28];
#pragma unroll
    for (int it = 0; it < 7; ++it) {
        const float4 a = *reinterpret_cast<const float4*>(c.xs + part * 896 + it * 128 + c.lane * 4);
        xr[it * 4 + 0] = a.x; xr[it * 4 + 1] = a.y; xr[it * 4 + 2] = a.z; xr[it * 4 + 3] = a.w;
    }
    for (int q = 0; q < g.nchunks; ++q, ++c.it) {
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        const bool valid = (q * 4 + slot) < nloc;
        wait_full(P, c, stage, parity);
        float acc = 0.f;
        if (valid) {
            const uint2* wp = reinterpret_cast<const uint2*>(c.smem + OFF_RING + stage * STAGE_BYTES + slot * (INTER * 2) + part * 1792) + c.lane;
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int it = 0; it < 7; ++it) {
                const uint2 w = wp[it * 32];
                if (it & 1) a1 = dot4(w, xr + it * 4, a1); else a0 = dot4(w, xr + it * 4, a0);
            }
            acc = a0 + a1;
        }
        acc = warp_sum(acc);
        if (c.lane == 0 && valid) c.res[(q * 4 + slot) * 4 + part] = acc;
        release_stage(c, stage);
    }
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nloc) {
        const float y = c.res[c.tid * 4] + c.res[c.tid * 4 + 1] + c.res[c.tid * 4 + 2] + c.res[c.tid * 4 + 3] + rs;
        reinterpret_cast<__nv_bfloat16*>(P.hidden)[g.r0 + c.tid] = __float2bfloat16_rn(y);
    }
}

// final norm (f32, not rounded) + LM head + argmax, lowest index winning exact ties
// (reference: megakernel/kernel.cu:763-826, 905-920)
__device__ void phase_lm(const DecodeParams& P, Ctx& c) {
    const Geo g = phase_geo(T_LM, c.cta, c.G, P.vocab);
    const int nloc = g.r1 - g.r0;
    float w0, w1;
    load_norm_w(P.final_norm, c.tid, w0, w1);
    grid_sync(P, c);
    stage_rmsnorm(c, reinterpret_cast<const __nv_bfloat16*>(P.hidden), w0, w1, false, c.cta == 0 ? P.normalized : nullptr);
    trace_point(P, c);
    float xr[32];
    load_x1024(c, xr);
    const bool penal = (P.rep_penalty > 1.0f) && (P.seen_mask != nullptr);
    float bestv = -INFINITY;
    int besti = 0x7fffffff;
    for (int q = 0; q < g.nchunks; ++q, ++c.it) {
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        const int row = g.r0 + q * 16 + c.warp;
        const bool valid = (q * 16 + c.warp) < nloc;
        float seen = 0.f;
        if (penal && valid) seen = __ldcg(P.seen_mask + row);
        wait_full(P, c, stage, parity);
        float acc = 0.f;
        if (valid) acc = dot_row1024(c.smem + OFF_RING + stage * STAGE_BYTES + c.warp * 2048, c.lane, xr);
        acc = warp_sum(acc);
        if (valid) {
            if (seen > 0.f) acc = (acc > 0.f) ? acc / P.rep_penalty : acc * P.rep_penalty;
            if (acc > bestv) { bestv = acc; besti = row; }
        }
        release_stage(c, stage);
    }
    trace_point(P, c);
    int* resi = reinterpret_cast<int*>(c.res) + 32;
    if (c.lane == 0) { c.res[c.warp] = bestv; resi[c.warp] = besti; }
    named_bar_sync(1, NCT);
    if (c.warp == 0) {
        float v = (c.lane < NCW) ? c.res[c.lane] : -INFINITY;
        int i = (c.lane < NCW) ? resi[c.lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, i, o);
            if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
        }
        if (c.lane == 0) {
            P.ws->argmax_val[c.cta] = v;
            P.ws->argmax_idx[c.cta] = i;
            __threadfence();
            const uint32_t old = atomicAdd(&P.ws->lm_count, 1u);
            c.misc[MISC_LAST] = (old == (uint32_t)c.G - 1u) ? 1 : 0;
        }
    }
    named_bar_sync(1, NCT);
    if (c.misc[MISC_LAST] && c.warp == 0) {
        __threadfence();
        float v = -INFINITY;
        int i = 0x7fffffff;
        for (int b = c.lane; b < c.G; b += 32) {
            const float ov = __ldcg(P.ws->argmax_val + b);
            const int oi = __ldcg(P.ws->argmax_idx + b);
            if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, i, o);
            if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
        }
        if (c.lane == 0) {
            *P.out_token = i;
            if (P.token_feedback) *P.token_feedback = i;
            if (P.out_tokens_slot) *P.out_tokens_slot = i;
            // every CTA has passed its last barrier: leave the workspace zeroed for the next launch
            P.ws->bar = 0u;
            P.ws->lm_count = 0u;
        }
    }
}

__global__ void __launch_bounds__(NTHREADS, 1) decode_megakernel_bf16(const __grid_constant__ DecodeParams P) {
    extern __shared__ __align__(1024) char smem[];
    Ctx c;
    c.smem = smem;
    c.xs = reinterpret_cast<float*>(smem + OFF_SCRATCH);
    c.res = reinterpret_cast<float*>(smem + OFF_RES);
    c.red = reinterpret_cast<float*>(smem + OFF_RED);
    c.misc = reinterpret_cast<volatile int*>(smem + OFF_MISC);
    c.ring0 = smem_u32(smem + OFF_RING);
    c.full0 = smem_u32(smem + OFF_BAR);
    c.empty0 = c.full0 + NSTAGE * 8;
    c.tid = threadIdx.x; c.warp = threadIdx.x >> 5; c.lane = threadIdx.x & 31;
    c.cta = blockIdx.x; c.G = gridDim.x;
    c.it = 0; c.epoch = 0; c.trace_slot = 0;

    // The pointer table is read on every chunk; keep it in shared memory (the acquire loads of the
    // grid barrier keep invalidating L1, so a global copy would cost an L2 round trip each time).
    LayerWeights* s_layers = reinterpret_cast<LayerWeights*>(smem + OFF_LAYERS);
    for (int i = threadIdx.x; i < P.num_layers * (int)(sizeof(LayerWeights) / 16); i += NTHREADS)
        reinterpret_cast<uint4*>(s_layers)[i] = __ldg(reinterpret_cast<const uint4*>(P.layers) + i);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(c.full0 + s * 8, 1);
            mbar_init(c.empty0 + s * 8, NCW);
        }
        c.misc[MISC_ABORT] = 0;
        c.misc[MISC_LAST] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    int token = P.token_ptr ? __ldcg(P.token_ptr) : P.token_val;
    token = token < 0 ? 0 : (token >= P.vocab ? P.vocab - 1 : token);
    const __nv_bfloat16* embed_row = reinterpret_cast<const __nv_bfloat16*>(P.embed) + (size_t)token * HIDDEN;

    if (c.warp == NCW) {
        // ===== producer warp =====
        const uint64_t pol_stream = l2_policy_evict_first();
        const uint64_t pol_keep = l2_policy_evict_last();
        int dn_idx = 0;
        for (int layer = 0; layer < P.num_layers; ++layer) {
            const LayerWeights& lw = s_layers[layer];
            if (lw.layer_type == 0) {
                producer_phase(P, c, T_DN_IN, lw, dn_idx, pol_stream, pol_keep);
                producer_phase(P, c, T_DN_REC, lw, dn_idx, pol_stream, pol_keep);
                producer_phase(P, c, T_DN_OUT, lw, dn_idx, pol_stream, pol_keep);
                ++dn_idx;
            } else {
                producer_phase(P, c, T_FA_IN, lw, dn_idx, pol_stream, pol_keep);
                producer_phase(P, c, T_FA_OUT, lw, dn_idx, pol_stream, pol_keep);
            }
            producer_phase(P, c, T_GATEUP, lw, dn_idx, pol_stream, pol_keep);
            producer_phase(P, c, T_DOWN, lw, dn_idx, pol_stream, pol_keep);
        }
        producer_phase(P, c, T_LM, s_layers[0], 0, pol_stream, pol_keep);
    } else {
        // ===== consumer warps =====
        if (c.cta == 0 && c.tid == 0 && P.seen_mask && P.rep_penalty > 1.0f) P.seen_mask[token] = 1.0f;
        int dn_idx = 0, fa_idx = 0;
        for (int layer = 0; layer < P.num_layers; ++layer) {
            const LayerWeights& lw = s_layers[layer];
            const __nv_bfloat16* h_in = (layer == 0) ? embed_row : reinterpret_cast<const __nv_bfloat16*>(P.hidden);
            if (lw.layer_type == 0) {
                phase_dn_in(P, c, lw, dn_idx, h_in, layer == 0);
                phase_dn_rec(P, c, dn_idx);
                phase_dn_out(P, c, lw, h_in);
                ++dn_idx;
            } else {
                phase_fa_in(P, c, lw, h_in, layer == 0);
                phase_fa_att(P, c, lw, fa_idx);
                phase_fa_out(P, c, lw, h_in);
                ++fa_idx;
            }
            phase_gateup(P, c, lw);
            phase_down(P, c);
        }
        phase_lm(P, c);
    }
    __syncthreads();
    if (c.misc[MISC_ABORT]) {
        // a wait ran out: give bulk copies that are still in flight time to land before the CTA exits
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 50000ull) {}
    }
}

}  // namespace

size_t decode_smem_bytes() { return SMEM_BYTES; }

int decode_max_grid() {
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cudaFuncSetAttribute(decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_megakernel_bf16, NTHREADS, SMEM_BYTES) != cudaSuccess)
        return 0;
    int g = sms * per_sm;
    return g > MAX_GRID ? MAX_GRID : g;
}

cudaError_t launch_decode_kernel(const DecodeParams& p, int grid, cudaStream_t stream) {
    static bool inv_freq_done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !inv_freq_done[dev]) {
        float tab[FA_ROT / 2];
        for (int i = 0; i < FA_ROT / 2; ++i) tab[i] = (float)(1.0 / pow(ROPE_THETA, (2.0 * i) / FA_ROT));
        e = cudaMemcpyToSymbol(c_inv_freq, tab, sizeof(tab));
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(decode_megakernel_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        inv_freq_done[dev] = true;
    }
    void* args[] = {(void*)&p};
    return cudaLaunchCooperativeKernel((const void*)decode_megakernel_bf16, dim3(grid), dim3(NTHREADS), args,
                                       SMEM_BYTES, stream);
}

}  // namespace mk
