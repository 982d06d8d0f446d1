// Causal GQA attention for prefill on the 5th-generation tensor cores (dense mode).
//
// One CTA = 32 consecutive query positions x the 4 query heads of one KV head = 128 rows, one row per TMEM lane.
//   warp 0      TMA: the Q tile once, then K tiles (lane 0) and V tiles (lane 1) of 64 keys into two-stage rings with
//               barriers of their own (128-byte swizzle); the two K stages are rows 0-63 / 64-127 of one operand
//   warp 1      one thread issues tcgen05.mma: S = Q K^T for a PAIR of tiles at once (M128 N128, K = 256 in 16
//               steps, over both K stages into the two adjacent score buffers in tensor memory; a lone last tile
//               M128 N64), and O += P V per tile (M128 N256, K = 64 in 4 steps; P is read from tensor memory, V
//               MN-major, i.e. as it lies in the cache: keys x dims)
//   warps 2-9   softmax, two threads per row (warps 2-5 take score columns 0-31, warps 6-9 columns 32-63 of each
//               tile, same TMEM lanes), two tiles per pass: tcgen05.ld the scores, running maximum (exchanged
//               through shared memory) and sum, probabilities rounded to bf16 pairs into one of four buffers in
//               tensor memory (the A operand of P V), and the epilogue
// The score MMAs of the next pair are issued before the P V MMAs of this pair (their buffers are free as soon as the
// softmax has loaded this pair's scores), so the tensor pipe works while the softmax threads process the pair.  The
// output accumulator is rescaled only when a row maximum grows by more than 2^8
// since the last rescale (probabilities then stay below 2^8, exact enough in bf16/f32): with a causal mask the
// maximum settles after the first tiles, so the TMEM round trip of a rescale is rare.
// Every wait is bounded; on expiry the kernel sets *err and leaves.
// (reference arithmetic: softmax(q k^T / 16) v * sigmoid(gate), megakernel/prefill.cu:1202-1236)
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mk_common.cuh"
#include "mk_prefill.h"

namespace mk {
namespace {

constexpr int TQ = 32;                         // query positions per CTA
constexpr int TK = 64;                         // keys per tile
constexpr int Q_BYTES = 128 * 512;             // 4 dim-blocks x [128 rows x 128 B]
constexpr int KV_BYTES = TK * 512;             // 4 dim-blocks x [64 keys x 128 B]
constexpr int P_BYTES = 128 * 128;             // [128 rows x 64 keys] bf16
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_BYTES;                     // 2 stages
constexpr int OFF_V = OFF_K + 2 * KV_BYTES;                // 2 stages
constexpr int OFF_P = OFF_V + 2 * KV_BYTES;
constexpr int OFF_BARS = OFF_P + P_BYTES;
constexpr int BAR_BYTES = 256;                             // barriers, tensor-memory slot, tile count
constexpr int OFF_LIST = OFF_BARS + BAR_BYTES + 2048;            // after the barriers and the 2 x 2 x 128 floats of row-maximum exchange;
                                                           // block-sparse mode: up to 2048 tile ids (u16)
constexpr int FA5_SMEM = OFF_LIST + 4096 + 1024;           // + alignment slack
constexpr uint32_t TM_COLS = 512;
constexpr uint32_t TM_S0 = 0, TM_O = 128;                  // score buffers at columns 0 and 64, output at 128..383
constexpr uint32_t TM_P = 384;                             // probabilities, bf16 pairs: four buffers of 32 columns (64 keys)

__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar) : "memory");
}
// K-major operand, 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart
__device__ __forceinline__ uint64_t desc_k(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3ffffu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}
// MN-major operand, 128-byte swizzle: 64 MN elements per 128-byte row, K rows 128 bytes apart in groups of 8
// (1024 bytes per group); blocks of 64 MN elements `mn_block_bytes` apart
__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr, uint32_t mn_block_bytes) {
    return (uint64_t)((saddr & 0x3ffffu) >> 4) | ((uint64_t)(mn_block_bytes >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ uint32_t idesc(int m, int n, bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma5(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc) : "memory");
}
// 2^x on the special-function unit alone (exp2f wraps the same instruction in a range fix-up for denormal results,
// four more instructions per probability; results below 2^-126 are flushed to zero, which is what a probability that
// small rounds to in bf16 anyway)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// the same with the A operand in tensor memory (row = lane, two bf16 of consecutive k per 32-bit column)
__device__ __forceinline__ void mma5_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
                 ::"r"(d), "r"(a_tmem), "l"(b), "r"(id), "r"(acc) : "memory");
}
#define TM_ST16(taddr, v)                                                                                              \
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"                  \
                 ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),           \
                   "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]) : "memory")
__device__ __forceinline__ void commit5(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool waitb(uint32_t bar, uint32_t parity, int* err) {
    for (uint32_t n = 0; n < (1u << 24); ++n)
        if (mbar_try_wait(bar, parity)) return true;
    atomicExch(err, 3);
    return false;
}
#define TM_LD64(taddr, v)                                                                                              \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 "                                                            \
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31," \
                 "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];" \
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]),   \
                   "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),    \
                   "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),   \
                   "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]), "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]),   \
                   "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]), "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]),   \
                   "=r"(v[46]), "=r"(v[47]), "=r"(v[48]), "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]),   \
                   "=r"(v[55]), "=r"(v[56]), "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])    \
                 : "r"(taddr) : "memory")
#define TM_ST64(taddr, v)                                                                                              \
    asm volatile("tcgen05.st.sync.aligned.32x32b.x64.b32 [%64], "                                                     \
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31," \
                 "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63};" \
                 ::"r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),           \
                   "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]),  \
                   "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),  \
                   "r"(v[30]), "r"(v[31]), "r"(v[32]), "r"(v[33]), "r"(v[34]), "r"(v[35]), "r"(v[36]), "r"(v[37]), "r"(v[38]), "r"(v[39]),  \
                   "r"(v[40]), "r"(v[41]), "r"(v[42]), "r"(v[43]), "r"(v[44]), "r"(v[45]), "r"(v[46]), "r"(v[47]), "r"(v[48]), "r"(v[49]),  \
                   "r"(v[50]), "r"(v[51]), "r"(v[52]), "r"(v[53]), "r"(v[54]), "r"(v[55]), "r"(v[56]), "r"(v[57]), "r"(v[58]), "r"(v[59]),  \
                   "r"(v[60]), "r"(v[61]), "r"(v[62]), "r"(v[63]), "r"(taddr) : "memory")

#define TM_LD32(taddr, v)                                                                                              \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "                                                            \
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];" \
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]),   \
                   "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),    \
                   "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),   \
                   "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])                                                                      \
                 : "r"(taddr) : "memory")

// map_q: 2-D view of the qkv buffer restricted to the query heads: (dims 0..4095, tokens), box 64 x 32;
// map_k0/1, map_v0/1: 2-D views of the two KV heads of one layer's cache: (256 dims, S rows), box 64 x 64; rows
// past the prompt read as zeros, so stale cache contents never meet a zero probability.
__global__ void __launch_bounds__(320, 1)
k_fa_tcgen05(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k0,
             const __grid_constant__ CUtensorMap map_k1, const __grid_constant__ CUtensorMap map_v0,
             const __grid_constant__ CUtensorMap map_v1, const __nv_bfloat16* __restrict__ qkv,
             __nv_bfloat16* __restrict__ out, int S, int* err, const uint32_t* __restrict__ mask, int nblk, int nwords) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ char smem_raw[];
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sb = smem_u32(smem);
    const uint32_t bars = sb + OFF_BARS;
    // K and V stages have barriers of their own: a K stage is free as soon as the score MMA that read it is done (one
    // tile earlier than the V stage of the same tile), so the next K tile is requested that much sooner -- with one pair
    // of barriers for both, every score MMA waited for a K tile that had been requested only when the previous P V ended.
    const uint32_t q_full = bars, k_full0 = bars + 8, k_empty0 = bars + 24, s_full0 = bars + 40, s_empty0 = bars + 56,
                   v_full0 = bars + 120, v_empty0 = bars + 136;
    // Per probability buffer b = tile & 3: p_full(b) = the softmax has written the tile's probabilities, pv_done(b) =
    // the P V product that read them is complete.  (One barrier per buffer: the softmax runs up to a pair of tiles
    // ahead of the P V products, and a parity wait cannot tell a phase from the one two phases later.)
    auto p_full = [&](int b) { return bars + 160 + 8 * (uint32_t)b; };
    auto pv_done = [&](int b) { return bars + 192 + 8 * (uint32_t)b; };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BARS + 96);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qblk = gridDim.x - 1 - blockIdx.x, g = blockIdx.y;
    const int q0 = qblk * TQ;
    const int last_q = min(q0 + TQ, S) - 1;
    int ntiles = last_q / TK + 1;
    // block-sparse mode: mask[head][query block of 128][word], one bit per key block of 128.  The CTA walks the
    // union of the blocks its four heads keep; a head that dropped a block gets zero probabilities for it.
    unsigned short* tlist = reinterpret_cast<unsigned short*>(smem + OFF_LIST);
    int* tcount = reinterpret_cast<int*>(smem + OFF_BARS + 112);
    const uint32_t* m0 = nullptr;
    size_t hstride = 0;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (mask) {
        m0 = mask + ((size_t)(g * 4) * nblk + (q0 >> 7)) * nwords;
        hstride = (size_t)nblk * nwords;
        if (threadIdx.x == 64) {
            int n = 0;
            for (int w = 0; w < nwords; ++w) {
                uint32_t u = m0[w] | m0[w + hstride] | m0[w + 2 * hstride] | m0[w + 3 * hstride];
                while (u) {
                    const int b = __ffs(u) - 1;
                    u &= u - 1;
                    const int t0 = (w * 32 + b) * 2;
                    if (t0 * TK <= last_q) tlist[n++] = (unsigned short)t0;
                    if ((t0 + 1) * TK <= last_q) tlist[n++] = (unsigned short)(t0 + 1);
                }
            }
            *tcount = n;
        }
    }

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(k_full0 + 8 * s, 1); mbar_init(k_empty0 + 8 * s, 1);
            mbar_init(v_full0 + 8 * s, 1); mbar_init(v_empty0 + 8 * s, 1);
            mbar_init(s_full0 + 8 * s, 1); mbar_init(s_empty0 + 8 * s, 256);
        }
        for (int b = 0; b < 4; ++b) { mbar_init(p_full(b), 256); mbar_init(pv_done(b), 1); }
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(TM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
    if (mask) ntiles = *tcount;
    auto tile_of = [&](int j) { return mask ? (int)tlist[j] : j; };
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            // Q tile: row = head * 32 + position; dim-block b of head hh is one box of 64 dims x 32 positions
            mbar_expect_tx(q_full, Q_BYTES);
            for (int hh = 0; hh < 4; ++hh)
                for (int b = 0; b < 4; ++b)
                    tma2d(sb + OFF_Q + b * (128 * 128) + hh * (32 * 128), &map_q, (g * 4 + hh) * 512 + b * 64, q0, q_full);
            const CUtensorMap* mk_ = g ? &map_k1 : &map_k0;
            for (int j = 0; j < ntiles && ok; ++j) {
                const int s = j & 1;
                ok = waitb(k_empty0 + 8 * s, ((j >> 1) & 1) ^ 1u, err);
                if (!ok) break;
                mbar_expect_tx(k_full0 + 8 * s, KV_BYTES);
                for (int b = 0; b < 4; ++b)      // dim-block b: 128 rows of 128 bytes, stage s = rows 64 s .. 64 s + 63
                    tma2d(sb + OFF_K + b * (2 * TK * 128) + s * (TK * 128), mk_, b * 64, tile_of(j) * TK, k_full0 + 8 * s);
            }
        } else if (lane == 1) {          // the V tiles go through a second thread: a wait for a V stage never delays a K request
            const CUtensorMap* mv_ = g ? &map_v1 : &map_v0;
            for (int j = 0; j < ntiles && ok; ++j) {
                const int s = j & 1;
                ok = waitb(v_empty0 + 8 * s, ((j >> 1) & 1) ^ 1u, err);
                if (!ok) break;
                mbar_expect_tx(v_full0 + 8 * s, KV_BYTES);
                for (int b = 0; b < 4; ++b)
                    tma2d(sb + OFF_V + s * KV_BYTES + b * (TK * 128), mv_, b * 64, tile_of(j) * TK, v_full0 + 8 * s);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t id_s = idesc(128, TK, false), id_o = idesc(128, 256, true);
            // The two K stages are rows 0-63 and 64-127 of ONE K-major operand per dim-block, and the two score buffers are
            // adjacent columns: the scores of a pair of tiles are one sequence of 16 instructions 128 keys wide instead of
            // two sequences 64 wide (an instruction costs about the same either way).
            const uint32_t id_s2 = idesc(128, 2 * TK, false);
            auto issue_s = [&](int j) {          // one tile (the last of an odd count): stage and score buffer j & 1
                const int s = j & 1;
                const uint32_t qb = sb + OFF_Q, kb = sb + OFF_K + s * (TK * 128);
#pragma unroll
                for (int ks = 0; ks < 16; ++ks)
                    mma5(tmem + TM_S0 + s * TK, desc_k(qb + (ks >> 2) * (128 * 128) + (ks & 3) * 32),
                         desc_k(kb + (ks >> 2) * (2 * TK * 128) + (ks & 3) * 32), id_s, ks ? 1u : 0u);
                commit5(s_full0 + 8 * s);
                commit5(k_empty0 + 8 * s);
            };
            auto issue_s_pair = [&]() {          // tiles (even, odd): both stages, both score buffers
                const uint32_t qb = sb + OFF_Q, kb = sb + OFF_K;
#pragma unroll
                for (int ks = 0; ks < 16; ++ks)
                    mma5(tmem + TM_S0, desc_k(qb + (ks >> 2) * (128 * 128) + (ks & 3) * 32),
                         desc_k(kb + (ks >> 2) * (2 * TK * 128) + (ks & 3) * 32), id_s2, ks ? 1u : 0u);
                commit5(s_full0); commit5(s_full0 + 8);
                commit5(k_empty0); commit5(k_empty0 + 8);
            };
            ok = waitb(q_full, 0, err) && waitb(k_full0, 0, err);
            if (ok && ntiles > 1) ok = waitb(k_full0 + 8, 0, err);
            if (ok) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                if (ntiles > 1) issue_s_pair(); else issue_s(0);
            }
            // The softmax threads take the tiles two at a time (one pass of barrier hops and tensor-memory round trips
            // per 128 keys): per pair, first the score products of the NEXT pair -- their buffers are free as soon as the
            // softmax has loaded this pair's scores -- then the two P V products of this pair.
            for (int jp = 0; jp < ntiles && ok; jp += 2) {
                if (jp + 2 < ntiles) {
                    const bool pair = jp + 3 < ntiles;
                    const uint32_t ph = ((jp + 2) >> 1) & 1, ph_read = (jp >> 1) & 1;
                    ok = waitb(k_full0, ph, err) && waitb(s_empty0, ph_read, err);
                    if (ok && pair) ok = waitb(k_full0 + 8, ph, err) && waitb(s_empty0 + 8, ph_read, err);
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    if (pair) issue_s_pair(); else issue_s(jp + 2);
                }
                for (int t = jp; t < min(jp + 2, ntiles) && ok; ++t) {
                    const int s = t & 1, pb = t & 3;
                    ok = waitb(v_full0 + 8 * s, (t >> 1) & 1, err) && waitb(p_full(pb), (t >> 2) & 1, err);
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t vb = sb + OFF_V + s * KV_BYTES;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)   // 16 keys = 8 columns of the probability buffer per step
                        mma5_ta(tmem + TM_O, tmem + TM_P + (uint32_t)pb * 32 + kk * 8, desc_mn(vb + kk * (16 * 128), TK * 128), id_o, (t | kk) ? 1u : 0u);
                    commit5(v_empty0 + 8 * s);
                    commit5(pv_done(pb));
                }
            }
        }
    } else {
        const int r = (warp & 3) * 32 + lane;                 // row = TMEM lane
        const int half = (warp - 2) >> 2;                      // which 32 of the tile's 64 score columns
        const int hh = r >> 5, qi = r & 31, qpos = q0 + qi;
        const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const float sc = 0.0625f * 1.4426950408889634f;       // 1/sqrt(256) * log2(e)
        float* xbuf = reinterpret_cast<float*>(smem + OFF_BARS + BAR_BYTES);      // [pass parity][2 halves][128 rows]
        float m_ref = -1e30f, lsum = 0.f;
        // A wait that ran out must not make one warp leave the loop while the others sit in the named barrier
        // below: from then on this warp skips every wait (its results are garbage, *err is set) but keeps step.
        bool dead = false;
        auto wait_all = [&](uint32_t bar, uint32_t parity) {
            if (!dead && !__all_sync(0xffffffffu, waitb(bar, parity, err))) dead = true;
        };
        for (int jp = 0; jp < ntiles; jp += 2) {
            const bool two = jp + 1 < ntiles;                  // tiles jp (score buffer 0) and jp + 1 (score buffer 1)
            float* xmax = xbuf + ((jp >> 1) & 1) * 256;
            wait_all(s_full0, (jp >> 1) & 1);
            if (two) wait_all(s_full0 + 8, (jp >> 1) & 1);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint32_t va[32], vb[32];
            TM_LD32(lane_addr + TM_S0 + half * 32, va);
            if (two) TM_LD32(lane_addr + TM_S0 + TK + half * 32, vb);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            mbar_arrive(s_empty0);
            if (two) mbar_arrive(s_empty0 + 8);
            float hmax = -1e30f;
            {
                const int tj = tile_of(jp), key0 = tj * TK + half * 32;
                const bool dropped = mask && !((m0[hh * hstride + (tj >> 6)] >> ((tj >> 1) & 31)) & 1u);   // this head dropped the block
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    float x = __uint_as_float(va[k]) * sc;
                    if (key0 + k > qpos || dropped) x = -1e30f;
                    va[k] = __float_as_uint(x);
                    hmax = fmaxf(hmax, x);
                }
            }
            if (two) {
                const int tj = tile_of(jp + 1), key0 = tj * TK + half * 32;
                const bool dropped = mask && !((m0[hh * hstride + (tj >> 6)] >> ((tj >> 1) & 31)) & 1u);
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    float x = __uint_as_float(vb[k]) * sc;
                    if (key0 + k > qpos || dropped) x = -1e30f;
                    vb[k] = __float_as_uint(x);
                    hmax = fmaxf(hmax, x);
                }
            }
            // row maximum over both halves (and both tiles)
            xmax[half * 128 + r] = hmax;
            named_bar_sync(1, 256);
            const float tmax = fmaxf(hmax, xmax[(half ^ 1) * 128 + r]);
            // the probability buffers of these two tiles were last read by the P V products of tiles jp - 4 and jp - 3
            if (jp >= 4) {
                wait_all(pv_done(jp & 3), ((jp - 4) >> 2) & 1);
                if (two) wait_all(pv_done((jp + 1) & 3), ((jp - 3) >> 2) & 1);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            }
            // tcgen05.ld / st are warp-wide: the decision to rescale is taken per warp, every lane takes part
            // with its own factor (1 for a row whose maximum did not move); each half rescales 128 output columns
            const bool grow = tmax > m_ref + 8.0f;
            if (__any_sync(0xffffffffu, grow)) {
                if (jp >= 1) {
                    // the output accumulator is rescaled in place: every P V issued so far must be complete
                    wait_all(pv_done((jp - 1) & 3), ((jp - 1) >> 2) & 1);
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const float f = grow ? exp2f(m_ref - tmax) : 1.0f;
                    lsum *= f;
#pragma unroll 1
                    for (int c = 0; c < 2; ++c) {
                        uint32_t o[64];
                        TM_LD64(lane_addr + TM_O + half * 128 + c * 64, o);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                        for (int k = 0; k < 64; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * f);
                        TM_ST64(lane_addr + TM_O + half * 128 + c * 64, o);
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                }
                if (grow) m_ref = tmax;
            }
            // probabilities -> bf16 pairs into this thread's 16 columns of the tiles' tensor-memory buffers (the A operand of P V)
            {
                uint32_t w[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float p0 = ex2_approx(__uint_as_float(va[2 * e]) - m_ref);
                    const float p1 = ex2_approx(__uint_as_float(va[2 * e + 1]) - m_ref);
                    const __nv_bfloat162 pp = __floats2bfloat162_rn(p0, p1);
                    w[e] = *reinterpret_cast<const uint32_t*>(&pp);
                    lsum += bf_lo(w[e]) + bf_hi(w[e]);
                }
                TM_ST16(lane_addr + TM_P + (uint32_t)(jp & 3) * 32 + half * 16, w);
            }
            if (two) {
                uint32_t w[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float p0 = ex2_approx(__uint_as_float(vb[2 * e]) - m_ref);
                    const float p1 = ex2_approx(__uint_as_float(vb[2 * e + 1]) - m_ref);
                    const __nv_bfloat162 pp = __floats2bfloat162_rn(p0, p1);
                    w[e] = *reinterpret_cast<const uint32_t*>(&pp);
                    lsum += bf_lo(w[e]) + bf_hi(w[e]);
                }
                TM_ST16(lane_addr + TM_P + (uint32_t)((jp + 1) & 3) * 32 + half * 16, w);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            mbar_arrive(p_full(jp & 3));
            if (two) mbar_arrive(p_full((jp + 1) & 3));
        }
        // epilogue: O / l * sigmoid(gate) -> bf16; the row sum is the two halves' sums
        wait_all(pv_done((ntiles - 1) & 3), ((ntiles - 1) >> 2) & 1);
        float* xsum = xbuf + ((((ntiles - 1) >> 1) + 1) & 1) * 256;       // the exchange buffer the last pass did not use
        xsum[half * 128 + r] = lsum;
        named_bar_sync(1, 256);
        if (!dead) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const float inv = 1.0f / (lsum + xsum[(half ^ 1) * 128 + r]);
            const int head = g * 4 + hh;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                uint32_t o[64];
                const int col0 = half * 128 + c * 64;
                TM_LD64(lane_addr + TM_O + col0, o);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (qpos < S) {
                    const __nv_bfloat16* gate = qkv + (size_t)qpos * FA_QKV_ROWS + head * 2 * FA_HEAD_DIM + FA_HEAD_DIM + col0;
                    __nv_bfloat16* dst = out + (size_t)qpos * FA_Q_SIZE + head * FA_HEAD_DIM + col0;
#pragma unroll
                    for (int k8 = 0; k8 < 8; ++k8) {
                        const uint4 gu = *reinterpret_cast<const uint4*>(gate + k8 * 8);
                        const uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w};
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const __nv_bfloat162 pp = __floats2bfloat162_rn(
                                __uint_as_float(o[k8 * 8 + 2 * e]) * inv * sigmoid_f(bf_lo(gw[e])),
                                __uint_as_float(o[k8 * 8 + 2 * e + 1]) * inv * sigmoid_f(bf_hi(gw[e])));
                            w[e] = *reinterpret_cast<const uint32_t*>(&pp);
                        }
                        *reinterpret_cast<uint4*>(dst + k8 * 8) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TM_COLS) : "memory");
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn5() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess) fn = (EncodeTiledFn)p;
    }
    return fn;
}
// (cols x rows) bf16 matrix with row pitch `pitch` elements; box = 64 cols x box_rows, 128-byte swizzle
bool map2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t pitch, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn5();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t fa_prefill_tcgen05(const void* qkv, const void* kc, const void* vc, void* out, int S, int max_seq, int* err,
                               const uint32_t* mask, cudaStream_t stream) {
    const int nblk = (S + 127) / 128, nwords = (nblk + 31) / 32;
    if (mask && nblk > 1024) return cudaErrorInvalidValue;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(k_fa_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize, FA5_SMEM);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    CUtensorMap mq, k0, k1, v0, v1;
    const __nv_bfloat16* K = (const __nv_bfloat16*)kc;
    const __nv_bfloat16* V = (const __nv_bfloat16*)vc;
    const size_t head = (size_t)max_seq * FA_HEAD_DIM;
    // rows beyond S (qkv buffer, caches) are zero-filled by TMA
    if (!map2d(&mq, qkv, FA_QPROJ, (uint64_t)S, FA_QKV_ROWS, TQ) || !map2d(&k0, K, FA_HEAD_DIM, (uint64_t)S, FA_HEAD_DIM, TK) ||
        !map2d(&k1, K + head, FA_HEAD_DIM, (uint64_t)S, FA_HEAD_DIM, TK) || !map2d(&v0, V, FA_HEAD_DIM, (uint64_t)S, FA_HEAD_DIM, TK) ||
        !map2d(&v1, V + head, FA_HEAD_DIM, (uint64_t)S, FA_HEAD_DIM, TK))
        return cudaErrorInvalidValue;
    return launch_pdl(k_fa_tcgen05, dim3((S + TQ - 1) / TQ, FA_KV_HEADS), 320, FA5_SMEM, stream, mq, k0, k1, v0, v1,
                      (const __nv_bfloat16*)qkv, (__nv_bfloat16*)out, S, err, mask, nblk, nwords);
}

}  // namespace mk
