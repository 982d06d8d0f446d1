// Batched decode step: B independent sequences advance by one token each and share every weight pass.
// Included by prefill_bf16.cu inside namespace mk { namespace { (it reuses that file's row-wise kernels).
//
// The reference has no batch dimension in any op (megakernel/torch_bindings.cpp:569-675 are all batch 1); the
// batched step keeps the reference's per-sequence state layouts and puts a leading batch dimension on them:
//   tokens int32 [B], positions int32 [B] (each sequence has its own length),
//   fa_k_cache / fa_v_cache bf16 [B][n_fa][2][max_seq][256], dn_states f32 [B][n_dn][16][128][128],
//   conv_bufs f32 [B][n_dn][6144][4].
// Row-wise work (norms, gates, SwiGLU) treats the batch as B rows, the projections stream each matrix once; the
// kernels below do the per-sequence work: conv window, recurrent state update, attention over each sequence's own
// cache, and the LM head with one argmax per sequence.  Rounding points are those of the prompt path.

constexpr int BATCH_MAX = 16;

// The whole token mixer of a Gated DeltaNet layer for one (sequence, head) per block, 16 warps (two blocks per SM):
//   gates from the raw beta / alpha products, causal conv1d (window of four inputs) + SiLU + L2 norms with the
//   shifted window written back, one gated-delta-rule step on the head's 128 x 128 state (warp = eight value rows,
//   lane = four keys; the rows are requested before anything else so that their latency hides the rest), and the
//   gated RMSNorm of the head's output, written as bf16 for the out projection.
// Arithmetic: k_dn_gates_mma's epilogue, k_dn_preproject at t = 0 + k_dn_conv_state with S = 1, one iteration of
// k_dn_scan, k_dn_gated_norm.  The step is bound by the state traffic (2 x 64 KB per block).
// qkv, z: bf16 [B][6144], [B][2048]; graw: f32 [B][32] = W_b x | W_a x; act: bf16 [B][2048].
__global__ void __launch_bounds__(512, 2) k_dnb_layer(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ z,
                                                    const float* __restrict__ graw, const __nv_bfloat16* __restrict__ conv_w,
                                                    const __nv_bfloat16* __restrict__ a_log, const __nv_bfloat16* __restrict__ dt_bias,
                                                    const __nv_bfloat16* __restrict__ norm_w, float* __restrict__ conv_state,
                                                    size_t conv_seq_stride, float* __restrict__ state, size_t state_seq_stride,
                                                    __nv_bfloat16* __restrict__ act) {
    pdl_launch_next();
    const int b = blockIdx.x, h = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ __align__(16) float qs[DN_KEY], ks[DN_KEY], vs[DN_VAL], os[DN_VAL];
    __shared__ float red[3][4];
    __shared__ float gate[4];                                 // beta, decay, q.k
    constexpr int RW = 8;                                     // value rows per warp
    float* sbase = state + (size_t)b * state_seq_stride + ((size_t)h * DN_VAL + warp * RW) * DN_KEY;
    float4 s[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) s[r] = reinterpret_cast<const float4*>(sbase + r * DN_KEY)[lane];
    // neither the state nor the conv window is written by the projection kernel before this one: both are requested
    // here, ahead of the wait
    float* cs = conv_state + (size_t)b * conv_seq_stride;
    float4 win[3];
    uint2 cw[3];
    if (threadIdx.x < 128) {
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            const int ch = r * DN_QK + h * DN_KEY + threadIdx.x;
            win[r] = *reinterpret_cast<const float4*>(cs + ch * 4);
            cw[r] = __ldg(reinterpret_cast<const uint2*>(conv_w) + ch);
        }
    }
    pdl_wait_prior();
    if (threadIdx.x < 128) {
        const int c = threadIdx.x;
        float val[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            const int ch = r * DN_QK + h * DN_KEY + c;
            const uint2 wr = cw[r];
            const float w4[4] = {bf_lo(wr.x), bf_hi(wr.x), bf_lo(wr.y), bf_hi(wr.y)};
            const float4 old = win[r];
            const float x[4] = {old.y, old.z, old.w, ld_bf(qkv + (size_t)b * DN_CONV_CH + ch)};
            float co = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) co += x[k] * w4[k];
            val[r] = silu_f(co);
            *reinterpret_cast<float4*>(cs + ch * 4) = make_float4(x[0], x[1], x[2], x[3]);
        }
        float sq = warp_sum(val[0] * val[0]), sk = warp_sum(val[1] * val[1]), sqk = warp_sum(val[0] * val[1]);
        if ((c & 31) == 0) { red[0][c >> 5] = sq; red[1][c >> 5] = sk; red[2][c >> 5] = sqk; }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        sq = red[0][0] + red[0][1] + red[0][2] + red[0][3];
        sk = red[1][0] + red[1][1] + red[1][2] + red[1][3];
        sqk = red[2][0] + red[2][1] + red[2][2] + red[2][3];
        const float qn = rsqrtf(sq + 1e-6f) * 0.08838834764831845f, kn = rsqrtf(sk + 1e-6f);
        qs[c] = val[0] * qn;
        ks[c] = val[1] * kn;
        vs[c] = val[2];
        if (c == 0) gate[2] = sqk * qn * kn;
    } else if (threadIdx.x == 128) {
        gate[0] = 1.0f / (1.0f + expf(-graw[b * 32 + h]));
        const float x = graw[b * 32 + 16 + h] + ld_bf(dt_bias + h);
        const float sp = (x > 20.0f) ? x : log1pf(expf(x));
        gate[1] = expf(-expf(ld_bf(a_log + h)) * sp);
    }
    __syncthreads();
    const float4 q4 = reinterpret_cast<const float4*>(qs)[lane], k4 = reinterpret_cast<const float4*>(ks)[lane];
    const float beta = gate[0], decay = gate[1], qk = gate[2];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const int row = warp * RW + r;
        float stk = s[r].x * k4.x + s[r].y * k4.y + s[r].z * k4.z + s[r].w * k4.w;
        float sqv = s[r].x * q4.x + s[r].y * q4.y + s[r].z * q4.z + s[r].w * q4.w;
#pragma unroll
        for (int of = 16; of > 0; of >>= 1) {
            stk += __shfl_xor_sync(0xffffffffu, stk, of);
            sqv += __shfl_xor_sync(0xffffffffu, sqv, of);
        }
        const float err = (vs[row] - decay * stk) * beta;
        s[r].x = fmaf(s[r].x, decay, k4.x * err); s[r].y = fmaf(s[r].y, decay, k4.y * err);
        s[r].z = fmaf(s[r].z, decay, k4.z * err); s[r].w = fmaf(s[r].w, decay, k4.w * err);
        if (lane == 0) os[row] = decay * sqv + err * qk;
        reinterpret_cast<float4*>(sbase + r * DN_KEY)[lane] = s[r];
    }
    __syncthreads();
    if (warp == 0) {
        const size_t off = (size_t)b * DN_V + h * DN_VAL;
        const float4 o4 = reinterpret_cast<const float4*>(os)[lane];
        const uint2 z2 = reinterpret_cast<const uint2*>(z + off)[lane];
        const uint2 w2 = __ldg(reinterpret_cast<const uint2*>(norm_w) + lane);
        const float ss = warp_sum(o4.x * o4.x + o4.y * o4.y + o4.z * o4.z + o4.w * o4.w);
        const float rstd = rsqrtf(ss * (1.0f / DN_VAL) + RMS_EPS);
        const __nv_bfloat162 p0 = __floats2bfloat162_rn(o4.x * rstd * bf_lo(w2.x) * silu_f(bf_lo(z2.x)),
                                                        o4.y * rstd * bf_hi(w2.x) * silu_f(bf_hi(z2.x)));
        const __nv_bfloat162 p1 = __floats2bfloat162_rn(o4.z * rstd * bf_lo(w2.y) * silu_f(bf_lo(z2.y)),
                                                        o4.w * rstd * bf_hi(w2.y) * silu_f(bf_hi(z2.y)));
        uint2 r;
        r.x = *reinterpret_cast<const uint32_t*>(&p0); r.y = *reinterpret_cast<const uint32_t*>(&p1);
        reinterpret_cast<uint2*>(act + off)[lane] = r;
    }
}

// Attention of one new query per sequence over that sequence's cache (positions 0 .. pos[b], the new key and
// value already appended).  Block = (sequence, query head), sixteen warps stride over the keys eight at a time with an
// online softmax each (lane = 8 of the 256 dimensions), then merge through shared memory.
// out[b][head][256] = softmax(q k^T / 16) v * sigmoid(gate), bf16.
constexpr int FAB_WARPS = 16, FAB_UN = 8;      // the kernel is a chain of cache-row round trips: keep many rows in flight
__global__ void __launch_bounds__(FAB_WARPS * 32) k_fab_attention(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ kc,
                                                       const __nv_bfloat16* __restrict__ vc, size_t seq_stride,
                                                       const int* __restrict__ pos, int max_seq, __nv_bfloat16* __restrict__ out) {
    pdl_launch_next();
    const int b = blockIdx.x, hq = blockIdx.y, g = hq >> 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = min(max(pos[b], 0), max_seq - 1) + 1;       // positions were advanced a whole step ago
    const __nv_bfloat16* qrow = qkv + (size_t)b * FA_QKV_ROWS + hq * 2 * FA_HEAD_DIM;
    const __nv_bfloat16* kb = kc + (size_t)b * seq_stride + (size_t)g * max_seq * FA_HEAD_DIM;
    const __nv_bfloat16* vb = vc + (size_t)b * seq_stride + (size_t)g * max_seq * FA_HEAD_DIM;
    // Rows 0 .. n-2 of the cache are older than this step (the kernel before this one appends row n-1 only): ask for
    // them to be brought into L2 while that kernel runs.  One block per KV head does it, at most 1 MB per tensor.
    if (threadIdx.x == 0 && (hq & 3) == 0 && n > 1) {
        const uint32_t bytes = (uint32_t)min(n - 1, 2048) * FA_HEAD_DIM * 2;
        l2_prefetch(kb, bytes);
        l2_prefetch(vb, bytes);
    }
    pdl_wait_prior();
    float q[8];
    {
        const uint4 u = reinterpret_cast<const uint4*>(qrow)[lane];
        q[0] = bf_lo(u.x); q[1] = bf_hi(u.x); q[2] = bf_lo(u.y); q[3] = bf_hi(u.y);
        q[4] = bf_lo(u.z); q[5] = bf_hi(u.z); q[6] = bf_lo(u.w); q[7] = bf_hi(u.w);
    }
    float m = -INFINITY, l = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j0 = warp; j0 < n; j0 += FAB_WARPS * FAB_UN) {
        uint4 ku[FAB_UN], vu[FAB_UN];
        float s[FAB_UN];
#pragma unroll
        for (int u = 0; u < FAB_UN; ++u) {
            const int j = j0 + FAB_WARPS * u;
            const bool in = j < n;
            ku[u] = in ? __ldg(reinterpret_cast<const uint4*>(kb + (size_t)j * FA_HEAD_DIM) + lane) : make_uint4(0, 0, 0, 0);
            vu[u] = in ? __ldg(reinterpret_cast<const uint4*>(vb + (size_t)j * FA_HEAD_DIM) + lane) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < FAB_UN; ++u) s[u] = dot8(ku[u], q, 0.f);
#pragma unroll
        for (int of = 16; of > 0; of >>= 1) {
#pragma unroll
            for (int u = 0; u < FAB_UN; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], of);
        }
        float mn = m;
#pragma unroll
        for (int u = 0; u < FAB_UN; ++u) {
            s[u] = (j0 + FAB_WARPS * u < n) ? s[u] * 0.0625f : -INFINITY;
            mn = fmaxf(mn, s[u]);
        }
        const float corr = __expf(m - mn);          // first pass: exp(-inf) = 0
        l *= corr;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= corr;
#pragma unroll
        for (int u = 0; u < FAB_UN; ++u) {
            const float p = __expf(s[u] - mn);
            l += p;
            const uint32_t w[4] = {vu[u].x, vu[u].y, vu[u].z, vu[u].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                acc[2 * e] = fmaf(p, bf_lo(w[e]), acc[2 * e]);
                acc[2 * e + 1] = fmaf(p, bf_hi(w[e]), acc[2 * e + 1]);
            }
        }
        m = mn;
    }
    __shared__ float sm_m[FAB_WARPS], sm_l[FAB_WARPS];
    __shared__ float sm_acc[FAB_WARPS][FA_HEAD_DIM];
    if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
#pragma unroll
    for (int e = 0; e < 8; ++e) sm_acc[warp][lane * 8 + e] = acc[e];
    __syncthreads();
    const int d = threadIdx.x;                       // one output dimension per thread (the first 256)
    if (d >= FA_HEAD_DIM) return;
    float mm = sm_m[0];
#pragma unroll
    for (int w = 1; w < FAB_WARPS; ++w) mm = fmaxf(mm, sm_m[w]);
    float tot = 0.f, ov = 0.f;
#pragma unroll
    for (int w = 0; w < FAB_WARPS; ++w) {
        const float f = (sm_m[w] == -INFINITY) ? 0.f : __expf(sm_m[w] - mm);
        tot += sm_l[w] * f;
        ov += sm_acc[w][d] * f;
    }
    const float gate = ld_bf(qrow + FA_HEAD_DIM + d);
    out[(size_t)b * FA_Q_SIZE + hq * FA_HEAD_DIM + d] = __float2bfloat16_rn(ov / tot * (1.0f / (1.0f + __expf(-gate))));
}

// LM head for NB rows of activations at once: every vocabulary row is read once and multiplied with all NB
// activation vectors (f32, staged in shared memory in the order the lanes read them).  Warp = two vocabulary rows
// per iteration.  Per block and sequence the best logit (lowest index on ties) goes to bval / bidx [NB][grid].
template <int NB>
__global__ void __launch_bounds__(256) k_lm_head_batch(const float* __restrict__ x, int B, const __nv_bfloat16* __restrict__ W,
                                                       int vocab, float* __restrict__ bval, int* __restrict__ bidx) {
    pdl_enter();
    extern __shared__ __align__(16) float4 xs[];      // [NB][8 pieces][32 lanes]: piece 2i + half = dims i*256 + lane*8 + half*4 ..
    __shared__ float sv[8][NB];
    __shared__ int si[8][NB];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int idx = threadIdx.x; idx < NB * 256; idx += 256) {
        const int b = idx >> 8, r = idx & 255, piece = r >> 5, ln = r & 31;
        xs[idx] = (b < B) ? *reinterpret_cast<const float4*>(x + (size_t)b * HIDDEN + (piece >> 1) * 256 + ln * 8 + (piece & 1) * 4)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    float best[NB];
    int besti[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) { best[b] = -INFINITY; besti[b] = 0x7fffffff; }
    for (int row0 = (blockIdx.x * 8 + warp) * 2; row0 < vocab; row0 += gridDim.x * 16) {
        const bool two = row0 + 1 < vocab;
        const uint4* wp0 = reinterpret_cast<const uint4*>(W + (size_t)row0 * HIDDEN) + lane;
        const uint4* wp1 = wp0 + (two ? HIDDEN / 8 : 0);
        uint4 wa[4], wb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) { wa[i] = __ldg(wp0 + i * 32); wb[i] = __ldg(wp1 + i * 32); }
        float a0[NB], a1[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) { a0[b] = 0.f; a1[b] = 0.f; }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float fa[8] = {bf_lo(wa[i].x), bf_hi(wa[i].x), bf_lo(wa[i].y), bf_hi(wa[i].y),
                                 bf_lo(wa[i].z), bf_hi(wa[i].z), bf_lo(wa[i].w), bf_hi(wa[i].w)};
            const float fb[8] = {bf_lo(wb[i].x), bf_hi(wb[i].x), bf_lo(wb[i].y), bf_hi(wb[i].y),
                                 bf_lo(wb[i].z), bf_hi(wb[i].z), bf_lo(wb[i].w), bf_hi(wb[i].w)};
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const float4 x0 = xs[(b * 8 + 2 * i) * 32 + lane], x1 = xs[(b * 8 + 2 * i + 1) * 32 + lane];
                a0[b] = fmaf(fa[0], x0.x, a0[b]); a0[b] = fmaf(fa[1], x0.y, a0[b]); a0[b] = fmaf(fa[2], x0.z, a0[b]); a0[b] = fmaf(fa[3], x0.w, a0[b]);
                a0[b] = fmaf(fa[4], x1.x, a0[b]); a0[b] = fmaf(fa[5], x1.y, a0[b]); a0[b] = fmaf(fa[6], x1.z, a0[b]); a0[b] = fmaf(fa[7], x1.w, a0[b]);
                a1[b] = fmaf(fb[0], x0.x, a1[b]); a1[b] = fmaf(fb[1], x0.y, a1[b]); a1[b] = fmaf(fb[2], x0.z, a1[b]); a1[b] = fmaf(fb[3], x0.w, a1[b]);
                a1[b] = fmaf(fb[4], x1.x, a1[b]); a1[b] = fmaf(fb[5], x1.y, a1[b]); a1[b] = fmaf(fb[6], x1.z, a1[b]); a1[b] = fmaf(fb[7], x1.w, a1[b]);
            }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float v0 = warp_sum(a0[b]), v1 = warp_sum(a1[b]);
            if (v0 > best[b]) { best[b] = v0; besti[b] = row0; }
            if (two && v1 > best[b]) { best[b] = v1; besti[b] = row0 + 1; }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int b = 0; b < NB; ++b) { sv[warp][b] = best[b]; si[warp][b] = besti[b]; }
    }
    __syncthreads();
    if (threadIdx.x < NB && threadIdx.x < B) {
        const int b = threadIdx.x;
        float bv = sv[0][b];
        int bi = si[0][b];
        for (int w = 1; w < 8; ++w)
            if (sv[w][b] > bv || (sv[w][b] == bv && si[w][b] < bi)) { bv = sv[w][b]; bi = si[w][b]; }
        bval[(size_t)b * gridDim.x + blockIdx.x] = bv;
        bidx[(size_t)b * gridDim.x + blockIdx.x] = bi;
    }
}

// ---- projections of a batched step ---------------------------------------------------------------------------
// C[b][n] = sum_k A[b][k] W[n][k] (+ R[b][n]) for B <= 16 rows of activations: pure weight streaming, so the kernel is
// built around reading W once at full rate, not around the tensor cores' peak.  One CTA per 16 rows of W, its eight
// warps split K; W goes straight from global memory into mma.sync A fragments (the k order inside a fragment is
// permuted so that a lane reads 16 contiguous bytes of a row: a dot product does not care, and the activations are
// permuted the same way), the activations sit in shared memory as the B operand (batch = the n8 columns), f32
// partial sums of the warps meet in shared memory.  Several matrices that share A (the input projections of a
// layer) run as segments of one launch.
// kind: 0 = bf16 output (+ residual R), 1 = f32 output, 2 = SwiGLU pair: C = bf16(silu(bf16(W x)) * bf16(W2 x)), the
// rounding points of a bf16 gate | up projection followed by k_silu_mul.
struct SkinnySeg { const __nv_bfloat16* W; const __nv_bfloat16* W2; void* C; const __nv_bfloat16* R; int N; int ldc; int kind; };
struct SkinnyArgs { SkinnySeg seg[4]; int nseg; };

// norm_w != null: A is the residual stream [B][1024] and the staged activations are its RMSNorm (weights norm_w),
// exactly k_rmsnorm's arithmetic; every CTA normalises for itself (B x 1024 values: less than a launch costs) and
// keeps the result in shared memory.  norm_w == null: every lane reads its B fragments straight from A (L2
// hits), together with the weights of the same k steps.
// ks > 1 (single plain segment with few rows): ks CTAs share a row group, each takes a slice of K and leaves f32
// partial sums in `part`; the CTA that arrives last at the group's counter adds them in slice order (same result
// whichever CTA that is), applies the residual and writes.  The counter resets itself.
// Persistent: a CTA walks over its share of the (row group, K slice) items; the activations are staged once and the
// weight stream of the next item is already in flight while the current one is reduced and written.
template <int NT>      // n8 tiles over the batch: 1 for B <= 8, 2 for B <= 16
__global__ void __launch_bounds__(256, 2) k_skinny_proj(const __nv_bfloat16* __restrict__ A, const __nv_bfloat16* __restrict__ norm_w,
                                                                      int B, int K, int lda, SkinnyArgs args, int items, int ks,
                                                                      float* __restrict__ part, int* __restrict__ counters) {
    pdl_launch_next();
    // The weights do not depend on the previous kernel: ask for this CTA's row groups (16 rows x K, contiguous)
    // to be brought into L2 while the predecessor is still finishing.
    if (threadIdx.x < 32) {
        const int mine_ = (items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
        for (int j = threadIdx.x; j < mine_; j += 32) {
            const int gg = blockIdx.x + j * gridDim.x;
            if (gg % ks) continue;                           // one CTA of a K-split group asks for the whole group
            int grp = gg / ks, si = 0;
            while (si + 1 < args.nseg && grp >= args.seg[si].N / 16) { grp -= args.seg[si].N / 16; ++si; }
            l2_prefetch(args.seg[si].W + (size_t)grp * 16 * K, 16u * K * 2u);
            if (args.seg[si].kind == 2) l2_prefetch(args.seg[si].W2 + (size_t)grp * 16 * K, 16u * K * 2u);
        }
    }
    pdl_wait_prior();
    extern __shared__ __align__(16) uint4 as[];              // norm mode: [NT * 8][K / 8 + 4] activations, rows >= B zero
    __shared__ float red[8][NT * 8][17];
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int rs = K / 8 + 4;                                // row stride in 16-byte units (+64 B: no bank conflicts)
    const int nst_all = K / 32;                              // a step = 32 k: 64 contiguous bytes of each of 16 rows
    const bool direct = norm_w == nullptr;
    const bool pair = args.seg[0].kind == 2;                 // a pair launch has a single segment
    // a pair splits the warps: 0-3 stream the 16 rows of W, 4-7 the 16 rows of W2, each group splits K four ways
    const int kw = pair ? (warp & 3) : warp, nkw = pair ? 4 : 8;
    const int FG = ((nst_all + ks - 1) / ks + 4 * nkw - 1) / (4 * nkw);      // fetches (of four k steps per warp) per item
    const int mine = (items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

    struct Item { const uint4 *w0, *w1; int st_lo, nst, n0, si, kp, ggrp; };
    auto locate = [&](int j) {
        Item it;
        const int gg = blockIdx.x + j * gridDim.x;
        it.kp = gg % ks; it.ggrp = gg / ks;
        int grp = it.ggrp, si = 0;
        while (si + 1 < args.nseg && grp >= args.seg[si].N / 16) { grp -= args.seg[si].N / 16; ++si; }
        it.si = si; it.n0 = grp * 16;
        const __nv_bfloat16* Wm = (pair && warp >= 4) ? args.seg[si].W2 : args.seg[si].W;
        it.w0 = reinterpret_cast<const uint4*>(Wm + (size_t)(it.n0 + g) * K) + tig;
        it.w1 = reinterpret_cast<const uint4*>(Wm + (size_t)(it.n0 + g + 8) * K) + tig;
        it.st_lo = (it.kp * nst_all) / ks; it.nst = ((it.kp + 1) * nst_all) / ks;
        return it;
    };
    const uint4* arow[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) arow[t] = reinterpret_cast<const uint4*>(A + (size_t)min(t * 8 + g, B - 1) * lda) + tig;
    uint4 lo[4], hi[4], bfr[NT][4];
    auto fetch = [&](int q) {                                // q-th fetch of this warp's stream
        const Item it = locate(q / FG);
        const int st0 = it.st_lo + kw + (q % FG) * 4 * nkw;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int st = st0 + nkw * u;
            if (st < it.nst) { lo[u] = __ldcs(it.w0 + st * 4); hi[u] = __ldcs(it.w1 + st * 4); }
            else { lo[u] = make_uint4(0, 0, 0, 0); hi[u] = make_uint4(0, 0, 0, 0); }
            if (direct) {
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    bfr[t][u] = (st < it.nst && t * 8 + g < B) ? __ldg(arow[t] + st * 4) : make_uint4(0, 0, 0, 0);
            }
        }
    };
    if (mine > 0) fetch(0);                                  // weights are on their way while the activations are staged
    if (!direct) {
        for (int b = warp; b < NT * 8; b += 8) {
            if (b < B) rmsnorm_row(reinterpret_cast<const uint4*>(A + (size_t)b * lda), norm_w, as + b * rs, lane);
            else { for (int i = lane; i < K / 8; i += 32) as[b * rs + i] = make_uint4(0, 0, 0, 0); }
        }
        __syncthreads();                                     // activations staged
    }
    const int b = threadIdx.x >> 4, n = threadIdx.x & 15;    // epilogue: 256 threads = 16 batch columns x 16 rows
    const bool writer = threadIdx.x < NT * 8 * 16 && b < B;
    for (int j = 0; j < mine; ++j) {
        const Item it = locate(j);
        float acc[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t) { acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f; }
        for (int f = 0; f < FG; ++f) {
            const int q = j * FG + f;
            uint4 clo[4], chi[4], cb[NT][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                clo[u] = lo[u]; chi[u] = hi[u];
#pragma unroll
                for (int t = 0; t < NT; ++t) cb[t][u] = bfr[t][u];
            }
            if (q + 1 < mine * FG) fetch(q + 1);             // next fetch in flight while this one is multiplied
            const int st0 = it.st_lo + kw + f * 4 * nkw;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int st = st0 + nkw * u;
                if (st < it.nst) {
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const uint4 bb = direct ? cb[t][u] : as[(t * 8 + g) * rs + st * 4 + tig];
                        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                                     : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                                     : "r"(clo[u].x), "r"(chi[u].x), "r"(clo[u].y), "r"(chi[u].y), "r"(bb.x), "r"(bb.y));
                        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                                     : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                                     : "r"(clo[u].z), "r"(chi[u].z), "r"(clo[u].w), "r"(chi[u].w), "r"(bb.z), "r"(bb.w));
                    }
                }
            }
        }
        // accumulator element e of tile t: W row g + 8 (e >> 1), batch column 8 t + 2 tig + (e & 1)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int e = 0; e < 4; ++e) red[warp][t * 8 + 2 * tig + (e & 1)][g + 8 * (e >> 1)] = acc[t][e];
        }
        __syncthreads();
        const SkinnySeg& sg = args.seg[it.si];
        const size_t o = (size_t)b * sg.ldc + it.n0 + n;
        const int bc = b & (NT * 8 - 1);
        if (ks > 1) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) v += red[w][bc][n];
            float* mypart = part + ((size_t)it.ggrp * ks) * 256;
            if (writer) mypart[it.kp * 256 + threadIdx.x] = v;
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) {
                const int old = atomicAdd(counters + it.ggrp, 1);
                s_last = (old == ks - 1);
                if (old == ks - 1) counters[it.ggrp] = 0;
            }
            __syncthreads();
            if (s_last && writer) {
                __threadfence();
                float tot = 0.f;
                for (int p = 0; p < ks; ++p) tot += __ldcg(mypart + p * 256 + threadIdx.x);
                if (sg.R) tot += ld_bf(sg.R + o);
                reinterpret_cast<__nv_bfloat16*>(sg.C)[o] = __float2bfloat16_rn(tot);
            }
        } else if (writer) {
            if (pair) {
                const float gsum = (red[0][bc][n] + red[1][bc][n]) + (red[2][bc][n] + red[3][bc][n]);
                const float usum = (red[4][bc][n] + red[5][bc][n]) + (red[6][bc][n] + red[7][bc][n]);
                const float gv = __bfloat162float(__float2bfloat16_rn(gsum)), uv = __bfloat162float(__float2bfloat16_rn(usum));
                reinterpret_cast<__nv_bfloat16*>(sg.C)[o] = __float2bfloat16_rn(silu_f(gv) * uv);
            } else {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) v += red[w][bc][n];
                if (sg.R) v += ld_bf(sg.R + o);
                if (sg.kind == 1) reinterpret_cast<float*>(sg.C)[o] = v;
                else reinterpret_cast<__nv_bfloat16*>(sg.C)[o] = __float2bfloat16_rn(v);
            }
        }
        __syncthreads();                                     // red and s_last are reused by the next item
    }
}

// Projections that read the residual stream (K = 1024: DeltaNet / attention input matrices, gate and up): the same
// fragment scheme as k_skinny_proj, one item per CTA and no loop at all: a warp's share of K is four k steps, whose
// weights are requested before the kernel even waits for its predecessor (weights are constants), the RMSNorm of the
// B rows (k_rmsnorm's arithmetic) is staged in shared memory meanwhile.  Three CTAs per SM, so nearly
// every item of the largest launch is resident at once.  A SwiGLU pair puts 8 gate rows and the matching 8 up rows
// into one 16-row tile, so silu(g) * u happens in the epilogue of the thread that owns both.
template <int NT>
__global__ void __launch_bounds__(256, 3) k_skinny_norm(const __nv_bfloat16* __restrict__ A, const __nv_bfloat16* __restrict__ norm_w,
                                                                      int B, SkinnyArgs args) {
    pdl_launch_next();
    constexpr int K = HIDDEN, RS = K / 8 + 4;
    extern __shared__ __align__(16) uint4 as[];              // [NT * 8][RS] normalised activations, rows >= B zero
    __shared__ float red[8][NT * 8][17];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const bool pair = args.seg[0].kind == 2;                 // a pair launch has a single segment
    const int rows = pair ? 8 : 16;
    int grp = blockIdx.x, si = 0;
    while (si + 1 < args.nseg && grp >= args.seg[si].N / rows) { grp -= args.seg[si].N / rows; ++si; }
    const SkinnySeg& sg = args.seg[si];
    const int n0 = grp * rows;
    const uint4* w0 = reinterpret_cast<const uint4*>(sg.W + (size_t)(n0 + g) * K) + tig;
    const uint4* w1 = reinterpret_cast<const uint4*>(pair ? sg.W2 + (size_t)(n0 + g) * K : sg.W + (size_t)(n0 + g + 8) * K) + tig;
    uint4 lo[4], hi[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) { lo[u] = __ldcs(w0 + (warp + 8 * u) * 4); hi[u] = __ldcs(w1 + (warp + 8 * u) * 4); }
    pdl_wait_prior();
    for (int b = warp; b < NT * 8; b += 8) {
        if (b < B) rmsnorm_row(reinterpret_cast<const uint4*>(A + (size_t)b * K), norm_w, as + b * RS, lane);
        else { for (int i = lane; i < K / 8; i += 32) as[b * RS + i] = make_uint4(0, 0, 0, 0); }
    }
    __syncthreads();
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) { acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f; }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const uint4 bb = as[(t * 8 + g) * RS + (warp + 8 * u) * 4 + tig];
            asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                         : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                         : "r"(lo[u].x), "r"(hi[u].x), "r"(lo[u].y), "r"(hi[u].y), "r"(bb.x), "r"(bb.y));
            asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                         : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                         : "r"(lo[u].z), "r"(hi[u].z), "r"(lo[u].w), "r"(hi[u].w), "r"(bb.z), "r"(bb.w));
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][t * 8 + 2 * tig + (e & 1)][g + 8 * (e >> 1)] = acc[t][e];
    }
    __syncthreads();
    const int b = threadIdx.x >> 4, n = threadIdx.x & 15;
    if (threadIdx.x < NT * 8 * 16 && b < B) {
        if (pair) {
            if (n < 8) {
                float gsum = 0.f, usum = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) { gsum += red[w][b][n]; usum += red[w][b][n + 8]; }
                const float gv = __bfloat162float(__float2bfloat16_rn(gsum)), uv = __bfloat162float(__float2bfloat16_rn(usum));
                reinterpret_cast<__nv_bfloat16*>(sg.C)[(size_t)b * sg.ldc + n0 + n] = __float2bfloat16_rn(silu_f(gv) * uv);
            }
        } else {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) v += red[w][b][n];
            const size_t o = (size_t)b * sg.ldc + n0 + n;
            if (sg.R) v += ld_bf(sg.R + o);
            if (sg.kind == 1) reinterpret_cast<float*>(sg.C)[o] = v;
            else reinterpret_cast<__nv_bfloat16*>(sg.C)[o] = __float2bfloat16_rn(v);
        }
    }
}

// host side: launch the segments (all N multiples of 16, K a multiple of 32, at most 4 segments)
constexpr int SKINNY_MAX_GROUPS = 1024;      // row groups a K-split launch may have (counters, partial sums)
struct SkinnyWs { float* part = nullptr; int* counters = nullptr; bool attr = false; };
SkinnyWs g_skinny[64];

inline cudaError_t skinny_proj(const void* A, const void* norm_w, int B, int K, int lda, const SkinnyArgs& args, cudaStream_t stream) {
    int groups = 0;
    for (int i = 0; i < args.nseg; ++i) {
        if (args.seg[i].N % 16) return cudaErrorInvalidValue;
        groups += args.seg[i].N / 16;
    }
    if (K % 32 || lda % 8 || B < 1 || B > 16 || groups == 0 || K > INTER || (norm_w && K != HIDDEN)) return cudaErrorInvalidValue;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    SkinnyWs& ws = g_skinny[dev];
    if (!ws.attr) {
        cudaError_t e = cudaFuncSetAttribute(k_skinny_proj<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * (HIDDEN / 8 + 4) * 16);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_skinny_proj<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 16 * (HIDDEN / 8 + 4) * 16);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_skinny_norm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 16 * (HIDDEN / 8 + 4) * 16);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_skinny_norm<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 16 * (HIDDEN / 8 + 4) * 16);
        if (e == cudaSuccess) e = cudaMalloc((void**)&ws.part, (size_t)SKINNY_MAX_GROUPS * 256 * 4);
        if (e == cudaSuccess) e = cudaMalloc((void**)&ws.counters, SKINNY_MAX_GROUPS * 4);
        if (e == cudaSuccess) e = cudaMemset(ws.counters, 0, SKINNY_MAX_GROUPS * 4);
        if (e != cudaSuccess) return e;
        ws.attr = true;
    }
    // few row groups (the 1024-row out / o / down projections): split K over CTAs until about 256 of them stream
    int ks = 1;
    if (args.nseg == 1 && args.seg[0].kind == 0 && !norm_w) {
        ks = 256 / groups;
        const int max_ks = (K / 32) / 8;                     // at least eight k steps (one per warp) per CTA
        if (ks > max_ks) ks = max_ks;
        if (ks < 1) ks = 1;
        if (groups * ks > SKINNY_MAX_GROUPS) ks = 1;
    }
    const int nt = B <= 8 ? 1 : 2;
    if (norm_w) {
        const bool pair = args.seg[0].kind == 2;
        if (pair && args.nseg != 1) return cudaErrorInvalidValue;
        const int ctas = pair ? args.seg[0].N / 8 : groups;
        const size_t sm = (size_t)nt * 8 * (HIDDEN / 8 + 4) * 16;
        if (nt == 1) return launch_pdl(k_skinny_norm<1>, ctas, 256, sm, stream, (const __nv_bfloat16*)A, (const __nv_bfloat16*)norm_w, B, args);
        return launch_pdl(k_skinny_norm<2>, ctas, 256, sm, stream, (const __nv_bfloat16*)A, (const __nv_bfloat16*)norm_w, B, args);
    }
    const size_t smem = 0;
    static int sms = 0;
    if (!sms && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return cudaErrorInvalidDevice;
    const int items = groups * ks, slots = sms * 2;
    const int grid = items < slots ? items : slots;
    if (nt == 1) return launch_pdl(k_skinny_proj<1>, grid, 256, smem, stream, (const __nv_bfloat16*)A, (const __nv_bfloat16*)norm_w, B, K, lda, args, items, ks, ws.part, ws.counters);
    return launch_pdl(k_skinny_proj<2>, grid, 256, smem, stream, (const __nv_bfloat16*)A, (const __nv_bfloat16*)norm_w, B, K, lda, args, items, ks, ws.part, ws.counters);
}

// The 1024-row projections back into the residual stream (out / o: K = 2048, down: K = 3584): few rows, long K.
// One CTA per 8 rows of W (the other half of the m16 tile stays zero: the tensor cores are nowhere near the
// limit, parallelism is), eight warps split K, and the whole kernel is straight-line: every weight a lane will ever
// need (STEPS x 16 bytes) is requested before the kernel waits for its predecessor, the activations are staged in
// shared memory after the wait while those loads land, then MMAs, one shared-memory sum, residual add, store.
// With 128 CTAs the entire matrix is in flight at once.  C doubles as the residual (read and written in place).
template <int NT, int STEPS>   // K = 256 * STEPS
__global__ void __launch_bounds__(256, 2) k_skinny_res(const __nv_bfloat16* __restrict__ A, int B, const __nv_bfloat16* __restrict__ W,
                                                       __nv_bfloat16* C, int ldc, int* __restrict__ err) {
    pdl_launch_next();
    constexpr int K = 256 * STEPS, RS = K / 8 + 4;
    extern __shared__ __align__(16) uint4 as[];              // [NT * 8][RS] activations, rows >= B zero
    __shared__ float red[8][NT * 8][9];
    __shared__ __align__(8) unsigned long long bar_mem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int n0 = blockIdx.x * 8;
    const uint4* w0 = reinterpret_cast<const uint4*>(W + (size_t)(n0 + g) * K) + tig;
    uint4 lo[STEPS];
#pragma unroll
    for (int u = 0; u < STEPS; ++u) lo[u] = __ldcs(w0 + (warp + 8 * u) * 4);
    const uint32_t bar = smem_u32(&bar_mem);
    if (threadIdx.x == 0) { mbar_init(bar, 1); fence_mbar_init(); }
    for (int i = threadIdx.x; i < (NT * 8 - B) * (K / 8); i += 256) {
        const int b = B + i / (K / 8), c = i % (K / 8);
        as[b * RS + c] = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();                                         // barrier initialised, padding rows written
    pdl_wait_prior();
    // the B activation rows arrive as B bulk copies (one thread issues them; no per-thread load / store round trips)
    if (threadIdx.x == 0) {
        mbar_expect_tx(bar, (uint32_t)B * K * 2);
        const uint64_t pol = l2_policy_evict_last();
        for (int b = 0; b < B; ++b) bulk_g2s(smem_u32(as + b * RS), A + (size_t)b * K, K * 2, bar, pol);
    }
    if (!mbar_wait(bar, 0) && threadIdx.x == 0) *err = 5;    // bounded: gives up and reports instead of hanging
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) { acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f; }
#pragma unroll
    for (int u = 0; u < STEPS; ++u) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const uint4 bb = as[(t * 8 + g) * RS + (warp + 8 * u) * 4 + tig];
            asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                         : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                         : "r"(lo[u].x), "r"(0u), "r"(lo[u].y), "r"(0u), "r"(bb.x), "r"(bb.y));
            asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                         : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                         : "r"(lo[u].z), "r"(0u), "r"(lo[u].w), "r"(0u), "r"(bb.z), "r"(bb.w));
        }
    }
    // accumulator elements 0, 1 of tile t: W row g, batch columns 8 t + 2 tig, + 1 (elements 2, 3 belong to the zero rows)
#pragma unroll
    for (int t = 0; t < NT; ++t) { red[warp][t * 8 + 2 * tig][g] = acc[t][0]; red[warp][t * 8 + 2 * tig + 1][g] = acc[t][1]; }
    __syncthreads();
    const int b = threadIdx.x >> 3, n = threadIdx.x & 7;
    if (threadIdx.x < NT * 8 * 8 && b < B) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += red[w][b][n];
        const size_t o = (size_t)b * ldc + n0 + n;
        C[o] = __float2bfloat16_rn(v + ld_bf(C + o));
    }
}

template <int NT, int STEPS>
inline cudaError_t launch_skinny_res(const void* A, int B, const void* W, void* C, int N, int ldc, int* err, cudaStream_t stream) {
    constexpr size_t smem = (size_t)NT * 8 * (256 * STEPS / 8 + 4) * 16;
    static bool attr[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(k_skinny_res<NT, STEPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    return launch_pdl(k_skinny_res<NT, STEPS>, N / 8, 256, smem, stream, (const __nv_bfloat16*)A, B, (const __nv_bfloat16*)W,
                      (__nv_bfloat16*)C, ldc, err);
}

// C[b][n] += sum_k A[b][k] W[n][k] for K = 2048 or 3584, N a multiple of 8
inline cudaError_t skinny_res(const void* A, int B, int K, const void* W, void* C, int N, int ldc, int* err, cudaStream_t stream) {
    if (B < 1 || B > 16 || N % 8 || (K != 2048 && K != 3584) || !err) return cudaErrorInvalidValue;
    if (B <= 8) return K == 2048 ? launch_skinny_res<1, 8>(A, B, W, C, N, ldc, err, stream) : launch_skinny_res<1, 14>(A, B, W, C, N, ldc, err, stream);
    return K == 2048 ? launch_skinny_res<2, 8>(A, B, W, C, N, ldc, err, stream) : launch_skinny_res<2, 14>(A, B, W, C, N, ldc, err, stream);
}

// LM head of a batched step on the tensor cores: the same fragment scheme as k_skinny_proj, but a warp keeps a
// 16-row group of the vocabulary to itself over all of K = 1024 (no cross-warp sum), the f32 activations enter as two
// bf16 terms (x = hi + lo, relative error 2^-16) accumulated into the same f32 sums, and the epilogue is a running
// argmax per sequence (lowest index on ties).  Persistent: the warps stride over the 16-row groups, the weight
// stream is prefetched across group boundaries.  Per block and sequence the best logit goes to bval / bidx [B][grid].
template <int NT>
__global__ void __launch_bounds__(256, 2) k_lm_head_mma(const float* __restrict__ x, int B, const __nv_bfloat16* __restrict__ W,
                                                        int vocab, float* __restrict__ bval, int* __restrict__ bidx) {
    pdl_launch_next();
    constexpr int RS = HIDDEN / 8 + 4;                        // row stride in 16-byte units (+64 B: no bank conflicts)
    extern __shared__ __align__(16) uint4 xh[];               // hi [NT * 8][RS], then lo [NT * 8][RS]
    __shared__ float sv[8][NT * 8];
    __shared__ int si[8][NT * 8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int ngroups = (vocab + 15) / 16, nwarps = gridDim.x * 8, wg = blockIdx.x * 8 + warp;
    const int mine = wg < ngroups ? (ngroups - wg + nwarps - 1) / nwarps : 0;       // groups of this warp
    constexpr int FG = HIDDEN / 32 / 4;                       // fetches of four k steps per group: 8
    uint4 lo[4], hi[4];
    auto fetch = [&](int q) {                                 // q-th fetch of this warp's stream
        const int n0 = (wg + (q / FG) * nwarps) * 16, st0 = (q % FG) * 4;
        const uint4* w0 = reinterpret_cast<const uint4*>(W + (size_t)min(n0 + g, vocab - 1) * HIDDEN) + tig;
        const uint4* w1 = reinterpret_cast<const uint4*>(W + (size_t)min(n0 + g + 8, vocab - 1) * HIDDEN) + tig;
#pragma unroll
        for (int u = 0; u < 4; ++u) { lo[u] = __ldcs(w0 + (st0 + u) * 4); hi[u] = __ldcs(w1 + (st0 + u) * 4); }
    };
    if (mine > 0) fetch(0);                                  // weights first: they do not depend on the previous kernel
    pdl_wait_prior();
    uint4* xlo = xh + NT * 8 * RS;
    for (int i = threadIdx.x; i < NT * 8 * (HIDDEN / 8); i += 256) {
        const int b = i / (HIDDEN / 8), c = i - b * (HIDDEN / 8);
        uint32_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
        if (b < B) {
            const float4 a = *reinterpret_cast<const float4*>(x + (size_t)b * HIDDEN + c * 8);
            const float4 d = *reinterpret_cast<const float4*>(x + (size_t)b * HIDDEN + c * 8 + 4);
            const float v[8] = {a.x, a.y, a.z, a.w, d.x, d.y, d.z, d.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 hh = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
                const __nv_bfloat162 ll = __floats2bfloat162_rn(v[2 * e] - __low2float(hh), v[2 * e + 1] - __high2float(hh));
                h[e] = *reinterpret_cast<const uint32_t*>(&hh);
                l[e] = *reinterpret_cast<const uint32_t*>(&ll);
            }
        }
        xh[b * RS + c] = make_uint4(h[0], h[1], h[2], h[3]);
        xlo[b * RS + c] = make_uint4(l[0], l[1], l[2], l[3]);
    }
    __syncthreads();
    float best[NT][2];
    int besti[NT][2];
#pragma unroll
    for (int t = 0; t < NT; ++t) { best[t][0] = best[t][1] = -INFINITY; besti[t][0] = besti[t][1] = 0x7fffffff; }
    float acc[NT][4];
    for (int q = 0; q < mine * FG; ++q) {
        const int st0 = (q % FG) * 4;
        if (st0 == 0) {
#pragma unroll
            for (int t = 0; t < NT; ++t) { acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f; }
        }
        uint4 clo[4], chi[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) { clo[u] = lo[u]; chi[u] = hi[u]; }
        if (q + 1 < mine * FG) fetch(q + 1);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int off = (t * 8 + g) * RS + (st0 + u) * 4 + tig;
                const uint4 bh = xh[off], bl = xlo[off];
                asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                             : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                             : "r"(clo[u].x), "r"(chi[u].x), "r"(clo[u].y), "r"(chi[u].y), "r"(bh.x), "r"(bh.y));
                asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                             : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                             : "r"(clo[u].z), "r"(chi[u].z), "r"(clo[u].w), "r"(chi[u].w), "r"(bh.z), "r"(bh.w));
                asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                             : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                             : "r"(clo[u].x), "r"(chi[u].x), "r"(clo[u].y), "r"(chi[u].y), "r"(bl.x), "r"(bl.y));
                asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                             : "+f"(acc[t][0]), "+f"(acc[t][1]), "+f"(acc[t][2]), "+f"(acc[t][3])
                             : "r"(clo[u].z), "r"(chi[u].z), "r"(clo[u].w), "r"(chi[u].w), "r"(bl.z), "r"(bl.w));
            }
        }
        if (st0 == (FG - 1) * 4) {
            // group done: element e of tile t = logit of row n0 + g + 8 (e >> 1) for sequence 8 t + 2 tig + (e & 1)
            const int n0 = (wg + (q / FG) * nwarps) * 16;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int r0 = n0 + g, r1 = n0 + g + 8;
                    float v = r0 < vocab ? acc[t][c] : -INFINITY;
                    int ix = r0;
                    const float v1 = r1 < vocab ? acc[t][2 + c] : -INFINITY;
                    if (v1 > v) { v = v1; ix = r1; }
#pragma unroll
                    for (int of = 4; of < 32; of <<= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, v, of);
                        const int oi = __shfl_xor_sync(0xffffffffu, ix, of);
                        if (ov > v || (ov == v && oi < ix)) { v = ov; ix = oi; }
                    }
                    if (v > best[t][c] || (v == best[t][c] && ix < besti[t][c])) { best[t][c] = v; besti[t][c] = ix; }
                }
            }
        }
    }
    if (g == 0) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int c = 0; c < 2; ++c) { sv[warp][t * 8 + 2 * tig + c] = best[t][c]; si[warp][t * 8 + 2 * tig + c] = besti[t][c]; }
        }
    }
    __syncthreads();
    if (threadIdx.x < NT * 8 && threadIdx.x < B) {
        const int b = threadIdx.x;
        float bv = sv[0][b];
        int bi = si[0][b];
        for (int w = 1; w < 8; ++w)
            if (sv[w][b] > bv || (sv[w][b] == bv && si[w][b] < bi)) { bv = sv[w][b]; bi = si[w][b]; }
        bval[(size_t)b * gridDim.x + blockIdx.x] = bv;
        bidx[(size_t)b * gridDim.x + blockIdx.x] = bi;
    }
}

// After a step of a multi-step run: the chosen tokens become the next inputs, every sequence moves on by one.
__global__ void k_batch_advance(int* __restrict__ tokens, const int* __restrict__ chosen, int* __restrict__ positions,
                                int* __restrict__ log_row, int B) {
    pdl_enter();
    const int b = threadIdx.x;
    if (b >= B) return;
    const int t = chosen[b];
    tokens[b] = t;
    positions[b] += 1;
    if (log_row) log_row[b] = t;
}

int g_batch_res_kernel = 1;        // projections into the residual stream: 0 = K split over CTAs, otherwise the straight-line 8-row kernel
int g_batch_lm_mma = 1;            // LM head of the batched step: 1 = tensor cores (bf16 hi + lo), 0 = f32 CUDA cores
struct BatchWs { float *normed_f32 = nullptr, *bval = nullptr, *graw = nullptr; int *bidx = nullptr, *chosen = nullptr; };
BatchWs g_bws[64];

cudaError_t ensure_batch_ws(BatchWs& w) {
    if (w.normed_f32) return cudaSuccess;
    cudaError_t e = cudaMalloc((void**)&w.normed_f32, (size_t)BATCH_MAX * HIDDEN * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&w.bval, (size_t)BATCH_MAX * LM_BLOCKS * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&w.bidx, (size_t)BATCH_MAX * LM_BLOCKS * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&w.chosen, BATCH_MAX * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&w.graw, BATCH_MAX * 32 * 4);
    return e;
}

// One step for B sequences.  tokens / positions / output_tokens: device int32 [B].
template <typename LayerSource>
int decode_batch_core(const int* tokens, const int* positions, int* output_tokens, int B, const void* embed_weight,
                      LayerSource source, int num_layers, int n_fa, int n_dn, const void* final_norm_w, const void* lm_head_w,
                      void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs, void* final_normed,
                      void* hidden_bf16_out, int max_seq_len, int vocab, int dev, cudaStream_t stream) {
    PrefillWs& w = g_pws[dev];
    BatchWs& bw = g_bws[dev];
    PF_CHECK(ensure_ws(w, B < 64 ? 64 : B, stream, true), "step workspace (grow it with mk_prefill_reserve() before capturing a graph)");
    PF_CHECK(ensure_batch_ws(bw), "batch workspace");
    static bool attr[64] = {false};
    if (!attr[dev]) {
        PF_CHECK(cudaFuncSetAttribute(k_lm_head_batch<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 16 * 256 * 16), "lm head smem");
        PF_CHECK(cudaFuncSetAttribute(k_lm_head_mma<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * 8 * (HIDDEN / 8 + 4) * 16), "lm head smem");
        attr[dev] = true;
    }
    typedef __nv_bfloat16 bf;
    // projections: up to four matrices that share the activations per launch
    auto proj = [&](const void* A, const void* norm_w, int K, std::initializer_list<SkinnySeg> segs) {
        SkinnyArgs a;
        a.nseg = 0;
        for (const SkinnySeg& sg : segs) a.seg[a.nseg++] = sg;
        return skinny_proj(A, norm_w, B, K, K, a, stream);
    };
    auto blocks_for_warps = [&](long long nw) { return (unsigned)((nw + 7) / 8); };
    const size_t kv_seq = (size_t)n_fa * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;          // elements per sequence
    const size_t st_seq = (size_t)n_dn * DN_HEADS * DN_VAL * DN_KEY, cv_seq = (size_t)n_dn * DN_CONV_CH * DN_CONV_K;

    const bool res_kernel = g_batch_res_kernel != 0;          // out / o / down: straight-line kernel unless switched off
    launch_pdl(k_embed, B, 128, 0, stream, tokens, (const bf*)embed_weight, w.hidden, B, vocab);
    int dn_idx = 0, fa_idx = 0;
    for (int li = 0; li < num_layers; ++li) {
        LayerView lv;
        const int rc = source(li, lv);
        if (rc != MK_OK) return rc;
        // every input projection normalises the residual stream itself (lv.in_norm / lv.post_norm)
        if (lv.type == 0) {
            float* state = (float*)dn_states + (size_t)dn_idx * DN_HEADS * DN_VAL * DN_KEY;
            float* cstate = (float*)conv_bufs + (size_t)dn_idx * DN_CONV_CH * DN_CONV_K;
            PF_CHECK(proj(w.hidden, lv.in_norm, HIDDEN, {{(const bf*)lv.w_qkv, nullptr, w.wide, nullptr, DN_CONV_CH, DN_CONV_CH, 0},
                                                         {(const bf*)lv.w_z, nullptr, w.z, nullptr, DN_V, DN_V, 0},
                                                         {(const bf*)lv.w_b, nullptr, bw.graw, nullptr, 16, 32, 1},
                                                         {(const bf*)lv.w_a, nullptr, bw.graw + 16, nullptr, 16, 32, 1}}),
                     "DeltaNet input projections");
            launch_pdl(k_dnb_layer, dim3(B, DN_HEADS), 512, 0, stream, (const bf*)w.wide, (const bf*)w.z, (const float*)bw.graw,
                       (const bf*)lv.conv_w, (const bf*)lv.a_log, (const bf*)lv.dt_bias, (const bf*)lv.dn_norm, cstate, cv_seq, state,
                       st_seq, w.act);
            if (res_kernel) PF_CHECK(skinny_res(w.act, B, DN_V, lv.w_out, w.hidden, HIDDEN, HIDDEN, w.err, stream), "out projection");
            else PF_CHECK(proj(w.act, nullptr, DN_V, {{(const bf*)lv.w_out, nullptr, w.hidden, w.hidden, HIDDEN, HIDDEN, 0}}), "out projection");
            ++dn_idx;
        } else {
            bf* kc = (bf*)fa_k_cache + (size_t)fa_idx * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;
            bf* vc = (bf*)fa_v_cache + (size_t)fa_idx * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;
            if (lv.w_faqkv) {
                PF_CHECK(proj(w.hidden, lv.in_norm, HIDDEN, {{(const bf*)lv.w_faqkv, nullptr, w.wide, nullptr, FA_QKV_ROWS, FA_QKV_ROWS, 0}}),
                         "q, k, v projections");
            } else {
                PF_CHECK(proj(w.hidden, lv.in_norm, HIDDEN,
                              {{(const bf*)lv.w_q, nullptr, w.wide, nullptr, FA_QPROJ, FA_QKV_ROWS, 0},
                               {(const bf*)lv.w_k, nullptr, w.wide + FA_QPROJ, nullptr, FA_KV_SIZE, FA_QKV_ROWS, 0},
                               {(const bf*)lv.w_v, nullptr, w.wide + FA_QPROJ + FA_KV_SIZE, nullptr, FA_KV_SIZE, FA_QKV_ROWS, 0}}),
                         "q, k, v projections");
            }
            launch_pdl(k_fa_norm_rope, blocks_for_warps((long long)B * 12), 256, 0, stream, w.wide, (const bf*)lv.q_norm,
                       (const bf*)lv.k_norm, kc, vc, B, max_seq_len, positions, kv_seq);
            launch_pdl(k_fab_attention, dim3(B, FA_Q_HEADS), FAB_WARPS * 32, 0, stream, (const bf*)w.wide, (const bf*)kc, (const bf*)vc, kv_seq,
                       positions, max_seq_len, w.act);
            if (res_kernel) PF_CHECK(skinny_res(w.act, B, FA_Q_SIZE, lv.w_o, w.hidden, HIDDEN, HIDDEN, w.err, stream), "o projection");
            else PF_CHECK(proj(w.act, nullptr, FA_Q_SIZE, {{(const bf*)lv.w_o, nullptr, w.hidden, w.hidden, HIDDEN, HIDDEN, 0}}), "o projection");
            ++fa_idx;
        }
        // gate and up rows meet in one CTA, which applies SwiGLU before it writes
        const bf* wg = lv.w_gateup ? (const bf*)lv.w_gateup : (const bf*)lv.w_gate;
        const bf* wu = lv.w_gateup ? (const bf*)lv.w_gateup + (size_t)INTER * HIDDEN : (const bf*)lv.w_up;
        PF_CHECK(proj(w.hidden, lv.post_norm, HIDDEN, {{wg, wu, w.act, nullptr, INTER, INTER, 2}}), "gate and up projections");
        if (res_kernel) PF_CHECK(skinny_res(w.act, B, INTER, lv.w_down, w.hidden, HIDDEN, HIDDEN, w.err, stream), "down projection");
        else PF_CHECK(proj(w.act, nullptr, INTER, {{(const bf*)lv.w_down, nullptr, w.hidden, w.hidden, HIDDEN, HIDDEN, 0}}), "down projection");
    }
    launch_pdl(k_final_norm, B, 512, 0, stream, w.hidden, (const bf*)final_norm_w, bw.normed_f32, (bf*)final_normed, (bf*)hidden_bf16_out);
    constexpr int LMB = 296;                                  // two persistent blocks per SM
    constexpr int LM_SMEM1 = 2 * 8 * (HIDDEN / 8 + 4) * 16, LM_SMEM2 = 2 * LM_SMEM1;
    if (g_batch_lm_mma) {
        if (B <= 8) launch_pdl(k_lm_head_mma<1>, LMB, 256, LM_SMEM1, stream, (const float*)bw.normed_f32, B, (const bf*)lm_head_w, vocab, bw.bval, bw.bidx);
        else launch_pdl(k_lm_head_mma<2>, LMB, 256, LM_SMEM2, stream, (const float*)bw.normed_f32, B, (const bf*)lm_head_w, vocab, bw.bval, bw.bidx);
        launch_pdl(k_lm_reduce, B, 32, 0, stream, bw.bval, bw.bidx, LMB, output_tokens);
    } else {
        if (B <= 8) launch_pdl(k_lm_head_batch<8>, LM_BLOCKS, 256, 8 * 256 * 16, stream, bw.normed_f32, B, (const bf*)lm_head_w, vocab, bw.bval, bw.bidx);
        else launch_pdl(k_lm_head_batch<16>, LM_BLOCKS / 2, 256, 16 * 256 * 16, stream, bw.normed_f32, B, (const bf*)lm_head_w, vocab, bw.bval, bw.bidx);
        launch_pdl(k_lm_reduce, B, 32, 0, stream, bw.bval, bw.bidx, B <= 8 ? LM_BLOCKS : LM_BLOCKS / 2, output_tokens);
    }
    PF_CHECK(cudaGetLastError(), "batched step launch");
    return MK_OK;
}
