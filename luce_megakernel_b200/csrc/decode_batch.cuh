// Batched decode step: B independent sequences advance by one token each and share every weight pass.
// Included by prefill_bf16.cu inside namespace mk { namespace { (it reuses that file's row-wise kernels).
//
// The reference has no batch dimension in any op (megakernel/torch_bindings.cpp:569-675 are all batch 1); the
// batched step keeps the reference's per-sequence state layouts and puts a leading batch dimension on them:
//   tokens int32 [B], positions int32 [B] (each sequence has its own length),
//   fa_k_cache / fa_v_cache bf16 [B][n_fa][2][max_seq][256], dn_states f32 [B][n_dn][16][128][128],
//   conv_bufs f32 [B][n_dn][6144][4].
// Row-wise work (norms, projections as tcgen05 GEMMs with M = B, gates, SwiGLU) treats the batch as B rows; the
// kernels below do the per-sequence work: conv window, recurrent state update, attention over each sequence's own
// cache, and the LM head with one argmax per sequence.  Rounding points are those of the prompt path.

constexpr int BATCH_MAX = 16;

// Causal conv1d (window of four inputs) + SiLU + L2 norms for the new token of every sequence, and the shifted
// window written back.  Block = (sequence, head), thread c = channel c of q, k and v of that head.
// Same arithmetic as k_dn_preproject at t = 0 followed by k_dn_conv_state with S = 1.
__global__ void k_dnb_conv(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ conv_w,
                           float* __restrict__ conv_state, size_t seq_stride, float* __restrict__ pre, float* __restrict__ kq) {
    pdl_enter();
    const int b = blockIdx.x, h = blockIdx.y, c = threadIdx.x;
    float* cs = conv_state + (size_t)b * seq_stride;
    __shared__ float red[3][4];
    float val[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        const int ch = r * DN_QK + h * DN_KEY + c;
        const uint2 wr = __ldg(reinterpret_cast<const uint2*>(conv_w) + ch);
        const float w4[4] = {bf_lo(wr.x), bf_hi(wr.x), bf_lo(wr.y), bf_hi(wr.y)};
        const float4 old = *reinterpret_cast<const float4*>(cs + ch * 4);
        const float x[4] = {old.y, old.z, old.w, ld_bf(qkv + (size_t)b * DN_CONV_CH + ch)};
        float co = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) co += x[k] * w4[k];
        val[r] = silu_f(co);
        *reinterpret_cast<float4*>(cs + ch * 4) = make_float4(x[0], x[1], x[2], x[3]);
    }
    float sq = warp_sum(val[0] * val[0]), sk = warp_sum(val[1] * val[1]), sqk = warp_sum(val[0] * val[1]);
    if ((c & 31) == 0) { red[0][c >> 5] = sq; red[1][c >> 5] = sk; red[2][c >> 5] = sqk; }
    __syncthreads();
    sq = red[0][0] + red[0][1] + red[0][2] + red[0][3];
    sk = red[1][0] + red[1][1] + red[1][2] + red[1][3];
    sqk = red[2][0] + red[2][1] + red[2][2] + red[2][3];
    const float qn = rsqrtf(sq + 1e-6f) * 0.08838834764831845f, kn = rsqrtf(sk + 1e-6f);
    float* dst = pre + (size_t)b * DN_CONV_CH + h * DN_KEY + c;
    dst[0] = val[0] * qn;
    dst[DN_QK] = val[1] * kn;
    dst[2 * DN_QK] = val[2];
    if (c == 0) kq[(b * 16 + h) * 4 + 2] = sqk * qn * kn;
}

// One gated-delta-rule step per sequence.  Block = (sequence, head, 16 value rows), warp = one value row, lane =
// four keys: the state row is read once, updated and written back (the step is bound by that traffic:
// 2 x 1 MB per sequence and layer).  Arithmetic as one iteration of k_dn_scan.
__global__ void __launch_bounds__(512) k_dnb_step(const float* __restrict__ pre, const float* __restrict__ gates,
                                                  float* __restrict__ state, size_t seq_stride, float* __restrict__ o) {
    pdl_enter();
    const int b = blockIdx.x >> 7, hb = blockIdx.x & 127;
    const int h = hb >> 3, slice = hb & 7;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = slice * 16 + warp;
    float* srow = state + (size_t)b * seq_stride + ((size_t)h * DN_VAL + row) * DN_KEY;
    float4 s = reinterpret_cast<const float4*>(srow)[lane];
    const float* tok = pre + (size_t)b * DN_CONV_CH;
    const float4 q4 = reinterpret_cast<const float4*>(tok + h * DN_KEY)[lane];
    const float4 k4 = reinterpret_cast<const float4*>(tok + DN_QK + h * DN_KEY)[lane];
    const float vj = tok[2 * DN_QK + h * DN_VAL + row];
    const float4 gt = *reinterpret_cast<const float4*>(gates + ((size_t)b * 16 + h) * 4);     // beta, decay, q.k
    float stk = s.x * k4.x + s.y * k4.y + s.z * k4.z + s.w * k4.w;
    float sqv = s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w;
#pragma unroll
    for (int of = 16; of > 0; of >>= 1) {
        stk += __shfl_xor_sync(0xffffffffu, stk, of);
        sqv += __shfl_xor_sync(0xffffffffu, sqv, of);
    }
    const float err = (vj - gt.y * stk) * gt.x;
    s.x = fmaf(s.x, gt.y, k4.x * err); s.y = fmaf(s.y, gt.y, k4.y * err);
    s.z = fmaf(s.z, gt.y, k4.z * err); s.w = fmaf(s.w, gt.y, k4.w * err);
    if (lane == 0) o[(size_t)b * DN_V + h * DN_VAL + row] = gt.y * sqv + err * gt.z;
    reinterpret_cast<float4*>(srow)[lane] = s;
}

// Attention of one new query per sequence over that sequence's cache (positions 0 .. pos[b], the new key and
// value already appended).  Block = (sequence, query head), eight warps stride over the keys four at a time with an
// online softmax each (lane = 8 of the 256 dimensions), then merge through shared memory.
// out[b][head][256] = softmax(q k^T / 16) v * sigmoid(gate), bf16.
__global__ void __launch_bounds__(256) k_fab_attention(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ kc,
                                                       const __nv_bfloat16* __restrict__ vc, size_t seq_stride,
                                                       const int* __restrict__ pos, int max_seq, __nv_bfloat16* __restrict__ out) {
    pdl_enter();
    const int b = blockIdx.x, hq = blockIdx.y, g = hq >> 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = min(max(pos[b], 0), max_seq - 1) + 1;
    const __nv_bfloat16* qrow = qkv + (size_t)b * FA_QKV_ROWS + hq * 2 * FA_HEAD_DIM;
    const __nv_bfloat16* kb = kc + (size_t)b * seq_stride + (size_t)g * max_seq * FA_HEAD_DIM;
    const __nv_bfloat16* vb = vc + (size_t)b * seq_stride + (size_t)g * max_seq * FA_HEAD_DIM;
    float q[8];
    {
        const uint4 u = reinterpret_cast<const uint4*>(qrow)[lane];
        q[0] = bf_lo(u.x); q[1] = bf_hi(u.x); q[2] = bf_lo(u.y); q[3] = bf_hi(u.y);
        q[4] = bf_lo(u.z); q[5] = bf_hi(u.z); q[6] = bf_lo(u.w); q[7] = bf_hi(u.w);
    }
    float m = -INFINITY, l = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j0 = warp; j0 < n; j0 += 32) {
        uint4 ku[4], vu[4];
        float s[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = j0 + 8 * u;
            const bool in = j < n;
            ku[u] = in ? __ldg(reinterpret_cast<const uint4*>(kb + (size_t)j * FA_HEAD_DIM) + lane) : make_uint4(0, 0, 0, 0);
            vu[u] = in ? __ldg(reinterpret_cast<const uint4*>(vb + (size_t)j * FA_HEAD_DIM) + lane) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) s[u] = dot8(ku[u], q, 0.f);
#pragma unroll
        for (int of = 16; of > 0; of >>= 1) {
#pragma unroll
            for (int u = 0; u < 4; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], of);
        }
        float mn = m;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            s[u] = (j0 + 8 * u < n) ? s[u] * 0.0625f : -INFINITY;
            mn = fmaxf(mn, s[u]);
        }
        const float corr = __expf(m - mn);          // first pass: exp(-inf) = 0
        l *= corr;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= corr;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
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
    __shared__ float sm_m[8], sm_l[8];
    __shared__ float sm_acc[8][FA_HEAD_DIM];
    if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
#pragma unroll
    for (int e = 0; e < 8; ++e) sm_acc[warp][lane * 8 + e] = acc[e];
    __syncthreads();
    const int d = threadIdx.x;                       // one output dimension per thread
    float mm = sm_m[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mm = fmaxf(mm, sm_m[w]);
    float tot = 0.f, ov = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
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

struct BatchWs { float *normed_f32 = nullptr, *bval = nullptr; int *bidx = nullptr, *chosen = nullptr; };
BatchWs g_bws[64];

cudaError_t ensure_batch_ws(BatchWs& w) {
    if (w.normed_f32) return cudaSuccess;
    cudaError_t e = cudaMalloc((void**)&w.normed_f32, (size_t)BATCH_MAX * HIDDEN * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&w.bval, (size_t)BATCH_MAX * LM_BLOCKS * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&w.bidx, (size_t)BATCH_MAX * LM_BLOCKS * 4);
    if (e == cudaSuccess) e = cudaMalloc((void**)&w.chosen, BATCH_MAX * 4);
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
    PF_CHECK(ensure_ws(w, B < 64 ? 64 : B), "step workspace");
    PF_CHECK(ensure_batch_ws(bw), "batch workspace");
    static bool attr[64] = {false};
    if (!attr[dev]) {
        PF_CHECK(cudaFuncSetAttribute(k_lm_head_batch<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 16 * 256 * 16), "lm head smem");
        attr[dev] = true;
    }
    typedef __nv_bfloat16 bf;
    auto gemm = [&](const void* A, const void* W, void* C, const void* R, int N, int K, int ldc) {
        gemm_set_small_m_split(true);
        const cudaError_t e = gemm_bf16_tn(A, W, C, R, B, N, K, K, ldc, w.err, stream);
        gemm_set_small_m_split(false);
        return e;
    };
    auto blocks_for_warps = [&](long long nw) { return (unsigned)((nw + 7) / 8); };
    const size_t kv_seq = (size_t)n_fa * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;          // elements per sequence
    const size_t st_seq = (size_t)n_dn * DN_HEADS * DN_VAL * DN_KEY, cv_seq = (size_t)n_dn * DN_CONV_CH * DN_CONV_K;

    launch_pdl(k_embed, B, 128, 0, stream, tokens, (const bf*)embed_weight, w.hidden, B, vocab);
    int dn_idx = 0, fa_idx = 0;
    for (int li = 0; li < num_layers; ++li) {
        LayerView lv;
        const int rc = source(li, lv);
        if (rc != MK_OK) return rc;
        launch_pdl(k_rmsnorm, blocks_for_warps(B), 256, 0, stream, w.hidden, (const bf*)lv.in_norm, w.normed, B);
        if (lv.type == 0) {
            float* state = (float*)dn_states + (size_t)dn_idx * DN_HEADS * DN_VAL * DN_KEY;
            float* cstate = (float*)conv_bufs + (size_t)dn_idx * DN_CONV_CH * DN_CONV_K;
            PF_CHECK(gemm(w.normed, lv.w_qkv, w.wide, nullptr, DN_CONV_CH, HIDDEN, DN_CONV_CH), "gemm qkv");
            PF_CHECK(gemm(w.normed, lv.w_z, w.z, nullptr, DN_V, HIDDEN, DN_V), "gemm z");
            launch_pdl(k_dn_gates_mma, (unsigned)((B + 15) / 16), 128, 0, stream, w.normed, (const bf*)lv.w_b, (const bf*)lv.w_a,
                       (const bf*)lv.a_log, (const bf*)lv.dt_bias, w.beta, B);
            launch_pdl(k_dnb_conv, dim3(B, DN_HEADS), 128, 0, stream, w.wide, (const bf*)lv.conv_w, cstate, cv_seq, w.pre, w.beta);
            launch_pdl(k_dnb_step, (unsigned)(B * 128), 512, 0, stream, w.pre, w.beta, state, st_seq, w.o);
            launch_pdl(k_dn_gated_norm, blocks_for_warps((long long)B * DN_HEADS), 256, 0, stream, w.o, w.z, (const bf*)lv.dn_norm, w.act, B);
            PF_CHECK(gemm(w.act, lv.w_out, w.hidden, w.hidden, HIDDEN, DN_V, HIDDEN), "gemm out");
            ++dn_idx;
        } else {
            bf* kc = (bf*)fa_k_cache + (size_t)fa_idx * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;
            bf* vc = (bf*)fa_v_cache + (size_t)fa_idx * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;
            if (lv.w_faqkv) {
                PF_CHECK(gemm(w.normed, lv.w_faqkv, w.wide, nullptr, FA_QKV_ROWS, HIDDEN, FA_QKV_ROWS), "gemm fa qkv");
            } else {
                PF_CHECK(gemm(w.normed, lv.w_q, w.wide, nullptr, FA_QPROJ, HIDDEN, FA_QKV_ROWS), "gemm q");
                PF_CHECK(gemm(w.normed, lv.w_k, w.wide + FA_QPROJ, nullptr, FA_KV_SIZE, HIDDEN, FA_QKV_ROWS), "gemm k");
                PF_CHECK(gemm(w.normed, lv.w_v, w.wide + FA_QPROJ + FA_KV_SIZE, nullptr, FA_KV_SIZE, HIDDEN, FA_QKV_ROWS), "gemm v");
            }
            launch_pdl(k_fa_norm_rope, blocks_for_warps((long long)B * 12), 256, 0, stream, w.wide, (const bf*)lv.q_norm,
                       (const bf*)lv.k_norm, kc, vc, B, max_seq_len, positions, kv_seq);
            launch_pdl(k_fab_attention, dim3(B, FA_Q_HEADS), 256, 0, stream, (const bf*)w.wide, (const bf*)kc, (const bf*)vc, kv_seq,
                       positions, max_seq_len, w.act);
            PF_CHECK(gemm(w.act, lv.w_o, w.hidden, w.hidden, HIDDEN, FA_Q_SIZE, HIDDEN), "gemm o");
            ++fa_idx;
        }
        launch_pdl(k_rmsnorm, blocks_for_warps(B), 256, 0, stream, w.hidden, (const bf*)lv.post_norm, w.normed, B);
        if (lv.w_gateup) {
            PF_CHECK(gemm(w.normed, lv.w_gateup, w.wide, nullptr, 2 * INTER, HIDDEN, 2 * INTER), "gemm gate_up");
        } else {
            PF_CHECK(gemm(w.normed, lv.w_gate, w.wide, nullptr, INTER, HIDDEN, 2 * INTER), "gemm gate");
            PF_CHECK(gemm(w.normed, lv.w_up, w.wide + INTER, nullptr, INTER, HIDDEN, 2 * INTER), "gemm up");
        }
        launch_pdl(k_silu_mul, (unsigned)(((size_t)B * (INTER / 8) + 255) / 256), 256, 0, stream, w.wide, w.act, B);
        PF_CHECK(gemm(w.act, lv.w_down, w.hidden, w.hidden, HIDDEN, INTER, HIDDEN), "gemm down");
    }
    launch_pdl(k_final_norm, B, 512, 0, stream, w.hidden, (const bf*)final_norm_w, bw.normed_f32, (bf*)final_normed, (bf*)hidden_bf16_out);
    if (B <= 8) launch_pdl(k_lm_head_batch<8>, LM_BLOCKS, 256, 8 * 256 * 16, stream, bw.normed_f32, B, (const bf*)lm_head_w, vocab, bw.bval, bw.bidx);
    else launch_pdl(k_lm_head_batch<16>, LM_BLOCKS / 2, 256, 16 * 256 * 16, stream, bw.normed_f32, B, (const bf*)lm_head_w, vocab, bw.bval, bw.bidx);
    launch_pdl(k_lm_reduce, B, 32, 0, stream, bw.bval, bw.bidx, B <= 8 ? LM_BLOCKS : LM_BLOCKS / 2, output_tokens);
    PF_CHECK(cudaGetLastError(), "batched step launch");
    return MK_OK;
}
