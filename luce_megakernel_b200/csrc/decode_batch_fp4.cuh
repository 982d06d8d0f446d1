// Batched decode step on the NVFP4 format with a per-tensor scale (e2m1 in 16-element blocks, E4M3 block scales in
// plain rows, fp32 scale per matrix).  Included by prefill_bf16.cu after decode_batch.cuh, inside namespace mk { namespace {.
//
// Same kernel sequence and the same fragment scheme as the bf16 step (decode_batch.cuh): a lane that read 16 contiguous
// bytes of a bf16 weight row (8 weights) now reads the 4 bytes that hold the same 8 weights, plus the E4M3 scale of
// their block; byte permutes turn the codes into f16 (mk_common.cuh), one half-precision multiply applies the block
// scale exactly, the products go through mma.sync m16n8k16 in f16 with f32 accumulation and the matrix's fp32 scale
// multiplies the finished sums.  Activations are the bf16-rounded values of the bf16 step, held as f16 (exact).
// beta / alpha projections, norms, conv stay bf16 and use the bf16 kernels.  No counterpart in the reference (all of
// its ops are batch 1, megakernel/torch_bindings.cpp:569-675, and its NVFP4 decode has no tensor scale).

struct Fp4Mat { const uint8_t* packed; const uint8_t* scales; const float* ts; };     // [N][K/2], [N][K/16], scalar
struct SkinnySegFp4 { Fp4Mat W, W2; void* C; int N; int ldc; int kind; };             // kind 0: bf16 out; 2: SwiGLU pair (W gate, W2 up)
struct SkinnyArgsFp4 { SkinnySegFp4 seg[3]; int nseg; };

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3]) : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// eight bf16 values (one uint4) -> the same values as f16 (exact unless below 6e-8 in magnitude)
__device__ __forceinline__ uint4 bf16x8_to_f16x8(const uint4& u) {
    const uint32_t q[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __half2 h = __floats2half2_rn(bf_lo(q[e]), bf_hi(q[e]));
        o[e] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// rmsnorm_row with the result (rounded to bf16 first, like the bf16 step) stored as f16
__device__ __forceinline__ void rmsnorm_row_f16(const uint4* __restrict__ src, const __nv_bfloat16* __restrict__ w, uint4* dst, int lane) {
    float v[32];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 u = src[i * 32 + lane];
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) { v[i * 8 + 2 * e] = bf_lo(q[e]); v[i * 8 + 2 * e + 1] = bf_hi(q[e]); }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss * (1.0f / HIDDEN) + RMS_EPS);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 wu = __ldg(reinterpret_cast<const uint4*>(w) + i * 32 + lane);
        const uint32_t wq[4] = {wu.x, wu.y, wu.z, wu.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __half2 p = __floats2half2_rn(round_bf16(v[i * 8 + 2 * e] * rstd * (1.0f + bf_lo(wq[e]))),
                                                round_bf16(v[i * 8 + 2 * e + 1] * rstd * (1.0f + bf_hi(wq[e]))));
            o[e] = *reinterpret_cast<const uint32_t*>(&p);
        }
        dst[i * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// One MMA pair for 8 weights per row: codes of rows g (w_lo) and g + 8 (w_hi; 0 = no second row), their block scales,
// and the 8 activations of n8-tile column g (bb).
__device__ __forceinline__ void fp4_mma_pair(float (&acc)[4], uint32_t w_lo, uint32_t w_hi, __half2 s_lo, __half2 s_hi, const uint4& bb) {
    uint32_t ra[4], rb[4];
    e2m1x8_to_f16x2x4(w_lo, ra);
    e2m1x8_to_f16x2x4(w_hi, rb);
    mma_f16(acc, hmul2_bits(ra[0], s_lo), hmul2_bits(rb[0], s_hi), hmul2_bits(ra[1], s_lo), hmul2_bits(rb[1], s_hi), bb.x, bb.y);
    mma_f16(acc, hmul2_bits(ra[2], s_lo), hmul2_bits(rb[2], s_hi), hmul2_bits(ra[3], s_lo), hmul2_bits(rb[3], s_hi), bb.z, bb.w);
}

// Projections that read the residual stream (K = 1024), FP4 weights: k_skinny_norm's scheme.  One CTA per 16 rows of
// a segment (or 8 gate + 8 up rows of a SwiGLU pair), eight warps split K, everything a lane needs of W is requested
// before the dependency wait.
template <int NT>
__global__ void __launch_bounds__(256, 3) k_skinny_norm_fp4(const __nv_bfloat16* __restrict__ A, const __nv_bfloat16* __restrict__ norm_w,
                                                            int B, SkinnyArgsFp4 args) {
    pdl_launch_next();
    constexpr int K = HIDDEN, RS = K / 8 + 4;
    extern __shared__ __align__(16) uint4 as[];              // [NT * 8][RS] normalised activations as f16, rows >= B zero
    __shared__ float red[8][NT * 8][17];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const bool pair = args.seg[0].kind == 2;
    const int rows = pair ? 8 : 16;
    int grp = blockIdx.x, si = 0;
    while (si + 1 < args.nseg && grp >= args.seg[si].N / rows) { grp -= args.seg[si].N / rows; ++si; }
    const SkinnySegFp4& sg = args.seg[si];
    const int n0 = grp * rows;
    const Fp4Mat& m1 = pair ? sg.W2 : sg.W;
    const int r1 = pair ? n0 + g : n0 + g + 8;
    const uint32_t* p0 = reinterpret_cast<const uint32_t*>(sg.W.packed + (size_t)(n0 + g) * (K / 2)) + tig;
    const uint32_t* p1 = reinterpret_cast<const uint32_t*>(m1.packed + (size_t)r1 * (K / 2)) + tig;
    const unsigned short* s0 = reinterpret_cast<const unsigned short*>(sg.W.scales + (size_t)(n0 + g) * (K / 16));
    const unsigned short* s1 = reinterpret_cast<const unsigned short*>(m1.scales + (size_t)r1 * (K / 16));
    uint32_t lo[4], hi[4];
    unsigned short slo[4], shi[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        lo[u] = __ldcs(p0 + (warp + 8 * u) * 4); hi[u] = __ldcs(p1 + (warp + 8 * u) * 4);
        slo[u] = __ldg(s0 + warp + 8 * u); shi[u] = __ldg(s1 + warp + 8 * u);
    }
    const float t0 = __ldg(sg.W.ts) * TS_SCALE_FOLD, t1 = __ldg(m1.ts) * TS_SCALE_FOLD;
    pdl_wait_prior();
    for (int b = warp; b < NT * 8; b += 8) {
        if (b < B) rmsnorm_row_f16(reinterpret_cast<const uint4*>(A + (size_t)b * K), norm_w, as + b * RS, lane);
        else { for (int i = lane; i < K / 8; i += 32) as[b * RS + i] = make_uint4(0, 0, 0, 0); }
    }
    __syncthreads();
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) { acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f; }
    const int sh = (tig >> 1) * 8;                           // a lane's 8 weights lie in block 2 (warp + 8 u) + (tig >> 1) of the row
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const __half2 h0 = e4m3_to_h2_div256((uint32_t)slo[u] >> sh), h1 = e4m3_to_h2_div256((uint32_t)shi[u] >> sh);
#pragma unroll
        for (int t = 0; t < NT; ++t) fp4_mma_pair(acc[t], lo[u], hi[u], h0, h1, as[(t * 8 + g) * RS + (warp + 8 * u) * 4 + tig]);
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
                const float gv = round_bf16(gsum * t0), uv = round_bf16(usum * t1);
                reinterpret_cast<__nv_bfloat16*>(sg.C)[(size_t)b * sg.ldc + n0 + n] = __float2bfloat16_rn(silu_f(gv) * uv);
            }
        } else {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) v += red[w][b][n];
            reinterpret_cast<__nv_bfloat16*>(sg.C)[(size_t)b * sg.ldc + n0 + n] = __float2bfloat16_rn(v * t0);
        }
    }
}

// The 1024-row projections back into the residual stream (K = 2048 or 3584), FP4 weights: k_skinny_res's scheme.
template <int NT, int STEPS>   // K = 256 * STEPS
__global__ void __launch_bounds__(256, 2) k_skinny_res_fp4(const __nv_bfloat16* __restrict__ A, int B, Fp4Mat W, __nv_bfloat16* C, int ldc,
                                                           int* __restrict__ err) {
    pdl_launch_next();
    constexpr int K = 256 * STEPS, RS = K / 8 + 4;
    extern __shared__ __align__(16) uint4 as[];              // [NT * 8][RS] activations (bf16 on arrival, f16 after the conversion pass)
    __shared__ float red[8][NT * 8][9];
    __shared__ __align__(8) unsigned long long bar_mem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int n0 = blockIdx.x * 8;
    const uint32_t* p0 = reinterpret_cast<const uint32_t*>(W.packed + (size_t)(n0 + g) * (K / 2)) + tig;
    const unsigned short* s0 = reinterpret_cast<const unsigned short*>(W.scales + (size_t)(n0 + g) * (K / 16));
    uint32_t lo[STEPS];
    unsigned short slo[STEPS];
#pragma unroll
    for (int u = 0; u < STEPS; ++u) { lo[u] = __ldcs(p0 + (warp + 8 * u) * 4); slo[u] = __ldg(s0 + warp + 8 * u); }
    const float ts = __ldg(W.ts) * TS_SCALE_FOLD;
    const uint32_t bar = smem_u32(&bar_mem);
    if (threadIdx.x == 0) { mbar_init(bar, 1); fence_mbar_init(); }
    for (int i = threadIdx.x; i < (NT * 8 - B) * (K / 8); i += 256) {
        const int b = B + i / (K / 8), c = i % (K / 8);
        as[b * RS + c] = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
    pdl_wait_prior();
    if (threadIdx.x == 0) {
        mbar_expect_tx(bar, (uint32_t)B * K * 2);
        const uint64_t pol = l2_policy_evict_last();
        for (int b = 0; b < B; ++b) bulk_g2s(smem_u32(as + b * RS), A + (size_t)b * K, K * 2, bar, pol);
    }
    if (!mbar_wait(bar, 0) && threadIdx.x == 0) *err = 5;
    for (int i = threadIdx.x; i < B * (K / 8); i += 256) {   // bf16 -> f16 in place
        const int b = i / (K / 8), c = i % (K / 8);
        as[b * RS + c] = bf16x8_to_f16x8(as[b * RS + c]);
    }
    __syncthreads();
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) { acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f; }
    const int sh = (tig >> 1) * 8;
    const __half2 hz = e4m3_to_h2_div256(0u);
#pragma unroll
    for (int u = 0; u < STEPS; ++u) {
        const __half2 h0 = e4m3_to_h2_div256((uint32_t)slo[u] >> sh);
#pragma unroll
        for (int t = 0; t < NT; ++t) fp4_mma_pair(acc[t], lo[u], 0u, h0, hz, as[(t * 8 + g) * RS + (warp + 8 * u) * 4 + tig]);
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) { red[warp][t * 8 + 2 * tig][g] = acc[t][0]; red[warp][t * 8 + 2 * tig + 1][g] = acc[t][1]; }
    __syncthreads();
    const int b = threadIdx.x >> 3, n = threadIdx.x & 7;
    if (threadIdx.x < NT * 8 * 8 && b < B) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += red[w][b][n];
        const size_t o = (size_t)b * ldc + n0 + n;
        C[o] = __float2bfloat16_rn(v * ts + ld_bf(C + o));
    }
}

template <int NT, int STEPS>
inline cudaError_t launch_skinny_res_fp4(const void* A, int B, const Fp4Mat& W, void* C, int N, int ldc, int* err, cudaStream_t stream) {
    constexpr size_t smem = (size_t)NT * 8 * (256 * STEPS / 8 + 4) * 16;
    static bool attr[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(k_skinny_res_fp4<NT, STEPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    return launch_pdl(k_skinny_res_fp4<NT, STEPS>, N / 8, 256, smem, stream, (const __nv_bfloat16*)A, B, W, (__nv_bfloat16*)C, ldc, err);
}

inline cudaError_t skinny_res_fp4(const void* A, int B, int K, const Fp4Mat& W, void* C, int N, int ldc, int* err, cudaStream_t stream) {
    if (B < 1 || B > 16 || N % 8 || (K != 2048 && K != 3584) || !err) return cudaErrorInvalidValue;
    if (B <= 8) return K == 2048 ? launch_skinny_res_fp4<1, 8>(A, B, W, C, N, ldc, err, stream) : launch_skinny_res_fp4<1, 14>(A, B, W, C, N, ldc, err, stream);
    return K == 2048 ? launch_skinny_res_fp4<2, 8>(A, B, W, C, N, ldc, err, stream) : launch_skinny_res_fp4<2, 14>(A, B, W, C, N, ldc, err, stream);
}

inline cudaError_t skinny_norm_fp4(const void* A, const void* norm_w, int B, const SkinnyArgsFp4& args, cudaStream_t stream) {
    const bool pair = args.seg[0].kind == 2;
    if (pair && args.nseg != 1) return cudaErrorInvalidValue;
    int ctas = 0;
    for (int i = 0; i < args.nseg; ++i) {
        if (args.seg[i].N % 16) return cudaErrorInvalidValue;
        ctas += args.seg[i].N / (pair ? 8 : 16);
    }
    static bool attr[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_skinny_norm_fp4<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 16 * (HIDDEN / 8 + 4) * 16);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_skinny_norm_fp4<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 16 * (HIDDEN / 8 + 4) * 16);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    const int nt = B <= 8 ? 1 : 2;
    const size_t sm = (size_t)nt * 8 * (HIDDEN / 8 + 4) * 16;
    if (nt == 1) return launch_pdl(k_skinny_norm_fp4<1>, ctas, 256, sm, stream, (const __nv_bfloat16*)A, (const __nv_bfloat16*)norm_w, B, args);
    return launch_pdl(k_skinny_norm_fp4<2>, ctas, 256, sm, stream, (const __nv_bfloat16*)A, (const __nv_bfloat16*)norm_w, B, args);
}

// LM head of a batched step, FP4 weights: k_lm_head_mma's scheme (a warp keeps a 16-row group of the vocabulary over
// all of K, activations as two f16 terms hi + lo, running argmax per sequence, lowest index on ties).
template <int NT>
__global__ void __launch_bounds__(256, 2) k_lm_head_mma_fp4(const float* __restrict__ x, int B, Fp4Mat W, int vocab,
                                                            float* __restrict__ bval, int* __restrict__ bidx) {
    pdl_launch_next();
    constexpr int RS = HIDDEN / 8 + 4;
    extern __shared__ __align__(16) uint4 xh[];               // hi [NT * 8][RS], then lo [NT * 8][RS]
    __shared__ float sv[8][NT * 8];
    __shared__ int si[8][NT * 8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int ngroups = (vocab + 15) / 16, nwarps = gridDim.x * 8, wg = blockIdx.x * 8 + warp;
    const int mine = wg < ngroups ? (ngroups - wg + nwarps - 1) / nwarps : 0;
    constexpr int FG = HIDDEN / 32 / 4;                       // fetches of four k steps per group: 8
    uint32_t lo[4], hi[4];
    unsigned short slo[4], shi[4];
    auto fetch = [&](int q) {
        const int n0 = (wg + (q / FG) * nwarps) * 16, st0 = (q % FG) * 4;
        const size_t ra = (size_t)min(n0 + g, vocab - 1), rb = (size_t)min(n0 + g + 8, vocab - 1);
        const uint32_t* w0 = reinterpret_cast<const uint32_t*>(W.packed + ra * (HIDDEN / 2)) + tig;
        const uint32_t* w1 = reinterpret_cast<const uint32_t*>(W.packed + rb * (HIDDEN / 2)) + tig;
        const unsigned short* s0 = reinterpret_cast<const unsigned short*>(W.scales + ra * (HIDDEN / 16));
        const unsigned short* s1 = reinterpret_cast<const unsigned short*>(W.scales + rb * (HIDDEN / 16));
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            lo[u] = __ldcs(w0 + (st0 + u) * 4); hi[u] = __ldcs(w1 + (st0 + u) * 4);
            slo[u] = __ldg(s0 + st0 + u); shi[u] = __ldg(s1 + st0 + u);
        }
    };
    if (mine > 0) fetch(0);
    const float ts = __ldg(W.ts) * TS_SCALE_FOLD;
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
                const __half2 hh = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
                const __half2 ll = __floats2half2_rn(v[2 * e] - __low2float(hh), v[2 * e + 1] - __high2float(hh));
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
    const int sh = (tig >> 1) * 8;
    for (int q = 0; q < mine * FG; ++q) {
        const int st0 = (q % FG) * 4;
        if (st0 == 0) {
#pragma unroll
            for (int t = 0; t < NT; ++t) { acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f; }
        }
        uint32_t clo[4], chi[4];
        unsigned short cs0[4], cs1[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) { clo[u] = lo[u]; chi[u] = hi[u]; cs0[u] = slo[u]; cs1[u] = shi[u]; }
        if (q + 1 < mine * FG) fetch(q + 1);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const __half2 h0 = e4m3_to_h2_div256((uint32_t)cs0[u] >> sh), h1 = e4m3_to_h2_div256((uint32_t)cs1[u] >> sh);
            uint32_t ra[4], rb[4];
            e2m1x8_to_f16x2x4(clo[u], ra);
            e2m1x8_to_f16x2x4(chi[u], rb);
            const uint32_t a0 = hmul2_bits(ra[0], h0), a1 = hmul2_bits(rb[0], h1), a2 = hmul2_bits(ra[1], h0), a3 = hmul2_bits(rb[1], h1);
            const uint32_t c0 = hmul2_bits(ra[2], h0), c1 = hmul2_bits(rb[2], h1), c2 = hmul2_bits(ra[3], h0), c3 = hmul2_bits(rb[3], h1);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int off = (t * 8 + g) * RS + (st0 + u) * 4 + tig;
                const uint4 bh = xh[off], bl = xlo[off];
                mma_f16(acc[t], a0, a1, a2, a3, bh.x, bh.y);
                mma_f16(acc[t], c0, c1, c2, c3, bh.z, bh.w);
                mma_f16(acc[t], a0, a1, a2, a3, bl.x, bl.y);
                mma_f16(acc[t], c0, c1, c2, c3, bl.z, bl.w);
            }
        }
        if (st0 == (FG - 1) * 4) {
            const int n0 = (wg + (q / FG) * nwarps) * 16;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int r0 = n0 + g, r1 = n0 + g + 8;
                    float v = r0 < vocab ? acc[t][c] * ts : -INFINITY;
                    int ix = r0;
                    const float v1 = r1 < vocab ? acc[t][2 + c] * ts : -INFINITY;
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

// Host view of one entry of the 224-byte table
struct LayerViewFp4 {
    int type;
    const void *in_norm, *post_norm, *w_b, *w_a, *conv_w, *a_log, *dt_bias, *dn_norm, *q_norm, *k_norm;
    Fp4Mat qkv, z, out, q, k, v, o, gate, up, down;
};
inline Fp4Mat fp4_mat(const void* const* p) {
    return Fp4Mat{(const uint8_t*)p[0], (const uint8_t*)p[1], (const float*)p[2]};
}
inline LayerViewFp4 view_of_fp4(const LayerWeightsNVFP4TS& e) {
    LayerViewFp4 v{};
    v.type = e.layer_type;
    const void* const* p = e.ptrs;
    if (e.layer_type == 0) {
        v.in_norm = p[0]; v.qkv = fp4_mat(p + 1); v.z = fp4_mat(p + 4); v.w_b = p[7]; v.w_a = p[8]; v.conv_w = p[9]; v.a_log = p[10];
        v.dt_bias = p[11]; v.dn_norm = p[12]; v.out = fp4_mat(p + 13); v.post_norm = p[16]; v.gate = fp4_mat(p + 17);
        v.up = fp4_mat(p + 20); v.down = fp4_mat(p + 23);
    } else {
        v.in_norm = p[0]; v.q = fp4_mat(p + 1); v.k = fp4_mat(p + 4); v.v = fp4_mat(p + 7); v.q_norm = p[10]; v.k_norm = p[11];
        v.o = fp4_mat(p + 12); v.post_norm = p[15]; v.gate = fp4_mat(p + 16); v.up = fp4_mat(p + 19); v.down = fp4_mat(p + 22);
    }
    return v;
}

// One step for B sequences on the tensor-scale NVFP4 weights; same kernel sequence as decode_batch_core (one more
// launch per DeltaNet layer: the bf16 beta / alpha projections).
inline int decode_batch_core_fp4(const int* tokens, const int* positions, int* output_tokens, int B, const void* embed_weight,
                                 const LayerWeightsNVFP4TS* host_layers, int num_layers, int n_fa, int n_dn, const void* final_norm_w,
                                 const Fp4Mat& lm, void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
                                 void* final_normed, void* hidden_bf16_out, int max_seq_len, int vocab, int dev, cudaStream_t stream) {
    PrefillWs& w = g_pws[dev];
    BatchWs& bw = g_bws[dev];
    PF_CHECK(ensure_ws(w, B < 64 ? 64 : B, stream, true), "step workspace (grow it with mk_prefill_reserve() before capturing a graph)");
    PF_CHECK(ensure_batch_ws(bw), "batch workspace");
    static bool attr[64] = {false};
    if (!attr[dev]) {
        PF_CHECK(cudaFuncSetAttribute(k_lm_head_mma_fp4<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * 8 * (HIDDEN / 8 + 4) * 16), "lm head smem");
        attr[dev] = true;
    }
    typedef __nv_bfloat16 bf;
    auto blocks_for_warps = [&](long long nw) { return (unsigned)((nw + 7) / 8); };
    const size_t kv_seq = (size_t)n_fa * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;
    const size_t st_seq = (size_t)n_dn * DN_HEADS * DN_VAL * DN_KEY, cv_seq = (size_t)n_dn * DN_CONV_CH * DN_CONV_K;
    launch_pdl(k_embed, B, 128, 0, stream, tokens, (const bf*)embed_weight, w.hidden, B, vocab);
    int dn_idx = 0, fa_idx = 0;
    for (int li = 0; li < num_layers; ++li) {
        const LayerViewFp4 lv = view_of_fp4(host_layers[li]);
        if (lv.type == 0) {
            float* state = (float*)dn_states + (size_t)dn_idx * DN_HEADS * DN_VAL * DN_KEY;
            float* cstate = (float*)conv_bufs + (size_t)dn_idx * DN_CONV_CH * DN_CONV_K;
            SkinnyArgsFp4 a;
            a.nseg = 2;
            a.seg[0] = SkinnySegFp4{lv.qkv, Fp4Mat{}, w.wide, DN_CONV_CH, DN_CONV_CH, 0};
            a.seg[1] = SkinnySegFp4{lv.z, Fp4Mat{}, w.z, DN_V, DN_V, 0};
            PF_CHECK(skinny_norm_fp4(w.hidden, lv.in_norm, B, a, stream), "DeltaNet input projections");
            SkinnyArgs g2;
            g2.nseg = 2;
            g2.seg[0] = SkinnySeg{(const bf*)lv.w_b, nullptr, bw.graw, nullptr, 16, 32, 1};
            g2.seg[1] = SkinnySeg{(const bf*)lv.w_a, nullptr, bw.graw + 16, nullptr, 16, 32, 1};
            PF_CHECK(skinny_proj(w.hidden, lv.in_norm, B, HIDDEN, HIDDEN, g2, stream), "beta / alpha projections");
            launch_pdl(k_dnb_layer, dim3(B, DN_HEADS), 512, 0, stream, (const bf*)w.wide, (const bf*)w.z, (const float*)bw.graw,
                       (const bf*)lv.conv_w, (const bf*)lv.a_log, (const bf*)lv.dt_bias, (const bf*)lv.dn_norm, cstate, cv_seq, state,
                       st_seq, w.act);
            PF_CHECK(skinny_res_fp4(w.act, B, DN_V, lv.out, w.hidden, HIDDEN, HIDDEN, w.err, stream), "out projection");
            ++dn_idx;
        } else {
            bf* kc = (bf*)fa_k_cache + (size_t)fa_idx * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;
            bf* vc = (bf*)fa_v_cache + (size_t)fa_idx * FA_KV_HEADS * max_seq_len * FA_HEAD_DIM;
            SkinnyArgsFp4 a;
            a.nseg = 3;
            a.seg[0] = SkinnySegFp4{lv.q, Fp4Mat{}, w.wide, FA_QPROJ, FA_QKV_ROWS, 0};
            a.seg[1] = SkinnySegFp4{lv.k, Fp4Mat{}, w.wide + FA_QPROJ, FA_KV_SIZE, FA_QKV_ROWS, 0};
            a.seg[2] = SkinnySegFp4{lv.v, Fp4Mat{}, w.wide + FA_QPROJ + FA_KV_SIZE, FA_KV_SIZE, FA_QKV_ROWS, 0};
            PF_CHECK(skinny_norm_fp4(w.hidden, lv.in_norm, B, a, stream), "q, k, v projections");
            launch_pdl(k_fa_norm_rope, blocks_for_warps((long long)B * 12), 256, 0, stream, w.wide, (const bf*)lv.q_norm,
                       (const bf*)lv.k_norm, kc, vc, B, max_seq_len, positions, kv_seq);
            launch_pdl(k_fab_attention, dim3(B, FA_Q_HEADS), FAB_WARPS * 32, 0, stream, (const bf*)w.wide, (const bf*)kc, (const bf*)vc, kv_seq,
                       positions, max_seq_len, w.act);
            PF_CHECK(skinny_res_fp4(w.act, B, FA_Q_SIZE, lv.o, w.hidden, HIDDEN, HIDDEN, w.err, stream), "o projection");
            ++fa_idx;
        }
        SkinnyArgsFp4 gu;
        gu.nseg = 1;
        gu.seg[0] = SkinnySegFp4{lv.gate, lv.up, w.act, INTER, INTER, 2};
        PF_CHECK(skinny_norm_fp4(w.hidden, lv.post_norm, B, gu, stream), "gate and up projections");
        PF_CHECK(skinny_res_fp4(w.act, B, INTER, lv.down, w.hidden, HIDDEN, HIDDEN, w.err, stream), "down projection");
    }
    launch_pdl(k_final_norm, B, 512, 0, stream, w.hidden, (const bf*)final_norm_w, bw.normed_f32, (bf*)final_normed, (bf*)hidden_bf16_out);
    constexpr int LMB = 296;
    constexpr int LM_SMEM1 = 2 * 8 * (HIDDEN / 8 + 4) * 16, LM_SMEM2 = 2 * LM_SMEM1;
    if (B <= 8) launch_pdl(k_lm_head_mma_fp4<1>, LMB, 256, LM_SMEM1, stream, (const float*)bw.normed_f32, B, lm, vocab, bw.bval, bw.bidx);
    else launch_pdl(k_lm_head_mma_fp4<2>, LMB, 256, LM_SMEM2, stream, (const float*)bw.normed_f32, B, lm, vocab, bw.bval, bw.bidx);
    launch_pdl(k_lm_reduce, B, 32, 0, stream, bw.bval, bw.bidx, LMB, output_tokens);
    PF_CHECK(cudaGetLastError(), "batched step launch");
    return MK_OK;
}
