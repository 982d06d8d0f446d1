// Device code of the decode megakernel.  Included twice by decode_bf16.cu, once per value of
// MK_TRACE, inside a namespace of its own: the timeline stamps cost instruction-cache space, so
// the variant without them is the one that normally runs.
// ---- weight format of this variant -----------------------------------------------------------
// MK_WFMT 0: bf16 rows of K*2 bytes, contiguous in the ring stage.
// MK_WFMT 1: NVFP4 layer weights: packed rows of K/2 bytes placed at a stride of K/2+16 bytes (so
//            that the 8 rows a quarter-warp reads hit different banks), followed by the fp16 group
//            scales of the chunk's rows (K/16 bytes per row); lanes 0-15 of the producer issue the
//            data rows, lanes 16-31 the scale rows.  beta / alpha projections stay bf16 and are
//            computed outside the ring; the LM head uses the 16-block E4M3 format.
#if MK_WFMT == 0
typedef LayerWeights LW;
constexpr int NSTAGE = 6;                               // ring stages
constexpr int STAGE_BYTES = 32768;
constexpr int IN_ROWS_DN = DN_IN_ROWS;                  // qkv | z | beta | alpha
constexpr int LM_RPC = 16;                              // LM-head rows per ring chunk
__device__ __forceinline__ constexpr int row_bytes(int K) { return K * 2; }
__device__ __forceinline__ constexpr int row_stride(int K) { return K * 2; }
#elif MK_WFMT == 1
typedef LayerWeightsNVFP4 LW;
constexpr int NSTAGE = 6;
constexpr int STAGE_BYTES = 32768;
// slots of the NVFP4 table: a quantised matrix takes (data, scales) (reference: megakernel/model_nvfp4.py:274-311)
enum { DN_IN_NORM = 0, DN_W_QKV = 1, DN_W_Z = 3, DN_W_B = 5, DN_W_A = 6, DN_CONV_W = 7, DN_A_LOG = 8, DN_DT_BIAS = 9,
       DN_NORM_W = 10, DN_W_OUT = 11, DN_POST_NORM = 13, DN_W_GATE = 14, DN_W_UP = 16, DN_W_DOWN = 18 };
enum { FA_IN_NORM = 0, FA_W_Q = 1, FA_W_K = 3, FA_W_V = 5, FA_Q_NORM = 7, FA_K_NORM = 8, FA_W_O = 9, FA_POST_NORM = 11,
       FA_W_GATE = 12, FA_W_UP = 14, FA_W_DOWN = 16 };
constexpr int IN_ROWS_DN = DN_CONV_CH + DN_V;           // qkv | z
constexpr int LM_RPC = 64;
__device__ __forceinline__ constexpr int row_bytes(int K) { return K / 2; }
__device__ __forceinline__ constexpr int row_stride(int K) { return K / 2 + 16; }
__device__ __forceinline__ constexpr int scale_bytes(int K) { return K / 16; }
#else
// MK_WFMT 2: e2m1 values in 16-element blocks, E4M3 block scales stored row-major ([rows][K/16] bytes), an fp32 scale
// per matrix.  A ring chunk is R consecutive packed rows (R * K/2 bytes, no padding) followed by the R rows of
// block scales (R * K/16 bytes): two bulk copies per matrix the chunk touches.  R = 64 for K = 1024, 32 for
// K = 2048, 16 for K = 3584, so every phase of a layer is ONE chunk per CTA.  The table entry has three slots per
// quantised matrix: packed data, row-major scales, pointer to the tensor scale.
// MK_WFMT 3: the same quantised values, multiplied on the block-scaled 5th-generation tensor cores (tcgen05.mma
// kind::mxf4nvf4, accumulators and block scales in tensor memory).  The table's first slot of every phase's matrix
// group points at an array of per-CTA chunk IMAGES instead of plain rows: image c holds the rows CTA c owns in that
// phase, already in the shared-memory layout the MMA reads (K-major, 128-byte swizzle, 256 values per 128-byte row
// segment, k-tile after k-tile), followed by the rows' block scales in the order tcgen05.cp lays them into tensor
// memory, so that a phase is ONE bulk copy per CTA.  Images are built for a grid of exactly U_CTAS CTAs.  The
// activation vector is the B operand: quantised on the fly into up to eight NVFP4 residual terms (term n+1 encodes
// six times what term n left over), one MMA column each, recombined after the product.
typedef LayerWeightsNVFP4TS LW;
#if MK_WFMT == 3
constexpr int NSTAGE = 4;                               // the attention phase needs four chunks resident at once
constexpr int STAGE_BYTES = 36864;                      // 56 rows of K = 1024: 28 KB of codes + 16 scale units of 512 B
#else
constexpr int NSTAGE = 5;
constexpr int STAGE_BYTES = 36864;                      // 64 rows of K = 1024: 32 KB of codes + 4 KB of scales
#endif
enum { DN_IN_NORM = 0, DN_W_QKV = 1, DN_W_Z = 4, DN_W_B = 7, DN_W_A = 8, DN_CONV_W = 9, DN_A_LOG = 10, DN_DT_BIAS = 11,
       DN_NORM_W = 12, DN_W_OUT = 13, DN_POST_NORM = 16, DN_W_GATE = 17, DN_W_UP = 20, DN_W_DOWN = 23 };
enum { FA_IN_NORM = 0, FA_W_Q = 1, FA_W_K = 4, FA_W_V = 7, FA_Q_NORM = 10, FA_K_NORM = 11, FA_W_O = 12, FA_POST_NORM = 15,
       FA_W_GATE = 16, FA_W_UP = 19, FA_W_DOWN = 22 };
constexpr int IN_ROWS_DN = DN_CONV_CH + DN_V;           // qkv | z (beta / alpha stay bf16, outside the ring)
#if MK_WFMT == 3
constexpr int LM_RPC = 56;                              // LM-head rows per chunk image
constexpr int UP_ROW0 = 28;                             // local row of the first up-projection row in a gate|up chunk
#else
constexpr int LM_RPC = 64;
constexpr int UP_ROW0 = 32;
#endif
__device__ __forceinline__ constexpr int row_bytes(int K) { return K / 2; }
__device__ __forceinline__ constexpr int scale_bytes(int K) { return K / 16; }
__device__ __forceinline__ constexpr int rows_per_chunk(int K) { return K == 1024 ? 64 : (K == 2048 ? 32 : 16); }
#if MK_WFMT == 3
constexpr int U_CTAS = 148;                             // the grid the chunk images are cut for
constexpr int U_OFF_B = NSTAGE * STAGE_BYTES;           // activation terms: 8 rows x K/2 bytes, swizzled like the weights
constexpr int U_B_BYTES = 8 * (INTER / 2);
constexpr int U_OFF_SFB = U_OFF_B + U_B_BYTES;          // their block scales: one 512-byte copy unit per MMA step (64 k)
constexpr int U_SFB_BYTES = (INTER / 64) * 512;
constexpr int U_OFF_BARS = U_OFF_SFB + U_SFB_BYTES;     // barriers: product done [2], accumulator drained [2], activation ready
constexpr int U_OFF_TMEM = U_OFF_BARS + 40;             // tensor-memory base address
constexpr int U_OFF_AMAX = U_OFF_BARS + 64;             // per-warp maxima of the staged activation [16]
static_assert(U_OFF_AMAX + 64 <= RING_BYTES, "tensor-core operands do not fit behind the ring");
// tensor-memory columns: accumulator buffers at 0 and 32 (8 columns each); block scales take four columns per MMA
// step and operand (the unit one tcgen05.cp writes, which is also the alignment the MMA is given): weights from
// column 64, activation from column 288, 56 steps each at most
constexpr uint32_t U_TM_COLS = 512;
constexpr uint32_t U_TM_SFA = 64, U_TM_SFB = 288;
// padded row count of a CTA's chunk per phase, and the image size (codes + scales)
__device__ __forceinline__ constexpr int u_rp(int type) {
    return (type == T_DN_IN || type == T_GATEUP || type == T_LM) ? 56 : type == T_FA_IN ? 40 : 8;
}
__device__ __forceinline__ constexpr int u_k(int type) {           // K of the whole product
    return (type == T_DN_OUT || type == T_FA_OUT) ? 2048 : type == T_DOWN ? INTER : HIDDEN;
}
__device__ __forceinline__ constexpr int u_kc(int type) {          // K of one chunk image: the down projection takes two
    return type == T_DOWN ? INTER / 2 : u_k(type);
}
__device__ __forceinline__ constexpr int u_img_bytes(int type) {
    return u_rp(type) * (u_kc(type) / 2) + (u_kc(type) / 64) * 512;
}
static_assert(u_img_bytes(T_GATEUP) <= STAGE_BYTES && u_img_bytes(T_DOWN) <= STAGE_BYTES && u_img_bytes(T_DN_OUT) <= STAGE_BYTES,
              "image exceeds a ring stage");
#endif
#endif
static_assert(NSTAGE * STAGE_BYTES <= RING_BYTES && NSTAGE <= MAX_STAGES, "ring does not fit its region");

struct Geo {
    int r0, r1;       // rows (or outputs for gate/up, first unit for the recurrence)
    int nchunks;
};

__device__ __forceinline__ void split_rows(int n, int G, int c, int& a, int& b) {
    // n <= 248320 rows (or whatever the vocabulary is) times at most 256 CTAs fits 32 bits
    a = (int)(((unsigned)n * (unsigned)c) / (unsigned)G);
    b = (int)(((unsigned)n * (unsigned)(c + 1)) / (unsigned)G);
}

// attention units: (KV head, chunk of positions); a unit's K and V rows travel through the ring in tiles of
// 64 positions, four ring chunks per tile: K rows 0-31, K rows 32-63, V rows 0-31, V rows 32-63
constexpr int ATT_ROW_STRIDE = FA_HEAD_DIM * 2 + 16;      // (row stride of the query / probability scratch tiles)
// A K or V chunk in a ring stage: 32 positions x 256 dims as four boxes of 64 dims (32 rows x 128 bytes = 4 KB each,
// 128-byte swizzle), the layout cp.async.bulk.tensor writes: 16-byte piece c of row r of a box sits at piece c ^ (r & 7).
// Four tensor copies per chunk instead of one bulk copy per row: a CTA issues a copy only every ~0.1 us, and 128 row
// copies per tile made the tile arrive ~3 us after the attention phase had started.
__device__ __forceinline__ uint32_t att_tile_off(int rr, int bytecol) {
    return (uint32_t)(((bytecol >> 7) << 12) + rr * 128 + ((((bytecol >> 4) & 7) ^ (rr & 7)) << 4));
}
__device__ __forceinline__ int att_num_chunks(int L) {
    int nc = (L + ATT_CHUNK_POS - 1) / ATT_CHUNK_POS;
    return nc < 1 ? 1 : (nc > ATT_MAX_CHUNKS ? ATT_MAX_CHUNKS : nc);
}
__device__ __forceinline__ void att_unit_range(int L, int u, int& g, int& ch, int& p_lo, int& p_hi) {
    const int NC = att_num_chunks(L), per = (L + NC - 1) / NC;
    g = u / NC; ch = u % NC;
    p_lo = ch * per; p_hi = min(L, p_lo + per);
}

__device__ __forceinline__ Geo phase_geo(int type, int cta, int G, int vocab, int pos = 0) {
    Geo g;
    g.r0 = g.r1 = 0;
    g.nchunks = 0;
    switch (type) {
#if MK_WFMT >= 2
        case T_DN_IN:  split_rows(IN_ROWS_DN, G, cta, g.r0, g.r1);  g.nchunks = (g.r1 - g.r0 + 63) >> 6; break;
        case T_FA_IN:  split_rows(FA_QKV_ROWS, G, cta, g.r0, g.r1); g.nchunks = (g.r1 - g.r0 + 63) >> 6; break;
        case T_DN_OUT:
        case T_FA_OUT: split_rows(HIDDEN, G, cta, g.r0, g.r1);      g.nchunks = (g.r1 - g.r0 + 31) >> 5; break;
        case T_GATEUP: split_rows(INTER, G, cta, g.r0, g.r1);       g.nchunks = (g.r1 - g.r0 + 31) >> 5; break;
#if MK_WFMT == 3
        case T_DOWN:   split_rows(HIDDEN, G, cta, g.r0, g.r1);      g.nchunks = 2; break;      // two K halves
#else
        case T_DOWN:   split_rows(HIDDEN, G, cta, g.r0, g.r1);      g.nchunks = (g.r1 - g.r0 + 15) >> 4; break;
#endif
#else
        case T_DN_IN:  split_rows(IN_ROWS_DN, G, cta, g.r0, g.r1);  g.nchunks = (g.r1 - g.r0 + 15) >> 4; break;
        case T_FA_IN:  split_rows(FA_QKV_ROWS, G, cta, g.r0, g.r1); g.nchunks = (g.r1 - g.r0 + 15) >> 4; break;
        case T_DN_OUT:
        case T_FA_OUT: split_rows(HIDDEN, G, cta, g.r0, g.r1);      g.nchunks = (g.r1 - g.r0 + 7) >> 3; break;
        case T_GATEUP: split_rows(INTER, G, cta, g.r0, g.r1);       g.nchunks = (g.r1 - g.r0 + 7) >> 3; break;
        case T_DOWN:   split_rows(HIDDEN, G, cta, g.r0, g.r1);      g.nchunks = (g.r1 - g.r0 + 3) >> 2; break;
#endif
        case T_LM:     split_rows(vocab, G, cta, g.r0, g.r1);       g.nchunks = (g.r1 - g.r0 + LM_RPC - 1) / LM_RPC; break;
        case T_DN_REC: g.r0 = cta; g.nchunks = (cta < 128) ? (128 - cta + G - 1) / G : 0; break;
        case T_FA_ATT: {
            const int L = pos + 1;
            if (cta < FA_KV_HEADS * att_num_chunks(L)) {      // at most one unit per CTA (grids hold >= 129 CTAs)
                int gg, ch, lo, hi;
                att_unit_range(L, cta, gg, ch, lo, hi);
                g.r0 = lo; g.r1 = hi;
                g.nchunks = 4 * ((hi - lo + 63) >> 6);
            }
            break;
        }
        default: break;
    }
    return g;
}

// Source of what producer lane `lane` copies for chunk q: returns bytes (0 = nothing) and the
// ring offset.  bf16: lane = row slot.  NVFP4: lanes 0-15 = packed rows, lanes 16-31 = their scales.
__device__ __forceinline__ uint32_t chunk_slot_src(int type, const LW& lw, const DecodeParams& P,
                                                   const Geo& g, int q, int lane, int G, int dn_idx,
                                                   const char*& src, uint32_t& dst_off, int cta_of_geo, int pos) {
    if (type == T_FA_ATT) return 0;      // attention tiles travel as tensor copies (producer_phase)
#if MK_WFMT >= 2
    if (type == T_DN_REC) {
        if (lane != 0) return 0;
        const int u = g.r0 + q * G;
        const int h = u >> 3, sl = u & 7;
        src = (const char*)(P.dn_states + ((size_t)(dn_idx * DN_HEADS + h) * DN_VAL + sl * 16) * DN_KEY);
        dst_off = 0;
        return 16 * DN_KEY * 4;
    }
#if MK_WFMT == 3
    {
        // one image per CTA and phase (per chunk for the LM head), copied as it lies
        if (lane != 0 || q >= g.nchunks) return 0;
        const bool dn = (lw.layer_type == 0);
        const uint32_t img = (uint32_t)u_img_bytes(type);
        if (type == T_LM) {
            src = (const char*)P.lm_head + ((size_t)cta_of_geo * P.lm_image_chunks + q) * img;
        } else {
            int slot;
            switch (type) {
                case T_DN_IN: slot = DN_W_QKV; break;
                case T_FA_IN: slot = FA_W_Q; break;
                case T_DN_OUT: slot = DN_W_OUT; break;
                case T_FA_OUT: slot = FA_W_O; break;
                case T_GATEUP: slot = dn ? (int)DN_W_GATE : (int)FA_W_GATE; break;
                case T_DOWN: slot = dn ? (int)DN_W_DOWN : (int)FA_W_DOWN; break;
                default: return 0;
            }
            src = (const char*)lw.ptrs[slot] + ((size_t)cta_of_geo * g.nchunks + q) * img;
        }
        dst_off = 0;
        return img;
    }
#else
    {
        // Stage layout: the chunk's R rows of packed codes, contiguous (R * K/2 bytes), then their R rows of block scales.
        // lane = 2 * segment + kind: segment = a matrix the chunk's rows fall into (at most 3; gate / up for the SwiGLU
        // phase), kind 0 = packed rows, 1 = scales.  Few copies per chunk on purpose: a CTA can issue a bulk copy only
        // every ~0.1 us, and an earlier layout with eight padded row groups (17-19 copies per chunk) spent over 2 us
        // per chunk just issuing them; the bank conflicts of the unpadded rows are avoided on the reading side instead.
        const int seg = lane >> 1, kind = lane & 1;
        if (seg >= 3) return 0;
        // matrix segments of the phase's concatenated row space: [0, h0) [h0, h1) [h1, h2), table slots i0 i1 i2
        int K = HIDDEN, nseg = 1, h0 = 0, h1 = 0, h2 = 0, i0 = -1, i1 = -1, i2 = -1;
        const bool dn = (lw.layer_type == 0);
        bool gateup = false;
        switch (type) {
            case T_DN_IN: nseg = 2; i0 = DN_W_QKV; h0 = DN_CONV_CH; i1 = DN_W_Z; h1 = DN_CONV_CH + DN_V; break;
            case T_FA_IN: nseg = 3; i0 = FA_W_Q; h0 = FA_QPROJ; i1 = FA_W_K; h1 = FA_QPROJ + FA_KV_SIZE; i2 = FA_W_V; h2 = FA_QKV_ROWS; break;
            case T_DN_OUT: i0 = DN_W_OUT; K = 2048; h0 = HIDDEN; break;
            case T_FA_OUT: i0 = FA_W_O; K = 2048; h0 = HIDDEN; break;
            case T_GATEUP: gateup = true; nseg = 2; i0 = dn ? (int)DN_W_GATE : (int)FA_W_GATE; i1 = dn ? (int)DN_W_UP : (int)FA_W_UP; break;
            case T_DOWN: i0 = dn ? (int)DN_W_DOWN : (int)FA_W_DOWN; K = INTER; h0 = HIDDEN; break;
            case T_LM: h0 = P.vocab; break;
            default: return 0;
        }
        if (seg >= nseg) return 0;
        const int R = rows_per_chunk(K);
        const uint32_t sc_off = (uint32_t)R * row_bytes(K);
        const char* base;
        if (type == T_LM) base = (const char*)(kind ? P.lm_scales : P.lm_head);
        else base = (const char*)lw.ptrs[(seg == 0 ? i0 : (seg == 1 ? i1 : i2)) + kind];
        const uint32_t unit = kind ? scale_bytes(K) : row_bytes(K);
        const uint32_t region = kind ? sc_off : 0u;
        if (gateup) {
            // outputs [oa, ob) of this chunk: gate rows at stage rows 0.., the matching up rows at stage rows 32..
            const int oa = g.r0 + q * 32, ob = min(g.r1, oa + 32);
            if (ob <= oa) return 0;
            src = base + (size_t)oa * unit;
            dst_off = region + (uint32_t)(seg * 32) * unit;
            return (uint32_t)(ob - oa) * unit;
        }
        const int ra = g.r0 + q * R, rb = min(g.r1, ra + R);
        const int lo_s = seg == 0 ? 0 : (seg == 1 ? h0 : h1), hi_s = seg == 0 ? h0 : (seg == 1 ? h1 : h2);
        const int a = max(ra, lo_s), b = min(rb, hi_s);
        if (b <= a) return 0;
        src = base + (size_t)(a - lo_s) * unit;
        dst_off = region + (uint32_t)(a - ra) * unit;
        return (uint32_t)(b - a) * unit;
    }
#endif   // MK_WFMT == 3
#else
#if MK_WFMT == 0
    const int slot = lane, kind = 0;
#else
    const int slot = lane & 15, kind = lane >> 4;
#endif
    int K = HIDDEN, rpc = 16, idx = -1, rr = 0;     // matrix slot index in the table and row inside it
    switch (type) {
        case T_DN_IN: {
            const int r = g.r0 + q * 16 + slot;
            if (slot >= 16 || r >= g.r1) return 0;
            if (r < DN_CONV_CH) { idx = DN_W_QKV; rr = r; }
            else if (r < DN_CONV_CH + DN_V) { idx = DN_W_Z; rr = r - DN_CONV_CH; }
            else if (r < DN_CONV_CH + DN_V + DN_HEADS) { idx = DN_W_B; rr = r - DN_CONV_CH - DN_V; }
            else { idx = DN_W_A; rr = r - DN_CONV_CH - DN_V - DN_HEADS; }
            break;
        }
        case T_FA_IN: {
            const int r = g.r0 + q * 16 + slot;
            if (slot >= 16 || r >= g.r1) return 0;
            if (r < FA_QPROJ) { idx = FA_W_Q; rr = r; }
            else if (r < FA_QPROJ + FA_KV_SIZE) { idx = FA_W_K; rr = r - FA_QPROJ; }
            else { idx = FA_W_V; rr = r - FA_QPROJ - FA_KV_SIZE; }
            break;
        }
        case T_DN_OUT:
        case T_FA_OUT: {
            const int r = g.r0 + q * 8 + slot;
            if (slot >= 8 || r >= g.r1) return 0;
            idx = (type == T_DN_OUT) ? (int)DN_W_OUT : (int)FA_W_O; rr = r; K = 2048; rpc = 8;
            break;
        }
        case T_GATEUP: {
            const int o = g.r0 + q * 8 + (slot & 7);
            if (slot >= 16 || o >= g.r1) return 0;
            const bool dn = (lw.layer_type == 0);
            idx = slot < 8 ? (dn ? (int)DN_W_GATE : (int)FA_W_GATE) : (dn ? (int)DN_W_UP : (int)FA_W_UP); rr = o;
            break;
        }
        case T_DOWN: {
            const int r = g.r0 + q * 4 + slot;
            if (slot >= 4 || r >= g.r1) return 0;
            idx = (lw.layer_type == 0) ? (int)DN_W_DOWN : (int)FA_W_DOWN; rr = r; K = INTER; rpc = 4;
            break;
        }
        case T_LM: {
#if MK_WFMT == 0
            const int r = g.r0 + q * 16 + slot;
            if (slot >= 16 || r >= g.r1) return 0;
            src = (const char*)P.lm_head + (size_t)r * (HIDDEN * 2); dst_off = slot * (HIDDEN * 2);
            return HIDDEN * 2;
#else
            // (MK_WFMT 1) packed LM-head rows are read one row per warp step: no padding, one copy per chunk
            if (lane != 0) return 0;
            const int r = g.r0 + q * LM_RPC;
            const int n = min(LM_RPC, g.r1 - r);
            src = (const char*)P.lm_head + (size_t)r * (HIDDEN / 2); dst_off = 0;
            return (uint32_t)n * (HIDDEN / 2);
#endif
        }
        case T_DN_REC: {
            if (lane != 0) return 0;
            const int u = g.r0 + q * G;           // unit = (head, 16-row value slice)
            const int h = u >> 3, sl = u & 7;
            src = (const char*)(P.dn_states + ((size_t)(dn_idx * DN_HEADS + h) * DN_VAL + sl * 16) * DN_KEY);
            dst_off = 0;
            return 16 * DN_KEY * 4;
        }
        default: return 0;
    }
#if MK_WFMT == 0
    (void)rpc; (void)kind;
    src = (const char*)lw.ptrs[idx] + (size_t)rr * row_bytes(K);
    dst_off = slot * row_stride(K);
    return row_bytes(K);
#else
    if (kind == 0) {
        src = (const char*)lw.ptrs[idx] + (size_t)rr * row_bytes(K);
        dst_off = slot * row_stride(K);
        return row_bytes(K);
    }
    src = (const char*)lw.ptrs[idx + 1] + (size_t)rr * scale_bytes(K);
    dst_off = rpc * row_stride(K) + slot * scale_bytes(K);
    return scale_bytes(K);
#endif
#endif   // MK_WFMT >= 2
}

struct Ctx {
    char* smem;
    float* xs;            // scratch as floats
    float* part;          // per-chunk, per-warp partial row sums (half in use by the current phase)
    float* part_base;
    uint32_t part_flip;
    float* red;
    volatile int* misc;
    uint32_t full0, empty0, ring0;
    int tid, warp, lane, cta, G;
    uint32_t it;          // ring chunk counter (producer and consumers advance it identically)
    uint32_t seq;         // decode steps completed on this workspace before the current one
    uint32_t trace_slot;
    uint32_t where;       // (layer << 4) | phase of the schedule this thread is in; bit 15: producer warp (diagnostics)
    int pos;              // position of the token being decoded in this step
    int step;             // index of the step inside this launch
    const float* rope;    // shared memory: cos[32] | sin[32] of pos * inv_freq_i, recomputed every step
    // tcgen05 variant only
    float amax;           // largest |value| this thread staged for the coming row product
    uint32_t mma_n;       // row products issued so far: selects the accumulator buffer and the barrier phases
    uint32_t tmem;        // base address of the CTA's tensor-memory allocation
    float inv_g;          // 1 / normalisation factor of the staged activation
    unsigned long long wf_cycles;   // traced variants: SM clocks this thread spent waiting for ring chunks to land
    uint32_t wf_count;              // ... and how many waits did not find their chunk already there
    uint32_t wf_calls;              // ... out of how many
    uint32_t dirty_stages;          // producer warp: ring stages whose last occupant the consumers wrote into
};

// A bounded wait ran out (or another CTA reported one): from here on every wait of this CTA
// returns at once and the launch drains; the status reaches the host when the kernel ends.
// Kept tiny and inline: a call here would cost a register save/restore at every wait site.
__device__ __forceinline__ void fail(const DecodeParams& P, Ctx& c, uint32_t code) {
    if (c.misc[MISC_ABORT] == 0) c.misc[MISC_DETAIL] = (int)(c.where | ((uint32_t)c.step << 16));
    c.misc[MISC_ABORT] = (int)code;
    P.ws->abort_flag = 1u;
}

// Optional timeline: thread 0 of each CTA appends the global timer at four points of every phase.
__device__ __forceinline__ void trace_point(const DecodeParams& P, Ctx& c) {
    if (MK_TRACE && P.trace) {
        if (c.tid == 0 && c.trace_slot < (uint32_t)P.trace_slots)
            P.trace[(size_t)c.cta * P.trace_slots + c.trace_slot] = globaltimer_ns();
        c.trace_slot++;
    }
}

__device__ __forceinline__ void wait_full(const DecodeParams& P, Ctx& c, uint32_t stage, uint32_t parity) {
#if MK_TRACE
    // mbarrier.try_wait may itself suspend the thread for a while before it answers: time the whole call
    const long long t0 = clock64();
    c.wf_calls++;
    bool done = mbar_try_wait(c.full0 + stage * 8, parity);
    if (!done && !c.misc[MISC_ABORT] && !mbar_wait(c.full0 + stage * 8, parity, P.mbar_limit_tries)) fail(P, c, ST_MBAR_TIMEOUT);
    const unsigned long long dt = (unsigned long long)(clock64() - t0);
    if (dt > 400ull) {                                         // more than ~0.2 us: the chunk was not there yet
        c.wf_cycles += dt; c.wf_count++;
        if (c.tid == 0) reinterpret_cast<volatile int*>(c.smem + OFF_DBG)[c.where & 15u] += (int)dt;    // ... by phase type (thread 0 only)
    }
#else
    if (mbar_try_wait(c.full0 + stage * 8, parity)) return;
    if (c.misc[MISC_ABORT]) return;
    if (!mbar_wait(c.full0 + stage * 8, parity, P.mbar_limit_tries)) fail(P, c, ST_MBAR_TIMEOUT);
#endif
}

__device__ __forceinline__ void release_stage(Ctx& c, uint32_t stage) {
    __syncwarp();
    if (c.lane == 0) mbar_arrive(c.empty0 + stage * 8);
}

// ---- flagged activation words --------------------------------------------------------------

__device__ __forceinline__ uint32_t epoch_of(const Ctx& c, int layer) { return ((c.seq + 1u) << 5) | (uint32_t)(layer + 1); }

__device__ __forceinline__ void st_flagged(unsigned long long* p, float v, uint32_t epoch) {
    const unsigned long long w = ((unsigned long long)epoch << 32) | (unsigned long long)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ void ld_word2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// (Tried and dropped, both slower on B200: keeping two or three loads of a polled word in flight, staggered by a
// fraction of an L2 round trip, and moving the retry loops out of line -- a call from this 96-register kernel
// sends the caller's live registers through local memory, and the retry loop is the common case, not the rare one.)
// Slow path of a poll (every 1024 failed tries): bounded by P.poll_limit_cycles (about 2 s of SM clock by
// default), gives up at once if another CTA gave up.
__device__ __forceinline__ bool poll_give_up(const DecodeParams& P, Ctx& c, uint64_t& t0) {
    if (c.misc[MISC_ABORT]) return true;
    const uint64_t now = (uint64_t)clock64();
    if (t0 == 0) t0 = now;
    if (now - t0 > P.poll_limit_cycles || *((volatile uint32_t*)&P.ws->abort_flag) != 0u) {
        fail(P, c, ST_GRID_TIMEOUT);
        return true;
    }
    return false;
}

__device__ __forceinline__ float poll1(const DecodeParams& P, Ctx& c, const unsigned long long* p, uint32_t epoch) {
    unsigned long long w = ld_word(p);
    if ((uint32_t)(w >> 32) != epoch) {
        uint64_t t0 = 0;
        uint32_t n = 0;
        do {
            if ((++n & 1023u) == 0 && poll_give_up(P, c, t0)) break;
            MK_POLL_BACKOFF();
            w = ld_word(p);
        } while ((uint32_t)(w >> 32) != epoch);
    }
    return __uint_as_float((uint32_t)w);
}

// two consecutive words (p must be 16-byte aligned)
__device__ __forceinline__ float2 poll2(const DecodeParams& P, Ctx& c, const unsigned long long* p, uint32_t epoch) {
    unsigned long long a, b;
    ld_word2(p, a, b);
    if ((uint32_t)(a >> 32) != epoch || (uint32_t)(b >> 32) != epoch) {
        uint64_t t0 = 0;
        uint32_t n = 0;
        do {
            if ((++n & 1023u) == 0 && poll_give_up(P, c, t0)) break;
            MK_POLL_BACKOFF();
            ld_word2(p, a, b);
        } while ((uint32_t)(a >> 32) != epoch || (uint32_t)(b >> 32) != epoch);
    }
    return make_float2(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)b));
}

// Batched polls: all loads are issued before any epoch is checked, so the N words cost one
// L2 round trip instead of N.  W = words per load (1 or 2); words of one load are consecutive.
template <int N>
__device__ __forceinline__ void poll1_batch(const DecodeParams& P, Ctx& c, const unsigned long long* const (&p)[N],
                                            uint32_t epoch, float (&out)[N]) {
    unsigned long long w[N];
    uint64_t t0 = 0;
    uint32_t n = 0;
#pragma unroll 1
    while (true) {
#pragma unroll
        for (int i = 0; i < N; ++i) w[i] = ld_word(p[i]);
        bool ok = true;
#pragma unroll
        for (int i = 0; i < N; ++i) ok = ok && ((uint32_t)(w[i] >> 32) == epoch);
        if (ok) break;
        if ((++n & 1023u) == 0 && poll_give_up(P, c, t0)) break;
        MK_POLL_BACKOFF();
    }
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = __uint_as_float((uint32_t)w[i]);
}

template <int N>
__device__ __forceinline__ void poll2_batch(const DecodeParams& P, Ctx& c, const unsigned long long* const (&p)[N],
                                            uint32_t epoch, float2 (&out)[N]) {
    unsigned long long a[N], b[N];
    uint64_t t0 = 0;
    uint32_t n = 0;
#pragma unroll 1
    while (true) {
#pragma unroll
        for (int i = 0; i < N; ++i) ld_word2(p[i], a[i], b[i]);
        bool ok = true;
#pragma unroll
        for (int i = 0; i < N; ++i) ok = ok && ((uint32_t)(a[i] >> 32) == epoch) && ((uint32_t)(b[i] >> 32) == epoch);
        if (ok) break;
        if ((++n & 1023u) == 0 && poll_give_up(P, c, t0)) break;
        MK_POLL_BACKOFF();
    }
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = make_float2(__uint_as_float((uint32_t)a[i]), __uint_as_float((uint32_t)b[i]));
}

// ---- producer ---------------------------------------------------------------------------

// What producer lane `lane` moves for chunk q, with runs of consecutive slots whose sources and ring
// destinations are contiguous (consecutive rows of one matrix) merged into ONE transfer issued by the run's
// first lane: the issue rate, not the size, limits a CTA.  Returns this lane's bytes; `head` says whether the
// lane issues, `run_bytes` how much.
__device__ __forceinline__ uint32_t chunk_runs(const DecodeParams& P, Ctx& c, int type, const LW& lw, const Geo& g, int q,
                                               int idx, int pos, const char*& src, uint32_t& dst_off, bool& head,
                                               uint32_t& run_bytes) {
    uint32_t bytes = chunk_slot_src(type, lw, P, g, q, c.lane, c.G, idx, src, dst_off, c.cta, pos);
    if (bytes && (((uintptr_t)src) & 15u)) { fail(P, c, ST_MISALIGNED); bytes = 0; }
#if MK_WFMT >= 2
    // every lane already describes a whole run (a row group, or a matrix's scale rows) of its own size: no merging
    // (two matrices that happen to lie back to back in memory must not be taken for one run of equal pieces)
    if (type != T_FA_ATT) {
        head = bytes != 0;
        run_bytes = bytes;
        return bytes;
    }
#endif
    const unsigned long long prev_src = __shfl_up_sync(0xffffffffu, (unsigned long long)(uintptr_t)src, 1);
    const uint32_t prev_bytes = __shfl_up_sync(0xffffffffu, bytes, 1);
    const uint32_t prev_dst = __shfl_up_sync(0xffffffffu, dst_off, 1);
    head = bytes && (c.lane == 0 || prev_bytes == 0 ||
                     prev_src + prev_bytes != (unsigned long long)(uintptr_t)src ||
                     prev_dst + prev_bytes != dst_off);
    const uint32_t heads = __ballot_sync(0xffffffffu, head);
    const uint32_t valid = __ballot_sync(0xffffffffu, bytes != 0);
    const uint32_t above = (c.lane == 31) ? 0u : ~((2u << c.lane) - 1u);
    const uint32_t stop = (heads | ~valid) & above;
    const int end = stop ? (__ffs(stop) - 1) : 32;
    run_bytes = bytes * (uint32_t)(end - c.lane);
    return bytes;
}

__device__ __forceinline__ void producer_phase(const DecodeParams& P, Ctx& c, int type, const LW& lw, int dn_idx,
                               uint64_t pol_stream, uint64_t pol_keep) {
    const Geo g = phase_geo(type, c.cta, c.G, P.vocab, c.pos);
    // State rows and cache rows were written with ordinary stores, possibly by an earlier step of this launch.  The
    // writers released (ring barrier / ready word) long before this warp acquired the stage it is about to fill; the
    // proxy fence orders those writes before the bulk copies below, which read through the async proxy.  (A fence
    // on the writers' side would sit on the critical path: it waits for their stores to complete.)
    if (type == T_DN_REC || type == T_FA_ATT) fence_proxy_async();
#pragma unroll 1
    for (int q = 0; q < g.nchunks; ++q, ++c.it) {
        if (c.misc[MISC_ABORT]) continue;
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        if (c.lane == 0 && !mbar_wait(c.empty0 + stage * 8, parity ^ 1u, P.mbar_limit_tries)) fail(P, c, ST_MBAR_TIMEOUT);
        __syncwarp();
        // The attention phase patches and pads its K/V tile in place, with ordinary stores into the ring stage.  Those
        // stores were released through the stage's "empty" barrier, acquired just above; the proxy fence orders them
        // before the bulk copies that now overwrite the stage (async proxy).  It sits here, in the warp that runs
        // ahead, because on the consumers' side it cost 1.8 us per attention layer on the critical path.
        if (c.dirty_stages & (1u << stage)) { fence_proxy_async(); c.dirty_stages &= ~(1u << stage); }
        if (type == T_FA_ATT) {
            // chunk q = tile * 4 + {K lo, K hi, V lo, V hi} of this CTA's unit (dn_idx carries the attention layer index):
            // 32 positions from p0 as four 64-dim boxes, lanes 0-3; rows past the unit's last position come along and are
            // masked by the consumers; a chunk that starts past it completes with nothing
            c.dirty_stages |= 1u << stage;
            if (c.misc[MISC_ABORT]) continue;
            const int kvh = c.cta / att_num_chunks(c.pos + 1), part = q & 3;
            const int p0 = g.r0 + (q >> 2) * 64 + (part & 1) * 32;
            const bool any = p0 < g.r1;
            if (c.lane == 0) mbar_expect_tx(c.full0 + stage * 8, any ? 32u * FA_HEAD_DIM * 2u : 0u);
            __syncwarp();
            if (any && c.lane < 4) {
                const CUtensorMap* map = (part & 2) ? &P.map_v : &P.map_k;
                const int row = (dn_idx * FA_KV_HEADS + kvh) * P.max_seq_len + p0;
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                    ::"r"(c.ring0 + stage * STAGE_BYTES + c.lane * 4096), "l"(map), "r"(64 * c.lane), "r"(row), "r"(c.full0 + stage * 8)
                    : "memory");
            }
            continue;
        }
        const char* src = nullptr;
        uint32_t dst_off = 0, run_bytes = 0;
        bool head = false;
        const uint32_t bytes = chunk_runs(P, c, type, lw, g, q, dn_idx, c.pos, src, dst_off, head, run_bytes);
        const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
        if (c.misc[MISC_ABORT]) continue;
        if (c.lane == 0) mbar_expect_tx(c.full0 + stage * 8, total);
        __syncwarp();
        if (head)
            bulk_g2s(c.ring0 + stage * STAGE_BYTES + dst_off, src, run_bytes, c.full0 + stage * 8,
                     (type == T_DN_REC || type == T_FA_ATT) ? pol_keep : pol_stream);
    }
}

// ---- tensor-core row products ---------------------------------------------------------------

#if MK_WFMT == 0
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// An f32 activation is carried through the bf16 MMA as three bf16 terms that add up to it
// exactly: each term keeps the next 8 leading mantissa bits (truncation, no rounding), so
// hi + mid + lo == x.  The terms occupy MMA columns 0, 1, 2; columns 3..7 are zero.
__device__ __forceinline__ void split3(float x, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
    hi = __float_as_uint(x) & 0xffff0000u;
    const float r1 = x - __uint_as_float(hi);
    mid = __float_as_uint(r1) & 0xffff0000u;
    const float r2 = r1 - __uint_as_float(mid);
    lo = __float_as_uint(r2) & 0xffff0000u;
}
#else
// NVFP4 weights are exact in f16 (e2m1 codes 0..6), so this variant multiplies in f16: the
// activation is split into three f16 terms (round to nearest; the sum reproduces x to about
// 2^-30 relative unless a term underflows below 6e-8, far under the bf16 tolerances).
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// terms returned in the upper 16 bits, like the bf16 variant
__device__ __forceinline__ void split3(float x, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
    const __half h = __float2half_rn(x);
    const float r1 = x - __half2float(h);
    const __half m = __float2half_rn(r1);
    const float r2 = r1 - __half2float(m);
    const __half l = __float2half_rn(r2);
    hi = (uint32_t)__half_as_ushort(h) << 16;
    mid = (uint32_t)__half_as_ushort(m) << 16;
    lo = (uint32_t)__half_as_ushort(l) << 16;
}

// two e2m1 codes (one byte, low nibble first) -> f16x2
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
    const __half2_raw h = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)(byte & 0xffu), __NV_E2M1);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

#endif

// Staging of a warp's K-slice: three planes of XK bf16.  Elements e, e+1 (e even) as one word.
__device__ __forceinline__ void stage_pair(uint32_t* xw, int e, float x0, float x1) {
    uint32_t h0, m0, l0, h1, m1, l1;
    split3(x0, h0, m0, l0);
    split3(x1, h1, m1, l1);
    xw[e >> 1] = __byte_perm(h0, h1, 0x7632);
    xw[(XK >> 1) + (e >> 1)] = __byte_perm(m0, m1, 0x7632);
    xw[XK + (e >> 1)] = __byte_perm(l0, l1, 0x7632);
}
__device__ __forceinline__ void stage_one(uint32_t* xw, int e, float x) {
    uint32_t h, m, l;
    split3(x, h, m, l);
    unsigned short* p = reinterpret_cast<unsigned short*>(xw);
    p[e] = (unsigned short)(h >> 16);
    p[XK + e] = (unsigned short)(m >> 16);
    p[2 * XK + e] = (unsigned short)(l >> 16);
}

// B fragments of this warp's K-slice.  Thread (g = lane/4, t = lane%4) reads the 16-byte weight
// chunks t, t+4, ... of a row, i.e. elements 8(t+4i)..+7; chunk i feeds MMA 2i (first four
// elements) and MMA 2i+1 (last four).  The k order inside an MMA is a permutation shared by both
// operands, so any consistent assignment is valid: the same 16 bytes of plane g are the B words.
template <int NLOAD>
__device__ __forceinline__ void load_bfrags(const uint32_t* xw, int lane, uint32_t (&b)[2 * NLOAD][2]) {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t* plane = xw + (g < 3 ? g : 0) * (XK >> 1);
#pragma unroll
    for (int i = 0; i < NLOAD; ++i) {
        uint4 v = *reinterpret_cast<const uint4*>(plane + 4 * (t + 4 * i));
        if (g >= 3) v = make_uint4(0, 0, 0, 0);
        b[2 * i][0] = v.x; b[2 * i][1] = v.y;
        b[2 * i + 1][0] = v.z; b[2 * i + 1][1] = v.w;
    }
}

#if MK_WFMT == 0
// One ring chunk times the activation: rows of `rowbytes` bytes, this warp's K-slice starting
// `kofs` bytes into each row.  ROWS = 16: tile rows g and g+8; ROWS = 8: row g; ROWS = 4: rows g < 4.
// Odd g read their chunks rotated by one so that the two rows of a quarter-warp hit different
// banks (all rows alias: the row stride is a multiple of 128 bytes).  Writes the warp's partial
// sums of tile rows into `out[0..15]`.  (Inlined: as a called function it cost ~0.18 us per chunk, the caller's
// live registers going through local memory around every call.)
template <int NLOAD, int ROWS>
__device__ __forceinline__ void mma_chunk(const char* stage, int K, int warp, int lane,
                                          const uint32_t (&b)[2 * NLOAD][2], float* out) {
    const int g = lane >> 2, t = lane & 3, odd = g & 1;
    const int rowbytes = row_stride(K), kofs = warp * NLOAD * 64;      // 32*NLOAD elements of 2 bytes per warp
    const bool live = (ROWS >= 8) || (g < 4);
    const char* r0 = stage + g * rowbytes + kofs + 16 * t;
    const char* r1 = r0 + 8 * rowbytes;
    uint4 A0[NLOAD], A1[NLOAD];
#pragma unroll
    for (int s = 0; s < NLOAD; ++s) {
        int i = s + odd;
        if (i >= NLOAD) i -= NLOAD;
        A0[s] = live ? *reinterpret_cast<const uint4*>(r0 + 64 * i) : make_uint4(0, 0, 0, 0);
        if (ROWS == 16) A1[s] = *reinterpret_cast<const uint4*>(r1 + 64 * i);
        else A1[s] = make_uint4(0, 0, 0, 0);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < NLOAD; ++i) {
        constexpr int N = NLOAD;
        const int so = (i + N - 1) % N;      // slot holding chunk i for odd g
        uint4 a, d;
        a.x = odd ? A0[so].x : A0[i].x; a.y = odd ? A0[so].y : A0[i].y;
        a.z = odd ? A0[so].z : A0[i].z; a.w = odd ? A0[so].w : A0[i].w;
        if (ROWS == 16) {
            d.x = odd ? A1[so].x : A1[i].x; d.y = odd ? A1[so].y : A1[i].y;
            d.z = odd ? A1[so].z : A1[i].z; d.w = odd ? A1[so].w : A1[i].w;
        } else {
            d = make_uint4(0, 0, 0, 0);
        }
        mma_16816(acc, a.x, d.x, a.y, d.y, b[2 * i][0], b[2 * i][1]);
        mma_16816(acc2, a.z, d.z, a.w, d.w, b[2 * i + 1][0], b[2 * i + 1][1]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] += acc2[k];
    // columns 0,1 (hi, mid) sit in the t = 0 lane, column 2 (lo) in the t = 1 lane
    float s0 = acc[0] + (t == 0 ? acc[1] : 0.f);
    float s1 = acc[2] + (t == 0 ? acc[3] : 0.f);
    s0 += __shfl_down_sync(0xffffffffu, s0, 1);
    s1 += __shfl_down_sync(0xffffffffu, s1, 1);
    if (t == 0) {
        out[g] = s0;
        if (ROWS == 16) out[g + 8] = s1;
    }
}

// Two 4-row chunks (the down projection) as ONE 8-row tile: lane groups 0-3 read the rows of the first chunk, 4-7 the
// rows of the second, so the pair costs the MMAs of one chunk instead of two half-empty tiles one after the other.
template <int NLOAD>
__device__ __forceinline__ void mma_chunk_pair4(const char* stage0, const char* stage1, int K, int warp, int lane,
                                                const uint32_t (&b)[2 * NLOAD][2], float* out0, float* out1) {
    const int g = lane >> 2, t = lane & 3, odd = g & 1;
    const int rowbytes = row_stride(K), kofs = warp * NLOAD * 64;
    const char* r0 = (g < 4 ? stage0 + g * rowbytes : stage1 + (g - 4) * rowbytes) + kofs + 16 * t;
    uint4 A0[NLOAD];
#pragma unroll
    for (int s = 0; s < NLOAD; ++s) {
        int i = s + odd;
        if (i >= NLOAD) i -= NLOAD;
        A0[s] = *reinterpret_cast<const uint4*>(r0 + 64 * i);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < NLOAD; ++i) {
        constexpr int N = NLOAD;
        const int so = (i + N - 1) % N;
        uint4 a;
        a.x = odd ? A0[so].x : A0[i].x; a.y = odd ? A0[so].y : A0[i].y;
        a.z = odd ? A0[so].z : A0[i].z; a.w = odd ? A0[so].w : A0[i].w;
        mma_16816(acc, a.x, 0u, a.y, 0u, b[2 * i][0], b[2 * i][1]);
        mma_16816(acc2, a.z, 0u, a.w, 0u, b[2 * i + 1][0], b[2 * i + 1][1]);
    }
    float s0 = (acc[0] + acc2[0]) + (t == 0 ? acc[1] + acc2[1] : 0.f);
    s0 += __shfl_down_sync(0xffffffffu, s0, 1);
    if (t == 0) {
        if (g < 4) out0[g] = s0;
        else out1[g - 4] = s0;
    }
}

#elif MK_WFMT == 1
// NVFP4 version of the chunk product.  Stage: packed rows at a stride of K/2+16 bytes, then the
// fp16 scales of the chunk's rows.  The 16-byte weight chunk i of the bf16 layout (8 elements) is
// one 32-bit word of nibbles here; the 32 elements the four lanes of a row cover in chunk i are
// exactly quantisation group warp*NLOAD+i, so the two MMAs of a chunk go into a fresh accumulator
// that is then scaled by the group's scale of each row: the dequantised value never has to be
// rounded.  The row stride keeps the 8 rows of a quarter-warp on different banks.
template <int NLOAD, int ROWS>
__device__ __forceinline__ void mma_chunk(const char* stage, int K, int warp, int lane,
                                          const uint32_t (&b)[2 * NLOAD][2], float* out) {
    const int g = lane >> 2, t = lane & 3;
    const bool live = (ROWS >= 8) || (g < 4);
    const int stride = row_stride(K);
    const char* r0 = stage + g * stride + warp * (NLOAD * 16) + 4 * t;
    const char* r1 = r0 + 8 * stride;
    const unsigned short* sc0 = reinterpret_cast<const unsigned short*>(stage + ROWS * stride + g * scale_bytes(K)) + warp * NLOAD;
    const unsigned short* sc1 = sc0 + 8 * (scale_bytes(K) / 2);
    uint32_t w0[NLOAD], w1[NLOAD];
    float s0[NLOAD], s1[NLOAD];
#pragma unroll
    for (int i = 0; i < NLOAD; ++i) {
        w0[i] = live ? *reinterpret_cast<const uint32_t*>(r0 + 16 * i) : 0u;
        s0[i] = live ? __half2float(__ushort_as_half(sc0[i])) : 0.f;
        if (ROWS == 16) { w1[i] = *reinterpret_cast<const uint32_t*>(r1 + 16 * i); s1[i] = __half2float(__ushort_as_half(sc1[i])); }
        else { w1[i] = 0u; s1[i] = 0.f; }
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < NLOAD; ++i) {
        float tmp[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t ra[4], rb[4] = {0u, 0u, 0u, 0u};
        e2m1x8_to_f16x2x4(w0[i], ra);
        if (ROWS == 16) e2m1x8_to_f16x2x4(w1[i], rb);
        mma_16816(tmp, ra[0], rb[0], ra[1], rb[1], b[2 * i][0], b[2 * i][1]);
        mma_16816(tmp, ra[2], rb[2], ra[3], rb[3], b[2 * i + 1][0], b[2 * i + 1][1]);
        acc[0] = fmaf(s0[i], tmp[0], acc[0]); acc[1] = fmaf(s0[i], tmp[1], acc[1]);
        acc[2] = fmaf(s1[i], tmp[2], acc[2]); acc[3] = fmaf(s1[i], tmp[3], acc[3]);
    }
    float q0 = acc[0] + (t == 0 ? acc[1] : 0.f);
    float q1 = acc[2] + (t == 0 ? acc[3] : 0.f);
    q0 += __shfl_down_sync(0xffffffffu, q0, 1);
    q1 += __shfl_down_sync(0xffffffffu, q1, 1);
    if (t == 0) {
        out[g] = q0;
        if (ROWS == 16) out[g + 8] = q1;
    }
}
#endif

#if MK_WFMT == 2
// ---- tensor-scale NVFP4: one chunk per phase, warps split it into row tiles x K parts ------------------------
// A chunk holds R consecutive rows (64 / 32 / 16 for K = 1024 / 2048 / 3584), unpadded.  RT row tiles of 16 rows x KS
// parts of the K dimension of 256 elements (8 segments of 32) make RT * KS working warps (16, 8 or 14 of the 16).
// Rows are a multiple of 128 bytes apart, so the eight rows a quarter-warp reads at once would collide on the same
// banks; instead lane group g reads segment i ^ g in step i (eight different 16-byte columns: no conflict) and a
// three-stage network of selects puts the words back in segment order.
// Activations: part p of the K dimension is staged as three f16 planes of 256 elements (hi / mid / lo terms) at
// xs + p * 384 words, written by whichever warps own those elements and read by the RT warps of that part.
template <int PK>
__device__ __forceinline__ void stage_pair_ts(Ctx& c, int e, float x0, float x1) {
    uint32_t* xw = reinterpret_cast<uint32_t*>(c.xs) + (e / PK) * (3 * PK / 2);
    const int l = e % PK;
    uint32_t h0, m0, l0, h1, m1, l1;
    split3(x0, h0, m0, l0);
    split3(x1, h1, m1, l1);
    xw[l >> 1] = __byte_perm(h0, h1, 0x7632);
    xw[(PK >> 1) + (l >> 1)] = __byte_perm(m0, m1, 0x7632);
    xw[PK + (l >> 1)] = __byte_perm(l0, l1, 0x7632);
}
template <int PK>
__device__ __forceinline__ void stage_one_ts(Ctx& c, int e, float x) {
    unsigned short* p = reinterpret_cast<unsigned short*>(reinterpret_cast<uint32_t*>(c.xs) + (e / PK) * (3 * PK / 2));
    const int l = e % PK;
    uint32_t h, m, lo;
    split3(x, h, m, lo);
    p[l] = (unsigned short)(h >> 16);
    p[PK + l] = (unsigned short)(m >> 16);
    p[2 * PK + l] = (unsigned short)(lo >> 16);
}
__device__ __forceinline__ void load_bfrags_ts(const uint32_t* xw, int lane, uint32_t (&b)[16][2]) {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t* plane = xw + (g < 3 ? g : 0) * 128;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint4 v = *reinterpret_cast<const uint4*>(plane + 4 * (t + 4 * i));
        if (g >= 3) v = make_uint4(0, 0, 0, 0);
        b[2 * i][0] = v.x; b[2 * i][1] = v.y;
        b[2 * i + 1][0] = v.z; b[2 * i + 1][1] = v.w;
    }
}
// w[i] holds segment i ^ g on entry and segment i on return
__device__ __forceinline__ void unxor8(uint32_t (&w)[8], int g) {
#pragma unroll
    for (int bit = 1; bit < 8; bit <<= 1) {
        const bool sw = (g & bit) != 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if ((i & bit) == 0) {
                const uint32_t a = w[i], d = w[i | bit];
                w[i] = sw ? d : a;
                w[i | bit] = sw ? a : d;
            }
        }
    }
}

// The chunk in `stage` times the staged activation; warp (kq, T) = warp / RT, warp % RT leaves its partial sums of
// tile T's 16 rows (8 when !TWO: the phase has at most 8 rows) in out[0..15].
template <int RT, bool TWO>
__device__ __forceinline__ void mma_chunk_ts(const char* stage, const uint32_t* xw, int K, int warp, int lane, float* out) {
    const int g = lane >> 2, t = lane & 3, T = warp % RT, kq = warp / RT;
    const int rb = K / 2, sb = K / 16;
    uint32_t b[16][2];
    load_bfrags_ts(xw, lane, b);
    const char* r0 = stage + (16 * T + g) * rb + kq * 128 + 4 * t;
    const unsigned char* sc0 = reinterpret_cast<const unsigned char*>(stage) + rows_per_chunk(K) * rb + (16 * T + g) * sb + kq * 16;
    uint32_t w0[8], w1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        w0[i] = *reinterpret_cast<const uint32_t*>(r0 + 16 * (i ^ g));
        w1[i] = TWO ? *reinterpret_cast<const uint32_t*>(r0 + 8 * rb + 16 * (i ^ g)) : 0u;
    }
    const uint4 sa = *reinterpret_cast<const uint4*>(sc0);
    const uint4 sd = TWO ? *reinterpret_cast<const uint4*>(sc0 + 8 * sb) : make_uint4(0, 0, 0, 0);
    unxor8(w0, g);
    if (TWO) unxor8(w1, g);
    const uint32_t aw[4] = {sa.x, sa.y, sa.z, sa.w}, dw[4] = {sd.x, sd.y, sd.z, sd.w};
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
    const int sh = (t >> 1) * 8;          // lanes t = 0,1 hold elements of the segment's first block, t = 2,3 of its second
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const __half2 h0 = e4m3_to_h2_div256((aw[i >> 1] >> (16 * (i & 1))) >> sh);
        const __half2 h1 = e4m3_to_h2_div256((dw[i >> 1] >> (16 * (i & 1))) >> sh);
        uint32_t ra[4], rbv[4] = {0u, 0u, 0u, 0u};
        e2m1x8_to_f16x2x4(w0[i], ra);
        if (TWO) e2m1x8_to_f16x2x4(w1[i], rbv);
        mma_16816(acc, hmul2_bits(ra[0], h0), TWO ? hmul2_bits(rbv[0], h1) : 0u, hmul2_bits(ra[1], h0), TWO ? hmul2_bits(rbv[1], h1) : 0u,
                  b[2 * i][0], b[2 * i][1]);
        mma_16816(acc2, hmul2_bits(ra[2], h0), TWO ? hmul2_bits(rbv[2], h1) : 0u, hmul2_bits(ra[3], h0), TWO ? hmul2_bits(rbv[3], h1) : 0u,
                  b[2 * i + 1][0], b[2 * i + 1][1]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] += acc2[k];
    float q0 = acc[0] + (t == 0 ? acc[1] : 0.f);
    float q1 = acc[2] + (t == 0 ? acc[3] : 0.f);
    q0 += __shfl_down_sync(0xffffffffu, q0, 1);
    q1 += __shfl_down_sync(0xffffffffu, q1, 1);
    if (t == 0) { out[g] = q0; if (TWO) out[g + 8] = q1; }
}

// One-chunk phase.  `sync_parts`: the staged activation was written by other warps than the ones that read it.
template <int RT, int KS, bool TWO>
__device__ __forceinline__ void mma_phase_ts(const DecodeParams& P, Ctx& c, int nchunks, int K, bool sync_parts) {
    c.part = c.part_base + ((c.part_flip++ & 1u) ? PART_HALF : 0);
    if (sync_parts) named_bar_sync(1, NCT);
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(c.xs) + (c.warp / RT) * 384;
    if (nchunks > 1) { fail(P, c, ST_MISALIGNED); nchunks = 1; }   // never reached for grids >= MIN_GRID
    if (nchunks > 0) {
        const uint32_t stage = c.it % NSTAGE;
        wait_full(P, c, stage, (c.it / NSTAGE) & 1u);
        if (c.warp < RT * KS)
            mma_chunk_ts<RT, TWO>(c.smem + OFF_RING + stage * STAGE_BYTES, xw, K, c.warp, c.lane, c.part + c.warp * 16);
        release_stage(c, stage);
        ++c.it;
    }
}
// sum over the K parts of stage row r of the chunk
template <int RT, int KS>
__device__ __forceinline__ float part_sum_ts(const Ctx& c, int r) {
    const int T = r >> 4, idx = r & 15;
    float s = 0.f;
#pragma unroll
    for (int kq = 0; kq < KS; ++kq) s += c.part[(kq * RT + T) * 16 + idx];
    return s;
}
// the matrix's fp32 scale times the 2^8 the block scales were divided by
__device__ __forceinline__ float tensor_scale_of(const LW& lw, int slot) {
    return __ldg(reinterpret_cast<const float*>(lw.ptrs[slot + 2])) * TS_SCALE_FOLD;
}
#endif

#if MK_WFMT == 3
// ---- tensor-scale NVFP4 on tcgen05: the CTA's rows of a phase x the activation as NVFP4 residual terms ---------
// A (weights): the chunk image in the ring stage, M = 128 rows of which the first u_rp(type) are real (what lies
// behind them in shared memory feeds accumulator rows nobody reads).  B (activation): up to 8 rows, one per residual
// term, quantised by the consumer warps into U_OFF_B / U_OFF_SFB.  D: 128 lanes x 8 columns of tensor memory, one of
// two buffers.  Block scales: one tcgen05.cp (32 lanes x 16 bytes, replicated to the four lane quadrants) per MMA step
// and operand fills four columns: row r of the operand reads lane r % 32, column r / 32, one byte per 16-value block.
template <int PK>
__device__ __forceinline__ void stage_pair_ts(Ctx& c, int e, float x0, float x1) {
    reinterpret_cast<float2*>(c.xs)[e >> 1] = make_float2(x0, x1);
    c.amax = fmaxf(c.amax, fmaxf(fabsf(x0), fabsf(x1)));
}
template <int PK>
__device__ __forceinline__ void stage_one_ts(Ctx& c, int e, float x) {
    c.xs[e] = x;
    c.amax = fmaxf(c.amax, fabsf(x));
}

__device__ __forceinline__ uint64_t u_desc_sw128(uint32_t saddr) {   // K-major, 128-byte swizzle, 8-row groups 1024 B apart
    return (uint64_t)((saddr & 0x3ffffu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}
__device__ __forceinline__ uint64_t u_desc_sf(uint32_t saddr) {      // 32 rows of 16 bytes, no swizzle, 8-row groups 128 B apart
    return (uint64_t)((saddr & 0x3ffffu) >> 4) | ((uint64_t)(128 >> 4) << 32) | ((uint64_t)1 << 46);
}
// kind::mxf4nvf4, e2m1 x e2m1, E4M3 block scales, K-major operands, M = 128, N = 8
constexpr uint32_t U_IDESC = (1u << 7) | (1u << 10) | ((8u >> 3) << 17) | ((128u >> 4) << 24);
__device__ __forceinline__ void u_mma(uint32_t d, uint64_t ad, uint64_t bd, uint32_t sfa, uint32_t sfb, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d), "l"(ad), "l"(bd), "r"(U_IDESC), "r"(acc), "r"(sfa), "r"(sfb) : "memory");
}
__device__ __forceinline__ void u_cp_sf(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void u_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void u_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void u_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float e4m3_value(uint32_t code) {       // code << 7 read as f16 is the value / 256
    return __half2float(__ushort_as_half((unsigned short)(code << 7))) * 256.0f;
}
// eight floats -> eight e2m1 codes, element 0 in the low nibble (round to nearest even, saturating at 6)
__device__ __forceinline__ uint32_t f32x8_to_e2m1x8(const float (&v)[8]) {
    uint32_t w;
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
        "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
        : "=r"(w)
        : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
    return w;
}

// The staged f32 vector (c.xs[0..K)) -> P.act_terms NVFP4 terms in the B operand layout.  Two threads per 16-element
// block.  x is first scaled by g = 192 / max|x|, so that block scales start at or below 32 whatever the vector's
// magnitude.  All terms of a block share ONE scale s = E4M3 rounded UP from max|g x| / 6; with u_0 = g x / s (|u_0| <= 6)
//   code_n = e2m1_rne(u_n),   u_1 = 4 (u_0 - code_0),   u_{n+1} = 8 (u_n - code_n)  for n >= 1:
// the first residual is at most 1 (half the widest e2m1 gap), so |u_1| <= 4, and from there on residuals are at most
// 1/2, so every |u_n| <= 4: nothing ever saturates and every step is exact in f32.  Hence
//   x = (s / g) (code_0 + code_1 / 4 + code_2 / 32 + code_3 / 256 + ...)   up to the last residual, <= s / (g 4 8^(T-1)).
// Ends by arriving on the "activation ready" barrier the MMA warp waits on; sets c.inv_g.
__device__ __forceinline__ void u_prepare_acts(const DecodeParams& P, Ctx& c, int K) {
    float* wmax = reinterpret_cast<float*>(c.smem + U_OFF_AMAX);
    const float m = warp_max(c.amax);
    c.amax = 0.f;
    if (c.lane == 0) wmax[c.warp] = m;
    named_bar_sync(1, NCT);                       // the vector is staged, the warp maxima are written
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < NCW; ++i) am = fmaxf(am, wmax[i]);
    const float g = (am > 0.f && am < 3.0e38f) ? 192.0f / am : 1.0f;
    c.inv_g = 1.0f / g;
    const int b = c.tid >> 1, h = c.tid & 1;
    if (b < K / 16) {
        float u[8];
        {
            const float4 a = *reinterpret_cast<const float4*>(c.xs + 16 * b + 8 * h);
            const float4 d = *reinterpret_cast<const float4*>(c.xs + 16 * b + 8 * h + 4);
            u[0] = a.x * g; u[1] = a.y * g; u[2] = a.z * g; u[3] = a.w * g;
            u[4] = d.x * g; u[5] = d.y * g; u[6] = d.z * g; u[7] = d.w * g;
        }
        float a = fmaxf(fmaxf(fmaxf(fabsf(u[0]), fabsf(u[1])), fmaxf(fabsf(u[2]), fabsf(u[3]))),
                        fmaxf(fmaxf(fabsf(u[4]), fabsf(u[5])), fmaxf(fabsf(u[6]), fabsf(u[7]))));
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
        const float t = a * (1.0f / 6.0f);
        uint32_t code = (uint32_t)__nv_cvt_float_to_fp8(t, __NV_SATFINITE, __NV_E4M3);
        float sv = e4m3_value(code);
        if (sv < t && code < 0x7eu) { ++code; sv = e4m3_value(code); }
        if (code == 0u) { code = 1u; sv = 0.001953125f; }
        const float inv = 1.0f / sv;
#pragma unroll
        for (int i = 0; i < 8; ++i) u[i] *= inv;
        const int bb = b & 15;
        char* brow = c.smem + U_OFF_B + (b >> 4) * 1024 + (bb & 1) * 8 + h * 4;
        unsigned char* sfb = reinterpret_cast<unsigned char*>(c.smem) + U_OFF_SFB + (b >> 2) * 512 + (b & 3);
        const int terms = P.act_terms;
#pragma unroll 1
        for (int n = 0; n < terms; ++n) {
            const uint32_t w = f32x8_to_e2m1x8(u);
            uint32_t hh[4];
            e2m1x8_to_f16x2x4(w, hh);
            const float up = n ? 8.0f : 4.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hh[i]));
                u[2 * i] = (u[2 * i] - f.x) * up;
                u[2 * i + 1] = (u[2 * i + 1] - f.y) * up;
            }
            *reinterpret_cast<uint32_t*>(brow + n * 128 + (((bb >> 1) ^ n) << 4)) = w;
            if (h == 0) sfb[n * 16] = (unsigned char)code;
        }
    }
    fence_proxy_async();                          // the tensor core reads shared memory through the async proxy
    __syncwarp();
    if (c.lane == 0) mbar_arrive(smem_u32(c.smem + U_OFF_BARS) + 32);
}

// ---- the MMA warp's side ---------------------------------------------------------------------------------------
// Descriptors advance by plain additions on their low words: a K-major 128-byte-swizzled operand moves 32 bytes (2
// units of 16) per MMA step inside a k-tile; a scale unit is 512 bytes (32 units).
__device__ __forceinline__ uint64_t u_desc(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }
constexpr uint32_t U_HI_SW128 = (1024u >> 4) | (1u << 14) | (2u << 29);
constexpr uint32_t U_HI_SF = (128u >> 4) | (1u << 14);

// (Keeping these two loops rolled, four operations per trip, is no faster: a tcgen05.cp or tcgen05.mma of this size costs
// about 42 ns on the tensor pipe however its issue is coded.)
template <int N>
__device__ __forceinline__ void u_copy_units(uint32_t taddr, uint32_t saddr) {
    const uint32_t lo = (saddr & 0x3ffffu) >> 4;
#pragma unroll
    for (int i = 0; i < N; ++i) u_cp_sf(taddr + 4 * i, u_desc(lo + 32 * i, U_HI_SF));
}
// NS MMA steps of one chunk image of RP rows at a_s; ks0 = first step's index within the product
template <int NS, int RP>
__device__ __forceinline__ void u_mma_steps(uint32_t d_t, uint32_t a_s, uint32_t b_s, uint32_t sfa_t, uint32_t sfb_t, int ks0) {
    const uint32_t a_lo = ((a_s & 0x3ffffu) >> 4) | (1u << 16);
    const uint32_t b_lo = (((b_s + (ks0 >> 2) * 1024) & 0x3ffffu) >> 4) | (1u << 16);
    static_assert(NS % 4 == 0, "whole k-tiles");
#pragma unroll
    for (int kl = 0; kl < NS; ++kl)
        // (spreading the steps over several accumulator column groups changes nothing: a step costs about 42 ns
        // whether or not it depends on the one before)
        u_mma(d_t, u_desc(a_lo + (kl >> 2) * (RP * 128 / 16) + (kl & 3) * 2, U_HI_SW128),
              u_desc(b_lo + (kl >> 2) * (1024 / 16) + (kl & 3) * 2, U_HI_SW128), sfa_t + 4 * (ks0 + kl), sfb_t + 4 * (ks0 + kl),
              (ks0 + kl) ? 1u : 0u);
}

__device__ __forceinline__ void u_wait(const DecodeParams& P, Ctx& c, uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return;
    if (c.misc[MISC_ABORT]) return;
    if (!mbar_wait(bar, parity, P.mbar_limit_tries)) fail(P, c, ST_MBAR_TIMEOUT);
}

// One projection phase (or one LM-head chunk when `lm`): weight scales go to tensor memory as soon as the chunk has
// landed and the previous product no longer reads that region; the MMAs follow the activation.
//   barriers at U_OFF_BARS: +0,+8 product m done (by parity of m); +16,+24 accumulator buffer drained; +32 activation ready
__device__ __forceinline__ void u_mma_phase(const DecodeParams& P, Ctx& c, int type, int nchunks, uint32_t& m, uint32_t& an,
                                            bool lm_chunk, bool lm_first) {
    const uint32_t ubar = smem_u32(c.smem + U_OFF_BARS);
    const int K = u_k(type);
    const uint32_t d_t = c.tmem + 32u * (m & 1u);
    const uint32_t sfa_t = c.tmem + U_TM_SFA + ((K == HIDDEN) ? 64u * (m & 1u) : 0u), sfb_t = c.tmem + U_TM_SFB;
    const uint32_t b_s = smem_u32(c.smem + U_OFF_B), sfb_s = smem_u32(c.smem + U_OFF_SFB);
    // region of the weight scales is free: inside the LM head regions alternate and product m - 2 has been read back
    // (waited for below); everywhere else the previous product must have finished
    if (lm_chunk && !lm_first) {
        if (m >= 2u) u_wait(P, c, ubar + 16 + 8 * (m & 1u), ((m >> 1) - 1u) & 1u);
    } else if (m >= 1u) {
        u_wait(P, c, ubar + 8 * ((m - 1u) & 1u), ((m - 1u) >> 1) & 1u);
    }
    for (int q = 0; q < nchunks; ++q) {
        const uint32_t itq = c.it + q, stage = itq % NSTAGE;
        wait_full(P, c, stage, (itq / NSTAGE) & 1u);
        const uint32_t a_s = c.ring0 + stage * STAGE_BYTES;
        u_fence_after();
        switch (type) {
            case T_FA_IN:  u_copy_units<16>(sfa_t, a_s + 40 * 512); break;
            case T_DN_OUT:
            case T_FA_OUT: u_copy_units<32>(sfa_t, a_s + 8 * 1024); break;
            case T_DOWN:   u_copy_units<28>(sfa_t + 4 * 28 * q, a_s + 8 * 896); break;
            default:       u_copy_units<16>(sfa_t, a_s + 56 * 512); break;       // qkv|z, gate|up, LM head
        }
    }
    if (!lm_chunk || lm_first) {
        u_wait(P, c, ubar + 32, an & 1u);          // the activation operand is in shared memory
        ++an;
        u_fence_after();
        switch (K) {
            case HIDDEN: u_copy_units<16>(sfb_t, sfb_s); break;
            case 2048:   u_copy_units<32>(sfb_t, sfb_s); break;
            default:     u_copy_units<56>(sfb_t, sfb_s); break;
        }
    }
    if (m >= 2u) u_wait(P, c, ubar + 16 + 8 * (m & 1u), ((m >> 1) - 1u) & 1u);   // accumulator buffer drained
    u_fence_after();
    for (int q = 0; q < nchunks; ++q) {
        const uint32_t a_s = c.ring0 + ((c.it + q) % NSTAGE) * STAGE_BYTES;
        switch (type) {
            case T_FA_IN:  u_mma_steps<16, 40>(d_t, a_s, b_s, sfa_t, sfb_t, 0); break;
            case T_DN_OUT:
            case T_FA_OUT: u_mma_steps<32, 8>(d_t, a_s, b_s, sfa_t, sfb_t, 0); break;
            case T_DOWN:   u_mma_steps<28, 8>(d_t, a_s, b_s, sfa_t, sfb_t, 28 * q); break;
            default:       u_mma_steps<16, 56>(d_t, a_s, b_s, sfa_t, sfb_t, 0); break;
        }
    }
    u_commit(ubar + 8 * (m & 1u));
    c.it += nchunks;
    ++m;
}

// Everyone: wait for product m.
__device__ __forceinline__ void u_wait_product(const DecodeParams& P, Ctx& c, uint32_t m) {
    u_wait(P, c, smem_u32(c.smem + U_OFF_BARS) + 8 * (m & 1u), (m >> 1) & 1u);
    u_fence_after();
}

// Warps 0 and 1: row 32 warp + lane of product m, the terms recombined; then the buffer is handed back.
__device__ __forceinline__ float u_read_row(Ctx& c, uint32_t m) {
    uint32_t v[8];
    __syncwarp();
    const uint32_t taddr = c.tmem + ((uint32_t)(32 * c.warp) << 16) + 32u * (m & 1u);
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    u_fence_before();
    __syncwarp();
    if (c.lane == 0) mbar_arrive(smem_u32(c.smem + U_OFF_BARS) + 16 + 8 * (m & 1u));
    float y = __uint_as_float(v[0]), f = 0.25f;
#pragma unroll
    for (int n = 1; n < 8; ++n) { y = fmaf(__uint_as_float(v[n]), f, y); f *= 0.125f; }
    return y * c.inv_g;
}

// One projection phase, consumer side: same call as the mma.sync variant (whose warp split the template arguments
// describe).
template <int RT, int KS, bool TWO>
__device__ __forceinline__ void mma_phase_ts(const DecodeParams& P, Ctx& c, int nchunks, int K, bool sync_parts) {
    (void)sync_parts;
    c.part = c.part_base + ((c.part_flip++ & 1u) ? PART_HALF : 0);
    u_prepare_acts(P, c, K);
    trace_point(P, c);
    if (nchunks > 2) { fail(P, c, ST_MISALIGNED); nchunks = 2; }
    if (nchunks > 0) {
        const uint32_t m = c.mma_n++;
        u_wait_product(P, c, m);
        trace_point(P, c);
        if (c.warp < 2) c.part[32 * c.warp + c.lane] = u_read_row(c, m);
        for (int q = 0; q < nchunks; ++q, ++c.it) release_stage(c, c.it % NSTAGE);
    }
}
template <int RT, int KS>
__device__ __forceinline__ float part_sum_ts(const Ctx& c, int r) { return c.part[r]; }
__device__ __forceinline__ float tensor_scale_of(const LW& lw, int slot) {
    return __ldg(reinterpret_cast<const float*>(lw.ptrs[slot + 2]));
}
#endif

#if MK_WFMT < 2
// Runs all chunks of a phase; partial sums land in part[(q * 16 + warp) * 16 + tile_row].
template <int NLOAD, int ROWS>
__device__ __forceinline__ void mma_phase(const DecodeParams& P, Ctx& c, int nchunks_in, int K) {
    int nchunks = nchunks_in;
    // alternate halves: a slow warp may still be reading the previous phase's sums in its epilogue
    c.part = c.part_base + ((c.part_flip++ & 1u) ? PART_HALF : 0);
    uint32_t b[2 * NLOAD][2];
    load_bfrags<NLOAD>(reinterpret_cast<const uint32_t*>(c.xs) + c.warp * XSW, c.lane, b);
    if (nchunks > 4) { fail(P, c, ST_MISALIGNED); nchunks = 4; }   // never reached for grids >= MIN_GRID
    // Chunks two at a time: the weights are in the ring long before the activation is (the waits below practically
    // never block), so what a chunk costs is its own dependent chain load -> MMA -> shuffle -> store; two independent
    // chains in flight per warp hide most of one of them.
    int q = 0;
    // (all four chunks of an input projection in one go measured no better than two pairs)
#pragma unroll 1
    for (; q + 2 <= nchunks; q += 2, c.it += 2) {
        const uint32_t s0 = c.it % NSTAGE, s1 = (c.it + 1) % NSTAGE;
        wait_full(P, c, s0, (c.it / NSTAGE) & 1u);
        wait_full(P, c, s1, ((c.it + 1) / NSTAGE) & 1u);
#if MK_WFMT == 0
        if (ROWS == 4) {
            mma_chunk_pair4<NLOAD>(c.smem + OFF_RING + s0 * STAGE_BYTES, c.smem + OFF_RING + s1 * STAGE_BYTES, K, c.warp, c.lane, b,
                                   c.part + (q * NCW + c.warp) * 16, c.part + ((q + 1) * NCW + c.warp) * 16);
        } else
#endif
        {
            mma_chunk<NLOAD, ROWS>(c.smem + OFF_RING + s0 * STAGE_BYTES, K, c.warp, c.lane, b, c.part + (q * NCW + c.warp) * 16);
            mma_chunk<NLOAD, ROWS>(c.smem + OFF_RING + s1 * STAGE_BYTES, K, c.warp, c.lane, b, c.part + ((q + 1) * NCW + c.warp) * 16);
        }
        release_stage(c, s0);
        release_stage(c, s1);
    }
    if (q < nchunks) {
        const uint32_t stage = c.it % NSTAGE;
        wait_full(P, c, stage, (c.it / NSTAGE) & 1u);
        mma_chunk<NLOAD, ROWS>(c.smem + OFF_RING + stage * STAGE_BYTES, K, c.warp, c.lane, b, c.part + (q * NCW + c.warp) * 16);
        release_stage(c, stage);
        ++c.it;
    }
}

__device__ __forceinline__ float part_sum(const Ctx& c, int q, int row) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) s += c.part[(q * NCW + w) * 16 + row];
    return s;
}
#endif

// ---- activation staging -----------------------------------------------------------------

__device__ __forceinline__ void load_norm_w(const void* w, int tid, float& w0, float& w1) {
    const uint32_t raw = __ldg(reinterpret_cast<const uint32_t*>(w) + tid);
    w0 = 1.0f + bf_lo(raw);
    w1 = 1.0f + bf_hi(raw);
}

// Thread tid fetches elements (2 tid, 2 tid + 1) of the residual stream: from the embedding row
// for the first layer, else from the flagged words of the previous down-projection.
__device__ __forceinline__ float2 fetch_hidden2(const DecodeParams& P, Ctx& c, const __nv_bfloat16* embed_row,
                                                const unsigned long long* words, uint32_t epoch) {
    if (embed_row) {
        const uint32_t raw = __ldg(reinterpret_cast<const uint32_t*>(embed_row) + c.tid);
        return make_float2(bf_lo(raw), bf_hi(raw));
    }
    return poll2(P, c, words + 2 * c.tid, epoch);
}

// RMSNorm of the 1024-vector held two elements per thread; result (optionally rounded to bf16)
// goes to this warp's staging slice, whose 64 elements are exactly the warp's K-slice.
// reference: megakernel/kernel.cu:189-231
__device__ __forceinline__ float2 rmsnorm_to_slice(Ctx& c, float2 v, float w0, float w1, bool round_to_bf16) {
    const float ss = warp_sum(v.x * v.x + v.y * v.y);
    if (c.lane == 0) c.red[c.warp] = ss;
    named_bar_sync(1, NCT);
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < NCW; ++i) tot += c.red[i];
    const float rstd = rsqrtf(tot * (1.0f / HIDDEN) + RMS_EPS);
    float x0 = v.x * rstd * w0, x1 = v.y * rstd * w1;
    if (round_to_bf16) { x0 = round_bf16(x0); x1 = round_bf16(x1); }
#if MK_WFMT >= 2
    stage_pair_ts<256>(c, 2 * c.tid, x0, x1);    // read by other warps: mma_phase_ts syncs
#else
    stage_pair(reinterpret_cast<uint32_t*>(c.xs) + c.warp * XSW, 2 * c.lane, x0, x1);
    __syncwarp();
#endif
    return make_float2(x0, x1);
}

// ---- phases -----------------------------------------------------------------------------

__device__ __forceinline__ void phase_dn_in(const DecodeParams& P, Ctx& c, const LW& lw, int layer, int dn_idx,
                            const __nv_bfloat16* embed_row) {
    const Geo g = phase_geo(T_DN_IN, c.cta, c.G, P.vocab);
    const int nloc = g.r1 - g.r0;
    const uint32_t ep = epoch_of(c, layer);
    trace_point(P, c);
    float w0, w1;
    load_norm_w(lw.ptrs[DN_IN_NORM], c.tid, w0, w1);
    // epilogue inputs that do not depend on this token: conv window and taps of the row this thread finishes
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
#if MK_WFMT >= 2
    const float ts_in = (c.tid < nloc) ? tensor_scale_of(lw, r < DN_CONV_CH ? (int)DN_W_QKV : (int)DN_W_Z) : 0.f;
#endif
#if MK_WFMT >= 1
    // beta / alpha projections are bf16 rows outside the ring: CTA c < 32 owns row c of [Wb; Wa];
    // every thread multiplies its two activations with its two weights (fetched before the wait)
    uint32_t ba_w = 0u;
    if (c.cta < 2 * DN_HEADS)
        ba_w = __ldg(reinterpret_cast<const uint32_t*>(lw.ptrs[c.cta < DN_HEADS ? (int)DN_W_B : (int)DN_W_A]) +
                     (size_t)(c.cta & (DN_HEADS - 1)) * (HIDDEN / 2) + c.tid);
    if (c.tid == NCT - 1 && c.cta >= DN_HEADS && c.cta < 2 * DN_HEADS) {
        a_log = bf2f(reinterpret_cast<const __nv_bfloat16*>(lw.ptrs[DN_A_LOG])[c.cta - DN_HEADS]);
        dt_b = bf2f(reinterpret_cast<const __nv_bfloat16*>(lw.ptrs[DN_DT_BIAS])[c.cta - DN_HEADS]);
    }
#endif
    const float2 v = fetch_hidden2(P, c, embed_row, P.ws->x_hidden[1], epoch_of(c, layer - 1));
    const float2 xn = rmsnorm_to_slice(c, v, w0, w1, true);
#if MK_WFMT >= 1
    if (c.cta < 2 * DN_HEADS) {
        const float pd = warp_sum(bf_lo(ba_w) * xn.x + bf_hi(ba_w) * xn.y);
        if (c.lane == 0) c.red[16 + c.warp] = pd;
    }
#else
    (void)xn;
#endif
    trace_point(P, c);
#if MK_WFMT >= 2
    mma_phase_ts<4, 4, true>(P, c, g.nchunks, HIDDEN, true);
#else
    mma_phase<2, 16>(P, c, g.nchunks, HIDDEN);
#endif
    trace_point(P, c);
    named_bar_sync(1, NCT);
#if MK_WFMT >= 1
    if (c.tid == NCT - 1 && c.cta < 2 * DN_HEADS) {
        float val = 0.f;
#pragma unroll
        for (int i = 0; i < NCW; ++i) val += c.red[16 + i];
        if (c.cta < DN_HEADS) {
            st_flagged(P.ws->x_dnin + DN_CONV_CH + DN_V + c.cta, 1.0f / (1.0f + expf(-val)), ep);
        } else {
            const float x = val + dt_b;
            const float sp = (x > 20.0f) ? x : log1pf(expf(x));
            st_flagged(P.ws->x_dnin + DN_CONV_CH + DN_V + c.cta, expf(-expf(a_log) * sp), ep);
        }
    }
#endif
    if (c.tid < nloc) {
#if MK_WFMT >= 2
        const float val = part_sum_ts<4, 4>(c, c.tid) * ts_in;
#else
        const float val = part_sum(c, c.tid >> 4, c.tid & 15);
#endif
        if (r < DN_CONV_CH) {
            // shift the 4-tap window, append, dot with the taps, SiLU (reference: megakernel/kernel.cu:640-646)
            const float4 ns = make_float4(cs.y, cs.z, cs.w, val);
            *reinterpret_cast<float4*>(conv_row) = ns;
            const float co = ns.x * bf_lo(cw.x) + ns.y * bf_hi(cw.x) + ns.z * bf_lo(cw.y) + ns.w * bf_hi(cw.y);
            st_flagged(P.ws->x_dnin + r, silu_f(co), ep);
        } else if (r < DN_CONV_CH + DN_V) {
            st_flagged(P.ws->x_dnin + r, val, ep);
        }
#if MK_WFMT == 0
        else if (r < DN_CONV_CH + DN_V + DN_HEADS) {
            st_flagged(P.ws->x_dnin + r, 1.0f / (1.0f + expf(-val)), ep);
        } else {
            // decay = exp(-exp(A_log) * softplus(a + dt_bias)) (reference: megakernel/kernel.cu:653-657)
            const float x = val + dt_b;
            const float sp = (x > 20.0f) ? x : log1pf(expf(x));
            st_flagged(P.ws->x_dnin + r, expf(-expf(a_log) * sp), ep);
        }
#endif
    }
    trace_point(P, c);
}

// Gated delta rule for one token; unit = (head, 16 value rows), one warp per value row.
// State row j is contiguous over the key index (reference: megakernel/kernel.cu:686-713).
// The unit's inputs (q and k of the head, 16 v values, beta, decay) are fetched once per CTA --
// one word pair per thread -- and shared through shared memory: every REC CTA polling every word
// with every warp would put thousands of pollers on the same few L2 lines.
__device__ __forceinline__ void phase_dn_rec(const DecodeParams& P, Ctx& c, int layer, int dn_idx) {
    const Geo g = phase_geo(T_DN_REC, c.cta, c.G, P.vocab);
    const uint32_t ep = epoch_of(c, layer);
    float* sh = c.xs;        // [0,128) q, [128,256) k, [256,272) v, [272] beta, [273] decay
    trace_point(P, c);
#pragma unroll 1
    for (int qi = 0; qi < g.nchunks; ++qi, ++c.it) {
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        const int u = g.r0 + qi * c.G;
        const int h = u >> 3, j0 = (u & 7) * 16;
        const unsigned long long* X = P.ws->x_dnin;
        if (c.tid < 128) {
            const unsigned long long* src = (c.tid < 64) ? X + h * DN_KEY + 2 * c.tid
                                                         : X + DN_QK + h * DN_KEY + 2 * (c.tid - 64);
            const float2 v = poll2(P, c, src, ep);
            reinterpret_cast<float2*>(sh)[c.tid] = v;
        } else if (c.tid < 128 + 18) {
            const int k = c.tid - 128;
            const unsigned long long* src = (k < 16) ? X + 2 * DN_QK + h * DN_VAL + j0 + k
                                           : (k == 16) ? X + DN_CONV_CH + DN_V + h
                                                       : X + DN_CONV_CH + DN_V + DN_HEADS + h;
            sh[256 + k] = poll1(P, c, src, ep);
        }
        named_bar_sync(1, NCT);
        const int j = j0 + c.warp;
        const float4 q4 = reinterpret_cast<const float4*>(sh)[c.lane];
        const float4 k4 = reinterpret_cast<const float4*>(sh + 128)[c.lane];
        const float vj = sh[256 + c.warp], beta = sh[272], decay = sh[273];
        float sq = q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w;
        float sk = k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w;
        float kq = q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w;
        sq = warp_sum(sq); sk = warp_sum(sk); kq = warp_sum(kq);
        const float qn = rsqrtf(sq + 1e-6f) * 0.08838834764831845f;   // 1/sqrt(128)
        const float kn = rsqrtf(sk + 1e-6f);
        kq *= qn * kn;
        if (qi == 0) trace_point(P, c);
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
        if (c.lane == 0) st_flagged(P.ws->x_o + h * DN_VAL + j, decay * sqv + err * kq, ep);
        if (qi == 0) trace_point(P, c);
        release_stage(c, stage);
        if (qi + 1 < g.nchunks) named_bar_sync(1, NCT);     // the shared inputs are rewritten by the next unit
    }
    if (g.nchunks == 0) { trace_point(P, c); trace_point(P, c); }
    trace_point(P, c);
}

// out-projection (K = 2048, 8 rows per chunk) + residual -> bf16-rounded hidden words
__device__ __forceinline__ void outproj_rows(const DecodeParams& P, Ctx& c, const Geo& g, int type, float resid, uint32_t ep,
                                             float tscale) {
    (void)type; (void)tscale;
    const int nloc = g.r1 - g.r0;
#if MK_WFMT >= 2
    mma_phase_ts<1, 8, false>(P, c, g.nchunks, 2048, true);
#else
    mma_phase<4, 8>(P, c, g.nchunks, 2048);
#endif
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nloc) {
#if MK_WFMT >= 2
        const float y = part_sum_ts<1, 8>(c, c.tid) * tscale + resid;
#else
        const float y = part_sum(c, c.tid >> 3, c.tid & 7) + resid;
#endif
        st_flagged(P.ws->x_hidden[0] + g.r0 + c.tid, round_bf16(y), ep);
    }
    trace_point(P, c);
}

__device__ __forceinline__ float fetch_resid_in(const DecodeParams& P, Ctx& c, const __nv_bfloat16* embed_row, int row,
                                                int layer) {
    if (embed_row) return bf2f(embed_row[row]);
    return poll1(P, c, P.ws->x_hidden[1] + row, epoch_of(c, layer - 1));
}

// out-proj of a DeltaNet layer; staging fuses the gated RMSNorm (plain weight) * SiLU(z): warp w
// owns head w, whose 128 values are exactly its K-slice (reference: megakernel/kernel.cu:715-741)
__device__ __forceinline__ void phase_dn_out(const DecodeParams& P, Ctx& c, const LW& lw, int layer,
                             const __nv_bfloat16* embed_row) {
    const Geo g = phase_geo(T_DN_OUT, c.cta, c.G, P.vocab);
    const uint32_t ep = epoch_of(c, layer);
    trace_point(P, c);
    const uint2 nwr = __ldg(reinterpret_cast<const uint2*>(lw.ptrs[DN_NORM_W]) + c.lane);
    float resid = 0.f;
    if (c.tid < g.r1 - g.r0) resid = fetch_resid_in(P, c, embed_row, g.r0 + c.tid, layer);
    {
        const int h = c.warp;
        const unsigned long long* Z = P.ws->x_dnin + DN_CONV_CH + h * DN_VAL + 4 * c.lane;
        const unsigned long long* O = P.ws->x_o + h * DN_VAL + 4 * c.lane;
        const unsigned long long* const p2[4] = {Z, Z + 2, O, O + 2};
        float2 v2[4];
        poll2_batch<4>(P, c, p2, ep, v2);
        const float2 za = v2[0], zb = v2[1], oa = v2[2], ob = v2[3];
        const float ss = warp_sum(oa.x * oa.x + oa.y * oa.y + ob.x * ob.x + ob.y * ob.y);
        const float rstd = rsqrtf(ss * (1.0f / DN_VAL) + RMS_EPS);
        float4 x;
        x.x = oa.x * rstd * bf_lo(nwr.x) * silu_f(za.x);
        x.y = oa.y * rstd * bf_hi(nwr.x) * silu_f(za.y);
        x.z = ob.x * rstd * bf_lo(nwr.y) * silu_f(zb.x);
        x.w = ob.y * rstd * bf_hi(nwr.y) * silu_f(zb.y);
#if MK_WFMT >= 2
        stage_pair_ts<256>(c, 128 * c.warp + 4 * c.lane, x.x, x.y);
        stage_pair_ts<256>(c, 128 * c.warp + 4 * c.lane + 2, x.z, x.w);
#else
        uint32_t* xw = reinterpret_cast<uint32_t*>(c.xs) + c.warp * XSW;
        stage_pair(xw, 4 * c.lane, x.x, x.y);
        stage_pair(xw, 4 * c.lane + 2, x.z, x.w);
        __syncwarp();
#endif
    }
    trace_point(P, c);
#if MK_WFMT >= 2
    outproj_rows(P, c, g, T_DN_OUT, resid, ep, tensor_scale_of(lw, DN_W_OUT));
#else
    outproj_rows(P, c, g, T_DN_OUT, resid, ep, 1.0f);
#endif
}

__device__ __forceinline__ void phase_fa_in(const DecodeParams& P, Ctx& c, const LW& lw, int layer,
                            const __nv_bfloat16* embed_row) {
    const Geo g = phase_geo(T_FA_IN, c.cta, c.G, P.vocab);
    const int nloc = g.r1 - g.r0;
    const uint32_t ep = epoch_of(c, layer);
    trace_point(P, c);
    float w0, w1;
    load_norm_w(lw.ptrs[FA_IN_NORM], c.tid, w0, w1);
    const float2 v = fetch_hidden2(P, c, embed_row, P.ws->x_hidden[1], epoch_of(c, layer - 1));
    rmsnorm_to_slice(c, v, w0, w1, true);
    trace_point(P, c);
#if MK_WFMT >= 2
    float ts_in = 0.f;
    if (c.tid < nloc) {
        const int r = g.r0 + c.tid;
        ts_in = tensor_scale_of(lw, r < FA_QPROJ ? (int)FA_W_Q : (r < FA_QPROJ + FA_KV_SIZE ? (int)FA_W_K : (int)FA_W_V));
    }
    mma_phase_ts<4, 4, true>(P, c, g.nchunks, HIDDEN, true);
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nloc) st_flagged(P.ws->x_fain + g.r0 + c.tid, part_sum_ts<4, 4>(c, c.tid) * ts_in, ep);
#else
    mma_phase<2, 16>(P, c, g.nchunks, HIDDEN);
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nloc)      // rows 0..4095: per head [q(256) | gate(256)]; then k[512], v[512]
        st_flagged(P.ws->x_fain + g.r0 + c.tid, part_sum(c, c.tid >> 4, c.tid & 15), ep);
#endif
    trace_point(P, c);
}

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
    f[0] = bf_lo(u.x); f[1] = bf_hi(u.x); f[2] = bf_lo(u.y); f[3] = bf_hi(u.y);
    f[4] = bf_lo(u.z); f[5] = bf_hi(u.z); f[6] = bf_lo(u.w); f[7] = bf_hi(u.w);
}

// per-head RMSNorm(1+w) + partial RoPE on lane-strided dims d = lane + 32 e
// (dims i and i+32 of the rotary pair sit in the same lane).  reference: megakernel/kernel.cu:462-499
__device__ __forceinline__ void head_norm_rope(const DecodeParams& P, Ctx& c, const unsigned long long* src, uint32_t ep,
                                               const void* wn, int pos, float* n) {
    float ss = 0.f;
    {
        const unsigned long long* b0 = src + c.lane;
        const unsigned long long* const p1[8] = {b0, b0 + 32, b0 + 64, b0 + 96, b0 + 128, b0 + 160, b0 + 192, b0 + 224};
        float v[8];
        poll1_batch<8>(P, c, p1, ep, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) { n[e] = v[e]; ss += v[e] * v[e]; }
    }
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss * (1.0f / FA_HEAD_DIM) + RMS_EPS);
#pragma unroll
    for (int e = 0; e < 8; ++e)
        n[e] = n[e] * rstd * (1.0f + bf2f(reinterpret_cast<const __nv_bfloat16*>(wn)[c.lane + 32 * e]));
    (void)pos;
    const float cs = c.rope[c.lane], sn = c.rope[32 + c.lane];      // this step's position, computed at step start
    const float a = n[0], b = n[1];
    n[0] = a * cs - b * sn;
    n[1] = b * cs + a * sn;
}

// Split-KV decode attention.  Unit = (KV head, chunk of positions), one unit per CTA at most.  The unit's
// K and V rows arrive through the weight ring (issued by the producer warp long before the query exists),
// the row of the current position is patched in shared memory by the unit that owns it (and appended to the
// cache).  The 4 query heads of the KV head are rows of one MMA tile: rows 0-3 carry the bf16 head of each
// (scaled) query, rows 4-7 the bf16 remainder, so q . k keeps ~16 mantissa bits; the softmax weights take the
// same two-row form into P . V.  Warps 0-3 each compute all scores and 64 of the 256 output dims; there is no
// cross-warp merge.  Each unit leaves (m, l, o[256]) per head in the workspace and publishes its ready word;
// the o-proj phase merges the chunks.  reference: megakernel/kernel.cu:506-560
__device__ __forceinline__ void att_mma(float (&c4)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c4[0]), "+f"(c4[1]), "+f"(c4[2]), "+f"(c4[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void att_ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void att_ldsm4t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
// x as a pair (bf16 head, bf16 remainder); `lo_part` selects which one this lane carries
__device__ __forceinline__ uint32_t att_pack(float x, float y, bool lo_part) {
    const __nv_bfloat16 xh = __float2bfloat16_rn(x), yh = __float2bfloat16_rn(y);
    __nv_bfloat162 r = lo_part ? __floats2bfloat162_rn(x - __bfloat162float(xh), y - __bfloat162float(yh))
                               : __halves2bfloat162(xh, yh);
    return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ void phase_fa_att(const DecodeParams& P, Ctx& c, const LW& lw, int layer, int fa_idx) {
    const int pos = c.pos, L = pos + 1;
    const uint32_t ep = epoch_of(c, layer);
    const Geo geo = phase_geo(T_FA_ATT, c.cta, c.G, P.vocab, pos);
    // scratch: query tile [8 rows][264] bf16 (rows 0-3 heads, 4-7 remainders), probability tile [8][72] bf16,
    // the current position's key / value row, per-warp row maxima and sums
    constexpr int QROW = FA_HEAD_DIM + 8, PROW = 64 + 8;
    __nv_bfloat16* qt = reinterpret_cast<__nv_bfloat16*>(c.xs);
    __nv_bfloat16* pt = qt + 8 * QROW;
    __nv_bfloat16* krow = pt + 8 * PROW;
    __nv_bfloat16* vrow = krow + FA_HEAD_DIM;
    float* smax = reinterpret_cast<float*>(vrow + FA_HEAD_DIM);      // [4 warps][4 heads]
    float* ssum = smax + 16;
    trace_point(P, c);
    if (geo.nchunks == 0) { trace_point(P, c); trace_point(P, c); }
    if (geo.nchunks > 0) {
        const int u = c.cta;
        int g, ch, p_lo, p_hi;
        att_unit_range(L, u, g, ch, p_lo, p_hi);
        const bool owner = (pos >= p_lo && pos < p_hi);
        // The first K/V tile does not depend on this step's projections (the producer fetched it from the caches long
        // ago): take it over and pad it while the query is still on its way.
        {
#pragma unroll
            for (int k = 0; k < 4; ++k) wait_full(P, c, (c.it + k) % NSTAGE, ((c.it + k) / NSTAGE) & 1u);
            const int nvalid0 = min(64, p_hi - p_lo);
            if (nvalid0 < 64 && c.warp >= 6) {
                for (int r = nvalid0 + (c.warp - 6); r < 64; r += NCW - 6) {
                    char* dst = c.smem + OFF_RING + ((c.it + 2 + (r >> 5)) % NSTAGE) * STAGE_BYTES + att_tile_off(r & 31, 16 * c.lane);
                    *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
                }
            }
        }
        const int r_own = pos - p_lo;                 // row of the current position, if it lies in the first tile
        const bool patch0 = owner && r_own < 64;
        if (c.warp < 4) {
            float n[8];
            head_norm_rope(P, c, P.ws->x_fain + (g * FA_GQA + c.warp) * 2 * FA_HEAD_DIM, ep, lw.ptrs[FA_Q_NORM], pos, n);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float x = n[e] * 0.0625f;                       // 1 / sqrt(head_dim), exact
                const __nv_bfloat16 hi = __float2bfloat16_rn(x);
                qt[c.warp * QROW + c.lane + 32 * e] = hi;
                qt[(c.warp + 4) * QROW + c.lane + 32 * e] = __float2bfloat16_rn(x - __bfloat162float(hi));
            }
        } else if (c.warp == 4 && owner) {
            float n[8];
            head_norm_rope(P, c, P.ws->x_fain + FA_QPROJ + g * FA_HEAD_DIM, ep, lw.ptrs[FA_K_NORM], pos, n);
            __nv_bfloat16* Kb = reinterpret_cast<__nv_bfloat16*>(P.k_cache) + ((size_t)(fa_idx * FA_KV_HEADS + g) * P.max_seq_len + pos) * FA_HEAD_DIM;
#pragma unroll
            char* tile = c.smem + OFF_RING + ((c.it + (r_own >> 5)) % NSTAGE) * STAGE_BYTES;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const __nv_bfloat16 v = __float2bfloat16_rn(n[e]);
                const int d = c.lane + 32 * e;
                Kb[d] = v;
                krow[d] = v;
                // straight into the tile (the producer fences before it refills the stage)
                if (patch0) *reinterpret_cast<__nv_bfloat16*>(tile + att_tile_off(r_own & 31, 2 * d) + ((2 * d) & 15)) = v;
            }
        } else if (c.warp == 5 && owner) {
            const unsigned long long* b0 = P.ws->x_fain + FA_QPROJ + FA_KV_SIZE + g * FA_HEAD_DIM + c.lane;
            const unsigned long long* const p1[8] = {b0, b0 + 32, b0 + 64, b0 + 96, b0 + 128, b0 + 160, b0 + 192, b0 + 224};
            float v[8];
            poll1_batch<8>(P, c, p1, ep, v);
            __nv_bfloat16* Vb = reinterpret_cast<__nv_bfloat16*>(P.v_cache) + ((size_t)(fa_idx * FA_KV_HEADS + g) * P.max_seq_len + pos) * FA_HEAD_DIM;
#pragma unroll
            char* tile = c.smem + OFF_RING + ((c.it + 2 + (r_own >> 5)) % NSTAGE) * STAGE_BYTES;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const __nv_bfloat16 b = __float2bfloat16_rn(v[e]);
                const int d = c.lane + 32 * e;
                Vb[d] = b;
                vrow[d] = b;
                if (patch0) *reinterpret_cast<__nv_bfloat16*>(tile + att_tile_off(r_own & 31, 2 * d) + ((2 * d) & 15)) = b;
            }
        }
        named_bar_sync(1, NCT);
        trace_point(P, c);                 // query / key / value of this position ready

        const int g8 = c.lane >> 2, t4 = c.lane & 3;
        const bool lo_part = g8 >= 4;
        float oacc[4][4];                  // warps 0-7: output dims [32 warp, 32 warp + 32)
#pragma unroll
        for (int n = 0; n < 4; ++n) { oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f; }
        float mrun = -1e30f, lrun = 0.f;
        const int ntile = geo.nchunks >> 2;
#pragma unroll 1
        for (int tile = 0; tile < ntile; ++tile) {
            uint32_t stg[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t itk = c.it + k;
                wait_full(P, c, itk % NSTAGE, (itk / NSTAGE) & 1u);
                stg[k] = smem_u32(c.smem + OFF_RING + (itk % NSTAGE) * STAGE_BYTES);
            }
            const int tbase = p_lo + tile * 64, nvalid = min(64, p_hi - tbase);
            // patch the row of the current position, zero the value rows past the end of the chunk (first tile: done above)
            if (tile > 0 && owner && pos >= tbase && pos < tbase + 64 && c.warp >= 4 && c.warp < 6) {
                const int r = pos - tbase;
                char* dst = c.smem + OFF_RING + ((c.it + (c.warp == 4 ? 0 : 2) + (r >> 5)) % NSTAGE) * STAGE_BYTES + att_tile_off(r & 31, 16 * c.lane);
                const uint4* srcv = reinterpret_cast<const uint4*>(c.warp == 4 ? krow : vrow);
                *reinterpret_cast<uint4*>(dst) = srcv[c.lane];      // (the producer fences before it refills this stage)
            }
            if (tile > 0 && nvalid < 64 && c.warp >= 6) {
                for (int r = nvalid + (c.warp - 6); r < 64; r += NCW - 6) {
                    char* dst = c.smem + OFF_RING + ((c.it + 2 + (r >> 5)) % NSTAGE) * STAGE_BYTES + att_tile_off(r & 31, 16 * c.lane);
                    *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
                }
            }
            if (tile > 0) named_bar_sync(1, NCT);
            if (tile == 0) trace_point(P, c);      // first K/V tile landed and patched
            float sc[2][2];
            if (c.warp < 4) {
                // scores of keys [16 warp, 16 warp + 16): rows = (head, part)
                float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                const int brow = (c.lane & 7) + (c.lane >> 4) * 8, bcol = ((c.lane >> 3) & 1) * 16;
                const uint32_t kb = stg[c.warp >> 1];
                const int krow_i = (c.warp & 1) * 16 + brow;
                const uint32_t* qrow = reinterpret_cast<const uint32_t*>(qt + g8 * QROW) + t4;
#pragma unroll
                for (int ks = 0; ks < 16; ++ks) {
                    uint32_t b0, b1, b2, b3;
                    att_ldsm4(kb + att_tile_off(krow_i, bcol + ks * 32), b0, b1, b2, b3);
                    const uint32_t a0 = qrow[ks * 8], a2 = qrow[ks * 8 + 4];
                    att_mma(acc[0], a0, a2, b0, b1);
                    att_mma(acc[1], a0, a2, b2, b3);
                }
                float tmax = -1e30f;
#pragma unroll
                for (int n = 0; n < 2; ++n) {
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        float v = acc[n][e] + __shfl_xor_sync(0xffffffffu, acc[n][e], 16);   // head + remainder rows
                        if (c.warp * 16 + n * 8 + 2 * t4 + e >= nvalid) v = -1e30f;
                        sc[n][e] = v;
                        tmax = fmaxf(tmax, v);
                    }
                }
                tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
                tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
                if (!lo_part && t4 == 0) smax[c.warp * 4 + g8] = tmax;
                named_bar_sync(2, 128);
                const int h = g8 & 3;
                const float mn = fmaxf(fmaxf(fmaxf(smax[h], smax[4 + h]), fmaxf(smax[8 + h], smax[12 + h])), mrun);
                float rs = 0.f;
#pragma unroll
                for (int n = 0; n < 2; ++n) {
                    const float p0 = __expf(sc[n][0] - mn), p1 = __expf(sc[n][1] - mn);
                    rs += p0 + p1;
                    *reinterpret_cast<uint32_t*>(pt + g8 * PROW + c.warp * 16 + n * 8 + 2 * t4) = att_pack(p0, p1, lo_part);
                }
                rs += __shfl_xor_sync(0xffffffffu, rs, 1);
                rs += __shfl_xor_sync(0xffffffffu, rs, 2);
                if (!lo_part && t4 == 0) ssum[c.warp * 4 + g8] = rs;
            }
            if (c.warp < 8) {
                named_bar_sync(3, 256);
                const int h = g8 & 3;
                const float mn = fmaxf(fmaxf(fmaxf(smax[h], smax[4 + h]), fmaxf(smax[8 + h], smax[12 + h])), mrun);
                const float corr = __expf(mrun - mn);
                lrun = lrun * corr + (ssum[h] + ssum[4 + h]) + (ssum[8 + h] + ssum[12 + h]);
                mrun = mn;
#pragma unroll
                for (int n = 0; n < 4; ++n) { oacc[n][0] *= corr; oacc[n][1] *= corr; }
                const int trow = (c.lane & 7) + ((c.lane >> 3) & 1) * 8, tcol = (c.lane >> 4) * 16;
                const uint32_t* prow = reinterpret_cast<const uint32_t*>(pt + g8 * PROW) + t4;
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint32_t a0 = prow[ks * 8], a2 = prow[ks * 8 + 4];
#pragma unroll
                    for (int np = 0; np < 2; ++np) {
                        uint32_t b0, b1, b2, b3;
                        att_ldsm4t(stg[2 + (ks >> 1)] + att_tile_off((ks & 1) * 16 + trow, (c.warp * 32 + np * 16) * 2 + tcol), b0, b1, b2, b3);
                        att_mma(oacc[2 * np], a0, a2, b0, b1);
                        att_mma(oacc[2 * np + 1], a0, a2, b2, b3);
                    }
                }
            }
            named_bar_sync(1, NCT);
#pragma unroll
            for (int k = 0; k < 4; ++k) release_stage(c, (c.it + k) % NSTAGE);
            c.it += 4;
        }
        if (c.warp < 8) {
            float* dst = P.ws->attn_part + ((size_t)(g * FA_GQA + (g8 & 3)) * ATT_MAX_CHUNKS + ch) * ATT_PART_STRIDE;
#pragma unroll
            for (int n = 0; n < 4; ++n) {
                const float o0 = oacc[n][0] + __shfl_xor_sync(0xffffffffu, oacc[n][0], 16);
                const float o1 = oacc[n][1] + __shfl_xor_sync(0xffffffffu, oacc[n][1], 16);
                if (!lo_part) *reinterpret_cast<float2*>(dst + 4 + c.warp * 32 + n * 8 + 2 * t4) = make_float2(o0, o1);
            }
            if (c.warp == 0 && !lo_part && t4 == 0) { dst[0] = mrun; dst[1] = lrun; }
        }
        named_bar_sync(1, NCT);
        if (c.tid == 0)       // the partials of this unit are complete: publish (release orders the CTA's stores)
            asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(P.ws->att_ready + u), "r"(ep) : "memory");
    }
    trace_point(P, c);
}

// o-proj of an attention layer; staging waits for the attention units, merges their chunks and
// applies the sigmoid gate: warp w owns dims (w&1)*128.. of head w/2, which is its K-slice
// (reference: megakernel/kernel.cu:542-570)
__device__ __forceinline__ void phase_fa_out(const DecodeParams& P, Ctx& c, const LW& lw, int layer,
                             const __nv_bfloat16* embed_row) {
    const Geo g = phase_geo(T_FA_OUT, c.cta, c.G, P.vocab);
    const int NC = att_num_chunks(c.pos + 1);
    const uint32_t ep = epoch_of(c, layer);
    trace_point(P, c);
    float resid = 0.f;
    if (c.tid < g.r1 - g.r0) resid = fetch_resid_in(P, c, embed_row, g.r0 + c.tid, layer);
    {
        const int head = c.warp >> 1, d4 = (c.warp & 1) * 128 + 4 * c.lane;
        const unsigned long long* G4 = P.ws->x_fain + head * 2 * FA_HEAD_DIM + FA_HEAD_DIM + d4;
        const float2 ga = poll2(P, c, G4, ep), gb = poll2(P, c, G4 + 2, ep);
        if (c.warp == 0 && c.lane < FA_KV_HEADS * NC) {   // one warp waits for the attention units of this layer
            uint64_t t0 = 0;
            uint32_t n = 0;
            while (ld_acquire_gpu(P.ws->att_ready + c.lane) != ep)
                if ((++n & 1023u) == 0 && poll_give_up(P, c, t0)) break;
        }
        named_bar_sync(1, NCT);
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
        const float inv = 1.0f / den;
        float4 x;
        x.x = o.x * inv * sigmoid_f(ga.x); x.y = o.y * inv * sigmoid_f(ga.y);
        x.z = o.z * inv * sigmoid_f(gb.x); x.w = o.w * inv * sigmoid_f(gb.y);
#if MK_WFMT >= 2
        stage_pair_ts<256>(c, 128 * c.warp + 4 * c.lane, x.x, x.y);
        stage_pair_ts<256>(c, 128 * c.warp + 4 * c.lane + 2, x.z, x.w);
#else
        uint32_t* xw = reinterpret_cast<uint32_t*>(c.xs) + c.warp * XSW;
        stage_pair(xw, 4 * c.lane, x.x, x.y);
        stage_pair(xw, 4 * c.lane + 2, x.z, x.w);
        __syncwarp();
#endif
    }
    trace_point(P, c);
#if MK_WFMT >= 2
    outproj_rows(P, c, g, T_FA_OUT, resid, ep, tensor_scale_of(lw, FA_W_O));
#else
    outproj_rows(P, c, g, T_FA_OUT, resid, ep, 1.0f);
#endif
}

// post norm + SiLU(Wg x) * (Wu x): tile rows 0-7 are gate rows, 8-15 the matching up rows
// (reference: megakernel/kernel.cu:313-347, 572-578)
__device__ __forceinline__ void phase_gateup(const DecodeParams& P, Ctx& c, const LW& lw, int layer) {
    const Geo g = phase_geo(T_GATEUP, c.cta, c.G, P.vocab);
    const int nout = g.r1 - g.r0;
    const uint32_t ep = epoch_of(c, layer);
    trace_point(P, c);
    float w0, w1;
    load_norm_w(lw.ptrs[lw.layer_type == 0 ? (int)DN_POST_NORM : (int)FA_POST_NORM], c.tid, w0, w1);
    const float2 v = poll2(P, c, P.ws->x_hidden[0] + 2 * c.tid, ep);
    rmsnorm_to_slice(c, v, w0, w1, true);
    trace_point(P, c);
#if MK_WFMT >= 2
    const bool dnl = (lw.layer_type == 0);
    const float ts_g = tensor_scale_of(lw, dnl ? (int)DN_W_GATE : (int)FA_W_GATE);
    const float ts_u = tensor_scale_of(lw, dnl ? (int)DN_W_UP : (int)FA_W_UP);
    mma_phase_ts<4, 4, true>(P, c, g.nchunks, HIDDEN, true);
#else
    mma_phase<2, 16>(P, c, g.nchunks, HIDDEN);
#endif
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nout) {
#if MK_WFMT >= 2
        const float gv = part_sum_ts<4, 4>(c, c.tid) * ts_g;
        const float uv = part_sum_ts<4, 4>(c, UP_ROW0 + c.tid) * ts_u;
#else
        const float gv = part_sum(c, c.tid >> 3, c.tid & 7);
        const float uv = part_sum(c, c.tid >> 3, 8 + (c.tid & 7));
#endif
        st_flagged(P.ws->x_mlp + g.r0 + c.tid, silu_f(gv) * uv, ep);
    }
    trace_point(P, c);
}

// down projection (K = 3584, 4 rows per chunk) + residual (reference: megakernel/kernel.cu:350-384)
__device__ __forceinline__ void phase_down(const DecodeParams& P, Ctx& c, const LW& lw, int layer) {
    (void)lw;
    const Geo g = phase_geo(T_DOWN, c.cta, c.G, P.vocab);
    const int nloc = g.r1 - g.r0;
    const uint32_t ep = epoch_of(c, layer);
    trace_point(P, c);
    float resid = 0.f;
    if (c.tid < nloc) resid = poll1(P, c, P.ws->x_hidden[0] + g.r0 + c.tid, ep);
    {
        float xv[7];
        const unsigned long long* base = P.ws->x_mlp + c.warp * XK + c.lane;
        const unsigned long long* const p1[7] = {base, base + 32, base + 64, base + 96, base + 128, base + 160, base + 192};
        poll1_batch<7>(P, c, p1, ep, xv);
#if MK_WFMT >= 2
#pragma unroll
        for (int k = 0; k < 7; ++k) stage_one_ts<256>(c, 224 * c.warp + c.lane + 32 * k, xv[k]);
#else
        uint32_t* xw = reinterpret_cast<uint32_t*>(c.xs) + c.warp * XSW;
#pragma unroll
        for (int k = 0; k < 7; ++k) stage_one(xw, c.lane + 32 * k, xv[k]);
#endif
        __syncwarp();
    }
    trace_point(P, c);
#if MK_WFMT >= 2
    const float ts_d = tensor_scale_of(lw, lw.layer_type == 0 ? (int)DN_W_DOWN : (int)FA_W_DOWN);
    mma_phase_ts<1, 14, false>(P, c, g.nchunks, INTER, true);
#else
    mma_phase<7, 4>(P, c, g.nchunks, INTER);
#endif
    trace_point(P, c);
    named_bar_sync(1, NCT);
    if (c.tid < nloc) {
#if MK_WFMT >= 2
        const float y = part_sum_ts<1, 14>(c, c.tid) * ts_d + resid;
#else
        const float y = part_sum(c, c.tid >> 2, c.tid & 3) + resid;
#endif
        st_flagged(P.ws->x_hidden[1] + g.r0 + c.tid, round_bf16(y), ep);
    }
    trace_point(P, c);
}

// ---- LM head: scalar streaming rows (one warp per ring slot) --------------------------------

__device__ __forceinline__ float dot_row1024(const char* row, int lane, const float* xr) {
    const uint4* wp = reinterpret_cast<const uint4*>(row) + lane;
    const uint4 w0 = wp[0], w1 = wp[32], w2 = wp[64], w3 = wp[96];
    float a0 = dot8(w0, xr, 0.f), a1 = dot8(w1, xr + 8, 0.f);
    a0 = dot8(w2, xr + 16, a0); a1 = dot8(w3, xr + 24, a1);
    return a0 + a1;
}

// final norm (f32, not rounded) + LM head + argmax, lowest index winning exact ties
// (reference: megakernel/kernel.cu:763-826, 905-920)
__device__ __forceinline__ void phase_lm(const DecodeParams& P, Ctx& c) {
    const Geo g = phase_geo(T_LM, c.cta, c.G, P.vocab);
    const int nloc = g.r1 - g.r0;
    trace_point(P, c);
    float w0, w1;
    load_norm_w(P.final_norm, c.tid, w0, w1);
    const float2 v = poll2(P, c, P.ws->x_hidden[1] + 2 * c.tid, epoch_of(c, P.num_layers - 1));
    {
        const float ss = warp_sum(v.x * v.x + v.y * v.y);
        if (c.lane == 0) c.red[c.warp] = ss;
        named_bar_sync(1, NCT);
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < NCW; ++i) tot += c.red[i];
        const float rstd = rsqrtf(tot * (1.0f / HIDDEN) + RMS_EPS);
        const float2 x = make_float2(v.x * rstd * w0, v.y * rstd * w1);
        reinterpret_cast<float2*>(c.xs)[c.tid] = x;
        if (c.cta == 0) {     // outputs of the reference signature: last hidden (bf16) and its final norm (f32)
            reinterpret_cast<float2*>(P.normalized)[c.tid] = x;
            reinterpret_cast<__nv_bfloat162*>(P.hidden)[c.tid] = __floats2bfloat162_rn(v.x, v.y);
        }
        named_bar_sync(1, NCT);
    }
    trace_point(P, c);
    float bestv = -INFINITY;
    int besti = 0x7fffffff;
#if MK_WFMT == 0
    float xr[32];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const float4 a = *reinterpret_cast<const float4*>(c.xs + it * 256 + c.lane * 8);
        const float4 b = *reinterpret_cast<const float4*>(c.xs + it * 256 + c.lane * 8 + 4);
        xr[it * 8 + 0] = a.x; xr[it * 8 + 1] = a.y; xr[it * 8 + 2] = a.z; xr[it * 8 + 3] = a.w;
        xr[it * 8 + 4] = b.x; xr[it * 8 + 5] = b.y; xr[it * 8 + 6] = b.z; xr[it * 8 + 7] = b.w;
    }
    const bool penal = (P.rep_penalty > 1.0f) && (P.seen_mask != nullptr);
#pragma unroll 1
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
            if (P.logits_out && c.lane == 0) P.logits_out[row] = acc;
            if (acc > bestv) { bestv = acc; besti = row; }
        }
        release_stage(c, stage);
    }
#elif MK_WFMT == 3
    // LM head on tcgen05: the final-normed vector is quantised once; the MMA warp works through the CTA's chunk images
    // (56 rows each) on its own, two accumulator buffers ahead at most, while warps 0 and 1 read the products back.
    {
        const float2 xv = reinterpret_cast<const float2*>(c.xs)[c.tid];
        c.amax = fmaxf(fabsf(xv.x), fabsf(xv.y));
        u_prepare_acts(P, c, HIDDEN);
    }
    const float ts_lm = __ldg(P.lm_tensor_scale);
#pragma unroll 1
    for (int q = 0; q < g.nchunks; ++q, ++c.it) {
        const uint32_t m = c.mma_n++;
        u_wait_product(P, c, m);
        if (c.warp < 2) {
            const float acc = u_read_row(c, m) * ts_lm;
            const int lr = q * LM_RPC + c.tid;
            if (c.tid < LM_RPC && lr < nloc) {
                if (P.logits_out) P.logits_out[g.r0 + lr] = acc;
                if (acc > bestv) { bestv = acc; besti = g.r0 + lr; }
            }
        }
        release_stage(c, c.it % NSTAGE);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bestv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ov > bestv || (ov == bestv && oi < besti)) { bestv = ov; besti = oi; }
    }
#elif MK_WFMT == 2
    // LM head in the tensor-scale format on the tensor cores: a chunk is 64 packed rows with their block scales,
    // processed like a K = 1024 layer chunk (4 row tiles x 4 K parts); the final-normed vector (f32) is staged once
    // as three f16 terms.  Partial sums alternate between the two halves of `part` from chunk to chunk, so one
    // CTA barrier per chunk is enough: rows are finished by threads 0-63 while the warps start the next chunk.
    {
        const float2 xv = reinterpret_cast<const float2*>(c.xs)[c.tid];
        named_bar_sync(1, NCT);                                   // everyone has read the f32 vector: reuse the scratch
        stage_pair_ts<256>(c, 2 * c.tid, xv.x, xv.y);
        named_bar_sync(1, NCT);
    }
    const uint32_t* xw_lm = reinterpret_cast<const uint32_t*>(c.xs) + (c.warp / 4) * (3 * 256 / 2);
    const float ts_lm = __ldg(P.lm_tensor_scale) * TS_SCALE_FOLD;
#pragma unroll 1
    for (int q = 0; q < g.nchunks; ++q, ++c.it) {
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        c.part = c.part_base + ((c.part_flip++ & 1u) ? PART_HALF : 0);
        wait_full(P, c, stage, parity);
        mma_chunk_ts<4, true>(c.smem + OFF_RING + stage * STAGE_BYTES, xw_lm, HIDDEN, c.warp, c.lane, c.part + c.warp * 16);
        release_stage(c, stage);
        named_bar_sync(1, NCT);
        const int lr = q * LM_RPC + c.tid;
        if (c.tid < LM_RPC && lr < nloc) {
            const float acc = part_sum_ts<4, 4>(c, c.tid) * ts_lm;
            if (P.logits_out) P.logits_out[g.r0 + lr] = acc;
            if (acc > bestv) { bestv = acc; besti = g.r0 + lr; }
        }
    }
    // every thread holds the best of its own rows: make it warp-uniform, like the other variants leave it
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bestv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ov > bestv || (ov == bestv && oi < besti)) { bestv = ov; besti = oi; }
    }
#else
    // LM head in the 16-block E4M3 format: a chunk is 64 packed rows (512 bytes each); a warp takes
    // rows warp, warp+16, ...; a lane owns 32 weights = two blocks, whose scales are adjacent
    // bytes of the tiled scale array and are fetched from global memory ahead of the ring wait.
    float xr[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float4 a = *reinterpret_cast<const float4*>(c.xs + 32 * c.lane + 4 * j);
        xr[4 * j] = a.x; xr[4 * j + 1] = a.y; xr[4 * j + 2] = a.z; xr[4 * j + 3] = a.w;
    }
    const uint8_t* lm_scales = reinterpret_cast<const uint8_t*>(P.lm_scales);
#pragma unroll 1
    for (int q = 0; q < g.nchunks; ++q, ++c.it) {
        const uint32_t stage = c.it % NSTAGE, parity = (c.it / NSTAGE) & 1u;
        unsigned short sc[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int lr = q * LM_RPC + c.warp + 16 * k;
            const int row = g.r0 + lr;
            sc[k] = 0;
            if (lr < nloc) {
                const size_t idx = ((size_t)(row >> 7) * (HIDDEN >> 6) + (c.lane >> 1)) * 512 + (size_t)(row & 31) * 16 +
                                   (size_t)((row & 127) >> 5) * 4 + ((2 * c.lane) & 3);
                sc[k] = __ldg(reinterpret_cast<const unsigned short*>(lm_scales + idx));
            }
        }
        wait_full(P, c, stage, parity);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int lr = q * LM_RPC + c.warp + 16 * k;
            const bool valid = lr < nloc;
            float acc = 0.f;
            if (valid) {
                const uint4 pk = *(reinterpret_cast<const uint4*>(c.smem + OFF_RING + stage * STAGE_BYTES + (c.warp + 16 * k) * (HIDDEN / 2)) + c.lane);
                const __half_raw h0 = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)(sc[k] & 0xff), __NV_E4M3);
                const __half_raw h1 = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)(sc[k] >> 8), __NV_E4M3);
                const float s0 = __half2float(*reinterpret_cast<const __half*>(&h0)), s1 = __half2float(*reinterpret_cast<const __half*>(&h1));
                const uint32_t wv[4] = {pk.x, pk.y, pk.z, pk.w};
                float a0 = 0.f, a1 = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float part = 0.f;
#pragma unroll
                    for (int bb = 0; bb < 4; ++bb) {
                        const uint32_t hh = e2m1x2_to_f16x2(wv[i] >> (8 * bb));
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hh));
                        part = fmaf(f.x, xr[8 * i + 2 * bb], part);
                        part = fmaf(f.y, xr[8 * i + 2 * bb + 1], part);
                    }
                    if (i < 2) a0 += part; else a1 += part;
                }
                acc = a0 * s0 + a1 * s1;
            }
            acc = warp_sum(acc);
            if (P.logits_out && valid && c.lane == 0) P.logits_out[g.r0 + lr] = acc;
            if (valid && acc > bestv) { bestv = acc; besti = g.r0 + lr; }
        }
        release_stage(c, stage);
    }
#endif
    trace_point(P, c);
    c.part = c.part_base + ((c.part_flip++ & 1u) ? PART_HALF : 0);
    int* resi = reinterpret_cast<int*>(c.part) + 32;
    if (c.lane == 0) { c.part[c.warp] = bestv; resi[c.warp] = besti; }
    named_bar_sync(1, NCT);
    if (c.warp == 0) {
        float bv = (c.lane < NCW) ? c.part[c.lane] : -INFINITY;
        int bi = (c.lane < NCW) ? resi[c.lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (c.lane == 0) {
            P.ws->argmax_val[c.cta] = bv;
            P.ws->argmax_idx[c.cta] = bi;
            __threadfence();
            const uint32_t old = atomicAdd(&P.ws->lm_count, 1u);
            c.misc[MISC_LAST] = (old == (uint32_t)c.G - 1u) ? 1 : 0;
        }
    }
    named_bar_sync(1, NCT);
    if (c.misc[MISC_LAST] && c.warp == 0) {
        __threadfence();
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int b = c.lane; b < c.G; b += 32) {
            const float ov = __ldcg(P.ws->argmax_val + b);
            const int oi = __ldcg(P.ws->argmax_idx + b);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (c.lane == 0) {
            // a wait ran out somewhere in this launch: the argmax was taken over garbage, report -1 instead
            if (*((volatile uint32_t*)&P.ws->abort_flag) != 0u) bi = -1;
            P.out_token[c.step] = bi;
            if (P.token_feedback) *P.token_feedback = bi;
            if (P.host_token && c.step == P.steps - 1) {        // a host thread spins on the ticket (mk_decode_step_host)
                *((volatile int*)P.host_token) = bi;
                __threadfence_system();
                *((volatile uint32_t*)P.host_token + 1) = P.host_ticket;
            }
            // every CTA has finished this step: re-arm the workspace, then hand the token to the next step of this
            // launch (every CTA waits for this word before it touches the workspace again)
            P.ws->lm_count = 0u;
            P.ws->seq = c.seq + 1u;
            __threadfence();
            st_flagged(&P.ws->next_token, __int_as_float(bi), ((c.seq + 2u) << 5));
        }
    }
    trace_point(P, c);
}

#if MK_WFMT == 0 && MK_TRACE == 0
// The kernel's poll of a flagged word, on a word whose epoch never comes: see launch_wait_selftest().
__global__ void wait_selftest_kernel(const __grid_constant__ DecodeParams P) {
    __shared__ int misc[8];
    Ctx c;
    c.misc = misc;
    c.tid = threadIdx.x; c.warp = 0; c.lane = threadIdx.x; c.cta = blockIdx.x; c.G = gridDim.x;
    c.seq = __ldcg(&P.ws->seq);
    c.where = 0; c.step = 0;
    if (threadIdx.x == 0) { misc[MISC_ABORT] = 0; misc[MISC_DETAIL] = 0; }
    __syncthreads();
    // epoch of a layer index no phase ever publishes: the word keeps whatever epoch it had
    (void)poll1(P, c, P.ws->x_mlp + blockIdx.x, epoch_of(c, 30));
    __syncthreads();
    if (threadIdx.x == 0 && misc[MISC_ABORT] && P.host_status) {
        *((volatile uint32_t*)P.host_status) = (uint32_t)misc[MISC_ABORT];
        __threadfence_system();
    }
}
#endif

#if MK_WFMT == 3
constexpr int NTHR = NTHREADS + 32;        // + the warp that issues the tensor-core work
#else
constexpr int NTHR = NTHREADS;
#endif
__global__ void __launch_bounds__(NTHR, 1) decode_megakernel_bf16(const __grid_constant__ DecodeParams P) {
    extern __shared__ __align__(1024) char smem[];
    Ctx c;
    c.smem = smem;
    c.xs = reinterpret_cast<float*>(smem + OFF_SCRATCH);
    c.part_base = reinterpret_cast<float*>(smem + OFF_PART);
    c.part = c.part_base;
    c.part_flip = 0;
    c.red = reinterpret_cast<float*>(smem + OFF_RED);
    c.misc = reinterpret_cast<volatile int*>(smem + OFF_MISC);
    c.ring0 = smem_u32(smem + OFF_RING);
    c.full0 = smem_u32(smem + OFF_BAR);
    c.empty0 = c.full0 + NSTAGE * 8;
    c.tid = threadIdx.x; c.warp = threadIdx.x >> 5; c.lane = threadIdx.x & 31;
    c.cta = blockIdx.x; c.G = gridDim.x;
    c.it = 0; c.trace_slot = 0;
    c.seq = __ldcg(&P.ws->seq);
    c.pos = P.position; c.step = 0; c.where = 0;
    c.wf_cycles = 0; c.wf_count = 0; c.wf_calls = 0; c.dirty_stages = 0;
    float* s_rope = reinterpret_cast<float*>(smem + OFF_ROPE);
    c.rope = s_rope;

    // The pointer table is read on every chunk; keep it in shared memory.
    LW* s_layers = reinterpret_cast<LW*>(smem + OFF_LAYERS);
    for (int i = threadIdx.x; i < P.num_layers * (int)(sizeof(LW) / 16); i += NTHR)
        reinterpret_cast<uint4*>(s_layers)[i] = __ldg(reinterpret_cast<const uint4*>(P.layers) + i);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(c.full0 + s * 8, 1);
            mbar_init(c.empty0 + s * 8, NCW);
        }
        c.misc[MISC_ABORT] = 0;
        c.misc[MISC_LAST] = 0;
        c.misc[MISC_DETAIL] = 0;
#if MK_TRACE
        for (int k = 0; k < 16; ++k) reinterpret_cast<volatile int*>(smem + OFF_DBG)[k] = 0;
#endif
#if MK_WFMT == 3
        const uint32_t ubar = smem_u32(smem + U_OFF_BARS);
        mbar_init(ubar, 1); mbar_init(ubar + 8, 1);             // product done (tcgen05.commit)
        mbar_init(ubar + 16, 2); mbar_init(ubar + 24, 2);       // accumulator buffer read back by warps 0 and 1
        mbar_init(ubar + 32, NCW);                              // activation operand written by the consumer warps
#endif
        fence_mbar_init();
    }
#if MK_WFMT == 3
    c.amax = 0.f; c.mma_n = 0; c.inv_g = 1.0f;
    // activation operand and its scales start as zeros: rows of unused residual terms must stay zero
    for (int i = threadIdx.x; i < (U_B_BYTES + U_SFB_BYTES) / 16; i += NTHR)
        reinterpret_cast<uint4*>(smem + U_OFF_B)[i] = make_uint4(0, 0, 0, 0);
    if (c.warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem + U_OFF_TMEM)), "r"(U_TM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_proxy_async();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    c.tmem = *reinterpret_cast<volatile uint32_t*>(smem + U_OFF_TMEM);
#else
    __syncthreads();
#endif

    if (c.warp == NCW) {
        // ===== producer warp =====
        // Walks the weight schedule of every step of the launch; it never needs the token, so it runs ahead of the
        // consumers across step boundaries (the next step's first layer streams in while the argmax finishes).
        const uint64_t pol_stream = l2_policy_evict_first();
        const uint64_t pol_keep = l2_policy_evict_last();
#pragma unroll 1
        for (int step = 0; step < P.steps; ++step) {
            c.pos = P.position + step;
            c.step = step;
            int dn_idx = 0, fa_idx = 0;
            for (int layer = 0; layer <= P.num_layers; ++layer) {
                const bool lm = (layer == P.num_layers);
                const LW& lw = s_layers[lm ? 0 : layer];
                const bool dn = (lw.layer_type == 0);
                const int nph = 5 - (lm ? 4 : 0);
#pragma unroll 1
                for (int ph = 0; ph < nph; ++ph) {
                    int type;
                    if (lm) type = T_LM;
                    else if (dn) type = (ph == 0) ? T_DN_IN : (ph == 1) ? T_DN_REC : (ph == 2) ? T_DN_OUT : (ph == 3) ? T_GATEUP : T_DOWN;
                    else type = (ph == 0) ? T_FA_IN : (ph == 1) ? T_FA_ATT : (ph == 2) ? T_FA_OUT : (ph == 3) ? T_GATEUP : T_DOWN;
                    c.where = 0x8000u | ((uint32_t)layer << 4) | (uint32_t)type;
                    producer_phase(P, c, type, lw, dn ? dn_idx : fa_idx, pol_stream, pol_keep);
                }
                if (!lm) { if (dn) ++dn_idx; else ++fa_idx; }
            }
        }
#if MK_WFMT == 3
    } else if (c.warp == NCW + 1) {
        // ===== MMA warp: one thread walks the same schedule and issues the tensor-core work of every projection =====
        if (c.lane == 0) {
            uint32_t m = 0, an = 0;
#pragma unroll 1
            for (int step = 0; step < P.steps; ++step) {
                c.pos = P.position + step;
                c.step = step;
                for (int layer = 0; layer < P.num_layers; ++layer) {
                    const bool dn = (s_layers[layer].layer_type == 0);
#pragma unroll 1
                    for (int ph = 0; ph < 5; ++ph) {
                        int type;
                        if (dn) type = (ph == 0) ? T_DN_IN : (ph == 1) ? T_DN_REC : (ph == 2) ? T_DN_OUT : (ph == 3) ? T_GATEUP : T_DOWN;
                        else type = (ph == 0) ? T_FA_IN : (ph == 1) ? T_FA_ATT : (ph == 2) ? T_FA_OUT : (ph == 3) ? T_GATEUP : T_DOWN;
                        c.where = 0x4000u | ((uint32_t)layer << 4) | (uint32_t)type;
                        const Geo g = phase_geo(type, c.cta, c.G, P.vocab, c.pos);
                        if (ph == 1) c.it += g.nchunks;               // recurrence / attention chunks: not this warp's
                        else if (g.nchunks > 0) u_mma_phase(P, c, type, g.nchunks, m, an, false, false);
                    }
                }
                c.where = 0x4000u | ((uint32_t)P.num_layers << 4) | T_LM;
                const Geo g = phase_geo(T_LM, c.cta, c.G, P.vocab, c.pos);
                for (int q = 0; q < g.nchunks; ++q) u_mma_phase(P, c, T_LM, 1, m, an, true, q == 0);
            }
        }
#endif
    } else {
        // ===== consumer warps =====
#pragma unroll 1
        for (int step = 0; step < P.steps; ++step) {
            c.step = step;
            c.pos = P.position + step;
            // this step's token: the launch argument, or the previous step's argmax handed over through the workspace
            if (c.tid == 0) {
                int t;
                if (step == 0) t = P.token_ptr ? __ldcg(P.token_ptr) : P.token_val;
                else t = __float_as_int(poll1(P, c, &P.ws->next_token, (c.seq + 1u) << 5));
                c.misc[MISC_TOKEN] = t < 0 ? 0 : (t >= P.vocab ? P.vocab - 1 : t);
            }
            // rotary angles of this position (reference: megakernel/kernel.cu:468-470): angle in f32, accurate sincosf
            if (c.warp == NCW - 1) {
                float sn, cs;
                sincosf((float)c.pos * P.rope_inv_freq[c.lane], &sn, &cs);
                s_rope[c.lane] = cs;
                s_rope[32 + c.lane] = sn;
            }
            named_bar_sync(1, NCT);
            const int token = c.misc[MISC_TOKEN];
            const __nv_bfloat16* embed_row = reinterpret_cast<const __nv_bfloat16*>(P.embed) + (size_t)token * HIDDEN;
            if (c.cta == 0 && c.tid == 0 && P.seen_mask && P.rep_penalty > 1.0f) P.seen_mask[token] = 1.0f;
            int dn_idx = 0, fa_idx = 0;
#pragma unroll 1
            for (int layer = 0; layer < P.num_layers; ++layer) {
                const LW& lw = s_layers[layer];
                const __nv_bfloat16* erow = (layer == 0) ? embed_row : nullptr;
                const uint32_t wl = (uint32_t)layer << 4;
                if (lw.layer_type == 0) {
                    c.where = wl | T_DN_IN;  phase_dn_in(P, c, lw, layer, dn_idx, erow);
                    c.where = wl | T_DN_REC; phase_dn_rec(P, c, layer, dn_idx);
                    c.where = wl | T_DN_OUT; phase_dn_out(P, c, lw, layer, erow);
                    ++dn_idx;
                } else {
                    c.where = wl | T_FA_IN;  phase_fa_in(P, c, lw, layer, erow);
                    c.where = wl | T_FA_ATT; phase_fa_att(P, c, lw, layer, fa_idx);
                    c.where = wl | T_FA_OUT; phase_fa_out(P, c, lw, layer, erow);
                    ++fa_idx;
                }
                c.where = wl | T_GATEUP; phase_gateup(P, c, lw, layer);
                c.where = wl | T_DOWN;   phase_down(P, c, lw, layer);
            }
            c.where = ((uint32_t)P.num_layers << 4) | T_LM;
            phase_lm(P, c);
            ++c.seq;
        }
    }
#if MK_WFMT == 3
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
#endif
    __syncthreads();
#if MK_WFMT == 3
    if (c.warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(c.tmem), "r"(U_TM_COLS) : "memory");
    }
#endif
#if MK_TRACE
    // last three trace slots of the CTA: thread 0's waits for ring chunks (calls, SM clocks blocked, calls that blocked)
    if (P.trace && threadIdx.x == 0 && P.trace_slots >= 3) {
        P.trace[(size_t)c.cta * P.trace_slots + P.trace_slots - 3] = c.wf_calls;
        if (P.trace_slots >= 32)
            for (int k = 0; k < 16; ++k)
                P.trace[(size_t)c.cta * P.trace_slots + P.trace_slots - 32 + k] = (unsigned long long)reinterpret_cast<volatile int*>(c.smem + OFF_DBG)[k];
        P.trace[(size_t)c.cta * P.trace_slots + P.trace_slots - 2] = c.wf_cycles;
        P.trace[(size_t)c.cta * P.trace_slots + P.trace_slots - 1] = c.wf_count;
    }
#endif
    if (c.misc[MISC_ABORT]) {
        if (threadIdx.x == 0 && P.host_status) {
            // low byte: ST code; bits 8-11 phase, 12-18 layer, 23 producer warp, 24-31 step (where the first wait gave up)
            const uint32_t d = (uint32_t)c.misc[MISC_DETAIL];
            *((volatile uint32_t*)P.host_status) = ((uint32_t)c.misc[MISC_ABORT] & 0xffu) | ((d & 0x7fffu) << 8) |
                                                   ((d & 0x8000u) << 8) | ((d >> 16) << 24);
            __threadfence_system();
        }
        // a wait ran out: give bulk copies that are still in flight time to land before the CTA exits
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 50000ull) {}
    }
}

