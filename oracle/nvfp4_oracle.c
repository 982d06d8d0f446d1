/* CPU restatement of the reference's two NVFP4 weight formats.  TEST INFRASTRUCTURE ONLY: the
 * checker for the CUDA quantisers / dequantising kernels; the product never calls it.
 *
 * Format A, layer weights (reference: megakernel/kernel_gb10_nvfp4.cu:1764-1817):
 *   groups of `group_size` along K; scale = amax/6 (1 if the group is all zero) stored as fp16;
 *   code = sign | magnitude index by the thresholds 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5 applied
 *   to x * (1/scale) with the UNROUNDED f32 scale (half-way cases go up in magnitude);
 *   byte = element 2i in the low nibble, element 2i+1 in the high nibble.
 * Format B, LM head / tensor-core layout (reference: megakernel/kernel_gb10_nvfp4.cu:1373-1437):
 *   blocks of 16 along K; scale = max(amax * (1/6), 2^-28) rounded to E4M3 (round to nearest
 *   even, saturating to 448); value = x * (1/decoded_scale) rounded to e2m1 (nearest even code,
 *   saturating to 6); scales stored in 128-row x 4-column tiles of 512 bytes at
 *   tile*512 + (row%32)*16 + ((row%128)/32)*4 + (col%4).
 * Dequantised value of both: LUT{0,.5,1,1.5,2,3,4,6}[code&7] * (-1 if code&8) * scale
 * (reference: megakernel/kernel_gb10_nvfp4.cu:80-83, 528-552, 1439-1456).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bf16_to_f32(uint16_t v) { uint32_t u = (uint32_t)v << 16; float f; memcpy(&f, &u, 4); return f; }

/* IEEE f32 -> f16, round to nearest even (what __float2half does) */
static uint16_t f32_to_f16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t exp = (int32_t)((x >> 23) & 0xff) - 127 + 15;
    uint32_t man = x & 0x7fffffu;
    if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0));
    if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    if (exp <= 0) {
        if (exp < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - exp;
        uint32_t half = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u), mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1u))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t half = ((uint32_t)exp << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++;
    return (uint16_t)(sign | half);
}
static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1f, man = h & 0x3ffu, x;
    if (exp == 0) {
        if (man == 0) x = sign;
        else { int e = -1; do { man <<= 1; e++; } while (!(man & 0x400u)); x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13); }
    } else if (exp == 31) x = sign | 0x7f800000u | (man << 13);
    else x = sign | ((exp - 15 + 127) << 23) | (man << 13);
    float f; memcpy(&f, &x, 4); return f;
}

/* E4M3 (bias 7, no infinities, max 448) */
float mk_oracle_e4m3_to_f32(uint8_t c) {
    int sign = c >> 7, exp = (c >> 3) & 0xf, man = c & 7;
    float v;
    if (exp == 0) v = ldexpf((float)man, -9);
    else if (exp == 15 && man == 7) v = NAN;
    else v = ldexpf(1.0f + man / 8.0f, exp - 7);
    return sign ? -v : v;
}
/* round to nearest even, saturate to +-448 */
uint8_t mk_oracle_f32_to_e4m3(float f) {
    uint8_t sign = signbit(f) ? 0x80 : 0;
    float a = fabsf(f);
    if (isnan(f)) return (uint8_t)(sign | 0x7f);
    if (a >= 448.0f) return (uint8_t)(sign | 0x7e);
    if (a < ldexpf(1.0f, -6)) {                       /* subnormal range: multiples of 2^-9 */
        float q = a * 512.0f;                         /* exact */
        float r = nearbyintf(q);                      /* default rounding mode: nearest even */
        int m = (int)r;                               /* 0..8; 8 = smallest normal */
        return (uint8_t)(sign | m);
    }
    int e; float fr = frexpf(a, &e);                  /* a = fr * 2^e, fr in [0.5,1) */
    float m = fr * 2.0f;  e -= 1;                     /* m in [1,2) */
    float q = (m - 1.0f) * 8.0f;
    int mi = (int)nearbyintf(q);
    if (mi == 8) { mi = 0; e += 1; }
    int be = e + 7;
    if (be > 15 || (be == 15 && mi == 7)) return (uint8_t)(sign | 0x7e);
    return (uint8_t)(sign | (be << 3) | mi);
}

static const float E2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

/* format A code: thresholds, half-way cases up in magnitude (reference :1764-1776) */
static unsigned code_a(float x) {
    float ax = fabsf(x);
    unsigned mag = ax < 0.25f ? 0 : ax < 0.75f ? 1 : ax < 1.25f ? 2 : ax < 1.75f ? 3 : ax < 2.5f ? 4 : ax < 3.5f ? 5 : ax < 5.0f ? 6 : 7;
    return (x < 0.0f) ? (mag | 8u) : mag;
}
/* format B code: nearest representable, ties to the even code, saturating (cvt.rn.satfinite.e2m1x2) */
uint8_t mk_oracle_f32_to_e2m1(float x) {
    unsigned sign = signbit(x) ? 8u : 0u;
    float ax = fabsf(x);
    unsigned mag;
    if (isnan(x)) return (uint8_t)(sign | 7u);
    if (ax <= 0.25f) mag = 0;            /* tie 0.25 -> 0 (even) */
    else if (ax < 0.75f) mag = 1;
    else if (ax <= 1.25f) mag = 2;       /* ties 0.75 -> 1.0, 1.25 -> 1.0 */
    else if (ax < 1.75f) mag = 3;
    else if (ax <= 2.5f) mag = 4;        /* ties 1.75 -> 2.0, 2.5 -> 2.0 */
    else if (ax < 3.5f) mag = 5;
    else if (ax <= 5.0f) mag = 6;        /* ties 3.5 -> 4.0, 5.0 -> 4.0 */
    else mag = 7;
    return (uint8_t)(sign | mag);
}

void mk_oracle_quantize_a(const uint16_t* w, int rows, int cols, int group, uint8_t* packed, uint16_t* scales) {
    int gpr = cols / group;
    for (int r = 0; r < rows; ++r)
        for (int g = 0; g < gpr; ++g) {
            const uint16_t* src = w + (size_t)r * cols + (size_t)g * group;
            uint8_t* dst = packed + (size_t)r * (cols / 2) + (size_t)g * (group / 2);
            float amax = 0.0f;
            for (int i = 0; i < group; ++i) amax = fmaxf(amax, fabsf(bf16_to_f32(src[i])));
            float scale = (amax > 0.0f) ? (amax / 6.0f) : 1.0f;
            scales[(size_t)r * gpr + g] = f32_to_f16(scale);
            if (amax == 0.0f) { memset(dst, 0, group / 2); continue; }
            float inv = 1.0f / scale;
            for (int i = 0; i < group; i += 2) {
                unsigned lo = code_a(bf16_to_f32(src[i]) * inv), hi = code_a(bf16_to_f32(src[i + 1]) * inv);
                dst[i / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
}

size_t mk_oracle_scale_index_b(int row, int scale_col, int cols) {
    int tiles_per_row = cols / 64;
    size_t tile = (size_t)(row / 128) * tiles_per_row + (scale_col >> 2);
    return tile * 512 + (size_t)(row & 31) * 16 + (size_t)((row & 127) >> 5) * 4 + (scale_col & 3);
}

void mk_oracle_quantize_b(const uint16_t* w, int rows, int cols, uint8_t* packed, uint8_t* scales) {
    const float sixth = 1.0f / 6.0f, floor_s = 1.0f / (float)(1 << 28);
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < cols / 16; ++b) {
            const uint16_t* src = w + (size_t)r * cols + (size_t)b * 16;
            float amax = 0.0f;
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(bf16_to_f32(src[i])));
            uint8_t sc = mk_oracle_f32_to_e4m3(fmaxf(amax * sixth, floor_s));
            float dec = mk_oracle_e4m3_to_f32(sc);
            float inv = (dec > 0.0f) ? (1.0f / dec) : 0.0f;
            uint8_t* dst = packed + (size_t)r * (cols / 2) + (size_t)b * 8;
            for (int i = 0; i < 16; i += 2) {
                unsigned lo = mk_oracle_f32_to_e2m1(bf16_to_f32(src[i]) * inv);
                unsigned hi = mk_oracle_f32_to_e2m1(bf16_to_f32(src[i + 1]) * inv);
                dst[i / 2] = (uint8_t)(lo | (hi << 4));
            }
            scales[mk_oracle_scale_index_b(r, b, cols)] = sc;
        }
}

static float deq(unsigned code, float scale) { float v = E2M1[code & 7u] * scale; return (code & 8u) ? -v : v; }

void mk_oracle_dequantize_a(const uint8_t* packed, const uint16_t* scales, int rows, int cols, int group, float* out) {
    int gpr = cols / group;
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) {
            uint8_t byte = packed[(size_t)r * (cols / 2) + c / 2];
            unsigned code = (c & 1) ? (byte >> 4) : (byte & 15u);
            out[(size_t)r * cols + c] = deq(code, f16_to_f32(scales[(size_t)r * gpr + c / group]));
        }
}

void mk_oracle_dequantize_b(const uint8_t* packed, const uint8_t* scales, int rows, int cols, float* out) {
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) {
            uint8_t byte = packed[(size_t)r * (cols / 2) + c / 2];
            unsigned code = (c & 1) ? (byte >> 4) : (byte & 15u);
            out[(size_t)r * cols + c] = deq(code, mk_oracle_e4m3_to_f32(scales[mk_oracle_scale_index_b(r, c / 16, cols)]));
        }
}

/* Format B with a per-tensor scale (the "e2m1 values in 16-element blocks, FP8 E4M3 block scales, fp32 per-tensor
 * scale" format).  The reference has no per-tensor scale (its 16-block quantiser, kernel_gb10_nvfp4.cu:1373-1437,
 * stores block scales directly; alpha = 1 at :451): parity unpinned, this restatement is the definition the CUDA
 * kernels are held to bit for bit.
 *   s_t   = amax(tensor) / (6 * 448)   (1 for an all-zero tensor)      -- the largest block scale lands on 448
 *   block = E4M3( max((amax(block) / 6) / s_t, 2^-28) ),  dec = decoded block scale
 *   code  = e2m1_rne( x * (1 / (dec * s_t)) ),  value = e2m1(code) * (dec * s_t)
 * every operation a single IEEE f32 operation in the order written. */
float mk_oracle_tensor_scale(const uint16_t* w, int rows, int cols) {
    float amax = 0.0f;
    for (size_t i = 0; i < (size_t)rows * cols; ++i) amax = fmaxf(amax, fabsf(bf16_to_f32(w[i])));
    return amax > 0.0f ? amax / 2688.0f : 1.0f;
}

void mk_oracle_quantize_ts(const uint16_t* w, int rows, int cols, uint8_t* packed, uint8_t* scales, float* tensor_scale) {
    const float sixth = 1.0f / 6.0f, floor_s = 1.0f / (float)(1 << 28);
    const float st = mk_oracle_tensor_scale(w, rows, cols);
    *tensor_scale = st;
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < cols / 16; ++b) {
            const uint16_t* src = w + (size_t)r * cols + (size_t)b * 16;
            float amax = 0.0f;
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(bf16_to_f32(src[i])));
            float rel = (amax * sixth) / st;
            uint8_t sc = mk_oracle_f32_to_e4m3(fmaxf(rel, floor_s));
            float eff = mk_oracle_e4m3_to_f32(sc) * st;
            float inv = (eff > 0.0f) ? (1.0f / eff) : 0.0f;
            uint8_t* dst = packed + (size_t)r * (cols / 2) + (size_t)b * 8;
            for (int i = 0; i < 16; i += 2) {
                unsigned lo = mk_oracle_f32_to_e2m1(bf16_to_f32(src[i]) * inv);
                unsigned hi = mk_oracle_f32_to_e2m1(bf16_to_f32(src[i + 1]) * inv);
                dst[i / 2] = (uint8_t)(lo | (hi << 4));
            }
            scales[mk_oracle_scale_index_b(r, b, cols)] = sc;
        }
}

void mk_oracle_dequantize_ts(const uint8_t* packed, const uint8_t* scales, float tensor_scale, int rows, int cols, float* out) {
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) {
            uint8_t byte = packed[(size_t)r * (cols / 2) + c / 2];
            unsigned code = (c & 1) ? (byte >> 4) : (byte & 15u);
            out[(size_t)r * cols + c] = deq(code, mk_oracle_e4m3_to_f32(scales[mk_oracle_scale_index_b(r, c / 16, cols)]) * tensor_scale);
        }
}

uint16_t mk_oracle_f32_to_f16(float f) { return f32_to_f16(f); }
float mk_oracle_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
