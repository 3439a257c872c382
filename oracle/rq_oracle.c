/*
 * rq_oracle.c -- CPU oracle (test infrastructure only; see rq_oracle.h).
 *
 * Compiled with -ffp-contract=off so that every a*b+c below rounds twice,
 * exactly like the reference's Rust code (rustc never contracts), except
 * where fmaf() is written out to restate an explicit FMA instruction.
 */
#include "rq_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define QK4_0 32
#define BS_Q4_0 18
#define QK_K 256
#define BS_Q4_K 144
#define BS_Q3_K 110
#define QK8_0 32
#define BS_Q8_0 34
#define BS_Q6_K 210
#define BS_Q5_K 176
#define BS_Q2_K 84

/* ------------------------------------------------------------------ f16 */

float rqo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
    if (e == 0) {
        /* zero / subnormal: m * 2^-24, exact in f32 */
        float v = (float)m * 5.9604644775390625e-08f;
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* IEEE binary16 from binary32, round to nearest even (what half::f16::from_f32
 * and numpy's astype(float16) do). */
uint16_t rqo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) /* inf / nan */
        return sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u);
    if (ax >= 0x477ff000u) /* >= 65520 rounds to inf */
        return sign | 0x7c00u;
    if (ax < 0x38800000u) { /* below 2^-14: half subnormal or zero */
        if (ax <= 0x33000000u) /* <= 2^-25 (tie at 2^-25 goes to even = 0) */
            return sign;
        uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
        int E = (int)(ax >> 23) - 127;  /* -25 .. -15 */
        int shift = -(E + 1);           /* 14 .. 24 */
        uint32_t h = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return sign | (uint16_t)h;
    }
    uint32_t h = ((ax >> 23) - 112u) << 10 | ((ax & 0x7fffffu) >> 13);
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return sign | (uint16_t)h;
}

void rqo_f32_to_f16_n(const float* x, uint16_t* h, int64_t n) {
    for (int64_t i = 0; i < n; i++) h[i] = rqo_f32_to_f16(x[i]);
}
void rqo_f16_to_f32_n(const uint16_t* h, float* x, int64_t n) {
    for (int64_t i = 0; i < n; i++) x[i] = rqo_f16_to_f32(h[i]);
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline void wr16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

int64_t rqo_block_bytes(int type) {
    switch (type) {
    case RQO_Q4_0: return BS_Q4_0;
    case RQO_Q4_K: return BS_Q4_K;
    case RQO_Q3_K: return BS_Q3_K;
    case RQO_Q8_0: return BS_Q8_0;
    case RQO_Q6_K: return BS_Q6_K;
    case RQO_Q5_K: return BS_Q5_K;
    case RQO_Q2_K: return BS_Q2_K;
    default: return 0;
    }
}
int64_t rqo_block_elems(int type) {
    switch (type) {
    case RQO_Q4_0: return QK4_0;
    case RQO_Q8_0: return QK8_0;
    case RQO_Q4_K: case RQO_Q3_K: case RQO_Q6_K: case RQO_Q5_K: case RQO_Q2_K: return QK_K;
    default: return 0;
    }
}

/* round to nearest, ties to even (lrintf under the default rounding mode;
 * the GPU quantizer uses __float2int_rn, the same rounding). */
static inline int nearest_int(float v) { return (int)lrintf(v); }

/* ------------------------------------------------------------- Q4_0 */

/* q4_kernel.rs:137-163: d = max_signed / -8, id = 1/d,
 * q = clamp(x*id + 8.5, 0, 15) as u8 (truncation), lo nibble = element i,
 * hi nibble = element i+16. */
static void quantize_q4_0_block(const float* chunk, uint8_t* blk) {
    float max_abs = 0.0f, max_signed = 0.0f;
    for (int i = 0; i < QK4_0; i++) {
        float a = fabsf(chunk[i]);
        if (a > max_abs) { max_abs = a; max_signed = chunk[i]; }
    }
    float d = max_signed / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    wr16(blk, rqo_f32_to_f16(d));
    for (int i = 0; i < QK4_0 / 2; i++) {
        float a = chunk[i] * id + 8.5f;
        float b = chunk[i + QK4_0 / 2] * id + 8.5f;
        /* Rust f32::clamp then `as u8`: NaN -> 0 */
        a = (a != a) ? 0.0f : (a < 0.0f ? 0.0f : (a > 15.0f ? 15.0f : a));
        b = (b != b) ? 0.0f : (b < 0.0f ? 0.0f : (b > 15.0f ? 15.0f : b));
        blk[2 + i] = (uint8_t)((uint8_t)a | ((uint8_t)b << 4));
    }
}

static void dequantize_q4_0_block(const uint8_t* blk, float* y) {
    float d = rqo_f16_to_f32(rd16(blk));
    for (int i = 0; i < QK4_0 / 2; i++) {
        y[i] = d * (float)((int)(blk[2 + i] & 0x0f) - 8);
        y[i + QK4_0 / 2] = d * (float)((int)(blk[2 + i] >> 4) - 8);
    }
}

/* ------------------------------------------------------------- Q8_0 */
/* Block of 32: f16 d, 32 int8.  Quantizer of GGML's quantize_row_q8_0_ref /
 * candle's BlockQ8_0::from_float: d = amax / 127, id = 1/d (0 for a zero
 * block), q = round(x * id) with ties away from zero (roundf / f32::round).
 * Dequantization: w = d * q. */
static void quantize_q8_0_block(const float* x, uint8_t* blk) {
    float amax = 0.0f;
    for (int i = 0; i < QK8_0; i++) amax = fmaxf(amax, fabsf(x[i]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    wr16(blk, rqo_f32_to_f16(d));
    for (int i = 0; i < QK8_0; i++) blk[2 + i] = (uint8_t)(int8_t)roundf(x[i] * id);
}

static void dequantize_q8_0_block(const uint8_t* blk, float* y) {
    const float d = rqo_f16_to_f32(rd16(blk));
    for (int i = 0; i < QK8_0; i++) y[i] = d * (float)(int8_t)blk[2 + i];
}

/* ------------------------------------------------------------- Q6_K */
/* Super-block of 256 (GGML block_q6_K): ql[128] low 4 bits, qh[64] high 2
 * bits, scales[16] int8 (one per 16 elements), f16 d.  Half n (128 elements)
 * uses ql[64n..], qh[32n..], scales[8n..]; for l < 32:
 *   element 128n+l    = (ql[l]    & 15) | ((qh[l] >> 0) & 3) << 4, scale is+0
 *   element 128n+l+32 = (ql[l+32] & 15) | ((qh[l] >> 2) & 3) << 4, scale is+2
 *   element 128n+l+64 = (ql[l]    >> 4) | ((qh[l] >> 4) & 3) << 4, scale is+4
 *   element 128n+l+96 = (ql[l+32] >> 4) | ((qh[l] >> 6) & 3) << 4, scale is+6
 * with is = l / 16; w = (d * sc) * (q - 32) (GGML dequantize_row_q6_K and
 * gguf-py's order).  The quantizer is this project's own deterministic rule
 * (one int8 scale per 16 elements from the sub-block's largest magnitude). */
static int q6k_index(int i, int* lb, int* hb, int* hshift, int* hi_nib, int* sidx) {
    const int n = i / 128, r = i % 128, quarter = r / 32, l = r % 32;
    *lb = 64 * n + l + ((quarter & 1) ? 32 : 0);
    *hb = 128 + 32 * n + l;
    *hshift = 2 * quarter;
    *hi_nib = quarter >= 2;
    *sidx = 8 * n + l / 16 + 2 * quarter;
    return 0;
}

static void dequantize_q6_k_block(const uint8_t* blk, float* y) {
    const float d = rqo_f16_to_f32(rd16(blk + 208));
    for (int i = 0; i < QK_K; i++) {
        int lb, hb, hs, hn, si;
        q6k_index(i, &lb, &hb, &hs, &hn, &si);
        const int lo = hn ? (blk[lb] >> 4) : (blk[lb] & 15);
        const int q = (lo | (((blk[hb] >> hs) & 3) << 4)) - 32;
        const float sc = (float)(int8_t)blk[192 + si];
        y[i] = (d * sc) * (float)q;
    }
}

static void quantize_q6_k_block(const float* x, uint8_t* blk) {
    memset(blk, 0, BS_Q6_K);
    float scale[16], amax_all = 0.0f;
    for (int j = 0; j < 16; j++) {
        float amax = 0.0f;
        for (int k = 0; k < 16; k++) amax = fmaxf(amax, fabsf(x[16 * j + k]));
        scale[j] = amax / 31.0f;  /* q - 32 in [-31, 31] */
        amax_all = fmaxf(amax_all, scale[j]);
    }
    const float d = amax_all / 127.0f;
    const uint16_t dh = rqo_f32_to_f16(d);
    const float df = rqo_f16_to_f32(dh);
    wr16(blk + 208, dh);
    int sc[16];
    for (int j = 0; j < 16; j++) {
        int v = df != 0.0f ? nearest_int(scale[j] / df) : 0;
        sc[j] = v > 127 ? 127 : (v < -128 ? -128 : v);
        blk[192 + j] = (uint8_t)(int8_t)sc[j];
    }
    for (int i = 0; i < QK_K; i++) {
        const int j = i / 16;
        const float dl = df * (float)sc[j];
        int q = dl != 0.0f ? nearest_int(x[i] / dl) : 0;
        q = q < -32 ? -32 : (q > 31 ? 31 : q);
        const int u = q + 32;  /* 0..63 */
        int lb, hb, hs, hn, si;
        q6k_index(i, &lb, &hb, &hs, &hn, &si);
        blk[lb] |= (uint8_t)(hn ? ((u & 15) << 4) : (u & 15));
        blk[hb] |= (uint8_t)((u >> 4) << hs);
    }
}

/* ------------------------------------------------------------- Q4_K */
/* Super-block of 256: f16 d, f16 dmin, 12 bytes of 6-bit (scale, min) for 8
 * sub-blocks of 32, 128 bytes of nibbles.  Nibble layout: group g (0..3) owns
 * qs[32g .. 32g+31]; low nibble of byte j is element 64g+j (sub-block 2g),
 * high nibble is element 64g+32+j (sub-block 2g+1).
 * w = (d*sc)*q - (dmin*m), two f32 roundings (GGML / gguf-py order). */

static void q4k_get_scale_min(int j, const uint8_t* s, int* sc, int* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static void dequantize_q4_k_block(const uint8_t* blk, float* y) {
    float d = rqo_f16_to_f32(rd16(blk));
    float dmin = rqo_f16_to_f32(rd16(blk + 2));
    const uint8_t* sc = blk + 4;
    const uint8_t* qs = blk + 16;
    for (int g = 0; g < 4; g++) {
        int s0, m0, s1, m1;
        q4k_get_scale_min(2 * g, sc, &s0, &m0);
        q4k_get_scale_min(2 * g + 1, sc, &s1, &m1);
        float d0 = d * (float)s0, mm0 = dmin * (float)m0;
        float d1 = d * (float)s1, mm1 = dmin * (float)m1;
        for (int j = 0; j < 32; j++) {
            y[64 * g + j] = d0 * (float)(qs[32 * g + j] & 0x0f) - mm0;
            y[64 * g + 32 + j] = d1 * (float)(qs[32 * g + j] >> 4) - mm1;
        }
    }
}

/* This project's own deterministic Q4_K quantizer (candle's source is not
 * available).  Per sub-block: range [min(mn,0), mx] -> scale=(mx-lo)/15,
 * min=-lo; scales and mins to 6 bits against the super-block maxima; then
 * q = clamp(rint((x + dmin*m)/(d*sc)), 0, 15) with the stored f16 values.
 * The GPU quantizer (rustyllm_b200/csrc/rq_layout.cu) performs the same f32
 * operations. */
static void quantize_q4_k_block(const float* x, uint8_t* blk) {
    float scale[8], mins[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int s = 0; s < 8; s++) {
        float mn = x[32 * s], mx = x[32 * s];
        for (int i = 1; i < 32; i++) {
            float v = x[32 * s + i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.0f) mn = 0.0f;
        scale[s] = (mx - mn) / 15.0f;
        mins[s] = -mn;
        if (scale[s] > max_scale) max_scale = scale[s];
        if (mins[s] > max_min) max_min = mins[s];
    }
    float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
    float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
    int ls[8], lm[8];
    for (int s = 0; s < 8; s++) {
        int a = nearest_int(inv_scale * scale[s]);
        int b = nearest_int(inv_min * mins[s]);
        ls[s] = a > 63 ? 63 : a;
        lm[s] = b > 63 ? 63 : b;
    }
    uint16_t dh = rqo_f32_to_f16(max_scale / 63.0f);
    uint16_t mh = rqo_f32_to_f16(max_min / 63.0f);
    wr16(blk, dh);
    wr16(blk + 2, mh);
    uint8_t* sc = blk + 4;
    for (int j = 0; j < 4; j++) {
        sc[j] = (uint8_t)(ls[j] | ((ls[j + 4] >> 4) << 6));
        sc[j + 4] = (uint8_t)(lm[j] | ((lm[j + 4] >> 4) << 6));
        sc[j + 8] = (uint8_t)((ls[j + 4] & 0x0f) | ((lm[j + 4] & 0x0f) << 4));
    }
    float d = rqo_f16_to_f32(dh), dmin = rqo_f16_to_f32(mh);
    uint8_t L[256];
    for (int s = 0; s < 8; s++) {
        float dl = d * (float)ls[s];
        float ml = dmin * (float)lm[s];
        for (int i = 0; i < 32; i++) {
            int q = 0;
            if (dl != 0.0f) {
                q = nearest_int((x[32 * s + i] + ml) / dl);
                q = q < 0 ? 0 : (q > 15 ? 15 : q);
            }
            L[32 * s + i] = (uint8_t)q;
        }
    }
    uint8_t* qs = blk + 16;
    for (int g = 0; g < 4; g++)
        for (int j = 0; j < 32; j++)
            qs[32 * g + j] = (uint8_t)(L[64 * g + j] | (L[64 * g + 32 + j] << 4));
}

/* ------------------------------------------------------------- Q5_K */
/* Super-block of 256: f16 d, f16 dmin, the 12 bytes of 6-bit (scale, min)
 * of Q4_K, qh[32], qs[128].  Element 64g+j (sub-block 2g) = low nibble of
 * qs[32g+j] | bit 2g of qh[j] << 4; element 64g+32+j (sub-block 2g+1) = high
 * nibble | bit 2g+1 of qh[j] << 4.  w = (d*sc)*q - (dmin*m) (gguf-py's
 * Q5_K.dequantize_blocks).  The quantizer is this project's Q4_K rule with
 * 5-bit q (unpinned). */
static void dequantize_q5_k_block(const uint8_t* blk, float* y) {
    float d = rqo_f16_to_f32(rd16(blk));
    float dmin = rqo_f16_to_f32(rd16(blk + 2));
    const uint8_t* sc = blk + 4;
    const uint8_t* qh = blk + 16;
    const uint8_t* qs = blk + 48;
    for (int g = 0; g < 4; g++) {
        int s0, m0, s1, m1;
        q4k_get_scale_min(2 * g, sc, &s0, &m0);
        q4k_get_scale_min(2 * g + 1, sc, &s1, &m1);
        float d0 = d * (float)s0, mm0 = dmin * (float)m0;
        float d1 = d * (float)s1, mm1 = dmin * (float)m1;
        for (int j = 0; j < 32; j++) {
            int q0 = (qs[32 * g + j] & 0x0f) | (((qh[j] >> (2 * g)) & 1) << 4);
            int q1 = (qs[32 * g + j] >> 4) | (((qh[j] >> (2 * g + 1)) & 1) << 4);
            y[64 * g + j] = d0 * (float)q0 - mm0;
            y[64 * g + 32 + j] = d1 * (float)q1 - mm1;
        }
    }
}

static void quantize_q5_k_block(const float* x, uint8_t* blk) {
    memset(blk, 0, BS_Q5_K);
    float scale[8], mins[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int s = 0; s < 8; s++) {
        float mn = x[32 * s], mx = x[32 * s];
        for (int i = 1; i < 32; i++) {
            float v = x[32 * s + i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.0f) mn = 0.0f;
        scale[s] = (mx - mn) / 31.0f;
        mins[s] = -mn;
        if (scale[s] > max_scale) max_scale = scale[s];
        if (mins[s] > max_min) max_min = mins[s];
    }
    float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
    float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
    int ls[8], lm[8];
    for (int s = 0; s < 8; s++) {
        int a = nearest_int(inv_scale * scale[s]);
        int b = nearest_int(inv_min * mins[s]);
        ls[s] = a > 63 ? 63 : a;
        lm[s] = b > 63 ? 63 : b;
    }
    uint16_t dh = rqo_f32_to_f16(max_scale / 63.0f);
    uint16_t mh = rqo_f32_to_f16(max_min / 63.0f);
    wr16(blk, dh);
    wr16(blk + 2, mh);
    uint8_t* sc = blk + 4;
    for (int j = 0; j < 4; j++) {
        sc[j] = (uint8_t)(ls[j] | ((ls[j + 4] >> 4) << 6));
        sc[j + 4] = (uint8_t)(lm[j] | ((lm[j + 4] >> 4) << 6));
        sc[j + 8] = (uint8_t)((ls[j + 4] & 0x0f) | ((lm[j + 4] & 0x0f) << 4));
    }
    float d = rqo_f16_to_f32(dh), dmin = rqo_f16_to_f32(mh);
    uint8_t* qh = blk + 16;
    uint8_t* qs = blk + 48;
    for (int s = 0; s < 8; s++) {
        float dl = d * (float)ls[s];
        float ml = dmin * (float)lm[s];
        for (int i = 0; i < 32; i++) {
            int q = 0;
            if (dl != 0.0f) {
                q = nearest_int((x[32 * s + i] + ml) / dl);
                q = q < 0 ? 0 : (q > 31 ? 31 : q);
            }
            const int g = s / 2;
            qs[32 * g + i] |= (uint8_t)((s & 1) ? ((q & 15) << 4) : (q & 15));
            qh[i] |= (uint8_t)((q >> 4) << s);
        }
    }
}

/* ------------------------------------------------------------- Q2_K */
/* Super-block of 256: scales[16] (low nibble: scale, high nibble: min of a
 * 16-element sub-block), qs[64] (2-bit), f16 d, f16 dmin.  Element
 * 128n+32j+l = (qs[32n+l] >> 2j) & 3 of sub-block (128n+32j+l)/16;
 * w = (d*sc)*q - (dmin*m) (gguf-py's Q2_K.dequantize_blocks).  The
 * quantizer is this project's own rule (unpinned). */
static void dequantize_q2_k_block(const uint8_t* blk, float* y) {
    const uint8_t* sc = blk;
    const uint8_t* qs = blk + 16;
    float d = rqo_f16_to_f32(rd16(blk + 80));
    float dmin = rqo_f16_to_f32(rd16(blk + 82));
    for (int n = 0; n < 2; n++)
        for (int j = 0; j < 4; j++)
            for (int l = 0; l < 32; l++) {
                const int e = 128 * n + 32 * j + l, s = e / 16;
                const float dl = d * (float)(sc[s] & 15), ml = dmin * (float)(sc[s] >> 4);
                y[e] = dl * (float)((qs[32 * n + l] >> (2 * j)) & 3) - ml;
            }
}

static void quantize_q2_k_block(const float* x, uint8_t* blk) {
    memset(blk, 0, BS_Q2_K);
    float scale[16], mins[16];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int s = 0; s < 16; s++) {
        float mn = x[16 * s], mx = x[16 * s];
        for (int i = 1; i < 16; i++) {
            float v = x[16 * s + i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.0f) mn = 0.0f;
        scale[s] = (mx - mn) / 3.0f;
        mins[s] = -mn;
        if (scale[s] > max_scale) max_scale = scale[s];
        if (mins[s] > max_min) max_min = mins[s];
    }
    float inv_scale = max_scale > 0.0f ? 15.0f / max_scale : 0.0f;
    float inv_min = max_min > 0.0f ? 15.0f / max_min : 0.0f;
    int ls[16], lm[16];
    for (int s = 0; s < 16; s++) {
        int a = nearest_int(inv_scale * scale[s]);
        int b = nearest_int(inv_min * mins[s]);
        ls[s] = a > 15 ? 15 : a;
        lm[s] = b > 15 ? 15 : b;
        blk[s] = (uint8_t)(ls[s] | (lm[s] << 4));
    }
    uint16_t dh = rqo_f32_to_f16(max_scale / 15.0f);
    uint16_t mh = rqo_f32_to_f16(max_min / 15.0f);
    wr16(blk + 80, dh);
    wr16(blk + 82, mh);
    float d = rqo_f16_to_f32(dh), dmin = rqo_f16_to_f32(mh);
    uint8_t* qs = blk + 16;
    for (int e = 0; e < 256; e++) {
        const int s = e / 16;
        const float dl = d * (float)ls[s], ml = dmin * (float)lm[s];
        int q = 0;
        if (dl != 0.0f) {
            q = nearest_int((x[e] + ml) / dl);
            q = q < 0 ? 0 : (q > 3 ? 3 : q);
        }
        const int n = e / 128, j = (e % 128) / 32, l = e % 32;
        qs[32 * n + l] |= (uint8_t)(q << (2 * j));
    }
}

/* ------------------------------------------------------------- Q3_K */
/* Super-block of 256: hmask[32], qs[64], scales[12], f16 d (110 bytes).
 * Element i: h=i/128, s=(i%128)/32, j=i%32; low 2 bits (qs[32h+j] >> 2s)&3;
 * high bit (hmask[j] >> (i/32))&1; q = low - (high ? 0 : 4) in [-4, 3].
 * Sub-block of 16 = i/16; 6-bit scale stored +32: low nibble in byte
 * (s<8 ? s : s-8) (low/high half), high 2 bits in byte 8+(s%4) at 2*(s/4).
 * w = (d*scale)*q (gguf-py order). */

static void q3k_scales(const uint8_t* sb, int* out) {
    for (int s = 0; s < 16; s++) {
        int lo = s < 8 ? (sb[s] & 0x0f) : (sb[s - 8] >> 4);
        int hi = (sb[8 + (s % 4)] >> (2 * (s / 4))) & 3;
        out[s] = (lo | (hi << 4)) - 32;
    }
}

static void dequantize_q3_k_block(const uint8_t* blk, float* y) {
    const uint8_t* hm = blk;
    const uint8_t* qs = blk + 32;
    int sc[16];
    q3k_scales(blk + 96, sc);
    float d = rqo_f16_to_f32(rd16(blk + 108));
    for (int i = 0; i < 256; i++) {
        int h = i / 128, s = (i % 128) / 32, j = i % 32;
        int low = (qs[32 * h + j] >> (2 * s)) & 3;
        int hb = (hm[j] >> (i / 32)) & 1;
        int q = low - (hb ? 0 : 4);
        float dl = d * (float)sc[i / 16];
        y[i] = dl * (float)q;
    }
}

/* This project's own Q3_K quantizer: per sub-block of 16 the element of
 * largest magnitude maps to -4 (scale = v/-4); the 16 scales go to 6-bit
 * signed with iscale = -32/max_scale, d = f16(1/iscale); then
 * q = clamp(rint(x / (d*l)), -4, 3). */
static void quantize_q3_k_block(const float* x, uint8_t* blk) {
    float scale[16];
    float max_scale = 0.0f, amax_scale = 0.0f;
    for (int s = 0; s < 16; s++) {
        float ma = 0.0f, mv = 0.0f;
        for (int i = 0; i < 16; i++) {
            float v = x[16 * s + i];
            float a = fabsf(v);
            if (a > ma) { ma = a; mv = v; }
        }
        scale[s] = mv / -4.0f;
        float as = fabsf(scale[s]);
        if (as > amax_scale) { amax_scale = as; max_scale = scale[s]; }
    }
    memset(blk, 0, BS_Q3_K);
    int ls[16];
    float iscale = max_scale != 0.0f ? -32.0f / max_scale : 0.0f;
    for (int s = 0; s < 16; s++) {
        int l = nearest_int(iscale * scale[s]);
        ls[s] = l < -32 ? -32 : (l > 31 ? 31 : l);
    }
    uint16_t dh = rqo_f32_to_f16(iscale != 0.0f ? 1.0f / iscale : 0.0f);
    uint8_t* sb = blk + 96;
    for (int s = 0; s < 16; s++) {
        int v = ls[s] + 32;
        if (s < 8) sb[s] |= (uint8_t)(v & 0x0f);
        else sb[s - 8] |= (uint8_t)((v & 0x0f) << 4);
        sb[8 + (s % 4)] |= (uint8_t)((v >> 4) << (2 * (s / 4)));
    }
    wr16(blk + 108, dh);
    float d = rqo_f16_to_f32(dh);
    uint8_t* hm = blk;
    uint8_t* qs = blk + 32;
    for (int i = 0; i < 256; i++) {
        float dl = d * (float)ls[i / 16];
        int q = 0;
        if (dl != 0.0f) {
            q = nearest_int(x[i] / dl);
            q = q < -4 ? -4 : (q > 3 ? 3 : q);
        }
        int u = q + 4; /* 0..7 */
        int h = i / 128, s = (i % 128) / 32, j = i % 32;
        qs[32 * h + j] |= (uint8_t)((u & 3) << (2 * s));
        hm[j] |= (uint8_t)((u >> 2) << (i / 32));
    }
}

/* ------------------------------------------------------ generic entry */

int rqo_quantize(int type, const float* x, int64_t rows, int64_t in, uint8_t* out) {
    int64_t be = rqo_block_elems(type), bb = rqo_block_bytes(type);
    if (!be || in % be) return -1;
    int64_t nb = in / be;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++) {
            const float* src = x + r * in + b * be;
            uint8_t* dst = out + (r * nb + b) * bb;
            if (type == RQO_Q4_0) quantize_q4_0_block(src, dst);
            else if (type == RQO_Q8_0) quantize_q8_0_block(src, dst);
            else if (type == RQO_Q4_K) quantize_q4_k_block(src, dst);
            else if (type == RQO_Q6_K) quantize_q6_k_block(src, dst);
            else if (type == RQO_Q5_K) quantize_q5_k_block(src, dst);
            else if (type == RQO_Q2_K) quantize_q2_k_block(src, dst);
            else quantize_q3_k_block(src, dst);
        }
    return 0;
}

int rqo_dequantize(int type, const uint8_t* blocks, int64_t rows, int64_t in, float* out) {
    int64_t be = rqo_block_elems(type), bb = rqo_block_bytes(type);
    if (!be || in % be) return -1;
    int64_t nb = in / be;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* src = blocks + (r * nb + b) * bb;
            float* dst = out + r * in + b * be;
            if (type == RQO_Q4_0) dequantize_q4_0_block(src, dst);
            else if (type == RQO_Q8_0) dequantize_q8_0_block(src, dst);
            else if (type == RQO_Q4_K) dequantize_q4_k_block(src, dst);
            else if (type == RQO_Q6_K) dequantize_q6_k_block(src, dst);
            else if (type == RQO_Q5_K) dequantize_q5_k_block(src, dst);
            else if (type == RQO_Q2_K) dequantize_q2_k_block(src, dst);
            else dequantize_q3_k_block(src, dst);
        }
    return 0;
}

static void dequantize_row(int type, const uint8_t* row, int64_t in, float* out) {
    rqo_dequantize(type, row, 1, in, out);
}

int rqo_matmul_ref(int type, const uint8_t* blocks, int64_t out, int64_t in,
                   const float* x, int64_t M, float* y, int acc64) {
    int64_t be = rqo_block_elems(type), bb = rqo_block_bytes(type);
    if (!be || in % be) return -1;
    int64_t row_bytes = in / be * bb;
    float* w = (float*)malloc(sizeof(float) * (size_t)in);
    if (!w) return -2;
    for (int64_t o = 0; o < out; o++) {
        dequantize_row(type, blocks + o * row_bytes, in, w);
        for (int64_t m = 0; m < M; m++) {
            const float* xr = x + m * in;
            if (acc64) {
                double acc = 0.0;
                for (int64_t k = 0; k < in; k++) acc += (double)xr[k] * (double)w[k];
                y[m * out + o] = (float)acc;
            } else {
                float acc = 0.0f;
                for (int64_t k = 0; k < in; k++) acc += xr[k] * w[k];
                y[m * out + o] = acc;
            }
        }
    }
    free(w);
    return 0;
}

/* ------------------------------------------- q4_kernel.rs dot restatements */

/* q4_kernel.rs:274-293: block_sum over i of x[i]*lo + x[i+16]*hi, then
 * sum += scale * block_sum. */
float rqo_dot_q4_0_scalar(const uint8_t* w_row, const float* x_row, int64_t blocks_per_row) {
    float sum = 0.0f;
    for (int64_t b = 0; b < blocks_per_row; b++) {
        const uint8_t* blk = w_row + b * BS_Q4_0;
        float scale = rqo_f16_to_f32(rd16(blk));
        const float* xb = x_row + b * QK4_0;
        float block_sum = 0.0f;
        for (int i = 0; i < QK4_0 / 2; i++) {
            float lo = (float)((int)(blk[2 + i] & 0x0f) - 8);
            float hi = (float)((int)(blk[2 + i] >> 4) - 8);
            block_sum += xb[i] * lo;
            block_sum += xb[i + QK4_0 / 2] * hi;
        }
        sum += scale * block_sum;
    }
    return sum;
}

/* q4_kernel.rs:300-360: eight f32 lanes; per block the weight is (q-8)*scale
 * (one rounding), then fused multiply-add into lane c of four vectors
 * (x[0..8] with low nibbles of bytes 0..7, x[8..16] with low nibbles of bytes
 * 8..15, x[16..24] / x[24..32] with the high nibbles), then a left-to-right
 * horizontal sum of the eight lanes. */
float rqo_dot_q4_0_avx2order(const uint8_t* w_row, const float* x_row, int64_t blocks_per_row) {
    float acc[8] = {0};
    for (int64_t b = 0; b < blocks_per_row; b++) {
        const uint8_t* blk = w_row + b * BS_Q4_0;
        float scale = rqo_f16_to_f32(rd16(blk));
        const uint8_t* qs = blk + 2;
        const float* xb = x_row + b * QK4_0;
        for (int v = 0; v < 4; v++) {
            for (int c = 0; c < 8; c++) {
                int byte = (v & 1) * 8 + c;
                int q = (v < 2) ? (qs[byte] & 0x0f) : (qs[byte] >> 4);
                float w = (float)(q - 8) * scale;
                acc[c] = fmaf(w, xb[8 * v + c], acc[c]);
            }
        }
    }
    float s = 0.0f;
    for (int c = 0; c < 8; c++) s += acc[c];
    return s;
}

/* Dequant-fused f32 dot with eight lanes for the K-quants (CPU baseline:
 * the weight value is the exact GGML dequant, accumulated with fmaf). */
static float dot_kquant_f32(int type, const uint8_t* w_row, const float* x, int64_t nb) {
    float acc[8] = {0};
    float w[256];
    const int be = (int)rqo_block_elems(type);
    for (int64_t b = 0; b < nb; b++) {
        if (type == RQO_Q4_K) dequantize_q4_k_block(w_row + b * BS_Q4_K, w);
        else if (type == RQO_Q6_K) dequantize_q6_k_block(w_row + b * BS_Q6_K, w);
        else if (type == RQO_Q8_0) dequantize_q8_0_block(w_row + b * BS_Q8_0, w);
        else if (type == RQO_Q5_K) dequantize_q5_k_block(w_row + b * BS_Q5_K, w);
        else if (type == RQO_Q2_K) dequantize_q2_k_block(w_row + b * BS_Q2_K, w);
        else dequantize_q3_k_block(w_row + b * BS_Q3_K, w);
        const float* xb = x + b * be;
        for (int i = 0; i < be; i += 8)
            for (int c = 0; c < 8; c++) acc[c] = fmaf(w[i + c], xb[i + c], acc[c]);
    }
    float s = 0.0f;
    for (int c = 0; c < 8; c++) s += acc[c];
    return s;
}

typedef struct {
    int type;
    const uint8_t* blocks;
    int64_t out, in, n, row_bytes, nb, chunk, nchunks;
    const float* x;
    float* y;
    int64_t next; /* atomic chunk counter */
} lin_job;

static void* lin_worker(void* arg) {
    lin_job* j = (lin_job*)arg;
    for (;;) {
        int64_t c = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
        if (c >= j->nchunks) break;
        int64_t start = c * j->chunk, end = start + j->chunk;
        if (end > j->n * j->out) end = j->n * j->out;
        for (int64_t pos = start; pos < end; pos++) {
            int64_t b = pos / j->out, o = pos % j->out;
            const uint8_t* wr = j->blocks + o * j->row_bytes;
            const float* xr = j->x + b * j->in;
            float v;
            if (j->type == RQO_Q4_0) v = rqo_dot_q4_0_avx2order(wr, xr, j->nb);
            else v = dot_kquant_f32(j->type, wr, xr, j->nb);
            j->y[pos] = v;
        }
    }
    return NULL;
}

int rqo_linear_threaded(int type, const uint8_t* blocks, int64_t out, int64_t in,
                        const float* x, int64_t M, float* y, int nthreads) {
    int64_t be = rqo_block_elems(type), bb = rqo_block_bytes(type);
    if (!be || in % be || M <= 0 || out <= 0) return -1;
    if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    lin_job j;
    j.type = type; j.blocks = blocks; j.out = out; j.in = in; j.n = M;
    j.nb = in / be; j.row_bytes = j.nb * bb; j.x = x; j.y = y; j.next = 0;
    /* q4_kernel.rs:208-210 */
    int64_t total = M * out;
    int64_t chunk = total / ((int64_t)nthreads * 4);
    if (chunk < 8) chunk = 8;
    if (chunk > total) chunk = total;
    if (chunk < 1) chunk = 1;
    j.chunk = chunk;
    j.nchunks = (total + chunk - 1) / chunk;
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < nthreads; t++)
        if (pthread_create(&th[started], NULL, lin_worker, &j) == 0) started++;
    lin_worker(&j);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return 0;
}

/* The same products as rqo_linear_threaded, computed faster for M > 1:
 * each weight row is dequantized once and dotted with every activation row.
 * The dot is the 8-lane fmaf order of dot_kquant_f32 / the AVX2-order Q4_0
 * dot (element i into lane i % 8, lanes summed in order), and the dequant is
 * exact, so every output has the bits rqo_linear_threaded gives it.  Used by
 * the layer and model oracles, where M is a prompt or a batch of tokens. */
static float dot_lanes8_fma(const float* w, const float* x, int64_t n) {
    float acc[8] = {0};
    for (int64_t i = 0; i < n; i += 8)
        for (int c = 0; c < 8; c++) acc[c] = fmaf(w[i + c], x[i + c], acc[c]);
    float s = 0.0f;
    for (int c = 0; c < 8; c++) s += acc[c];
    return s;
}

typedef struct {
    int type;
    const uint8_t* blocks;
    int64_t out, in, M, row_bytes;
    const float* x;
    float* y;
    int64_t next; /* atomic row-chunk counter */
} rows_job;

static void* rows_worker(void* arg) {
    rows_job* j = (rows_job*)arg;
    float* w = (float*)malloc(sizeof(float) * (size_t)j->in);
    if (!w) return NULL;
    const int64_t chunk = 16;
    for (;;) {
        int64_t c = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
        int64_t o0 = c * chunk;
        if (o0 >= j->out) break;
        int64_t o1 = o0 + chunk < j->out ? o0 + chunk : j->out;
        for (int64_t o = o0; o < o1; o++) {
            dequantize_row(j->type, j->blocks + o * j->row_bytes, j->in, w);
            for (int64_t m = 0; m < j->M; m++) j->y[m * j->out + o] = dot_lanes8_fma(w, j->x + m * j->in, j->in);
        }
    }
    free(w);
    return NULL;
}

int rqo_linear_rows(int type, const uint8_t* blocks, int64_t out, int64_t in, const float* x, int64_t M,
                    float* y, int nthreads) {
    int64_t be = rqo_block_elems(type), bb = rqo_block_bytes(type);
    if (!be || in % be || M <= 0 || out <= 0) return -1;
    if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    rows_job j;
    j.type = type; j.blocks = blocks; j.out = out; j.in = in; j.M = M;
    j.row_bytes = in / be * bb; j.x = x; j.y = y; j.next = 0;
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < nthreads; t++)
        if (pthread_create(&th[started], NULL, rows_worker, &j) == 0) started++;
    rows_worker(&j);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return 0;
}

/* ------------------------------------------------------------------ MoE */

float rqo_silu(float x) { return x / (1.0f + expf(-x)); }

/* ------------------------------------------- ParallelLinear (F16 weights) */

/* parallel_linear.rs:33-94: the f16 row is converted to an f32 scratch row
 * (half's convert_to_f32_slice, exact), then the dot product.  A build with
 * the avx2 and fma target features (the configuration the AVX2 figures of
 * q4_kernel.rs:31-39 come from) runs dot_f32_avx2_fma: eight f32 lanes
 * accumulate element 8i+c into lane c with a fused multiply-add
 * (_mm256_fmadd_ps, :80-84), the lanes are summed left to right
 * (buf.iter().sum(), :87-89) and a scalar tail adds a[i]*b[i] (two
 * roundings, :91-94).  Without those features the scalar loop of :48-55 runs:
 * sum += x[k]*w[k] in ascending k, two roundings each. */
static float dot_f16_scalar(const float* x, const float* w, int64_t n) {
    float sum = 0.0f;
    for (int64_t k = 0; k < n; k++) sum += x[k] * w[k];
    return sum;
}

static float dot_f16_lanes8(const float* x, const float* w, int64_t n) {
    float acc[8] = {0};
    const int64_t chunks = n / 8;
    for (int64_t i = 0; i < chunks; i++)
        for (int c = 0; c < 8; c++) acc[c] = fmaf(x[8 * i + c], w[8 * i + c], acc[c]);
    float sum = -0.0f;
    for (int c = 0; c < 8; c++) sum += acc[c];
    for (int64_t i = chunks * 8; i < n; i++) sum += x[i] * w[i];
    return sum;
}

typedef struct {
    const uint16_t* w;
    int64_t out, in, n, chunk, nchunks;
    const float* x;
    float* y;
    int avx2;
    int64_t next; /* atomic chunk counter */
} pl_job;

static void* pl_worker(void* arg) {
    pl_job* j = (pl_job*)arg;
    float* scratch = (float*)malloc(sizeof(float) * (size_t)j->in);
    if (!scratch) return NULL;
    for (;;) {
        int64_t c = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
        if (c >= j->nchunks) break;
        int64_t start = c * j->chunk, end = start + j->chunk;
        if (end > j->n * j->out) end = j->n * j->out;
        for (int64_t pos = start; pos < end; pos++) {
            int64_t b = pos / j->out, o = pos % j->out;
            rqo_f16_to_f32_n(j->w + o * j->in, scratch, j->in);
            j->y[pos] = j->avx2 ? dot_f16_lanes8(j->x + b * j->in, scratch, j->in)
                                : dot_f16_scalar(j->x + b * j->in, scratch, j->in);
        }
    }
    free(scratch);
    return NULL;
}

/* parallel_linear.rs:191-295: y[b][j] = dot_f16_f32(W[j], x[b]) over the
 * flattened n*out outputs in chunks of max(total / (4 workers), 8) (:223-225);
 * the n == 1 fast path (:239-259) computes the same values. */
int rqo_parallel_linear_f16(const uint16_t* w, int64_t out, int64_t in, const float* x, int64_t n,
                            float* y, int avx2, int nthreads) {
    if (out <= 0 || in <= 0 || n <= 0) return -1;
    if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pl_job j;
    j.w = w; j.out = out; j.in = in; j.n = n; j.x = x; j.y = y; j.avx2 = avx2; j.next = 0;
    int64_t total = n * out;
    int64_t chunk = total / ((int64_t)nthreads * 4);
    if (chunk < 8) chunk = 8;
    if (chunk > total) chunk = total;
    if (chunk < 1) chunk = 1;
    j.chunk = chunk;
    j.nchunks = (total + chunk - 1) / chunk;
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < nthreads; t++)
        if (pthread_create(&th[started], NULL, pl_worker, &j) == 0) started++;
    pl_worker(&j);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return 0;
}

/* Router logits: the gate of SparseMoe is a ParallelLinear (F16 weight,
 * streaming_mixtral.rs:265,283), so logits[t][e] = dot_f16_f32(wr[e], x[t])
 * in the AVX2 lane order. */
void rqo_router_logits(const float* x, int64_t T, int64_t H, const uint16_t* wr16, int E, float* logits) {
    rqo_parallel_linear_f16(wr16, E, H, x, T, logits, 1, 1);
}

/* streaming_mixtral.rs:284-303: softmax_last_dim, then per token a stable
 * sort of expert indices by probability descending (total_cmp), take top_k,
 * sum the selected probabilities in rank order, weight = p / sum. */
void rqo_route_topk(const float* logits, int64_t T, int E, int k, int32_t* ids, float* weights) {
    float p[256];
    int order[256];
    for (int64_t t = 0; t < T; t++) {
        const float* l = logits + t * E;
        float mx = l[0];
        for (int e = 1; e < E; e++) if (l[e] > mx) mx = l[e];
        float sum = 0.0f;
        for (int e = 0; e < E; e++) { p[e] = expf(l[e] - mx); sum += p[e]; }
        for (int e = 0; e < E; e++) p[e] = p[e] / sum;
        /* stable insertion sort, descending */
        for (int e = 0; e < E; e++) {
            int pos = e;
            while (pos > 0 && p[order[pos - 1]] < p[e]) { order[pos] = order[pos - 1]; pos--; }
            order[pos] = e;
        }
        float s = 0.0f;
        for (int r = 0; r < k; r++) s += p[order[r]];
        for (int r = 0; r < k; r++) {
            ids[t * k + r] = order[r];
            weights[t * k + r] = p[order[r]] / s;
        }
    }
}

void rqo_permute(const int32_t* ids, const float* weights, int64_t T, int E, int k,
                 int32_t* offsets, int32_t* rows, float* slot_w) {
    int64_t pos = 0;
    for (int e = 0; e < E; e++) {
        offsets[e] = (int32_t)pos;
        for (int64_t t = 0; t < T; t++)
            for (int r = 0; r < k; r++)
                if (ids[t * k + r] == e) {
                    rows[pos] = (int32_t)t;
                    if (slot_w) slot_w[pos] = weights[t * k + r];
                    pos++;
                }
    }
    offsets[E] = (int32_t)pos;
}

int rqo_moe_forward(const float* x, int64_t T, int64_t H, int64_t F, int E, int k,
                    const uint16_t* wr, int wtype, const uint8_t* const* w1,
                    const uint8_t* const* w3, const uint8_t* const* w2, float* y,
                    int32_t* ids_out, int32_t* perm_out, int32_t* offsets_out,
                    int nthreads) {
    if (E > 256 || k > E || H % 4) return -1;
    float* logits = (float*)malloc(sizeof(float) * (size_t)(T * E));
    int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * (size_t)(T * k));
    float* wts = (float*)malloc(sizeof(float) * (size_t)(T * k));
    int32_t* rows = (int32_t*)malloc(sizeof(int32_t) * (size_t)(T * k));
    float* sw = (float*)malloc(sizeof(float) * (size_t)(T * k));
    int32_t offs[257];
    float* xin = (float*)malloc(sizeof(float) * (size_t)(T * H));
    float* g = (float*)malloc(sizeof(float) * (size_t)(T * F));
    float* u = (float*)malloc(sizeof(float) * (size_t)(T * F));
    float* o = (float*)malloc(sizeof(float) * (size_t)(T * H));
    if (!logits || !ids || !wts || !rows || !sw || !xin || !g || !u || !o) return -2;
    rqo_router_logits(x, T, H, wr, E, logits);
    rqo_route_topk(logits, T, E, k, ids, wts);
    rqo_permute(ids, wts, T, E, k, offs, rows, sw);
    memset(y, 0, sizeof(float) * (size_t)(T * H));
    for (int e = 0; e < E; e++) {
        int64_t n = offs[e + 1] - offs[e];
        if (n == 0) continue;
        for (int64_t i = 0; i < n; i++)
            memcpy(xin + i * H, x + (int64_t)rows[offs[e] + i] * H, sizeof(float) * (size_t)H);
        if (wtype == RQO_F16) {  /* the reference's experts: ParallelLinear (streaming_mixtral.rs:231-257) */
            rqo_parallel_linear_f16((const uint16_t*)w1[e], F, H, xin, n, g, 1, nthreads);
            rqo_parallel_linear_f16((const uint16_t*)w3[e], F, H, xin, n, u, 1, nthreads);
        } else {
            rqo_linear_rows(wtype, w1[e], F, H, xin, n, g, nthreads);
            rqo_linear_rows(wtype, w3[e], F, H, xin, n, u, nthreads);
        }
        for (int64_t i = 0; i < n * F; i++) g[i] = rqo_silu(g[i]) * u[i];
        if (wtype == RQO_F16) rqo_parallel_linear_f16((const uint16_t*)w2[e], H, F, g, n, o, 1, nthreads);
        else rqo_linear_rows(wtype, w2[e], H, F, g, n, o, nthreads);
        for (int64_t i = 0; i < n; i++) {
            float wv = sw[offs[e] + i];
            float* yr = y + (int64_t)rows[offs[e] + i] * H;
            for (int64_t c = 0; c < H; c++) yr[c] = yr[c] + o[i * H + c] * wv;
        }
    }
    if (ids_out) memcpy(ids_out, ids, sizeof(int32_t) * (size_t)(T * k));
    if (perm_out) memcpy(perm_out, rows, sizeof(int32_t) * (size_t)(T * k));
    if (offsets_out) memcpy(offsets_out, offs, sizeof(int32_t) * (size_t)(E + 1));
    free(logits); free(ids); free(wts); free(rows); free(sw); free(xin); free(g); free(u); free(o);
    return 0;
}

/* ------------------------------------------------------------ Llama loop */
/* The quantized Llama forward of src/streaming_quantized.rs:193-317,611-633
 * on the CPU, f32 throughout: RmsNorm (candle_nn::ops::rms_norm order:
 * m = sqrt(sum(x^2)/n + eps), y = x / m * w), q/k/v/o and MLP linears by the
 * dequantize-then-dot path, non-interleaved RoPE from f32 tables built like
 * QuantStreamCache::new, causal GQA attention with softmax, silu(g) * u,
 * residual adds, final norm, F16 lm_head, first-index argmax. */

struct rqo_llama {
    int64_t H, I, nh, nkv, hd, nl, vocab, max_seq;
    float eps, theta;
    int wtype;
    const uint8_t** w;   /* [nl][7] */
    const float** rms1;  /* [nl] */
    const float** rms2;
    const uint16_t* emb;
    const float* lnf;
    const uint16_t* head;
    float *kc, *vc;      /* [nl][nkv][max_seq][hd] */
    float *cs, *sn;      /* [max_seq][hd/2] */
};

rqo_llama* rqo_llama_create(int64_t H, int64_t I, int64_t nh, int64_t nkv, int64_t hd, int64_t nl,
                            int64_t vocab, int64_t max_seq, float eps, float theta, int wtype) {
    rqo_llama* m = (rqo_llama*)calloc(1, sizeof(rqo_llama));
    if (!m) return NULL;
    m->H = H; m->I = I; m->nh = nh; m->nkv = nkv; m->hd = hd; m->nl = nl; m->vocab = vocab;
    m->max_seq = max_seq; m->eps = eps; m->theta = theta; m->wtype = wtype;
    m->w = (const uint8_t**)calloc((size_t)(nl * 7), sizeof(void*));
    m->rms1 = (const float**)calloc((size_t)nl, sizeof(void*));
    m->rms2 = (const float**)calloc((size_t)nl, sizeof(void*));
    m->kc = (float*)calloc((size_t)(nl * nkv * max_seq * hd), sizeof(float));
    m->vc = (float*)calloc((size_t)(nl * nkv * max_seq * hd), sizeof(float));
    int64_t half = hd / 2;
    m->cs = (float*)malloc(sizeof(float) * (size_t)(max_seq * half));
    m->sn = (float*)malloc(sizeof(float) * (size_t)(max_seq * half));
    for (int64_t i = 0; i < half; i++) {
        float inv = 1.0f / powf(theta, (float)(2 * i) / (float)hd);
        for (int64_t p = 0; p < max_seq; p++) {
            float a = (float)p * inv;
            m->cs[p * half + i] = cosf(a);
            m->sn[p * half + i] = sinf(a);
        }
    }
    return m;
}

void rqo_llama_free(rqo_llama* m) {
    if (!m) return;
    free(m->w); free(m->rms1); free(m->rms2); free(m->kc); free(m->vc); free(m->cs); free(m->sn);
    free(m);
}

int rqo_llama_set_layer(rqo_llama* m, int64_t l, const uint8_t* const* w7, const float* rms1,
                        const float* rms2) {
    if (l < 0 || l >= m->nl) return -1;
    for (int i = 0; i < 7; i++) m->w[l * 7 + i] = w7[i];
    m->rms1[l] = rms1;
    m->rms2[l] = rms2;
    return 0;
}

void rqo_llama_set_embedding(rqo_llama* m, const uint16_t* emb) { m->emb = emb; }
void rqo_llama_set_head(rqo_llama* m, const float* lnf, const uint16_t* head) { m->lnf = lnf; m->head = head; }

static void rms_norm(const float* x, const float* w, int64_t n, float eps, float* y) {
    float sum2 = 0.0f;
    for (int64_t i = 0; i < n; i++) sum2 += x[i] * x[i];
    float mden = sqrtf(sum2 / (float)n + eps);
    for (int64_t i = 0; i < n; i++) y[i] = x[i] / mden * w[i];
}

void rqo_llama_embed(const rqo_llama* m, const int32_t* tokens, int64_t T, float* x) {
    for (int64_t t = 0; t < T; t++)
        for (int64_t i = 0; i < m->H; i++) x[t * m->H + i] = rqo_f16_to_f32(m->emb[(int64_t)tokens[t] * m->H + i]);
}

/* QBlock::forward (src/streaming_quantized.rs:305-317) of layer l over the
 * hidden rows x[T][H] at positions pos..pos+T-1, in place; the layer's keys
 * and values are written into its cache at those positions. */
int rqo_llama_layer(rqo_llama* m, int64_t l, float* x, int64_t T, int64_t pos, int nthreads) {
    const int64_t H = m->H, I = m->I, nh = m->nh, nkv = m->nkv, hd = m->hd, half = hd / 2;
    const int64_t nq = nh * hd, nk = nkv * hd, rep = nh / nkv;
    if (l < 0 || l >= m->nl || pos < 0 || pos + T > m->max_seq) return -1;
    const uint8_t* const* W = m->w + l * 7;
    for (int i = 0; i < 7; i++)
        if (!W[i]) return -1;
    float* h = (float*)calloc((size_t)(T * H), sizeof(float));
    float* q = (float*)malloc(sizeof(float) * (size_t)(T * nq));
    float* k = (float*)malloc(sizeof(float) * (size_t)(T * nk));
    float* v = (float*)malloc(sizeof(float) * (size_t)(T * nk));
    float* a = (float*)malloc(sizeof(float) * (size_t)(T * nq));
    float* o = (float*)malloc(sizeof(float) * (size_t)(T * H));
    float* g = (float*)malloc(sizeof(float) * (size_t)(T * I));
    float* u = (float*)malloc(sizeof(float) * (size_t)(T * I));
    float* sc = (float*)malloc(sizeof(float) * (size_t)m->max_seq);
    if (!h || !q || !k || !v || !a || !o || !g || !u || !sc) return -2;
    float* kc = m->kc + l * nkv * m->max_seq * hd;
    float* vc = m->vc + l * nkv * m->max_seq * hd;
    for (int64_t t = 0; t < T; t++) rms_norm(x + t * H, m->rms1[l], H, m->eps, h + t * H);
    rqo_linear_rows(m->wtype, W[0], nq, H, h, T, q, nthreads);
    rqo_linear_rows(m->wtype, W[1], nk, H, h, T, k, nthreads);
    rqo_linear_rows(m->wtype, W[2], nk, H, h, T, v, nthreads);
    for (int64_t t = 0; t < T; t++) {
        int64_t p = pos + t;
        const float* c = m->cs + p * half;
        const float* s = m->sn + p * half;
        for (int64_t hh = 0; hh < nh; hh++) {
            float* qh = q + (t * nh + hh) * hd;
            for (int64_t i = 0; i < half; i++) {
                float a0 = qh[i], b0 = qh[i + half];
                qh[i] = a0 * c[i] - b0 * s[i];
                qh[i + half] = a0 * s[i] + b0 * c[i];
            }
        }
        for (int64_t kh = 0; kh < nkv; kh++) {
            const float* ks = k + (t * nkv + kh) * hd;
            const float* vs = v + (t * nkv + kh) * hd;
            float* kd = kc + (kh * m->max_seq + p) * hd;
            float* vd = vc + (kh * m->max_seq + p) * hd;
            for (int64_t i = 0; i < half; i++) {
                float a0 = ks[i], b0 = ks[i + half];
                kd[i] = a0 * c[i] - b0 * s[i];
                kd[i + half] = a0 * s[i] + b0 * c[i];
            }
            for (int64_t i = 0; i < hd; i++) vd[i] = vs[i];
        }
    }
    float sq = sqrtf((float)hd);
    for (int64_t t = 0; t < T; t++) {
        int64_t L = pos + t + 1;
        for (int64_t hh = 0; hh < nh; hh++) {
            const float* qh = q + (t * nh + hh) * hd;
            int64_t kh = hh / rep;
            const float* K = kc + kh * m->max_seq * hd;
            const float* V = vc + kh * m->max_seq * hd;
            float mx = -INFINITY;
            for (int64_t j = 0; j < L; j++) {
                float acc = 0.0f;
                for (int64_t d = 0; d < hd; d++) acc += qh[d] * K[j * hd + d];
                sc[j] = acc / sq;
                if (sc[j] > mx) mx = sc[j];
            }
            float sum = 0.0f;
            for (int64_t j = 0; j < L; j++) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
            for (int64_t j = 0; j < L; j++) sc[j] = sc[j] / sum;
            float* ah = a + (t * nh + hh) * hd;
            for (int64_t d = 0; d < hd; d++) {
                float acc = 0.0f;
                for (int64_t j = 0; j < L; j++) acc += sc[j] * V[j * hd + d];
                ah[d] = acc;
            }
        }
    }
    rqo_linear_rows(m->wtype, W[3], H, nq, a, T, o, nthreads);
    for (int64_t i = 0; i < T * H; i++) x[i] = o[i] + x[i];
    for (int64_t t = 0; t < T; t++) rms_norm(x + t * H, m->rms2[l], H, m->eps, h + t * H);
    rqo_linear_rows(m->wtype, W[4], I, H, h, T, g, nthreads);
    rqo_linear_rows(m->wtype, W[5], I, H, h, T, u, nthreads);
    for (int64_t i = 0; i < T * I; i++) g[i] = rqo_silu(g[i]) * u[i];
    rqo_linear_rows(m->wtype, W[6], H, I, g, T, o, nthreads);
    for (int64_t i = 0; i < T * H; i++) x[i] = o[i] + x[i];
    free(h); free(q); free(k); free(v); free(a); free(o); free(g); free(u); free(sc);
    return 0;
}

/* f16 -> f32 of every half, for the lm_head rows (same values as rqo_f16_to_f32) */
static float g_f16_table[65536];
static pthread_once_t g_f16_once = PTHREAD_ONCE_INIT;
static void f16_table_init(void) {
    for (uint32_t i = 0; i < 65536u; i++) g_f16_table[i] = rqo_f16_to_f32((uint16_t)i);
}

typedef struct {
    const rqo_llama* m;
    const float* hn;  /* [T][H] normed rows */
    int64_t T;
    float* lg;        /* [T][vocab] */
    int64_t next;
} head_job;

static void* head_worker(void* arg) {
    head_job* j = (head_job*)arg;
    const int64_t H = j->m->H, V = j->m->vocab, chunk = 64;
    for (;;) {
        int64_t r0 = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED) * chunk;
        if (r0 >= V) break;
        int64_t r1 = r0 + chunk < V ? r0 + chunk : V;
        for (int64_t r = r0; r < r1; r++) {
            const uint16_t* row = j->m->head + r * H;
            for (int64_t t = 0; t < j->T; t++) {
                const float* h = j->hn + t * H;
                float acc = 0.0f;
                for (int64_t i = 0; i < H; i++) acc += h[i] * g_f16_table[row[i]];
                j->lg[t * V + r] = acc;
            }
        }
    }
    return NULL;
}

/* ln_f and the F16 lm_head (src/streaming_quantized.rs:630-632) of every row
 * of x[T][H]: logits[T][vocab] (may be NULL) and the first-index argmax of
 * each row. */
int rqo_llama_head(const rqo_llama* m, const float* x, int64_t T, float* logits, int32_t* argmax, int nthreads) {
    const int64_t H = m->H, V = m->vocab;
    pthread_once(&g_f16_once, f16_table_init);
    float* hn = (float*)malloc(sizeof(float) * (size_t)(T * H));
    float* lg = logits ? logits : (float*)malloc(sizeof(float) * (size_t)(T * V));
    if (!hn || !lg) return -2;
    for (int64_t t = 0; t < T; t++) rms_norm(x + t * H, m->lnf, H, m->eps, hn + t * H);
    if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    head_job j = {m, hn, T, lg, 0};
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < nthreads; t++)
        if (pthread_create(&th[started], NULL, head_worker, &j) == 0) started++;
    head_worker(&j);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    for (int64_t t = 0; t < T; t++) {
        const float* r = lg + t * V;
        int32_t best = 0;
        for (int64_t v = 1; v < V; v++)
            if (r[v] > r[best]) best = (int32_t)v;
        argmax[t] = best;
    }
    free(hn);
    if (!logits) free(lg);
    return 0;
}

/* forward(input_ids, index_pos) (src/streaming_quantized.rs:622-633):
 * logits_last [vocab] of the last position (may be NULL); next: argmax. */
int rqo_llama_forward(rqo_llama* m, const int32_t* tokens, int64_t T, int64_t pos,
                      float* logits_last, int32_t* next, int nthreads) {
    if (pos + T > m->max_seq || T < 1) return -1;
    float* x = (float*)malloc(sizeof(float) * (size_t)(T * m->H));
    if (!x) return -2;
    rqo_llama_embed(m, tokens, T, x);
    int rc = 0;
    for (int64_t l = 0; l < m->nl && !rc; l++) rc = rqo_llama_layer(m, l, x, T, pos, nthreads);
    int32_t best = 0;
    if (!rc) rc = rqo_llama_head(m, x + (T - 1) * m->H, 1, logits_last, &best, nthreads);
    if (!rc && next) *next = best;
    free(x);
    return rc;
}
