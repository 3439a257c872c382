// rq_mv_common.cuh -- per-lane dot-product pieces shared by the matvec
// kernels (register-streaming fallback in rq_matvec.cu, bulk-copy pipeline in
// rq_mv_pipe.cu).
//
// A K-slice is 2048 elements.  Within a slice lane l owns 64 elements:
//   Q4_K: group l (super-block l/4, 64-element group l%4): 32 quant bytes
//         [32l, 32l+32) of the slice, header of super-block l/4;
//   Q3_K: quarter l%4 of super-block l/4 (h = bit 1, u = bit 0): elements
//         128h + 32s + 16u + jj (s, jj in 0..3, 0..15);
//   Q4_0: blocks 2l and 2l+1 of the slice.
// The activation planes of those 64 elements stay in registers (48 words)
// for every row the lane processes.
#pragma once

#include "rq_internal.cuh"

namespace rq {

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// d1*65536 + d2*256 + d3 with one final rounding
__device__ __forceinline__ float fix24(int d1, int d2, int d3) {
    return fmaf((float)d1, 65536.0f, (float)(d2 * 256 + d3));
}

// ------------------------------------------------------ transpose reduction
// v[0..N) are this lane's partials for N rows.  Afterwards v[0] holds the
// full 32-lane sum of row row_of_lane<N>(lane), on the lanes for which
// lane_writes<N>(lane) is true.
template <int N, int CNT, int OFF>
__device__ __forceinline__ void transpose_reduce_step(float (&v)[N], int lane) {
    if constexpr (OFF > 0) {
        if constexpr (CNT > 1) {
            constexpr int HALF = CNT / 2;
            const bool upper = (lane & OFF) != 0;
#pragma unroll
            for (int i = 0; i < HALF; i++) {
                const float send = upper ? v[i] : v[i + HALF];
                const float keep = upper ? v[i + HALF] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
            }
            transpose_reduce_step<N, HALF, OFF / 2>(v, lane);
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], OFF);
            transpose_reduce_step<N, 1, OFF / 2>(v, lane);
        }
    }
}

template <int N>
__device__ __forceinline__ void transpose_reduce(float (&v)[N], int lane) {
    transpose_reduce_step<N, N, 16>(v, lane);
}

template <int N>
__device__ __forceinline__ int row_of_lane(int lane) {
    int row = 0, cnt = N;
#pragma unroll
    for (int off = 16; off >= 1 && cnt > 1; off >>= 1) {
        cnt >>= 1;
        if (lane & off) row += cnt;
    }
    return row;
}

template <int N>
__device__ __forceinline__ bool lane_writes(int lane) {
    constexpr int used = (N >= 32) ? 5 : (N >= 16) ? 4 : (N >= 8) ? 3 : (N >= 4) ? 2 : (N >= 2) ? 1 : 0;
    return (lane & ((1 << (5 - used)) - 1)) == 0;
}

// --------------------------------------------------------- x staging
// Stage the 32 values v (one block of row m, block b) into the planes and
// stats of xq; the arithmetic of the staged form (see rq_internal.cuh).
__device__ __forceinline__ void stage_block(const float (&v)[32], int64_t m, int64_t b, int64_t in,
                                            int8_t* __restrict__ planes, float4* __restrict__ stats) {
    float amax = 0.0f, sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; k++) { amax = fmaxf(amax, fabsf(v[k])); sa += v[k]; }
#pragma unroll
    for (int k = 16; k < 32; k++) { amax = fmaxf(amax, fabsf(v[k])); sb += v[k]; }
    const float inv = amax > 0.0f ? kXQScale / amax : 0.0f;
    const float sx = amax / kXQScale;
    uint32_t p1[8], p2[8], p3[8];
#pragma unroll
    for (int k = 0; k < 8; k++) { p1[k] = 0u; p2[k] = 0u; p3[k] = 0u; }
#pragma unroll
    for (int k = 0; k < 32; k++) {
        const int X = __float2int_rn(v[k] * inv);
        const int x3 = (X << 24) >> 24;  // balanced base-256 digits
        const int t1 = (X - x3) >> 8;
        const int x2 = (t1 << 24) >> 24;
        const int x1 = (t1 - x2) >> 8;
        p1[k / 4] |= (uint32_t)(x1 & 255) << (8 * (k % 4));
        p2[k / 4] |= (uint32_t)(x2 & 255) << (8 * (k % 4));
        p3[k / 4] |= (uint32_t)(x3 & 255) << (8 * (k % 4));
    }
    uint4* d1 = reinterpret_cast<uint4*>(planes + (m * 3 + 0) * in + b * 32);
    uint4* d2 = reinterpret_cast<uint4*>(planes + (m * 3 + 1) * in + b * 32);
    uint4* d3 = reinterpret_cast<uint4*>(planes + (m * 3 + 2) * in + b * 32);
    d1[0] = make_uint4(p1[0], p1[1], p1[2], p1[3]); d1[1] = make_uint4(p1[4], p1[5], p1[6], p1[7]);
    d2[0] = make_uint4(p2[0], p2[1], p2[2], p2[3]); d2[1] = make_uint4(p2[4], p2[5], p2[6], p2[7]);
    d3[0] = make_uint4(p3[0], p3[1], p3[2], p3[3]); d3[1] = make_uint4(p3[4], p3[5], p3[6], p3[7]);
    stats[m * (in / 32) + b] = make_float4(sx, sa, sb, 0.0f);
}

__device__ __forceinline__ void load_block(const float* src, float (&v)[32]) {
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float4 f = reinterpret_cast<const float4*>(src)[k];
            v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int k = 0; k < 32; k++) v[k] = src[k];
    }
}

// ------------------------------------------------------------------- Q4_K

struct Q4KLane {
    uint32_t p[3][16];  // planes of elements 64g .. 64g+63 of the super-block
    float sxl, xsl, sxh, xsh;
    uint32_t mL, mH;
    int sh;
    bool hiG;
};

__device__ __forceinline__ void q4k_lane_setup(Q4KLane& L, const int8_t* planes,
                                               const float4* stats, int64_t in, int64_t sb,
                                               int g) {
    const int64_t pos = sb * 256 + 64 * g;
#pragma unroll
    for (int p = 0; p < 3; p++) {
        const uint4* src = reinterpret_cast<const uint4*>(planes + p * in + pos);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint4 u = src[k];
            L.p[p][4 * k] = u.x; L.p[p][4 * k + 1] = u.y;
            L.p[p][4 * k + 2] = u.z; L.p[p][4 * k + 3] = u.w;
        }
    }
    const float4 lo = stats[sb * 8 + 2 * g];
    const float4 hi = stats[sb * 8 + 2 * g + 1];
    L.sxl = lo.x;
    L.xsl = lo.y + lo.z;
    L.sxh = hi.x * 0.0625f;  // high nibbles are masked in place: 16*q
    L.xsh = hi.y + hi.z;
    L.hiG = g >= 2;
    L.sh = 16 * (g & 1);
    L.mL = L.hiG ? 0x0F0Fu : 0x3F3Fu;
    L.mH = L.hiG ? 0x3030u : 0u;
}

// One row: 32 quant bytes (qa, qb) of the lane's group and the super-block
// header h.  Returns the lane's contribution to y[row].
__device__ __forceinline__ float q4k_lane_row(const Q4KLane& L, uint4 qa, uint4 qb, uint4 h) {
    const uint32_t wv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int l1 = 0, l2 = 0, l3 = 0, h1 = 0, h2 = 0, h3 = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t lo = wv[k] & 0x0F0F0F0Fu;
        const uint32_t hi = wv[k] & 0xF0F0F0F0u;
        l1 = dp4a_us(lo, L.p[0][k], l1);
        l2 = dp4a_us(lo, L.p[1][k], l2);
        l3 = dp4a_us(lo, L.p[2][k], l3);
        h1 = dp4a_us(hi, L.p[0][8 + k], h1);
        h2 = dp4a_us(hi, L.p[1][8 + k], h2);
        h3 = dp4a_us(hi, L.p[2][8 + k], h3);
    }
    const float fl = fix24(l1, l2, l3) * L.sxl;
    const float fh = fix24(h1, h2, h3) * L.sxh;
    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
    // 6-bit (scale, min) of sub-blocks 2g, 2g+1 (GGML Q4_K packing)
    const uint32_t A = L.hiG ? h.w : h.y;
    const uint32_t B = L.hiG ? (h.w >> 4) : h.z;
    const uint32_t scp = ((A >> L.sh) & L.mL) | ((h.y >> (L.sh + 2)) & L.mH);
    const uint32_t mp = ((B >> L.sh) & L.mL) | ((h.z >> (L.sh + 2)) & L.mH);
    const float sc0 = (float)(scp & 0xFFu), sc1 = (float)((scp >> 8) & 0xFFu);
    const float m0 = (float)(mp & 0xFFu), m1 = (float)((mp >> 8) & 0xFFu);
    return dd.x * fmaf(sc0, fl, sc1 * fh) - dd.y * fmaf(m0, L.xsl, m1 * L.xsh);
}

// Q4_K lane for the shared-memory pipeline.  The lane's 32 quant bytes are
// read as two 16-byte halves in a lane-dependent order (half h1 first, h1 =
// bit 2 of the lane) so each quarter-warp's 128-bit shared loads hit distinct
// banks; the activation words are stored in the same order at set-up, so no
// per-row register swap is needed.  The four 6-bit values of sub-blocks
// (2g, 2g+1) are gathered with two byte permutes and lane-constant masks.
struct Q4KPLane {
    uint32_t xa[3][8];  // half A: [plane][0..3 low-nibble words, 4..7 high-nibble words]
    uint32_t xb[3][8];  // half B
    float sxl, xsl, sxh, xsh;
    uint32_t sel1, sel2, mA, mB, mC;
    bool hiG;
};

__device__ __forceinline__ void q4kp_lane_setup(Q4KPLane& L, const int8_t* planes,
                                                const float4* stats, int64_t in, int64_t sb,
                                                int g, int h1, bool valid) {
    const int64_t pos = sb * 256 + 64 * g;
#pragma unroll
    for (int p = 0; p < 3; p++) {
        const int8_t* base = planes + p * in + pos;
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int hsel = half == 0 ? h1 : 1 - h1;
            uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = make_uint4(0u, 0u, 0u, 0u);
            if (valid) {
                lo = *reinterpret_cast<const uint4*>(base + 16 * hsel);
                hi = *reinterpret_cast<const uint4*>(base + 32 + 16 * hsel);
            }
            uint32_t* dst = half == 0 ? L.xa[p] : L.xb[p];
            dst[0] = lo.x; dst[1] = lo.y; dst[2] = lo.z; dst[3] = lo.w;
            dst[4] = hi.x; dst[5] = hi.y; dst[6] = hi.z; dst[7] = hi.w;
        }
    }
    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
    if (valid) {
        lo = stats[sb * 8 + 2 * g];
        hi = stats[sb * 8 + 2 * g + 1];
    }
    L.sxl = lo.x;
    L.xsl = lo.y + lo.z;
    L.sxh = hi.x * 0.0625f;  // high nibbles are masked in place: 16*q
    L.xsh = hi.y + hi.z;
    L.hiG = g >= 2;
    const uint32_t j = 2u * (uint32_t)(g & 1);
    // g < 2:  bytes [s[j], s[j+1], s[j+4], s[j+5]] of (h.y, h.z)
    // g >= 2: bytes [s[j+8], s[j+9], s[j+8], s[j+9]] of h.w (j relative), and
    //         top bits from [s[j], s[j+1], s[j+4], s[j+5]] of (h.y, h.z)
    const uint32_t yz = j | ((j + 1) << 4) | ((j + 4) << 8) | ((j + 5) << 12);
    L.sel1 = L.hiG ? (j | ((j + 1) << 4) | (j << 8) | ((j + 1) << 12)) : yz;
    L.sel2 = yz;
    L.mA = L.hiG ? 0x00000F0Fu : 0x3F3F3F3Fu;
    L.mB = L.hiG ? 0x0F0F0000u : 0u;
    L.mC = L.hiG ? 0x30303030u : 0u;
}

__device__ __forceinline__ float q4kp_lane_row(const Q4KPLane& L, uint4 qa, uint4 qb, uint4 h,
                                               float part) {
    const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w};
    const uint32_t wb[4] = {qb.x, qb.y, qb.z, qb.w};
    int l1 = 0, l2 = 0, l3 = 0, h1 = 0, h2 = 0, h3 = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t lo = wa[k] & 0x0F0F0F0Fu, hi = wa[k] & 0xF0F0F0F0u;
        l1 = dp4a_us(lo, L.xa[0][k], l1);
        l2 = dp4a_us(lo, L.xa[1][k], l2);
        l3 = dp4a_us(lo, L.xa[2][k], l3);
        h1 = dp4a_us(hi, L.xa[0][4 + k], h1);
        h2 = dp4a_us(hi, L.xa[1][4 + k], h2);
        h3 = dp4a_us(hi, L.xa[2][4 + k], h3);
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t lo = wb[k] & 0x0F0F0F0Fu, hi = wb[k] & 0xF0F0F0F0u;
        l1 = dp4a_us(lo, L.xb[0][k], l1);
        l2 = dp4a_us(lo, L.xb[1][k], l2);
        l3 = dp4a_us(lo, L.xb[2][k], l3);
        h1 = dp4a_us(hi, L.xb[0][4 + k], h1);
        h2 = dp4a_us(hi, L.xb[1][4 + k], h2);
        h3 = dp4a_us(hi, L.xb[2][4 + k], h3);
    }
    const float fl = fix24(l1, l2, l3) * L.sxl;
    const float fh = fix24(h1, h2, h3) * L.sxh;
    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
    const uint32_t x1 = __byte_perm(L.hiG ? h.w : h.y, h.z, L.sel1);
    const uint32_t x2 = __byte_perm(h.y, h.z, L.sel2);
    const uint32_t w = (x1 & L.mA) | ((x1 >> 4) & L.mB) | ((x2 >> 2) & L.mC);  // [sc0, sc1, m0, m1]
    const float sc0 = (float)(w & 0xFFu), sc1 = (float)((w >> 8) & 0xFFu);
    const float m0 = (float)((w >> 16) & 0xFFu), m1 = (float)(w >> 24);
    part = fmaf(dd.x, fmaf(sc0, fl, sc1 * fh), part);
    return fmaf(-dd.y, fmaf(m0, L.xsl, m1 * L.xsh), part);
}

// Selectors that gather the four 6-bit values (scale, min) of the sub-block
// pair (2g, 2g+1) of a Q4_K header with two byte permutes (GGML packing; the
// same decode as Q4KPLane, for kernels that keep g per warp).
struct Q4KScaleSel {
    uint32_t sel1, sel2, mA, mB, mC;
    bool hiG;
};

__device__ __forceinline__ Q4KScaleSel q4k_scale_sel(int g) {
    Q4KScaleSel S;
    S.hiG = g >= 2;
    const uint32_t j = 2u * (uint32_t)(g & 1);
    const uint32_t yz = j | ((j + 1) << 4) | ((j + 4) << 8) | ((j + 5) << 12);
    S.sel1 = S.hiG ? (j | ((j + 1) << 4) | (j << 8) | ((j + 1) << 12)) : yz;
    S.sel2 = yz;
    S.mA = S.hiG ? 0x00000F0Fu : 0x3F3F3F3Fu;
    S.mB = S.hiG ? 0x0F0F0000u : 0u;
    S.mC = S.hiG ? 0x30303030u : 0u;
    return S;
}

// bytes [sc(2g), sc(2g+1), m(2g), m(2g+1)] of header h
__device__ __forceinline__ uint32_t q4k_scales(const Q4KScaleSel& S, uint4 h) {
    const uint32_t x1 = __byte_perm(S.hiG ? h.w : h.y, h.z, S.sel1);
    const uint32_t x2 = __byte_perm(h.y, h.z, S.sel2);
    return (x1 & S.mA) | ((x1 >> 4) & S.mB) | ((x2 >> 2) & S.mC);
}

// ------------------------------------------------------------------- Q3_K

// Q3_K on the expanded device layout (rq_internal.cuh): q + 4 as nibbles in
// Q4_K's arrangement, 16 int8 scales and d per super-block.  The lane is the
// Q4_K pipeline lane's data path (group g = lane % 4 of the super-block,
// halves in order h1) with one accumulator chain per 16-element sub-block:
// A lo = sub-block 4g + h1, B lo = 4g + 1 - h1, A hi = 4g + 2 + h1,
// B hi = 4g + 3 - h1, each scaled by its int8 scale, and the -4 offset of
// q + 4 taken from the 16-element sums of the staged activations.
struct Q3KLane {
    uint32_t xa[3][8];  // half A: [plane][0..3 low-nibble words, 4..7 high-nibble words]
    uint32_t xb[3][8];  // half B
    float sxl, sxh;     // block scales of the low / high 32 elements (sxh / 16: nibbles in place)
    float xs[4];        // 4 * sum of x over the sub-blocks A lo, B lo, A hi, B hi
    uint32_t sel;       // byte permute putting the four scales in that order
};

__device__ __forceinline__ void q3k_lane_setup(Q3KLane& L, const int8_t* planes, const float4* stats, int64_t in,
                                               int64_t sb, int g, int h1, bool valid) {
    const int64_t pos = sb * 256 + 64 * g;
#pragma unroll
    for (int p = 0; p < 3; p++) {
        const int8_t* base = planes + p * in + pos;
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int hsel = half == 0 ? h1 : 1 - h1;
            uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = make_uint4(0u, 0u, 0u, 0u);
            if (valid) {
                lo = *reinterpret_cast<const uint4*>(base + 16 * hsel);
                hi = *reinterpret_cast<const uint4*>(base + 32 + 16 * hsel);
            }
            uint32_t* dst = half == 0 ? L.xa[p] : L.xb[p];
            dst[0] = lo.x; dst[1] = lo.y; dst[2] = lo.z; dst[3] = lo.w;
            dst[4] = hi.x; dst[5] = hi.y; dst[6] = hi.z; dst[7] = hi.w;
        }
    }
    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
    if (valid) {
        lo = stats[sb * 8 + 2 * g];
        hi = stats[sb * 8 + 2 * g + 1];
    }
    L.sxl = lo.x;
    L.sxh = hi.x * 0.0625f;
    L.xs[0] = 4.0f * (h1 ? lo.z : lo.y);
    L.xs[1] = 4.0f * (h1 ? lo.y : lo.z);
    L.xs[2] = 4.0f * (h1 ? hi.z : hi.y);
    L.xs[3] = 4.0f * (h1 ? hi.y : hi.z);
    L.sel = h1 ? 0x2301u : 0x3210u;
}

// One row: the lane's 32 nibble bytes (qa: half A, qb: half B), the header
// word holding the int8 scales of sub-blocks 4g..4g+3 and the word holding d.
__device__ __forceinline__ float q3k_lane_row(const Q3KLane& L, uint4 qa, uint4 qb, uint32_t scw, uint32_t dw) {
    const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w};
    const uint32_t wb[4] = {qb.x, qb.y, qb.z, qb.w};
    int al[3] = {0, 0, 0}, ah[3] = {0, 0, 0}, bl[3] = {0, 0, 0}, bh[3] = {0, 0, 0};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t lo = wa[k] & 0x0F0F0F0Fu, hi = wa[k] & 0xF0F0F0F0u;
#pragma unroll
        for (int p = 0; p < 3; p++) {
            al[p] = dp4a_us(lo, L.xa[p][k], al[p]);
            ah[p] = dp4a_us(hi, L.xa[p][4 + k], ah[p]);
        }
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t lo = wb[k] & 0x0F0F0F0Fu, hi = wb[k] & 0xF0F0F0F0u;
#pragma unroll
        for (int p = 0; p < 3; p++) {
            bl[p] = dp4a_us(lo, L.xb[p][k], bl[p]);
            bh[p] = dp4a_us(hi, L.xb[p][4 + k], bh[p]);
        }
    }
    const uint32_t sc = __byte_perm(scw, 0u, L.sel);
    const float s0 = (float)((int)(sc << 24) >> 24), s1 = (float)((int)(sc << 16) >> 24);
    const float s2 = (float)((int)(sc << 8) >> 24), s3 = (float)((int)sc >> 24);
    float part = s0 * fmaf(fix24(al[0], al[1], al[2]), L.sxl, -L.xs[0]);
    part = fmaf(s1, fmaf(fix24(bl[0], bl[1], bl[2]), L.sxl, -L.xs[1]), part);
    part = fmaf(s2, fmaf(fix24(ah[0], ah[1], ah[2]), L.sxh, -L.xs[2]), part);
    part = fmaf(s3, fmaf(fix24(bh[0], bh[1], bh[2]), L.sxh, -L.xs[3]), part);
    return __half2float(__ushort_as_half((unsigned short)(dw & 0xFFFFu))) * part;
}

// ------------------------------------------------------------------- Q4_0

struct Q40Lane {
    uint32_t p[3][16];
    float sx0, sx1, xs0, xs1;
    bool has1;
};

__device__ __forceinline__ void q40_lane_setup(Q40Lane& L, const int8_t* planes,
                                               const float4* stats, int64_t in, int64_t nblk,
                                               int64_t b0) {
    L.has1 = b0 + 1 < nblk;
#pragma unroll
    for (int p = 0; p < 3; p++) {
        const uint4* src = reinterpret_cast<const uint4*>(planes + p * in + b0 * 32);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            uint4 v = (k < 2 || L.has1) ? src[k] : make_uint4(0u, 0u, 0u, 0u);
            L.p[p][4 * k] = v.x; L.p[p][4 * k + 1] = v.y;
            L.p[p][4 * k + 2] = v.z; L.p[p][4 * k + 3] = v.w;
        }
    }
    const float4 st0 = stats[b0];
    const float4 st1 = L.has1 ? stats[b0 + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
    L.sx0 = st0.x * 0.0625f;
    L.sx1 = st1.x * 0.0625f;
    L.xs0 = 8.0f * (st0.y + st0.z);
    L.xs1 = 8.0f * (st1.y + st1.z);
}

// qa, qb: quant bytes of blocks b0, b0+1; d0, d1: their f16 scales.
__device__ __forceinline__ float q40_lane_row(const Q40Lane& L, uint4 qa, uint4 qb, uint16_t d0b,
                                              uint16_t d1b) {
    const uint32_t wv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int a[2][3];
#pragma unroll
    for (int blk = 0; blk < 2; blk++) {
        int e1 = 0, e2 = 0, e3 = 0, f1 = 0, f2 = 0, f3 = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t w = wv[4 * blk + k];
            const uint32_t lo = w & 0x0F0F0F0Fu, hi = w & 0xF0F0F0F0u;
            e1 = dp4a_us(lo, L.p[0][8 * blk + k], e1);
            e2 = dp4a_us(lo, L.p[1][8 * blk + k], e2);
            e3 = dp4a_us(lo, L.p[2][8 * blk + k], e3);
            f1 = dp4a_us(hi, L.p[0][8 * blk + 4 + k], f1);
            f2 = dp4a_us(hi, L.p[1][8 * blk + 4 + k], f2);
            f3 = dp4a_us(hi, L.p[2][8 * blk + 4 + k], f3);
        }
        a[blk][0] = 16 * e1 + f1;  // 16 * sum(q * x_plane)
        a[blk][1] = 16 * e2 + f2;
        a[blk][2] = 16 * e3 + f3;
    }
    const float d0 = __half2float(__ushort_as_half(d0b));
    const float d1 = __half2float(__ushort_as_half(d1b));
    const float v0 = fmaf(fix24(a[0][0], a[0][1], a[0][2]), L.sx0, -L.xs0);
    const float v1 = fmaf(fix24(a[1][0], a[1][1], a[1][2]), L.sx1, -L.xs1);
    return fmaf(d0, v0, d1 * v1);
}

// ------------------------------------------------------------------- Q8_0
// Lane of blocks b0, b0+1 (64 weights): signed int8 weights times the three
// signed activation planes by dp4a; w = d * q.  Lanes with bit 1 set take
// the two blocks in swapped order (first = b0+1) so a quarter-warp's
// 128-bit shared loads spread over twice as many banks.
struct Q80Lane {
    uint32_t p[3][16];  // [plane][first block 0..7, second block 8..15]
    float sx0, sx1;     // plane scales of the first / second block
    bool swp, has1;
};

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ void q80_lane_setup(Q80Lane& L, const int8_t* planes, const float4* stats, int64_t in,
                                               int64_t nblk, int64_t b0, bool valid, bool swp) {
    L.has1 = valid && b0 + 1 < nblk;
    L.swp = swp && L.has1;
    const int64_t fb = L.swp ? b0 + 1 : b0, sb = L.swp ? b0 : b0 + 1;
#pragma unroll
    for (int p = 0; p < 3; p++) {
        const uint4* f = reinterpret_cast<const uint4*>(planes + p * in + fb * 32);
        const uint4* s = reinterpret_cast<const uint4*>(planes + p * in + sb * 32);
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const uint4 a = valid ? f[k] : make_uint4(0u, 0u, 0u, 0u);
            const uint4 b = L.has1 ? s[k] : make_uint4(0u, 0u, 0u, 0u);
            L.p[p][4 * k] = a.x; L.p[p][4 * k + 1] = a.y; L.p[p][4 * k + 2] = a.z; L.p[p][4 * k + 3] = a.w;
            L.p[p][8 + 4 * k] = b.x; L.p[p][8 + 4 * k + 1] = b.y; L.p[p][8 + 4 * k + 2] = b.z;
            L.p[p][8 + 4 * k + 3] = b.w;
        }
    }
    L.sx0 = valid ? stats[fb].x : 0.0f;
    L.sx1 = L.has1 ? stats[sb].x : 0.0f;
}

// w0..w3: the first block's 32 quant bytes (w0, w1) then the second's
// (w2, w3); dd: the pair's f16 scales (b0 low, b0+1 high).
__device__ __forceinline__ float q80_lane_row(const Q80Lane& L, uint4 w0, uint4 w1, uint4 w2, uint4 w3,
                                              uint32_t dd) {
    const uint32_t a[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const uint32_t b[8] = {w2.x, w2.y, w2.z, w2.w, w3.x, w3.y, w3.z, w3.w};
    int e1 = 0, e2 = 0, e3 = 0, f1 = 0, f2 = 0, f3 = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        e1 = dp4a_ss(a[k], L.p[0][k], e1);
        e2 = dp4a_ss(a[k], L.p[1][k], e2);
        e3 = dp4a_ss(a[k], L.p[2][k], e3);
        f1 = dp4a_ss(b[k], L.p[0][8 + k], f1);
        f2 = dp4a_ss(b[k], L.p[1][8 + k], f2);
        f3 = dp4a_ss(b[k], L.p[2][8 + k], f3);
    }
    const uint16_t lo = (uint16_t)(dd & 0xFFFFu), hi = (uint16_t)(dd >> 16);
    const float d0 = __half2float(__ushort_as_half(L.swp ? hi : lo));
    const float d1 = L.has1 ? __half2float(__ushort_as_half(L.swp ? lo : hi)) : 0.0f;
    return fmaf(d0, fix24(e1, e2, e3) * L.sx0, d1 * (fix24(f1, f2, f3) * L.sx1));
}

// ------------------------------------------------------------------- Q6_K
// Lane g (0..3) of super-block sb: half n = g / 2, offset l0 = 16 (g & 1);
// its 64 weights are the four groups of 16 at 128n + 32j + l0 (j = 0..3,
// sub-block scale 8n + (g & 1) + 2j).  The 6-bit q of group j is the low
// (j < 2) or high nibble of ql[64n + 32 (j & 1) + l0 ..] with bits 2j, 2j+1
// of qh[32n + l0 ..] on top; w = (d * sc) * (q - 32), so per group
// d * sc * (sx * sum(q X) - 32 * sum(x)) with the group's x sum from the
// block stats.
struct Q6KLane {
    uint32_t p[3][16];  // [plane][group j words 4j .. 4j+3]
    float sx[4], s32[4];  // per group: plane scale, 32 * sum(x)
};

// xmul: factor on the group sums (32 for Q6_K's q - 32, 1 for Q2_K's min)
__device__ __forceinline__ void q6k_lane_setup(Q6KLane& L, const int8_t* planes, const float4* stats, int64_t in,
                                               int64_t sb, int g, bool valid, float xmul = 32.0f) {
    const int n = g >> 1, l0 = 16 * (g & 1);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int64_t blk = sb * 8 + 4 * n + j;  // 32-element block of group j
#pragma unroll
        for (int p = 0; p < 3; p++) {
            const uint4 v = valid ? *reinterpret_cast<const uint4*>(planes + p * in + blk * 32 + l0)
                                  : make_uint4(0u, 0u, 0u, 0u);
            L.p[p][4 * j] = v.x; L.p[p][4 * j + 1] = v.y; L.p[p][4 * j + 2] = v.z; L.p[p][4 * j + 3] = v.w;
        }
        const float4 st = valid ? stats[blk] : make_float4(0.f, 0.f, 0.f, 0.f);
        L.sx[j] = st.x;
        L.s32[j] = xmul * (l0 ? st.z : st.y);
    }
}

// a: ql bytes of groups 0 / 2 (low / high nibbles), b: of groups 1 / 3,
// h: the qh bytes; sc01 / sc23: the header words holding scales 8n .. 8n+3,
// 8n+4 .. 8n+7; dw: the word holding d; gs = g & 1.
__device__ __forceinline__ float q6k_lane_row(const Q6KLane& L, uint4 a, uint4 b, uint4 h, uint32_t sc01,
                                              uint32_t sc23, uint32_t dw, int gs) {
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w}, hw[4] = {h.x, h.y, h.z, h.w};
    int acc[4][3];
#pragma unroll
    for (int j = 0; j < 4; j++) acc[j][0] = acc[j][1] = acc[j][2] = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t q0 = (aw[k] & 0x0F0F0F0Fu) | ((hw[k] << 4) & 0x30303030u);
        const uint32_t q1 = (bw[k] & 0x0F0F0F0Fu) | ((hw[k] << 2) & 0x30303030u);
        const uint32_t q2 = ((aw[k] >> 4) & 0x0F0F0F0Fu) | (hw[k] & 0x30303030u);
        const uint32_t q3 = ((bw[k] >> 4) & 0x0F0F0F0Fu) | ((hw[k] >> 2) & 0x30303030u);
        const uint32_t qv[4] = {q0, q1, q2, q3};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            acc[j][0] = dp4a_us(qv[j], L.p[0][4 * j + k], acc[j][0]);
            acc[j][1] = dp4a_us(qv[j], L.p[1][4 * j + k], acc[j][1]);
            acc[j][2] = dp4a_us(qv[j], L.p[2][4 * j + k], acc[j][2]);
        }
    }
    // scales of groups j = 0..3: bytes gs, gs + 2 of sc01, then of sc23
    const int sh = 8 * gs;
    const float s0 = (float)(int8_t)(sc01 >> sh), s1 = (float)(int8_t)(sc01 >> (sh + 16));
    const float s2 = (float)(int8_t)(sc23 >> sh), s3 = (float)(int8_t)(sc23 >> (sh + 16));
    const float v0 = fmaf(fix24(acc[0][0], acc[0][1], acc[0][2]), L.sx[0], -L.s32[0]);
    const float v1 = fmaf(fix24(acc[1][0], acc[1][1], acc[1][2]), L.sx[1], -L.s32[1]);
    const float v2 = fmaf(fix24(acc[2][0], acc[2][1], acc[2][2]), L.sx[2], -L.s32[2]);
    const float v3 = fmaf(fix24(acc[3][0], acc[3][1], acc[3][2]), L.sx[3], -L.s32[3]);
    const float d = __half2float(__ushort_as_half((uint16_t)(dw & 0xFFFFu)));
    return d * fmaf(s0, v0, fmaf(s1, v1, fmaf(s2, v2, s3 * v3)));
}

// ------------------------------------------------------------------- Q5_K
// The Q4_K pipeline lane with a fifth bit: q = nibble | (bit 2g or 2g+1 of
// qh[j]) << 4 for the low / high nibble of qs[32g + j].  The lane reads the
// qh bytes j of its two 16-byte halves in the same half order as its qs
// bytes; a lane-constant rotation brings bit 2g (2g+1) of every qh byte to
// bit 4, so each 5-bit word costs one more shift and a 3-input logic op.
// High nibbles are shifted down (16 q would not fit a byte), so both
// sub-blocks use the plain plane scale.
struct Q5KLane {
    Q4KPLane b;
    uint32_t rl, rh;  // rotate-right amounts for the low / high sub-block's bit
};

__device__ __forceinline__ void q5k_lane_setup(Q5KLane& L, const int8_t* planes, const float4* stats, int64_t in,
                                               int64_t sb, int g, int h1, bool valid) {
    q4kp_lane_setup(L.b, planes, stats, in, sb, g, h1, valid);
    L.b.sxh = valid ? stats[sb * 8 + 2 * g + 1].x : 0.0f;
    L.rl = (uint32_t)(2 * g - 4) & 31u;
    L.rh = (uint32_t)(2 * g - 3) & 31u;
}

__device__ __forceinline__ float q5k_lane_row(const Q5KLane& L, uint4 qa, uint4 qb, uint4 ha, uint4 hb, uint4 h) {
    const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w}, wb[4] = {qb.x, qb.y, qb.z, qb.w};
    const uint32_t xa[4] = {ha.x, ha.y, ha.z, ha.w}, xb[4] = {hb.x, hb.y, hb.z, hb.w};
    int l1 = 0, l2 = 0, l3 = 0, h1 = 0, h2 = 0, h3 = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t lo = (wa[k] & 0x0F0F0F0Fu) | (__funnelshift_r(xa[k], xa[k], L.rl) & 0x10101010u);
        const uint32_t hi = ((wa[k] >> 4) & 0x0F0F0F0Fu) | (__funnelshift_r(xa[k], xa[k], L.rh) & 0x10101010u);
        l1 = dp4a_us(lo, L.b.xa[0][k], l1);
        l2 = dp4a_us(lo, L.b.xa[1][k], l2);
        l3 = dp4a_us(lo, L.b.xa[2][k], l3);
        h1 = dp4a_us(hi, L.b.xa[0][4 + k], h1);
        h2 = dp4a_us(hi, L.b.xa[1][4 + k], h2);
        h3 = dp4a_us(hi, L.b.xa[2][4 + k], h3);
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t lo = (wb[k] & 0x0F0F0F0Fu) | (__funnelshift_r(xb[k], xb[k], L.rl) & 0x10101010u);
        const uint32_t hi = ((wb[k] >> 4) & 0x0F0F0F0Fu) | (__funnelshift_r(xb[k], xb[k], L.rh) & 0x10101010u);
        l1 = dp4a_us(lo, L.b.xb[0][k], l1);
        l2 = dp4a_us(lo, L.b.xb[1][k], l2);
        l3 = dp4a_us(lo, L.b.xb[2][k], l3);
        h1 = dp4a_us(hi, L.b.xb[0][4 + k], h1);
        h2 = dp4a_us(hi, L.b.xb[1][4 + k], h2);
        h3 = dp4a_us(hi, L.b.xb[2][4 + k], h3);
    }
    const float fl = fix24(l1, l2, l3) * L.b.sxl;
    const float fh = fix24(h1, h2, h3) * L.b.sxh;
    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
    const uint32_t x1 = __byte_perm(L.b.hiG ? h.w : h.y, h.z, L.b.sel1);
    const uint32_t x2 = __byte_perm(h.y, h.z, L.b.sel2);
    const uint32_t w = (x1 & L.b.mA) | ((x1 >> 4) & L.b.mB) | ((x2 >> 2) & L.b.mC);  // [sc0, sc1, m0, m1]
    const float sc0 = (float)(w & 0xFFu), sc1 = (float)((w >> 8) & 0xFFu);
    const float m0 = (float)((w >> 16) & 0xFFu), m1 = (float)(w >> 24);
    return dd.x * fmaf(sc0, fl, sc1 * fh) - dd.y * fmaf(m0, L.b.xsl, m1 * L.b.xsh);
}

// ------------------------------------------------------------------- Q2_K
// Lane g (0..3) of super-block sb owns the same four 16-weight groups as a
// Q6_K lane: 128n + 32j + l0 + (0..15), n = g / 2, l0 = 16 (g & 1), sub-block
// 8n + 2j + (g & 1).  Group j's 2-bit q are bits 2j, 2j+1 of the 16 bytes
// qs[32n + l0 ..]; w = (d * (sc & 15)) * q - dmin * (sc >> 4), so per group
// d * sc * sx * sum(q X) - dmin * m * sum(x).
using Q2KLane = Q6KLane;

// q: the lane's 16 qs bytes; sc01 / sc23: header words holding the scale
// bytes 8n .. 8n+3 and 8n+4 .. 8n+7; dw: the word holding (d, dmin).
__device__ __forceinline__ float q2k_lane_row(const Q2KLane& L, uint4 q, uint32_t sc01, uint32_t sc23, uint32_t dw,
                                              int gs) {
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    int acc[4][3];
#pragma unroll
    for (int j = 0; j < 4; j++) acc[j][0] = acc[j][1] = acc[j][2] = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t qv = (qw[k] >> (2 * j)) & 0x03030303u;
            acc[j][0] = dp4a_us(qv, L.p[0][4 * j + k], acc[j][0]);
            acc[j][1] = dp4a_us(qv, L.p[1][4 * j + k], acc[j][1]);
            acc[j][2] = dp4a_us(qv, L.p[2][4 * j + k], acc[j][2]);
        }
    }
    // scale bytes of groups j = 0..3: bytes gs, gs + 2 of sc01, then of sc23
    const int sh = 8 * gs;
    const uint32_t b0 = sc01 >> sh, b1 = sc01 >> (sh + 16), b2 = sc23 >> sh, b3 = sc23 >> (sh + 16);
    const float v0 = fix24(acc[0][0], acc[0][1], acc[0][2]) * L.sx[0];
    const float v1 = fix24(acc[1][0], acc[1][1], acc[1][2]) * L.sx[1];
    const float v2 = fix24(acc[2][0], acc[2][1], acc[2][2]) * L.sx[2];
    const float v3 = fix24(acc[3][0], acc[3][1], acc[3][2]) * L.sx[3];
    const float dot = fmaf((float)(b0 & 15u), v0, fmaf((float)(b1 & 15u), v1,
                      fmaf((float)(b2 & 15u), v2, (float)(b3 & 15u) * v3)));
    const float mins = fmaf((float)((b0 >> 4) & 15u), L.s32[0], fmaf((float)((b1 >> 4) & 15u), L.s32[1],
                       fmaf((float)((b2 >> 4) & 15u), L.s32[2], (float)((b3 >> 4) & 15u) * L.s32[3])));
    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&dw));
    return fmaf(dd.x, dot, -dd.y * mins);
}

}  // namespace rq
