// rq_layout.cu -- GGML <-> device layout, exact dequantization, and the
// on-device quantizers.
//
// This translation unit is compiled with -fmad=false and spells every
// rounding step with __f*_rn intrinsics: dequantization must be bit-identical
// to GGML's (w = (d*sc)*q - (dmin*m), two roundings), and the quantizers must
// produce the same bytes as the CPU quantizer on the same f32 input.

#include <algorithm>

#include "rq_internal.cuh"

namespace rq {
namespace {

// --------------------------------------------------------------- repacking

// Map byte b of a GGML block to (is_header, offset) in the device layout.
__device__ __forceinline__ bool ggml_byte_slot(int type, int b, int* off) {
    if (type == RQ_Q4_K || type == RQ_Q5_K) {  // [d dmin scales(12)] [qs 128] / [qh 32][qs 128]
        if (b < 16) { *off = b; return true; }
        *off = b - 16; return false;
    }
    if (type == RQ_Q6_K) {  // [ql 128][qh 64][scales 16][d 2]
        if (b < 192) { *off = b; return false; }
        *off = b - 192; return true;  // scales 0..15, d 16..17
    }
    if (type == RQ_Q2_K) {  // [scales 16][qs 64][d 2][dmin 2]
        if (b < 16) { *off = b; return true; }
        if (b < 80) { *off = b - 16; return false; }
        *off = b - 64; return true;  // d 16..17, dmin 18..19
    }
    // Q4_0: [d 2][qs 16]; Q8_0: [d 2][qs 32]
    if (b < 2) { *off = b; return true; }
    *off = b - 2; return false;
}

__global__ void repack_kernel(int type, int bb, int qsb, int hb, const uint8_t* __restrict__ raw,
                              uint8_t* __restrict__ qs, uint8_t* __restrict__ hdr, int64_t blk0,
                              int64_t nbytes) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (; i < nbytes; i += stride) {
        int64_t blk = i / bb + blk0;
        int b = (int)(i % bb);
        int off;
        if (ggml_byte_slot(type, b, &off)) hdr[blk * hb + off] = raw[i];
        else qs[blk * qsb + off] = raw[i];
    }
}

__global__ void unpack_kernel(int type, int bb, int qsb, int hb, uint8_t* __restrict__ raw,
                              const uint8_t* __restrict__ qs, const uint8_t* __restrict__ hdr,
                              int64_t blk0, int64_t nbytes) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (; i < nbytes; i += stride) {
        int64_t blk = i / bb + blk0;
        int b = (int)(i % bb);
        int off;
        raw[i] = ggml_byte_slot(type, b, &off) ? hdr[blk * hb + off] : qs[blk * qsb + off];
    }
}

// Q3_K expanded layout (rq_internal.cuh): per super-block 128 nibble bytes
// of q + 4 in Q4_K's arrangement and 20 header bytes (16 int8 scales, d).

// q + 4 (0..7) of element e of a GGML Q3_K block: 2 low bits from qs
// (byte 32 (c / 4) + e % 32, shift 2 (c % 4)), bit 2 from hmask (byte e % 32,
// bit c), c = e / 32 -- GGML's dequantize_row_q3_K order.
__device__ __forceinline__ int q3k_raw_q4(const uint8_t* blk, int e) {
    const int c = e / 32, j = e % 32;
    const int low = (blk[32 + 32 * (c / 4) + j] >> (2 * (c % 4))) & 3;
    const int hb = (blk[j] >> c) & 1;
    return low | (hb << 2);
}

// The 6-bit scale (0..63) of 16-element sub-block i of a GGML Q3_K block.
__device__ __forceinline__ int q3k_raw_scale(const uint8_t* blk, int i) {
    const uint8_t* sc = blk + 96;
    const int lo = i < 8 ? (sc[i] & 15) : (sc[i - 8] >> 4);
    const int hi = (sc[8 + i % 4] >> (2 * (i / 4))) & 3;
    return lo | (hi << 4);
}

// q + 4 of element e of an expanded super-block (qs part).
__device__ __forceinline__ int q3k_exp_q4(const uint8_t* q, int e) {
    const int c4 = e / 64, w = e % 64;
    const uint8_t b = q[32 * c4 + (w % 32)];
    return w < 32 ? (b & 15) : (b >> 4);
}

// GGML Q3_K blocks -> expanded layout; one thread per output byte (128 qs
// bytes + 20 header bytes per super-block).
__global__ void q3k_expand_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ qs,
                                  uint8_t* __restrict__ hdr, int64_t blk0, int64_t nsb) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (; i < nsb * 148; i += stride) {
        const int64_t sb = i / 148;
        const int b = (int)(i % 148);
        const uint8_t* blk = raw + sb * 110;
        if (b < 128) {
            const int e0 = 64 * (b / 32) + b % 32;
            qs[(blk0 + sb) * 128 + b] = (uint8_t)(q3k_raw_q4(blk, e0) | (q3k_raw_q4(blk, e0 + 32) << 4));
        } else {
            const int h = b - 128;
            uint8_t v = 0;
            if (h < 16) v = (uint8_t)(int8_t)(q3k_raw_scale(blk, h) - 32);
            else if (h < 18) v = blk[108 + h - 16];
            hdr[(blk0 + sb) * 20 + h] = v;
        }
    }
}

// Expanded layout -> GGML Q3_K blocks; one thread per GGML byte.
__global__ void q3k_contract_kernel(uint8_t* __restrict__ raw, const uint8_t* __restrict__ qs,
                                    const uint8_t* __restrict__ hdr, int64_t blk0, int64_t nsb) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (; i < nsb * 110; i += stride) {
        const int64_t sb = i / 110;
        const int b = (int)(i % 110);
        const uint8_t* q = qs + (blk0 + sb) * 128;
        const uint8_t* h = hdr + (blk0 + sb) * 20;
        int v = 0;
        if (b < 32) {  // hmask byte b: bit c = bit 2 of element 32 c + b
            for (int c = 0; c < 8; c++) v |= ((q3k_exp_q4(q, 32 * c + b) >> 2) & 1) << c;
        } else if (b < 96) {  // qs byte: half hh, column j, four 2-bit fields
            const int hh = (b - 32) / 32, j = (b - 32) % 32;
            for (int s = 0; s < 4; s++) v |= (q3k_exp_q4(q, 32 * (4 * hh + s) + j) & 3) << (2 * s);
        } else if (b < 108) {  // packed 6-bit scales
            const int k = b - 96;
            if (k < 8) {
                v = ((((int)(int8_t)h[k]) + 32) & 15) | (((((int)(int8_t)h[k + 8]) + 32) & 15) << 4);
            } else {
                for (int qd = 0; qd < 4; qd++) v |= (((((int)(int8_t)h[4 * qd + k - 8]) + 32) >> 4) & 3) << (2 * qd);
            }
        } else {
            v = h[16 + b - 108];
        }
        raw[sb * 110 + b] = (uint8_t)v;
    }
}

// ----------------------------------------------------------- dequantization

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t* s, int* sc, int* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// One thread per 32 output elements.
__global__ void dequant_kernel(int type, const uint8_t* __restrict__ qs,
                               const uint8_t* __restrict__ hdr, int64_t out, int64_t in,
                               float* __restrict__ y) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t n32 = out * in / 32;
    if (t >= n32) return;
    float v[32];
    if (type == RQ_Q4_K) {
        int64_t sbi = t / 8;  // super-block index, row-major over [out][nblk]
        int s = (int)(t % 8); // sub-block
        const uint8_t* h = hdr + sbi * 16;
        const uint8_t* q = qs + sbi * 128 + 32 * (s / 2);
        float d = h2f((uint16_t)(h[0] | (h[1] << 8)));
        float dmin = h2f((uint16_t)(h[2] | (h[3] << 8)));
        int sc, m;
        q4k_scale_min(s, h + 4, &sc, &m);
        float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
        int shift = (s & 1) * 4;
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = __fsub_rn(__fmul_rn(d1, (float)((q[j] >> shift) & 15)), m1);
    } else if (type == RQ_Q3_K) {  // w = (d * sc) * (q - 4), expanded layout
        int64_t sbi = t / 8;
        int c = (int)(t % 8);  // 32-element chunk
        const uint8_t* q = qs + sbi * 128;
        const uint8_t* h = hdr + sbi * 20;
        float d = h2f((uint16_t)(h[16] | (h[17] << 8)));
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int sub = 2 * c + half;  // 16-element sub-block
            float dl = __fmul_rn(d, (float)(int8_t)h[sub]);
#pragma unroll
            for (int jj = 0; jj < 16; jj++) {
                const int j = 16 * half + jj;
                v[j] = __fmul_rn(dl, (float)(q3k_exp_q4(q, 32 * c + j) - 4));
            }
        }
    } else if (type == RQ_Q5_K) {  // w = (d * sc) * q - (dmin * m), q = nibble | qh bit << 4
        int64_t sbi = t / 8;
        int s = (int)(t % 8);
        const uint8_t* qh = qs + sbi * 160;
        const uint8_t* q = qh + 32 + 32 * (s / 2);
        const uint8_t* h = hdr + sbi * 16;
        float d = h2f((uint16_t)(h[0] | (h[1] << 8)));
        float dmin = h2f((uint16_t)(h[2] | (h[3] << 8)));
        int sc, m;
        q4k_scale_min(s, h + 4, &sc, &m);
        float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
        int shift = (s & 1) * 4;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int qv = ((q[j] >> shift) & 15) | (((qh[j] >> s) & 1) << 4);
            v[j] = __fsub_rn(__fmul_rn(d1, (float)qv), m1);
        }
    } else if (type == RQ_Q2_K) {  // w = (d * (sc & 15)) * q - (dmin * (sc >> 4))
        int64_t sbi = t / 8;
        int c = (int)(t % 8);  // 32-element chunk: half n = c / 4, shift 2 (c % 4)
        const uint8_t* q = qs + sbi * 64 + 32 * (c / 4);
        const uint8_t* h = hdr + sbi * 20;
        float d = h2f((uint16_t)(h[16] | (h[17] << 8)));
        float dmin = h2f((uint16_t)(h[18] | (h[19] << 8)));
        const int shift = 2 * (c % 4);
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int sc = h[2 * c + half];
            const float dl = __fmul_rn(d, (float)(sc & 15)), ml = __fmul_rn(dmin, (float)(sc >> 4));
#pragma unroll
            for (int jj = 0; jj < 16; jj++) {
                const int j = 16 * half + jj;
                v[j] = __fsub_rn(__fmul_rn(dl, (float)((q[j] >> shift) & 3)), ml);
            }
        }
    } else if (type == RQ_Q8_0) {  // w = d * q
        const int8_t* q = reinterpret_cast<const int8_t*>(qs + t * 32);
        float d = h2f((uint16_t)(hdr[2 * t] | (hdr[2 * t + 1] << 8)));
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = __fmul_rn(d, (float)q[j]);
    } else if (type == RQ_Q6_K) {  // w = (d * sc) * (q - 32), GGML dequantize_row_q6_K
        int64_t sbi = t / 8;
        int c = (int)(t % 8);  // 32-element chunk: half n = c / 4, quarter = c % 4
        const uint8_t* ql = qs + sbi * 192;
        const uint8_t* qh = ql + 128;
        const uint8_t* h = hdr + sbi * 20;
        float d = h2f((uint16_t)(h[16] | (h[17] << 8)));
        const int n = c / 4, quarter = c % 4;
#pragma unroll
        for (int l = 0; l < 32; l++) {
            const uint8_t lb = ql[64 * n + l + ((quarter & 1) ? 32 : 0)];
            const int lo = quarter >= 2 ? (lb >> 4) : (lb & 15);
            const int q = (lo | (((qh[32 * n + l] >> (2 * quarter)) & 3) << 4)) - 32;
            const float sc = (float)(int8_t)h[8 * n + l / 16 + 2 * quarter];
            v[l] = __fmul_rn(__fmul_rn(d, sc), (float)q);
        }
    } else {  // Q4_0
        const uint8_t* q = qs + t * 16;
        float d = h2f((uint16_t)(hdr[2 * t] | (hdr[2 * t + 1] << 8)));
#pragma unroll
        for (int j = 0; j < 16; j++) {
            v[j] = __fmul_rn(d, (float)((q[j] & 15) - 8));
            v[j + 16] = __fmul_rn(d, (float)((q[j] >> 4) - 8));
        }
    }
    float4* dst = reinterpret_cast<float4*>(y + t * 32);
#pragma unroll
    for (int k = 0; k < 8; k++) dst[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}

// --------------------------------------------------------------- quantizers
//
// Same f32 operations, in the same order, as the CPU quantizer
// (quantize_q4_k_block / quantize_q3_k_block / the Q4_0 rule of
// src/q4_kernel.rs:137-163), so equal input gives equal bytes.

// Q4_K: one warp per super-block; lane l holds elements 8l..8l+7
// (sub-block l/4, group l/8).
__global__ void quant_q4k_kernel(const float* __restrict__ x, int64_t nsb_total,
                                 uint8_t* __restrict__ qs, uint8_t* __restrict__ hdr) {
    int64_t sbi = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
    int lane = threadIdx.x & 31;
    if (sbi >= nsb_total) return;  // warp-uniform
    const float4* src = reinterpret_cast<const float4*>(x + sbi * 256 + 8 * lane);
    float4 a = src[0], b = src[1];
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float mn = v[0], mx = v[0];
#pragma unroll
    for (int i = 1; i < 8; i++) { mn = fminf(mn, v[i]); mx = fmaxf(mx, v[i]); }
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (mn > 0.0f) mn = 0.0f;
    float scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    float mins = -mn;
    float max_scale = scale, max_min = mins;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, o));
        max_min = fmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, o));
    }
    // the CPU quantizer starts both maxima at +0.0 and only replaces them
    // with larger values: an all-zero (or all -0.0) set stays +0.0
    if (!(max_scale > 0.0f)) max_scale = 0.0f;
    if (!(max_min > 0.0f)) max_min = 0.0f;
    float inv_scale = max_scale > 0.0f ? __fdiv_rn(63.0f, max_scale) : 0.0f;
    float inv_min = max_min > 0.0f ? __fdiv_rn(63.0f, max_min) : 0.0f;
    int ls = min(63, __float2int_rn(__fmul_rn(inv_scale, scale)));
    int lm = min(63, __float2int_rn(__fmul_rn(inv_min, mins)));
    __half dh = __float2half_rn(__fdiv_rn(max_scale, 63.0f));
    __half mh = __float2half_rn(__fdiv_rn(max_min, 63.0f));
    float d = __half2float(dh), dmin = __half2float(mh);
    float dl = __fmul_rn(d, (float)ls), ml = __fmul_rn(dmin, (float)lm);
    uint32_t pk[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int q = 0;
        if (dl != 0.0f) q = min(15, max(0, __float2int_rn(__fdiv_rn(__fadd_rn(v[i], ml), dl))));
        pk[i / 4] |= (uint32_t)q << (8 * (i % 4));
    }
    // lanes with (l%8) < 4 hold low nibbles of bytes 8*(l%8)..+7 of group l/8,
    // the partner lane l^4 the high nibbles.
    uint32_t p0 = __shfl_xor_sync(0xffffffffu, pk[0], 4);
    uint32_t p1 = __shfl_xor_sync(0xffffffffu, pk[1], 4);
    if ((lane & 7) < 4) {
        uint2 outv = make_uint2(pk[0] | (p0 << 4), pk[1] | (p1 << 4));
        *reinterpret_cast<uint2*>(qs + sbi * 128 + 32 * (lane / 8) + 8 * (lane & 7)) = outv;
    }
    int all_ls[8], all_lm[8];
#pragma unroll
    for (int s = 0; s < 8; s++) {
        all_ls[s] = __shfl_sync(0xffffffffu, ls, 4 * s);
        all_lm[s] = __shfl_sync(0xffffffffu, lm, 4 * s);
    }
    if (lane == 0) {
        uint8_t hb[16];
        uint16_t dbits = __half_as_ushort(dh), mbits = __half_as_ushort(mh);
        hb[0] = (uint8_t)dbits; hb[1] = (uint8_t)(dbits >> 8);
        hb[2] = (uint8_t)mbits; hb[3] = (uint8_t)(mbits >> 8);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            hb[4 + j] = (uint8_t)(all_ls[j] | ((all_ls[j + 4] >> 4) << 6));
            hb[8 + j] = (uint8_t)(all_lm[j] | ((all_lm[j + 4] >> 4) << 6));
            hb[12 + j] = (uint8_t)((all_ls[j + 4] & 15) | ((all_lm[j + 4] & 15) << 4));
        }
        uint4 hv;
        hv.x = hb[0] | (hb[1] << 8) | (hb[2] << 16) | ((uint32_t)hb[3] << 24);
        hv.y = hb[4] | (hb[5] << 8) | (hb[6] << 16) | ((uint32_t)hb[7] << 24);
        hv.z = hb[8] | (hb[9] << 8) | (hb[10] << 16) | ((uint32_t)hb[11] << 24);
        hv.w = hb[12] | (hb[13] << 8) | (hb[14] << 16) | ((uint32_t)hb[15] << 24);
        *reinterpret_cast<uint4*>(hdr + sbi * 16) = hv;
    }
}

// Q3_K: one warp per super-block; lane l holds elements 8l..8l+7
// (16-element sub-block l/2; 32-element chunk c = l/4: h = c/4, s = c%4;
// byte offset j = 8*(l%4) .. +7).
__global__ void quant_q3k_kernel(const float* __restrict__ x, int64_t nsb_total,
                                 uint8_t* __restrict__ qs, uint8_t* __restrict__ hdr) {
    int64_t sbi = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
    int lane = threadIdx.x & 31;
    if (sbi >= nsb_total) return;
    const float4* src = reinterpret_cast<const float4*>(x + sbi * 256 + 8 * lane);
    float4 a = src[0], b = src[1];
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float ma = 0.0f, mv = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float av = fabsf(v[i]);
        if (av > ma) { ma = av; mv = v[i]; }
    }
    // sub-block = lanes (2k, 2k+1); the first strict maximum wins
    float ma_o = __shfl_xor_sync(0xffffffffu, ma, 1);
    float mv_o = __shfl_xor_sync(0xffffffffu, mv, 1);
    if (lane & 1) {  // upper half: keep own only if strictly larger than lower
        if (!(ma > ma_o)) { ma = ma_o; mv = mv_o; }
    } else {
        if (ma_o > ma) { ma = ma_o; mv = mv_o; }
    }
    float scale = __fdiv_rn(mv, -4.0f);
    // first sub-block with the largest |scale|
    float best = fabsf(scale);
    float best_s = scale;
    int best_i = lane >> 1;
#pragma unroll
    for (int o = 2; o < 32; o <<= 1) {
        float ob = __shfl_xor_sync(0xffffffffu, best, o);
        float os = __shfl_xor_sync(0xffffffffu, best_s, o);
        int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (ob > best || (ob == best && oi < best_i)) { best = ob; best_s = os; best_i = oi; }
    }
    float max_scale = best > 0.0f ? best_s : 0.0f;
    float iscale = max_scale != 0.0f ? __fdiv_rn(-32.0f, max_scale) : 0.0f;
    int l = __float2int_rn(__fmul_rn(iscale, scale));
    l = max(-32, min(31, l));
    __half dh = __float2half_rn(iscale != 0.0f ? __fdiv_rn(1.0f, iscale) : 0.0f);
    float d = __half2float(dh);
    float dl = __fmul_rn(d, (float)l);
    // expanded layout: element 8 lane + i is nibble (q + 4) of byte
    // 32 (lane / 8) + 8 (lane % 4) + i, the low nibble for lane % 8 < 4
    unsigned long long part = 0ull;
    const int nshift = (lane & 4) ? 4 : 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int q = 0;
        if (dl != 0.0f) q = max(-4, min(3, __float2int_rn(__fdiv_rn(v[i], dl))));
        part |= (unsigned long long)((q + 4) << nshift) << (8 * i);
    }
    part |= __shfl_xor_sync(0xffffffffu, part, 4);
    if (!(lane & 4))
        *reinterpret_cast<unsigned long long*>(qs + sbi * 128 + 32 * (lane / 8) + 8 * (lane & 3)) = part;
    int all_l[16];
#pragma unroll
    for (int k = 0; k < 16; k++) all_l[k] = __shfl_sync(0xffffffffu, l, 2 * k);
    if (lane == 0) {
        uint32_t w[5];
#pragma unroll
        for (int k = 0; k < 4; k++)
            w[k] = (uint32_t)(uint8_t)(int8_t)all_l[4 * k] | ((uint32_t)(uint8_t)(int8_t)all_l[4 * k + 1] << 8) |
                   ((uint32_t)(uint8_t)(int8_t)all_l[4 * k + 2] << 16) |
                   ((uint32_t)(uint8_t)(int8_t)all_l[4 * k + 3] << 24);
        w[4] = (uint32_t)__half_as_ushort(dh);
        uint32_t* hp = reinterpret_cast<uint32_t*>(hdr + sbi * 20);
#pragma unroll
        for (int k = 0; k < 5; k++) hp[k] = w[k];
    }
}

// Q4_0: one thread per 32-element block (src/q4_kernel.rs:137-163).
__global__ void quant_q40_kernel(const float* __restrict__ x, int64_t nblk_total,
                                 uint8_t* __restrict__ qs, uint8_t* __restrict__ hdr) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nblk_total) return;
    const float* c = x + t * 32;
    float max_abs = 0.0f, max_signed = 0.0f;
    for (int i = 0; i < 32; i++) {
        float a = fabsf(c[i]);
        if (a > max_abs) { max_abs = a; max_signed = c[i]; }
    }
    float d = __fdiv_rn(max_signed, -8.0f);
    float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    // the header array is 256-byte aligned, so block t's f16 scale is a
    // naturally aligned 16-bit word
    reinterpret_cast<__half*>(hdr)[t] = __float2half_rn(d);
    uint8_t* q = qs + t * 16;
    for (int i = 0; i < 16; i++) {
        float a = __fadd_rn(__fmul_rn(c[i], id), 8.5f);
        float b = __fadd_rn(__fmul_rn(c[i + 16], id), 8.5f);
        a = (a != a) ? 0.0f : fminf(fmaxf(a, 0.0f), 15.0f);
        b = (b != b) ? 0.0f : fminf(fmaxf(b, 0.0f), 15.0f);
        q[i] = (uint8_t)(__float2uint_rz(a) | (__float2uint_rz(b) << 4));
    }
}

// Q8_0: one thread per 32-element block (GGML quantize_row_q8_0_ref /
// candle BlockQ8_0::from_float): d = amax / 127, q = round(x / d) with ties
// away from zero.
__global__ void quant_q80_kernel(const float* __restrict__ x, int64_t nblk_total, uint8_t* __restrict__ qs,
                                 uint8_t* __restrict__ hdr) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nblk_total) return;
    const float* c = x + t * 32;
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(c[i]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    reinterpret_cast<__half*>(hdr)[t] = __float2half_rn(d);
    int8_t* q = reinterpret_cast<int8_t*>(qs + t * 32);
    for (int i = 0; i < 32; i++) q[i] = (int8_t)(int)roundf(__fmul_rn(c[i], id));
}

// Q6_K: one thread per super-block, the oracle's rule: per 16 elements
// scale = amax / 31, d = max scale / 127 (as f16), sc = rint(scale / d)
// (int8), q = rint(x / (d sc)) in [-32, 31] stored as q + 32.
__global__ void quant_q6k_kernel(const float* __restrict__ x, int64_t nsb, uint8_t* __restrict__ qs,
                                 uint8_t* __restrict__ hdr) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nsb) return;
    const float* c = x + t * 256;
    float scale[16], amax_all = 0.0f;
    for (int j = 0; j < 16; j++) {
        float amax = 0.0f;
        for (int k = 0; k < 16; k++) amax = fmaxf(amax, fabsf(c[16 * j + k]));
        scale[j] = __fdiv_rn(amax, 31.0f);
        amax_all = fmaxf(amax_all, scale[j]);
    }
    const __half dh = __float2half_rn(__fdiv_rn(amax_all, 127.0f));
    const float df = __half2float(dh);
    uint8_t* h = hdr + t * 20;
    int sc[16];
    for (int j = 0; j < 16; j++) {
        int v = df != 0.0f ? __float2int_rn(__fdiv_rn(scale[j], df)) : 0;
        sc[j] = v > 127 ? 127 : (v < -128 ? -128 : v);
        h[j] = (uint8_t)(int8_t)sc[j];
    }
    const uint16_t db = __half_as_ushort(dh);
    h[16] = (uint8_t)(db & 255u);
    h[17] = (uint8_t)(db >> 8);
    h[18] = h[19] = 0;
    uint8_t* ql = qs + t * 192;
    uint8_t* qh = ql + 128;
    for (int i = 0; i < 192; i++) ql[i] = 0;
    for (int i = 0; i < 256; i++) {
        const int j = i / 16;
        const float dl = __fmul_rn(df, (float)sc[j]);
        int q = dl != 0.0f ? __float2int_rn(__fdiv_rn(c[i], dl)) : 0;
        q = q < -32 ? -32 : (q > 31 ? 31 : q);
        const int u = q + 32;
        const int n = i / 128, r = i % 128, quarter = r / 32, l = r % 32;
        const int lb = 64 * n + l + ((quarter & 1) ? 32 : 0);
        ql[lb] |= (uint8_t)(quarter >= 2 ? ((u & 15) << 4) : (u & 15));
        qh[32 * n + l] |= (uint8_t)((u >> 4) << (2 * quarter));
    }
}

// Q5_K: one warp per super-block, the Q4_K rule with 5-bit q (scale =
// (max - min) / 31); lane l holds elements 8l..8l+7 (sub-block l/4).
__global__ void quant_q5k_kernel(const float* __restrict__ x, int64_t nsb_total,
                                 uint8_t* __restrict__ qs, uint8_t* __restrict__ hdr) {
    int64_t sbi = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
    int lane = threadIdx.x & 31;
    if (sbi >= nsb_total) return;  // warp-uniform
    const float4* src = reinterpret_cast<const float4*>(x + sbi * 256 + 8 * lane);
    float4 a = src[0], b = src[1];
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float mn = v[0], mx = v[0];
#pragma unroll
    for (int i = 1; i < 8; i++) { mn = fminf(mn, v[i]); mx = fmaxf(mx, v[i]); }
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (mn > 0.0f) mn = 0.0f;
    float scale = __fdiv_rn(__fsub_rn(mx, mn), 31.0f);
    float mins = -mn;
    float max_scale = scale, max_min = mins;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, o));
        max_min = fmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, o));
    }
    if (!(max_scale > 0.0f)) max_scale = 0.0f;
    if (!(max_min > 0.0f)) max_min = 0.0f;
    float inv_scale = max_scale > 0.0f ? __fdiv_rn(63.0f, max_scale) : 0.0f;
    float inv_min = max_min > 0.0f ? __fdiv_rn(63.0f, max_min) : 0.0f;
    int ls = min(63, __float2int_rn(__fmul_rn(inv_scale, scale)));
    int lm = min(63, __float2int_rn(__fmul_rn(inv_min, mins)));
    __half dh = __float2half_rn(__fdiv_rn(max_scale, 63.0f));
    __half mh = __float2half_rn(__fdiv_rn(max_min, 63.0f));
    float d = __half2float(dh), dmin = __half2float(mh);
    float dl = __fmul_rn(d, (float)ls), ml = __fmul_rn(dmin, (float)lm);
    const int s = lane / 4;
    uint32_t pk[2] = {0u, 0u};
    unsigned long long hp = 0ull;  // bit s of qh bytes 8 (l % 4) .. +7
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int q = 0;
        if (dl != 0.0f) q = min(31, max(0, __float2int_rn(__fdiv_rn(__fadd_rn(v[i], ml), dl))));
        pk[i / 4] |= (uint32_t)(q & 15) << (8 * (i % 4));
        hp |= (unsigned long long)((q >> 4) << s) << (8 * i);
    }
    uint32_t p0 = __shfl_xor_sync(0xffffffffu, pk[0], 4);
    uint32_t p1 = __shfl_xor_sync(0xffffffffu, pk[1], 4);
    // the 8 sub-blocks' bits of one qh byte sit on lanes differing in bits 2..4
    hp |= __shfl_xor_sync(0xffffffffu, hp, 4);
    hp |= __shfl_xor_sync(0xffffffffu, hp, 8);
    hp |= __shfl_xor_sync(0xffffffffu, hp, 16);
    uint8_t* base = qs + sbi * 160;
    if (lane < 4) *reinterpret_cast<unsigned long long*>(base + 8 * lane) = hp;
    if ((lane & 7) < 4) {
        uint2 outv = make_uint2(pk[0] | (p0 << 4), pk[1] | (p1 << 4));
        *reinterpret_cast<uint2*>(base + 32 + 32 * (lane / 8) + 8 * (lane & 7)) = outv;
    }
    int all_ls[8], all_lm[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        all_ls[k] = __shfl_sync(0xffffffffu, ls, 4 * k);
        all_lm[k] = __shfl_sync(0xffffffffu, lm, 4 * k);
    }
    if (lane == 0) {
        uint8_t hb[16];
        uint16_t dbits = __half_as_ushort(dh), mbits = __half_as_ushort(mh);
        hb[0] = (uint8_t)dbits; hb[1] = (uint8_t)(dbits >> 8);
        hb[2] = (uint8_t)mbits; hb[3] = (uint8_t)(mbits >> 8);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            hb[4 + j] = (uint8_t)(all_ls[j] | ((all_ls[j + 4] >> 4) << 6));
            hb[8 + j] = (uint8_t)(all_lm[j] | ((all_lm[j + 4] >> 4) << 6));
            hb[12 + j] = (uint8_t)((all_ls[j + 4] & 15) | ((all_lm[j + 4] & 15) << 4));
        }
        uint4 hv;
        hv.x = hb[0] | (hb[1] << 8) | (hb[2] << 16) | ((uint32_t)hb[3] << 24);
        hv.y = hb[4] | (hb[5] << 8) | (hb[6] << 16) | ((uint32_t)hb[7] << 24);
        hv.z = hb[8] | (hb[9] << 8) | (hb[10] << 16) | ((uint32_t)hb[11] << 24);
        hv.w = hb[12] | (hb[13] << 8) | (hb[14] << 16) | ((uint32_t)hb[15] << 24);
        *reinterpret_cast<uint4*>(hdr + sbi * 16) = hv;
    }
}

// Q2_K: one thread per super-block, the oracle's rule: per 16 elements
// scale = (max - min) / 3 and min = -min(0, smallest), 4-bit ls / lm
// against the super-block maxima, q = rint((x + dmin lm) / (d ls)) in 0..3.
__global__ void quant_q2k_kernel(const float* __restrict__ x, int64_t nsb, uint8_t* __restrict__ qs,
                                 uint8_t* __restrict__ hdr) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nsb) return;
    const float* c = x + t * 256;
    float scale[16], mins[16], max_scale = 0.0f, max_min = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        float mn = c[16 * j], mx = c[16 * j];
#pragma unroll
        for (int k = 1; k < 16; k++) { mn = fminf(mn, c[16 * j + k]); mx = fmaxf(mx, c[16 * j + k]); }
        if (mn > 0.0f) mn = 0.0f;
        scale[j] = __fdiv_rn(__fsub_rn(mx, mn), 3.0f);
        mins[j] = -mn;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (mins[j] > max_min) max_min = mins[j];
    }
    const float inv_scale = max_scale > 0.0f ? __fdiv_rn(15.0f, max_scale) : 0.0f;
    const float inv_min = max_min > 0.0f ? __fdiv_rn(15.0f, max_min) : 0.0f;
    const __half dh = __float2half_rn(__fdiv_rn(max_scale, 15.0f));
    const __half mh = __float2half_rn(__fdiv_rn(max_min, 15.0f));
    const float d = __half2float(dh), dmin = __half2float(mh);
    // header words: scales 0..15, then (d, dmin); quant words: 64 bytes, byte
    // 32n + l holds the 2-bit q of elements 128n + 32 sh + l at bits 2 sh
    uint32_t hw[5] = {0u, 0u, 0u, 0u, 0u}, qw[16];
#pragma unroll
    for (int k = 0; k < 16; k++) qw[k] = 0u;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const int ls = min(15, __float2int_rn(__fmul_rn(inv_scale, scale[j])));
        const int lm = min(15, __float2int_rn(__fmul_rn(inv_min, mins[j])));
        hw[j / 4] |= (uint32_t)(ls | (lm << 4)) << (8 * (j % 4));
        const float dl = __fmul_rn(d, (float)ls), ml = __fmul_rn(dmin, (float)lm);
        const int n = j / 8, sh = (j % 8) / 2, l0 = 16 * (j % 2);
#pragma unroll
        for (int k = 0; k < 16; k++) {
            int v = 0;
            if (dl != 0.0f) v = min(3, max(0, __float2int_rn(__fdiv_rn(__fadd_rn(c[16 * j + k], ml), dl))));
            const int byte = 32 * n + l0 + k;
            qw[byte / 4] |= (uint32_t)v << (8 * (byte % 4) + 2 * sh);
        }
    }
    hw[4] = (uint32_t)__half_as_ushort(dh) | ((uint32_t)__half_as_ushort(mh) << 16);
    // 20 t is a multiple of 4 and the header array is 256-byte aligned
    uint32_t* hp = reinterpret_cast<uint32_t*>(hdr + t * 20);
#pragma unroll
    for (int k = 0; k < 5; k++) hp[k] = hw[k];
    uint4* qp = reinterpret_cast<uint4*>(qs + t * 64);
#pragma unroll
    for (int k = 0; k < 4; k++) qp[k] = make_uint4(qw[4 * k], qw[4 * k + 1], qw[4 * k + 2], qw[4 * k + 3]);
}

int grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    return (int)(g > (1 << 30) ? (1 << 30) : g);
}

}  // namespace

int launch_repack(const rq_weight* w, const uint8_t* raw_dev, int64_t row0, int64_t rows,
                  cudaStream_t st) {
    TypeInfo ti = type_info(w->type);
    int64_t nbytes = rows * w->nblk * ti.block_bytes;
    if (nbytes == 0) return RQ_OK;
    if (w->type == RQ_Q3_K) {
        const int64_t nsb = rows * w->nblk;
        const int64_t grid = std::min<int64_t>((nsb * 148 + 255) / 256, 148 * 64);
        q3k_expand_kernel<<<(unsigned)grid, 256, 0, st>>>(raw_dev, w->qs, w->hdr, row0 * w->nblk, nsb);
        return cuda_error(cudaGetLastError(), "Q3_K expand kernel");
    }
    int64_t grid = (nbytes + 255) / 256;
    if (grid > 148 * 64) grid = 148 * 64;
    repack_kernel<<<(unsigned)grid, 256, 0, st>>>(w->type, ti.block_bytes, ti.qs_bytes, ti.hdr_bytes,
                                                  raw_dev, w->qs, w->hdr, row0 * w->nblk, nbytes);
    return cuda_error(cudaGetLastError(), "repack kernel");
}

int launch_unpack(const rq_weight* w, uint8_t* raw_dev, int64_t row0, int64_t rows,
                  cudaStream_t st) {
    TypeInfo ti = type_info(w->type);
    int64_t nbytes = rows * w->nblk * ti.block_bytes;
    if (nbytes == 0) return RQ_OK;
    if (w->type == RQ_Q3_K) {
        const int64_t nsb = rows * w->nblk;
        const int64_t grid = std::min<int64_t>((nsb * 110 + 255) / 256, 148 * 64);
        q3k_contract_kernel<<<(unsigned)grid, 256, 0, st>>>(raw_dev, w->qs, w->hdr, row0 * w->nblk, nsb);
        return cuda_error(cudaGetLastError(), "Q3_K contract kernel");
    }
    int64_t grid = (nbytes + 255) / 256;
    if (grid > 148 * 64) grid = 148 * 64;
    unpack_kernel<<<(unsigned)grid, 256, 0, st>>>(w->type, ti.block_bytes, ti.qs_bytes, ti.hdr_bytes,
                                                  raw_dev, w->qs, w->hdr, row0 * w->nblk, nbytes);
    return cuda_error(cudaGetLastError(), "unpack kernel");
}

int launch_dequant(const rq_weight* w, float* y, cudaStream_t st) {
    int64_t n32 = w->out * w->in / 32;
    if (n32 == 0) return RQ_OK;
    dequant_kernel<<<grid_for(n32, 256), 256, 0, st>>>(w->type, w->qs, w->hdr, w->out, w->in, y);
    return cuda_error(cudaGetLastError(), "dequant kernel");
}

int launch_quantize(const rq_weight* w, const float* x, cudaStream_t st) {
    if (w->out * w->in == 0) return RQ_OK;
    if (w->type == RQ_Q8_0) {
        int64_t nb = w->out * w->nblk;
        quant_q80_kernel<<<grid_for(nb, 128), 128, 0, st>>>(x, nb, w->qs, w->hdr);
    } else if (w->type == RQ_Q6_K) {
        int64_t nsb = w->out * w->nblk;
        quant_q6k_kernel<<<grid_for(nsb, 128), 128, 0, st>>>(x, nsb, w->qs, w->hdr);
    } else if (w->type == RQ_Q2_K) {
        int64_t nsb = w->out * w->nblk;
        quant_q2k_kernel<<<grid_for(nsb, 128), 128, 0, st>>>(x, nsb, w->qs, w->hdr);
    } else if (w->type == RQ_Q5_K) {
        int64_t threads = w->out * w->nblk * 32;
        quant_q5k_kernel<<<grid_for(threads, 256), 256, 0, st>>>(x, w->out * w->nblk, w->qs, w->hdr);
    } else if (w->type == RQ_Q4_K || w->type == RQ_Q3_K) {
        int64_t nsb = w->out * w->nblk;
        int64_t threads = nsb * 32;
        if (w->type == RQ_Q4_K)
            quant_q4k_kernel<<<grid_for(threads, 256), 256, 0, st>>>(x, nsb, w->qs, w->hdr);
        else
            quant_q3k_kernel<<<grid_for(threads, 256), 256, 0, st>>>(x, nsb, w->qs, w->hdr);
    } else {
        int64_t nb = w->out * w->nblk;
        quant_q40_kernel<<<grid_for(nb, 128), 128, 0, st>>>(x, nb, w->qs, w->hdr);
    }
    return cuda_error(cudaGetLastError(), "quantize kernel");
}

}  // namespace rq
