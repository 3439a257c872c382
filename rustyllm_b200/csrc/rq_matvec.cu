// rq_matvec.cu -- activation staging and the M=1 decode matvec kernels
// (Q4_K, Q3_K, Q4_0) for sm_100a.
//
// Design (HBM-bound: one pass over the packed weights, nothing dequantized is
// ever written back):
//   * The activation row is staged once per call into 24-bit fixed point per
//     32-element block (three int8 planes, see rq_internal.cuh), so the inner
//     product of 4-bit quants with x is exact integer arithmetic: dp4a on the
//     nibbles as they sit in the packed bytes (low nibbles masked in place,
//     high nibbles masked in place and carried as 16*q).
//   * A CTA owns R consecutive output rows and all of K.  K is cut into
//     slices of 2048 elements (8 super-blocks); warp w takes slices
//     w, w+NW, ...  Within a slice lane l owns one 64-element group, keeps
//     that group's activation planes in registers for all R rows, and streams
//     the weights with 128-bit loads (each warp load is 1 KB contiguous).
//   * Per-row lane partials are folded with a transpose reduction
//     (R values over 32 lanes in R-1 shuffles), then across warps through
//     shared memory in a fixed order, so results are deterministic.

#include "rq_internal.cuh"

namespace rq {
namespace {

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// ------------------------------------------------------ activation staging

// One thread per 32-element block of one activation row.
__global__ void xquant_kernel(const float* __restrict__ x, int64_t M, int64_t in,
                              int8_t* __restrict__ planes, float4* __restrict__ stats) {
    int64_t nb = in / 32;
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= M * nb) return;
    int64_t m = t / nb, b = t % nb;
    const float* src = x + m * in + b * 32;
    float v[32];
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
#pragma unroll
        for (int k = 0; k < 8; k++) {
            float4 f = reinterpret_cast<const float4*>(src)[k];
            v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int k = 0; k < 32; k++) v[k] = src[k];
    }
    float amax = 0.0f, sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; k++) { amax = fmaxf(amax, fabsf(v[k])); sa += v[k]; }
#pragma unroll
    for (int k = 16; k < 32; k++) { amax = fmaxf(amax, fabsf(v[k])); sb += v[k]; }
    float inv = amax > 0.0f ? kXQScale / amax : 0.0f;
    float sx = amax / kXQScale;
    uint32_t p1[8], p2[8], p3[8];
#pragma unroll
    for (int k = 0; k < 8; k++) { p1[k] = 0u; p2[k] = 0u; p3[k] = 0u; }
#pragma unroll
    for (int k = 0; k < 32; k++) {
        int X = __float2int_rn(v[k] * inv);
        int x3 = (X << 24) >> 24;           // balanced base-256 digits
        int t1 = (X - x3) >> 8;
        int x2 = (t1 << 24) >> 24;
        int x1 = (t1 - x2) >> 8;
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
    stats[t] = make_float4(sx, sa, sb, 0.0f);
}

// ----------------------------------------------------- transpose reduction
//
// v[0..N) are this lane's partials for N rows.  After the call v[0] holds the
// full 32-lane sum of row row_of_lane<N>(lane).
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
    // lanes that hold a row after the reduction: the low bits not used to
    // index rows are zero
    constexpr int used = (N >= 32) ? 5 : (N >= 16) ? 4 : (N >= 8) ? 3 : (N >= 4) ? 2 : (N >= 2) ? 1 : 0;
    return (lane & ((1 << (5 - used)) - 1)) == 0;
}

// ---------------------------------------------------------- shared pieces

struct GroupX {      // activation planes of one 64-element group, one token
    uint32_t p[3][16];
};

__device__ __forceinline__ void load_group_x(GroupX& gx, const int8_t* planes, int64_t in,
                                             int64_t pos) {
#pragma unroll
    for (int p = 0; p < 3; p++) {
        const uint4* src = reinterpret_cast<const uint4*>(planes + p * in + pos);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            uint4 u = src[k];
            gx.p[p][4 * k] = u.x; gx.p[p][4 * k + 1] = u.y;
            gx.p[p][4 * k + 2] = u.z; gx.p[p][4 * k + 3] = u.w;
        }
    }
}

__device__ __forceinline__ float fix24(int d1, int d2, int d3) {
    // d1*65536 + d2*256 + d3 with one final rounding
    return fmaf((float)d1, 65536.0f, (float)(d2 * 256 + d3));
}

// ================================================================== Q4_K

template <int R>
__global__ void __launch_bounds__(256, 2)
mv_q4k_kernel(const uint8_t* __restrict__ qs, const uint8_t* __restrict__ hdr,
              const int8_t* __restrict__ planes, const float4* __restrict__ stats,
              float* __restrict__ y, int64_t out, int64_t nsb, int64_t in) {
    __shared__ float red[8][R];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int64_t row0 = (int64_t)blockIdx.x * R;
    const int64_t nslice = (nsb + 7) / 8;
    float part[R];
#pragma unroll
    for (int r = 0; r < R; r++) part[r] = 0.0f;

    for (int64_t s = warp; s < nslice; s += nw) {
        const int64_t gidx = s * 32 + lane;
        const int64_t sb = gidx >> 2;
        const int g = (int)(gidx & 3);
        if (sb < nsb) {
            GroupX gx;
            load_group_x(gx, planes, in, sb * 256 + 64 * g);
            const float4 st_lo = stats[sb * 8 + 2 * g];
            const float4 st_hi = stats[sb * 8 + 2 * g + 1];
            const float sxl = st_lo.x, xsl = st_lo.y + st_lo.z;
            const float sxh = st_hi.x * 0.0625f, xsh = st_hi.y + st_hi.z;
            // scale/min unpacking constants for sub-blocks 2g, 2g+1
            const bool hiG = g >= 2;
            const int sh = 16 * (g & 1);
            const uint32_t mL = hiG ? 0x0F0Fu : 0x3F3Fu;
            const uint32_t mH = hiG ? 0x3030u : 0u;
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int64_t row = row0 + r;
                if (row < out) {
                    const int64_t bi = row * nsb + sb;
                    const uint8_t* wp = qs + bi * 128 + 32 * g;
                    const uint4 qa = ldg_stream(wp);
                    const uint4 qb = ldg_stream(wp + 16);
                    const uint4 h = ldg_stream(hdr + bi * 16);
                    const uint32_t wv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    int l1 = 0, l2 = 0, l3 = 0, h1 = 0, h2 = 0, h3 = 0;
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const uint32_t lo = wv[k] & 0x0F0F0F0Fu;
                        const uint32_t hi = wv[k] & 0xF0F0F0F0u;
                        l1 = dp4a_us(lo, gx.p[0][k], l1);
                        l2 = dp4a_us(lo, gx.p[1][k], l2);
                        l3 = dp4a_us(lo, gx.p[2][k], l3);
                        h1 = dp4a_us(hi, gx.p[0][8 + k], h1);
                        h2 = dp4a_us(hi, gx.p[1][8 + k], h2);
                        h3 = dp4a_us(hi, gx.p[2][8 + k], h3);
                    }
                    const float fl = fix24(l1, l2, l3) * sxl;
                    const float fh = fix24(h1, h2, h3) * sxh;
                    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                    const uint32_t A = hiG ? h.w : h.y;
                    const uint32_t B = hiG ? (h.w >> 4) : h.z;
                    const uint32_t scp = ((A >> sh) & mL) | ((h.y >> (sh + 2)) & mH);
                    const uint32_t mp = ((B >> sh) & mL) | ((h.z >> (sh + 2)) & mH);
                    const float sc0 = (float)(scp & 0xFFu), sc1 = (float)((scp >> 8) & 0xFFu);
                    const float m0 = (float)(mp & 0xFFu), m1 = (float)((mp >> 8) & 0xFFu);
                    part[r] += dd.x * fmaf(sc0, fl, sc1 * fh) - dd.y * fmaf(m0, xsl, m1 * xsh);
                }
            }
        }
    }
    transpose_reduce<R>(part, lane);
    if (lane_writes<R>(lane)) red[warp][row_of_lane<R>(lane)] = part[0];
    __syncthreads();
    if (threadIdx.x < R) {
        float acc = 0.0f;
        for (int w = 0; w < nw; w++) acc += red[w][threadIdx.x];
        const int64_t row = row0 + threadIdx.x;
        if (row < out) y[row] = acc;
    }
}

// ================================================================== Q3_K
// Lane owns quarter qq of a super-block: h = qq>>1, u = qq&1, i.e. elements
// 128h + 32s + 16u + jj (s = 0..3, jj = 0..15): qs bytes [32h+16u, +16),
// hmask bytes [16u, +16) (bit 4h+s), 16-element sub-blocks 8h + 2s + u.

template <int R>
__global__ void __launch_bounds__(256, 2)
mv_q3k_kernel(const uint8_t* __restrict__ qs, const uint8_t* __restrict__ hdr,
              const int8_t* __restrict__ planes, const float4* __restrict__ stats,
              float* __restrict__ y, int64_t out, int64_t nsb, int64_t in) {
    __shared__ float red[8][R];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int64_t row0 = (int64_t)blockIdx.x * R;
    const int64_t nslice = (nsb + 7) / 8;
    float part[R];
#pragma unroll
    for (int r = 0; r < R; r++) part[r] = 0.0f;

    for (int64_t s0 = warp; s0 < nslice; s0 += nw) {
        const int64_t gidx = s0 * 32 + lane;
        const int64_t sb = gidx >> 2;
        const int qq = (int)(gidx & 3), h = qq >> 1, u = qq & 1;
        if (sb < nsb) {
            uint32_t xp[3][4][4];  // [plane][run s][word]
            float sx[4], xs16[4];
#pragma unroll
            for (int s = 0; s < 4; s++) {
                const int64_t pos = sb * 256 + 128 * h + 32 * s + 16 * u;
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    const uint4 v = *reinterpret_cast<const uint4*>(planes + p * in + pos);
                    xp[p][s][0] = v.x; xp[p][s][1] = v.y; xp[p][s][2] = v.z; xp[p][s][3] = v.w;
                }
                const float4 st = stats[sb * 8 + 4 * h + s];
                sx[s] = st.x;
                xs16[s] = u ? st.z : st.y;
            }
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int64_t row = row0 + r;
                if (row < out) {
                    const int64_t bi = row * nsb + sb;
                    const uint8_t* base = qs + bi * 96;
                    const uint4 hm = ldg_stream(base + 16 * u);
                    const uint4 qv = ldg_stream(base + 32 + 32 * h + 16 * u);
                    const uint4 hd = ldg_stream(hdr + bi * 16);
                    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
                    const uint32_t hw[4] = {hm.x, hm.y, hm.z, hm.w};
                    const float d = __half2float(__ushort_as_half((unsigned short)(hd.w & 0xFFFFu)));
                    const uint32_t lo8[2] = {hd.x, hd.y};
                    float acc = 0.0f;
#pragma unroll
                    for (int s = 0; s < 4; s++) {
                        int a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const uint32_t hq = (hw[c] >> (4 * h)) & 0x0F0F0F0Fu;
                            const uint32_t ql = (qw[c] >> (2 * s)) & 0x03030303u;
                            const uint32_t hb = (s <= 2 ? (hq << (2 - s)) : (hq >> 1)) & 0x04040404u;
                            const uint32_t q = ql | hb;  // q + 4 in 0..7
                            a1 = dp4a_us(q, xp[0][s][c], a1);
                            a2 = dp4a_us(q, xp[1][s][c], a2);
                            a3 = dp4a_us(q, xp[2][s][c], a3);
                        }
                        // 6-bit scale of sub-block 8h + 2s + u
                        const int k = u + 2 * s;  // 0..7
                        const int lo4 = (int)((lo8[k >> 2] >> (8 * (k & 3) + 4 * h)) & 15u);
                        const int kb = u + 2 * (s & 1);  // byte 8 + kb
                        const int hi2 = (int)((hd.z >> (8 * kb + 2 * (2 * h + (s >> 1)))) & 3u);
                        const float scale = (float)((lo4 | (hi2 << 4)) - 32);
                        acc = fmaf(scale, fmaf(fix24(a1, a2, a3), sx[s], -4.0f * xs16[s]), acc);
                    }
                    part[r] = fmaf(d, acc, part[r]);
                }
            }
        }
    }
    transpose_reduce<R>(part, lane);
    if (lane_writes<R>(lane)) red[warp][row_of_lane<R>(lane)] = part[0];
    __syncthreads();
    if (threadIdx.x < R) {
        float acc = 0.0f;
        for (int w = 0; w < nw; w++) acc += red[w][threadIdx.x];
        const int64_t row = row0 + threadIdx.x;
        if (row < out) y[row] = acc;
    }
}

// ================================================================== Q4_0
// Lane owns two consecutive 32-element blocks (one 64-element group).

template <int R>
__global__ void __launch_bounds__(256, 2)
mv_q40_kernel(const uint8_t* __restrict__ qs, const uint8_t* __restrict__ hdr,
              const int8_t* __restrict__ planes, const float4* __restrict__ stats,
              float* __restrict__ y, int64_t out, int64_t nblk, int64_t in) {
    __shared__ float red[8][R];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int64_t row0 = (int64_t)blockIdx.x * R;
    const int64_t ngroups = (nblk + 1) / 2;
    const int64_t nslice = (ngroups + 31) / 32;
    float part[R];
#pragma unroll
    for (int r = 0; r < R; r++) part[r] = 0.0f;

    for (int64_t s = warp; s < nslice; s += nw) {
        const int64_t gidx = s * 32 + lane;
        const int64_t b0 = 2 * gidx;
        if (b0 < nblk) {
            const bool has1 = b0 + 1 < nblk;
            GroupX gx;
            if (has1) {
                load_group_x(gx, planes, in, b0 * 32);
            } else {  // ragged tail: one block only
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    const uint4* src = reinterpret_cast<const uint4*>(planes + p * in + b0 * 32);
#pragma unroll
                    for (int k = 0; k < 2; k++) {
                        uint4 v = src[k];
                        gx.p[p][4 * k] = v.x; gx.p[p][4 * k + 1] = v.y;
                        gx.p[p][4 * k + 2] = v.z; gx.p[p][4 * k + 3] = v.w;
                    }
#pragma unroll
                    for (int k = 8; k < 16; k++) gx.p[p][k] = 0u;
                }
            }
            const float4 st0 = stats[b0];
            const float4 st1 = has1 ? stats[b0 + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
            const float sx0 = st0.x * 0.0625f, sx1 = st1.x * 0.0625f;
            const float xs0 = 8.0f * (st0.y + st0.z), xs1 = 8.0f * (st1.y + st1.z);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int64_t row = row0 + r;
                if (row < out) {
                    const int64_t bi = row * nblk + b0;
                    const uint4 qa = ldg_stream(qs + bi * 16);
                    const uint4 qb = has1 ? ldg_stream(qs + bi * 16 + 16) : make_uint4(0u, 0u, 0u, 0u);
                    const uint16_t d0b = *reinterpret_cast<const uint16_t*>(hdr + bi * 2);
                    const uint16_t d1b = has1 ? *reinterpret_cast<const uint16_t*>(hdr + bi * 2 + 2) : (uint16_t)0;
                    const uint32_t wv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    int a[2][3];
#pragma unroll
                    for (int blk = 0; blk < 2; blk++) {
                        int e1 = 0, e2 = 0, e3 = 0, f1 = 0, f2 = 0, f3 = 0;
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const uint32_t w = wv[4 * blk + k];
                            const uint32_t lo = w & 0x0F0F0F0Fu, hi = w & 0xF0F0F0F0u;
                            e1 = dp4a_us(lo, gx.p[0][8 * blk + k], e1);
                            e2 = dp4a_us(lo, gx.p[1][8 * blk + k], e2);
                            e3 = dp4a_us(lo, gx.p[2][8 * blk + k], e3);
                            f1 = dp4a_us(hi, gx.p[0][8 * blk + 4 + k], f1);
                            f2 = dp4a_us(hi, gx.p[1][8 * blk + 4 + k], f2);
                            f3 = dp4a_us(hi, gx.p[2][8 * blk + 4 + k], f3);
                        }
                        a[blk][0] = 16 * e1 + f1;  // 16 * sum(q * x_plane)
                        a[blk][1] = 16 * e2 + f2;
                        a[blk][2] = 16 * e3 + f3;
                    }
                    const float d0 = __half2float(__ushort_as_half(d0b));
                    const float d1 = __half2float(__ushort_as_half(d1b));
                    const float v0 = fmaf(fix24(a[0][0], a[0][1], a[0][2]), sx0, -xs0);
                    const float v1 = fmaf(fix24(a[1][0], a[1][1], a[1][2]), sx1, -xs1);
                    part[r] += fmaf(d0, v0, d1 * v1);
                }
            }
        }
    }
    transpose_reduce<R>(part, lane);
    if (lane_writes<R>(lane)) red[warp][row_of_lane<R>(lane)] = part[0];
    __syncthreads();
    if (threadIdx.x < R) {
        float acc = 0.0f;
        for (int w = 0; w < nw; w++) acc += red[w][threadIdx.x];
        const int64_t row = row0 + threadIdx.x;
        if (row < out) y[row] = acc;
    }
}

template <int R>
int launch_mv_r(const rq_weight* w, XQ xq, float* y, int nw, cudaStream_t st) {
    const int64_t grid = (w->out + R - 1) / R;
    const dim3 g((unsigned)grid), b((unsigned)(nw * 32));
    if (w->type == RQ_Q4_K)
        mv_q4k_kernel<R><<<g, b, 0, st>>>(w->qs, w->hdr, xq.planes, xq.stats, y, w->out, w->nblk, w->in);
    else if (w->type == RQ_Q3_K)
        mv_q3k_kernel<R><<<g, b, 0, st>>>(w->qs, w->hdr, xq.planes, xq.stats, y, w->out, w->nblk, w->in);
    else
        mv_q40_kernel<R><<<g, b, 0, st>>>(w->qs, w->hdr, xq.planes, xq.stats, y, w->out, w->nblk, w->in);
    return cuda_error(cudaGetLastError(), "matvec kernel");
}

}  // namespace

int launch_xquant(const float* x, int64_t M, int64_t in, XQ xq, cudaStream_t st) {
    int64_t n = M * (in / 32);
    if (n == 0) return RQ_OK;
    xquant_kernel<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(x, M, in, xq.planes, xq.stats);
    return cuda_error(cudaGetLastError(), "xquant kernel");
}

// M=1 matvec for one activation row: xq must hold that row.
int launch_matvec(const rq_weight* w, XQ xq, float* y, int sm_count, cudaStream_t st) {
    // K slices of 2048 elements; warps per CTA = slices / ceil(slices/8)
    const int64_t elems_per_slice = 2048;
    const int64_t nslice = (w->in + elems_per_slice - 1) / elems_per_slice;
    const int64_t rounds = (nslice + 7) / 8;
    const int nw = (int)((nslice + rounds - 1) / rounds);
    const int64_t want = 2 * (int64_t)sm_count;
    if (w->out / 16 >= want) return launch_mv_r<16>(w, xq, y, nw, st);
    if (w->out / 8 >= want) return launch_mv_r<8>(w, xq, y, nw, st);
    return launch_mv_r<4>(w, xq, y, nw, st);
}

int launch_linear(const rq_weight* w, XQ xq, float* y, int64_t M, int sm_count,
                  cudaStream_t st) {
    for (int64_t m = 0; m < M; m++) {
        XQ row{xq.planes + m * 3 * w->in, xq.stats + m * (w->in / 32)};
        int rc = launch_matvec(w, row, y + m * w->out, sm_count, st);
        if (rc) return rc;
    }
    return RQ_OK;
}

}  // namespace rq
