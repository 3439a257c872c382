// rq_pipe_lane.cuh -- the consumer-lane side of the bulk-copy pipelines
// (M=1 matvec, decode step): which bytes of a staged weight row a lane
// reads, and its activation registers for K-slice s (2048 elements).
#pragma once

#include "rq_mv_common.cuh"

namespace rq {

template <int TYPE>
struct LaneOf;
template <>
struct LaneOf<RQ_Q4_K> { using T = Q4KPLane; };
template <>
struct LaneOf<RQ_Q3_K> { using T = Q3KLane; };
template <>
struct LaneOf<RQ_Q4_0> { using T = Q40Lane; };
template <>
struct LaneOf<RQ_Q8_0> { using T = Q80Lane; };
template <>
struct LaneOf<RQ_Q6_K> { using T = Q6KLane; };
template <>
struct LaneOf<RQ_Q5_K> { using T = Q5KLane; };
template <>
struct LaneOf<RQ_Q2_K> { using T = Q2KLane; };

// Per-lane constants of K-slice s: activation planes and the lane's
// shared-memory byte offsets inside a row.  Lanes past the end of a partial
// slice get zero activations and read the slice's first block, so the row
// loop needs no per-lane branch.
struct LaneOffsets {
    uint32_t qa, qb, h;
    uint32_t q3;  // Q6_K / Q5_K: offset of the lane's (first) qh bytes
    uint32_t hd;  // Q6_K / Q2_K: offset of the super-block's d
    int gs;       // Q6_K / Q2_K: g & 1
};

template <int TYPE>
__device__ __forceinline__ void lane_setup(typename LaneOf<TYPE>::T& L, LaneOffsets& o, int64_t nblk, int64_t in,
                                           const XQ& xq, int s, int lane) {
    if constexpr (TYPE == RQ_Q8_0) {
        // blocks b0, b0+1 of slice s (64 blocks of 32 per slice)
        const int64_t b0 = (int64_t)s * 64 + 2 * lane;
        const bool valid = b0 < nblk;
        const uint32_t l = valid ? (uint32_t)lane : 0u;
        const bool swp = (l >> 1) & 1u;
        q80_lane_setup(L, xq.planes, xq.stats, in, nblk, valid ? b0 : (int64_t)s * 64, valid, swp);
        o.qa = (uint32_t)(s * 2048) + 64u * l + (L.swp ? 32u : 0u);  // the first block's 32 bytes
        o.qb = o.qa ^ 32u;                                             // the second block's
        o.h = (uint32_t)(s * 128) + 4u * l;
    } else if constexpr (TYPE == RQ_Q6_K) {
        // super-block 8s + lane / 4, lane g = lane % 4 (192 quant + 20 header bytes each)
        const int64_t sb = (int64_t)s * 8 + (lane >> 2);
        const bool valid = sb < nblk;
        const uint32_t sbl = valid ? (uint32_t)(lane >> 2) : 0u;
        const int g = lane & 3, n = g >> 1, l0 = 16 * (g & 1);
        q6k_lane_setup(L, xq.planes, xq.stats, in, valid ? sb : (int64_t)s * 8, g, valid);
        const uint32_t base = (uint32_t)(s * 8 * 192) + 192u * sbl;
        o.qa = base + 64u * (uint32_t)n + (uint32_t)l0;
        o.qb = o.qa + 32u;
        o.q3 = base + 128u + 32u * (uint32_t)n + (uint32_t)l0;
        o.h = (uint32_t)(s * 8 * 20) + 20u * sbl + 8u * (uint32_t)n;
        o.hd = (uint32_t)(s * 8 * 20) + 20u * sbl + 16u;
        o.gs = g & 1;
    } else if constexpr (TYPE == RQ_Q2_K) {
        // super-block 8s + lane / 4, lane g = lane % 4 (64 quant + 20 header bytes each)
        const int64_t sb = (int64_t)s * 8 + (lane >> 2);
        const bool valid = sb < nblk;
        const uint32_t sbl = valid ? (uint32_t)(lane >> 2) : 0u;
        const int g = lane & 3, n = g >> 1, l0 = 16 * (g & 1);
        q6k_lane_setup(L, xq.planes, xq.stats, in, valid ? sb : (int64_t)s * 8, g, valid, 1.0f);
        o.qa = (uint32_t)(s * 8 * 64) + 64u * sbl + 32u * (uint32_t)n + (uint32_t)l0;
        o.qb = o.qa;
        o.h = (uint32_t)(s * 8 * 20) + 20u * sbl + 8u * (uint32_t)n;
        o.hd = (uint32_t)(s * 8 * 20) + 20u * sbl + 16u;
        o.gs = g & 1;
    } else if constexpr (TYPE == RQ_Q5_K) {
        // super-block 8s + lane / 4, group g = lane % 4, half order h1 = bit 2
        // of the lane (160 quant bytes: qh[32] then qs[128]; 16 header bytes)
        const int64_t sb = (int64_t)s * 8 + (lane >> 2);
        const bool valid = sb < nblk;
        const uint32_t sbl = valid ? (uint32_t)(lane >> 2) : 0u;
        const int g = lane & 3, h1 = (lane >> 2) & 1;
        q5k_lane_setup(L, xq.planes, xq.stats, in, valid ? sb : 0, g, h1, valid);
        const uint32_t base = (uint32_t)(s * 8 * 160) + 160u * sbl;
        o.qa = base + 32u + 32u * (uint32_t)g + 16u * (uint32_t)h1;
        o.qb = o.qa ^ 16u;
        o.q3 = base + 16u * (uint32_t)h1;
        o.h = (uint32_t)(s * 128) + 16u * sbl;
    } else if constexpr (TYPE == RQ_Q4_0) {
        const int64_t b0 = (int64_t)s * 64 + 2 * lane;
        const bool valid = b0 < nblk;
        if (valid) {
            q40_lane_setup(L, xq.planes, xq.stats, in, nblk, b0);
        } else {
#pragma unroll
            for (int q = 0; q < 3; q++)
#pragma unroll
                for (int w = 0; w < 16; w++) L.p[q][w] = 0u;
            L.sx0 = L.sx1 = L.xs0 = L.xs1 = 0.0f;
            L.has1 = false;
        }
        const uint32_t l = valid ? (uint32_t)lane : 0u;
        o.qa = (uint32_t)(s * 1024) + 32u * l + 16u * ((l >> 2) & 1u);
        o.qb = o.qa ^ 16u;
        o.h = (uint32_t)(s * 128) + 4u * l;
    } else {
        const int64_t sb = (int64_t)s * 8 + (lane >> 2);
        const bool valid = sb < nblk;
        const uint32_t sbl = valid ? (uint32_t)(lane >> 2) : 0u;
        if constexpr (TYPE == RQ_Q4_K) {
            q4kp_lane_setup(L, xq.planes, xq.stats, in, valid ? sb : 0, lane & 3, (lane >> 2) & 1, valid);
            o.qa = (uint32_t)(s * 1024) + 128u * sbl + 32u * (uint32_t)(lane & 3) + 16u * ((lane >> 2) & 1u);
            o.qb = o.qa ^ 16u;
        } else {
            // Q3_K, expanded: Q4_K's nibble offsets, 20-byte headers
            q3k_lane_setup(L, xq.planes, xq.stats, in, valid ? sb : 0, lane & 3, (lane >> 2) & 1, valid);
            o.qa = (uint32_t)(s * 1024) + 128u * sbl + 32u * (uint32_t)(lane & 3) + 16u * ((lane >> 2) & 1u);
            o.qb = o.qa ^ 16u;
            o.h = (uint32_t)(s * 8 * 20) + 20u * sbl + 4u * (uint32_t)(lane & 3);
            o.hd = (uint32_t)(s * 8 * 20) + 20u * sbl + 16u;
            return;
        }
        o.h = (uint32_t)(s * 128) + 16u * sbl;
    }
}

// Lane contribution of one row held in shared memory (q: the row's quant
// bytes, h: its header bytes).
template <int TYPE>
__device__ __forceinline__ float lane_row(const typename LaneOf<TYPE>::T& L, const LaneOffsets& o,
                                          const uint8_t* q, const uint8_t* h) {
    if constexpr (TYPE == RQ_Q2_K) {
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(h + o.h);
        return q2k_lane_row(L, *reinterpret_cast<const uint4*>(q + o.qa), hw[0], hw[1],
                            *reinterpret_cast<const uint32_t*>(h + o.hd), o.gs);
    }
    const uint4 a = *reinterpret_cast<const uint4*>(q + o.qa);
    const uint4 b = *reinterpret_cast<const uint4*>(q + o.qb);
    if constexpr (TYPE == RQ_Q2_K) {
        return 0.0f;  // handled above
    } else if constexpr (TYPE == RQ_Q5_K) {
        const uint4 ha = *reinterpret_cast<const uint4*>(q + o.q3);
        const uint4 hb = *reinterpret_cast<const uint4*>(q + (o.q3 ^ 16u));
        return q5k_lane_row(L, a, b, ha, hb, *reinterpret_cast<const uint4*>(h + o.h));
    } else if constexpr (TYPE == RQ_Q8_0) {
        const uint4 a1 = *reinterpret_cast<const uint4*>(q + o.qa + 16);
        const uint4 b1 = *reinterpret_cast<const uint4*>(q + o.qb + 16);
        return q80_lane_row(L, a, a1, b, b1, *reinterpret_cast<const uint32_t*>(h + o.h));
    } else if constexpr (TYPE == RQ_Q6_K) {
        const uint4 hh = *reinterpret_cast<const uint4*>(q + o.q3);
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(h + o.h);
        const uint32_t dw = *reinterpret_cast<const uint32_t*>(h + o.hd);
        return q6k_lane_row(L, a, b, hh, hw[0], hw[1], dw, o.gs);
    } else if constexpr (TYPE == RQ_Q4_K) {
        return q4kp_lane_row(L, a, b, *reinterpret_cast<const uint4*>(h + o.h), 0.0f);
    } else if constexpr (TYPE == RQ_Q3_K) {
        return q3k_lane_row(L, a, b, *reinterpret_cast<const uint32_t*>(h + o.h),
                            *reinterpret_cast<const uint32_t*>(h + o.hd));
    } else {
        // a is the half selected by lane bit 2; swap back to blocks (b0, b0+1)
        const bool swap = (o.qa & 16u) != 0u;
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(h + o.h);
        return q40_lane_row(L, swap ? b : a, swap ? a : b, (uint16_t)(dd & 0xFFFFu),
                            L.has1 ? (uint16_t)(dd >> 16) : (uint16_t)0);
    }
}

}  // namespace rq
