// rq_mm_skinny.cu -- Q4_K matmul for 9..16 activation rows (speculative
// verify batches, short prompt chunks) on the 5th-gen tensor cores, in one
// pass over the weights.
//
// The kernel is built around the cost per weight, not per MMA, and around
// one measured limit: the single warp that issues the MMAs pays ~30-130
// cycles for every tcgen05 instruction (MMA or commit) and every mbarrier
// wait, whatever the operand source (TMEM or shared memory), the spacing of
// dependent MMAs or the number of issuing warps, so a 128-row super-block
// (17 MMAs of 2048 weights) costs ~2100 cycles, ~1.7 TB/s of Q4_K at any M.
// The kernel therefore waits and commits once per half super-block.  Below
// 9 rows the mma.sync kernel, whose 8-row tiles cost the same, is faster;
// from 9 to 16 rows this one is (one pass instead of two).
//   * The 4-bit quants enter the MMA as they are: a nibble's bit pattern
//     in a 16-bit lane is the f16 subnormal q * 2^-24, a high nibble masked
//     in place is 16 q * 2^-24; one shift and four masks turn a word of 8
//     weights into four f16x2 operand words (no multiply, no conversion).
//   * Each of the 8 sub-blocks of a super-block accumulates into its own
//     TMEM accumulator (K = 32: two MMAs), so the MMAs never wait on one
//     another, and the sub-block scales sc_j (6-bit) are
//     applied in the epilogue: y += d * sum_j sc_j P1_j - dmin * P2 with
//     P2 = [m_0..7, m_0..7] . [bsum_hi ; bsum_lo] (one K = 16 MMA) exactly
//     as in rq_mm_tc.cu.  Every operand is exact; the activations arrive as
//     x / s = hi + lo in f16 (stacked along N: the MMA's N is 32 for the
//     16 token columns).
//   * Persistent CTAs take equal ranges of (128-row tile, super-block)
//     units over all jobs, so 1024-row and 28672-row weights alike fill the
//     148 SMs.  A tile cut between CTAs is finished by the last CTA to
//     arrive (an atomic count per tile), which sums the pieces from a
//     workspace in CTA order: the result does not depend on timing.
//
// Warp roles (18 warps, one CTA per SM):
//   0      TMA producer: ring R (one super-block of 128 rows: quant bytes,
//          headers, the block-sum operand B2), ring C (two 64-element chunks
//          of x_hi / x_lo: B1, half a super-block).
//   1      TMEM allocation, all MMAs (one elected lane), commits.
//   2..9   expand: warp w writes TMEM lanes 32 (w % 4) .. +31 (rows); the
//          two warps of a lane quarter take the two 64-element chunks of a
//          half super-block (both nibbles: 32 of the half's 64 A-slot
//          columns each); the first also writes A2 (the m values).
//   10..17 epilogue: two warps per lane quarter, each reads 2 of the 4
//          sub-block accumulators of each half and releases the half as soon
//          as it has read it; running totals stay in registers and the two
//          warps' totals are added once per tile piece.
// TMEM columns: [8 chains x 32 | P2 16] (two halves of 4 chains), then na A
// slots of 64 (128 f16 of K per row).  Every mbarrier wait is bounded; on expiry
// the CTA records the error and skips work, and TMEM is always released.

#include <string.h>

#include <algorithm>

#include "rq_async.cuh"
#include "rq_mv_common.cuh"
#include "rq_tcgen05.cuh"

namespace rq {
namespace {

using namespace tc;

constexpr int kWarpsSK = 18;
constexpr int kThreadsSK = 32 * kWarpsSK;
constexpr int kExpWarp0 = 2, kEpiWarp0 = 10;
constexpr int kChains = 8;  // one accumulator per sub-block
constexpr int kMaxR = 8, kMaxC = 8, kMaxA = 6;
constexpr int kSmemSK = 227 * 1024;
constexpr float kSub = 16777216.0f;  // 2^24: f16 subnormal n * 2^-24 -> n
constexpr int kNT = 16;              // token columns per tile (x_hi and x_lo: MMA N = 32)

struct SKJob {
    float* y;
    const float* add;
    const uint8_t* hdr;  // [out][nblk][16]
    int64_t out;
    int tok0, M;
    int t0;  // first tile of the job in the global tile order
};

struct alignas(64) SKParams {
    CUtensorMap wq[kMaxJobs];  // quant bytes [out][nblk*128], box 128 x 128, 128-byte swizzle
    CUtensorMap wh[kMaxJobs];  // headers [out][nblk*16], box 16 x 128
    CUtensorMap xhi, xlo;      // staged x planes [rows][in] f16, box 64 x nt, 128-byte swizzle
    CUtensorMap bs;            // block sums [rows][nblk*16] f16, box 16 x 16, 32-byte swizzle
    SKJob jobs[kMaxJobs];
    const float* xscale;
    int* err;
    float* ws;  // tile pieces: slot (tile + cta) of [nt][128] floats
    int* cnt;   // arrivals per tile (reset by the last arrival)
    long long units;
    int njobs, nblk, nb, na, nr, nc;
    uint32_t buf_cols, acol0, tmem_cols;
    uint32_t r_bytes, r_hdr, r_b2, r_a2, c_bytes, ring_off, c_off;
};

// A CTA's share: units [U b / G, U (b+1) / G) of the (tile, super-block)
// order, walked as segments of consecutive super-blocks of one tile.
struct Seg {
    int t, sb0, sb1;
};
struct Segs {
    long long u, u1;
    __device__ __forceinline__ void start(const SKParams& p) {
        u = p.units * (long long)blockIdx.x / gridDim.x;
        u1 = p.units * (long long)(blockIdx.x + 1) / gridDim.x;
    }
    __device__ __forceinline__ bool next(const SKParams& p, Seg& s) {
        if (u >= u1) return false;
        s.t = (int)(u / p.nblk);
        s.sb0 = (int)(u - (long long)s.t * p.nblk);
        const long long e = min(u1, (long long)(s.t + 1) * p.nblk);
        s.sb1 = s.sb0 + (int)(e - u);
        u = e;
        return true;
    }
};

__device__ __forceinline__ int job_of(const SKParams& p, int t) {
    int j = 0;
    while (j + 1 < p.njobs && t >= p.jobs[j + 1].t0) j++;
    return j;
}

// the CTA whose share holds unit x
__device__ __forceinline__ long long cta_of(const SKParams& p, long long x) {
    return ((x + 1) * (long long)gridDim.x + p.units - 1) / p.units - 1;
}

__global__ void __launch_bounds__(kThreadsSK, 1) mm_skinny_kernel(const __grid_constant__ SKParams p) {
    constexpr int NT = kNT;
    constexpr uint32_t N1 = 2 * NT;   // P1 columns per chain: x_hi tokens, then x_lo tokens
    constexpr uint32_t kEpiPerSB = 8;  // epilogue warps that read one super-block
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    uint8_t* smem = smem_raw + pad;
    const uint32_t sbase = raw + pad;
    // first 1 KB: rfull, rempty [kMaxR]; cfull, cempty [kMaxC]; aready,
    // aempty [kMaxA]; accfull, accempty [2]; the TMEM address; a flag
    const uint32_t rfull0 = sbase, rempty0 = rfull0 + 8 * kMaxR;
    const uint32_t cfull0 = rempty0 + 8 * kMaxR, cempty0 = cfull0 + 8 * kMaxC;
    const uint32_t aready0 = cempty0 + 8 * kMaxC, aempty0 = aready0 + 8 * kMaxA;
    const uint32_t accfull0 = aempty0 + 8 * kMaxA, accempty0 = accfull0 + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (accempty0 + 16 - sbase));
    volatile int* last_flag = reinterpret_cast<volatile int*>(smem + (accempty0 + 20 - sbase));
    float* ered = reinterpret_cast<float*>(smem + 1024);  // [128 rows][NT]: the high half's totals
    const uint32_t ringr = sbase + p.ring_off, ringc = ringr + p.c_off;
    const uint8_t* ringr_p = smem + p.ring_off;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nblk = p.nblk;

    if (threadIdx.x == 0) {
        // an R stage is free once the MMAs have read it (one commit) and
        // the epilogue warps of its super-block have read the header
        for (int i = 0; i < p.nr; i++) {
            mbar_init(rfull0 + 8 * i, 1);
            mbar_init(rempty0 + 8 * i, 1 + kEpiPerSB);
        }
        for (int i = 0; i < p.nc; i++) {
            mbar_init(cfull0 + 8 * i, 1);
            mbar_init(cempty0 + 8 * i, 1);
        }
        for (int i = 0; i < p.na; i++) {
            mbar_init(aready0 + 8 * i, 8);
            mbar_init(aempty0 + 8 * i, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(accfull0 + 8 * b, 1);
            mbar_init(accempty0 + 8 * b, kEpiPerSB);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the staged activations are written by the preceding kernel in the stream
    asm volatile("griddepcontrol.wait;" ::: "memory");

    Segs sg;
    sg.start(p);
    Seg s;
    if (warp == 0) {
        // -------------------------------------------------------------- TMA
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first(), pol_h = policy_evict_normal();
            const uint64_t pol_x = policy_evict_last();
            const uint32_t rtx = kRowsTC * 128 + kRowsTC * 16 + 16 * 32;
            const uint32_t ctx = 4u * 128u * NT;  // two chunks of x_hi and x_lo
            Ring rr, cr;
            int ri = 0, ci = 0;
            bool ok = true;
            while (ok && sg.next(p, s)) {
                const int j = job_of(p, s.t);
                const int row0 = (s.t - p.jobs[j].t0) * kRowsTC, tok = p.jobs[j].tok0;
                for (int sb = s.sb0; sb < s.sb1 && ok; sb++, ri++, rr.next(p.nr)) {
                    if (rr.u > 0 && !wait_err(rempty0 + 8 * rr.i, (rr.u - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = ringr + (uint32_t)rr.i * p.r_bytes;
                    const uint32_t fb = rfull0 + 8 * rr.i;
                    mbar_expect_tx(fb, rtx);
                    tma_load_2d(st, &p.wq[j], sb * 128, row0, fb, pol_w);
                    tma_load_2d(st + p.r_hdr, &p.wh[j], sb * 16, row0, fb, pol_h);
                    tma_load_2d(st + p.r_b2, &p.bs, sb * 16, tok, fb, pol_x);
                    for (int h = 0; h < 2; h++, ci++, cr.next(p.nc)) {
                        if (cr.u > 0 && !wait_err(cempty0 + 8 * cr.i, (cr.u - 1) & 1, p.err)) {
                            ok = false;
                            break;
                        }
                        const uint32_t sc = ringc + (uint32_t)cr.i * p.c_bytes;
                        const uint32_t cb = cfull0 + 8 * cr.i;
                        mbar_expect_tx(cb, ctx);
#pragma unroll
                        for (int c = 0; c < 2; c++) {
                            const int x = (4 * sb + 2 * h + c) * 64;
                            tma_load_2d(sc + 256u * NT * c, &p.xhi, x, tok, cb, pol_x);
                            tma_load_2d(sc + 256u * NT * c + 128u * NT, &p.xlo, x, tok, cb, pol_x);
                        }
                    }
                }
            }
            // no copy may still be in flight when the CTA exits
            for (int k = max(0, ri - p.nr); k < ri; k++)
                if (!mbar_wait(rfull0 + 8 * (k % p.nr), (k / p.nr) & 1)) ok = false;
            for (int k = max(0, ci - p.nc); k < ci; k++)
                if (!mbar_wait(cfull0 + 8 * (k % p.nc), (k / p.nc) & 1)) ok = false;
            if (!ok && p.err) atomicExch(p.err, 1);
        }
    } else if (warp == 1) {
        // -------------------------------------------------------------- MMA
        // Per half super-block h (chunks 2h, 2h+1, sub-blocks 4h .. 4h+3):
        // wait for its accumulator half, activation stage and A slot, issue
        // the first K step of the four sub-blocks, then the second, and
        // commit each ring once.  Every tcgen05 instruction costs tens of
        // cycles to issue, so the kernel issues as few as it can.
        const uint32_t idesc1 = umma_idesc(N1), idesc2 = umma_idesc(16);
        Ring rr, cr, ar;
        int ksb = 0;  // super-blocks done: the parity of the accumulator halves
        bool ok = true;
        while (sg.next(p, s)) {
            for (int sb = s.sb0; sb < s.sb1; sb++, rr.next(p.nr), ksb++) {
                for (int h = 0; h < 2; h++, cr.next(p.nc), ar.next(p.na)) {
                    // half h of the accumulators is free once the epilogue has read it
                    if (ok && ksb > 0 && !wait_err(accempty0 + 8 * h, (ksb - 1) & 1, p.err)) ok = false;
                    if (ok && !wait_err(cfull0 + 8 * cr.i, cr.u & 1, p.err)) ok = false;
                    if (ok && !wait_err(aready0 + 8 * ar.i, ar.u & 1, p.err)) ok = false;
                    ok = __all_sync(0xffffffffu, ok);
                    tmem_fence_after();
                    const uint32_t sc = ringc + (uint32_t)cr.i * p.c_bytes;
                    const uint32_t acol = tmem + p.acol0 + 64u * (uint32_t)ar.i;
                    if (elect_one()) {
                        if (ok) {
#pragma unroll
                            for (int k2 = 0; k2 < 2; k2++)
#pragma unroll
                                for (int i = 0; i < 4; i++) {
                                    // sub-block 4h + i: chunk c = i / 2, nibble half i % 2
                                    const int c = i >> 1, nh = i & 1, kk = 2 * nh + k2;
                                    const uint32_t d = tmem + (uint32_t)(4 * h + i) * N1;
                                    umma_f16_ts(d, acol + 32u * (uint32_t)c + 8u * kk,
                                                desc_sw128(sc + 256u * NT * (uint32_t)c + 32u * kk), idesc1,
                                                (uint32_t)k2);
                                }
                            if (h == 1) {
                                const uint32_t st = ringr + (uint32_t)rr.i * p.r_bytes;
                                umma_f16(tmem + kChains * N1, desc_sw32(st + p.r_a2), desc_sw32(st + p.r_b2), idesc2,
                                         0u);
                            }
                        }
                        umma_commit(cempty0 + 8 * cr.i);
                        umma_commit(aempty0 + 8 * ar.i);
                        if (h == 1) umma_commit(rempty0 + 8 * rr.i);
                        umma_commit(accfull0 + 8 * h);
                    }
                    __syncwarp();
                }
            }
        }
        if (!ok && lane == 0 && p.err) atomicExch(p.err, 1);
    } else if (warp < kEpiWarp0) {
        // ----------------------------------------------------------- expand
        // Warp w writes TMEM lanes 32 (w % 4) .. +31 (rows r); the two warps
        // of a lane quarter take alternate chunks (par 0: chunks 0, 2 of every
        // super-block, par 1: chunks 1, 3), both nibbles of each (32
        // columns), and store both chunks before waiting for the stores.
        const int q = warp & 3, par = (warp - kExpWarp0) >> 2;  // par: chunk 2h + par of half h
        const int r = 32 * q + lane;
        const uint32_t swz = (uint32_t)(r & 7);
        const uint32_t lane_a = tmem + ((uint32_t)(32 * q) << 16) + p.acol0;
        Ring rr, ar;  // ar: the A slot of the current half super-block
        bool ok = true;
        while (sg.next(p, s)) {
            for (int sb = s.sb0; sb < s.sb1; sb++, rr.next(p.nr)) {
                if (ok && !wait_err(rfull0 + 8 * rr.i, rr.u & 1, p.err)) ok = false;
                const uint8_t* rst = ringr_p + (size_t)rr.i * p.r_bytes;
                if (ok && par == 0) {
                    // A2 row r: [m_0..7, m_0..7] as f16 subnormals (32-byte
                    // swizzle; both 16-byte halves are equal)
                    const uint4 hd = *reinterpret_cast<const uint4*>(rst + p.r_hdr + r * 16);
                    uint32_t m[4];
#pragma unroll
                    for (int g = 0; g < 4; g++) {
                        const uint32_t w = q4k_scales(q4k_scale_sel(g), hd);
                        m[g] = ((w >> 16) & 0xFFu) | ((w >> 24) << 16);
                    }
                    const uint4 mv = make_uint4(m[0], m[1], m[2], m[3]);
                    uint8_t* a2 = const_cast<uint8_t*>(rst) + p.r_a2 + (r >> 3) * 256 + (r & 7) * 32;
                    *reinterpret_cast<uint4*>(a2) = mv;
                    *reinterpret_cast<uint4*>(a2 + 16) = mv;
                    // generic-proxy writes become visible to the tensor core
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
                for (int h = 0; h < 2; h++, ar.next(p.na)) {
                    if (ok && ar.u > 0 && !wait_err(aempty0 + 8 * ar.i, (ar.u - 1) & 1, p.err)) ok = false;
                    ok = __all_sync(0xffffffffu, ok);  // tcgen05.st is warp-wide
                    tmem_fence_after();
                    if (ok) {
                        // the chunk's 32 quant bytes of row r: 16-byte chunks
                        // 2cq, 2cq+1 of the row's 128-byte-swizzled line
                        const int cq = 2 * h + par;
                        const uint8_t* qrow = rst + r * 128;
                        const uint4 qa = *reinterpret_cast<const uint4*>(qrow + (((2 * cq) ^ swz) << 4));
                        const uint4 qb = *reinterpret_cast<const uint4*>(qrow + (((2 * cq + 1) ^ swz) << 4));
                        const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                        uint32_t o[32];
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            // bytes b0..b3: (b0, b2) and (b1, b3) in 16-bit
                            // lanes, i.e. elements (e0, e2), (e1, e3); low
                            // nibbles are K 0..31 of the chunk, high 32..63
                            const uint32_t v = qw[i] >> 8;
                            o[2 * i] = qw[i] & 0x000F000Fu;
                            o[2 * i + 1] = v & 0x000F000Fu;
                            o[16 + 2 * i] = qw[i] & 0x00F000F0u;
                            o[17 + 2 * i] = v & 0x00F000F0u;
                        }
                        // TMEM column c of the chunk holds K positions 2c, 2c+1
                        tmem_st32u(lane_a + 64u * (uint32_t)ar.i + 32u * (uint32_t)par, o);
                        tmem_wait_st();
                    }
                    tmem_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(aready0 + 8 * ar.i);
                }
            }
        }
        if (!ok && lane == 0 && p.err) atomicExch(p.err, 1);
    } else {
        // ------------------------------------------------------------ epilogue
        // Each warp reads 4 of the 8 chains of every super-block, the low
        // half also P2.  The header comes from the R stage, which the
        // epilogue releases together with the MMA.
        const int q = warp & 3, half = (warp - kEpiWarp0) >> 2;
        const int r = 32 * q + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        Ring rr;
        int ksb = 0;  // super-blocks done: the parity of the accumulator halves
        bool ok = true;
        while (sg.next(p, s)) {
            const int j = job_of(p, s.t);
            const SKJob& jb = p.jobs[j];
            const int64_t row = (int64_t)(s.t - jb.t0) * kRowsTC + r;
            const bool live = row < jb.out;
            float tot[NT];
#pragma unroll
            for (int i = 0; i < NT; i++) tot[i] = 0.0f;
            for (int sb = s.sb0; sb < s.sb1; sb++, rr.next(p.nr), ksb++) {
                // sub-block scales: chain c = sub-block c, its coefficient
                // d 2^24 sc_c (1/16 more for odd c: high nibbles are 16 q);
                // this warp reads chains 2e, 2e + 1 and 4 + 2e, 5 + 2e
                float kc[4], fm = 0.0f;
                for (int h = 0; h < 2; h++) {
                    if (ok && !wait_err(accfull0 + 8 * h, ksb & 1, p.err)) ok = false;
                    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-wide
                    tmem_fence_after();
                    if (h == 0) {
                        const uint4 hd =
                            *reinterpret_cast<const uint4*>(ringr_p + (size_t)rr.i * p.r_bytes + p.r_hdr + r * 16);
                        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hd.x));
                        const float fd = dm.x * kSub;
                        fm = -dm.y * kSub;
#pragma unroll
                        for (int g = 0; g < 2; g++) {
                            const uint32_t w = q4k_scales(q4k_scale_sel(2 * g + half), hd);
                            kc[2 * g] = fd * (float)(w & 0xFFu);
                            kc[2 * g + 1] = fd * 0.0625f * (float)((w >> 8) & 0xFFu);
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(rempty0 + 8 * rr.i);  // the header is read
                    }
                    if (ok) {
                        // one 32-column chain at a time (96 registers per
                        // thread with 18 warps)
#pragma unroll
                        for (int c = 0; c < 2; c++) {
                            uint32_t ua[32];
                            tmem_ld32(lane_base + (uint32_t)(4 * h + 2 * half + c) * N1, ua);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 16; i++)
                                tot[i] = fmaf(kc[2 * h + c], __uint_as_float(ua[i]) + __uint_as_float(ua[16 + i]), tot[i]);
                        }
                        if (h == 1 && half == 0) {
                            uint32_t p2[16];
                            tmem_ld16(lane_base + kChains * N1, p2);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 16; i++) tot[i] = fmaf(fm, __uint_as_float(p2[i]), tot[i]);
                        }
                    }
                    // this half of the accumulators is read: the next MMAs
                    // may overwrite it
                    tmem_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(accempty0 + 8 * h);
                }
            }
            // ---- end of the tile piece: add the halves (low + high), then
            // write y, or the piece and count it
            if (half == 1) {
#pragma unroll
                for (int i = 0; i < NT; i++) ered[r * NT + i] = tot[i];
            }
            named_bar_sync(1, 256);
            if (half == 0) {
#pragma unroll
                for (int i = 0; i < NT; i++) tot[i] += ered[r * NT + i];
                const long long x0 = (long long)s.t * nblk;
                const long long bf = cta_of(p, x0), bl = cta_of(p, x0 + nblk - 1);
                const int P = (int)(bl - bf + 1);
                const float* xs = p.xscale + jb.tok0;
                if (P == 1) {
                    if (ok && live) {
#pragma unroll
                        for (int i = 0; i < NT; i++) {
                            if (i < jb.M) {
                                const int64_t o = (int64_t)i * jb.out + row;
                                const float v = tot[i] * xs[i];
                                jb.y[o] = jb.add ? v + jb.add[o] : v;
                            }
                        }
                    }
                } else {
                    float* wsl = p.ws + ((size_t)s.t + blockIdx.x) * (NT * 128);
#pragma unroll
                    for (int i = 0; i < NT; i++) wsl[i * 128 + r] = tot[i];
                    __threadfence();
                    named_bar_sync(2, 128);
                    if (warp == kEpiWarp0 && lane == 0) {
                        const int old = atomicAdd(p.cnt + s.t, 1);
                        *last_flag = old == P - 1;
                    }
                    named_bar_sync(2, 128);
                    if (*last_flag) {
                        __threadfence();
                        if (ok && live) {
                            for (int i = 0; i < NT && i < jb.M; i++) {
                                float v = 0.0f;
                                for (int pc = 0; pc < P; pc++)
                                    v += __ldcg(p.ws + ((size_t)s.t + bf + pc) * (NT * 128) + i * 128 + r);
                                const int64_t o = (int64_t)i * jb.out + row;
                                v *= xs[i];
                                jb.y[o] = jb.add ? v + jb.add[o] : v;
                            }
                        }
                        if (warp == kEpiWarp0 && lane == 0) p.cnt[s.t] = 0;
                    }
                }
            }
            // the combine buffer and the flag are reused by the next piece
            named_bar_sync(1, 256);
        }
        if (!ok && lane == 0 && p.err) atomicExch(p.err, 1);
    }
    // every MMA has completed (the epilogue waited for the last commit)
    // before the columns are released
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    __syncwarp();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols)
                     : "memory");
}

}  // namespace

int launch_mm_skinny(rq_ctx* ctx, const MMJobDesc* jobs, int njobs, XH xh, int64_t rows, cudaStream_t st, int* err) {
    if (njobs < 1 || njobs > kMaxJobs) return set_error(RQ_ERR_INVALID, "skinny matmul: %d jobs", njobs);
    const int64_t in = jobs[0].w->in, nblk = jobs[0].w->nblk;
    SKParams p;
    memset(&p, 0, sizeof p);
    int tiles = 0;
    for (int j = 0; j < njobs; j++) {
        const rq_weight* w = jobs[j].w;
        if (w->type != RQ_Q4_K || w->in != in)
            return set_error(RQ_ERR_INVALID, "skinny matmul: jobs need Q4_K weights with the same K");
        if (jobs[j].M < 1 || jobs[j].M > kSkinnyMaxM || jobs[j].tok0 < 0 || jobs[j].tok0 + jobs[j].M > rows)
            return set_error(RQ_ERR_INVALID, "skinny matmul: token rows [%d, %d) of %lld (at most %d per job)",
                             jobs[j].tok0, jobs[j].tok0 + jobs[j].M, (long long)rows, kSkinnyMaxM);
        int rc = encode(&p.wq[j], CU_TENSOR_MAP_DATA_TYPE_UINT8, w->qs, (uint64_t)(nblk * 128), (uint64_t)w->out,
                        (uint64_t)(nblk * 128), 128, kRowsTC, CU_TENSOR_MAP_SWIZZLE_128B, "quant bytes");
        if (!rc)
            rc = encode(&p.wh[j], CU_TENSOR_MAP_DATA_TYPE_UINT8, w->hdr, (uint64_t)(nblk * 16), (uint64_t)w->out,
                        (uint64_t)(nblk * 16), 16, kRowsTC, CU_TENSOR_MAP_SWIZZLE_NONE, "headers");
        if (rc) return rc;
        SKJob& t = p.jobs[j];
        t.y = jobs[j].y;
        t.add = jobs[j].add;
        t.hdr = w->hdr;
        t.out = w->out;
        t.tok0 = jobs[j].tok0;
        t.M = jobs[j].M;
        t.t0 = tiles;
        tiles += (int)((w->out + kRowsTC - 1) / kRowsTC);
    }
    const int nt = kNT;
    int rc = encode(&p.xhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh.v, (uint64_t)in, (uint64_t)rows, (uint64_t)(4 * in),
                    64, (uint32_t)nt, CU_TENSOR_MAP_SWIZZLE_128B, "activations (hi)");
    if (!rc)
        rc = encode(&p.xlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh.v + in, (uint64_t)in, (uint64_t)rows,
                    (uint64_t)(4 * in), 64, (uint32_t)nt, CU_TENSOR_MAP_SWIZZLE_128B, "activations (lo)");
    if (!rc)
        rc = encode(&p.bs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh.bs16, (uint64_t)(nblk * 16), (uint64_t)rows,
                    (uint64_t)(nblk * 32), 16, 16, CU_TENSOR_MAP_SWIZZLE_32B, "block sums");
    if (rc) return rc;
    p.units = (long long)tiles * nblk;
    const int grid = (int)std::min<long long>(ctx->sm_count, p.units);
    // split-K scratch: slot (tile + cta) of [nt][128] floats, a count per tile
    rc = ensure_skinny_scratch(ctx, (size_t)(tiles + grid) * nt * kRowsTC, tiles);
    if (rc) return rc;
    p.ws = ctx->sk_ws;
    p.cnt = ctx->sk_cnt;
    p.xscale = xh.scale;
    p.err = err;
    p.njobs = njobs;
    p.nblk = (int)nblk;
    // TMEM: [8 chains x 2 nt | P2 16] and na A slots of 64 (one per half
    // super-block)
    p.buf_cols = (uint32_t)(kChains * 2 * nt + 16);
    p.nb = 1;
    p.acol0 = (uint32_t)p.nb * p.buf_cols;
    p.na = std::min(kMaxA, (int)((512 - p.acol0) / 64));
    p.tmem_cols = 512;
    // R stage: quant 16 KB | headers 2 KB | B2 16 x 32 B | A2 4 KB; C stage
    // (half a super-block): two chunks of x_hi, x_lo nt x 128 B each; every
    // tile 1024-aligned
    auto al = [](uint32_t v) { return (v + 1023u) & ~1023u; };
    p.r_hdr = kRowsTC * 128;
    p.r_b2 = al(p.r_hdr + kRowsTC * 16);
    p.r_a2 = al(p.r_b2 + 16 * 32);
    p.r_bytes = al(p.r_a2 + kRowsTC * 32);
    p.c_bytes = al(4 * 128u * (uint32_t)nt);
    p.ring_off = 1024 + al(kRowsTC * 4u * (uint32_t)nt);
    p.nc = 4;
    const int avail = kSmemSK - 1024 - (int)p.ring_off - p.nc * (int)p.c_bytes;
    p.nr = std::min(kMaxR, avail / (int)p.r_bytes);
    if (p.nr < 2) return set_error(RQ_ERR_UNSUPPORTED, "skinny matmul: stages too large");
    p.c_off = (uint32_t)p.nr * p.r_bytes;
    const size_t smem = 1024 + (size_t)p.ring_off + p.c_off + (size_t)p.nc * p.c_bytes;

    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(mm_skinny_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemSK);
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(skinny matmul)");
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreadsSK);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_error(cudaLaunchKernelEx(&cfg, mm_skinny_kernel, p), "skinny matmul kernel");
}

}  // namespace rq
