// rq_mm_tc.cu -- Q4_K / Q3_K matmul for M >= 16 activation rows on the 5th-gen
// tensor cores: tcgen05.mma (kind::f16, f32 accumulators in TMEM).
//
// y[token][row] = x[token][:] . W[row][:] over K.  A CTA tile is 128 weight
// rows x nt tokens (nt = 16..112); persistent CTAs walk the tiles of up to 8
// jobs that share K.  With Q4_K's w = d * sc_j * q - dmin * m_j (super-block
// scales d, dmin; sub-block j's 6-bit sc_j, m_j; 4-bit q), one super-block
// (256 elements of K) contributes
//     d * sum_k (sc_j q)[row][k] x[token][k]  -  dmin * sum_j m_j bsum_j[token]
// where bsum_j is the sum of x over sub-block j.  Both sums run on the
// tensor core with EXACT weight operands: sc_j * q <= 945 and m_j <= 63 are
// integers below 1024, so their bit patterns are f16 subnormals n * 2^-24
// and the dequantization is three integer instructions per pair of
// elements (byte permute, nibble mask, multiply by sc_j) with no
// conversion.  The activations arrive split as x / s = hi + lo in f16 (s a
// power of two per token), the block sums as f16 hi / lo pairs, so
//   P1 = A1 . [x_hi ; x_lo]   (one MMA of N = 2 nt per 16 elements of K:
//                              the x_hi and x_lo rows stacked along N)
//   P2 = [m_0..7, m_0..7] . [bsum_hi 0..7, bsum_lo 0..7]   (one K=16 MMA)
// per super-block, and the epilogue adds d * 2^24 * (P1_hi + P1_lo) -
// dmin * 2^24 * P2 to a running f32 total in TMEM (round to nearest; each
// TMEM accumulator sees at most 16 MMAs, which keeps the tensor core's own
// accumulation rounding small).  After the last super-block
// y = s * total (+ residual).
//
// Q3_K (expanded device layout: q + 4 in 0..7 as Q4_K-ordered nibbles, 16
// signed int8 scales s_i per super-block, one per 16 elements, and d) runs
// the same kernel: w = d * s_i * (q - 4), and A1 = (q - 4) s_i + 128 is an
// integer in [4, 256] -- an exact f16 subnormal made by one multiply-add per
// pair of elements -- while A2 holds sixteen 128s, so
//     d * (P1 - P2) = d * sum_k (q - 4) s_i x_k
// and the epilogue takes d for both d and dmin.  Its 20-byte headers come in
// as 32-byte boxes from the 16-byte boundary at or below them.
//
// Warp roles (18 warps, one CTA per SM):
//   0      TMA producer.  Ring R, one super-block per stage: the 128 rows'
//          quant bytes (128-byte swizzle), headers, and the block-sum
//          operand B2 (32-byte swizzle).  Ring C, one 64-element chunk per
//          stage: the x_hi / x_lo tiles B1 (128-byte swizzle).
//   1      allocates TMEM and issues all MMAs from one elected lane; commits
//          each C stage, A slot and R stage back to their producers and each
//          super-block's accumulators to the epilogue.
//   2..9   expand a chunk's quant bytes straight into TMEM (tcgen05.st): the
//          A1 operand, 128 lanes = rows, 32 columns = 64 f16 per chunk; once
//          per super-block also the m values into A2 (shared memory, 32-byte
//          swizzle).  A1 in TMEM keeps the MMAs' shared-memory reads to the
//          activation tiles.
//   10..17 epilogue, two warps per TMEM lane quarter.
// TMEM columns: one or two accumulator buffers of [up to 4 independent K
// chains of P1 (2 nt each) | P2 (nt)], the running total (nt), and the A1
// slots (32 each).
// The activation staging stores every quad of elements as (e0, e2, e1, e3);
// A1 is written in the same order, so both operands agree on K.  Every
// mbarrier wait is bounded; on expiry the CTA records the error and skips
// work, and TMEM is always released.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <algorithm>

#include "rq_async.cuh"
#include "rq_mv_common.cuh"
#include "rq_tcgen05.cuh"

namespace rq {
namespace {

using namespace tc;

constexpr int kWarpsTC = 18;
constexpr int kThreadsTC = 32 * kWarpsTC;
constexpr int kDeqWarp0 = 2, kDeqWarps = 8;
constexpr int kEpiWarp0 = 10, kEpiWarps = 8;
static_assert(kDeqWarp0 + kDeqWarps == kEpiWarp0, "warp roles");
static_assert(kEpiWarp0 + kEpiWarps == kWarpsTC, "warp roles");
static_assert(kDeqWarp0 % 4 == 2 && kDeqWarps == 8 && kEpiWarps == 8,
              "two expand and two epilogue warps per TMEM lane quarter");
constexpr int kChunkK = 64;   // elements per chunk (one 128-byte swizzle row)
constexpr int kMaxNT = 112;   // tokens per tile; the MMA's N is 2 nt (x_hi and x_lo stacked)
constexpr int kMaxR = 4, kMaxC = 8, kMaxA = 4;
constexpr int kSmemBudgetTC = 226 * 1024;
constexpr float kSub = 16777216.0f;  // 2^24: f16 subnormal n * 2^-24 -> n
// header box per row and super-block: Q4_K's 16 bytes; Q3_K's 20 bytes
// (16 int8 scales, f16 d, 2 pad) read as the 32-byte box from the 16-byte
// boundary at or below them (TMA boxes start and end on 16-byte multiples)
template <bool Q3>
constexpr uint32_t kHdrBox = Q3 ? 32u : 16u;

struct TCJob {
    float* y;
    const float* add;
    const uint8_t* hdr;  // [out][nblk][16] (Q3_K: [20])
    int64_t out;
    int tok0, M;
    int nt;              // tokens per tile (MMA N, a multiple of 16)
    int rtiles, ttiles;  // 128-row tiles, nt-token tiles
    int t0;              // first tile index of this job
};

struct alignas(64) TCParams {
    CUtensorMap wq[kMaxJobs];  // quant bytes [out][nblk*128], box 128 x 128, 128-byte swizzle
    CUtensorMap wh[kMaxJobs];  // headers [out][nblk*16], box 16 x 128 (Q3_K: [out][nblk*20], box 32 x 128)
    CUtensorMap xhi[kMaxJobs];  // staged x, hi plane [rows][in] f16, box 64 x nt_j, 128-byte swizzle
    CUtensorMap xlo[kMaxJobs];
    CUtensorMap bs;            // block sums [rows][nblk*16] f16, box 16 x box, 32-byte swizzle
    TCJob jobs[kMaxJobs];
    const float* xscale;
    int* err;
    int njobs, ntiles, nblk, box, nr, nc, na, tmem_cols;
    int w_once;  // every job has one token tile: weights are read once, evict them first
    uint32_t r_bytes, r_hdr, r_b2, r_a2;  // R stage: quant at 0, headers, B2, A2
    uint32_t c_bytes;                     // C stage: B1 = x_hi rows, then x_lo rows (nt each)
    int nck, nb;        // K chains per super-block, accumulator buffers
    uint32_t buf_cols;  // columns of one buffer: nck chains of 2 box, then P2 (box)
    uint32_t tot_col, acol0;
    uint32_t c_off;                       // ring C after ring R
};

struct Tile {
    int j, rt, tt;
};

__device__ __forceinline__ Tile tile_of(const TCParams& p, int t) {
    int j = 0;
    while (j + 1 < p.njobs && t >= p.jobs[j + 1].t0) j++;
    // token tiles of one row tile are adjacent: CTAs that run at the same
    // time read the same weights, which HBM then delivers once
    const int local = t - p.jobs[j].t0;
    return Tile{j, local / p.jobs[j].ttiles, local % p.jobs[j].ttiles};
}

// Q3 = false: Q4_K weights; true: Q3_K in the expanded device layout
template <bool Q3>
__global__ void __launch_bounds__(kThreadsTC, 1) mm_tc_kernel(const __grid_constant__ TCParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    uint8_t* smem = smem_raw + pad;
    const uint32_t sbase = raw + pad;
    // barriers (first 1 KB): rfull, rempty [kMaxR]; cfull, cempty [kMaxC];
    // aready, aempty [kMaxA]; accfull, accempty [2]; the TMEM address slot
    const uint32_t rfull0 = sbase, rempty0 = rfull0 + 8 * kMaxR;
    const uint32_t cfull0 = rempty0 + 8 * kMaxR, cempty0 = cfull0 + 8 * kMaxC;
    const uint32_t aready0 = cempty0 + 8 * kMaxC, aempty0 = aready0 + 8 * kMaxA;
    const uint32_t accfull0 = aempty0 + 8 * kMaxA, accempty0 = accfull0 + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (accempty0 + 16 - sbase));
    const uint32_t ringr = sbase + 1024, ringc = ringr + p.c_off;
    uint8_t* ringr_p = smem + 1024;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nblk = p.nblk;

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nr; i++) {
            mbar_init(rfull0 + 8 * i, 1);
            mbar_init(rempty0 + 8 * i, 1);
        }
        for (int i = 0; i < p.nc; i++) {
            mbar_init(cfull0 + 8 * i, 1);
            mbar_init(cempty0 + 8 * i, 1);
        }
        for (int i = 0; i < p.na; i++) {
            mbar_init(aready0 + 8 * i, kDeqWarps);
            mbar_init(aempty0 + 8 * i, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(accfull0 + 8 * b, 1);
            mbar_init(accempty0 + 8 * b, kEpiWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the staged activations are written by the preceding kernel in the stream
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int box = p.box;
    const uint32_t acol0 = p.acol0;  // first A slot column
    if (warp == 0) {
        // -------------------------------------------------------------- TMA
        if (lane == 0) {
            const uint64_t pol_w = p.w_once ? policy_evict_first() : policy_evict_normal();
            const uint64_t pol_x = policy_evict_last();
            const uint32_t rtx = kRowsTC * 128 + kRowsTC * kHdrBox<Q3> + 32u * (uint32_t)box;
            Ring rr, cr;
            int ri = 0, ci = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
                const Tile tl = tile_of(p, t);
                const TCJob& jb = p.jobs[tl.j];
                const int row0 = tl.rt * kRowsTC, tok = jb.tok0 + tl.tt * jb.nt;
                const uint32_t ctx = 2u * 128u * (uint32_t)jb.nt;
                for (int sb = 0; sb < nblk && ok; sb++, ri++, rr.next(p.nr)) {
                    const int rs = rr.i, ru = rr.u;
                    if (ru > 0 && !wait_err(rempty0 + 8 * rs, (ru - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = ringr + (uint32_t)rs * p.r_bytes;
                    const uint32_t fb = rfull0 + 8 * rs;
                    mbar_expect_tx(fb, rtx);
                    tma_load_2d(st, &p.wq[tl.j], sb * 128, row0, fb, pol_w);
                    // Q3_K: the 20 header bytes of super-block sb lie in the
                    // 32-byte box that starts at the 16-byte boundary below them
                    tma_load_2d(st + p.r_hdr, &p.wh[tl.j], Q3 ? (sb * 20) & ~15 : sb * 16, row0, fb, pol_w);
                    tma_load_2d(st + p.r_b2, &p.bs, sb * 16, tok, fb, pol_x);
                    for (int cq = 0; cq < 4; cq++, ci++, cr.next(p.nc)) {
                        const int cs = cr.i, cu = cr.u;
                        if (cu > 0 && !wait_err(cempty0 + 8 * cs, (cu - 1) & 1, p.err)) {
                            ok = false;
                            break;
                        }
                        const uint32_t sc = ringc + (uint32_t)cs * p.c_bytes;
                        const uint32_t cb = cfull0 + 8 * cs;
                        mbar_expect_tx(cb, ctx);
                        tma_load_2d(sc, &p.xhi[tl.j], (4 * sb + cq) * kChunkK, tok, cb, pol_x);
                        tma_load_2d(sc + 128u * (uint32_t)jb.nt, &p.xlo[tl.j], (4 * sb + cq) * kChunkK, tok, cb,
                                    pol_x);
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
        // The whole warp runs the loop, so every operand is warp-uniform; one
        // elected lane issues each MMA and commit.
        Ring rr, cr, ar, br;  // R stages, C stages, A slots, accumulator buffers
        const int chm = p.nck - 1;  // nck is 1, 2 or 4
        bool ok = true;
        for (int t = blockIdx.x; t < p.ntiles; t += gridDim.x) {
            const int nt = p.jobs[tile_of(p, t).j].nt;
            const uint32_t idesc1 = umma_idesc(2 * nt), idesc2 = umma_idesc(nt);
            for (int sb = 0; sb < nblk; sb++, rr.next(p.nr), br.next(p.nb)) {
                const int b = br.i;
                // buffer b is free once the epilogue has read its previous super-block
                if (ok && br.u > 0 && !wait_err(accempty0 + 8 * b, (br.u - 1) & 1, p.err)) ok = false;
                ok = __all_sync(0xffffffffu, ok);
                tmem_fence_after();
                const uint32_t bcol = tmem + (uint32_t)b * p.buf_cols;
                for (int cq = 0; cq < 4; cq++, cr.next(p.nc), ar.next(p.na)) {
                    const int cs = cr.i, cu = cr.u;
                    const int as = ar.i, au = ar.u;
                    if (ok && !wait_err(cfull0 + 8 * cs, cu & 1, p.err)) ok = false;
                    if (ok && !wait_err(aready0 + 8 * as, au & 1, p.err)) ok = false;
                    ok = __all_sync(0xffffffffu, ok);
                    tmem_fence_after();
                    const uint32_t sc = ringc + (uint32_t)cs * p.c_bytes;
                    const uint32_t acol = tmem + acol0 + 32u * (uint32_t)as;
                    if (elect_one()) {
                        if (ok) {
#pragma unroll
                            for (int kk = 0; kk < kChunkK / 16; kk++) {
                                // K step 4 cq + kk of the super-block goes to chain
                                // (4 cq + kk) % nck: independent accumulators keep
                                // several MMAs in flight
                                const int step = 4 * cq + kk;
                                const uint32_t d = bcol + (uint32_t)((step & chm) * 2 * box);
                                umma_f16_ts(d, acol + 8u * kk, desc_sw128(sc + 32u * kk), idesc1,
                                            step > chm ? 1u : 0u);
                            }
                        }
                        // B1 and the A slot are free once these MMAs finish
                        umma_commit(cempty0 + 8 * cs);
                        umma_commit(aempty0 + 8 * as);
                    }
                    __syncwarp();
                }
                const int rs = rr.i;
                const uint32_t st = ringr + (uint32_t)rs * p.r_bytes;
                if (elect_one()) {
                    if (ok)
                        umma_f16(bcol + (uint32_t)(p.nck * 2 * box), desc_sw32(st + p.r_a2), desc_sw32(st + p.r_b2),
                                 idesc2, 0u);
                    umma_commit(rempty0 + 8 * rs);
                    umma_commit(accfull0 + 8 * b);
                }
                __syncwarp();
            }
        }
        if (!ok && lane == 0 && p.err) atomicExch(p.err, 1);
    } else if (warp < kEpiWarp0) {
        // ----------------------------------------------------------- expand
        // Warp w writes TMEM lanes 32 (w % 4) .. +31: row r of the tile, the
        // low (h = 0) or high (h = 1) nibbles of each 64-element chunk.
        const int q = warp & 3, h = (warp - kDeqWarp0) >> 2;
        const int r = 32 * q + lane;
        const uint32_t swz = (uint32_t)(r & 7);
        const uint32_t lane_a = tmem + ((uint32_t)(32 * q) << 16) + acol0 + 16u * (uint32_t)h;
        Ring rr, ar;
        bool ok = true;
        for (int tt = blockIdx.x; tt < p.ntiles; tt += gridDim.x) {
            for (int sb = 0; sb < nblk; sb++, rr.next(p.nr)) {
                const int rs = rr.i, ru = rr.u;
                if (ok && !wait_err(rfull0 + 8 * rs, ru & 1, p.err)) ok = false;
                uint8_t* rst = ringr_p + (size_t)rs * p.r_bytes;
                uint4 hd;
                if constexpr (Q3) {
                    // the 16 int8 scales at byte 4 (sb % 4) of the row's box
                    const uint32_t* h4 =
                        reinterpret_cast<const uint32_t*>(rst + p.r_hdr + r * 32 + 4 * (sb & 3));
                    hd = make_uint4(h4[0], h4[1], h4[2], h4[3]);
                } else {
                    hd = *reinterpret_cast<const uint4*>(rst + p.r_hdr + r * 16);
                }
                if (ok && h == 0 && Q3) {
                    // A2 row r: sixteen 128s (f16 subnormal 128 * 2^-24); with
                    // the block sums it removes the +128 bias of A1
                    const uint4 mv = make_uint4(0x00800080u, 0x00800080u, 0x00800080u, 0x00800080u);
                    uint8_t* a2 = rst + p.r_a2 + (r >> 3) * 256 + (r & 7) * 32;
                    *reinterpret_cast<uint4*>(a2) = mv;
                    *reinterpret_cast<uint4*>(a2 + 16) = mv;
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                } else if (ok && h == 0) {
                    // A2 row r: [m_0..7, m_0..7] as f16 subnormals (32-byte
                    // swizzle; both 16-byte halves are equal)
                    uint32_t m[4];
#pragma unroll
                    for (int g = 0; g < 4; g++) {
                        const uint32_t w = q4k_scales(q4k_scale_sel(g), hd);
                        m[g] = ((w >> 16) & 0xFFu) | ((w >> 24) << 16);
                    }
                    const uint4 mv = make_uint4(m[0], m[1], m[2], m[3]);
                    uint8_t* a2 = rst + p.r_a2 + (r >> 3) * 256 + (r & 7) * 32;
                    *reinterpret_cast<uint4*>(a2) = mv;
                    *reinterpret_cast<uint4*>(a2 + 16) = mv;
                    // generic-proxy writes become visible to the tensor core
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
                for (int cq = 0; cq < 4; cq++, ar.next(p.na)) {
                    const int as = ar.i, au = ar.u;
                    if (ok && au > 0 && !wait_err(aempty0 + 8 * as, (au - 1) & 1, p.err)) ok = false;
                    ok = __all_sync(0xffffffffu, ok);  // tcgen05.st is warp-wide
                    tmem_fence_after();
                    if (ok) {
                        // this chunk's 32 quant bytes of row r: 16-byte chunks
                        // 2cq, 2cq+1 of the row's 128-byte-swizzled line
                        const uint8_t* qrow = rst + r * 128;
                        const uint4 qa = *reinterpret_cast<const uint4*>(qrow + (((2 * cq) ^ swz) << 4));
                        const uint4 qb = *reinterpret_cast<const uint4*>(qrow + (((2 * cq + 1) ^ swz) << 4));
                        const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                        // per 16-byte half: A = q * s + c in both 16-bit lanes.
                        // Q4_K: s = sc_j (the half's 32-element sub-block), c = 0.
                        // Q3_K: the halves are 16-element sub-blocks 4cq + 2h and
                        // 4cq + 2h + 1 (q = stored q + 4 in 0..7, s the signed
                        // scale): A = (q - 4) s + 128 = q s + (128 - 4 s) lies in
                        // [4, 256] in each lane, so the packed 32-bit
                        // multiply-add is exact whatever the sign of s.
                        uint32_t sa, sb2, ca = 0u, cb = 0u;
                        if constexpr (Q3) {
                            const uint32_t sw = cq == 0 ? hd.x : cq == 1 ? hd.y : cq == 2 ? hd.z : hd.w;
                            const int s0 = (int)(int8_t)(uint8_t)(sw >> (16 * h));
                            const int s1 = (int)(int8_t)(uint8_t)(sw >> (16 * h + 8));
                            sa = (uint32_t)s0;
                            sb2 = (uint32_t)s1;
                            ca = (uint32_t)(128 - 4 * s0) * 0x00010001u;
                            cb = (uint32_t)(128 - 4 * s1) * 0x00010001u;
                        } else {
                            const uint32_t w = q4k_scales(q4k_scale_sel(cq), hd);
                            sa = sb2 = (w >> (8 * h)) & 0xFFu;
                        }
                        uint32_t o[16];
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            // bytes b0..b3 -> (e0, e2) and (e1, e3) in 16-bit lanes
                            uint32_t u0 = __byte_perm(qw[i], 0, 0x4240), u1 = __byte_perm(qw[i], 0, 0x4341);
                            if (h) {
                                u0 >>= 4;
                                u1 >>= 4;
                            }
                            const uint32_t s = i < 4 ? sa : sb2, c = i < 4 ? ca : cb;
                            o[2 * i] = (u0 & 0x000F000Fu) * s + c;
                            o[2 * i + 1] = (u1 & 0x000F000Fu) * s + c;
                        }
                        // TMEM column c of the slot holds K positions 2c, 2c+1
                        tmem_st16u(lane_a + 32u * (uint32_t)as, o);
                        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    }
                    tmem_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(aready0 + 8 * as);
                }
            }
        }
        if (!ok && lane == 0 && p.err) atomicExch(p.err, 1);
    } else {
        // ------------------------------------------------------------ epilogue
        // Warp w reads TMEM lanes 32 (w % 4) .. +31; the two warps of a lane
        // quarter take alternate 16-column groups.
        const int q = warp & 3, half = (warp - kEpiWarp0) >> 2;
        const int row_in = 32 * q + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        Ring br;
        bool ok = true;
        for (int t = blockIdx.x; t < p.ntiles; t += gridDim.x) {
            const Tile tl = tile_of(p, t);
            const TCJob& jb = p.jobs[tl.j];
            const int64_t row = (int64_t)tl.rt * kRowsTC + row_in;
            const bool live = row < jb.out;
            // per super-block: Q4_K (d, dmin) at byte 0 of its 16 header
            // bytes; Q3_K d at byte 16 of its 20 (the bias term scales by d)
            constexpr int hb = Q3 ? 20 : 16, hoff = Q3 ? 16 : 0;
            const uint8_t* hrow = jb.hdr + (live ? row : 0) * (int64_t)nblk * hb + hoff;
            const int nt0 = tl.tt * jb.nt;
            uint32_t dd = live ? __ldg(reinterpret_cast<const uint32_t*>(hrow)) : 0u;
            const int nt = jb.nt;
            for (int sb = 0; sb < nblk; sb++, br.next(p.nb)) {
                const int b = br.i;
                const bool first = sb == 0, last = sb == nblk - 1;
                const uint32_t dd_next =
                    (live && !last) ? __ldg(reinterpret_cast<const uint32_t*>(hrow + (sb + 1) * hb)) : 0u;
                const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&dd));
                const float fd = dm.x * kSub, fm = -(Q3 ? dm.x : dm.y) * kSub;
                if (ok && !wait_err(accfull0 + 8 * b, br.u & 1, p.err)) ok = false;
                ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld / st are warp-wide
                tmem_fence_after();
                const uint32_t bcol = lane_base + (uint32_t)b * p.buf_cols;
                if (ok) {
                    for (int n0 = 16 * half; n0 < nt; n0 += 32) {
                        // P1 = sum over the chains of (x_hi part + x_lo part)
                        float v1[16];
                        for (int c = 0; c < p.nck; c++) {
                            uint32_t uh[16], ul[16];
                            tmem_ld16(bcol + (uint32_t)(c * 2 * box + n0), uh);
                            tmem_ld16(bcol + (uint32_t)(c * 2 * box + nt + n0), ul);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 16; i++) {
                                const float hl = __uint_as_float(uh[i]) + __uint_as_float(ul[i]);
                                v1[i] = c == 0 ? hl : v1[i] + hl;
                            }
                        }
                        uint32_t u2[16], ua[16];
                        tmem_ld16(bcol + (uint32_t)(p.nck * 2 * box + n0), u2);
                        if (!first) tmem_ld16(lane_base + p.tot_col + (uint32_t)n0, ua);
                        tmem_wait_ld();
                        float a[16];
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            const float s = first ? 0.0f : __uint_as_float(ua[i]);
                            a[i] = fmaf(fm, __uint_as_float(u2[i]), fmaf(fd, v1[i], s));
                        }
                        if (!last) {
                            tmem_st16(lane_base + p.tot_col + (uint32_t)n0, a);
                            continue;
                        }
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            const int n = nt0 + n0 + i;
                            if (n < jb.M && live) {
                                const int64_t o = (int64_t)n * jb.out + row;
                                const float v = a[i] * p.xscale[jb.tok0 + n];
                                jb.y[o] = jb.add ? v + jb.add[o] : v;
                            }
                        }
                    }
                    if (!last) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                }
                tmem_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(accempty0 + 8 * b);
                dd = dd_next;
            }
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)p.tmem_cols)
                     : "memory");
}

}  // namespace

// Q3_K headers are 20 bytes per super-block: the tensor map's row pitch
// (nblk * 20 bytes) must be a multiple of 16
bool mm_tc_supported(const rq_weight* w) {
    return w->type == RQ_Q4_K || (w->type == RQ_Q3_K && w->nblk % 4 == 0);
}

int launch_mm_tc(const MMJobDesc* jobs, int njobs, XH xh, int64_t rows, int sm_count, cudaStream_t st, int* err) {
    if (njobs < 1 || njobs > kMaxJobs) return set_error(RQ_ERR_INVALID, "tensor-core matmul: %d jobs", njobs);
    const int64_t in = jobs[0].w->in, nblk = jobs[0].w->nblk;
    const bool q3 = jobs[0].w->type == RQ_Q3_K;
    TCParams p;
    memset(&p, 0, sizeof p);
    int tiles = 0, box = 16;
    p.w_once = 1;
    for (int j = 0; j < njobs; j++) {
        const rq_weight* w = jobs[j].w;
        if (!mm_tc_supported(w) || w->type != jobs[0].w->type || w->in != in)
            return set_error(RQ_ERR_INVALID,
                             "tensor-core matmul: jobs need Q4_K (or Q3_K, nblk %% 4 == 0) weights of one type "
                             "with the same K");
        if (jobs[j].M < 1 || jobs[j].tok0 < 0 || jobs[j].tok0 + jobs[j].M > rows)
            return set_error(RQ_ERR_INVALID, "tensor-core matmul: token rows [%d, %d) of %lld", jobs[j].tok0,
                             jobs[j].tok0 + jobs[j].M, (long long)rows);
        int rc = encode(&p.wq[j], CU_TENSOR_MAP_DATA_TYPE_UINT8, w->qs, (uint64_t)(nblk * 128), (uint64_t)w->out,
                        (uint64_t)(nblk * 128), 128, kRowsTC, CU_TENSOR_MAP_SWIZZLE_128B, "quant bytes");
        const uint64_t hrow = (uint64_t)nblk * (q3 ? 20 : 16);
        if (!rc)
            rc = encode(&p.wh[j], CU_TENSOR_MAP_DATA_TYPE_UINT8, w->hdr, hrow, (uint64_t)w->out, hrow,
                        q3 ? kHdrBox<true> : kHdrBox<false>, kRowsTC, CU_TENSOR_MAP_SWIZZLE_NONE, "headers");
        if (rc) return rc;
        TCJob& t = p.jobs[j];
        t.y = jobs[j].y;
        t.add = jobs[j].add;
        t.hdr = w->hdr;
        t.out = w->out;
        t.tok0 = jobs[j].tok0;
        t.M = jobs[j].M;
        t.rtiles = (int)((w->out + kRowsTC - 1) / kRowsTC);
        // even token tiles of at most kMaxNT, rounded up to the MMA's N step
        t.ttiles = (jobs[j].M + kMaxNT - 1) / kMaxNT;
        t.nt = ((jobs[j].M + t.ttiles - 1) / t.ttiles + 15) & ~15;
        box = std::max(box, t.nt);
        if (t.ttiles > 1) p.w_once = 0;
        t.t0 = tiles;
        tiles += t.rtiles * t.ttiles;
    }
    int rc = RQ_OK;
    for (int j = 0; j < njobs && !rc; j++) {
        rc = encode(&p.xhi[j], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh.v, (uint64_t)in, (uint64_t)rows,
                    (uint64_t)(4 * in), kChunkK, (uint32_t)p.jobs[j].nt, CU_TENSOR_MAP_SWIZZLE_128B,
                    "activations (hi)");
        if (!rc)
            rc = encode(&p.xlo[j], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh.v + in, (uint64_t)in, (uint64_t)rows,
                        (uint64_t)(4 * in), kChunkK, (uint32_t)p.jobs[j].nt, CU_TENSOR_MAP_SWIZZLE_128B,
                        "activations (lo)");
    }
    if (!rc)
        rc = encode(&p.bs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh.bs16, (uint64_t)(nblk * 16), (uint64_t)rows,
                    (uint64_t)(nblk * 32), 16, (uint32_t)box, CU_TENSOR_MAP_SWIZZLE_32B, "block sums");
    if (rc) return rc;
    p.xscale = xh.scale;
    p.err = err;
    p.njobs = njobs;
    p.ntiles = tiles;
    p.nblk = (int)nblk;
    p.box = box;
    // TMEM columns: nb buffers of [nck chains x 2 box | P2 box], the running
    // total (box), then na A slots of 32.  Chains hide the ~150-cycle latency
    // of dependent MMAs (an M=128 MMA of N = 2 box takes ~box cycles); two
    // buffers let the epilogue read one super-block while the next one runs.
    int nck = box <= 16 ? 4 : box <= 32 ? 2 : 1;
    int nb = 2, na = 0;
    for (;;) {
        const int used = nb * (nck * 2 * box + box) + box;
        na = std::min(kMaxA, (512 - used) / 32);
        if (na >= 2) break;
        if (nb == 2) {
            nb = 1;
        } else if (nck > 1) {
            nck--;
        } else {
            return set_error(RQ_ERR_UNSUPPORTED, "tensor-core matmul: %d tokens per tile", box);
        }
    }
    p.nck = nck;
    p.nb = nb;
    p.na = na;
    p.buf_cols = (uint32_t)(nck * 2 * box + box);
    p.tot_col = (uint32_t)nb * p.buf_cols;
    p.acol0 = p.tot_col + (uint32_t)box;
    p.tmem_cols = 32;
    while (p.tmem_cols < (int)p.acol0 + 32 * na) p.tmem_cols *= 2;
    // R stage: quant 16 KB | headers 2 KB (Q3_K 4 KB) | B2 box x 32 B | A2 4 KB
    // C stage: B1 hi, B1 lo nt x 128 B each (at most box); every tile 1024-aligned
    auto al = [](uint32_t v) { return (v + 1023u) & ~1023u; };
    p.r_hdr = kRowsTC * 128;
    p.r_b2 = al(p.r_hdr + kRowsTC * (q3 ? kHdrBox<true> : kHdrBox<false>));
    p.r_a2 = al(p.r_b2 + 32u * (uint32_t)box);
    p.r_bytes = al(p.r_a2 + kRowsTC * 32);
    p.c_bytes = al(2 * 128u * (uint32_t)box);
    const int avail = kSmemBudgetTC - 2048;
    p.nr = 3;
    p.nc = std::min(kMaxC, (avail - 3 * (int)p.r_bytes) / (int)p.c_bytes);
    if (p.nc < 3) {
        p.nr = 2;
        p.nc = std::min(kMaxC, (avail - 2 * (int)p.r_bytes) / (int)p.c_bytes);
    }
    if (p.nc < 2) return set_error(RQ_ERR_UNSUPPORTED, "tensor-core matmul: stages too large");
    p.c_off = (uint32_t)p.nr * p.r_bytes;
    const size_t smem = 2048 + (size_t)p.nr * p.r_bytes + (size_t)p.nc * p.c_bytes;
    const int grid = std::min(tiles, sm_count);

    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e =
            cudaFuncSetAttribute(mm_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudgetTC);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(mm_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudgetTC);
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(tensor-core matmul)");
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreadsTC);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_error(q3 ? cudaLaunchKernelEx(&cfg, mm_tc_kernel<true>, p) : cudaLaunchKernelEx(&cfg, mm_tc_kernel<false>, p),
                      "tensor-core matmul kernel");
}

}  // namespace rq
