// rq_mm_i8.cu -- Q4_K matmul for two activation rows (the speculative
// verify of a one-token draft, M = K + 1 = 2) on the int8 tensor cores:
// mma.sync m16n8k32, u8 weights x s8 activations -> s32, one weight pass.
//
// The work is HBM-bound, so the kernel keeps the M=1 pipeline's data path --
// one persistent CTA per SM owning a contiguous range of output rows, a
// producer lane streaming whole rows into a ring of shared-memory stages with
// bulk copies -- and replaces the per-row dp4a work by tensor-core tiles:
//
//   A (16 weight rows x 32 elements of K, u8): the 4-bit quants as they are.
//     A lane's 8 bytes of a 32-byte nibble group give both sub-blocks of the
//     group: low nibbles = sub-block 2c, high nibbles = 2c+1 (one mask or
//     shift-and-mask per 4 weights, no conversion).  Stages hold 16 rows;
//     each row is copied to its own shared-memory row padded by 32 bytes
//     (quants) / 16 bytes (headers), so the 8 rows a warp-wide load touches
//     fall in distinct banks.
//   B (32 elements x 8 columns, s8): column n = plane n / 2 of token n % 2
//     (columns 6, 7 zero), the activations staged in 24-bit fixed point as
//     three balanced bytes X = 65536 x1 + 256 x2 + x3 with one scale per
//     token and super-block (XQ2) -- the M=1 path's precision.  A warp owns a
//     K-slice of at most 4 super-blocks and holds that slice's B fragments
//     in registers for the whole launch.
//
// K-slot 4t + i of an MMA is element 8t + i of the sub-block and slot
// 16 + 4t + i element 8t + 4 + i (t = the lane's quad position): a thread's
// fragment registers then cover bytes 8t .. 8t+7 of a weight row and of an
// activation row, so both operands are single 8-byte loads.  Per sub-block
// the s32 tile is scaled by the row's 6-bit sc_j with an integer
// multiply-add (exact: |sum| < 2^31 over a super-block), and once per
// super-block the s32 sums become f32:
//   y += d * sx_tok * pw_plane * S  -  dmin * sum_j m_j * bsum_j
// with the min term from the f32 block sums of x.  At the end of a stage the
// three planes of a token are added over the lane quad, and each warp
// writes its K-slice partials of the 16 rows into a per-CTA table
// [row][slice][token]; after the last stage the slices are summed in order
// (deterministic) into y.  Every mbarrier wait is bounded (~1 s); on expiry
// the kernel sets the error word, drains its copies and returns.

#include <string.h>

#include <algorithm>

#include "rq_async.cuh"
#include "rq_internal.cuh"
#include "rq_tcgen05.cuh"

namespace rq {

// ---------------------------------------------------- activation staging

constexpr float kXQ3Scale = 8323072.0f;  // 127 * 65536: the three balanced bytes of X stay in [-127, 127]

size_t xq2_bytes(int64_t M, int64_t in) {
    size_t b = ((size_t)M * 3 * (size_t)in + 255) & ~(size_t)255;
    b += ((size_t)M * (size_t)(in / 256) * 4 + 255) & ~(size_t)255;
    b += (size_t)M * (size_t)(in / 32) * 4;
    return b;
}

XQ2 xq2_at(void* base, int64_t M, int64_t in) {
    uint8_t* p = (uint8_t*)base;
    XQ2 q;
    q.planes = (int8_t*)p;
    p += ((size_t)M * 3 * (size_t)in + 255) & ~(size_t)255;
    q.sx = (float*)p;
    p += ((size_t)M * (size_t)(in / 256) * 4 + 255) & ~(size_t)255;
    q.bsum = (float*)p;
    return q;
}

namespace {

// One warp per (token, super-block): lane l holds elements 8l .. 8l+7.
// X = rint(v * 127*65536 / amax) over the super-block, as three balanced
// bytes X = 65536 x1 + 256 x2 + x3 (stage_block's digits, one scale per 256
// elements instead of per 32), v = x or, with rms_w, the RMSNorm of x
// (xquant_rmsnorm_kernel's formula and sum of squares), or with up,
// silu(x) * up (x the gate rows); the f32 block sums
// of v are summed over the four lanes of a 32-element block.  Grid
// (ceil(nsb / 8), M), 256 threads: eight super-blocks of one token per CTA.
__global__ void xq2_stage_kernel(const float* __restrict__ x, int64_t in, XQ2 q, const float* __restrict__ rms_w,
                                 float eps, const float* __restrict__ up) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    __shared__ float wsum[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t nsb = in / 256, m = blockIdx.y;
    const float* row = x + m * in;
    float mden = 1.0f;
    if (rms_w) {
        float s2 = 0.0f;
        if ((in & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
            const float4* r4 = reinterpret_cast<const float4*>(row);
            for (int64_t i = threadIdx.x; i < in / 4; i += blockDim.x) {
                const float4 v = r4[i];
                s2 = fmaf(v.x, v.x, s2); s2 = fmaf(v.y, v.y, s2);
                s2 = fmaf(v.z, v.z, s2); s2 = fmaf(v.w, v.w, s2);
            }
        } else {
            for (int64_t i = threadIdx.x; i < in; i += blockDim.x) s2 = fmaf(row[i], row[i], s2);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        if (lane == 0) wsum[warp] = s2;
        __syncthreads();
        float tot = 0.0f;
        for (int k = 0; k < 8; k++) tot += wsum[k];
        mden = sqrtf(tot / (float)in + eps);
    }
    const int64_t sb = (int64_t)blockIdx.x * 8 + warp;
    if (sb >= nsb) return;
    const float* src = row + sb * 256 + 8 * lane;
    float v[8];
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        const float4 a = reinterpret_cast<const float4*>(src)[0], b = reinterpret_cast<const float4*>(src)[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = src[k];
    }
    if (rms_w) {
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = v[k] / mden * rms_w[sb * 256 + 8 * lane + k];
    }
    if (up) {  // SwiGLU: x is the gate row, v = silu(gate) * up (xquant_swiglu_kernel's formula)
        const float* u = up + m * in + sb * 256 + 8 * lane;
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = v[k] / (1.0f + expf(-v[k])) * u[k];
    }
    float amax = 0.0f, s = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        amax = fmaxf(amax, fabsf(v[k]));
        s += v[k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    const float inv = amax > 0.0f ? kXQ3Scale / amax : 0.0f;
    uint32_t p1[2] = {0u, 0u}, p2[2] = {0u, 0u}, p3[2] = {0u, 0u};
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int X = __float2int_rn(v[k] * inv);
        const int x3 = (X << 24) >> 24;  // balanced base-256 digits
        const int t1 = (X - x3) >> 8;
        const int x2 = (t1 << 24) >> 24;
        const int x1 = (t1 - x2) >> 8;
        p1[k / 4] |= (uint32_t)(x1 & 255) << (8 * (k % 4));
        p2[k / 4] |= (uint32_t)(x2 & 255) << (8 * (k % 4));
        p3[k / 4] |= (uint32_t)(x3 & 255) << (8 * (k % 4));
    }
    int8_t* base = q.planes + m * 3 * in + sb * 256 + 8 * lane;
    *reinterpret_cast<uint2*>(base) = make_uint2(p1[0], p1[1]);
    *reinterpret_cast<uint2*>(base + in) = make_uint2(p2[0], p2[1]);
    *reinterpret_cast<uint2*>(base + 2 * in) = make_uint2(p3[0], p3[1]);
    if ((lane & 3) == 0) q.bsum[m * (in / 32) + sb * 8 + lane / 4] = s;
    if (lane == 0) q.sx[m * nsb + sb] = amax / kXQ3Scale;
}

// ------------------------------------------------------------------ matmul

constexpr int kI8Cons = 8;         // consumer warps = K-slices
constexpr int kI8Threads = 32 * (1 + kI8Cons);
constexpr int kI8Rows = 16;        // weight rows per stage (one MMA tile)
constexpr int kI8MaxSB = 4;        // super-blocks per K-slice (K <= 8192)
constexpr int kI8QPad = 32, kI8HPad = 16;
constexpr int kI8Smem = 226 * 1024;  // dynamic part; a few static bytes besides
constexpr int kI8Bar = 2 * 16 * 8;  // up to 16 stages: full + empty barriers
constexpr int kI8MaxRowGroups = 256;  // arrival counters a split K may use

struct I8Job {
    const uint8_t* qs;
    const uint8_t* hdr;
    float* y;          // [M][out]
    const float* add;  // optional residual [M][out]: y = x W^T + add (may alias y)
    int64_t out;
};

struct I8Params {
    I8Job jobs[kMaxJobs];
    int njobs, M;
    int64_t in;
    int nsb;                    // super-blocks per row
    uint32_t qrow, hrow;        // device bytes per row
    uint32_t qstride, hstride;  // padded shared-memory row strides
    uint32_t stage_bytes, red_off, ring_off;
    int nstage;
    int RS;                     // weight rows per stage (<= 16, the MMA tile)
    uint32_t b_off, bstride;    // four-token kernel: staged activations [12][bstride] in shared memory
    uint32_t pr_off;            // four-token kernel: per-stage partial sums [2][16][8][4]
    int ks;                     // K-splits: CTA b takes K-range b % ks of row group b / ks
    int nsbr;                   // super-blocks per full row (nsb: per K-range)
    uint32_t qseg, hseg;        // device bytes of a K-range of a row
    uint32_t hsb;               // header bytes per super-block (Q4_K 16, Q3_K 20)
    float* part;                // ks > 1: partial y [ks][M][out]
    int* cnt;                   // ks > 1: arrivals per row group (zero between launches)
    XQ2 xq;
    int* err;
};

// rows of row group rg of nrg (the CTA's rows when K is not split)
__device__ __forceinline__ void i8_rows(const I8Job& j, int rg, int nrg, int64_t* rb, int* n) {
    const int64_t b = (int64_t)rg * j.out / nrg;
    const int64_t e = (int64_t)(rg + 1) * j.out / nrg;
    *rb = b;
    *n = (int)(e - b);
}

// K-split reduction: this CTA's partial rows are in part; the last of the
// ks CTAs of the row group to arrive sums the ks partials in split order
// (deterministic) into y.  Run by `nthr` threads (ct = 0..nthr-1) that
// synchronise with named barrier `bar`.
__device__ __forceinline__ void i8_ksplit_finish(const I8Params& p, int rgi, int nrg, int ct, int nthr, int bar,
                                                 int* s_last) {
    __threadfence();
    named_bar_sync(bar, nthr);
    if (ct == 0) {
        __threadfence();
        const int old = atomicAdd(p.cnt + rgi, 1);
        *s_last = old == p.ks - 1;
        if (old == p.ks - 1) atomicExch(p.cnt + rgi, 0);
    }
    named_bar_sync(bar, nthr);
    if (!*s_last) return;
    __threadfence();
    const I8Job& jb = p.jobs[0];
    int64_t rb;
    int nrows;
    i8_rows(jb, rgi, nrg, &rb, &nrows);
    for (int e = ct; e < nrows * p.M; e += nthr) {
        const int r = e / p.M, m = e % p.M;
        const int64_t o = (int64_t)m * jb.out + rb + r;
        float acc = 0.0f;
        for (int k = 0; k < p.ks; k++) acc += __ldcg(p.part + (int64_t)k * p.M * jb.out + o);
        jb.y[o] = jb.add ? acc + jb.add[o] : acc;
    }
}

__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// weight formats of the int8 kernels
constexpr int kI8Q4K = 0, kI8Q3K = 1, kI8Q40 = 2;

// signed s32 -> f32 for |v| < 2^22 without the conversion unit: v placed
// in the mantissa of 1.5 * 2^23, minus 1.5 * 2^23 (exact)
__device__ __forceinline__ float i2f_small(int v) {
    return __int_as_float(0x4B400000 + v) - 12582912.0f;
}

// m16n8k16 s8 x s8 -> s32 (a Q3_K 16-element sub-block per MMA)
__device__ __forceinline__ void mma_s8s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Q3_K quants (q + 4 in 0..7, three bits of each nibble) -> 32 (q - 4) as
// four signed bytes: the three bits moved to bits 5..7 of their byte, bit 7
// flipped.  Low nibbles (lo) or high nibbles (hi) of the word.
__device__ __forceinline__ uint32_t q3_lo(uint32_t w) { return ((w << 5) & 0xE0E0E0E0u) ^ 0x80808080u; }
__device__ __forceinline__ uint32_t q3_hi(uint32_t w) { return ((w << 1) & 0xE0E0E0E0u) ^ 0x80808080u; }

// signed byte J (compile-time) of a packed word
template <int J>
__device__ __forceinline__ int sbyte_of(uint32_t w) {
    return (int)(int8_t)(uint8_t)(w >> (8 * J));
}

// byte j (compile-time) of a packed word, zero-extended
template <int J>
__device__ __forceinline__ int byte_of(uint32_t w) {
    return (int)__byte_perm(w, 0u, 0x4440u + J);
}

// FMT kI8Q4K: Q4_K; kI8Q3K: Q3_K in the expanded device layout (m16n8k16
// per 16-element sub-block, no min term); kI8Q40: Q4_0 (one m16n8k32 per
// 32-element block, its f16 scale applied in f32, the -8 offset through the
// block sums)
template <int FMT>
__global__ void __launch_bounds__(kI8Threads, 1) mm_i8_kernel(const I8Params p) {
    constexpr bool Q3 = FMT == kI8Q3K, Q40 = FMT == kI8Q40;
    extern __shared__ __align__(128) uint8_t smem[];
    float* red = reinterpret_cast<float*>(smem + p.red_off);
    uint8_t* ring = smem + p.ring_off;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(smem), empty0 = full0 + 8 * 16;
    // K-split: this CTA's row group and K-range (super-blocks kb0 .. kb0 + nsb)
    const int ksi = blockIdx.x % p.ks, rgi = blockIdx.x / p.ks, nrg = gridDim.x / p.ks;
    const int kb0 = ksi * p.nsb;
    asm volatile("griddepcontrol.launch_dependents;");
    if (warp == 0) {
        if (lane < p.nstage) {
            mbar_init(full0 + 8 * lane, 1);
            mbar_init(empty0 + 8 * lane, kI8Cons);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int it = 0, slot = 0, use = 0;
            bool ok = true;
            for (int j = 0; j < p.njobs && ok; j++) {
                const I8Job& jb = p.jobs[j];
                int64_t rb;
                int nrows;
                i8_rows(jb, rgi, nrg, &rb, &nrows);
                for (int r0 = 0; r0 < nrows; r0 += p.RS, it++, slot = slot + 1 == p.nstage ? 0 : slot + 1,
                         use += slot == 0) {
                    if (use > 0 && !mbar_wait(empty0 + 8 * slot, (use - 1) & 1)) { ok = false; break; }
                    const int rows = min(p.RS, nrows - r0);
                    const uint32_t dst = smem_u32(ring) + (uint32_t)slot * p.stage_bytes;
                    const uint32_t hdst = dst + (uint32_t)p.RS * p.qstride;
                    mbar_expect_tx(full0 + 8 * slot, (uint32_t)rows * (p.qseg + p.hseg));
                    for (int r = 0; r < rows; r++) {
                        const int64_t row = rb + r0 + r;
                        bulk_g2s(dst + (uint32_t)r * p.qstride, jb.qs + row * p.qrow + (int64_t)kb0 * 128, p.qseg,
                                 full0 + 8 * slot, pol);
                        bulk_g2s(hdst + (uint32_t)r * p.hstride, jb.hdr + row * p.hrow + (int64_t)kb0 * p.hsb, p.hseg,
                                 full0 + 8 * slot, pol);
                    }
                }
            }
            for (int k = max(0, it - p.nstage); k < it; k++)
                if (!mbar_wait(full0 + 8 * (k % p.nstage), (k / p.nstage) & 1)) ok = false;
            if (!ok && p.err) atomicExch(p.err, 1);
        }
    } else {
        const int w = warp - 1;                 // K-slice
        const int g = lane >> 2, t = lane & 3;  // MMA group / quad position
        const int M = p.M;
        const int sb0 = w * p.nsb / kI8Cons, nsbw = (w + 1) * p.nsb / kI8Cons - sb0;
        asm volatile("griddepcontrol.wait;" ::: "memory");
        // B fragments of the slice: column g = plane g / 2 of token g % 2
        // (columns 6, 7 zero), elements 8t .. 8t+7 of each 32-element
        // sub-block (Q3_K: elements 4t .. 4t+3 and 16+4t .. 16+4t+3, the
        // k16 fragments of its two 16-element sub-blocks)
        uint32_t bf[kI8MaxSB][8][2];
        float coef[kI8MaxSB][2];  // sx * plane weight of columns 2t, 2t+1: plane t, tokens 0, 1
        {
            const int bp = g >> 1, bm = g & 1;
            const bool bvalid = bp < 3 && bm < M;
            const int8_t* bsrc =
                p.xq.planes + ((int64_t)bm * 3 + (bvalid ? bp : 0)) * p.in + (Q3 || Q40 ? 4 : 8) * t;
#pragma unroll
            for (int s = 0; s < kI8MaxSB; s++)
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    uint2 u = make_uint2(0u, 0u);
                    if (bvalid && s < nsbw) {
                        const int8_t* src = bsrc + ((int64_t)(kb0 + sb0 + s) * 8 + j) * 32;
                        if constexpr (Q3 || Q40)
                            u = make_uint2(*reinterpret_cast<const uint32_t*>(src),
                                           *reinterpret_cast<const uint32_t*>(src + 16));
                        else
                            u = *reinterpret_cast<const uint2*>(src);
                    }
                    bf[s][j][0] = u.x;
                    bf[s][j][1] = u.y;
                }
            // Q3_K: A carries 32 (q - 4), folded in here (exact)
            const float pw = (t == 0 ? 65536.0f : t == 1 ? 256.0f : 1.0f) * (Q3 ? 0.03125f : 1.0f);
#pragma unroll
            for (int s = 0; s < kI8MaxSB; s++)
#pragma unroll
                for (int c = 0; c < 2; c++)
                    coef[s][c] =
                        (t < 3 && c < M && s < nsbw) ? p.xq.sx[(int64_t)c * p.nsbr + kb0 + sb0 + s] * pw : 0.0f;
        }
        // block sums of this lane's token (t < M) over the slice, for the min term
        const bool tvalid = !Q3 && t < M;
        float bs[kI8MaxSB][8];
        {
            const float* bsum_t = p.xq.bsum + (int64_t)(tvalid ? t : 0) * (p.in / 32);
#pragma unroll
            for (int s = 0; s < kI8MaxSB; s++) {
                float4 b0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), b1 = b0;
                if (tvalid && s < nsbw) {
                    b0 = *reinterpret_cast<const float4*>(bsum_t + (int64_t)(kb0 + sb0 + s) * 8);
                    b1 = *reinterpret_cast<const float4*>(bsum_t + (int64_t)(kb0 + sb0 + s) * 8 + 4);
                }
                const float k8 = Q40 ? 8.0f : 1.0f;  // Q4_0: w = d (q - 8), the 8 folded in (exact)
                bs[s][0] = b0.x * k8; bs[s][1] = b0.y * k8; bs[s][2] = b0.z * k8; bs[s][3] = b0.w * k8;
                bs[s][4] = b1.x * k8; bs[s][5] = b1.y * k8; bs[s][6] = b1.z * k8; bs[s][7] = b1.w * k8;
            }
        }
        int slot = 0, use = 0, roff = 0;
        bool ok = true;
        for (int j = 0; j < p.njobs && ok; j++) {
            const I8Job& jb = p.jobs[j];
            int64_t rb;
            int nrows;
            i8_rows(jb, rgi, nrg, &rb, &nrows);
            for (int r0 = 0; r0 < nrows; r0 += p.RS, slot = slot + 1 == p.nstage ? 0 : slot + 1, use += slot == 0) {
                if (!mbar_wait(full0 + 8 * slot, use & 1)) {
                    if (lane == 0 && p.err) atomicExch(p.err, 1);
                    ok = false;
                    break;
                }
                const uint8_t* sq = ring + (size_t)slot * p.stage_bytes;
                const uint8_t* sh = sq + (size_t)p.RS * p.qstride;
                const int rows = min(p.RS, nrows - r0);
                // MMA rows past the stage's rows read its last row (results dropped)
                const int rA = min(g, rows - 1), rB = min(g + 8, rows - 1);
                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // rows g, g (cols 2t, 2t+1), g+8, g+8
                float mn[2] = {0.0f, 0.0f};               // min term of token t, rows g and g+8
#pragma unroll
                for (int s = 0; s < kI8MaxSB; s++) {
                    if (s < nsbw) {
                        const int sb = sb0 + s;
                        if constexpr (Q3) {
                            // 16 int8 scales (word c: sub-blocks 4c .. 4c+3), then d
                            const uint32_t* hg4 =
                                reinterpret_cast<const uint32_t*>(sh + (size_t)rA * p.hstride + sb * 20);
                            const uint32_t* h84 =
                                reinterpret_cast<const uint32_t*>(sh + (size_t)rB * p.hstride + sb * 20);
                            int ai[4] = {0, 0, 0, 0};
                            const uint8_t* qg = sq + (size_t)rA * p.qstride + sb * 128 + 4 * t;
                            const uint8_t* q8 = sq + (size_t)rB * p.qstride + sb * 128 + 4 * t;
#pragma unroll
                            for (int c = 0; c < 4; c++) {
                                // bytes 4t.. of the group's two 16-byte halves: low
                                // nibbles = sub-blocks 4c, 4c+1, high = 4c+2, 4c+3
                                const uint32_t wg0 = *reinterpret_cast<const uint32_t*>(qg + 32 * c);
                                const uint32_t wg1 = *reinterpret_cast<const uint32_t*>(qg + 32 * c + 16);
                                const uint32_t w80 = *reinterpret_cast<const uint32_t*>(q8 + 32 * c);
                                const uint32_t w81 = *reinterpret_cast<const uint32_t*>(q8 + 32 * c + 16);
                                const uint32_t scg = hg4[c], sc8 = h84[c];
                                int d[4];
                                mma_s8s8_k16(d, q3_lo(wg0), q3_lo(w80), bf[s][2 * c][0]);
                                ai[0] += d[0] * sbyte_of<0>(scg); ai[1] += d[1] * sbyte_of<0>(scg);
                                ai[2] += d[2] * sbyte_of<0>(sc8); ai[3] += d[3] * sbyte_of<0>(sc8);
                                mma_s8s8_k16(d, q3_lo(wg1), q3_lo(w81), bf[s][2 * c][1]);
                                ai[0] += d[0] * sbyte_of<1>(scg); ai[1] += d[1] * sbyte_of<1>(scg);
                                ai[2] += d[2] * sbyte_of<1>(sc8); ai[3] += d[3] * sbyte_of<1>(sc8);
                                mma_s8s8_k16(d, q3_hi(wg0), q3_hi(w80), bf[s][2 * c + 1][0]);
                                ai[0] += d[0] * sbyte_of<2>(scg); ai[1] += d[1] * sbyte_of<2>(scg);
                                ai[2] += d[2] * sbyte_of<2>(sc8); ai[3] += d[3] * sbyte_of<2>(sc8);
                                mma_s8s8_k16(d, q3_hi(wg1), q3_hi(w81), bf[s][2 * c + 1][1]);
                                ai[0] += d[0] * sbyte_of<3>(scg); ai[1] += d[1] * sbyte_of<3>(scg);
                                ai[2] += d[2] * sbyte_of<3>(sc8); ai[3] += d[3] * sbyte_of<3>(sc8);
                            }
                            const float dg = __half2float(*reinterpret_cast<const __half*>(hg4 + 4));
                            const float d8 = __half2float(*reinterpret_cast<const __half*>(h84 + 4));
                            acc[0] = fmaf((float)ai[0], dg * coef[s][0], acc[0]);
                            acc[1] = fmaf((float)ai[1], dg * coef[s][1], acc[1]);
                            acc[2] = fmaf((float)ai[2], d8 * coef[s][0], acc[2]);
                            acc[3] = fmaf((float)ai[3], d8 * coef[s][1], acc[3]);
                        } else if constexpr (Q40) {
                            // eight 32-element blocks: 16 quant bytes and an f16 d each
                            const uint4 hg = *reinterpret_cast<const uint4*>(sh + (size_t)rA * p.hstride + sb * 16);
                            const uint4 h8 = *reinterpret_cast<const uint4*>(sh + (size_t)rB * p.hstride + sb * 16);
                            const uint32_t dgw[4] = {hg.x, hg.y, hg.z, hg.w}, d8w[4] = {h8.x, h8.y, h8.z, h8.w};
                            const uint8_t* qg = sq + (size_t)rA * p.qstride + sb * 128 + 4 * t;
                            const uint8_t* q8 = sq + (size_t)rB * p.qstride + sb * 128 + 4 * t;
#pragma unroll
                            for (int j = 0; j < 8; j++) {
                                // bytes 4t..4t+3 of block j: low nibbles = elements
                                // 4t.., high nibbles = 16+4t.. (K slots as the B
                                // fragments)
                                const uint32_t wg = *reinterpret_cast<const uint32_t*>(qg + 16 * j);
                                const uint32_t w8 = *reinterpret_cast<const uint32_t*>(q8 + 16 * j);
                                const uint32_t a[4] = {wg & 0x0F0F0F0Fu, w8 & 0x0F0F0F0Fu, (wg >> 4) & 0x0F0F0F0Fu,
                                                       (w8 >> 4) & 0x0F0F0F0Fu};
                                int d[4];
                                mma_u8s8(d, a, bf[s][j][0], bf[s][j][1]);
                                const float2 dgp = __half22float2(*reinterpret_cast<const __half2*>(&dgw[j >> 1]));
                                const float2 d8p = __half22float2(*reinterpret_cast<const __half2*>(&d8w[j >> 1]));
                                const float dg = (j & 1) ? dgp.y : dgp.x, d8 = (j & 1) ? d8p.y : d8p.x;
                                acc[0] = fmaf(i2f_small(d[0]), dg * coef[s][0], acc[0]);
                                acc[1] = fmaf(i2f_small(d[1]), dg * coef[s][1], acc[1]);
                                acc[2] = fmaf(i2f_small(d[2]), d8 * coef[s][0], acc[2]);
                                acc[3] = fmaf(i2f_small(d[3]), d8 * coef[s][1], acc[3]);
                                mn[0] = fmaf(dg, bs[s][j], mn[0]);
                                mn[1] = fmaf(d8, bs[s][j], mn[1]);
                            }
                        } else {
                            const uint4 hg = *reinterpret_cast<const uint4*>(sh + (size_t)rA * p.hstride + sb * 16);
                            const uint4 h8 = *reinterpret_cast<const uint4*>(sh + (size_t)rB * p.hstride + sb * 16);
                            // Q4_K 6-bit scales and mins, four per word
                            const uint32_t scg0 = hg.y & 0x3F3F3F3Fu, mg0 = hg.z & 0x3F3F3F3Fu;
                            const uint32_t scg1 = (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u);
                            const uint32_t mg1 = ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u);
                            const uint32_t sc80 = h8.y & 0x3F3F3F3Fu, m80 = h8.z & 0x3F3F3F3Fu;
                            const uint32_t sc81 = (h8.w & 0x0F0F0F0Fu) | ((h8.y >> 2) & 0x30303030u);
                            const uint32_t m81 = ((h8.w >> 4) & 0x0F0F0F0Fu) | ((h8.z >> 2) & 0x30303030u);
                            int ai[4] = {0, 0, 0, 0};
                            const uint8_t* qg = sq + (size_t)rA * p.qstride + sb * 128 + 8 * t;
                            const uint8_t* q8 = sq + (size_t)rB * p.qstride + sb * 128 + 8 * t;
    #pragma unroll
                            for (int c = 0; c < 4; c++) {
                                const uint2 wg = *reinterpret_cast<const uint2*>(qg + 32 * c);
                                const uint2 w8 = *reinterpret_cast<const uint2*>(q8 + 32 * c);
                                const uint32_t alo[4] = {wg.x & 0x0F0F0F0Fu, w8.x & 0x0F0F0F0Fu, wg.y & 0x0F0F0F0Fu,
                                                         w8.y & 0x0F0F0F0Fu};
                                const uint32_t ahi[4] = {(wg.x >> 4) & 0x0F0F0F0Fu, (w8.x >> 4) & 0x0F0F0F0Fu,
                                                         (wg.y >> 4) & 0x0F0F0F0Fu, (w8.y >> 4) & 0x0F0F0F0Fu};
                                int d[4];
                                // sub-block 2c
                                mma_u8s8(d, alo, bf[s][2 * c][0], bf[s][2 * c][1]);
                                {
                                    const int sg = c < 2 ? (c == 0 ? byte_of<0>(scg0) : byte_of<2>(scg0))
                                                         : (c == 2 ? byte_of<0>(scg1) : byte_of<2>(scg1));
                                    const int s8 = c < 2 ? (c == 0 ? byte_of<0>(sc80) : byte_of<2>(sc80))
                                                         : (c == 2 ? byte_of<0>(sc81) : byte_of<2>(sc81));
                                    ai[0] += d[0] * sg;
                                    ai[1] += d[1] * sg;
                                    ai[2] += d[2] * s8;
                                    ai[3] += d[3] * s8;
                                }
                                // sub-block 2c + 1
                                mma_u8s8(d, ahi, bf[s][2 * c + 1][0], bf[s][2 * c + 1][1]);
                                {
                                    const int sg = c < 2 ? (c == 0 ? byte_of<1>(scg0) : byte_of<3>(scg0))
                                                         : (c == 2 ? byte_of<1>(scg1) : byte_of<3>(scg1));
                                    const int s8 = c < 2 ? (c == 0 ? byte_of<1>(sc80) : byte_of<3>(sc80))
                                                         : (c == 2 ? byte_of<1>(sc81) : byte_of<3>(sc81));
                                    ai[0] += d[0] * sg;
                                    ai[1] += d[1] * sg;
                                    ai[2] += d[2] * s8;
                                    ai[3] += d[3] * s8;
                                }
                            }
                            const float2 ddg = __half22float2(*reinterpret_cast<const __half2*>(&hg.x));
                            const float2 dd8 = __half22float2(*reinterpret_cast<const __half2*>(&h8.x));
                            acc[0] = fmaf((float)ai[0], ddg.x * coef[s][0], acc[0]);
                            acc[1] = fmaf((float)ai[1], ddg.x * coef[s][1], acc[1]);
                            acc[2] = fmaf((float)ai[2], dd8.x * coef[s][0], acc[2]);
                            acc[3] = fmaf((float)ai[3], dd8.x * coef[s][1], acc[3]);
                            {
                                // m_j as exact floats: byte j of the packed mins under
                                // the exponent of 2^23, minus 2^23 (no conversion unit)
                                float sg = 0.0f, s8 = 0.0f;
    #pragma unroll
                                for (int jj = 0; jj < 8; jj++) {
                                    const uint32_t wg = jj < 4 ? mg0 : mg1, w8 = jj < 4 ? m80 : m81;
                                    const float fg =
                                        __uint_as_float(__byte_perm(wg, 0x4B000000u, 0x7650u + (jj & 3))) - 8388608.0f;
                                    const float f8 =
                                        __uint_as_float(__byte_perm(w8, 0x4B000000u, 0x7650u + (jj & 3))) - 8388608.0f;
                                    sg = fmaf(fg, bs[s][jj], sg);
                                    s8 = fmaf(f8, bs[s][jj], s8);
                                }
                                mn[0] = fmaf(ddg.y, sg, mn[0]);
                                mn[1] = fmaf(dd8.y, s8, mn[1]);
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * slot);
                // the three planes of a token sit in lanes t = 0, 1, 2 of
                // the quad (lane 3 holds zeros): sum over the quad
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
                    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);
                }
                const int qb = lane & ~3;
                const float mA0 = __shfl_sync(0xffffffffu, mn[0], qb);
                const float mA1 = __shfl_sync(0xffffffffu, mn[0], qb + 1);
                const float mB0 = __shfl_sync(0xffffffffu, mn[1], qb);
                const float mB1 = __shfl_sync(0xffffffffu, mn[1], qb + 1);
                if (t == 0) {
                    float* rg = red + ((int64_t)(roff + r0 + g) * kI8Cons + w) * M;
                    float* r8 = red + ((int64_t)(roff + r0 + g + 8) * kI8Cons + w) * M;
                    if (g < rows) {
                        rg[0] = acc[0] - mA0;
                        if (M > 1) rg[1] = acc[1] - mA1;
                    }
                    if (g + 8 < rows) {
                        r8[0] = acc[2] - mB0;
                        if (M > 1) r8[1] = acc[3] - mB1;
                    }
                }
            }
            roff += nrows;
        }
    }
    __syncthreads();
    int roff = 0;
    for (int j = 0; j < p.njobs; j++) {
        int64_t rb;
        int nrows;
        i8_rows(p.jobs[j], rgi, nrg, &rb, &nrows);
        for (int e = threadIdx.x; e < nrows * p.M; e += blockDim.x) {
            const int r = e / p.M, m = e % p.M;
            float acc = 0.0f;
            for (int s = 0; s < kI8Cons; s++) acc += red[((int64_t)(roff + r) * kI8Cons + s) * p.M + m];
            const int64_t o = (int64_t)m * p.jobs[j].out + rb + r;
            if (p.ks > 1)
                p.part[(int64_t)ksi * p.M * p.jobs[j].out + o] = acc;
            else
                p.jobs[j].y[o] = p.jobs[j].add ? acc + p.jobs[j].add[o] : acc;
        }
        roff += nrows;
    }
    if (p.ks > 1) {
        __shared__ int s_last;
        i8_ksplit_finish(p, rgi, nrg, threadIdx.x, blockDim.x, 0, &s_last);
    }
}


// TMEM loads / stores of 8 and 16 32-bit columns (32x32b: lane i of the
// warp's lane quarter, one column per register)
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st8u(uint32_t taddr, const uint32_t* v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16p(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16p(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// ------------------------------------------------- three or four tokens
//
// The same data path and A operand; B has 12 columns, n = 4 p + m (plane p
// of token m), in two column groups of 8 (two MMAs per sub-block).  The 12
// activation rows are copied into shared memory once per CTA (a row per
// column, padded by 32 bytes: conflict-free 8-byte fragment loads) instead
// of registers.  The eight K-slice partials of a stage's rows are summed in
// slice order through a small double-buffered table after a barrier of the
// consumer warps, and y is written per stage.  A consumer that times out on
// a stage raises a shared abort flag and every warp then skips the rest of
// the work but still passes every barrier, so no barrier waits on a warp
// that left.
template <int FMT>
__global__ void __launch_bounds__(kI8Threads, 1) mm_i8x4_kernel(const I8Params p) {
    constexpr bool Q3 = FMT == kI8Q3K, Q40 = FMT == kI8Q40;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem + p.ring_off;
    float* pr = reinterpret_cast<float*>(smem + p.pr_off);
    __shared__ int s_abort;
    __shared__ uint32_t s_tmem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(smem), empty0 = full0 + 8 * 16;
    // K-split: this CTA's row group and K-range (super-blocks kb0 .. kb0 + nsb)
    const int ksi = blockIdx.x % p.ks, rgi = blockIdx.x / p.ks, nrg = gridDim.x / p.ks;
    const int kb0 = ksi * p.nsb;
    asm volatile("griddepcontrol.launch_dependents;");
    if (warp == 0) {
        if (lane < p.nstage) {
            mbar_init(full0 + 8 * lane, 1);
            mbar_init(empty0 + 8 * lane, kI8Cons);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x == 0) s_abort = 0;
    if (warp == 1) {  // the B fragments live in TMEM: 256 columns, freed by this warp at the end
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(256u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc::tmem_fence_before();
    __syncthreads();
    tc::tmem_fence_after();

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int it = 0, slot = 0, use = 0;
            bool ok = true;
            for (int j = 0; j < p.njobs && ok; j++) {
                const I8Job& jb = p.jobs[j];
                int64_t rb;
                int nrows;
                i8_rows(jb, rgi, nrg, &rb, &nrows);
                for (int r0 = 0; r0 < nrows; r0 += p.RS, it++, slot = slot + 1 == p.nstage ? 0 : slot + 1,
                         use += slot == 0) {
                    if (use > 0 && !mbar_wait(empty0 + 8 * slot, (use - 1) & 1)) { ok = false; break; }
                    const int rows = min(p.RS, nrows - r0);
                    const uint32_t dst = smem_u32(ring) + (uint32_t)slot * p.stage_bytes;
                    const uint32_t hdst = dst + (uint32_t)p.RS * p.qstride;
                    mbar_expect_tx(full0 + 8 * slot, (uint32_t)rows * (p.qseg + p.hseg));
                    for (int r = 0; r < rows; r++) {
                        const int64_t row = rb + r0 + r;
                        bulk_g2s(dst + (uint32_t)r * p.qstride, jb.qs + row * p.qrow + (int64_t)kb0 * 128, p.qseg,
                                 full0 + 8 * slot, pol);
                        bulk_g2s(hdst + (uint32_t)r * p.hstride, jb.hdr + row * p.hrow + (int64_t)kb0 * p.hsb, p.hseg,
                                 full0 + 8 * slot, pol);
                    }
                }
            }
            for (int k = max(0, it - p.nstage); k < it; k++)
                if (!mbar_wait(full0 + 8 * (k % p.nstage), (k / p.nstage) & 1)) ok = false;
            if (!ok && p.err) atomicExch(p.err, 1);
        }
        return;
    }
    const int w = warp - 1, ct = threadIdx.x - 32;
    const int g = lane >> 2, t = lane & 3;
    const int M = p.M;
    const int sb0 = w * p.nsb / kI8Cons, nsbw = (w + 1) * p.nsb / kI8Cons - sb0;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // B fragment columns of this lane: n0 = g and n1 = 8 + g, column n = 4 pl + m
    // the XQ2 row 3 m + pl (n1 only for pl = 2; absent tokens are zeros)
    const int n0 = g, n1 = 8 + g;
    const bool v0 = (n0 & 3) < M, v1 = (n1 >> 2) < 3 && (n1 & 3) < M;
    // This warp's TMEM lanes (32 (warp % 4) ..) and columns (warps 5..8
    // the second 128): per super-block s of the K-slice, 32 columns = for
    // each 32-element sub-block the lane's two B words of column n0, then of
    // n1 (Q4_K: bytes 8t .. 8t+7; Q3_K / Q4_0: bytes 4t .. 4t+3 of each
    // 16-element half).  Filled once, read back per super-block with two
    // tcgen05.ld of 16 columns, so the ring gets the shared memory.
    const uint32_t tb = s_tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (warp >= 5 ? 128u : 0u);
    {
        constexpr int lo_off = (Q3 || Q40) ? 4 : 8;
        const int8_t* src0 =
            p.xq.planes + (int64_t)(v0 ? 3 * (n0 & 3) + (n0 >> 2) : 0) * p.in + (int64_t)kb0 * 256 + lo_off * t;
        const int8_t* src1 =
            p.xq.planes + (int64_t)(v1 ? 3 * (n1 & 3) + (n1 >> 2) : 0) * p.in + (int64_t)kb0 * 256 + lo_off * t;
#pragma unroll
        for (int s = 0; s < kI8MaxSB; s++) {
            if (s < nsbw) {  // warp-uniform: tcgen05.st is warp-wide
                uint32_t v[32];
#pragma unroll
                for (int sub = 0; sub < 8; sub++) {
                    const int64_t ko = (int64_t)((sb0 + s) * 8 + sub) * 32;
                    uint2 b0 = make_uint2(0u, 0u), b1 = make_uint2(0u, 0u);
                    if constexpr (Q3 || Q40) {
                        if (v0)
                            b0 = make_uint2(*reinterpret_cast<const uint32_t*>(src0 + ko),
                                            *reinterpret_cast<const uint32_t*>(src0 + ko + 16));
                        if (v1)
                            b1 = make_uint2(*reinterpret_cast<const uint32_t*>(src1 + ko),
                                            *reinterpret_cast<const uint32_t*>(src1 + ko + 16));
                    } else {
                        if (v0) b0 = *reinterpret_cast<const uint2*>(src0 + ko);
                        if (v1) b1 = *reinterpret_cast<const uint2*>(src1 + ko);
                    }
                    v[4 * sub] = b0.x;
                    v[4 * sub + 1] = b0.y;
                    v[4 * sub + 2] = b1.x;
                    v[4 * sub + 3] = b1.y;
                }
                tc::tmem_st32u(tb + 32u * (uint32_t)s, v);
            }
        }
        tc::tmem_wait_st();
    }
    // the f32 factors of this lane's C columns (sx * plane weight, zero for
    // absent tokens) and its token's block sums are read per super-block
    // (L1-resident) to keep registers for the MMA tiles
    const int na0 = 2 * t, nb0 = 8 + 2 * t;  // first C column of the two groups
    // plane weights; Q3_K's A carries 32 (q - 4): 1/32 folded in (exact)
    const float pwa = ((na0 >> 2) == 0 ? 65536.0f : 256.0f) * (Q3 ? 0.03125f : 1.0f);
    const float pwb = Q3 ? 0.03125f : 1.0f;
    const bool ca0 = (na0 & 3) < M, ca1 = ((na0 + 1) & 3) < M;
    const bool cb0 = (nb0 >> 2) < 3 && (nb0 & 3) < M, cb1 = ((nb0 + 1) >> 2) < 3 && ((nb0 + 1) & 3) < M;
    const float* sxa0 = p.xq.sx + (int64_t)(ca0 ? (na0 & 3) : 0) * p.nsbr + kb0;
    const float* sxa1 = p.xq.sx + (int64_t)(ca1 ? ((na0 + 1) & 3) : 0) * p.nsbr + kb0;
    const float* sxb0 = p.xq.sx + (int64_t)(cb0 ? (nb0 & 3) : 0) * p.nsbr + kb0;
    const float* sxb1 = p.xq.sx + (int64_t)(cb1 ? ((nb0 + 1) & 3) : 0) * p.nsbr + kb0;
    const bool tvalid = !Q3 && t < M;
    const float* bsum_t = p.xq.bsum + (int64_t)(tvalid ? t : 0) * (p.in / 32) + (int64_t)kb0 * 8;
    int slot = 0, use = 0, par = 0;
    for (int j = 0; j < p.njobs; j++) {
        const I8Job& jb = p.jobs[j];
        int64_t rb;
        int nrows;
        i8_rows(jb, rgi, nrg, &rb, &nrows);
        for (int r0 = 0; r0 < nrows; r0 += p.RS, slot = slot + 1 == p.nstage ? 0 : slot + 1, use += slot == 0,
                 par ^= 1) {
            if (!*(volatile int*)&s_abort && !mbar_wait(full0 + 8 * slot, use & 1)) {
                if (lane == 0 && p.err) atomicExch(p.err, 1);
                *(volatile int*)&s_abort = 1;
            }
            const bool live = __all_sync(0xffffffffu, !*(volatile int*)&s_abort);  // warp-uniform
            const uint8_t* sq = ring + (size_t)slot * p.stage_bytes;
            const uint8_t* sh = sq + (size_t)p.RS * p.qstride;
            const int rows = min(p.RS, nrows - r0);
            const int rA = min(g, rows - 1), rB = min(g + 8, rows - 1);
            float acc0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, acc1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            float mn[2] = {0.0f, 0.0f};
#pragma unroll
            for (int s = 0; s < kI8MaxSB; s++) {
                if (live && s < nsbw) {
                    const int sb = sb0 + s;
                    // B words of the super-block's eight sub-blocks (TMEM): both halves
                    // requested before one wait, so one load latency per super-block
                    uint32_t bq[32];
                    const float cf0 = ca0 ? __ldg(sxa0 + sb) * pwa : 0.0f, cf1 = ca1 ? __ldg(sxa1 + sb) * pwa : 0.0f;
                    const float cg0 = cb0 ? __ldg(sxb0 + sb) * pwb : 0.0f, cg1 = cb1 ? __ldg(sxb1 + sb) * pwb : 0.0f;
                    if constexpr (Q3) {
                        const uint32_t* hg4 =
                            reinterpret_cast<const uint32_t*>(sh + (size_t)rA * p.hstride + sb * 20);
                        const uint32_t* h84 =
                            reinterpret_cast<const uint32_t*>(sh + (size_t)rB * p.hstride + sb * 20);
                        int a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
                        const uint8_t* qg = sq + (size_t)rA * p.qstride + sb * 128 + 4 * t;
                        const uint8_t* q8 = sq + (size_t)rB * p.qstride + sb * 128 + 4 * t;
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const uint32_t wq[4] = {*reinterpret_cast<const uint32_t*>(qg + 32 * c),
                                                    *reinterpret_cast<const uint32_t*>(qg + 32 * c + 16),
                                                    *reinterpret_cast<const uint32_t*>(q8 + 32 * c),
                                                    *reinterpret_cast<const uint32_t*>(q8 + 32 * c + 16)};
                            const uint32_t scg = hg4[c], sc8 = h84[c];
                            if (c == 0) {
                                tmem_ld16p(tb + 32u * (uint32_t)s, bq);
                                tmem_ld16p(tb + 32u * (uint32_t)s + 16u, bq + 16);
                                tc::tmem_wait_ld();
                            }
                            const uint32_t* bh = bq + 16 * (c >> 1);  // chunks 2c .. 2c+3
#pragma unroll
                            for (int q = 0; q < 4; q++) {
                                // sub-block 4c + q: low (q < 2) or high nibbles of
                                // half q & 1; its elements are half q & 1 of
                                // 32-element chunk 2c + q / 2
                                const uint32_t ag = q < 2 ? q3_lo(wq[q & 1]) : q3_hi(wq[q & 1]);
                                const uint32_t a8 = q < 2 ? q3_lo(wq[2 + (q & 1)]) : q3_hi(wq[2 + (q & 1)]);
                                const int cj = (2 * c + (q >> 1)) & 3;  // chunk within the loaded half
                                const uint32_t b0 = bh[4 * cj + (q & 1)], b1 = bh[4 * cj + 2 + (q & 1)];
                                int d0[4], d1[4];
                                mma_s8s8_k16(d0, ag, a8, b0);
                                mma_s8s8_k16(d1, ag, a8, b1);
                                const int sg = (int)(int8_t)(uint8_t)(scg >> (8 * q));
                                const int s8 = (int)(int8_t)(uint8_t)(sc8 >> (8 * q));
                                a0[0] += d0[0] * sg; a0[1] += d0[1] * sg; a0[2] += d0[2] * s8; a0[3] += d0[3] * s8;
                                a1[0] += d1[0] * sg; a1[1] += d1[1] * sg; a1[2] += d1[2] * s8; a1[3] += d1[3] * s8;
                            }
                        }
                        const float dg = __half2float(*reinterpret_cast<const __half*>(hg4 + 4));
                        const float d8 = __half2float(*reinterpret_cast<const __half*>(h84 + 4));
                        acc0[0] = fmaf((float)a0[0], dg * cf0, acc0[0]);
                        acc0[1] = fmaf((float)a0[1], dg * cf1, acc0[1]);
                        acc0[2] = fmaf((float)a0[2], d8 * cf0, acc0[2]);
                        acc0[3] = fmaf((float)a0[3], d8 * cf1, acc0[3]);
                        acc1[0] = fmaf((float)a1[0], dg * cg0, acc1[0]);
                        acc1[1] = fmaf((float)a1[1], dg * cg1, acc1[1]);
                        acc1[2] = fmaf((float)a1[2], d8 * cg0, acc1[2]);
                        acc1[3] = fmaf((float)a1[3], d8 * cg1, acc1[3]);
                    } else if constexpr (Q40) {
                        float bsv[8];
                        {
                            float4 bsa = make_float4(0.0f, 0.0f, 0.0f, 0.0f), bsb = bsa;
                            if (tvalid) {
                                bsa = __ldg(reinterpret_cast<const float4*>(bsum_t + (int64_t)sb * 8));
                                bsb = __ldg(reinterpret_cast<const float4*>(bsum_t + (int64_t)sb * 8 + 4));
                            }
                            bsv[0] = bsa.x; bsv[1] = bsa.y; bsv[2] = bsa.z; bsv[3] = bsa.w;
                            bsv[4] = bsb.x; bsv[5] = bsb.y; bsv[6] = bsb.z; bsv[7] = bsb.w;
                        }
                        const uint4 hg = *reinterpret_cast<const uint4*>(sh + (size_t)rA * p.hstride + sb * 16);
                        const uint4 h8 = *reinterpret_cast<const uint4*>(sh + (size_t)rB * p.hstride + sb * 16);
                        const uint32_t dgw[4] = {hg.x, hg.y, hg.z, hg.w}, d8w[4] = {h8.x, h8.y, h8.z, h8.w};
                        const uint8_t* qg = sq + (size_t)rA * p.qstride + sb * 128 + 4 * t;
                        const uint8_t* q8 = sq + (size_t)rB * p.qstride + sb * 128 + 4 * t;
                        float sgm = 0.0f, s8m = 0.0f;
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const uint32_t wg = *reinterpret_cast<const uint32_t*>(qg + 16 * j);
                            const uint32_t w8 = *reinterpret_cast<const uint32_t*>(q8 + 16 * j);
                            const uint32_t a[4] = {wg & 0x0F0F0F0Fu, w8 & 0x0F0F0F0Fu, (wg >> 4) & 0x0F0F0F0Fu,
                                                   (w8 >> 4) & 0x0F0F0F0Fu};
                            if (j == 0) {
                                tmem_ld16p(tb + 32u * (uint32_t)s, bq);
                                tmem_ld16p(tb + 32u * (uint32_t)s + 16u, bq + 16);
                                tc::tmem_wait_ld();
                            }
                            const uint32_t b00 = bq[4 * j], b01 = bq[4 * j + 1];
                            const uint32_t b10 = bq[4 * j + 2], b11 = bq[4 * j + 3];
                            int d0[4], d1[4];
                            mma_u8s8(d0, a, b00, b01);
                            mma_u8s8(d1, a, b10, b11);
                            const float2 dgp = __half22float2(*reinterpret_cast<const __half2*>(&dgw[j >> 1]));
                            const float2 d8p = __half22float2(*reinterpret_cast<const __half2*>(&d8w[j >> 1]));
                            const float dg = (j & 1) ? dgp.y : dgp.x, d8 = (j & 1) ? d8p.y : d8p.x;
                            acc0[0] = fmaf(i2f_small(d0[0]), dg * cf0, acc0[0]);
                            acc0[1] = fmaf(i2f_small(d0[1]), dg * cf1, acc0[1]);
                            acc0[2] = fmaf(i2f_small(d0[2]), d8 * cf0, acc0[2]);
                            acc0[3] = fmaf(i2f_small(d0[3]), d8 * cf1, acc0[3]);
                            acc1[0] = fmaf(i2f_small(d1[0]), dg * cg0, acc1[0]);
                            acc1[1] = fmaf(i2f_small(d1[1]), dg * cg1, acc1[1]);
                            acc1[2] = fmaf(i2f_small(d1[2]), d8 * cg0, acc1[2]);
                            acc1[3] = fmaf(i2f_small(d1[3]), d8 * cg1, acc1[3]);
                            sgm = fmaf(dg, bsv[j], sgm);
                            s8m = fmaf(d8, bsv[j], s8m);
                        }
                        // Q4_0: w = d (q - 8)
                        mn[0] = fmaf(8.0f, sgm, mn[0]);
                        mn[1] = fmaf(8.0f, s8m, mn[1]);
                    } else {
                        float4 bsa = make_float4(0.0f, 0.0f, 0.0f, 0.0f), bsb = bsa;
                        if (tvalid) {
                            bsa = __ldg(reinterpret_cast<const float4*>(bsum_t + (int64_t)sb * 8));
                            bsb = __ldg(reinterpret_cast<const float4*>(bsum_t + (int64_t)sb * 8 + 4));
                        }
                        const float bsv[8] = {bsa.x, bsa.y, bsa.z, bsa.w, bsb.x, bsb.y, bsb.z, bsb.w};
                        const uint4 hg = *reinterpret_cast<const uint4*>(sh + (size_t)rA * p.hstride + sb * 16);
                        const uint4 h8 = *reinterpret_cast<const uint4*>(sh + (size_t)rB * p.hstride + sb * 16);
                        const uint32_t scg0 = hg.y & 0x3F3F3F3Fu, mg0 = hg.z & 0x3F3F3F3Fu;
                        const uint32_t scg1 = (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u);
                        const uint32_t mg1 = ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u);
                        const uint32_t sc80 = h8.y & 0x3F3F3F3Fu, m80 = h8.z & 0x3F3F3F3Fu;
                        const uint32_t sc81 = (h8.w & 0x0F0F0F0Fu) | ((h8.y >> 2) & 0x30303030u);
                        const uint32_t m81 = ((h8.w >> 4) & 0x0F0F0F0Fu) | ((h8.z >> 2) & 0x30303030u);
                        int a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
                        const uint8_t* qg = sq + (size_t)rA * p.qstride + sb * 128 + 8 * t;
                        const uint8_t* q8 = sq + (size_t)rB * p.qstride + sb * 128 + 8 * t;
    #pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const uint2 wg = *reinterpret_cast<const uint2*>(qg + 32 * c);
                            const uint2 w8 = *reinterpret_cast<const uint2*>(q8 + 32 * c);
                            if (c == 0) {
                                tmem_ld16p(tb + 32u * (uint32_t)s, bq);
                                tmem_ld16p(tb + 32u * (uint32_t)s + 16u, bq + 16);
                                tc::tmem_wait_ld();
                            }
                            const uint32_t* bh = bq + 16 * (c >> 1);  // sub-blocks 2c .. 2c+3
                            const uint32_t alo[4] = {wg.x & 0x0F0F0F0Fu, w8.x & 0x0F0F0F0Fu, wg.y & 0x0F0F0F0Fu,
                                                     w8.y & 0x0F0F0F0Fu};
                            const uint32_t ahi[4] = {(wg.x >> 4) & 0x0F0F0F0Fu, (w8.x >> 4) & 0x0F0F0F0Fu,
                                                     (wg.y >> 4) & 0x0F0F0F0Fu, (w8.y >> 4) & 0x0F0F0F0Fu};
    #pragma unroll
                            for (int h = 0; h < 2; h++) {
                                const int sub = (2 * c + h) & 3;  // within the loaded half
                                const uint2 b0 = make_uint2(bh[4 * sub], bh[4 * sub + 1]);
                                const uint2 b1 = make_uint2(bh[4 * sub + 2], bh[4 * sub + 3]);
                                int d0[4], d1[4];
                                if (h == 0) {
                                    mma_u8s8(d0, alo, b0.x, b0.y);
                                    mma_u8s8(d1, alo, b1.x, b1.y);
                                } else {
                                    mma_u8s8(d0, ahi, b0.x, b0.y);
                                    mma_u8s8(d1, ahi, b1.x, b1.y);
                                }
                                const uint32_t wgs = c < 2 ? scg0 : scg1, w8s = c < 2 ? sc80 : sc81;
                                const int byte = (2 * c + h) & 3;
                                const int sg = (int)__byte_perm(wgs, 0u, 0x4440u + byte);
                                const int s8 = (int)__byte_perm(w8s, 0u, 0x4440u + byte);
                                a0[0] += d0[0] * sg; a0[1] += d0[1] * sg; a0[2] += d0[2] * s8; a0[3] += d0[3] * s8;
                                a1[0] += d1[0] * sg; a1[1] += d1[1] * sg; a1[2] += d1[2] * s8; a1[3] += d1[3] * s8;
                            }
                        }
                        const float2 ddg = __half22float2(*reinterpret_cast<const __half2*>(&hg.x));
                        const float2 dd8 = __half22float2(*reinterpret_cast<const __half2*>(&h8.x));
                        acc0[0] = fmaf((float)a0[0], ddg.x * cf0, acc0[0]);
                        acc0[1] = fmaf((float)a0[1], ddg.x * cf1, acc0[1]);
                        acc0[2] = fmaf((float)a0[2], dd8.x * cf0, acc0[2]);
                        acc0[3] = fmaf((float)a0[3], dd8.x * cf1, acc0[3]);
                        acc1[0] = fmaf((float)a1[0], ddg.x * cg0, acc1[0]);
                        acc1[1] = fmaf((float)a1[1], ddg.x * cg1, acc1[1]);
                        acc1[2] = fmaf((float)a1[2], dd8.x * cg0, acc1[2]);
                        acc1[3] = fmaf((float)a1[3], dd8.x * cg1, acc1[3]);
                        float sgm = 0.0f, s8m = 0.0f;
    #pragma unroll
                        for (int jj = 0; jj < 8; jj++) {
                            const uint32_t wg = jj < 4 ? mg0 : mg1, w8 = jj < 4 ? m80 : m81;
                            const float fg =
                                __uint_as_float(__byte_perm(wg, 0x4B000000u, 0x7650u + (jj & 3))) - 8388608.0f;
                            const float f8 =
                                __uint_as_float(__byte_perm(w8, 0x4B000000u, 0x7650u + (jj & 3))) - 8388608.0f;
                            sgm = fmaf(fg, bsv[jj], sgm);
                            s8m = fmaf(f8, bsv[jj], s8m);
                        }
                        mn[0] = fmaf(ddg.y, sgm, mn[0]);
                        mn[1] = fmaf(dd8.y, s8m, mn[1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * slot);
            // token 2t + c (t < 2): plane 0 in acc0 here, plane 1 in acc0 of
            // lane t + 2, plane 2 in acc1 here
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = acc0[i] + __shfl_xor_sync(0xffffffffu, acc0[i], 2) + acc1[i];
            const int qb = lane & ~3;
            const float mA0 = __shfl_sync(0xffffffffu, mn[0], qb + ((2 * t) & 3));
            const float mA1 = __shfl_sync(0xffffffffu, mn[0], qb + ((2 * t + 1) & 3));
            const float mB0 = __shfl_sync(0xffffffffu, mn[1], qb + ((2 * t) & 3));
            const float mB1 = __shfl_sync(0xffffffffu, mn[1], qb + ((2 * t + 1) & 3));
            float* buf = pr + par * (kI8Rows * kI8Cons * 4);
            if (t < 2) {
                const int m0 = 2 * t, m1 = 2 * t + 1;
                if (g < rows) {
                    buf[(g * kI8Cons + w) * 4 + m0] = v[0] - mA0;
                    buf[(g * kI8Cons + w) * 4 + m1] = v[1] - mA1;
                }
                if (g + 8 < rows) {
                    buf[((g + 8) * kI8Cons + w) * 4 + m0] = v[2] - mB0;
                    buf[((g + 8) * kI8Cons + w) * 4 + m1] = v[3] - mB1;
                }
            }
            named_bar_sync(1, 32 * kI8Cons);
            if (ct < rows * M && !*(volatile int*)&s_abort) {
                const int r = ct / M, m = ct % M;
                float acc = 0.0f;
                for (int s = 0; s < kI8Cons; s++) acc += buf[(r * kI8Cons + s) * 4 + m];
                const int64_t o = (int64_t)m * jb.out + rb + r0 + r;
                if (p.ks > 1)
                    p.part[(int64_t)ksi * M * jb.out + o] = acc;
                else
                    jb.y[o] = jb.add ? acc + jb.add[o] : acc;
            }
        }
    }
    if (p.ks > 1) {
        __shared__ int s_last;
        i8_ksplit_finish(p, rgi, nrg, ct, 32 * kI8Cons, 1, &s_last);
    }
    // every consumer's TMEM reads have completed (each was waited for)
    tc::tmem_fence_before();
    named_bar_sync(1, 32 * kI8Cons);
    tc::tmem_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(s_tmem), "r"(256u) : "memory");
}


// ------------------------------------------------- five to eight tokens
//
// The same data path and A operand; B has 24 columns in three column groups
// of 8, group p = activation plane p, column m = token m (absent tokens are
// zeros), so every sub-block takes three MMAs and a lane's C columns 2t,
// 2t+1 are tokens 2t, 2t+1 of every plane.  The lane's B words (per
// 32-element sub-block: two words for each of the three groups) live in
// TMEM: 512 columns, 256 per warp of a lane quarter, 64 per super-block
// (two halves of four sub-blocks, 24 words each, at 32-column offsets),
// filled once and read back with one 16- and one 8-column tcgen05.ld per
// half super-block.  The eight K-slice partials of a stage's rows are summed
// in slice order through a double-buffered table [row][slice][token] after
// a barrier of the consumer warps, and y is written per stage.

constexpr int kI8x8Cols = 512;  // TMEM columns of the eight-token form

template <int FMT>
__global__ void __launch_bounds__(kI8Threads, 1) mm_i8x8_kernel(const I8Params p) {
    constexpr bool Q3 = FMT == kI8Q3K, Q40 = FMT == kI8Q40;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem + p.ring_off;
    float* pr = reinterpret_cast<float*>(smem + p.pr_off);  // [2][kI8Rows][kI8Cons][8]
    __shared__ int s_abort;
    __shared__ uint32_t s_tmem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(smem), empty0 = full0 + 8 * 16;
    const int ksi = blockIdx.x % p.ks, rgi = blockIdx.x / p.ks, nrg = gridDim.x / p.ks;
    const int kb0 = ksi * p.nsb;
    asm volatile("griddepcontrol.launch_dependents;");
    if (warp == 0) {
        if (lane < p.nstage) {
            mbar_init(full0 + 8 * lane, 1);
            mbar_init(empty0 + 8 * lane, kI8Cons);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x == 0) s_abort = 0;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"((uint32_t)kI8x8Cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc::tmem_fence_before();
    __syncthreads();
    tc::tmem_fence_after();

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int it = 0, slot = 0, use = 0;
            bool ok = true;
            for (int j = 0; j < p.njobs && ok; j++) {
                const I8Job& jb = p.jobs[j];
                int64_t rb;
                int nrows;
                i8_rows(jb, rgi, nrg, &rb, &nrows);
                for (int r0 = 0; r0 < nrows; r0 += p.RS, it++, slot = slot + 1 == p.nstage ? 0 : slot + 1,
                         use += slot == 0) {
                    if (use > 0 && !mbar_wait(empty0 + 8 * slot, (use - 1) & 1)) { ok = false; break; }
                    const int rows = min(p.RS, nrows - r0);
                    const uint32_t dst = smem_u32(ring) + (uint32_t)slot * p.stage_bytes;
                    const uint32_t hdst = dst + (uint32_t)p.RS * p.qstride;
                    mbar_expect_tx(full0 + 8 * slot, (uint32_t)rows * (p.qseg + p.hseg));
                    for (int r = 0; r < rows; r++) {
                        const int64_t row = rb + r0 + r;
                        bulk_g2s(dst + (uint32_t)r * p.qstride, jb.qs + row * p.qrow + (int64_t)kb0 * 128, p.qseg,
                                 full0 + 8 * slot, pol);
                        bulk_g2s(hdst + (uint32_t)r * p.hstride, jb.hdr + row * p.hrow + (int64_t)kb0 * p.hsb, p.hseg,
                                 full0 + 8 * slot, pol);
                    }
                }
            }
            for (int k = max(0, it - p.nstage); k < it; k++)
                if (!mbar_wait(full0 + 8 * (k % p.nstage), (k / p.nstage) & 1)) ok = false;
            if (!ok && p.err) atomicExch(p.err, 1);
        }
        return;
    }
    const int w = warp - 1, ct = threadIdx.x - 32;
    const int g = lane >> 2, t = lane & 3;
    const int M = p.M;
    const int sb0 = w * p.nsb / kI8Cons, nsbw = (w + 1) * p.nsb / kI8Cons - sb0;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // B column g of group pl: token g of plane pl, XQ2 row 3 g + pl
    const bool vb = g < M;
    const uint32_t tb = s_tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (warp >= 5 ? 256u : 0u);
    {
        constexpr int lo_off = (Q3 || Q40) ? 4 : 8;
        const int8_t* src = p.xq.planes + (int64_t)(vb ? 3 * g : 0) * p.in + (int64_t)kb0 * 256 + lo_off * t;
#pragma unroll
        for (int s = 0; s < kI8MaxSB; s++) {
            if (s < nsbw) {  // warp-uniform: tcgen05.st is warp-wide
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    uint32_t v[24];
#pragma unroll
                    for (int sq = 0; sq < 4; sq++) {
                        const int sub = 4 * hf + sq;
                        const int64_t ko = (int64_t)((sb0 + s) * 8 + sub) * 32;
#pragma unroll
                        for (int pl = 0; pl < 3; pl++) {
                            uint2 b = make_uint2(0u, 0u);
                            if (vb) {
                                const int8_t* sp = src + (int64_t)pl * p.in + ko;
                                if constexpr (Q3 || Q40)
                                    b = make_uint2(*reinterpret_cast<const uint32_t*>(sp),
                                                   *reinterpret_cast<const uint32_t*>(sp + 16));
                                else
                                    b = *reinterpret_cast<const uint2*>(sp);
                            }
                            v[6 * sq + 2 * pl] = b.x;
                            v[6 * sq + 2 * pl + 1] = b.y;
                        }
                    }
                    const uint32_t col = tb + 64u * (uint32_t)s + 32u * (uint32_t)hf;
                    tmem_st16p(col, v);
                    tmem_st8u(col + 16u, v + 16);
                }
            }
        }
        tc::tmem_wait_st();
    }
    // f32 factors of this lane's C columns: token 2t + c of plane pl ->
    // sx[token][sb] * plane weight (zero for absent tokens), read per
    // super-block; Q3_K's A carries 32 (q - 4), folded in (exact)
    const float kq = Q3 ? 0.03125f : 1.0f;
    const float pw[3] = {65536.0f * kq, 256.0f * kq, 1.0f * kq};
    const bool tv0 = 2 * t < M, tv1 = 2 * t + 1 < M;
    const float* sx0 = p.xq.sx + (int64_t)(tv0 ? 2 * t : 0) * p.nsbr + kb0;
    const float* sx1 = p.xq.sx + (int64_t)(tv1 ? 2 * t + 1 : 0) * p.nsbr + kb0;
    const float* bs0 = p.xq.bsum + (int64_t)(tv0 ? 2 * t : 0) * (p.in / 32) + (int64_t)kb0 * 8;
    const float* bs1 = p.xq.bsum + (int64_t)(tv1 ? 2 * t + 1 : 0) * (p.in / 32) + (int64_t)kb0 * 8;
    int slot = 0, use = 0, par = 0;
    for (int j = 0; j < p.njobs; j++) {
        const I8Job& jb = p.jobs[j];
        int64_t rb;
        int nrows;
        i8_rows(jb, rgi, nrg, &rb, &nrows);
        for (int r0 = 0; r0 < nrows; r0 += p.RS, slot = slot + 1 == p.nstage ? 0 : slot + 1, use += slot == 0,
                 par ^= 1) {
            if (!*(volatile int*)&s_abort && !mbar_wait(full0 + 8 * slot, use & 1)) {
                if (lane == 0 && p.err) atomicExch(p.err, 1);
                *(volatile int*)&s_abort = 1;
            }
            const bool live = __all_sync(0xffffffffu, !*(volatile int*)&s_abort);  // warp-uniform
            const uint8_t* sq = ring + (size_t)slot * p.stage_bytes;
            const uint8_t* sh = sq + (size_t)p.RS * p.qstride;
            const int rows = min(p.RS, nrows - r0);
            const int rA = min(g, rows - 1), rB = min(g + 8, rows - 1);
            float acc[3][4];
#pragma unroll
            for (int pl = 0; pl < 3; pl++)
#pragma unroll
                for (int i = 0; i < 4; i++) acc[pl][i] = 0.0f;
            float mn[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};  // min / offset term: [row g, g+8][token 2t + c]
#pragma unroll
            for (int s = 0; s < kI8MaxSB; s++) {
                if (live && s < nsbw) {
                    const int sb = sb0 + s;
                    const float x0 = tv0 ? __ldg(sx0 + sb) : 0.0f, x1 = tv1 ? __ldg(sx1 + sb) : 0.0f;
                    float cf[3][2];
#pragma unroll
                    for (int pl = 0; pl < 3; pl++) {
                        cf[pl][0] = x0 * pw[pl];
                        cf[pl][1] = x1 * pw[pl];
                    }
                    const uint32_t colb = tb + 64u * (uint32_t)s;
                    // B words of the eight sub-blocks, [half][sub][plane][word]: both
                    // halves requested before one wait
                    uint32_t bq[48];
                    int a[3][4];
#pragma unroll
                    for (int pl = 0; pl < 3; pl++)
#pragma unroll
                        for (int i = 0; i < 4; i++) a[pl][i] = 0;
                    if constexpr (Q3) {
                        const uint32_t* hg4 =
                            reinterpret_cast<const uint32_t*>(sh + (size_t)rA * p.hstride + sb * 20);
                        const uint32_t* h84 =
                            reinterpret_cast<const uint32_t*>(sh + (size_t)rB * p.hstride + sb * 20);
                        const uint8_t* qg = sq + (size_t)rA * p.qstride + sb * 128 + 4 * t;
                        const uint8_t* q8 = sq + (size_t)rB * p.qstride + sb * 128 + 4 * t;
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const uint32_t wq[4] = {*reinterpret_cast<const uint32_t*>(qg + 32 * c),
                                                    *reinterpret_cast<const uint32_t*>(qg + 32 * c + 16),
                                                    *reinterpret_cast<const uint32_t*>(q8 + 32 * c),
                                                    *reinterpret_cast<const uint32_t*>(q8 + 32 * c + 16)};
                            const uint32_t scg = hg4[c], sc8 = h84[c];
                            if (c == 0) {
                                tmem_ld16p(colb, bq);
                                tmem_ld8(colb + 16u, bq + 16);
                                tmem_ld16p(colb + 32u, bq + 24);
                                tmem_ld8(colb + 48u, bq + 40);
                                tc::tmem_wait_ld();
                            }
                            const uint32_t* bh = bq + 24 * (c >> 1);  // chunks 2c .. 2c+3
#pragma unroll
                            for (int q = 0; q < 4; q++) {
                                const uint32_t ag = q < 2 ? q3_lo(wq[q & 1]) : q3_hi(wq[q & 1]);
                                const uint32_t a8 = q < 2 ? q3_lo(wq[2 + (q & 1)]) : q3_hi(wq[2 + (q & 1)]);
                                const int cj = (2 * c + (q >> 1)) & 3;
                                const int sg = (int)(int8_t)(uint8_t)(scg >> (8 * q));
                                const int s8 = (int)(int8_t)(uint8_t)(sc8 >> (8 * q));
#pragma unroll
                                for (int pl = 0; pl < 3; pl++) {
                                    int d[4];
                                    mma_s8s8_k16(d, ag, a8, bh[6 * cj + 2 * pl + (q & 1)]);
                                    a[pl][0] += d[0] * sg; a[pl][1] += d[1] * sg;
                                    a[pl][2] += d[2] * s8; a[pl][3] += d[3] * s8;
                                }
                            }
                        }
                        const float dg = __half2float(*reinterpret_cast<const __half*>(hg4 + 4));
                        const float d8 = __half2float(*reinterpret_cast<const __half*>(h84 + 4));
#pragma unroll
                        for (int pl = 0; pl < 3; pl++) {
                            acc[pl][0] = fmaf((float)a[pl][0], dg * cf[pl][0], acc[pl][0]);
                            acc[pl][1] = fmaf((float)a[pl][1], dg * cf[pl][1], acc[pl][1]);
                            acc[pl][2] = fmaf((float)a[pl][2], d8 * cf[pl][0], acc[pl][2]);
                            acc[pl][3] = fmaf((float)a[pl][3], d8 * cf[pl][1], acc[pl][3]);
                        }
                    } else if constexpr (Q40) {
                        const uint4 hg = *reinterpret_cast<const uint4*>(sh + (size_t)rA * p.hstride + sb * 16);
                        const uint4 h8 = *reinterpret_cast<const uint4*>(sh + (size_t)rB * p.hstride + sb * 16);
                        const uint32_t dgw[4] = {hg.x, hg.y, hg.z, hg.w}, d8w[4] = {h8.x, h8.y, h8.z, h8.w};
                        const uint8_t* qg = sq + (size_t)rA * p.qstride + sb * 128 + 4 * t;
                        const uint8_t* q8 = sq + (size_t)rB * p.qstride + sb * 128 + 4 * t;
#pragma unroll
                        for (int jb8 = 0; jb8 < 8; jb8++) {
                            const uint32_t wg = *reinterpret_cast<const uint32_t*>(qg + 16 * jb8);
                            const uint32_t w8 = *reinterpret_cast<const uint32_t*>(q8 + 16 * jb8);
                            const uint32_t am[4] = {wg & 0x0F0F0F0Fu, w8 & 0x0F0F0F0Fu, (wg >> 4) & 0x0F0F0F0Fu,
                                                    (w8 >> 4) & 0x0F0F0F0Fu};
                            if (jb8 == 0) {
                                tmem_ld16p(colb, bq);
                                tmem_ld8(colb + 16u, bq + 16);
                                tmem_ld16p(colb + 32u, bq + 24);
                                tmem_ld8(colb + 48u, bq + 40);
                                tc::tmem_wait_ld();
                            }
                            const float2 dgp = __half22float2(*reinterpret_cast<const __half2*>(&dgw[jb8 >> 1]));
                            const float2 d8p = __half22float2(*reinterpret_cast<const __half2*>(&d8w[jb8 >> 1]));
                            const float dg = (jb8 & 1) ? dgp.y : dgp.x, d8 = (jb8 & 1) ? d8p.y : d8p.x;
                            const uint32_t* bh = bq + 24 * (jb8 >> 2);
                            const int jj = jb8 & 3;
#pragma unroll
                            for (int pl = 0; pl < 3; pl++) {
                                int d[4];
                                mma_u8s8(d, am, bh[6 * jj + 2 * pl], bh[6 * jj + 2 * pl + 1]);
                                acc[pl][0] = fmaf(i2f_small(d[0]), dg * cf[pl][0], acc[pl][0]);
                                acc[pl][1] = fmaf(i2f_small(d[1]), dg * cf[pl][1], acc[pl][1]);
                                acc[pl][2] = fmaf(i2f_small(d[2]), d8 * cf[pl][0], acc[pl][2]);
                                acc[pl][3] = fmaf(i2f_small(d[3]), d8 * cf[pl][1], acc[pl][3]);
                            }
                            // Q4_0: w = d (q - 8), the offset through the block sums
                            const float b0v = tv0 ? __ldg(bs0 + (int64_t)sb * 8 + jb8) : 0.0f;
                            const float b1v = tv1 ? __ldg(bs1 + (int64_t)sb * 8 + jb8) : 0.0f;
                            mn[0][0] = fmaf(8.0f * dg, b0v, mn[0][0]);
                            mn[0][1] = fmaf(8.0f * dg, b1v, mn[0][1]);
                            mn[1][0] = fmaf(8.0f * d8, b0v, mn[1][0]);
                            mn[1][1] = fmaf(8.0f * d8, b1v, mn[1][1]);
                        }
                    } else {
                        const uint4 hg = *reinterpret_cast<const uint4*>(sh + (size_t)rA * p.hstride + sb * 16);
                        const uint4 h8 = *reinterpret_cast<const uint4*>(sh + (size_t)rB * p.hstride + sb * 16);
                        const uint32_t scg0 = hg.y & 0x3F3F3F3Fu, mg0 = hg.z & 0x3F3F3F3Fu;
                        const uint32_t scg1 = (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u);
                        const uint32_t mg1 = ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u);
                        const uint32_t sc80 = h8.y & 0x3F3F3F3Fu, m80 = h8.z & 0x3F3F3F3Fu;
                        const uint32_t sc81 = (h8.w & 0x0F0F0F0Fu) | ((h8.y >> 2) & 0x30303030u);
                        const uint32_t m81 = ((h8.w >> 4) & 0x0F0F0F0Fu) | ((h8.z >> 2) & 0x30303030u);
                        const uint8_t* qg = sq + (size_t)rA * p.qstride + sb * 128 + 8 * t;
                        const uint8_t* q8 = sq + (size_t)rB * p.qstride + sb * 128 + 8 * t;
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const uint2 wg = *reinterpret_cast<const uint2*>(qg + 32 * c);
                            const uint2 w8 = *reinterpret_cast<const uint2*>(q8 + 32 * c);
                            if (c == 0) {
                                tmem_ld16p(colb, bq);
                                tmem_ld8(colb + 16u, bq + 16);
                                tmem_ld16p(colb + 32u, bq + 24);
                                tmem_ld8(colb + 48u, bq + 40);
                                tc::tmem_wait_ld();
                            }
                            const uint32_t* bh = bq + 24 * (c >> 1);  // sub-blocks 2c .. 2c+3
                            const uint32_t alo[4] = {wg.x & 0x0F0F0F0Fu, w8.x & 0x0F0F0F0Fu, wg.y & 0x0F0F0F0Fu,
                                                     w8.y & 0x0F0F0F0Fu};
                            const uint32_t ahi[4] = {(wg.x >> 4) & 0x0F0F0F0Fu, (w8.x >> 4) & 0x0F0F0F0Fu,
                                                     (wg.y >> 4) & 0x0F0F0F0Fu, (w8.y >> 4) & 0x0F0F0F0Fu};
#pragma unroll
                            for (int h = 0; h < 2; h++) {
                                const int sub = (2 * c + h) & 3;  // within the loaded half
                                const uint32_t wgs = c < 2 ? scg0 : scg1, w8s = c < 2 ? sc80 : sc81;
                                const int byte = (2 * c + h) & 3;
                                const int sg = (int)__byte_perm(wgs, 0u, 0x4440u + byte);
                                const int s8 = (int)__byte_perm(w8s, 0u, 0x4440u + byte);
#pragma unroll
                                for (int pl = 0; pl < 3; pl++) {
                                    int d[4];
                                    if (h == 0)
                                        mma_u8s8(d, alo, bh[6 * sub + 2 * pl], bh[6 * sub + 2 * pl + 1]);
                                    else
                                        mma_u8s8(d, ahi, bh[6 * sub + 2 * pl], bh[6 * sub + 2 * pl + 1]);
                                    a[pl][0] += d[0] * sg; a[pl][1] += d[1] * sg;
                                    a[pl][2] += d[2] * s8; a[pl][3] += d[3] * s8;
                                }
                            }
                        }
                        const float2 ddg = __half22float2(*reinterpret_cast<const __half2*>(&hg.x));
                        const float2 dd8 = __half22float2(*reinterpret_cast<const __half2*>(&h8.x));
#pragma unroll
                        for (int pl = 0; pl < 3; pl++) {
                            acc[pl][0] = fmaf((float)a[pl][0], ddg.x * cf[pl][0], acc[pl][0]);
                            acc[pl][1] = fmaf((float)a[pl][1], ddg.x * cf[pl][1], acc[pl][1]);
                            acc[pl][2] = fmaf((float)a[pl][2], dd8.x * cf[pl][0], acc[pl][2]);
                            acc[pl][3] = fmaf((float)a[pl][3], dd8.x * cf[pl][1], acc[pl][3]);
                        }
                        // min term of tokens 2t, 2t+1: dmin * sum_j m_j bsum_j
                        float4 b0a = make_float4(0.0f, 0.0f, 0.0f, 0.0f), b0b = b0a, b1a = b0a, b1b = b0a;
                        if (tv0) {
                            b0a = __ldg(reinterpret_cast<const float4*>(bs0 + (int64_t)sb * 8));
                            b0b = __ldg(reinterpret_cast<const float4*>(bs0 + (int64_t)sb * 8 + 4));
                        }
                        if (tv1) {
                            b1a = __ldg(reinterpret_cast<const float4*>(bs1 + (int64_t)sb * 8));
                            b1b = __ldg(reinterpret_cast<const float4*>(bs1 + (int64_t)sb * 8 + 4));
                        }
                        const float bv0[8] = {b0a.x, b0a.y, b0a.z, b0a.w, b0b.x, b0b.y, b0b.z, b0b.w};
                        const float bv1[8] = {b1a.x, b1a.y, b1a.z, b1a.w, b1b.x, b1b.y, b1b.z, b1b.w};
                        float sg0 = 0.0f, sg1 = 0.0f, s80 = 0.0f, s81 = 0.0f;
#pragma unroll
                        for (int jj = 0; jj < 8; jj++) {
                            const uint32_t mw = jj < 4 ? mg0 : mg1, mw8 = jj < 4 ? m80 : m81;
                            const float fg =
                                __uint_as_float(__byte_perm(mw, 0x4B000000u, 0x7650u + (jj & 3))) - 8388608.0f;
                            const float f8 =
                                __uint_as_float(__byte_perm(mw8, 0x4B000000u, 0x7650u + (jj & 3))) - 8388608.0f;
                            sg0 = fmaf(fg, bv0[jj], sg0);
                            sg1 = fmaf(fg, bv1[jj], sg1);
                            s80 = fmaf(f8, bv0[jj], s80);
                            s81 = fmaf(f8, bv1[jj], s81);
                        }
                        mn[0][0] = fmaf(ddg.y, sg0, mn[0][0]);
                        mn[0][1] = fmaf(ddg.y, sg1, mn[0][1]);
                        mn[1][0] = fmaf(dd8.y, s80, mn[1][0]);
                        mn[1][1] = fmaf(dd8.y, s81, mn[1][1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * slot);
            // tokens 2t, 2t+1 of rows g, g+8: the three planes summed
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = acc[0][i] + acc[1][i] + acc[2][i];
            float* buf = pr + par * (kI8Rows * kI8Cons * 8);
            if (g < rows) {
                if (tv0) buf[(g * kI8Cons + w) * 8 + 2 * t] = v[0] - mn[0][0];
                if (tv1) buf[(g * kI8Cons + w) * 8 + 2 * t + 1] = v[1] - mn[0][1];
            }
            if (g + 8 < rows) {
                if (tv0) buf[((g + 8) * kI8Cons + w) * 8 + 2 * t] = v[2] - mn[1][0];
                if (tv1) buf[((g + 8) * kI8Cons + w) * 8 + 2 * t + 1] = v[3] - mn[1][1];
            }
            named_bar_sync(1, 32 * kI8Cons);
            if (ct < rows * M && !*(volatile int*)&s_abort) {
                const int r = ct / M, m = ct % M;
                float sum = 0.0f;
                for (int s = 0; s < kI8Cons; s++) sum += buf[(r * kI8Cons + s) * 8 + m];
                const int64_t o = (int64_t)m * jb.out + rb + r0 + r;
                if (p.ks > 1)
                    p.part[(int64_t)ksi * M * jb.out + o] = sum;
                else
                    jb.y[o] = jb.add ? sum + jb.add[o] : sum;
            }
        }
    }
    if (p.ks > 1) {
        __shared__ int s_last;
        i8_ksplit_finish(p, rgi, nrg, ct, 32 * kI8Cons, 1, &s_last);
    }
    tc::tmem_fence_before();
    named_bar_sync(1, 32 * kI8Cons);
    tc::tmem_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(s_tmem), "r"((uint32_t)kI8x8Cols)
                     : "memory");
}

}  // namespace

// K-splits for a row of nsb super-blocks: 1 when each of the 8 K-slice warps
// gets at most 4 super-blocks, else 4 (each CTA of a row group a quarter)
static int i8_ksplits(int64_t nsb) { return nsb <= (int64_t)kI8Cons * kI8MaxSB ? 1 : 4; }

bool mm_i8_supported(const rq_weight* w, int64_t M) {
    if ((w->type != RQ_Q4_K && w->type != RQ_Q3_K && w->type != RQ_Q4_0) || M < 2 || M > 8 || w->in % 256)
        return false;
    const int64_t nsb = w->in / 256;
    const int ks = i8_ksplits(nsb);
    if (nsb % ks) return false;
    const int64_t per = nsb / ks;
    // Q3_K's 20-byte headers: a K-range's header bytes are whole 16-byte
    // units (bulk copies) when it spans a multiple of 4 super-blocks
    if (w->type == RQ_Q3_K && per % 4) return false;
    // whole K-slices per warp when not split; split ranges up to 4 per warp
    return ks == 1 ? (per % kI8Cons == 0 && per / kI8Cons <= kI8MaxSB) : per <= (int64_t)kI8Cons * kI8MaxSB;
}

size_t mm_i8_scratch_floats(const rq_weight* w, int64_t M) {
    return i8_ksplits(w->in / 256) > 1 ? (size_t)4 * (size_t)M * (size_t)w->out : 0;
}

int launch_xq2_stage(const float* x, int64_t M, int64_t in, XQ2 q, cudaStream_t st, const float* rms_w,
                     float eps, const float* up) {
    if (M == 0 || in < 256) return RQ_OK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((in / 256 + 7) / 8), (unsigned)M);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_error(cudaLaunchKernelEx(&cfg, xq2_stage_kernel, x, in, q, rms_w, eps, up), "xq2 staging kernel");
}

int launch_mm_i8(const rq_weight* const* ws, float* const* ys, int njobs, int64_t M, XQ2 xq, int sm_count,
                 cudaStream_t st, int* err, const float* const* adds, float* part, int* cnt) {
    if (njobs < 1 || njobs > kMaxJobs) return set_error(RQ_ERR_INVALID, "int8 matmul: %d jobs", njobs);
    const rq_weight* w0 = ws[0];
    for (int j = 0; j < njobs; j++)
        if (!mm_i8_supported(ws[j], M) || ws[j]->in != w0->in || ws[j]->type != w0->type)
            return set_error(RQ_ERR_INVALID, "int8 matmul: unsupported weight or M = %lld", (long long)M);
    I8Params p;
    memset(&p, 0, sizeof p);
    p.njobs = njobs;
    p.M = (int)M;
    p.in = w0->in;
    p.nsbr = (int)(w0->in / 256);
    p.ks = i8_ksplits(p.nsbr);
    if (p.ks > 1 && (njobs != 1 || !part || !cnt))
        return set_error(RQ_ERR_INVALID, "int8 matmul: a split K needs one job and scratch");
    p.nsb = p.nsbr / p.ks;
    p.part = part;
    p.cnt = cnt;
    // per 256 elements: 128 quant bytes (Q4_0: 8 blocks of 16) and 16
    // header bytes (Q4_0: 8 f16 scales; Q3_K: 20)
    p.hsb = w0->type == RQ_Q3_K ? 20u : 16u;
    p.qrow = (uint32_t)(p.nsbr * 128);
    p.hrow = (uint32_t)(p.nsbr * p.hsb);
    p.qseg = (uint32_t)(p.nsb * 128);
    p.hseg = (uint32_t)(p.nsb * p.hsb);
    p.qstride = p.qseg + kI8QPad;
    p.hstride = p.hseg + kI8HPad;
    const uint32_t rowb = p.qstride + p.hstride;
    p.xq = xq;
    p.err = err;
    int64_t max_out = 0;
    for (int j = 0; j < njobs; j++) {
        p.jobs[j] = I8Job{ws[j]->qs, ws[j]->hdr, ys[j], adds ? adds[j] : nullptr, ws[j]->out};
        max_out = std::max(max_out, ws[j]->out);
    }
    // row groups x K-splits CTAs (a multiple of ks)
    const int nrg = (int)std::min<int64_t>(max_out, sm_count / p.ks);
    const int grid = nrg * p.ks;
    if (p.ks > 1 && nrg > kI8MaxRowGroups) return set_error(RQ_ERR_UNSUPPORTED, "int8 matmul: %d row groups", nrg);
    int64_t rows_cap = 0;
    for (int j = 0; j < njobs; j++) rows_cap += (ws[j]->out + nrg - 1) / nrg;
    // three to eight tokens: activations in TMEM, per-stage sums through a
    // partial table [2][rows][slices][4 or 8 tokens] ahead of the ring
    const bool x4 = M > 2, x8 = M > 4;
    if (x4) {
        p.pr_off = kI8Bar;
        p.ring_off = (uint32_t)((p.pr_off + 2 * kI8Rows * kI8Cons * (x8 ? 8 : 4) * 4 + 127) & ~127u);
    } else {
        const int64_t red_bytes = rows_cap * kI8Cons * M * 4;
        p.red_off = kI8Bar;
        p.ring_off = (uint32_t)((kI8Bar + red_bytes + 127) & ~(int64_t)127);
    }
    if (p.ring_off >= (uint32_t)kI8Smem) return set_error(RQ_ERR_UNSUPPORTED, "int8 matmul: partial table too large");
    // rows per stage: the most (<= 16) that leave three stages in flight,
    // else two stages of 16
    const int64_t room = kI8Smem - (int64_t)p.ring_off;
    int RS = (int)std::min<int64_t>(kI8Rows, room / (3 * (int64_t)rowb));
    if (RS < 12) RS = (int)std::min<int64_t>(kI8Rows, room / (2 * (int64_t)rowb));
    if (RS < 1) return set_error(RQ_ERR_UNSUPPORTED, "int8 matmul: rows of %u bytes too large", p.qrow + p.hrow);
    p.RS = RS;
    p.stage_bytes = ((uint32_t)RS * rowb + 127) & ~127u;
    const int nstage = std::min<int>((int)(room / p.stage_bytes), 16);
    if (nstage < 2) return set_error(RQ_ERR_UNSUPPORTED, "int8 matmul: rows of %u bytes too large", p.qrow + p.hrow);
    p.nstage = nstage;
    const size_t smem = p.ring_off + (size_t)nstage * p.stage_bytes;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaSuccess;
        const void* kerns[9] = {(const void*)mm_i8_kernel<kI8Q4K>,   (const void*)mm_i8_kernel<kI8Q3K>,
                                (const void*)mm_i8_kernel<kI8Q40>,   (const void*)mm_i8x4_kernel<kI8Q4K>,
                                (const void*)mm_i8x4_kernel<kI8Q3K>, (const void*)mm_i8x4_kernel<kI8Q40>,
                                (const void*)mm_i8x8_kernel<kI8Q4K>, (const void*)mm_i8x8_kernel<kI8Q3K>,
                                (const void*)mm_i8x8_kernel<kI8Q40>};
        for (int k = 0; k < 9 && e == cudaSuccess; k++)
            e = cudaFuncSetAttribute(kerns[k], cudaFuncAttributeMaxDynamicSharedMemorySize, kI8Smem);
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(int8 matmul)");
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kI8Threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (w0->type == RQ_Q3_K)
        e = x8 ? cudaLaunchKernelEx(&cfg, mm_i8x8_kernel<kI8Q3K>, p)
               : x4 ? cudaLaunchKernelEx(&cfg, mm_i8x4_kernel<kI8Q3K>, p)
                    : cudaLaunchKernelEx(&cfg, mm_i8_kernel<kI8Q3K>, p);
    else if (w0->type == RQ_Q4_0)
        e = x8 ? cudaLaunchKernelEx(&cfg, mm_i8x8_kernel<kI8Q40>, p)
               : x4 ? cudaLaunchKernelEx(&cfg, mm_i8x4_kernel<kI8Q40>, p)
                    : cudaLaunchKernelEx(&cfg, mm_i8_kernel<kI8Q40>, p);
    else
        e = x8 ? cudaLaunchKernelEx(&cfg, mm_i8x8_kernel<kI8Q4K>, p)
               : x4 ? cudaLaunchKernelEx(&cfg, mm_i8x4_kernel<kI8Q4K>, p)
                    : cudaLaunchKernelEx(&cfg, mm_i8_kernel<kI8Q4K>, p);
    return cuda_error(e, "int8 matmul kernel");
}

}  // namespace rq
