// rq_mm_small.cu -- Q4_K matmul for small batches (up to 8 activation rows
// per job) on the tensor cores: mma.sync m16n8k16, f16 x f16 -> f32.
//
// At M <= 8 the work is HBM-bound: every weight byte is read once and feeds
// at most 16 multiply-adds per weight.  The Q4_K scales change every 32
// weights of K, so each 32-deep product is rescaled in registers right after
// it is formed; mma.sync keeps its accumulator in registers for exactly that
// (a TMEM accumulator would need a tcgen05.ld per 32 weights of K).
//
// Operands.  A (weights): the 4-bit quants become exact f16 values in
// registers ((q & mask) | 0x6400 is 1024 + q as an f16, minus 1024; a high
// nibble masked in place gives 16 q the same way).  B (activations): each row
// is staged once as x / s = hi + lo, two f16 values per element, s a power of
// two per row; both products accumulate into one f32 accumulator, so the
// activation keeps ~22 significant bits.  Every weight and both activation
// halves are exact f16 operands and the products are exact; only the f32
// accumulation rounds.
//
// Data movement.  Weights and headers stream by 2-D tiled TMA
// (cp.async.bulk.tensor, no multicast) into a ring of shared-memory stages
// signalled by mbarriers (bounded waits); the staged activations (L2
// resident) are read straight from global memory one stage ahead.  A stage
// is up to 128 output rows (8 groups of 16) of one job x 512 elements of K
// (2 super-blocks = 8 sub-block pairs of 64):
//   A  quant bytes [super-block][128 rows][128 B], 128-byte swizzled, loaded
//      as boxes of 16..128 rows (one per set bit of the group count);
//   H  headers [128 rows][32 B].
// The 256 consumer threads first decode the stage's scales cooperatively
// (one (pair, row) entry each, four per thread) into a double-buffered table
// of (d*sc_lo, d*sc_hi/16, dmin*m_lo, dmin*m_hi); consumer warp w then owns
// sub-block pair w for every row group, so its activation fragments are
// loaded once per stage.  Accumulators (8 groups x 4 floats) live across the
// K loop of a row block; at the end of the block the 8 warps' partials are
// summed in warp order (deterministic) in the last stage's buffer.
//
// Fragment mapping.  MMA row m of a row group is weight row 2m (m < 8) or
// 2(m-8)+1, MMA column n is token n.  In k16 step s of a sub-block, thread
// t's K slots (2t, 2t+1) hold elements (8t+4s, 8t+4s+2) and slots (2t+8,
// 2t+9) hold (8t+4s+1, 8t+4s+3): one 32-bit word of quant bytes gives both
// pairs with one shift, and the staged activations store every quad of
// elements as (e0, e2, e1, e3) so one 128-bit load gives a thread's B
// fragments for both steps.  The 64-bit shared loads of the quant bytes
// touch 16 distinct bank pairs per half-warp under the 128-byte swizzle.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <algorithm>

#include "rq_async.cuh"
#include "rq_mv_common.cuh"

namespace rq {

size_t xh_bytes(int64_t rows, int64_t in) {
    size_t b = ((size_t)rows * 4 * (size_t)in + 255) & ~(size_t)255;  // f16 hi + lo
    b += ((size_t)rows * 4 + 255) & ~(size_t)255;                     // row scales
    b += ((size_t)rows * (size_t)(in / 32) * 4 + 255) & ~(size_t)255;  // block sums
    b += (size_t)rows * (size_t)(in / 256) * 32;                        // block sums, f16 hi / lo
    return b;
}

XH xh_at(void* base, int64_t rows, int64_t in) {
    uint8_t* p = (uint8_t*)base;
    XH x;
    x.v = (__half*)p;
    p += ((size_t)rows * 4 * (size_t)in + 255) & ~(size_t)255;
    x.scale = (float*)p;
    p += ((size_t)rows * 4 + 255) & ~(size_t)255;
    x.bsum = (float*)p;
    p += ((size_t)rows * (size_t)(in / 32) * 4 + 255) & ~(size_t)255;
    x.bs16 = (__half*)p;
    return x;
}

namespace {

// ------------------------------------------------------------------ staging
// One CTA per row: s = 2^e with amax < s <= 2 amax (1 for a zero row),
// v = x / s, hi = f16(v), lo = f16(v - hi), stored quad-permuted; block sums
// of v in element order, in f32 and as f16 hi / lo pairs grouped per
// super-block (the K = 16 operand of the tcgen05 kernel's min term).  The
// staged row is Op's value of each element: the input itself, its RMSNorm
// (x / sqrt(mean(x^2) + eps) * w, the order of xquant_rmsnorm_kernel) or
// SwiGLU (silu(gate) * up, silu(g) = g / (1 + exp(-g))).
struct OpPlain {
    const float* x;
    __device__ void setup(int64_t, int64_t, float*) {}
    __device__ float at(int64_t m, int64_t in, int64_t k) const { return x[m * in + k]; }
    __device__ void block(int64_t m, int64_t in, int64_t b, float (&v)[32]) const { load_block(x + m * in + 32 * b, v); }
};
struct OpRms {
    const float* x;
    const float* w;
    float eps;
    float mden;
    __device__ void setup(int64_t m, int64_t in, float* red) {
        const float* row = x + m * in;
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
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s2;
        __syncthreads();
        float tot = 0.0f;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) tot += red[k];
        mden = sqrtf(tot / (float)in + eps);
        __syncthreads();
    }
    __device__ float at(int64_t m, int64_t in, int64_t k) const { return x[m * in + k] / mden * w[k]; }
    __device__ void block(int64_t m, int64_t in, int64_t b, float (&v)[32]) const {
        float ww[32];
        load_block(x + m * in + 32 * b, v);
        load_block(w + 32 * b, ww);
#pragma unroll
        for (int k = 0; k < 32; k++) v[k] = v[k] / mden * ww[k];
    }
};
struct OpSwiglu {
    const float* g;
    const float* u;
    __device__ void setup(int64_t, int64_t, float*) {}
    __device__ float at(int64_t m, int64_t in, int64_t k) const {
        const float v = g[m * in + k];
        return v / (1.0f + expf(-v)) * u[m * in + k];
    }
    __device__ void block(int64_t m, int64_t in, int64_t b, float (&v)[32]) const {
        float uu[32];
        load_block(g + m * in + 32 * b, v);
        load_block(u + m * in + 32 * b, uu);
#pragma unroll
        for (int k = 0; k < 32; k++) v[k] = v[k] / (1.0f + expf(-v[k])) * uu[k];
    }
};

template <class Op>
__global__ void __launch_bounds__(256) xh_stage_kernel(Op op, int64_t in, __half* __restrict__ xh,
                                                       float* __restrict__ scale, float* __restrict__ bsum,
                                                       __half* __restrict__ bs16) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    __shared__ float red[8];
    const int64_t m = blockIdx.x;
    op.setup(m, in, red);
    float a = 0.0f;
    for (int64_t k = threadIdx.x; k < in; k += blockDim.x) a = fmaxf(a, fabsf(op.at(m, in, k)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
    __syncthreads();
    float amax = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) amax = fmaxf(amax, red[w]);
    int e = 0;
    if (amax > 0.0f) frexpf(amax, &e);  // amax = f 2^e, f in [0.5, 1)
    const float inv = ldexpf(1.0f, -e);
    if (threadIdx.x == 0) scale[m] = ldexpf(1.0f, e);
    __half* hi = xh + m * 2 * in;
    __half* lo = hi + in;
    for (int64_t b = threadIdx.x; b < in / 32; b += blockDim.x) {
        float s = 0.0f;
        __half h[32], l[32];
        float vb[32];
        op.block(m, in, b, vb);  // the values of at(), loaded as 16-byte vectors
#pragma unroll
        for (int k = 0; k < 32; k++) {
            const float t = vb[k] * inv;
            s += t;
            h[k] = __float2half_rn(t);
            l[k] = __float2half_rn(t - __half2float(h[k]));
        }
        // quad (e0, e1, e2, e3) is stored as (e0, e2, e1, e3)
        uint32_t ph[16], pl[16];
#pragma unroll
        for (int q = 0; q < 8; q++) {
            ph[2 * q] = (uint32_t)__half_as_ushort(h[4 * q]) | ((uint32_t)__half_as_ushort(h[4 * q + 2]) << 16);
            ph[2 * q + 1] = (uint32_t)__half_as_ushort(h[4 * q + 1]) | ((uint32_t)__half_as_ushort(h[4 * q + 3]) << 16);
            pl[2 * q] = (uint32_t)__half_as_ushort(l[4 * q]) | ((uint32_t)__half_as_ushort(l[4 * q + 2]) << 16);
            pl[2 * q + 1] = (uint32_t)__half_as_ushort(l[4 * q + 1]) | ((uint32_t)__half_as_ushort(l[4 * q + 3]) << 16);
        }
        uint4* dh = reinterpret_cast<uint4*>(hi + 32 * b);
        uint4* dl = reinterpret_cast<uint4*>(lo + 32 * b);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            dh[k] = make_uint4(ph[4 * k], ph[4 * k + 1], ph[4 * k + 2], ph[4 * k + 3]);
            dl[k] = make_uint4(pl[4 * k], pl[4 * k + 1], pl[4 * k + 2], pl[4 * k + 3]);
        }
        bsum[m * (in / 32) + b] = s;
        const __half sh = __float2half_rn(s);
        __half* b16 = bs16 + m * (in / 32) * 2 + (b >> 3) * 16 + (b & 7);
        b16[0] = sh;
        b16[8] = __float2half_rn(s - __half2float(sh));
    }
}

template <class Op>
int launch_stage(Op op, int64_t M, int64_t in, XH xh, cudaStream_t st) {
    if (M <= 0) return RQ_OK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)M);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_error(cudaLaunchKernelEx(&cfg, xh_stage_kernel<Op>, op, in, xh.v, xh.scale, xh.bsum, xh.bs16),
                      "x staging (f16)");
}

// ------------------------------------------------------------------- matmul

constexpr int kCons = 8;                  // consumer warps (one sub-block pair each)
constexpr int kThreadsMM = 32 * (1 + kCons);
constexpr int kCS = 2;                    // super-blocks per stage
constexpr int kRG = 8;                    // 16-row groups per block (at most)
constexpr int kMP = 8;                    // token rows per job
constexpr int kNH = 4;                    // box heights 16, 32, 64, 128 rows
constexpr uint32_t kABytes = kCS * kRG * 2048;           // 32768
constexpr uint32_t kHOff = kABytes;
constexpr uint32_t kHBytes = kRG * 16 * 16 * kCS;        // 4096
constexpr uint32_t kStageBytes = kHOff + kHBytes;        // 36864, a multiple of 1024
constexpr uint32_t kDecBytes = kCons * kRG * 16 * 16;    // 16384 per buffer
constexpr uint32_t kBarRegion = 1024;                    // up to 64 mbarriers
constexpr int kSmemBudgetMM = 227 * 1024;
static_assert(kCons * kRG * 16 * kMP * 4 <= (int)kABytes, "block partials fit in a stage");

struct MMJob {
    float* y;          // [M][out] rows of this job
    const float* add;  // optional residual with y's layout (may alias y)
    int64_t out;
    int64_t g0;        // first 16-row group of this job in the launch's group order
    int tok0, M;       // token rows [tok0, tok0 + M) of the staged activations
};

struct alignas(64) MMParams {
    CUtensorMap wq[kMaxJobs][kNH];  // quant bytes [out][nblk*128], box 128 x (16 << h), swizzle 128B
    CUtensorMap wh[kMaxJobs][kNH];  // headers     [out][nblk*16],  box 32 x (16 << h)
    MMJob jobs[kMaxJobs];
    const __half* xh;
    const float* xscale;
    const float* xbsum;
    int64_t in;
    int64_t gtot;
    int* err;
    int njobs;
    int nchunk;  // stages per row block = ceil(nblk / kCS)
    int nstage;
};

__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ uint4 ldg128(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ float2 ldg64f(const void* p) {
    float2 v;
    asm volatile("ld.global.nc.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
    return v;
}

// byte i of w as an exact float (0x4B0000bi is 2^23 + b_i)
template <int I>
__device__ __forceinline__ float byte_f32(uint32_t w) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u + I)) - 8388608.0f;
}

__device__ __forceinline__ void hmma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The stages of this CTA, in order.  The CTA owns groups
// [b*gtot/grid, (b+1)*gtot/grid) of the concatenated 16-row groups of all
// jobs; each job's share is cut into near-equal row blocks of at most kRG
// groups, and each block runs nchunk stages.
struct Sched {
    int64_t c0, c1;  // this CTA's group range
    int64_t lo, n;   // the current job's share [lo, lo + n)
    int64_t row0;    // first row of the current block
    int j, b, nb;    // job, block within the share, blocks in the share
    int ng, c;       // groups of the block, stage within the block
    bool valid;
};

__device__ __forceinline__ void sched_block(const MMParams& p, Sched& s) {
    const int64_t a = s.lo + (int64_t)s.b * s.n / s.nb, e = s.lo + (int64_t)(s.b + 1) * s.n / s.nb;
    s.row0 = (a - p.jobs[s.j].g0) * 16;
    s.ng = (int)(e - a);
    s.c = 0;
}

__device__ __forceinline__ void sched_job(const MMParams& p, Sched& s) {
    for (; s.j < p.njobs; s.j++) {
        const int64_t jg0 = p.jobs[s.j].g0, jg1 = jg0 + (p.jobs[s.j].out + 15) / 16;
        const int64_t lo = s.c0 > jg0 ? s.c0 : jg0, hi = s.c1 < jg1 ? s.c1 : jg1;
        if (lo < hi) {
            s.lo = lo;
            s.n = hi - lo;
            s.nb = (int)((s.n + kRG - 1) / kRG);
            s.b = 0;
            s.valid = true;
            sched_block(p, s);
            return;
        }
    }
    s.valid = false;
}

__device__ __forceinline__ void sched_start(const MMParams& p, Sched& s) {
    s.c0 = (int64_t)blockIdx.x * p.gtot / gridDim.x;
    s.c1 = (int64_t)(blockIdx.x + 1) * p.gtot / gridDim.x;
    s.j = 0;
    sched_job(p, s);
}

__device__ __forceinline__ void sched_next(const MMParams& p, Sched& s) {
    if (++s.c < p.nchunk) return;
    if (++s.b < s.nb) {
        sched_block(p, s);
        return;
    }
    s.j++;
    sched_job(p, s);
}

// The activation fragments of one stage for one thread: B words of the low
// and high sub-block (hi and lo halves of the staged value, both k16 steps)
// and the block sums of tokens 2t, 2t+1.
struct BFrag {
    uint4 lh, ll, hh, hl;  // [sub-block low/high][activation hi/lo]
    float2 s0, s1;         // block sums (low, high sub-block) of tokens 2t, 2t+1
};

struct MMLane {
    int g, t, sbl, gq;
    uint32_t a0, a1;     // quant bytes 8t..8t+7 of rows 2g, 2g+1 in a row-group box
    const __half* xrow;  // hi plane of token g of the job (clamped), at element 8t
    const float* bs0;    // block sums of tokens 2t, 2t+1 (clamped)
    const float* bs1;
};

// PAIR (jobs of at most 4 rows): MMA column 2t + h is half h (hi, lo) of
// token t, so one MMA serves both halves; thread (g, t) loads half g & 1 of
// token g >> 1 (L.xrow points at that plane) and the block sums of token t.
template <bool PAIR>
__device__ __forceinline__ BFrag load_b(const MMLane& L, int64_t in, int c) {
    const int64_t e0 = (int64_t)c * (kCS * 256) + 256 * L.sbl + 64 * L.gq;
    BFrag b;
    if (e0 >= in) {  // the pair lies in the zero-filled tail of the last stage
        b.lh = b.ll = b.hh = b.hl = make_uint4(0u, 0u, 0u, 0u);
        b.s0 = b.s1 = make_float2(0.f, 0.f);
        return b;
    }
    if constexpr (PAIR) {
        b.lh = ldg128(L.xrow + e0);
        b.hh = ldg128(L.xrow + e0 + 32);
        b.ll = b.hl = make_uint4(0u, 0u, 0u, 0u);
        b.s0 = ldg64f(L.bs0 + e0 / 32);
        b.s1 = make_float2(0.f, 0.f);
    } else {
        b.lh = ldg128(L.xrow + e0);
        b.ll = ldg128(L.xrow + in + e0);
        b.hh = ldg128(L.xrow + e0 + 32);
        b.hl = ldg128(L.xrow + in + e0 + 32);
        b.s0 = ldg64f(L.bs0 + e0 / 32);
        b.s1 = ldg64f(L.bs1 + e0 / 32);
    }
    return b;
}

// Shared-memory operands of row groups rg and rg+1 of one stage: quant words
// of rows 2g, 2g+1 and their decoded scales.
struct PairOps {
    uint2 w0[2], w1[2];
    uint4 q0[2], q1[2];
};

__device__ __forceinline__ void load_pair(PairOps& o, int rg0, uint32_t st, uint32_t dec, const MMLane& L) {
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const uint32_t A = st + (uint32_t)L.sbl * (kRG * 2048u) + (uint32_t)(rg0 + k) * 2048u;
        o.w0[k] = lds64(A + L.a0);
        o.w1[k] = lds64(A + L.a1);
        const uint32_t dq = dec + (uint32_t)((L.gq + 4 * L.sbl) * (kRG * 16) + (rg0 + k) * 16 + 2 * L.g) * 16u;
        o.q0[k] = lds128(dq);
        o.q1[k] = lds128(dq + 16);
    }
}

// Row groups rg0 and rg0+1 (the second may lie past the block's ng: it reads
// stale shared memory and its sums are discarded).  acc[rg][i]: weight row
// 2g + (i >> 1) of the group; token 2t + (i & 1), or with PAIR token t (i < 2).
template <bool PAIR>
__device__ __forceinline__ void compute_pair(float (&acc)[kRG][4], int rg0, const PairOps& o, const BFrag& b) {
    float dl[2][4], dh[2][4];
#pragma unroll
    for (int k = 0; k < 2; k++)
#pragma unroll
        for (int i = 0; i < 4; i++) dl[k][i] = dh[k][i] = 0.0f;
#pragma unroll
    for (int s = 0; s < 2; s++) {
        const uint32_t bh0 = s ? b.lh.z : b.lh.x, bh1 = s ? b.lh.w : b.lh.y;
        const uint32_t bl0 = s ? b.ll.z : b.ll.x, bl1 = s ? b.ll.w : b.ll.y;
        const uint32_t ch0 = s ? b.hh.z : b.hh.x, ch1 = s ? b.hh.w : b.hh.y;
        const uint32_t cl0 = s ? b.hl.z : b.hl.x, cl1 = s ? b.hl.w : b.hl.y;
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const uint32_t u0 = s ? o.w0[k].y : o.w0[k].x, u1 = s ? o.w1[k].y : o.w1[k].x;
            const uint32_t v0 = u0 >> 8, v1 = u1 >> 8;
            // the low nibble of a byte, as a 16-bit pattern, is the f16
            // subnormal q 2^-24; the high nibble in place is 16 q 2^-24
            const uint32_t la0 = u0 & 0x000F000Fu, la1 = u1 & 0x000F000Fu;
            const uint32_t la2 = v0 & 0x000F000Fu, la3 = v1 & 0x000F000Fu;
            const uint32_t ha0 = u0 & 0x00F000F0u, ha1 = u1 & 0x00F000F0u;
            const uint32_t ha2 = v0 & 0x00F000F0u, ha3 = v1 & 0x00F000F0u;
            hmma(dl[k], la0, la1, la2, la3, bh0, bh1);
            hmma(dh[k], ha0, ha1, ha2, ha3, ch0, ch1);
            if constexpr (!PAIR) {
                hmma(dl[k], la0, la1, la2, la3, bl0, bl1);
                hmma(dh[k], ha0, ha1, ha2, ha3, cl0, cl1);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 2; k++) {
        if constexpr (PAIR) {
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const uint4 q = j ? o.q1[k] : o.q0[k];
                // columns 2t, 2t+1 are the hi and lo halves of token t
                const float vl = dl[k][2 * j] + dl[k][2 * j + 1];
                const float vh = dh[k][2 * j] + dh[k][2 * j + 1];
                float a = acc[rg0 + k][j];
                a = fmaf(__uint_as_float(q.x), vl, a);
                a = fmaf(__uint_as_float(q.y), vh, a);
                a = fmaf(-__uint_as_float(q.z), b.s0.x, a);
                a = fmaf(-__uint_as_float(q.w), b.s0.y, a);
                acc[rg0 + k][j] = a;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint4 q = (i >> 1) ? o.q1[k] : o.q0[k];
                const float bsl = (i & 1) ? b.s1.x : b.s0.x, bsh = (i & 1) ? b.s1.y : b.s0.y;
                float a = acc[rg0 + k][i];
                a = fmaf(__uint_as_float(q.x), dl[k][i], a);
                a = fmaf(__uint_as_float(q.y), dh[k][i], a);
                a = fmaf(-__uint_as_float(q.z), bsl, a);
                a = fmaf(-__uint_as_float(q.w), bsh, a);
                acc[rg0 + k][i] = a;
            }
        }
    }
}

// Copies of one stage: for each set bit of ng (8, 4, 2, 1 groups) a box of
// the quant bytes of super-block 0, of super-block 1 and of the headers;
// lane i issues box i.
__device__ __forceinline__ void issue_stage(const MMParams& p, const Sched& s, uint32_t st, uint32_t fb, int lane,
                                            uint64_t pol) {
    const int ng = s.ng, c = s.c, j = s.j;
    if (lane == 0) mbar_expect_tx(fb, (uint32_t)ng * (kCS * 2048u + 512u));
    __syncwarp();
    int i = 0, gdone = 0;
#pragma unroll
    for (int h = kNH - 1; h >= 0; h--) {
        if (ng & (1 << h)) {
            const int y = (int)(s.row0 + gdone * 16);
            if (lane == i) tma_load_2d(st + (uint32_t)gdone * 2048u, &p.wq[j][h], (c * kCS) * 128, y, fb, pol);
            if (lane == i + 1)
                tma_load_2d(st + kRG * 2048u + (uint32_t)gdone * 2048u, &p.wq[j][h], (c * kCS + 1) * 128, y, fb, pol);
            if (lane == i + 2) tma_load_2d(st + kHOff + (uint32_t)gdone * 512u, &p.wh[j][h], c * kCS * 16, y, fb, pol);
            i += 3;
            gdone += 1 << h;
        }
    }
}

// Warp 0 streams the stages; warps 1..8 consume them.  9 warps: one
// scheduler holds 3 of them, so 168 registers per thread at most.
template <bool PAIR>
__global__ void __launch_bounds__(kThreadsMM, 1) mm_q4k_kernel(const __grid_constant__ MMParams p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled boxes
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    uint8_t* smem = smem_raw + pad;
    const uint32_t sbase = raw + pad;
    const uint32_t full0 = sbase, empty0 = sbase + 8u * (uint32_t)p.nstage;
    const uint32_t dec0 = sbase + kBarRegion;
    const uint32_t ring = dec0 + 2 * kDecBytes;
    uint8_t* ring_p = smem + kBarRegion + 2 * kDecBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    asm volatile("griddepcontrol.launch_dependents;");
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nstage; i++) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, kCons);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        // weights are written only by synchronous calls: stream them at once
        const uint64_t pol_w = policy_evict_first();
        Sched ps;
        sched_start(p, ps);
        int it = 0, slot = 0, phase = 0;
        bool ok = true;
        for (; ps.valid; sched_next(p, ps), it++) {
            int good = 1;
            if (lane == 0 && it >= p.nstage) good = mbar_wait(empty0 + 8 * slot, phase ^ 1) ? 1 : 0;
            good = __shfl_sync(0xffffffffu, good, 0);
            if (!good) {
                ok = false;
                break;
            }
            issue_stage(p, ps, ring + (uint32_t)slot * kStageBytes, full0 + 8 * slot, lane, pol_w);
            if (++slot == p.nstage) {
                slot = 0;
                phase ^= 1;
            }
        }
        // no copy may still be landing when the CTA exits
        if (lane == 0) {
            for (int k = max(0, it - p.nstage); k < it; k++)
                if (!mbar_wait(full0 + 8 * (k % p.nstage), (k / p.nstage) & 1)) ok = false;
            if (!ok && p.err) atomicExch(p.err, 1);
        }
        return;
    }

    // --------------------------------------------------------------- consumers
    // activations are written by the preceding kernel in the stream
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int cw = warp - 1, ct = threadIdx.x - 32;
    MMLane L;
    L.g = lane >> 2;
    L.t = lane & 3;
    L.sbl = cw >> 2;
    L.gq = cw & 3;
    {
        const uint32_t acol = (uint32_t)(32 * L.gq + 8 * L.t);
        L.a0 = (uint32_t)(2 * L.g) * 128u + (acol ^ (((uint32_t)(2 * L.g) & 7u) << 4));
        L.a1 = (uint32_t)(2 * L.g + 1) * 128u + (acol ^ (((uint32_t)(2 * L.g + 1) & 7u) << 4));
    }
    // this thread decodes the entries (pair dpair0 + 2i, row drow), i < 4
    const int drow = ct & 127, dpair0 = ct >> 7;
    const Q4KScaleSel dsel0 = q4k_scale_sel(dpair0 & 3);        // pairs dpair0, dpair0 + 4
    const Q4KScaleSel dsel1 = q4k_scale_sel((dpair0 + 2) & 3);  // pairs dpair0 + 2, dpair0 + 6
    Sched cs;
    sched_start(p, cs);
    int it = 0, slot = 0, phase = 0;
    bool ok = true;
    float acc[kRG][4];
    BFrag bcur;
    while (cs.valid) {
        const MMJob& jb = p.jobs[cs.j];
        if (cs.c == 0) {  // a new row block
            if constexpr (PAIR) {
                const int tb = jb.tok0 + min(L.g >> 1, jb.M - 1);
                L.xrow = p.xh + (int64_t)tb * 2 * p.in + (L.g & 1) * p.in + 8 * L.t;
                L.bs0 = p.xbsum + (int64_t)(jb.tok0 + min(L.t, jb.M - 1)) * (p.in / 32);
                L.bs1 = L.bs0;
            } else {
                const int tb = jb.tok0 + min(L.g, jb.M - 1);
                L.xrow = p.xh + (int64_t)tb * 2 * p.in + 8 * L.t;
                L.bs0 = p.xbsum + (int64_t)(jb.tok0 + min(2 * L.t, jb.M - 1)) * (p.in / 32);
                L.bs1 = p.xbsum + (int64_t)(jb.tok0 + min(2 * L.t + 1, jb.M - 1)) * (p.in / 32);
            }
#pragma unroll
            for (int rg = 0; rg < kRG; rg++)
#pragma unroll
                for (int i = 0; i < 4; i++) acc[rg][i] = 0.0f;
            bcur = load_b<PAIR>(L, p.in, 0);
        }
        const int ng = cs.ng;
        BFrag bnext = bcur;
        if (cs.c + 1 < p.nchunk) bnext = load_b<PAIR>(L, p.in, cs.c + 1);
        if (ok && !mbar_wait(full0 + 8 * slot, phase)) {
            ok = false;
            if (lane == 0 && p.err) atomicExch(p.err, 1);
        }
        const uint32_t st = ring + (uint32_t)slot * kStageBytes;
        const uint32_t dec = dec0 + (uint32_t)(it & 1) * kDecBytes;
        if (ok && drow < ng * 16) {
            // cooperative scale decode of the stage's headers
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int pair = dpair0 + 2 * i;
                const uint4 h = lds128(st + kHOff + (uint32_t)drow * 32u + 16u * (uint32_t)(pair >> 2));
                const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                const uint32_t w = q4k_scales((i & 1) ? dsel1 : dsel0, h);
                // the quants enter the products as q 2^-24 (16 q 2^-24 for
                // high nibbles): 2^24 and 2^20 restore them
                const float dq = dd.x * 16777216.0f;
                sts128(dec + (uint32_t)(pair * (kRG * 16) + drow) * 16u,
                       make_float4(dq * byte_f32<0>(w), dq * 0.0625f * byte_f32<1>(w), dd.y * byte_f32<2>(w),
                                   dd.y * byte_f32<3>(w)));
            }
        }
        named_bar_sync(1, kCons * 32);
        if (ok) {
#pragma unroll
            for (int rg = 0; rg < kRG; rg += 2) {
                if (rg < ng) {
                    PairOps ops;
                    load_pair(ops, rg, st, dec, L);
                    compute_pair<PAIR>(acc, rg, ops, bcur);
                }
            }
        }
        bcur = bnext;
        __syncwarp();
        const bool last = cs.c + 1 == p.nchunk;
        // a block's last stage is released after its reduction
        if (lane == 0 && !last) mbar_arrive(empty0 + 8 * slot);
        if (last) {
            // sum the 8 warps' partials in warp order, in this stage's buffer
            float* red = reinterpret_cast<float*>(ring_p + (size_t)slot * kStageBytes);
            named_bar_sync(1, kCons * 32);
#pragma unroll
            for (int rg = 0; rg < kRG; rg++) {
                if (rg < ng) {
                    if constexpr (PAIR) {
#pragma unroll
                        for (int j = 0; j < 2; j++) {
                            const int row = rg * 16 + 2 * L.g + j;
                            red[(cw * kRG * 16 + row) * kMP + L.t] = acc[rg][j];
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int row = rg * 16 + 2 * L.g + (i >> 1);
                            red[(cw * kRG * 16 + row) * kMP + 2 * L.t + (i & 1)] = acc[rg][i];
                        }
                    }
                }
            }
            named_bar_sync(1, kCons * 32);
            const int nrow = (int)min((int64_t)ng * 16, jb.out - cs.row0);
            for (int tk = 0; tk < jb.M; tk++) {
                const float sc = p.xscale[jb.tok0 + tk];
                for (int row = ct; row < nrow; row += kCons * 32) {
                    float s = 0.0f;
#pragma unroll
                    for (int w = 0; w < kCons; w++) s += red[(w * kRG * 16 + row) * kMP + tk];
                    const int64_t o = (int64_t)tk * jb.out + cs.row0 + row;
                    jb.y[o] = jb.add ? s * sc + jb.add[o] : s * sc;
                }
            }
            // the producer refills the buffer after all eight warps arrive
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * slot);
        }
        sched_next(p, cs);
        it++;
        if (++slot == p.nstage) {
            slot = 0;
            phase ^= 1;
        }
    }
}

using EncodeTiled = PFN_cuTensorMapEncodeTiled_v12000;

EncodeTiled encode_fn() {
    static EncodeTiled fn = []() -> EncodeTiled {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<EncodeTiled>(f);
    }();
    return fn;
}

int encode_2d(CUtensorMap* m, const void* base, uint64_t dim0, uint64_t dim1, uint64_t row_stride, uint32_t box0,
              uint32_t box1, CUtensorMapSwizzle sw, const char* what) {
    EncodeTiled fn = encode_fn();
    if (!fn) return set_error(RQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {dim0, dim1};
    const cuuint64_t strides[1] = {row_stride};
    const cuuint32_t box[2] = {box0, box1};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(RQ_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed: %d", what, (int)r);
    return RQ_OK;
}

}  // namespace

int launch_xh_stage(const float* x, int64_t M, int64_t in, XH xh, cudaStream_t st) {
    return launch_stage(OpPlain{x}, M, in, xh, st);
}

int launch_xh_stage_rmsnorm(const float* x, const float* w, float eps, int64_t M, int64_t in, XH xh,
                            cudaStream_t st) {
    return launch_stage(OpRms{x, w, eps, 0.0f}, M, in, xh, st);
}

int launch_xh_stage_swiglu(const float* gate, const float* up, int64_t M, int64_t in, XH xh, cudaStream_t st) {
    return launch_stage(OpSwiglu{gate, up}, M, in, xh, st);
}

bool mm_small_supported(const rq_weight* w) { return w->type == RQ_Q4_K; }

int launch_matmul_small(const rq_weight* w, XH xh, int64_t M, float* y, const float* add, int sm_count,
                        cudaStream_t st, int* err) {
    // tiles of kMP activation rows, up to kMaxJobs tiles per launch: each
    // launch reads the weights once per tile
    for (int64_t m0 = 0; m0 < M; m0 += (int64_t)kMP * kMaxJobs) {
        MMJobDesc jobs[kMaxJobs];
        int n = 0;
        for (int64_t t0 = m0; t0 < M && n < kMaxJobs; t0 += kMP, n++)
            jobs[n] = MMJobDesc{w, (int)t0, (int)std::min<int64_t>(kMP, M - t0), y + t0 * w->out,
                                add ? add + t0 * w->out : nullptr};
        int rc = launch_mm_small(jobs, n, xh, M, sm_count, st, err);
        if (rc) return rc;
    }
    return RQ_OK;
}

int launch_mm_small(const MMJobDesc* jobs, int njobs, XH xh, int64_t rows, int sm_count, cudaStream_t st,
                    int* err) {
    if (njobs < 1 || njobs > kMaxJobs) return set_error(RQ_ERR_INVALID, "small-M matmul: %d jobs", njobs);
    const int64_t in = jobs[0].w->in, nblk = jobs[0].w->nblk;
    MMParams p;
    memset(&p, 0, sizeof p);
    int64_t gtot = 0;
    for (int j = 0; j < njobs; j++) {
        const rq_weight* w = jobs[j].w;
        if (w->type != RQ_Q4_K || w->in != in)
            return set_error(RQ_ERR_INVALID, "small-M matmul: jobs need Q4_K weights with the same K");
        if (jobs[j].M < 1 || jobs[j].M > kMP || jobs[j].tok0 < 0 || jobs[j].tok0 + jobs[j].M > rows)
            return set_error(RQ_ERR_INVALID, "small-M matmul: token rows [%d, %d) of %lld", jobs[j].tok0,
                             jobs[j].tok0 + jobs[j].M, (long long)rows);
        for (int h = 0; h < kNH; h++) {
            int rc = encode_2d(&p.wq[j][h], w->qs, (uint64_t)(nblk * 128), (uint64_t)w->out, (uint64_t)(nblk * 128),
                               128, 16u << h, CU_TENSOR_MAP_SWIZZLE_128B, "quant bytes");
            if (!rc)
                rc = encode_2d(&p.wh[j][h], w->hdr, (uint64_t)(nblk * 16), (uint64_t)w->out, (uint64_t)(nblk * 16),
                               16 * kCS, 16u << h, CU_TENSOR_MAP_SWIZZLE_NONE, "headers");
            if (rc) return rc;
        }
        p.jobs[j].y = jobs[j].y;
        p.jobs[j].add = jobs[j].add;
        p.jobs[j].out = w->out;
        p.jobs[j].g0 = gtot;
        p.jobs[j].tok0 = jobs[j].tok0;
        p.jobs[j].M = jobs[j].M;
        gtot += (w->out + 15) / 16;
    }
    p.xh = xh.v;
    p.xscale = xh.scale;
    p.xbsum = xh.bsum;
    p.in = in;
    p.njobs = njobs;
    p.nchunk = (int)((nblk + kCS - 1) / kCS);
    p.gtot = gtot;
    p.err = err;
    const int nstage = (int)((kSmemBudgetMM - 1024 - kBarRegion - 2 * kDecBytes) / kStageBytes);
    // (a stage's buffer also holds its block's partial sums)
    p.nstage = std::min(nstage, 32);
    const size_t smem = 1024 + kBarRegion + 2 * kDecBytes + (size_t)p.nstage * kStageBytes;
    const int grid = (int)std::min<int64_t>(gtot, sm_count);

    // jobs of at most kMP / 2 rows put both activation halves in one MMA
    bool pair = true;
    for (int j = 0; j < njobs; j++) pair = pair && jobs[j].M <= kMP / 2;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(mm_q4k_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemBudgetMM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(mm_q4k_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudgetMM);
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(small-M matmul)");
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreadsMM);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_error(pair ? cudaLaunchKernelEx(&cfg, mm_q4k_kernel<true>, p)
                           : cudaLaunchKernelEx(&cfg, mm_q4k_kernel<false>, p),
                      "small-M matmul kernel");
}

}  // namespace rq
