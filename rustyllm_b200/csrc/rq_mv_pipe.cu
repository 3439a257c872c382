// rq_mv_pipe.cu -- M=1 matvec with weights staged through shared memory by
// bulk asynchronous copies (cp.async.bulk, the non-tensor TMA path).
//
// One persistent CTA per SM owns a contiguous range of output rows, so its
// weight bytes are two contiguous byte ranges (quant part and header part of
// the device layout).  Warp 0, lane 0 is the producer: it streams stages of
// RS whole rows into a ring of NSTAGE shared-memory buffers (~200 KB in
// flight per SM, independent of registers), signalling an mbarrier per stage
// with the byte count.  Consumer warp (s, g) keeps the activation planes of
// K-slice s in registers and processes rows g, g+G, ... of every stage, then
// releases the buffer through the stage's "empty" mbarrier.  Per-row lane
// partials are transpose-reduced within the warp and written to a per-CTA
// table [row][slice]; after the last stage the table is summed in slice
// order (deterministic) and y is written.
//
// Launched as a programmatic dependent of the activation-staging kernel: the
// producer starts streaming weights at once (weights do not depend on the
// preceding kernel), consumers wait (griddepcontrol.wait) before reading the
// planes.  Every mbarrier wait is bounded (~1 s); on expiry the kernel sets
// the error word, drains its in-flight copies and exits.

#include <algorithm>

#include "rq_mv_common.cuh"

namespace rq {
namespace {

// 16 warps per CTA (one producer, up to 15 consumers) keep the register
// budget at 128 per thread: the register file is split over four schedulers
// and a fifth resident warp on one of them would cap every thread at 96.
constexpr int kMaxConsumerWarps = 15;
constexpr int kThreads = 32 * (1 + kMaxConsumerWarps);
constexpr int kSmemBudget = 227 * 1024;
constexpr int kBarBytes = 2 * 32 * 8;  // up to 32 stages: full + empty barriers
constexpr long long kWaitCycles = 1ll << 31;

struct PipeParams {
    const uint8_t* qs;
    const uint8_t* hdr;
    const int8_t* planes;
    const float4* stats;
    float* y;
    int* err;
    int64_t out, nblk, in;
    int S, G, RS, nstage;
    uint32_t qrow, hrow;  // device bytes per weight row (quant part, header part)
    uint32_t stage_bytes, red_off, ring_off;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t a, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase with the given parity to complete; false after ~1 s.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity) {
    if (mbar_try_wait(a, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(a, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t mbar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(mbar), "l"(policy)
        : "memory");
}

template <int TYPE>
struct LaneOf;
template <>
struct LaneOf<RQ_Q4_K> { using T = Q4KPLane; };
template <>
struct LaneOf<RQ_Q3_K> { using T = Q3KLane; };
template <>
struct LaneOf<RQ_Q4_0> { using T = Q40Lane; };

// Set up lane data for K-slice s; returns whether the lane has valid data.
template <int TYPE>
__device__ __forceinline__ bool lane_setup(typename LaneOf<TYPE>::T& L, const PipeParams& p, int s,
                                           int lane) {
    if constexpr (TYPE == RQ_Q4_0) {
        const int64_t b0 = (int64_t)s * 64 + 2 * lane;
        if (b0 >= p.nblk) return false;
        q40_lane_setup(L, p.planes, p.stats, p.in, p.nblk, b0);
        return true;
    } else if constexpr (TYPE == RQ_Q4_K) {
        // lanes past the end of a partial slice get zero activations and read
        // the slice's first group, so the row loop needs no per-lane branch
        const int64_t sb = (int64_t)s * 8 + (lane >> 2);
        const bool valid = sb < p.nblk;
        q4kp_lane_setup(L, p.planes, p.stats, p.in, valid ? sb : 0, lane & 3, (lane >> 2) & 1, valid);
        return true;
    } else {
        const int64_t sb = (int64_t)s * 8 + (lane >> 2);
        if (sb >= p.nblk) return false;
        q3k_lane_setup(L, p.planes, p.stats, p.in, sb, lane & 3);
        return true;
    }
}

// Lane contribution of one row held in shared memory (sq: the row's quant
// bytes, sh: its header bytes).
template <int TYPE>
__device__ __forceinline__ float lane_row(const typename LaneOf<TYPE>::T& L, const uint8_t* sq,
                                          const uint8_t* sh, int s, int lane) {
    // the two 16-byte halves of a lane's 32 bytes are read in an order that
    // keeps each quarter-warp's 128-bit loads on distinct banks
    const int h1 = (lane >> 2) & 1;
    if constexpr (TYPE == RQ_Q4_K) {
        return 0.0f;  // Q4_K rows go through the hoisted path in the kernel
    } else if constexpr (TYPE == RQ_Q3_K) {
        const uint8_t* b = sq + s * 768 + 96 * (lane >> 2);
        const uint4 hm = *reinterpret_cast<const uint4*>(b + 16 * L.u);
        const uint4 qv = *reinterpret_cast<const uint4*>(b + 32 + 32 * L.h + 16 * L.u);
        const uint4 hd = *reinterpret_cast<const uint4*>(sh + s * 128 + 16 * (lane >> 2));
        return q3k_lane_row(L, hm, qv, hd);
    } else {
        // the pipeline takes Q4_0 only when blocks per row is a multiple of 8,
        // so both blocks of a lane exist
        const uint8_t* q = sq + s * 1024 + 32 * lane;
        const uint4 first = *reinterpret_cast<const uint4*>(q + 16 * h1);
        const uint4 second = *reinterpret_cast<const uint4*>(q + 16 * (1 - h1));
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(sh + s * 128 + 4 * lane);
        return q40_lane_row(L, h1 ? second : first, h1 ? first : second, (uint16_t)(dd & 0xFFFFu),
                            (uint16_t)(dd >> 16));
    }
}

template <int TYPE, int RPW>
__global__ void __launch_bounds__(kThreads, 1) mv_pipe_kernel(const PipeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    float* red = reinterpret_cast<float*>(smem + p.red_off);
    uint8_t* ring = smem + p.ring_off;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r_begin = (int64_t)blockIdx.x * p.out / gridDim.x;
    const int64_t r_end = (int64_t)(blockIdx.x + 1) * p.out / gridDim.x;
    const int nrows = (int)(r_end - r_begin);
    const int nst = (nrows + p.RS - 1) / p.RS;
    const uint32_t full0 = smem_u32(smem), empty0 = full0 + 8 * p.nstage;
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nstage; i++) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, p.S * p.G);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            uint64_t pol;
            asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
            int issued = 0;
            bool ok = true;
            for (int it = 0; it < nst; it++) {
                const int slot = it % p.nstage, use = it / p.nstage;
                if (use > 0 && !mbar_wait(empty0 + 8 * slot, (use - 1) & 1)) { ok = false; break; }
                const int rows = min(p.RS, nrows - it * p.RS);
                const int64_t r0 = r_begin + (int64_t)it * p.RS;
                const uint32_t qb = (uint32_t)rows * p.qrow, hb = (uint32_t)rows * p.hrow;
                const uint32_t dst = smem_u32(ring) + (uint32_t)slot * p.stage_bytes;
                mbar_expect_tx(full0 + 8 * slot, qb + hb);
                bulk_g2s(dst, p.qs + r0 * p.qrow, qb, full0 + 8 * slot, pol);
                bulk_g2s(dst + (uint32_t)p.RS * p.qrow, p.hdr + r0 * p.hrow, hb, full0 + 8 * slot, pol);
                issued = it + 1;
            }
            // let the next kernel in the stream start its own prologue
            asm volatile("griddepcontrol.launch_dependents;");
            // no bulk copy may still be landing when the CTA exits
            for (int it = max(0, issued - p.nstage); it < issued; it++)
                if (!mbar_wait(full0 + 8 * (it % p.nstage), (it / p.nstage) & 1)) ok = false;
            if (!ok && p.err) atomicExch(p.err, 1);
        }
    } else if (warp - 1 < p.S * p.G) {
        const int c = warp - 1;
        const int s = c % p.S, g = c / p.S;
        typename LaneOf<TYPE>::T L;
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const bool valid = lane_setup<TYPE>(L, p, s, lane);
        if constexpr (TYPE == RQ_Q4_K) {
            // lane-constant shared-memory offsets within a row
            const int64_t sbl = (int64_t)s * 8 + (lane >> 2) < p.nblk ? (lane >> 2) : 0;
            const uint32_t offA = (uint32_t)(s * 1024 + 128 * sbl + 32 * (lane & 3) + 16 * ((lane >> 2) & 1));
            const uint32_t offB = offA ^ 16u;
            const uint32_t offH = (uint32_t)(s * 128 + 16 * sbl);
            for (int it = 0; it < nst; it++) {
                const int slot = it % p.nstage, use = it / p.nstage;
                if (!mbar_wait(full0 + 8 * slot, use & 1)) {
                    if (lane == 0 && p.err) atomicExch(p.err, 1);
                    break;
                }
                const uint8_t* sq = ring + (size_t)slot * p.stage_bytes;
                const uint8_t* sh = sq + (size_t)p.RS * p.qrow;
                const int rows = min(p.RS, nrows - it * p.RS);
                float part[RPW];
#pragma unroll
                for (int j = 0; j < RPW; j++) {
                    const int r = g + j * p.G;  // warp-uniform
                    part[j] = 0.0f;
                    if (r < rows) {
                        const uint8_t* q = sq + (size_t)r * p.qrow;
                        const uint4 qa = *reinterpret_cast<const uint4*>(q + offA);
                        const uint4 qb = *reinterpret_cast<const uint4*>(q + offB);
                        const uint4 h = *reinterpret_cast<const uint4*>(sh + (size_t)r * p.hrow + offH);
                        part[j] = q4kp_lane_row(L, qa, qb, h, 0.0f);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * slot);
                transpose_reduce<RPW>(part, lane);
                if (lane_writes<RPW>(lane)) {
                    const int r = g + row_of_lane<RPW>(lane) * p.G;
                    if (r < rows) red[(it * p.RS + r) * p.S + s] = part[0];
                }
            }
        } else
        for (int it = 0; it < nst; it++) {
            const int slot = it % p.nstage, use = it / p.nstage;
            if (!mbar_wait(full0 + 8 * slot, use & 1)) {
                if (lane == 0 && p.err) atomicExch(p.err, 1);
                break;
            }
            const uint8_t* sq = ring + (size_t)slot * p.stage_bytes;
            const uint8_t* sh = sq + (size_t)p.RS * p.qrow;
            const int rows = min(p.RS, nrows - it * p.RS);
            float part[RPW];
#pragma unroll
            for (int j = 0; j < RPW; j++) {
                const int r = g + j * p.G;
                part[j] = (valid && r < rows)
                              ? lane_row<TYPE>(L, sq + (size_t)r * p.qrow, sh + (size_t)r * p.hrow, s, lane)
                              : 0.0f;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * slot);
            transpose_reduce<RPW>(part, lane);
            if (lane_writes<RPW>(lane)) {
                const int r = g + row_of_lane<RPW>(lane) * p.G;
                if (r < rows) red[(it * p.RS + r) * p.S + s] = part[0];
            }
        }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < nrows; t += blockDim.x) {
        float acc = 0.0f;
        for (int s = 0; s < p.S; s++) acc += red[t * p.S + s];
        p.y[r_begin + t] = acc;
    }
}

template <int TYPE, int RPW>
int launch_pipe_t(const PipeParams& p, int grid, int threads, size_t smem, cudaStream_t st) {
    static bool attr_set[64] = {};  // per instantiation and device, set before first launch
    auto kern = mv_pipe_kernel<TYPE, RPW>;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(mv_pipe)");
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_error(cudaLaunchKernelEx(&cfg, kern, p), "matvec pipeline kernel");
}

template <int TYPE>
int launch_pipe_type(const PipeParams& p, int rpw, int grid, int threads, size_t smem, cudaStream_t st) {
    if (rpw == 1) return launch_pipe_t<TYPE, 1>(p, grid, threads, smem, st);
    if (rpw == 2) return launch_pipe_t<TYPE, 2>(p, grid, threads, smem, st);
    return launch_pipe_t<TYPE, 4>(p, grid, threads, smem, st);
}

}  // namespace

bool pipe_supported(const rq_weight* w) {
    TypeInfo ti = type_info(w->type);
    const int64_t S = (w->in + 2047) / 2048;
    if (S > kMaxConsumerWarps) return false;
    const int64_t qrow = w->nblk * ti.qs_bytes, hrow = w->nblk * ti.hdr_bytes;
    if (qrow % 16 || hrow % 16) return false;  // bulk copies move 16-byte multiples
    if (qrow + hrow > 64 * 1024) return false;
    return true;
}

int launch_matvec_pipe(const rq_weight* w, XQ xq, float* y, int sm_count, cudaStream_t st,
                       int* err) {
    TypeInfo ti = type_info(w->type);
    PipeParams p;
    p.qs = w->qs;
    p.hdr = w->hdr;
    p.planes = xq.planes;
    p.stats = xq.stats;
    p.y = y;
    p.err = err;
    p.out = w->out;
    p.nblk = w->nblk;
    p.in = w->in;
    p.S = (int)((w->in + 2047) / 2048);
    p.G = std::max(1, kMaxConsumerWarps / p.S);
    p.qrow = (uint32_t)(w->nblk * ti.qs_bytes);
    p.hrow = (uint32_t)(w->nblk * ti.hdr_bytes);
    const uint32_t rowb = p.qrow + p.hrow;
    // RS = RPW * G whole rows per stage; four rows per consumer warp unless
    // a stage would exceed ~72 KB (at least three stages must fit)
    int rpw = 4;
    while (rpw > 1 && (uint64_t)rpw * p.G * rowb > 72 * 1024) rpw /= 2;
    p.RS = rpw * p.G;
    p.stage_bytes = (uint32_t)p.RS * rowb;
    int grid = (int)std::min<int64_t>(w->out, sm_count);
    // per-CTA partial table [rows][S] floats, at most 32 KB
    int64_t rows_cap = (w->out + grid - 1) / grid;
    while (rows_cap * p.S * 4 > 32 * 1024) {
        grid *= 2;
        rows_cap = (w->out + grid - 1) / grid;
    }
    p.red_off = kBarBytes;
    p.ring_off = (uint32_t)((kBarBytes + rows_cap * p.S * 4 + 127) & ~(int64_t)127);
    int nstage = (int)((kSmemBudget - p.ring_off) / p.stage_bytes);
    nstage = std::min(nstage, 32);
    if (nstage < 2) return set_error(RQ_ERR_UNSUPPORTED, "matvec pipeline: row of %u bytes too large", rowb);
    p.nstage = nstage;
    const size_t smem = p.ring_off + (size_t)nstage * p.stage_bytes;
    const int threads = 32 * (1 + p.S * p.G);
    switch (w->type) {
    case RQ_Q4_K: return launch_pipe_type<RQ_Q4_K>(p, rpw, grid, threads, smem, st);
    case RQ_Q3_K: return launch_pipe_type<RQ_Q3_K>(p, rpw, grid, threads, smem, st);
    default: return launch_pipe_type<RQ_Q4_0>(p, rpw, grid, threads, smem, st);
    }
}

}  // namespace rq
