// rq_mv_pipe.cu -- M=1 matvec with weights staged through shared memory by
// bulk asynchronous copies (cp.async.bulk, the non-tensor TMA path).
//
// One launch runs up to kMaxJobs independent matvecs with the same weight
// type and K (the q/k/v or gate/up linears of one layer, or the rows of a
// small batch).  One persistent CTA per SM owns a contiguous range of output
// rows of every job, so its weight bytes are contiguous byte ranges of the
// device layout.  Warp 0, lane 0 is the producer: it streams stages of RS
// whole rows, job after job without a pause, into a ring of NSTAGE
// shared-memory buffers (~200 KB in flight per SM, independent of
// registers), each stage signalling an mbarrier with its byte count.
// Consumer warp (s, g) owns K-slice s (2048 elements) and rows g, g+G, ... of
// every stage.  Each lane keeps the staged activation planes (24-bit fixed
// point in three int8 planes, written by the staging kernel) of its 64
// elements in registers, multiplies them with the 4-bit quants by dp4a, and
// releases the buffer through the stage's "empty" mbarrier.  Per-row lane partials are transpose-reduced within the
// warp into a per-CTA table [row][slice]; after the last stage the table is
// summed in slice order (deterministic) and y is written.
//
// Programmatic dependent launch: every CTA allows the next kernel in the
// stream to launch at once; the producer streams weights immediately
// (weights are written only by synchronous librq calls), while consumers
// wait (griddepcontrol.wait) for the staging kernel before reading planes.
// Every mbarrier wait is bounded (~1 s); on expiry the kernel sets the error
// word, drains its in-flight copies and exits.
//
// Fused all-reduce (row-parallel linears under tensor parallelism, one job):
// instead of writing its rows of y, a CTA stores its partial rows into slot
// [its rank] of every rank's NVLink exchange buffer (posted stores, no round
// trip), release-flags every peer, waits (acquire, bounded) for the peers'
// flags of the same CTA index -- every rank runs the same grid over the same
// rows -- and sums the W slots of its own buffer in rank order into y: the
// bits of the standalone one-shot all-reduce (rq_tp.cu), without its launch
// and with only local reads after the wait.

#include <string.h>

#include <algorithm>

#include "rq_async.cuh"
#include "rq_mv_common.cuh"
#include "rq_p2p.cuh"
#include "rq_pipe_lane.cuh"

namespace rq {
namespace {

// 16 warps per CTA (one producer, up to 15 consumers) keep the register
// budget at 128 per thread: the register file is split over four schedulers
// and a fifth resident warp on one of them would cap every thread at 96.
constexpr int kMaxConsumerWarps = 15;
constexpr int kThreads = 32 * (1 + kMaxConsumerWarps);
constexpr int kSmemBudget = 227 * 1024;
constexpr int kBarBytes = 2 * 32 * 8;  // up to 32 stages: full + empty barriers

struct PipeParams {
    PipeJob jobs[kMaxJobs];
    int njobs;
    int* err;
    int64_t nblk, in;
    int S, G, RS, nstage;
    uint32_t qrow, hrow;  // device bytes per weight row (quant part, header part)
    uint32_t stage_bytes, red_off, ring_off;
    int fuse;             // 1: all-reduce y over the ranks of ar (one job)
    P2PArgs ar;
    int dev_w;            // 1: weights resolved on the device (dw)
    PipeDevWeights dw;
    int sw;               // 1: SwiGLU staging epilogue (swg)
    PipeSwiglu swg;
    int cmb;              // 1: sparse-MoE combine epilogue (cm)
    PipeCombine cm;
    PipeNext nx;          // weights of the next launch to prefetch into L2 (nx.n = 0: none)
    int rms;              // 1: RMSNorm staging epilogue (rm)
    PipeRms rm;
    int rsi_on;           // 1: outputs divided by the staged vector's RMS (ri)
    PipeRmsIn ri;
};

// This CTA's rows of a job: an even split of the job's rows over the grid,
// the same range for every job of one shape.
__device__ __forceinline__ int64_t split_point(uint32_t i, int64_t out) {
    const uint64_t prod = (uint64_t)i * (uint64_t)out;
    // 32-bit division when it fits (every shape of a model): the 64-bit one
    // is a long instruction sequence on the producer's path to its first copy
    return prod <= 0xffffffffull ? (int64_t)((uint32_t)prod / gridDim.x) : (int64_t)(prod / gridDim.x);
}
__device__ __forceinline__ void job_rows(const PipeJob& j, int64_t* rb, int* n) {
    const int64_t b = split_point(blockIdx.x, j.out);
    const int64_t e = split_point(blockIdx.x + 1, j.out);
    *rb = b;
    *n = (int)(e - b);
}

// L2 prefetch of the next launch's weights (see PipeNext): this CTA index's
// first rows of each weight in a grid of gridDim.x CTAs, the budget split
// over the weights.
__device__ __forceinline__ void prefetch_next(const PipeNext& nx) {
    const uint32_t rowb = nx.qrow + nx.hrow;
    const int64_t per = (int64_t)(nx.budget / (uint32_t)nx.n / rowb);
    for (int i = 0; i < nx.n; i++) {
        const int64_t b = (int64_t)blockIdx.x * nx.out[i] / gridDim.x;
        const int64_t e = (int64_t)(blockIdx.x + 1) * nx.out[i] / gridDim.x;
        const int64_t rows = min(e - b, per);
        if (rows <= 0) continue;
        bulk_prefetch_l2(nx.qs[i] + b * nx.qrow, (uint32_t)(rows * nx.qrow));
        bulk_prefetch_l2(nx.hdr[i] + b * nx.hrow, (uint32_t)(rows * nx.hrow));
    }
}

// The fused all-reduce epilogue of one job (see the file comment); red holds
// this CTA's [row][slice] partials.
__device__ __forceinline__ void allreduce_rows(const PipeParams& p, const float* red) {
    // every thread orders its reads (the epoch word) after the previous grids
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const PipeJob& jb = p.jobs[0];
    int64_t rb;
    int nrows;
    job_rows(jb, &rb, &nrows);
    uint8_t* own = p.ar.base[p.ar.rank];
    uint32_t* ctl = reinterpret_cast<uint32_t*>(own + kP2PCtlOff);  // epoch, done, err
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(ctl);
    const int par = (int)(e & 1u);
    const int t = threadIdx.x, W = p.ar.world, me = p.ar.rank;
    const int64_t slot = (int64_t)me * jb.out;  // this rank's slot in every buffer
    for (int i = threadIdx.x; i < nrows; i += blockDim.x) {
        float acc = 0.0f;
        for (int s = 0; s < p.S; s++) acc += red[i * p.S + s];
        const float v = jb.add ? acc + jb.add[rb + i] : acc;
#pragma unroll
        for (int r = 0; r < kP2PMaxWorld; r++)
            if (r < W) reinterpret_cast<float*>(p.ar.base[r] + par * kP2PCap)[slot + rb + i] = v;
    }
    __syncthreads();
    const size_t fslot = ((size_t)par * kP2PFlagCTAs + blockIdx.x) * kP2PMaxWorld;
    if (t < W && t != me) {
        // this CTA's rows are in place: tell rank t
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t*>(p.ar.base[t] + kP2PFlagsOff) + fslot + me, e + 1u);
    }
    bool ok = true;
    if (t < W && t != me) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(own + kP2PFlagsOff) + fslot + t;
        const long long t0 = clock64();
        while ((int)(ld_acquire_sys(f) - (e + 1u)) < 0)
            if (clock64() - t0 > kWaitCycles) {
                ok = false;
                atomicExch(ctl + 2, 1u);
                break;
            }
    }
    ok = __syncthreads_and(ok);
    if (ok) {
        const float* mine = reinterpret_cast<const float*>(own + par * kP2PCap);
        for (int i = threadIdx.x; i < nrows; i += blockDim.x) {
            float acc = mine[rb + i];
#pragma unroll
            for (int r = 1; r < kP2PMaxWorld; r++)
                if (r < W) acc = acc + mine[(int64_t)r * jb.out + rb + i];
            jb.y[rb + i] = acc;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(ctl + 1, 1u) == gridDim.x - 1u) {
            atomicExch(ctl + 1, 0u);
            atomicAdd(ctl, 1u);
        }
    }
}

// SwiGLU staging after y is written (see PipeSwiglu): a thread per 32-row
// block this CTA touched adds the CTA's gate and up rows of the block to the
// block's arrival counter; the thread that brings it to 64 reads the block's
// 32 gate and 32 up values back from L2, stages silu(g) * u
// (xquant_swiglu_kernel's arithmetic) and zeroes the counter.
__device__ __forceinline__ void swiglu_blocks(const PipeParams& p) {
    __threadfence();  // this thread's y rows are visible before any count
    __syncthreads();
    const PipeJob& j0 = p.jobs[0];
    int64_t rb;
    int nrows;
    job_rows(j0, &rb, &nrows);
    if (nrows == 0) return;
    const int64_t nb = j0.out / 32, b0 = rb / 32;
    const int nbt = (int)((rb + nrows - 1) / 32 - b0 + 1), npair = p.njobs / 2;
    for (int i = threadIdx.x; i < npair * nbt; i += blockDim.x) {
        const int pr = i / nbt;
        const int64_t b = b0 + i % nbt;
        const int64_t lo = max(rb, 32 * b), hi = min(rb + nrows, 32 * b + 32);
        const int add = 2 * (int)(hi - lo);
        const int64_t row = p.swg.row0 + pr;
        int* cnt = p.swg.cnt + row * nb + b;
        __threadfence();
        if (atomicAdd(cnt, add) + add != 64) continue;
        __threadfence();
        const float* g = p.jobs[2 * pr].y + 32 * b;
        const float* u = p.jobs[2 * pr + 1].y + 32 * b;
        float v[32];
#pragma unroll
        for (int k = 0; k < 32; k++) {
            const float gv = __ldcg(g + k), uv = __ldcg(u + k);
            v[k] = gv / (1.0f + expf(-gv)) * uv;
        }
        stage_block(v, row, b, j0.out, p.swg.xq.planes, p.swg.xq.stats);
        atomicExch(cnt, 0);
    }
}

// RMSNorm staging (see PipeRms): after this CTA's y rows are written, each
// 32-row block they touch gets the number of rows written added to its
// arrival counter; the CTA that completes the block reads it back from L2,
// stages y * w (stage_block, as the staging kernel) and stores the block's
// sum of squares, then zeroes the counter.
__device__ __forceinline__ void rms_blocks(const PipeParams& p) {
    __threadfence();  // this thread's y rows are visible before any count
    __syncthreads();
    const PipeJob& j0 = p.jobs[0];
    int64_t rb;
    int nrows;
    job_rows(j0, &rb, &nrows);
    if (nrows == 0) return;
    const int64_t b0 = rb / 32;
    const int nbt = (int)((rb + nrows - 1) / 32 - b0 + 1);
    for (int i = threadIdx.x; i < nbt; i += blockDim.x) {
        const int64_t b = b0 + i;
        const int64_t lo = max(rb, 32 * b), hi = min(rb + nrows, 32 * b + 32);
        const int add = (int)(hi - lo);
        int* cnt = p.rm.cnt + b;
        __threadfence();
        if (atomicAdd(cnt, add) + add != 32) continue;
        __threadfence();
        const float* x = j0.y + 32 * b;
        float v[32], s2 = 0.0f;
#pragma unroll
        for (int k = 0; k < 32; k++) {
            const float xv = __ldcg(x + k);
            s2 = fmaf(xv, xv, s2);
            v[k] = xv * p.rm.w[32 * b + k];
        }
        stage_block(v, 0, b, j0.out, p.rm.xq.planes, p.rm.xq.stats);
        p.rm.ss[b] = s2;
        atomicExch(cnt, 0);
    }
}

// Sparse-MoE combine (see PipeCombine): the k slots of a token are
// consecutive jobs over the same rows of this CTA, so every output row is
// finished here: the slot outputs (partials summed in slice order, the bits
// of y) weighted and summed in ascending expert order from zero.
__device__ __forceinline__ void combine_rows(const PipeParams& p, const float* red) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // ids and wts of the routing kernel
    const int k = p.cm.k, ntok = p.njobs / k;
    int64_t rb;
    int nrows;
    job_rows(p.jobs[0], &rb, &nrows);
    const int64_t H = p.jobs[0].out;
    for (int tt = 0; tt < ntok; tt++) {
        const int s0 = p.cm.slot0 + tt * k;
        int ord[kMaxJobs];
        for (int r = 0; r < k; r++) ord[r] = r;
        for (int a = 1; a < k; a++)
            for (int b = a; b > 0 && p.cm.ids[s0 + ord[b - 1]] > p.cm.ids[s0 + ord[b]]; b--) {
                const int t = ord[b];
                ord[b] = ord[b - 1];
                ord[b - 1] = t;
            }
        float* out = p.cm.out + (int64_t)(s0 / k) * H;
        for (int i = threadIdx.x; i < nrows; i += blockDim.x) {
            float acc = 0.0f;
            for (int r = 0; r < k; r++) {
                const int j = tt * k + ord[r];
                float o = 0.0f;
                for (int s = 0; s < p.S; s++) o += red[(j * nrows + i) * p.S + s];
                acc = __fadd_rn(acc, __fmul_rn(o, p.cm.wts[s0 + ord[r]]));
            }
            out[rb + i] = acc;
        }
    }
}

template <int TYPE, int RPW>
__global__ void __launch_bounds__(kThreads, 1) mv_pipe_kernel(const PipeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    // the input's RMS divisor (rsi_on), after the barriers: the dynamic
    // allocation already takes the whole shared-memory budget
    float& s_rms = *reinterpret_cast<float*>(smem + kBarBytes);
    float* red = reinterpret_cast<float*>(smem + p.red_off);
    uint8_t* ring = smem + p.ring_off;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(smem), empty0 = full0 + 8 * p.nstage;
    // the next kernel in the stream may launch now; it waits for this grid
    // before touching anything this grid writes
    asm volatile("griddepcontrol.launch_dependents;");
    if (warp == 0) {  // one lane per stage
        if (lane < p.nstage) {
            mbar_init(full0 + 8 * lane, 1);
            mbar_init(empty0 + 8 * lane, p.S * p.G);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int it = 0, slot = 0, use = 0;  // stage count, ring slot, uses of the slot
            bool ok = true;
            // weights chosen on the device: the routing table comes from an
            // earlier kernel, so wait for it before the first copy
            if (p.dev_w) asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int j = 0; j < p.njobs && ok; j++) {
                const PipeJob& jb = p.jobs[j];
                int64_t rb;
                int nrows;
                job_rows(jb, &rb, &nrows);
                const uint8_t* jqs = jb.qs;
                const uint8_t* jhdr = jb.hdr;
                if (p.dev_w) {
                    const int e = p.dw.slot_e[p.dw.slot[j]];
                    jqs = p.dw.qs[p.dw.kind[j]][e];
                    jhdr = p.dw.hdr[p.dw.kind[j]][e];
                }
                for (int r0 = 0; r0 < nrows; r0 += p.RS, it++, slot = slot + 1 == p.nstage ? 0 : slot + 1,
                         use += slot == 0) {
                    if (use > 0 && !mbar_wait(empty0 + 8 * slot, (use - 1) & 1)) { ok = false; break; }
                    const int rows = min(p.RS, nrows - r0);
                    const int64_t row = rb + r0;
                    const uint32_t qb = (uint32_t)rows * p.qrow, hb = (uint32_t)rows * p.hrow;
                    const uint32_t dst = smem_u32(ring) + (uint32_t)slot * p.stage_bytes;
                    mbar_expect_tx(full0 + 8 * slot, qb + hb);
                    bulk_g2s(dst, jqs + row * p.qrow, qb, full0 + 8 * slot, pol);
                    bulk_g2s(dst + (uint32_t)p.RS * p.qrow, jhdr + row * p.hrow, hb, full0 + 8 * slot, pol);
                }
            }
            if (ok && p.nx.n > 0) prefetch_next(p.nx);
            // no bulk copy may still be landing when the CTA exits
            for (int k = max(0, it - p.nstage); k < it; k++)
                if (!mbar_wait(full0 + 8 * (k % p.nstage), (k / p.nstage) & 1)) ok = false;
            if (!ok && p.err) atomicExch(p.err, 1);
        }
    } else if (warp - 1 < p.S * p.G) {
        const int c = warp - 1;
        const int s = c % p.S, g = c / p.S;
        typename LaneOf<TYPE>::T L;
        LaneOffsets o;
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (p.rsi_on && c == 0) {
            // the staged vector's RMS: lane sums in a fixed order, then a
            // fixed shuffle tree (the same bits in every CTA and run)
            float t = 0.0f;
            for (int i = lane; i < p.ri.nb; i += 32) t += __ldcg(p.ri.ss + i);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
            if (lane == 0) s_rms = sqrtf(t / p.ri.n + p.ri.eps);
        }
        const int8_t* cur_x = nullptr;
        int slot = 0, use = 0, roff = 0;
        bool ok = true;
        for (int j = 0; j < p.njobs && ok; j++) {
            const PipeJob& jb = p.jobs[j];
            int64_t rb;
            int nrows;
            job_rows(jb, &rb, &nrows);
            if (jb.xq.planes != cur_x) {  // jobs that share x keep the planes
                lane_setup<TYPE>(L, o, p.nblk, p.in, jb.xq, s, lane);
                cur_x = jb.xq.planes;
            }
            for (int r0 = 0; r0 < nrows; r0 += p.RS, slot = slot + 1 == p.nstage ? 0 : slot + 1, use += slot == 0) {
                if (!mbar_wait(full0 + 8 * slot, use & 1)) {
                    if (lane == 0 && p.err) atomicExch(p.err, 1);
                    ok = false;
                    break;
                }
                const uint8_t* sq = ring + (size_t)slot * p.stage_bytes;
                const uint8_t* sh = sq + (size_t)p.RS * p.qrow;
                const int rows = min(p.RS, nrows - r0);
                float part[RPW];
#pragma unroll
                for (int i = 0; i < RPW; i++) {
                    const int r = g + i * p.G;  // warp-uniform
                    part[i] = r < rows ? lane_row<TYPE>(L, o, sq + (size_t)r * p.qrow, sh + (size_t)r * p.hrow)
                                       : 0.0f;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * slot);
                transpose_reduce<RPW>(part, lane);
                if (lane_writes<RPW>(lane)) {
                    const int r = g + row_of_lane<RPW>(lane) * p.G;
                    if (r < rows) red[(roff + r0 + r) * p.S + s] = part[0];
                }
            }
            roff += nrows;
        }
    }
    __syncthreads();
    if (p.fuse) {
        allreduce_rows(p, red);
        if (p.rms) rms_blocks(p);  // every rank holds the summed rows: each stages its own copy
        return;
    }
    if (p.cmb) {
        combine_rows(p, red);
        return;
    }
    int roff = 0;
    const float rdiv = p.rsi_on ? s_rms : 1.0f;
    for (int j = 0; j < p.njobs; j++) {
        int64_t rb;
        int nrows;
        job_rows(p.jobs[j], &rb, &nrows);
        const float* add = p.jobs[j].add;
        for (int t = threadIdx.x; t < nrows; t += blockDim.x) {
            float acc = 0.0f;
            for (int s = 0; s < p.S; s++) acc += red[(roff + t) * p.S + s];
            if (p.rsi_on) acc = acc / rdiv;
            p.jobs[j].y[rb + t] = add ? acc + add[rb + t] : acc;
        }
        roff += nrows;
    }
    if (p.sw) swiglu_blocks(p);
    if (p.rms) rms_blocks(p);
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

PipeNext pipe_next(const rq_weight* const* ws, int n, uint32_t budget) {
    PipeNext nx;
    memset(&nx, 0, sizeof nx);
    if (n < 1 || n > kMaxNext) return nx;
    const TypeInfo ti = type_info(ws[0]->type);
    for (int i = 0; i < n; i++)
        if (ws[i]->type != ws[0]->type || ws[i]->in != ws[0]->in) return nx;
    nx.qrow = (uint32_t)(ws[0]->nblk * ti.qs_bytes);
    nx.hrow = (uint32_t)(ws[0]->nblk * ti.hdr_bytes);
    if (nx.qrow % 16 || nx.hrow % 16) return nx;
    for (int i = 0; i < n; i++) {
        nx.qs[i] = ws[i]->qs;
        nx.hdr[i] = ws[i]->hdr;
        nx.out[i] = ws[i]->out;
    }
    nx.n = n;
    nx.budget = budget;
    return nx;
}

bool pipe_supported(const rq_weight* w) {
    TypeInfo ti = type_info(w->type);
    const int64_t S = (w->in + 2047) / 2048;
    if (S > kMaxConsumerWarps) return false;
    const int64_t qrow = w->nblk * ti.qs_bytes, hrow = w->nblk * ti.hdr_bytes;
    if (qrow % 16 || hrow % 16) return false;  // bulk copies move 16-byte multiples
    if (qrow + hrow > 64 * 1024) return false;
    return true;
}

int launch_matvec_pipe(const rq_weight* const* ws, const XQ* xqs, float* const* ys, int njobs,
                       int sm_count, cudaStream_t st, int* err, const float* const* adds, const P2PArgs* ar,
                       const PipeDevWeights* dw, const PipeSwiglu* sw, const PipeCombine* cmb,
                       const PipeNext* next, const PipeRms* rms, const PipeRmsIn* rsi) {
    if (njobs < 1 || njobs > kMaxJobs) return set_error(RQ_ERR_INVALID, "matvec pipeline: %d jobs", njobs);
    const rq_weight* w0 = ws[0];
    TypeInfo ti = type_info(w0->type);
    PipeParams p;
    p.njobs = njobs;
    for (int j = 0; j < njobs; j++) {
        p.jobs[j].qs = ws[j]->qs;
        p.jobs[j].hdr = ws[j]->hdr;
        p.jobs[j].xq = xqs[j];
        p.jobs[j].y = ys[j];
        p.jobs[j].add = adds ? adds[j] : nullptr;
        p.jobs[j].out = ws[j]->out;
    }
    p.err = err;
    p.dev_w = dw ? 1 : 0;
    if (dw) p.dw = *dw;
    bool same_shape = true;
    for (int j = 1; j < njobs; j++) same_shape = same_shape && ws[j]->out == w0->out;
    bool any_add = false;
    for (int j = 0; adds && j < njobs; j++) any_add = any_add || adds[j];
    p.sw = 0;
    p.cmb = 0;
    if (sw) {
        if (njobs % 2 || !same_shape || ar || cmb || any_add || w0->out % 32 || !sw->cnt || sw->row0 < 0)
            return set_error(RQ_ERR_INVALID, "matvec pipeline: SwiGLU staging needs gate/up pairs of one shape");
        p.sw = 1;
        p.swg = *sw;
    }
    if (cmb) {
        if (cmb->k < 1 || njobs % cmb->k || cmb->slot0 < 0 || cmb->slot0 % cmb->k || !same_shape || ar || any_add ||
            !cmb->ids || !cmb->wts || !cmb->out)
            return set_error(RQ_ERR_INVALID, "matvec pipeline: combine needs whole tokens of one shape");
        p.cmb = 1;
        p.cm = *cmb;
    }
    p.rms = 0;
    p.rsi_on = 0;
    if (rms) {
        if (njobs != 1 || cmb || sw || w0->out % 32 || !rms->cnt || !rms->ss || !rms->w)
            return set_error(RQ_ERR_INVALID, "matvec pipeline: RMSNorm staging needs one job of whole blocks");
        p.rms = 1;
        p.rm = *rms;
    }
    if (rsi) {
        if (ar || cmb || !rsi->ss || rsi->nb < 1 || !(rsi->n > 0.0f))
            return set_error(RQ_ERR_INVALID, "matvec pipeline: bad RMS input");
        p.rsi_on = 1;
        p.ri = *rsi;
    }
    memset(&p.nx, 0, sizeof p.nx);
    if (next && next->n > 0 && next->n <= kMaxNext && next->qrow % 16 == 0 && next->hrow % 16 == 0) p.nx = *next;
    p.nblk = w0->nblk;
    p.in = w0->in;
    p.S = (int)((w0->in + 2047) / 2048);
    p.G = std::max(1, kMaxConsumerWarps / p.S);
    p.qrow = (uint32_t)(w0->nblk * ti.qs_bytes);
    p.hrow = (uint32_t)(w0->nblk * ti.hdr_bytes);
    const uint32_t rowb = p.qrow + p.hrow;
    // RS = RPW * G whole rows per stage; four rows per consumer warp unless
    // a stage would exceed ~72 KB (at least three stages must fit)
    int rpw = 4;
    while (rpw > 1 && (uint64_t)rpw * p.G * rowb > 72 * 1024) rpw /= 2;
    p.RS = rpw * p.G;
    p.stage_bytes = (uint32_t)p.RS * rowb;
    int64_t max_out = 0;
    for (int j = 0; j < njobs; j++) max_out = std::max(max_out, ws[j]->out);
    int grid = (int)std::min<int64_t>(max_out, sm_count);
    // per-CTA partial table [rows of all jobs][S] floats, at most 32 KB
    auto rows_cap = [&](int gr) {
        int64_t r = 0;
        for (int j = 0; j < njobs; j++)
            r += (ws[j]->out + gr - 1) / gr;
        return r;
    };
    while (rows_cap(grid) * p.S * 4 > 32 * 1024) grid *= 2;
    p.fuse = 0;
    if (ar) {
        // every CTA must be resident at once (it waits for its peers), and
        // the flags and the exchange buffer must hold the grid and the rows
        if (njobs != 1 || grid > sm_count || grid > kP2PFlagCTAs || ar->world > kP2PMaxWorld ||
            (size_t)ar->world * w0->out * 4 > kP2PCap)
            return kPipeNotFusable;
        p.fuse = 1;
        p.ar = *ar;
    }
    p.red_off = kBarBytes + 16;  // 16 bytes of scalars after the barriers
    p.ring_off = (uint32_t)((p.red_off + rows_cap(grid) * p.S * 4 + 127) & ~(int64_t)127);
    int nstage = (int)((kSmemBudget - p.ring_off) / p.stage_bytes);
    nstage = std::min(nstage, 32);
    if (nstage < 2) return set_error(RQ_ERR_UNSUPPORTED, "matvec pipeline: row of %u bytes too large", rowb);
    p.nstage = nstage;
    const size_t smem = p.ring_off + (size_t)nstage * p.stage_bytes;
    const int threads = 32 * (1 + p.S * p.G);
    switch (w0->type) {
    case RQ_Q4_K: return launch_pipe_type<RQ_Q4_K>(p, rpw, grid, threads, smem, st);
    case RQ_Q3_K: return launch_pipe_type<RQ_Q3_K>(p, rpw, grid, threads, smem, st);
    case RQ_Q8_0: return launch_pipe_type<RQ_Q8_0>(p, rpw, grid, threads, smem, st);
    case RQ_Q6_K: return launch_pipe_type<RQ_Q6_K>(p, rpw, grid, threads, smem, st);
    case RQ_Q5_K: return launch_pipe_type<RQ_Q5_K>(p, rpw, grid, threads, smem, st);
    case RQ_Q2_K: return launch_pipe_type<RQ_Q2_K>(p, rpw, grid, threads, smem, st);
    default: return launch_pipe_type<RQ_Q4_0>(p, rpw, grid, threads, smem, st);
    }
}

}  // namespace rq
