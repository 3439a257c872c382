// rq_matvec.cu -- activation staging, the register-streaming M=1 matvec
// kernels (fallback for shapes the bulk-copy pipeline does not take), and the
// linear dispatch.
//
//   * The activation row is staged once per call into 24-bit fixed point per
//     32-element block (three int8 planes, see rq_internal.cuh), so the inner
//     product of 4-bit quants with x is exact integer arithmetic: dp4a on the
//     nibbles as they sit in the packed bytes.
//   * In the fallback kernels a CTA owns R consecutive rows and all of K;
//     warp w takes K-slices w, w+NW, ... and streams the weights with 128-bit
//     loads straight into registers.  Per-row lane partials are folded with a
//     transpose reduction, then across warps in shared memory in a fixed
//     order, so results are deterministic.

#include <algorithm>

#include "rq_mv_common.cuh"

namespace rq {
namespace {

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// ------------------------------------------------------ activation staging

// One thread per 32-element block of one activation row.  Launched as a
// programmatic dependent: it first waits for the preceding kernel (which may
// produce x), then lets the following matvec launch so that its weight
// streaming overlaps this kernel.
// RMSNorm fused into staging.  Grid (chunks, rows): every CTA reduces the
// whole row's sum of squares (the row is L2-resident and small), then stages
// its chunk of 32-element blocks.  y = (x / m) * w with
// m = sqrt(sum(x^2) / in + eps), the order of candle_nn::ops::rms_norm.
__global__ void xquant_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                      float eps, int64_t in, int8_t* __restrict__ planes,
                                      float4* __restrict__ stats) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    __shared__ float wsum[32];
    const int64_t m = blockIdx.y;
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
    if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = s2;
    __syncthreads();
    float tot = 0.0f;
    for (int k = 0; k < (int)(blockDim.x >> 5); k++) tot += wsum[k];
    const float mden = sqrtf(tot / (float)in + eps);
    const int64_t nb = in / 32;
    const int64_t per = (nb + gridDim.x - 1) / gridDim.x;
    const int64_t b0 = blockIdx.x * per, b1 = b0 + per < nb ? b0 + per : nb;
    for (int64_t b = b0 + threadIdx.x; b < b1; b += blockDim.x) {
        float v[32];
        load_block(row + b * 32, v);
#pragma unroll
        for (int k = 0; k < 32; k++) v[k] = v[k] / mden * w[b * 32 + k];
        stage_block(v, m, b, in, planes, stats);
    }
}

// SwiGLU fused into staging: v = silu(gate) * up, silu(g) = g / (1 + exp(-g)).
__global__ void xquant_swiglu_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                     int64_t M, int64_t in, int8_t* __restrict__ planes,
                                     float4* __restrict__ stats) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int64_t nb = in / 32;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= M * nb) return;
    const int64_t m = t / nb, b = t % nb;
    float g[32], u[32];
    load_block(gate + m * in + b * 32, g);
    load_block(up + m * in + b * 32, u);
#pragma unroll
    for (int k = 0; k < 32; k++) g[k] = g[k] / (1.0f + expf(-g[k])) * u[k];
    stage_block(g, m, b, in, planes, stats);
}

struct XRows {  // activation rows to stage: row m starts at x[m] (or x[0] + m*in)
    const float* x[kMaxJobs];
    int listed;    // 0: rows are consecutive from x[0]
};

__global__ void xquant_kernel(XRows rows, int64_t M, int64_t in, int8_t* __restrict__ planes,
                              float4* __restrict__ stats) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    int64_t nb = in / 32;
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= M * nb) return;
    int64_t m = t / nb, b = t % nb;
    const float* src = (rows.listed ? rows.x[m] : rows.x[0] + m * in) + b * 32;
    float v[32];
    load_block(src, v);
    stage_block(v, m, b, in, planes, stats);
}

// ------------------------------------------------- register-streaming kernels

template <int R>
__device__ __forceinline__ void finish_rows(float (&part)[R], float (*red)[R], int lane, int warp,
                                            int nw, int64_t row0, int64_t out, float* y) {
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
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int64_t s = warp; s < nslice; s += nw) {
        const int64_t gidx = s * 32 + lane;
        const int64_t sb = gidx >> 2;
        if (sb < nsb) {
            Q4KLane L;
            q4k_lane_setup(L, planes, stats, in, sb, (int)(gidx & 3));
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int64_t row = row0 + r;
                if (row < out) {
                    const int64_t bi = row * nsb + sb;
                    const uint8_t* wp = qs + bi * 128 + 32 * (gidx & 3);
                    part[r] += q4k_lane_row(L, ldg_stream(wp), ldg_stream(wp + 16),
                                            ldg_stream(hdr + bi * 16));
                }
            }
        }
    }
    finish_rows<R>(part, red, lane, warp, nw, row0, out, y);
}

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
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int64_t s0 = warp; s0 < nslice; s0 += nw) {
        const int64_t gidx = s0 * 32 + lane;
        const int64_t sb = gidx >> 2;
        if (sb < nsb) {
            // expanded layout: 128 nibble bytes and a 20-byte header per super-block
            const int g = (int)(gidx & 3), h1 = (lane >> 2) & 1;
            Q3KLane L;
            q3k_lane_setup(L, planes, stats, in, sb, g, h1, true);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int64_t row = row0 + r;
                if (row < out) {
                    const int64_t bi = row * nsb + sb;
                    const uint8_t* base = qs + bi * 128 + 32 * g;
                    const uint32_t* hw = reinterpret_cast<const uint32_t*>(hdr + bi * 20);
                    part[r] += q3k_lane_row(L, ldg_stream(base + 16 * h1), ldg_stream(base + 16 * (1 - h1)),
                                            hw[g], hw[4]);
                }
            }
        }
    }
    finish_rows<R>(part, red, lane, warp, nw, row0, out, y);
}

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
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int64_t s = warp; s < nslice; s += nw) {
        const int64_t b0 = 2 * (s * 32 + lane);
        if (b0 < nblk) {
            Q40Lane L;
            q40_lane_setup(L, planes, stats, in, nblk, b0);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int64_t row = row0 + r;
                if (row < out) {
                    const int64_t bi = row * nblk + b0;
                    const uint4 qa = ldg_stream(qs + bi * 16);
                    const uint4 qb = L.has1 ? ldg_stream(qs + bi * 16 + 16) : make_uint4(0u, 0u, 0u, 0u);
                    const uint16_t d0 = *reinterpret_cast<const uint16_t*>(hdr + bi * 2);
                    const uint16_t d1 = L.has1 ? *reinterpret_cast<const uint16_t*>(hdr + bi * 2 + 2)
                                               : (uint16_t)0;
                    part[r] += q40_lane_row(L, qa, qb, d0, d1);
                }
            }
        }
    }
    finish_rows<R>(part, red, lane, warp, nw, row0, out, y);
}

template <int R>
int launch_mv_r(const rq_weight* w, XQ xq, float* y, int nw, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((w->out + R - 1) / R));
    cfg.blockDim = dim3((unsigned)(nw * 32));
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (w->type == RQ_Q4_K)
        e = cudaLaunchKernelEx(&cfg, mv_q4k_kernel<R>, (const uint8_t*)w->qs, (const uint8_t*)w->hdr,
                               (const int8_t*)xq.planes, (const float4*)xq.stats, y, w->out, w->nblk, w->in);
    else if (w->type == RQ_Q3_K)
        e = cudaLaunchKernelEx(&cfg, mv_q3k_kernel<R>, (const uint8_t*)w->qs, (const uint8_t*)w->hdr,
                               (const int8_t*)xq.planes, (const float4*)xq.stats, y, w->out, w->nblk, w->in);
    else
        e = cudaLaunchKernelEx(&cfg, mv_q40_kernel<R>, (const uint8_t*)w->qs, (const uint8_t*)w->hdr,
                               (const int8_t*)xq.planes, (const float4*)xq.stats, y, w->out, w->nblk, w->in);
    return cuda_error(e, "matvec kernel");
}

// M=1 register-streaming matvec for one activation row.
int launch_matvec_regs(const rq_weight* w, XQ xq, float* y, int sm_count, cudaStream_t st) {
    const int64_t nslice = (w->in + 2047) / 2048;
    const int64_t rounds = (nslice + 7) / 8;
    const int nw = (int)((nslice + rounds - 1) / rounds);
    const int64_t want = 2 * (int64_t)sm_count;
    if (w->out / 16 >= want) return launch_mv_r<16>(w, xq, y, nw, st);
    if (w->out / 8 >= want) return launch_mv_r<8>(w, xq, y, nw, st);
    return launch_mv_r<4>(w, xq, y, nw, st);
}

}  // namespace

namespace {
int launch_xquant_impl(const XRows& rows, int64_t M, int64_t in, XQ xq, cudaStream_t st) {
    int64_t n = M * (in / 32);
    if (n == 0) return RQ_OK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((n + 127) / 128));
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_error(cudaLaunchKernelEx(&cfg, xquant_kernel, rows, M, in, xq.planes, xq.stats),
                      "xquant kernel");
}
}  // namespace

namespace {
cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, cudaStream_t st, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}
}  // namespace

int launch_xquant_rmsnorm(const float* x, const float* w, float eps, int64_t M, int64_t in, XQ xq,
                          cudaStream_t st) {
    if (M == 0) return RQ_OK;
    cudaLaunchAttribute attr[1];
    // 8 blocks of 32 per CTA: e.g. 32 CTAs of 256 threads for in = 8192
    const int64_t nb = in / 32;
    const unsigned chunks = (unsigned)std::max<int64_t>(1, (nb + 7) / 8);
    cudaLaunchConfig_t cfg = pdl_config(dim3(chunks, (unsigned)M), dim3(256), st, attr);
    return cuda_error(cudaLaunchKernelEx(&cfg, xquant_rmsnorm_kernel, x, w, eps, in, xq.planes, xq.stats),
                      "xquant rmsnorm kernel");
}

int launch_xquant_swiglu(const float* gate, const float* up, int64_t M, int64_t in, XQ xq,
                         cudaStream_t st) {
    const int64_t n = M * (in / 32);
    if (n == 0) return RQ_OK;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)((n + 127) / 128)), dim3(128), st, attr);
    return cuda_error(cudaLaunchKernelEx(&cfg, xquant_swiglu_kernel, gate, up, M, in, xq.planes, xq.stats),
                      "xquant swiglu kernel");
}

int launch_xquant(const float* x, int64_t M, int64_t in, XQ xq, cudaStream_t st) {
    XRows rows{};
    rows.x[0] = x;
    rows.listed = 0;
    return launch_xquant_impl(rows, M, in, xq, st);
}

int launch_xquant_rows(const float* const* xs, int n, int64_t in, XQ xq, cudaStream_t st) {
    if (n < 1 || n > kMaxJobs) return set_error(RQ_ERR_INVALID, "xquant: %d rows", n);
    XRows rows{};
    for (int j = 0; j < n; j++) rows.x[j] = xs[j];
    rows.listed = 1;
    return launch_xquant_impl(rows, n, in, xq, st);
}

int launch_linear(const rq_weight* w, XQ xq, float* y, int64_t M, int sm_count, cudaStream_t st, int* err,
                  const PipeNext* next) {
    if (pipe_supported(w)) {
        // every activation row is one job of the pipelined kernel
        for (int64_t m0 = 0; m0 < M; m0 += kMaxJobs) {
            const int n = (int)std::min<int64_t>(kMaxJobs, M - m0);
            const rq_weight* ws[kMaxJobs];
            XQ xqs[kMaxJobs];
            float* ys[kMaxJobs];
            for (int j = 0; j < n; j++) {
                ws[j] = w;
                xqs[j] = XQ{xq.planes + (m0 + j) * 3 * w->in, xq.stats + (m0 + j) * (w->in / 32)};
                ys[j] = y + (m0 + j) * w->out;
            }
            // the last launch prefetches the hinted weights
            int rc = launch_matvec_pipe(ws, xqs, ys, n, sm_count, st, err, nullptr, nullptr, nullptr, nullptr,
                                        nullptr, m0 + n == M ? next : nullptr);
            if (rc) return rc;
        }
        return RQ_OK;
    }
    if (w->type == RQ_Q8_0 || w->type == RQ_Q6_K || w->type == RQ_Q5_K || w->type == RQ_Q2_K)
        return set_error(RQ_ERR_UNSUPPORTED,
                         "%s matvec needs the pipelined kernel: in %lld must be a multiple of %d",
                         w->type == RQ_Q8_0 ? "Q8_0" : w->type == RQ_Q6_K ? "Q6_K" : w->type == RQ_Q5_K ? "Q5_K" : "Q2_K",
                         (long long)w->in,
                         w->type == RQ_Q8_0 || w->type == RQ_Q5_K ? 256 : 1024);
    for (int64_t m = 0; m < M; m++) {
        XQ row{xq.planes + m * 3 * w->in, xq.stats + m * (w->in / 32)};
        int rc = launch_matvec_regs(w, row, y + m * w->out, sm_count, st);
        if (rc) return rc;
    }
    return RQ_OK;
}

}  // namespace rq
