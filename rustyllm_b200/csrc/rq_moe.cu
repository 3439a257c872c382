// rq_moe.cu -- Mixtral sparse-MoE layer (SparseMoe::forward,
// src/streaming_mixtral.rs:280-319) on the GPU with quantized experts.
//
//   route:    logits[t][e] = x[t] . router[e] (warp per (t, e), the F16
//             ParallelLinear gate of the reference in its exact lane order,
//             so the logits carry its bits), softmax, top-k by descending score with ties to
//             the lower expert index (the stable sort of :292-294),
//             weights p / sum(p over the selected, in rank order) (:295-302)
//   permute:  per expert, the tokens that chose it in ascending token order
//             (:292-299), by a block-wide prefix scan over token flags
//   experts:  w2(silu(w1 x) * (w3 x)) (:250-256) as matvec jobs of the
//             pipelined kernel; each job reads the staged row of its token, so
//             no gathered copy of x is made
//   combine:  y[t] = sum over the token's experts in ascending expert order
//             of weight * out (the index_add order of :306-316)
// The host reads the per-expert counts after routing (the reference moves
// the routing table to the host too, :284-286) to build the job list.

#include <string.h>

#include <algorithm>
#include <vector>

#include "rq_async.cuh"
#include "rq_internal.cuh"
#include "rq_mv_common.cuh"

struct rq_moe {
    rq_ctx* ctx;
    int E, k;
    int64_t H, F;
    __half* router;  // [E][H], F16 as ParallelLinear::new stores it
    const uint8_t** wtab = nullptr;  // device [kind gate/up/down][qs/hdr][E] expert weight pointers
    std::vector<const rq_weight*> w1, w3, w2;  // NULL for experts of other ranks (expert parallel)
    int64_t dev_plan_max = 3;  // forwards of up to this many tokens plan on the device (rq_moe_set_device_plan)
    // per-forward routing buffers, T tokens (S = T k slots), grown on demand
    int64_t cap_t = 0;
    float* logits = nullptr;     // [T][E]
    int32_t* ids = nullptr;      // [T][k] expert ids in rank order
    float* wts = nullptr;        // [T][k]
    int32_t* offs = nullptr;     // [E+1]
    int32_t* perm = nullptr;     // [S] slot -> token (expert-major)
    float* slot_w = nullptr;     // [S]
    int32_t* tok_slot = nullptr; // [T][k] token -> its slots in ascending expert order
    int32_t* slot_e = nullptr;   // [S] expert of each slot
    float* xd = nullptr;         // [T][H] device copy of host x
    float* yd = nullptr;
    float* xg = nullptr;         // [S][H] token rows in slot order (send order under EP)
    float* o = nullptr;          // [S][H] expert outputs in slot order
    float* osend = nullptr;      // [S][H] expert outputs in send order (EP)
    int32_t* idx = nullptr;      // [S] gather indices
    int32_t* cnt = nullptr;      // [world][E] slot counts of every rank (EP)
    std::vector<void*> bufs_t;
    // expert-product buffers, R rows, grown on demand
    int64_t cap_r = 0;
    float* xr = nullptr;         // [R][H] received rows (EP)
    float* g = nullptr;          // [R][F]
    float* u = nullptr;
    float* fo = nullptr;         // [R][H]
    uint8_t* xq_x = nullptr;     // M=1 pipeline staging of the rows
    uint8_t* xq_h = nullptr;     // ... of the swiglu rows
    uint8_t* xh_x = nullptr;     // tensor-core staging of the rows
    uint8_t* xh_h = nullptr;     // ... of the swiglu rows
    int* swcnt = nullptr;        // [R][F/32] SwiGLU staging arrival counters (zero between launches)
    std::vector<void*> bufs_r;
};

namespace rq {
namespace {

// One CTA per token, one warp per expert (E <= 32).  The gate is the
// reference's ParallelLinear (streaming_mixtral.rs:265,283): F16 weights, and
// dot_f32_avx2_fma's arithmetic (parallel_linear.rs:64-94), restated exactly:
// lane c (c < 8) accumulates x[8i+c] * w[8i+c] with a fused multiply-add in
// ascending i, the eight lane sums are added left to right, and a tail of
// H % 8 elements adds x*w with two roundings.  So the logits carry the bits
// of the reference's CPU gate.  The chains are sequential by definition
// (H / 8 dependent FMAs each), so everything around them is kept off their
// path: the CTA copies a chunk of x and of every expert's row into shared
// memory with asynchronous 16-byte copies, all in flight at once (H = 4096
// with 8 experts is one chunk), and each chain lane loads 16 operands into
// registers before it runs their 16 FMAs.
constexpr int kRouterSmem = 96 * 1024;

__host__ __device__ inline int router_chunk(int E) {
    int ch = kRouterSmem / (4 + 2 * E);
    return ch - ch % 8;
}

// With planes given, the CTA also stages its token's row of x for the
// pipeline matvec (xquant_kernel's arithmetic) into row t of (planes, stats).
__global__ void router_kernel(const float* __restrict__ x, const __half* __restrict__ wr, int64_t H,
                              int E, int k, float* __restrict__ logits, int32_t* __restrict__ ids,
                              float* __restrict__ wts, int8_t* __restrict__ planes, float4* __restrict__ stats) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    extern __shared__ __align__(16) uint8_t rsm[];
    __shared__ float sl[32];
    const int64_t t = blockIdx.x;
    const int e = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ch = router_chunk(E);
    float* xs = reinterpret_cast<float*>(rsm);
    __half* ws = reinterpret_cast<__half*>(rsm + (size_t)ch * 4);
    const float* xr = x + t * H;
    const int64_t chunks8 = H / 8;  // elements covered by the eight chains
    float acc = 0.0f;
    for (int64_t c0 = 0; c0 < chunks8 * 8; c0 += ch) {
        const int64_t left = chunks8 * 8 - c0;
        const int n = (int)(left < ch ? left : ch);  // a multiple of 8
        __syncthreads();
        // x rows and the F16 rows are 16-byte aligned (H % 32 == 0, c0 % 8 == 0)
        for (int i = threadIdx.x; i < n / 4; i += blockDim.x) cp_async16(xs + 4 * i, xr + c0 + 4 * i);
        for (int i = threadIdx.x; i < E * (n / 8); i += blockDim.x) {
            const int r = i / (n / 8), q = i % (n / 8);
            cp_async16(ws + (size_t)r * ch + 8 * q, wr + (int64_t)r * H + c0 + 8 * q);
        }
        cp_async_commit();
        cp_async_wait_all();
        __syncthreads();
        if (e < E && lane < 8) {
            const __half* wrow = ws + (size_t)e * ch;
            const int n8 = n / 8;
            int i0 = 0;
            for (; i0 + 16 <= n8; i0 += 16) {
                float xv[16], wv[16];
#pragma unroll
                for (int u = 0; u < 16; u++) {
                    xv[u] = xs[8 * (i0 + u) + lane];
                    wv[u] = __half2float(wrow[8 * (i0 + u) + lane]);
                }
#pragma unroll
                for (int u = 0; u < 16; u++) acc = __fmaf_rn(xv[u], wv[u], acc);
            }
            for (; i0 < n8; i0++) acc = __fmaf_rn(xs[8 * i0 + lane], __half2float(wrow[8 * i0 + lane]), acc);
        }
    }
    if (e < E) {
        const __half* wrow = wr + (int64_t)e * H;
        float sum = -0.0f;
#pragma unroll
        for (int c = 0; c < 8; c++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, acc, c));
        for (int64_t i = chunks8 * 8; i < H; i++) sum = __fadd_rn(sum, __fmul_rn(xr[i], __half2float(wrow[i])));
        if (lane == 0) {
            sl[e] = sum;
            logits[t * E + e] = sum;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // softmax_last_dim, then the k best by score (ties -> lower index)
        float mx = sl[0];
        for (int j = 1; j < E; j++) mx = fmaxf(mx, sl[j]);
        float p[32], sum = 0.0f;
        for (int j = 0; j < E; j++) { p[j] = expf(sl[j] - mx); sum += p[j]; }
        for (int j = 0; j < E; j++) p[j] = p[j] / sum;
        int pick[32];
        unsigned used = 0u;
        for (int r = 0; r < k; r++) {
            int best = -1;
            for (int j = 0; j < E; j++)
                if (!(used >> j & 1u) && (best < 0 || sl[j] > sl[best])) best = j;
            pick[r] = best;
            used |= 1u << best;
        }
        float s = 0.0f;
        for (int r = 0; r < k; r++) s += p[pick[r]];
        for (int r = 0; r < k; r++) {
            ids[t * k + r] = pick[r];
            wts[t * k + r] = p[pick[r]] / s;
        }
    }
    if (planes)
        for (int64_t b = threadIdx.x; b < H / 32; b += blockDim.x) {
            float v[32];
            load_block(xr + b * 32, v);
            stage_block(v, t, b, H, planes, stats);
        }
}

// Single CTA: expert buckets in ascending token order.  offs[E+1];
// perm[slot] = token; slot_w[slot]; slot_e[slot] = its expert; tok_slot[t][r]
// = the token's slots sorted by expert id.
__global__ void permute_kernel(const int32_t* __restrict__ ids, const float* __restrict__ wts,
                               int64_t T, int E, int k, int32_t* __restrict__ offs,
                               int32_t* __restrict__ perm, float* __restrict__ slot_w,
                               int32_t* __restrict__ tok_slot, int32_t* __restrict__ slot_e) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    __shared__ int cnt[32];
    __shared__ int base[33];
    __shared__ int warp_sum[32][32];  // [warp][expert]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    if (tid < 32) cnt[tid] = 0;
    __syncthreads();
    // counts
    for (int64_t t = tid; t < T; t += blockDim.x)
        for (int r = 0; r < k; r++) atomicAdd(&cnt[ids[t * k + r]], 1);
    __syncthreads();
    if (tid == 0) {
        base[0] = 0;
        for (int e = 0; e < E; e++) base[e + 1] = base[e] + cnt[e];
        for (int e = 0; e <= E; e++) offs[e] = base[e];
    }
    __syncthreads();
    // ordered placement, one chunk of blockDim tokens at a time
    for (int64_t t0 = 0; t0 < T; t0 += blockDim.x) {
        const int64_t t = t0 + tid;
        unsigned mask = 0u;  // experts chosen by token t
        if (t < T)
            for (int r = 0; r < k; r++) mask |= 1u << ids[t * k + r];
        // per expert: rank of token t among chosen tokens of this chunk
        int rank[32];
        for (int e = 0; e < E; e++) {
            const unsigned bal = __ballot_sync(0xffffffffu, (mask >> e) & 1u);
            rank[e] = __popc(bal & ((1u << lane) - 1u));
            if (lane == 0) warp_sum[warp][e] = __popc(bal);
        }
        __syncthreads();
        for (int e = 0; e < E; e++) {
            int before = 0;
            for (int w = 0; w < warp; w++) before += warp_sum[w][e];
            rank[e] += before;
        }
        if (t < T) {
            int slots[32];
            for (int r = 0; r < k; r++) {
                const int e = ids[t * k + r];
                const int s = base[e] + rank[e];
                perm[s] = (int32_t)t;
                slot_w[s] = wts[t * k + r];
                slot_e[s] = e;
                slots[r] = s;
            }
            // ascending expert order == ascending slot order (buckets are expert-major)
            for (int a = 1; a < k; a++)
                for (int b = a; b > 0 && slots[b - 1] > slots[b]; b--) {
                    const int tmp = slots[b];
                    slots[b] = slots[b - 1];
                    slots[b - 1] = tmp;
                }
            for (int r = 0; r < k; r++) tok_slot[t * k + r] = slots[r];
        }
        __syncthreads();
        if (tid < 32 && tid < E) {
            int tot = 0;
            for (int w = 0; w < nw; w++) tot += warp_sum[w][tid];
            base[tid] += tot;
        }
        __syncthreads();
    }
}

// y[t][c] = sum_r slot_w[s_r] * o[s_r][c], slots in ascending expert order,
// starting from zero (ys.zeros_like then index_add per expert).
__global__ void combine_kernel(const float* __restrict__ o, const float* __restrict__ slot_w,
                               const int32_t* __restrict__ tok_slot, int64_t T, int k, int64_t H,
                               float* __restrict__ y) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int64_t t = blockIdx.y;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < H; c += (int64_t)gridDim.x * blockDim.x) {
        float acc = 0.0f;
        for (int r = 0; r < k; r++) {
            const int s = tok_slot[t * k + r];
            // index_add of outputs * weight (:313-315): two roundings
            acc = __fadd_rn(acc, __fmul_rn(o[(int64_t)s * H + c], slot_w[s]));
        }
        y[t * H + c] = acc;
    }
}

// dst[r] = src[idx[r]] for rows of H floats.
__global__ void gather_kernel(const float* __restrict__ src, const int32_t* __restrict__ idx, int64_t H,
                              float* __restrict__ dst) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int64_t r = blockIdx.y, t = idx[r];
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < H; c += (int64_t)gridDim.x * blockDim.x)
        dst[r * H + c] = src[t * H + c];
}

// g = silu(g) * up, silu(v) = v / (1 + exp(-v)) (streaming_mixtral.rs:250-256).
__global__ void swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, int64_t n) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = g[i];
        g[i] = v / (1.0f + expf(-v)) * u[i];
    }
}

cudaLaunchConfig_t pdl(dim3 grid, dim3 block, cudaStream_t st, cudaLaunchAttribute* attr) {
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

template <class T>
int grow(std::vector<void*>& bufs, T** p, size_t n) {
    cudaError_t e = cudaMalloc((void**)p, std::max<size_t>(n, 1) * sizeof(T));
    if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(moe)");
    bufs.push_back((void*)*p);
    return RQ_OK;
}

int ensure_t(rq_moe* m, int64_t T, int world) {
    if (T <= m->cap_t) return RQ_OK;
    for (void* p : m->bufs_t) cudaFree(p);
    m->bufs_t.clear();
    const int64_t S = T * m->k;
    auto& b = m->bufs_t;
    int rc = RQ_OK;
    if (!rc) rc = grow(b, &m->logits, (size_t)(T * m->E));
    if (!rc) rc = grow(b, &m->ids, (size_t)S);
    if (!rc) rc = grow(b, &m->wts, (size_t)S);
    if (!rc) rc = grow(b, &m->offs, (size_t)(m->E + 1));
    if (!rc) rc = grow(b, &m->perm, (size_t)S);
    if (!rc) rc = grow(b, &m->slot_w, (size_t)S);
    if (!rc) rc = grow(b, &m->tok_slot, (size_t)S);
    if (!rc) rc = grow(b, &m->slot_e, (size_t)S);
    if (!rc) rc = grow(b, &m->xd, (size_t)(T * m->H));
    if (!rc) rc = grow(b, &m->yd, (size_t)(T * m->H));
    if (!rc) rc = grow(b, &m->xg, (size_t)(S * m->H));
    if (!rc) rc = grow(b, &m->o, (size_t)(S * m->H));
    if (!rc) rc = grow(b, &m->osend, (size_t)(S * m->H));
    if (!rc) rc = grow(b, &m->idx, (size_t)S);
    if (!rc) rc = grow(b, &m->cnt, (size_t)(world * m->E));
    m->cap_t = rc ? 0 : T;
    return rc;
}

int ensure_r(rq_moe* m, int64_t R) {
    if (R <= m->cap_r) return RQ_OK;
    for (void* p : m->bufs_r) cudaFree(p);
    m->bufs_r.clear();
    auto& b = m->bufs_r;
    int rc = RQ_OK;
    if (!rc) rc = grow(b, &m->xr, (size_t)(R * m->H));
    if (!rc) rc = grow(b, &m->g, (size_t)(R * m->F));
    if (!rc) rc = grow(b, &m->u, (size_t)(R * m->F));
    if (!rc) rc = grow(b, &m->fo, (size_t)(R * m->H));
    if (!rc) rc = grow(b, &m->xq_x, xq_bytes(R, m->H));
    if (!rc) rc = grow(b, &m->xq_h, xq_bytes(R, m->F));
    if (!rc) rc = grow(b, &m->xh_x, xh_bytes(R, m->H));
    if (!rc) rc = grow(b, &m->xh_h, xh_bytes(R, m->F));
    if (!rc) rc = grow(b, &m->swcnt, (size_t)(R * (m->F / 32)));
    // zeroed before any stream of the caller can use them
    if (!rc) rc = cuda_error(cudaMemset(m->swcnt, 0, sizeof(int) * (size_t)(R * (m->F / 32))), "counter reset");
    if (!rc) rc = cuda_error(cudaDeviceSynchronize(), "counter reset");
    m->cap_r = rc ? 0 : R;
    return rc;
}

XQ xq_view(uint8_t* base, int64_t rows, int64_t in) {
    XQ q;
    q.planes = (int8_t*)base;
    q.stats = (float4*)(base + (((size_t)rows * 3 * in + 255) & ~(size_t)255));
    return q;
}

// jobs y_j = xq row r_j * W_j^T, batched kMaxJobs per launch (same in)
struct JobList {
    std::vector<const rq_weight*> w;
    std::vector<XQ> x;
    std::vector<float*> y;
};

// jobs with M_j <= 8 on the mma.sync kernel, larger ones on tcgen05 (not
// the split-K kernel: its piece boundaries depend on the other jobs of a
// launch, and a token must give the same bits in a layer call as in an
// expert-parallel one)
int run_mm_jobs(const std::vector<MMJobDesc>& J, XH xh, int64_t rows, int sm, cudaStream_t st, int* err) {
    std::vector<MMJobDesc> sm_jobs, tc_jobs;
    for (const MMJobDesc& j : J) (j.M >= kMinTcgenM ? tc_jobs : sm_jobs).push_back(j);
    for (size_t b = 0; b < sm_jobs.size(); b += kMaxJobs) {
        const int n = (int)std::min<size_t>(kMaxJobs, sm_jobs.size() - b);
        int rc = launch_mm_small(&sm_jobs[b], n, xh, rows, sm, st, err);
        if (rc) return rc;
    }
    for (size_t b = 0; b < tc_jobs.size(); b += kMaxJobs) {
        const int n = (int)std::min<size_t>(kMaxJobs, tc_jobs.size() - b);
        int rc = launch_mm_tc(&tc_jobs[b], n, xh, rows, sm, st, err);
        if (rc) return rc;
    }
    return RQ_OK;
}

int run_jobs(const JobList& J, int sm, cudaStream_t st, int* err) {
    for (size_t b = 0; b < J.w.size(); b += kMaxJobs) {
        const int n = (int)std::min<size_t>(kMaxJobs, J.w.size() - b);
        int rc;
        if (pipe_supported(J.w[b])) {
            rc = launch_matvec_pipe(&J.w[b], &J.x[b], &J.y[b], n, sm, st, err);
        } else {
            rc = RQ_OK;
            for (int j = 0; j < n && !rc; j++) rc = launch_linear(J.w[b + j], J.x[b + j], J.y[b + j], 1, sm, st, err);
        }
        if (rc) return rc;
    }
    return RQ_OK;
}

bool is_device(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

struct Guard {
    int prev = -1;
    explicit Guard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~Guard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// A run of rows of one expert inside a row buffer.
struct Seg {
    int e;
    int64_t start, n;
};

int launch_gather(const float* src, const int32_t* idx, int64_t rows, int64_t H, float* dst, cudaStream_t st) {
    if (rows == 0) return RQ_OK;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl(dim3((unsigned)std::min<int64_t>(32, (H + 255) / 256), (unsigned)rows), dim3(256), st, attr);
    return cuda_error(cudaLaunchKernelEx(&cfg, gather_kernel, src, idx, H, dst), "gather kernel");
}

// out[r] = FFN_e(rows[r]) for the R rows of the segments (expert e of each).
// Segments of at least kMinTensorM rows run on the tensor-core kernel in
// tiles of 8 rows; the others run one M=1 pipeline job per row.  Every row's
// result depends only on that row and on its segment's size, so a token gives
// the same bits in one layer call as in an expert-parallel one.
int expert_ffn(rq_moe* m, const float* rows, int64_t R, const std::vector<Seg>& segs, float* out, cudaStream_t st) {
    if (R == 0) return RQ_OK;
    const int64_t H = m->H, F = m->F;
    const int sm = m->ctx->sm_count;
    auto use_mm = [&](const Seg& sg) {
        const size_t e = (size_t)sg.e;
        return sg.n >= kMinTensorM && mm_small_supported(m->w1[e]) && mm_small_supported(m->w3[e]) &&
               mm_small_supported(m->w2[e]);
    };
    bool any_mm = false, any_pipe = false;
    for (const Seg& sg : segs) {
        if (sg.n == 0) continue;
        if (use_mm(sg)) any_mm = true;
        else any_pipe = true;
    }
    const XQ xqx = xq_view(m->xq_x, R, H), xqh = xq_view(m->xq_h, R, F);
    const XH xhx = xh_at(m->xh_x, R, H), xhh = xh_at(m->xh_h, R, F);
    int rc = RQ_OK;
    if (any_pipe) rc = launch_xquant(rows, R, H, xqx, st);
    if (!rc && any_mm) rc = launch_xh_stage(rows, R, H, xhx, st);
    if (rc) return rc;
    JobList up, down;
    std::vector<MMJobDesc> upm, downm;
    for (const Seg& sg : segs) {
        const size_t e = (size_t)sg.e;
        if (use_mm(sg) && sg.n >= kMinTcgenM) {
            upm.push_back(MMJobDesc{m->w1[e], (int)sg.start, (int)sg.n, m->g + sg.start * F, nullptr});
            upm.push_back(MMJobDesc{m->w3[e], (int)sg.start, (int)sg.n, m->u + sg.start * F, nullptr});
            downm.push_back(MMJobDesc{m->w2[e], (int)sg.start, (int)sg.n, out + sg.start * H, nullptr});
            continue;
        }
        if (use_mm(sg)) {
            for (int64_t t0 = sg.start; t0 < sg.start + sg.n; t0 += 8) {
                const int n = (int)std::min<int64_t>(8, sg.start + sg.n - t0);
                upm.push_back(MMJobDesc{m->w1[e], (int)t0, n, m->g + t0 * F, nullptr});
                upm.push_back(MMJobDesc{m->w3[e], (int)t0, n, m->u + t0 * F, nullptr});
                downm.push_back(MMJobDesc{m->w2[e], (int)t0, n, out + t0 * H, nullptr});
            }
            continue;
        }
        for (int64_t r = sg.start; r < sg.start + sg.n; r++) {
            const XQ xr{xqx.planes + r * 3 * H, xqx.stats + r * (H / 32)};
            up.w.push_back(m->w1[e]); up.x.push_back(xr); up.y.push_back(m->g + r * F);
            up.w.push_back(m->w3[e]); up.x.push_back(xr); up.y.push_back(m->u + r * F);
            down.w.push_back(m->w2[e]);
            down.x.push_back(XQ{xqh.planes + r * 3 * F, xqh.stats + r * (F / 32)});
            down.y.push_back(out + r * H);
        }
    }
    int* err = m->ctx->derr;
    rc = run_jobs(up, sm, st, err);
    if (!rc) rc = run_mm_jobs(upm, xhx, R, sm, st, err);
    cudaLaunchAttribute attr[1];
    if (!rc && any_mm) {
        cudaLaunchConfig_t cfg = pdl(dim3(1184), dim3(256), st, attr);
        rc = cuda_error(cudaLaunchKernelEx(&cfg, swiglu_kernel, m->g, (const float*)m->u, R * F), "swiglu kernel");
        if (!rc) rc = launch_xh_stage(m->g, R, F, xhh, st);
        if (!rc && any_pipe) rc = launch_xquant(m->g, R, F, xqh, st);
    } else if (!rc) {
        rc = launch_xquant_swiglu(m->g, m->u, R, F, xqh, st);
    }
    if (!rc) rc = run_jobs(down, sm, st, err);
    if (!rc) rc = run_mm_jobs(downm, xhh, R, sm, st, err);
    return rc;
}

// The T < kMinTensorM forward with the plan on the device: routing slots in
// token-major order (slot t k + r is the r-th pick of token t, its expert
// ids[slot]), token t's row staged by the router kernel into row t of xq_x.
// Gate and up of kMaxJobs / 2 slots per launch, silu(gate) * up staged in
// their epilogue into row `slot` of xq_h; then the down projections of
// kMaxJobs / k whole tokens per launch, the weighted combine in their
// epilogue, straight into y.  Three launches for T k <= kMaxJobs / 2 with the
// router: every slot's product has the bits of the host-planned path (the
// same kernels on the same rows), and combine sums in ascending expert order.
int expert_ffn_tokens(rq_moe* m, int64_t T, float* yd, cudaStream_t st) {
    const int64_t H = m->H, F = m->F, k = m->k, S = T * k;
    const int sm = m->ctx->sm_count;
    int* err = m->ctx->derr;
    const XQ xqx = xq_view(m->xq_x, T, H), xqh = xq_view(m->xq_h, S, F);
    PipeDevWeights dw;
    memset(&dw, 0, sizeof dw);
    dw.slot_e = m->ids;
    for (int kind = 0; kind < 3; kind++) {
        dw.qs[kind] = m->wtab + (size_t)(2 * kind) * m->E;
        dw.hdr[kind] = m->wtab + (size_t)(2 * kind + 1) * m->E;
    }
    const rq_weight* ws[kMaxJobs];
    XQ xs[kMaxJobs];
    float* ys[kMaxJobs];
    int rc = RQ_OK;
    for (int64_t s0 = 0; !rc && s0 < S; s0 += kMaxJobs / 2) {
        const int n = (int)std::min<int64_t>(kMaxJobs / 2, S - s0);
        for (int i = 0; i < n; i++) {
            const int64_t s = s0 + i, t = s / k;
            const XQ xr{xqx.planes + t * 3 * H, xqx.stats + t * (H / 32)};
            ws[2 * i] = m->w1[0];
            ws[2 * i + 1] = m->w3[0];
            xs[2 * i] = xs[2 * i + 1] = xr;
            ys[2 * i] = m->g + s * F;
            ys[2 * i + 1] = m->u + s * F;
            dw.slot[2 * i] = dw.slot[2 * i + 1] = (int)s;
            dw.kind[2 * i] = 0;
            dw.kind[2 * i + 1] = 1;
        }
        const PipeSwiglu sw{xqh, m->swcnt, (int)s0};
        rc = launch_matvec_pipe(ws, xs, ys, 2 * n, sm, st, err, nullptr, nullptr, &dw, &sw);
    }
    const int64_t per = kMaxJobs / k;  // whole tokens per down launch
    for (int64_t t0 = 0; !rc && t0 < T; t0 += per) {
        const int n = (int)(std::min<int64_t>(per, T - t0) * k);
        const int64_t s0 = t0 * k;
        for (int i = 0; i < n; i++) {
            const int64_t s = s0 + i;
            ws[i] = m->w2[0];
            xs[i] = XQ{xqh.planes + s * 3 * F, xqh.stats + s * (F / 32)};
            ys[i] = m->o + s * H;
            dw.slot[i] = (int)s;
            dw.kind[i] = 2;
        }
        const PipeCombine cb{m->ids, m->wts, yd, (int)k, (int)s0};
        rc = launch_matvec_pipe(ws, xs, ys, n, sm, st, err, nullptr, nullptr, &dw, nullptr, &cb);
    }
    return rc;
}

// Router of the T local tokens (logits, ids, wts), staging their rows into
// `stage` when given.
int launch_router(rq_moe* m, const float* xs, int64_t T, const XQ* stage, cudaStream_t st) {
    const int E = m->E, k = m->k;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl(dim3((unsigned)T), dim3((unsigned)(32 * E)), st, attr);
    const int ch = router_chunk(E);
    cfg.dynamicSmemBytes = (size_t)ch * 4 + (size_t)E * ch * 2;
    static bool attr_set[64] = {};  // per device, before the first launch
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRouterSmem);
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(router)");
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    return cuda_error(cudaLaunchKernelEx(&cfg, router_kernel, xs, (const __half*)m->router, m->H, E, k, m->logits,
                                         m->ids, m->wts, stage ? stage->planes : (int8_t*)nullptr,
                                         stage ? stage->stats : (float4*)nullptr),
                      "router kernel");
}

// Expert-major permutation of the routed slots (offs, perm, slot_w, tok_slot,
// slot_e).
int launch_permute(rq_moe* m, int64_t T, cudaStream_t st) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl(dim3(1), dim3(1024), st, attr);
    return cuda_error(cudaLaunchKernelEx(&cfg, permute_kernel, (const int32_t*)m->ids, (const float*)m->wts, T, m->E,
                                         m->k, m->offs, m->perm, m->slot_w, m->tok_slot, m->slot_e),
                      "permute kernel");
}

// Router and permutation of the T local tokens; with offs / perm given they
// are copied to the host (one stream synchronisation), else everything
// stays on the device.
int route(rq_moe* m, const float* xs, int64_t T, std::vector<int32_t>* offs, std::vector<int32_t>* perm,
          cudaStream_t st) {
    const int E = m->E, k = m->k;
    int rc = launch_router(m, xs, T, nullptr, st);
    if (!rc) rc = launch_permute(m, T, st);
    if (!offs) return rc;
    offs->assign((size_t)E + 1, 0);
    perm->assign((size_t)(T * k), 0);
    if (!rc) rc = cuda_error(cudaMemcpyAsync(offs->data(), m->offs, sizeof(int32_t) * (size_t)(E + 1),
                                             cudaMemcpyDeviceToHost, st), "offsets copy");
    if (!rc) rc = cuda_error(cudaMemcpyAsync(perm->data(), m->perm, sizeof(int32_t) * (size_t)(T * k),
                                             cudaMemcpyDeviceToHost, st), "perm copy");
    if (!rc) rc = cuda_error(cudaStreamSynchronize(st), "routing sync");
    return rc;
}

int combine(rq_moe* m, int64_t T, float* yd, cudaStream_t st) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl(dim3((unsigned)std::min<int64_t>(64, (m->H + 255) / 256), (unsigned)T), dim3(256),
                                 st, attr);
    return cuda_error(cudaLaunchKernelEx(&cfg, combine_kernel, (const float*)m->o, (const float*)m->slot_w,
                                         (const int32_t*)m->tok_slot, T, m->k, m->H, yd), "combine kernel");
}

// Shared front and back of both forwards: x to the device (when needed),
// then after `body` y back to the host and the routing outputs.
// With `fused` (the device-planned path of expert_ffn_tokens) the router
// stages the rows, the experts write y and the permutation runs only for
// perm_out; `body` is not called.
template <class Body>
int moe_call(rq_moe* m, const float* x, float* y, int64_t T, int32_t* ids_out, int32_t* perm_out, cudaStream_t st,
             int world, bool host_plan, bool fused, Body&& body) {
    int rc = ensure_t(m, T, world);
    if (rc) return rc;
    const int64_t H = m->H, S = T * m->k;
    const bool x_dev = is_device(x), y_dev = is_device(y);
    const float* xs = x;
    if (!x_dev || (reinterpret_cast<uintptr_t>(x) & 15)) {
        rc = cuda_error(cudaMemcpyAsync(m->xd, x, sizeof(float) * (size_t)(T * H), cudaMemcpyDefault, st), "x copy");
        if (rc) return rc;
        xs = m->xd;
    }
    float* yd = y_dev ? y : m->yd;
    std::vector<int32_t> offs, perm;
    if (fused) {
        rc = ensure_r(m, S);
        const XQ xqx = xq_view(m->xq_x, T, H);
        if (!rc) rc = launch_router(m, xs, T, &xqx, st);
        if (!rc) rc = expert_ffn_tokens(m, T, yd, st);
        if (!rc && perm_out) rc = launch_permute(m, T, st);
    } else {
        rc = route(m, xs, T, host_plan ? &offs : nullptr, host_plan ? &perm : nullptr, st);
        if (!rc) rc = body(xs, offs, perm);
        if (!rc) rc = combine(m, T, yd, st);
    }
    if (!rc && !y_dev)
        rc = cuda_error(cudaMemcpyAsync(y, yd, sizeof(float) * (size_t)(T * H), cudaMemcpyDeviceToHost, st), "y copy");
    if (!rc && ids_out)
        rc = cuda_error(cudaMemcpyAsync(ids_out, m->ids, sizeof(int32_t) * (size_t)S, cudaMemcpyDefault, st),
                        "ids copy");
    if (!rc && perm_out) {
        if (host_plan)
            memcpy(perm_out, perm.data(), sizeof(int32_t) * (size_t)S);
        else
            rc = cuda_error(cudaMemcpyAsync(perm_out, m->perm, sizeof(int32_t) * (size_t)S, cudaMemcpyDefault, st),
                            "perm copy");
    }
    if (!rc && (!y_dev || ids_out || (perm_out && !host_plan))) {
        rc = queue_error_readback(m->ctx, st);
        if (!rc) rc = cuda_error(cudaStreamSynchronize(st), "moe sync");
        if (!rc) rc = take_kernel_error(m->ctx, st, "rq_moe_forward");
    }
    return rc;
}

}  // namespace
}  // namespace rq

using namespace rq;

extern "C" {

int rq_moe_create(rq_ctx* ctx, int n_experts, int top_k, int64_t hidden, int64_t ffn,
                  const float* router_w, const rq_weight* const* w1, const rq_weight* const* w3,
                  const rq_weight* const* w2, rq_moe** out) {
    if (!ctx || !router_w || !w1 || !w3 || !w2 || !out)
        return set_error(RQ_ERR_INVALID, "rq_moe_create: NULL argument");
    *out = nullptr;
    if (n_experts < 1 || n_experts > 32 || top_k < 1 || top_k > n_experts)
        return set_error(RQ_ERR_INVALID, "rq_moe_create: need 1 <= top_k <= n_experts <= 32");
    if (hidden <= 0 || ffn <= 0 || hidden % 32 || ffn % 32)
        return set_error(RQ_ERR_INVALID, "rq_moe_create: hidden and ffn must be positive multiples of 32");
    const int W = tp_world(ctx), me = tp_rank(ctx);
    int present = -1;
    for (int e = 0; e < n_experts; e++) {
        if (!w1[e] && !w3[e] && !w2[e] && W > 1 && e % W != me) continue;  // another rank's expert
        if (!w1[e] || !w3[e] || !w2[e]) return set_error(RQ_ERR_INVALID, "rq_moe_create: expert %d missing", e);
        if (present < 0) present = e;
        if (w1[e]->out != ffn || w1[e]->in != hidden || w3[e]->out != ffn || w3[e]->in != hidden ||
            w2[e]->out != hidden || w2[e]->in != ffn)
            return set_error(RQ_ERR_INVALID, "rq_moe_create: expert %d shapes must be w1,w3 [%lld,%lld], w2 [%lld,%lld]",
                             e, (long long)ffn, (long long)hidden, (long long)hidden, (long long)ffn);
        if (w1[e]->type != w1[present]->type || w3[e]->type != w1[present]->type || w2[e]->type != w2[present]->type)
            return set_error(RQ_ERR_INVALID, "rq_moe_create: experts must share weight types");
    }
    Guard g(ctx->device);
    rq_moe* m = new (std::nothrow) rq_moe();
    if (!m) return set_error(RQ_ERR_OOM, "host allocation failed");
    m->ctx = ctx;
    m->E = n_experts;
    m->k = top_k;
    m->H = hidden;
    m->F = ffn;
    m->w1.assign(w1, w1 + n_experts);
    m->w3.assign(w3, w3 + n_experts);
    m->w2.assign(w2, w2 + n_experts);
    // ParallelLinear::new converts the gate weight to F16
    // (parallel_linear.rs:128-131): round to nearest even
    const size_t nr = (size_t)n_experts * (size_t)hidden;
    std::vector<float> rf(nr);
    std::vector<__half> rh(nr);
    cudaError_t e = cudaMemcpy(rf.data(), router_w, sizeof(float) * nr, cudaMemcpyDefault);
    for (size_t i = 0; e == cudaSuccess && i < nr; i++) rh[i] = __float2half_rn(rf[i]);
    if (e == cudaSuccess) e = cudaMalloc(&m->router, sizeof(__half) * nr);
    if (e == cudaSuccess) e = cudaMemcpy(m->router, rh.data(), sizeof(__half) * nr, cudaMemcpyHostToDevice);
    // per-expert weight pointers for the device-planned path:
    // [kind gate, up, down][qs, hdr][E]
    std::vector<const uint8_t*> tab((size_t)6 * n_experts, nullptr);
    for (int x = 0; x < n_experts; x++) {
        const rq_weight* trip[3] = {w1[x], w3[x], w2[x]};
        for (int kind = 0; kind < 3; kind++)
            if (trip[kind]) {
                tab[(size_t)(2 * kind) * n_experts + x] = trip[kind]->qs;
                tab[(size_t)(2 * kind + 1) * n_experts + x] = trip[kind]->hdr;
            }
    }
    if (e == cudaSuccess) e = cudaMalloc((void**)&m->wtab, sizeof(void*) * tab.size());
    if (e == cudaSuccess) e = cudaMemcpy(m->wtab, tab.data(), sizeof(void*) * tab.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (m->router) cudaFree(m->router);
        if (m->wtab) cudaFree(m->wtab);
        delete m;
        return cuda_error(e, "rq_moe_create router copy");
    }
    *out = m;
    return RQ_OK;
}

int rq_moe_free(rq_moe* m) {
    if (!m) return RQ_OK;
    Guard g(m->ctx->device);
    for (void* p : m->bufs_t) cudaFree(p);
    for (void* p : m->bufs_r) cudaFree(p);
    cudaFree(m->router);
    if (m->wtab) cudaFree(m->wtab);
    delete m;
    return RQ_OK;
}

/* Forwards of up to max_tokens tokens plan on the device: every routing
 * slot is one M=1 matvec job whose expert the kernel reads from the routing
 * table, so no host synchronisation, asynchronous and graph-capturable at
 * that T, but each slot streams its expert's weights (from about 4 tokens
 * the host plan, which reads each touched expert once per segment, is
 * faster).  Default and minimum 3 (below 4 tokens both plans are the same
 * kernels and bits). */
int rq_moe_set_device_plan(rq_moe* m, int64_t max_tokens) {
    if (!m || max_tokens < 0) return set_error(RQ_ERR_INVALID, "rq_moe_set_device_plan: bad argument");
    m->dev_plan_max = std::max<int64_t>(3, max_tokens);
    return RQ_OK;
}

int rq_moe_forward(rq_ctx* ctx, rq_moe* m, const float* x, float* y, int64_t T,
                   int32_t* expert_ids_out, int32_t* perm_out, void* stream) {
    if (!ctx || !m || !x || !y) return set_error(RQ_ERR_INVALID, "rq_moe_forward: NULL argument");
    if (T < 0) return set_error(RQ_ERR_INVALID, "rq_moe_forward: T = %lld", (long long)T);
    if (T == 0) return RQ_OK;
    for (int e = 0; e < m->E; e++)
        if (!m->w1[(size_t)e])
            return set_error(RQ_ERR_INVALID, "rq_moe_forward: expert %d is not on this rank (use rq_moe_forward_ep)", e);
    Guard gd(m->ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t S = T * m->k;
    // below kMinTensorM tokens no expert gets a tensor-core segment, so the
    // kernel of every slot is known without the routing: plan on the device
    // (up to dev_plan_max tokens when the caller asks for it: every slot an
    // M=1 job, asynchronous and graph-capturable at any T)
    bool dev_plan = T <= std::max<int64_t>(kMinTensorM - 1, m->dev_plan_max) && m->k <= kMaxJobs && m->F % 32 == 0;
    for (int e = 0; e < m->E && dev_plan; e++)
        dev_plan = pipe_supported(m->w1[(size_t)e]) && pipe_supported(m->w3[(size_t)e]) &&
                   pipe_supported(m->w2[(size_t)e]);
    return moe_call(m, x, y, T, expert_ids_out, perm_out, st, 1, !dev_plan, dev_plan,
                    [&](const float* xs, const std::vector<int32_t>& offs, const std::vector<int32_t>&) {
                        int rc = ensure_r(m, S);
                        // token rows in slot (expert-major) order
                        if (!rc) rc = launch_gather(xs, m->perm, S, m->H, m->xg, st);
                        if (rc) return rc;
                        std::vector<Seg> segs;
                        for (int e = 0; e < m->E; e++) {
                            const int64_t n = offs[(size_t)e + 1] - offs[(size_t)e];
                            if (n) segs.push_back(Seg{e, offs[(size_t)e], n});
                        }
                        return expert_ffn(m, m->xg, S, segs, m->o, st);
                    });
}

int rq_moe_forward_ep(rq_ctx* ctx, rq_moe* m, const float* x, float* y, int64_t T,
                      int32_t* expert_ids_out, int32_t* perm_out, void* stream) {
    if (!ctx || !m || (T > 0 && (!x || !y))) return set_error(RQ_ERR_INVALID, "rq_moe_forward_ep: NULL argument");
    if (T < 0) return set_error(RQ_ERR_INVALID, "rq_moe_forward_ep: T = %lld", (long long)T);
    if (!ctx->tp) return set_error(RQ_ERR_INVALID, "rq_moe_forward_ep: no communicator (rq_tp_init)");
    const int W = tp_world(ctx), me = tp_rank(ctx), E = m->E;
    for (int e = me; e < E; e += W)
        if (!m->w1[(size_t)e])
            return set_error(RQ_ERR_INVALID, "rq_moe_forward_ep: expert %d belongs to rank %d and is missing", e, me);
    Guard gd(m->ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    // every rank takes the same collective steps, also for T = 0
    const int64_t S = T * m->k, H = m->H;
    auto body = [&](const float* xs, const std::vector<int32_t>& offs, const std::vector<int32_t>& perm) {
        // slot counts of every rank
        std::vector<int32_t> mine((size_t)E);
        for (int e = 0; e < E; e++) mine[(size_t)e] = offs[(size_t)e + 1] - offs[(size_t)e];
        int rc = cuda_error(cudaMemcpyAsync(m->cnt + (size_t)me * E, mine.data(), sizeof(int32_t) * (size_t)E,
                                            cudaMemcpyHostToDevice, st), "counts copy");
        if (!rc) rc = tp_allgather_bytes(ctx, m->cnt + (size_t)me * E, m->cnt, (int64_t)sizeof(int32_t) * E, st);
        std::vector<int32_t> cnt((size_t)W * E);
        if (!rc) rc = cuda_error(cudaMemcpyAsync(cnt.data(), m->cnt, sizeof(int32_t) * cnt.size(),
                                                 cudaMemcpyDeviceToHost, st), "counts copy back");
        if (!rc) rc = cuda_error(cudaStreamSynchronize(st), "counts sync");
        if (rc) return rc;
        // send order: destination rank, then its experts ascending, then slots
        std::vector<int32_t> idx_send((size_t)S), pos_of_slot((size_t)S);
        std::vector<int64_t> sbytes((size_t)W, 0), soff((size_t)W, 0), rbytes((size_t)W, 0), roff((size_t)W, 0);
        int64_t p = 0;
        for (int d = 0; d < W; d++) {
            soff[(size_t)d] = p * H * 4;
            for (int e = d; e < E; e += W)
                for (int32_t sl = offs[(size_t)e]; sl < offs[(size_t)e + 1]; sl++, p++) {
                    idx_send[(size_t)p] = perm[(size_t)sl];
                    pos_of_slot[(size_t)sl] = (int32_t)p;
                }
            sbytes[(size_t)d] = p * H * 4 - soff[(size_t)d];
        }
        // receive layout: source rank, then this rank's experts ascending
        std::vector<Seg> segs;
        int64_t R = 0;
        for (int sr = 0; sr < W; sr++) {
            roff[(size_t)sr] = R * H * 4;
            for (int e = me; e < E; e += W) {
                const int64_t n = cnt[(size_t)sr * E + e];
                if (n) segs.push_back(Seg{e, R, n});
                R += n;
            }
            rbytes[(size_t)sr] = R * H * 4 - roff[(size_t)sr];
        }
        rc = ensure_r(m, R);
        if (!rc && S)
            rc = cuda_error(cudaMemcpyAsync(m->idx, idx_send.data(), sizeof(int32_t) * (size_t)S,
                                            cudaMemcpyHostToDevice, st), "send index copy");
        if (!rc) rc = launch_gather(xs, m->idx, S, H, m->xg, st);
        if (!rc) rc = tp_alltoallv_bytes(ctx, m->xg, sbytes.data(), soff.data(), m->xr, rbytes.data(), roff.data(), st);
        if (!rc) rc = expert_ffn(m, m->xr, R, segs, m->fo, st);
        // results back to their tokens' ranks, then into slot order
        if (!rc) rc = tp_alltoallv_bytes(ctx, m->fo, rbytes.data(), roff.data(), m->osend, sbytes.data(), soff.data(), st);
        if (!rc && S)
            rc = cuda_error(cudaMemcpyAsync(m->idx, pos_of_slot.data(), sizeof(int32_t) * (size_t)S,
                                            cudaMemcpyHostToDevice, st), "slot index copy");
        if (!rc) rc = launch_gather(m->osend, m->idx, S, H, m->o, st);
        return rc;
    };
    if (T == 0) {
        // no local tokens: still take part in the exchange
        int rc = ensure_t(m, 1, W);
        if (rc) return rc;
        std::vector<int32_t> offs((size_t)E + 1, 0), perm;
        return body(x, offs, perm);
    }
    return moe_call(m, x, y, T, expert_ids_out, perm_out, st, W, true, false, body);
}

}  // extern "C"
