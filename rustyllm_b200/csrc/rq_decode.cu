// rq_decode.cu -- one decode step (T = 1, one GPU) of the resident Llama
// loop in a single persistent launch.
//
// The launch chain of a step (8 kernels per layer) pays a fill and a drain of
// the weight stream at every kernel boundary.  Here one CTA per SM runs the
// whole step: warp 0, lane 0 streams the weight rows of every linear of
// every layer, in order, into a ring of shared-memory stages with bulk copies
// (the same per-CTA row shares and stage shapes as the M=1 pipeline), never
// waiting for activations -- only for free ring slots -- so the next linear's
// weights are already landing while the consumers finish the current one,
// run attention or the staging between linears.  The 15 consumer warps go
// through the phases of each layer separated by grid-wide barriers:
//
//   RMSNorm staging -> q/k/v -> attention -> o (+x) -> RMSNorm staging ->
//   gate/up -> SwiGLU staging -> down (+x)
//
// The step ends with the final RMSNorm, the F16 lm_head with its argmax, and
// the token bookkeeping.  Every phase uses the same thread-to-data mapping and
// arithmetic as the corresponding kernel of the launch chain (the Σx² of the
// staging with 256 threads, attention with kAttnThreads, the final norm as
// 1024 virtual threads), so the step computes the same bits.
//
// Every wait is bounded: mbarrier waits and grid barriers give up after
// ~1 s or as soon as another CTA has raised the error word, drain their
// copies and return; the host reads the error word after the step.

#include <algorithm>

#include "rq_async.cuh"
#include "rq_attn.cuh"
#include "rq_decode.cuh"
#include "rq_pipe_lane.cuh"

namespace rq {
namespace {

constexpr int kConsW = 15;                 // consumer warps
constexpr int kThreadsD = 32 * (1 + kConsW);
constexpr int kConsT = 32 * kConsW;        // 480 consumer threads
constexpr int kSmemBudgetD = 226 * 1024;  // dynamic part; a little static shared memory besides
constexpr int kRPW = 4;                    // rows per consumer warp per stage

__device__ __forceinline__ int64_t job_out(const DecParams& p, int j) {
    switch (j) {
    case 0: return p.nq;
    case 1:
    case 2: return p.nk;
    case 4:
    case 5: return p.I;
    default: return p.H;  // o, down
    }
}
__device__ __forceinline__ int job_cls(int j) { return j == 6 ? 1 : 0; }

// this CTA's contiguous share of `out` rows
__device__ __forceinline__ void rows_of(int64_t out, int64_t* rb, int* n) {
    const int64_t b = (int64_t)blockIdx.x * out / gridDim.x, e = (int64_t)(blockIdx.x + 1) * out / gridDim.x;
    *rb = b;
    *n = (int)(e - b);
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *(const volatile int*)p; }
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// mbarrier wait that also gives up once the error word is set
__device__ __forceinline__ bool mbar_wait_err(uint32_t a, uint32_t parity, const int* err) {
    if (mbar_try_wait(a, parity)) return true;
    const long long t0 = clock64();
    unsigned spins = 0;
    while (!mbar_try_wait(a, parity)) {
        if ((++spins & 255u) == 0u && ld_volatile(err)) return false;
        if (clock64() - t0 > kWaitCycles) return false;
    }
    return true;
}

// Grid-wide barrier of the consumer warps (the producer never joins): the
// arrival counter is zeroed before each launch, barrier n of the step waits
// for n * gridDim.x arrivals.  Release before arriving, acquire after.
__device__ __forceinline__ bool grid_sync(const DecParams& p, unsigned& nbar, int ct, volatile int* flag) {
    named_bar_sync(1, kConsT);
    nbar++;
    if (ct == 0) {
        int ok = ld_volatile(p.err) == 0;
        __threadfence();
        atomicAdd(p.bar, 1u);
        const unsigned target = nbar * gridDim.x;
        const long long t0 = clock64();
        unsigned spins = 0;
        while (ok && ld_acquire(p.bar) < target) {
            if ((++spins & 63u) == 0u) {
                if (ld_volatile(p.err)) ok = 0;
                else if (clock64() - t0 > kWaitCycles) {
                    atomicExch(p.err, 1);
                    ok = 0;
                }
            }
        }
        __threadfence();
        *flag = ok;
    }
    named_bar_sync(1, kConsT);
    return *flag != 0;
}

// Position in the ring of weight stages: slot, and how often the ring has
// wrapped (the slot's use count, whose parity is the mbarrier phase).
struct RingPos {
    int slot = 0, use = 0;
    __device__ __forceinline__ void next(int n) {
        if (++slot == n) {
            slot = 0;
            use++;
        }
    }
};

// ---------------------------------------------------------------- producer
template <int TYPE>
__device__ __noinline__ void produce(const DecParams& p, uint32_t full0, uint32_t empty0, uint32_t ring) {
    const uint64_t pol = policy_evict_first();
    int it = 0;
    RingPos rp;
    bool ok = true;
    for (int l = 0; l < p.n_layers && ok; l++) {
        const DecLayer& Ly = p.layers[l];
        for (int j = 0; j < 7 && ok; j++) {
            const int cls = job_cls(j);
            const uint32_t qrow = p.qrow[cls], hrow = p.hrow[cls];
            const int RS = p.RS[cls];
            int64_t rb;
            int n;
            rows_of(job_out(p, j), &rb, &n);
            for (int r0 = 0; r0 < n; r0 += RS, it++, rp.next(p.nslot)) {
                const int slot = rp.slot, use = rp.use;
                if (use > 0 && !mbar_wait_err(empty0 + 8 * slot, (use - 1) & 1, p.err)) {
                    ok = false;
                    break;
                }
                const int rows = min(RS, n - r0);
                const int64_t row = rb + r0;
                const uint32_t qb = (uint32_t)rows * qrow, hb = (uint32_t)rows * hrow;
                const uint32_t dst = ring + (uint32_t)slot * p.slot_bytes;
                mbar_expect_tx(full0 + 8 * slot, qb + hb);
                bulk_g2s(dst, Ly.qs[j] + row * qrow, qb, full0 + 8 * slot, pol);
                bulk_g2s(dst + (uint32_t)RS * qrow, Ly.hdr[j] + row * hrow, hb, full0 + 8 * slot, pol);
            }
        }
    }
    // no bulk copy may still be landing when the CTA exits
    for (int k = max(0, it - p.nslot); k < it; k++)
        if (!mbar_wait(full0 + 8 * (k % p.nslot), (k / p.nslot) & 1)) ok = false;
    if (!ok) atomicExch(p.err, 1);
}

// ----------------------------------------------------------- matvec phase
// Jobs j0 .. j0+nj-1 (same K) of layer Ly: every consumer warp waits for each
// stage and releases it; warps c < S*G compute (K-slice c % S, rows c / S,
// c / S + G, ...).  Epilogue: y = sum over slices in slice order (+ x for o
// and down).
template <int TYPE>
__device__ __noinline__ void matvec_phase(const DecParams& p, const XQ xsrc, int j0, int nj, RingPos& it, float* red,
                             const uint8_t* ring_p, uint32_t full0, uint32_t empty0, int cw, int lane, int ct,
                             bool& ok) {
    const int cls = job_cls(j0);
    const int S = p.S[cls], G = p.G[cls], RS = p.RS[cls];
    const int64_t in = cls ? p.I : p.H;
    const uint32_t qrow = p.qrow[cls], hrow = p.hrow[cls];
    const bool active = cw < S * G;
    const int s = cw % S, g = cw / S;
    typename LaneOf<TYPE>::T L;
    LaneOffsets o;
    if (active) lane_setup<TYPE>(L, o, p.nblk[cls], in, xsrc, s, lane);
    int roff = 0;
    for (int j = j0; j < j0 + nj; j++) {
        int64_t rb;
        int n;
        rows_of(job_out(p, j), &rb, &n);
        for (int r0 = 0; r0 < n; r0 += RS, it.next(p.nslot)) {
            const int slot = it.slot, use = it.use;
            if (ok && !mbar_wait_err(full0 + 8 * slot, use & 1, p.err)) {
                ok = false;
                if (lane == 0) atomicExch(p.err, 1);
            }
            if (ok && active) {
                const uint8_t* sq = ring_p + (size_t)slot * p.slot_bytes;
                const uint8_t* sh = sq + (size_t)RS * qrow;
                const int rows = min(RS, n - r0);
                float part[kRPW];
#pragma unroll
                for (int i = 0; i < kRPW; i++) {
                    const int r = g + i * G;
                    part[i] = r < rows ? lane_row<TYPE>(L, o, sq + (size_t)r * qrow, sh + (size_t)r * hrow) : 0.0f;
                }
                transpose_reduce<kRPW>(part, lane);
                if (lane_writes<kRPW>(lane)) {
                    const int r = g + row_of_lane<kRPW>(lane) * G;
                    if (r < rows) red[(roff + r0 + r) * S + s] = part[0];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * slot);
        }
        roff += n;
    }
    named_bar_sync(1, kConsT);
    roff = 0;
    for (int j = j0; j < j0 + nj; j++) {
        int64_t rb;
        int n;
        rows_of(job_out(p, j), &rb, &n);
        float* y = j == 0 ? p.q : j == 1 ? p.k : j == 2 ? p.v : j == 4 ? p.g : j == 5 ? p.u : p.x;
        const bool resid = j == 3 || j == 6;
        for (int t = ct; t < n; t += kConsT) {
            float acc = 0.0f;
            for (int k = 0; k < S; k++) acc += red[(roff + t) * S + k];
            y[rb + t] = resid ? acc + y[rb + t] : acc;
        }
        roff += n;
    }
}

// ------------------------------------------------------ the other phases

// RMSNorm staging of x with weight w into xq (the arithmetic of
// xquant_rmsnorm_kernel: Σx² by 256 threads over float4 chunks, then the
// blocks b = blockIdx.x, blockIdx.x + grid, ...).
__device__ __noinline__ void rmsnorm_stage(const DecParams& p, const float* w, int ct, float* wsum) {
    const int64_t H = p.H;
    if (ct < 256) {
        const float4* r4 = reinterpret_cast<const float4*>(p.x);
        float s2 = 0.0f;
        for (int64_t i = ct; i < H / 4; i += 256) {
            const float4 v = r4[i];
            s2 = fmaf(v.x, v.x, s2);
            s2 = fmaf(v.y, v.y, s2);
            s2 = fmaf(v.z, v.z, s2);
            s2 = fmaf(v.w, v.w, s2);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        if ((ct & 31) == 0) wsum[ct >> 5] = s2;
    }
    named_bar_sync(1, kConsT);
    float tot = 0.0f;
    for (int k = 0; k < 8; k++) tot += wsum[k];
    const float mden = sqrtf(tot / (float)H + p.eps);
    for (int64_t b = blockIdx.x + (int64_t)ct * gridDim.x; b < H / 32; b += (int64_t)kConsT * gridDim.x) {
        float v[32];
        load_block(p.x + b * 32, v);
#pragma unroll
        for (int k = 0; k < 32; k++) v[k] = v[k] / mden * w[b * 32 + k];
        stage_block(v, 0, b, H, p.xq.planes, p.xq.stats);
    }
}

// SwiGLU staging of (g, u) into xq (xquant_swiglu_kernel's arithmetic).
__device__ __noinline__ void swiglu_stage(const DecParams& p, int ct) {
    const int64_t I = p.I;
    for (int64_t b = blockIdx.x + (int64_t)ct * gridDim.x; b < I / 32; b += (int64_t)kConsT * gridDim.x) {
        float g[32], u[32];
        load_block(p.g + b * 32, g);
        load_block(p.u + b * 32, u);
#pragma unroll
        for (int k = 0; k < 32; k++) g[k] = g[k] / (1.0f + expf(-g[k])) * u[k];
        stage_block(g, 0, b, I, p.xq.planes, p.xq.stats);
    }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // order-preserving
    return ((unsigned long long)b << 32) | (0xFFFFFFFFu - idx);  // ties: lower index wins
}

// hf = rmsnorm(x, ln_f) into shared memory with rmsnorm_row_kernel's
// arithmetic (a 1024-thread block: 1024 strided partials, 32 warp butterflies,
// warp sums in order), then this CTA's lm_head rows, one warp per row
// (lm_head_kernel's per-row arithmetic), folded into *best.
__device__ __noinline__ void head_phase(const DecParams& p, int cw, int lane, int ct, float* hf, float* part,
                           unsigned long long* kb) {
    const int64_t H = p.H;
    for (int vt = ct; vt < 1024; vt += kConsT) {
        float s2 = 0.0f;
        for (int64_t i = vt; i < H; i += 1024) s2 = fmaf(p.x[i], p.x[i], s2);
        part[vt] = s2;
    }
    named_bar_sync(1, kConsT);
    for (int vw = cw; vw < 32; vw += kConsW) {  // virtual warp vw
        float s = part[vw * 32 + lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) part[1024 + vw] = s;
    }
    named_bar_sync(1, kConsT);
    float tot = 0.0f;
    for (int k = 0; k < 32; k++) tot += part[1024 + k];
    const float m = sqrtf(tot / (float)H + p.eps);
    for (int64_t i = ct; i < H; i += kConsT) hf[i] = p.x[i] / m * p.ln_f[i];
    named_bar_sync(1, kConsT);
    int64_t rb;
    int n;
    rows_of(p.vocab, &rb, &n);
    unsigned long long mykey = 0ull;
    for (int t = cw; t < n; t += kConsW) {
        const int64_t r = rb + t;
        const uint4* row = reinterpret_cast<const uint4*>(p.lm_head + r * H);
        float acc = 0.0f;
        for (int64_t c = lane; c < H / 8; c += 32) {
            uint4 u;
            asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                         : "l"(row + c));
            const float4 xa = reinterpret_cast<const float4*>(hf)[2 * c];
            const float4 xb = reinterpret_cast<const float4*>(hf)[2 * c + 1];
            const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            const float2 w2 = __half22float2(*reinterpret_cast<const __half2*>(&u.z));
            const float2 w3 = __half22float2(*reinterpret_cast<const __half2*>(&u.w));
            acc = fmaf(xa.x, w0.x, acc); acc = fmaf(xa.y, w0.y, acc);
            acc = fmaf(xa.z, w1.x, acc); acc = fmaf(xa.w, w1.y, acc);
            acc = fmaf(xb.x, w2.x, acc); acc = fmaf(xb.y, w2.y, acc);
            acc = fmaf(xb.z, w3.x, acc); acc = fmaf(xb.w, w3.y, acc);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            const unsigned long long key = argmax_key(acc, (uint32_t)r);
            mykey = key > mykey ? key : mykey;
        }
    }
    if (lane == 0) kb[cw] = mykey;
    named_bar_sync(1, kConsT);
    if (ct == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kConsW; w++) b = kb[w] > b ? kb[w] : b;
        atomicMax(p.best, b);
    }
}

template <int TYPE>
__global__ void __launch_bounds__(kThreadsD, 1) decode_step_kernel(const __grid_constant__ DecParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t full0 = smem_u32(smem), empty0 = full0 + 8 * p.nslot;
    float* red = reinterpret_cast<float*>(smem + p.red_off);
    float* scratch = reinterpret_cast<float*>(smem + p.scratch_off);
    uint8_t* ring_p = smem + p.ring_off;
    const uint32_t ring = smem_u32(ring_p);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ int flag;
    __shared__ float wsum[32];
    __shared__ unsigned long long kb[kConsW];
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nslot; i++) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, kConsW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == 0) {
        if (lane == 0) produce<TYPE>(p, full0, empty0, ring);
        return;
    }
    const int cw = warp - 1, ct = threadIdx.x - 32;
    unsigned nbar = 0;
    bool ok = true;
    RingPos it;
    // embedding row of the current token into x (this CTA's rows of x)
    {
        int32_t tok = p.tokens[0];
        tok = tok < 0 ? 0 : (tok >= p.vocab ? (int32_t)(p.vocab - 1) : tok);
        int64_t rb;
        int n;
        rows_of(p.H, &rb, &n);
        for (int t = ct; t < n; t += kConsT) p.x[rb + t] = __half2float(p.embed[(int64_t)tok * p.H + rb + t]);
    }
    ok = grid_sync(p, nbar, ct, &flag);
    for (int l = 0; l < p.n_layers; l++) {
        if (ok) rmsnorm_stage(p, p.layers[l].rms1, ct, wsum);
        ok = grid_sync(p, nbar, ct, &flag) && ok;
        matvec_phase<TYPE>(p, p.xq, 0, 3, it, red, ring_p, full0, empty0, cw, lane, ct, ok);
        ok = grid_sync(p, nbar, ct, &flag) && ok;
        if (ok && blockIdx.x < p.n_heads)
            attn_decode_head(p.q, p.k, p.v, p.layers[l].kc, p.layers[l].vc, p.rope_cos, p.rope_sin, p.pos,
                             (int)p.n_heads, (int)p.n_kv, (int)p.head_dim, (int)p.max_seq, p.xq.planes, p.xq.stats,
                             (int)blockIdx.x, ct, 1, scratch, wsum);
        ok = grid_sync(p, nbar, ct, &flag) && ok;
        matvec_phase<TYPE>(p, p.xq, 3, 1, it, red, ring_p, full0, empty0, cw, lane, ct, ok);
        ok = grid_sync(p, nbar, ct, &flag) && ok;
        if (ok) rmsnorm_stage(p, p.layers[l].rms2, ct, wsum);
        ok = grid_sync(p, nbar, ct, &flag) && ok;
        matvec_phase<TYPE>(p, p.xq, 4, 2, it, red, ring_p, full0, empty0, cw, lane, ct, ok);
        ok = grid_sync(p, nbar, ct, &flag) && ok;
        if (ok) swiglu_stage(p, ct);
        ok = grid_sync(p, nbar, ct, &flag) && ok;
        matvec_phase<TYPE>(p, p.xq, 6, 1, it, red, ring_p, full0, empty0, cw, lane, ct, ok);
        ok = grid_sync(p, nbar, ct, &flag) && ok;
    }
    // every weight stage is consumed: the ring holds the final norm's row
    float* hf = reinterpret_cast<float*>(ring_p);
    if (ok) head_phase(p, cw, lane, ct, hf, scratch, kb);
    ok = grid_sync(p, nbar, ct, &flag) && ok;
    if (ok && blockIdx.x == 0 && ct == 0) {
        const unsigned long long k = *p.best;
        const int32_t tok = (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        p.tokens[0] = tok;
        *p.pos += 1;
        const int nn = *p.nout;
        if (nn < p.max_seq) p.out[nn] = tok;
        *p.nout = nn + 1;
        *p.best = 0ull;
    }
}

}  // namespace

bool decode_plan(DecParams& p, int sm_count, size_t* smem) {
    if (p.type != RQ_Q4_K && p.type != RQ_Q3_K && p.type != RQ_Q4_0) return false;
    if (p.nq != p.H || p.head_dim % 32 || p.head_dim > 256 || p.n_heads > sm_count) return false;
    TypeInfo ti = type_info(p.type);
    const int64_t Ks[2] = {p.H, p.I};
    uint32_t slot = 0;
    for (int c = 0; c < 2; c++) {
        const int64_t S = (Ks[c] + 2047) / 2048;
        if (S > kConsW || Ks[c] % ti.block_elems) return false;
        p.S[c] = (int)S;
        p.G[c] = std::max(1, kConsW / p.S[c]);
        p.RS[c] = kRPW * p.G[c];
        p.nblk[c] = Ks[c] / ti.block_elems;
        p.qrow[c] = (uint32_t)(p.nblk[c] * ti.qs_bytes);
        p.hrow[c] = (uint32_t)(p.nblk[c] * ti.hdr_bytes);
        if (p.qrow[c] % 16 || p.hrow[c] % 16) return false;
        slot = std::max<uint32_t>(slot, (uint32_t)p.RS[c] * (p.qrow[c] + p.hrow[c]));
    }
    slot = (slot + 127) & ~127u;
    // partial-sum table: the largest phase's rows x slices
    auto share = [&](int64_t out) { return (out + sm_count - 1) / sm_count; };
    const int64_t red_f = std::max(std::max((share(p.nq) + 2 * share(p.nk)) * (int64_t)p.S[0], share(p.H) * p.S[0]),
                                   std::max(2 * share(p.I) * p.S[0], share(p.H) * p.S[1]));
    const size_t att_f = (size_t)attn_smem_floats(p.max_seq, p.head_dim);
    const size_t scr_f = std::max<size_t>(att_f, 1024 + 32);
    p.red_off = 1024;
    p.scratch_off = (uint32_t)((p.red_off + red_f * 4 + 127) & ~(int64_t)127);
    p.ring_off = (uint32_t)((p.scratch_off + scr_f * 4 + 127) & ~(size_t)127);
    const int64_t left = (int64_t)kSmemBudgetD - p.ring_off;
    const int nslot = (int)std::min<int64_t>(left / slot, 32);
    if (nslot < 2 || (size_t)nslot * slot < (size_t)p.H * 4) return false;  // the ring also holds hf
    p.slot_bytes = slot;
    p.nslot = nslot;
    *smem = p.ring_off + (size_t)nslot * slot;
    return true;
}

int launch_decode_step(const DecParams& p, int grid, size_t smem, cudaStream_t st) {
    const void* fn = p.type == RQ_Q4_K   ? (const void*)decode_step_kernel<RQ_Q4_K>
                     : p.type == RQ_Q3_K ? (const void*)decode_step_kernel<RQ_Q3_K>
                                         : (const void*)decode_step_kernel<RQ_Q4_0>;
    static bool attr_set[64][3] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int ti = p.type == RQ_Q4_K ? 0 : p.type == RQ_Q3_K ? 1 : 2;
    if (dev < 0 || dev >= 64 || !attr_set[dev][ti]) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudgetD);
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(decode step)");
        if (dev >= 0 && dev < 64) attr_set[dev][ti] = true;
    }
    int rc = cuda_error(cudaMemsetAsync(p.bar, 0, sizeof(unsigned), st), "barrier reset");
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreadsD);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    // every CTA must be resident at once: the grid barriers wait for all
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {const_cast<DecParams*>(&p)};
    return cuda_error(cudaLaunchKernelExC(&cfg, fn, args), "decode step kernel");
}

}  // namespace rq
