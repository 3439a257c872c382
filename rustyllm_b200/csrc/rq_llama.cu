// rq_llama.cu -- the quantized Llama decode loop on the GPU: the forward of
// StreamingLlamaQuantized (src/streaming_quantized.rs:622-729) with every
// QBlock resident (src/streaming_quantized.rs:282-318) and the greedy step of
// generate (src/streaming_quantized.rs:539-593).
//
// Per layer (T tokens):
//   stage(rmsnorm(x, rms_1))      -> q, k, v  (one batched matvec launch)
//   rope(q, k); append k, v to the layer's KV cache at pos .. pos+T-1
//   attention (GQA, causal, softmax in f32)  -> a
//   stage(a) -> o_proj, + residual x          (epilogue add)
//   stage(rmsnorm(x, rms_2))      -> gate, up (one batched launch)
//   stage(silu(gate) * up)        -> down, + residual x
// then rmsnorm(x[T-1], ln_f), the F16 lm_head matvec fused with a
// first-index argmax, and the device-side token / position update.  The
// decode step (T = 1) reads its token and position from device memory, so a
// whole step can be captured in one CUDA graph.
//
// Numerics follow the reference: activations, KV cache and attention in f32;
// embedding and lm_head weights F16 (exact GGUF F16 values, dequantized to
// f32 before use); RoPE tables computed on the host in f32 exactly as
// QuantStreamCache::new does.

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "rq_attn.cuh"
#include "rq_decode.cuh"
#include "rq_p2p.cuh"
#include "rq_mv_common.cuh"

struct rq_llama {
    rq_ctx* ctx;
    rq_llama_config cfg;
    struct Layer {
        const rq_weight* w[7];  // q, k, v, o, gate, up, down (borrowed)
        float* rms1;
        float* rms2;
        float* kc;  // [n_kv][max_seq][head_dim]
        float* vc;
    };
    std::vector<Layer> layers;
    __half* embed;    // [vocab][hidden]
    float* ln_f;      // [hidden]
    __half* lm_head;  // [vocab][hidden]
    float* rope_cos;  // [max_seq][head_dim/2]
    float* rope_sin;
    // activations
    float* x;     // [Tmax][hidden] residual stream
    float* q;     // [Tmax][n_heads*head_dim]
    float* k;     // [Tmax][n_kv*head_dim]
    float* v;
    float* att;   // [Tmax][n_heads*head_dim]
    float* g;     // [Tmax][intermediate]
    float* u;
    float* hf;    // [hidden] final normed row
    float* logits;  // [vocab / W]
    float* logits_all;  // [Tmax][vocab / W] (forward_all)
    unsigned long long* keys;  // [Tmax] per-position argmax keys (forward_all)
    int32_t* amax;             // [Tmax] per-position argmax tokens
    float* part;    // [Tmax][hidden] row-parallel partial sums (W > 1)
    int W, R;       // tensor-parallel world and rank
    int64_t nh_l, nkv_l, I_l, vocab_l;  // this rank's heads, kv heads, ffn rows, vocab rows
    rq::XQ xq;      // Tmax rows of max(hidden, intermediate)
    rq::XQ xqd;     // one row of the local intermediate: the down projection's input at decode
    int* swcnt;     // [I / 32] arrival counters of the decode SwiGLU staging (zero between launches)
    rq::XQ xqr;     // one row of the hidden size: the RMSNorm staging of the o / down epilogues at decode
    float* rss;     // [H / 32] its block sums of squares
    int* rcnt;      // [H / 32] its arrival counters (zero between launches)
    rq::PipeNext nx{};  // L2 prefetch hint for the decode matvec being launched (nx.n = 0: none)
    float* i8part;      // [4][8][hidden] split-K partial rows of the int8 down projection (T = 2..8)
    int* i8cnt;         // [256] its arrival counters (zero between launches)
    rq::XH xh;      // the same rows staged as f16 hi / lo (tensor-core prefill)
    // device state
    unsigned long long* best;  // packed (value, -index) of the argmax
    int32_t* tokens;           // [Tmax] current input tokens
    int32_t* pos;              // current position (KV length before this step)
    int32_t* out;              // [max_seq] generated tokens
    int32_t* nout;
    // one-launch decode step (rq_decode.cu)
    rq::DecLayer* dlayers;              // device copy of the per-layer table
    std::vector<rq::DecLayer> hlayers;  // host copy
    std::vector<bool> layer_set;
    unsigned* bar;                      // grid-barrier arrivals
    int* derr;                          // error word of the step
    bool fused = false;                 // rq_llama_set_fused
    std::vector<void*> allocs;
    std::vector<rq_weight*> owned;  // weights uploaded by rq_llama_load_gguf_dir
};

namespace rq {
namespace {

cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
}

// x[t][:] = f32(embed[tokens[t]][:])  (Embedding::forward over F16 weights
// dequantized to f32 by GgufLayer::tensor)
// The RMSNorm staging of PipeRms as a kernel (used when a tensor-parallel
// o / down projection falls back to the separate all-reduce): thread b
// stages x * w over block b and stores the block's sum of squares, the
// epilogue's arithmetic.
__global__ void rms_stage_kernel(const float* __restrict__ x, const float* __restrict__ w, int64_t H,
                                 int8_t* __restrict__ planes, float4* __restrict__ stats, float* __restrict__ ss) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= H / 32) return;
    float v[32], s2 = 0.0f;
#pragma unroll
    for (int k = 0; k < 32; k++) {
        const float xv = x[32 * b + k];
        s2 = fmaf(xv, xv, s2);
        v[k] = xv * w[32 * b + k];
    }
    stage_block(v, 0, b, H, planes, stats);
    ss[b] = s2;
}

__global__ void embed_kernel(const __half* __restrict__ emb, const int32_t* __restrict__ tokens,
                             int64_t T, int64_t hidden, int64_t vocab, float* __restrict__ x) {
    pdl_enter();
    const int64_t t = blockIdx.y;
    if (t >= T) return;
    int32_t tok = tokens[t];
    tok = tok < 0 ? 0 : (tok >= vocab ? (int32_t)(vocab - 1) : tok);
    const __half* row = emb + (int64_t)tok * hidden;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += (int64_t)gridDim.x * blockDim.x)
        x[t * hidden + i] = __half2float(row[i]);
}

// RoPE (candle_nn::rotary_emb::rope, non-interleaved halves) on q and k of
// token t at position pos+t, and the KV-cache append.
// grid (n_heads + n_kv, T), block head_dim/2.
__global__ void rope_append_kernel(float* __restrict__ q, const float* __restrict__ k,
                                   const float* __restrict__ v, float* __restrict__ kc,
                                   float* __restrict__ vc, const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, const int32_t* __restrict__ pos,
                                   int n_heads, int n_kv, int hd, int max_seq) {
    pdl_enter();
    const int hh = blockIdx.x, t = blockIdx.y, i = threadIdx.x, half = hd / 2;
    const int p = *pos + t;
    if (p >= max_seq || i >= half) return;
    const float c = cos_t[(int64_t)p * half + i], s = sin_t[(int64_t)p * half + i];
    if (hh < n_heads) {
        float* qh = q + ((int64_t)t * n_heads + hh) * hd;
        const float a = qh[i], b = qh[i + half];
        qh[i] = a * c - b * s;
        qh[i + half] = a * s + b * c;
    } else {
        const int kh = hh - n_heads;
        const float* kh_src = k + ((int64_t)t * n_kv + kh) * hd;
        const float* vh_src = v + ((int64_t)t * n_kv + kh) * hd;
        float* kdst = kc + ((int64_t)kh * max_seq + p) * hd;
        float* vdst = vc + ((int64_t)kh * max_seq + p) * hd;
        const float a = kh_src[i], b = kh_src[i + half];
        kdst[i] = a * c - b * s;
        kdst[i + half] = a * s + b * c;
        vdst[i] = vh_src[i];
        vdst[i + half] = vh_src[i + half];
    }
}

// Causal GQA attention for query token t of head h (QAttn::forward,
// src/streaming_quantized.rs:241-255): scores = q.k / sqrt(hd) over the
// pos+t+1 cached keys of kv head h / (n_heads / n_kv), softmax, weighted sum
// of values.  grid (n_heads, T), block 128, dynamic smem max_seq floats.
__global__ void attention_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                 const float* __restrict__ vc, const int32_t* __restrict__ pos,
                                 int n_heads, int n_kv, int hd, int max_seq, float* __restrict__ out) {
    pdl_enter();
    extern __shared__ float sc[];
    __shared__ float red[32];
    const int h = blockIdx.x, t = blockIdx.y;
    const int L = min(*pos + t + 1, max_seq);
    const int kh = h / (n_heads / n_kv);
    const float* qh = q + ((int64_t)t * n_heads + h) * hd;
    const float* K = kc + (int64_t)kh * max_seq * hd;
    const float* V = vc + (int64_t)kh * max_seq * hd;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const float inv_sqrt = 1.0f / sqrtf((float)hd);
    for (int j = warp; j < L; j += nw) {
        float acc = 0.0f;
        for (int d = lane; d < hd; d += 32) acc = fmaf(qh[d], K[(int64_t)j * hd + d], acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) sc[j] = acc * inv_sqrt;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < L; j += blockDim.x) mx = fmaxf(mx, sc[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < nw; w++) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float sum = 0.0f;
    for (int j = threadIdx.x; j < L; j += blockDim.x) {
        const float e = expf(sc[j] - mx);
        sc[j] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    sum = 0.0f;
    for (int w = 0; w < nw; w++) sum += red[w];
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.0f;
        for (int j = 0; j < L; j++) acc = fmaf(sc[j] / sum, V[(int64_t)j * hd + d], acc);
        out[((int64_t)t * n_heads + h) * hd + d] = acc;
    }
}

// Decode (T = 1) attention fused with RoPE, the KV-cache append and the
// staging of the head's output for o_proj (attn_decode_head): one CTA of
// kAttnThreads threads per head, dynamic smem attn_smem_floats floats.
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, float* __restrict__ kc,
    float* __restrict__ vc, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
    const int32_t* __restrict__ pos, int n_heads, int n_kv, int hd, int max_seq, int8_t* __restrict__ planes,
    float4* __restrict__ stats) {
    pdl_enter();
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[32];
    attn_decode_head(q, k, v, kc, vc, cos_t, sin_t, pos, n_heads, n_kv, hd, max_seq, planes, stats, (int)blockIdx.x,
                     (int)threadIdx.x, 0, sm, red);
}

// hf = rmsnorm(x[row], w) for one row (the lm_head input).
__global__ void rmsnorm_row_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                   float eps, int64_t hidden, float* __restrict__ y) {
    pdl_enter();
    __shared__ float wsum[32];
    float s2 = 0.0f;
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) s2 = fmaf(x[i], x[i], s2);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = s2;
    __syncthreads();
    float tot = 0.0f;
    for (int k = 0; k < (int)(blockDim.x >> 5); k++) tot += wsum[k];
    const float m = sqrtf(tot / (float)hidden + eps);
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) y[i] = x[i] / m * w[i];
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // order-preserving
    return ((unsigned long long)b << 32) | (0xFFFFFFFFu - idx);  // ties: lower index wins
}

// logits[r] = sum_k hf[k] * f32(W[r][k]) over an F16 [vocab][hidden] matrix,
// one warp per row, 16-byte streaming loads; the block's best (value, row +
// row_offset) is folded into *best with one atomicMax.  hidden % 8 == 0.
__global__ void __launch_bounds__(256) lm_head_kernel(const __half* __restrict__ W,
                                                      const float* __restrict__ hf, int64_t vocab,
                                                      int64_t hidden, int64_t row_offset,
                                                      float* __restrict__ logits,
                                                      unsigned long long* __restrict__ best) {
    extern __shared__ float xs[];
    pdl_enter();
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) xs[i] = hf[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long mykey = 0ull;
    for (int64_t r = (int64_t)blockIdx.x * 8 + warp; r < vocab; r += (int64_t)gridDim.x * 8) {
        const uint4* row = reinterpret_cast<const uint4*>(W + r * hidden);
        float acc = 0.0f;
        for (int64_t c = lane; c < hidden / 8; c += 32) {
            uint4 u;
            asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                         : "l"(row + c));
            const float4 xa = reinterpret_cast<const float4*>(xs)[2 * c];
            const float4 xb = reinterpret_cast<const float4*>(xs)[2 * c + 1];
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
            if (logits) logits[r] = acc;
            const unsigned long long key = argmax_key(acc, (uint32_t)(r + row_offset));
            mykey = key > mykey ? key : mykey;
        }
    }
    __shared__ unsigned long long kb[8];
    if (lane == 0) kb[warp] = mykey;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long k = kb[0];
        for (int w = 1; w < 8; w++) k = kb[w] > k ? kb[w] : k;
        atomicMax(best, k);
    }
}

// lm_head_kernel for NT rows of hf at once (the verify forward): the F16
// matrix is read once; every row's accumulation has the single-row order.
template <int NT>
__global__ void __launch_bounds__(256) lm_head_rows_kernel(const __half* __restrict__ W,
                                                           const float* __restrict__ hf, int64_t vocab,
                                                           int64_t hidden, int64_t row_offset,
                                                           float* __restrict__ logits,
                                                           unsigned long long* __restrict__ best) {
    extern __shared__ float xs[];  // [NT][hidden]
    pdl_enter();
    for (int64_t i = threadIdx.x; i < NT * hidden; i += blockDim.x) xs[i] = hf[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long mykey[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) mykey[t] = 0ull;
    for (int64_t r = (int64_t)blockIdx.x * 8 + warp; r < vocab; r += (int64_t)gridDim.x * 8) {
        const uint4* row = reinterpret_cast<const uint4*>(W + r * hidden);
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.0f;
        for (int64_t c = lane; c < hidden / 8; c += 32) {
            uint4 u;
            asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                         : "l"(row + c));
            const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            const float2 w2 = __half22float2(*reinterpret_cast<const __half2*>(&u.z));
            const float2 w3 = __half22float2(*reinterpret_cast<const __half2*>(&u.w));
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float4 xa = reinterpret_cast<const float4*>(xs + t * hidden)[2 * c];
                const float4 xb = reinterpret_cast<const float4*>(xs + t * hidden)[2 * c + 1];
                float a = acc[t];
                a = fmaf(xa.x, w0.x, a); a = fmaf(xa.y, w0.y, a);
                a = fmaf(xa.z, w1.x, a); a = fmaf(xa.w, w1.y, a);
                a = fmaf(xb.x, w2.x, a); a = fmaf(xb.y, w2.y, a);
                a = fmaf(xb.z, w3.x, a); a = fmaf(xb.w, w3.y, a);
                acc[t] = a;
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
        }
        if (lane == 0) {
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (logits) logits[t * vocab + r] = acc[t];
                const unsigned long long key = argmax_key(acc[t], (uint32_t)(r + row_offset));
                mykey[t] = key > mykey[t] ? key : mykey[t];
            }
        }
    }
    __shared__ unsigned long long kb[NT][8];
    if (lane == 0)
#pragma unroll
        for (int t = 0; t < NT; t++) kb[t][warp] = mykey[t];
    __syncthreads();
    if (threadIdx.x < NT) {
        unsigned long long k = kb[threadIdx.x][0];
        for (int w = 1; w < 8; w++) k = kb[threadIdx.x][w] > k ? kb[threadIdx.x][w] : k;
        atomicMax(best + threadIdx.x, k);
    }
}

// y[row] = rmsnorm(x[row], w) for every row (blockIdx.x), the math of
// rmsnorm_row_kernel.
__global__ void rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps,
                                    int64_t hidden, float* __restrict__ y) {
    pdl_enter();
    __shared__ float wsum[32];
    const float* xr = x + (int64_t)blockIdx.x * hidden;
    float* yr = y + (int64_t)blockIdx.x * hidden;
    float s2 = 0.0f;
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) s2 = fmaf(xr[i], xr[i], s2);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = s2;
    __syncthreads();
    float tot = 0.0f;
    for (int k = 0; k < (int)(blockDim.x >> 5); k++) tot += wsum[k];
    const float m = sqrtf(tot / (float)hidden + eps);
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) yr[i] = xr[i] / m * w[i];
}

// argmax tokens of T packed keys; the keys are cleared for the next call
__global__ void unpack_argmax_kernel(unsigned long long* keys, int T, int32_t* out) {
    pdl_enter();
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        out[t] = (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[t] & 0xFFFFFFFFull));
    }
}

// Greedy step bookkeeping: next token = argmax, appended to the output list;
// position advances by T; the argmax slot is cleared for the next step.
__global__ void finish_step_kernel(unsigned long long* best, int32_t* tokens, int32_t* pos,
                                   int32_t* out, int32_t* nout, int T, int max_out) {
    pdl_enter();
    const unsigned long long k = *best;
    const int32_t tok = (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    tokens[0] = tok;
    *pos += T;
    const int n = *nout;
    if (n < max_out) out[n] = tok;
    *nout = n + 1;
    *best = 0ull;
}

__global__ void add_rows_kernel(float* __restrict__ y, const float* __restrict__ a, int64_t n) {
    pdl_enter();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] += a[i];
}

int launch_simple(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args,
                  const char* what) {
    if (smem > 48 * 1024) {
        int rc = cuda_error(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), what);
        if (rc) return rc;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(grid, block, smem, st, attr);
    return cuda_error(cudaLaunchKernelExC(&cfg, fn, args), what);
}

// Decode (T = 1) prefetch hints: each matvec of the layer chain prefetches
// into L2 the first rows of the weights the next matvec reads (see
// PipeNext); the q/k/v matvec prefetches all of o_proj, whose launch waits
// for attention.  RQ_L2_PREFETCH=0 turns the hints off.
constexpr uint32_t kNextBudget = 128 * 1024;     // bytes per CTA across a launch boundary
constexpr uint32_t kNextBudgetAttn = 288 * 1024; // q/k/v -> o: attention runs in between

bool l2_prefetch_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("RQ_L2_PREFETCH");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

void set_next(rq_llama* m, const rq_weight* const* ws, int n, uint32_t budget) {
    m->nx = PipeNext{};
    if (n > 0 && l2_prefetch_enabled()) m->nx = pipe_next(ws, n, budget);
}

const PipeNext* next_hint(const rq_llama* m) { return m->nx.n > 0 ? &m->nx : nullptr; }


// Two- and three-token forwards (the verify of a one- or two-token draft)
// run the linears the int8 tensor-core kernel takes in one weight pass
// (rq_mm_i8.cu), its activation staging in m->xq's buffer.
bool i8_ok(const rq_weight* const* ws, int n, int64_t T) {
    if (T < 2 || T > 8) return false;
    for (int i = 0; i < n; i++)
        if (!mm_i8_supported(ws[i], T)) return false;
    return true;
}

XQ2 i8_stage(const rq_llama* m, int64_t T, int64_t in) { return xq2_at(m->xq.planes, T, in); }

// y_i[t] = x[t] W_i^T (+ add_i[t]) for the n weights (same in) and T staged rows.
int run_linears(rq_llama* m, int n, const rq_weight* const* ws, int64_t T, float* const* ys,
                const float* const* adds, cudaStream_t st) {
    const int64_t in = ws[0]->in;
    const int sm = m->ctx->sm_count;
    if (pipe_supported(ws[0])) {
        const rq_weight* jw[kMaxJobs];
        XQ jx[kMaxJobs];
        float* jy[kMaxJobs];
        const float* ja[kMaxJobs];
        int nj = 0;
        for (int64_t t = 0; t < T; t++)
            for (int i = 0; i < n; i++) {
                jw[nj] = ws[i];
                jx[nj] = XQ{m->xq.planes + t * 3 * in, m->xq.stats + t * (in / 32)};
                jy[nj] = ys[i] + t * ws[i]->out;
                ja[nj] = adds && adds[i] ? adds[i] + t * ws[i]->out : nullptr;
                if (++nj == kMaxJobs) {
                    int rc = launch_matvec_pipe(jw, jx, jy, nj, sm, st, m->derr, ja);
                    if (rc) return rc;
                    nj = 0;
                }
            }
        return nj ? launch_matvec_pipe(jw, jx, jy, nj, sm, st, m->derr, ja, nullptr, nullptr, nullptr, nullptr,
                                       T == 1 ? next_hint(m) : nullptr)
                  : RQ_OK;
    }
    for (int i = 0; i < n; i++) {
        if (adds && adds[i] && adds[i] != ys[i])
            return set_error(RQ_ERR_UNSUPPORTED, "llama: residual into a separate buffer needs the pipeline");
        if (adds && adds[i]) {
            // y += x W^T: compute into the scratch g, then add
            int rc = launch_linear(ws[i], m->xq, m->g, T, sm, st, m->derr);
            if (rc) return rc;
            int64_t cnt = T * ws[i]->out;
            float* y = ys[i];
            const float* a = m->g;
            void* args[] = {&y, &a, &cnt};
            rc = launch_simple((const void*)add_rows_kernel, dim3(256), dim3(256), 0, st, args, "add kernel");
            if (rc) return rc;
        } else {
            int rc = launch_linear(ws[i], m->xq, ys[i], T, sm, st, m->derr);
            if (rc) return rc;
        }
    }
    return RQ_OK;
}

// x = x + x_in W^T for a row-parallel weight (o_proj, down_proj).  One rank:
// the residual add is fused into the matvec epilogue.  W ranks: each rank's
// partial product (rank 0 also adds the residual) is summed into x by an
// all-reduce -- at T = 1 on the pipeline inside the matvec kernel itself,
// over the ranks' NVLink exchange regions.
int row_parallel(rq_llama* m, const rq_weight* w, int64_t T, cudaStream_t st, const XQ* staged = nullptr,
                 const PipeRms* rms = nullptr) {
    const XQ xin = staged ? *staged : m->xq;
    if (m->W == 1) {
        const rq_weight* w1[1] = {w};
        float* y1[1] = {m->x};
        const float* a1[1] = {m->x};
        if (staged || rms)  // rms: the next RMSNorm's input staged in the epilogue
            return launch_matvec_pipe(w1, &xin, y1, 1, m->ctx->sm_count, st, m->derr, a1, nullptr, nullptr, nullptr,
                                      nullptr, next_hint(m), rms);
        return run_linears(m, 1, w1, T, y1, a1, st);
    }
    const rq_weight* w1[1] = {w};
    P2PArgs ar;
    if (T == 1 && tp_fused_enabled(m->W) && pipe_supported(w) && tp_p2p_args(m->ctx, &ar)) {
        const XQ xq = xin;
        float* y = m->x;
        const float* add = m->R == 0 ? m->x : nullptr;
        const int rc = launch_matvec_pipe(w1, &xq, &y, 1, m->ctx->sm_count, st, m->derr, &add, &ar, nullptr,
                                          nullptr, nullptr, next_hint(m), rms);
        if (rc != kPipeNotFusable) return rc;
    }
    float* y1[1] = {m->part};
    const float* a1[1] = {m->R == 0 ? m->x : nullptr};
    int rc = staged ? launch_matvec_pipe(w1, &xin, y1, 1, m->ctx->sm_count, st, m->derr, a1, nullptr, nullptr,
                                         nullptr, nullptr, next_hint(m))
                    : run_linears(m, 1, w1, T, y1, a1, st);
    if (!rc) rc = tp_allreduce(m->ctx, m->part, m->x, T * m->cfg.hidden, 0, 0, st);
    if (!rc && rms) {  // the staging the fused epilogue would have done
        const float* x = m->x;
        const float* wr = rms->w;
        int64_t H = m->cfg.hidden;
        int8_t* planes = rms->xq.planes;
        float4* stats = rms->xq.stats;
        float* ss = rms->ss;
        void* args[] = {&x, &wr, &H, &planes, &stats, &ss};
        rc = launch_simple((const void*)rms_stage_kernel, dim3((unsigned)((H / 32 + 127) / 128)), dim3(128), 0, st,
                           args, "rms staging kernel");
    }
    return rc;
}

// Decode (T = 1): the gate/up matvec stages silu(gate) * up for the down
// projection in its own epilogue (no separate staging launch) when both
// weights run on the pipeline and the local intermediate size is a multiple
// of 32.
bool swiglu_in_epilogue(const rq_llama* m, const rq_weight* gate, const rq_weight* up, int64_t T) {
    return T == 1 && pipe_supported(gate) && pipe_supported(up) && gate->out == up->out && m->I_l % 32 == 0;
}

// Decode with every linear of layer l on the pipeline: the o and down
// matvecs (after their all-reduce under tensor parallelism, each rank
// staging its own copy) stage the next RMSNorm's input in their epilogue
// (PipeRms) and the q/k/v and gate/up matvecs divide by its RMS
// (PipeRmsIn), so no staging kernel runs between them (RQ_RMS_EPILOGUE=0
// restores the staging kernels).
bool rms_epilogue_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("RQ_RMS_EPILOGUE");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}
bool rms_in_epilogue(const rq_llama* m, int64_t l, int64_t T) {
    if (T != 1 || m->cfg.hidden % 32 || l < 0 || l >= m->cfg.n_layers || !rms_epilogue_enabled()) return false;
    const rq_llama::Layer& L = m->layers[(size_t)l];
    for (int i = 0; i < 7; i++)
        if (!pipe_supported(L.w[i])) return false;
    return swiglu_in_epilogue(m, L.w[4], L.w[5], T);
}

// y_i = x W_i^T (+ add_i) for the n Q4_K weights (same in) over the T rows
// staged in m->xh: one tcgen05 launch for T >= kMinTcgenM or 9 <= T <= 16
// (the split-K kernel), else mma.sync tiles of 8 rows, up to kMaxJobs tiles
// per launch.
int run_mm(rq_llama* m, int n, const rq_weight* const* ws, int64_t T, float* const* ys, const float* const* adds,
           cudaStream_t st) {
    const int sm = m->ctx->sm_count;
    std::vector<MMJobDesc> jobs;
    for (int i = 1; i < n; i++)
        if (ws[i]->type != ws[0]->type) {  // one launch per weight type
            for (int k = 0; k < n; k++) {
                int rc = run_mm(m, 1, &ws[k], T, &ys[k], adds ? &adds[k] : nullptr, st);
                if (rc) return rc;
            }
            return RQ_OK;
        }
    if (T >= kMinTcgenM || ws[0]->type == RQ_Q3_K) {  // Q3_K: tensor_prefill checked q3k_tensor_m
        for (int i = 0; i < n; i++) jobs.push_back(MMJobDesc{ws[i], 0, (int)T, ys[i], adds ? adds[i] : nullptr});
        return launch_mm_tc(jobs.data(), (int)jobs.size(), m->xh, T, sm, st, m->derr);
    }
    if (T >= kSkinnyMinM && T <= kSkinnyMaxM) {
        for (int i = 0; i < n; i++) jobs.push_back(MMJobDesc{ws[i], 0, (int)T, ys[i], adds ? adds[i] : nullptr});
        return launch_mm_skinny(m->ctx, jobs.data(), (int)jobs.size(), m->xh, T, st, m->derr);
    }
    for (int64_t t0 = 0; t0 < T; t0 += 8)
        for (int i = 0; i < n; i++) {
            const int64_t o = ws[i]->out;
            jobs.push_back(MMJobDesc{ws[i], (int)t0, (int)std::min<int64_t>(8, T - t0), ys[i] + t0 * o,
                                     adds && adds[i] ? adds[i] + t0 * o : nullptr});
        }
    for (size_t b = 0; b < jobs.size(); b += kMaxJobs) {
        const int nj = (int)std::min<size_t>(kMaxJobs, jobs.size() - b);
        int rc = launch_mm_small(&jobs[b], nj, m->xh, T, sm, st, m->derr);
        if (rc) return rc;
    }
    return RQ_OK;
}

// row_parallel on the tensor-core path: x = x + x_in W^T with x_in staged in
// m->xh (the residual add in the epilogue; under tensor parallelism rank 0
// adds it to its partial before the all-reduce).
int row_parallel_mm(rq_llama* m, const rq_weight* w, int64_t T, cudaStream_t st) {
    const rq_weight* w1[1] = {w};
    float* y1[1] = {m->W == 1 ? m->x : m->part};
    const float* a1[1] = {m->R == 0 ? m->x : nullptr};
    int rc = run_mm(m, 1, w1, T, y1, a1, st);
    if (!rc && m->W > 1) rc = tp_allreduce(m->ctx, m->part, m->x, T * m->cfg.hidden, 0, 0, st);
    return rc;
}

// Prompt chunks of T >= kMinTensorM tokens with Q4_K weights (Q3_K from
// kQ3TensorMinM tokens, on the tcgen05 kernel) run every linear on the
// f16 tensor-core kernels, one pass over the weights per chunk -- except
// chunks whose seven linears all take the int8 kernels (up to eight tokens),
// which stage the int8 planes instead (i8_ok).
bool tensor_prefill(const rq_llama* m, int64_t T, int64_t l) {
    if (T < kMinTensorM || !m->xh.v) return false;
    bool all_i8 = true;
    for (int i = 0; i < 7; i++) {
        const rq_weight* w = m->layers[(size_t)l].w[i];
        if (!mm_small_supported(w) && !q3k_tensor_m(w, T)) return false;
        all_i8 = all_i8 && mm_i8_supported(w, T);
    }
    return !all_i8;  // up to eight tokens: the int8 kernels where every linear takes them
}

// One forward over the T tokens in m->tokens at device position *m->pos.
int head_all(rq_llama* m, int64_t T, bool want_logits, cudaStream_t st);

int forward_device(rq_llama* m, int64_t T, bool want_logits, cudaStream_t st, bool all_positions = false) {
    const rq_llama_config& c = m->cfg;
    const int64_t H = c.hidden, I = m->I_l, nq = m->nh_l * c.head_dim, nk = m->nkv_l * c.head_dim;
    int rc;
    {
        const __half* emb = m->embed;
        const int32_t* tok = m->tokens;
        int64_t vocab = c.vocab, hidden = H;
        float* x = m->x;
        void* args[] = {&emb, &tok, &T, &hidden, &vocab, &x};
        rc = launch_simple((const void*)embed_kernel, dim3((unsigned)std::min<int64_t>(64, (H + 255) / 256), (unsigned)T),
                           dim3(256), 0, st, args, "embed kernel");
        if (rc) return rc;
    }
    for (int64_t l = 0; l < c.n_layers; l++) {
        rq_llama::Layer& L = m->layers[l];
        const bool tc = tensor_prefill(m, T, l);
        {
            const rq_weight* w3[3] = {L.w[0], L.w[1], L.w[2]};
            float* y3[3] = {m->q, m->k, m->v};
            if (tc) {
                rc = launch_xh_stage_rmsnorm(m->x, L.rms1, c.rms_eps, T, H, m->xh, st);
                if (!rc) rc = run_mm(m, 3, w3, T, y3, nullptr, st);
            } else if (i8_ok(w3, 3, T)) {
                const XQ2 q2 = i8_stage(m, T, H);
                rc = launch_xq2_stage(m->x, T, H, q2, st, L.rms1, c.rms_eps);
                if (!rc) rc = launch_mm_i8(w3, y3, 3, T, q2, m->ctx->sm_count, st, m->derr);
            } else if (l > 0 && rms_in_epilogue(m, l - 1, T) && rms_in_epilogue(m, l, T)) {
                // x * rms1 was staged by the previous down projection's epilogue
                const XQ in3[3] = {m->xqr, m->xqr, m->xqr};
                const PipeRmsIn ri{m->rss, (int)(H / 32), (float)H, c.rms_eps};
                set_next(m, &L.w[3], 1, kNextBudgetAttn);
                rc = launch_matvec_pipe(w3, in3, y3, 3, m->ctx->sm_count, st, m->derr, nullptr, nullptr, nullptr,
                                        nullptr, nullptr, next_hint(m), nullptr, &ri);
                set_next(m, nullptr, 0, 0);
            } else {
                rc = launch_xquant_rmsnorm(m->x, L.rms1, c.rms_eps, T, H, m->xq, st);
                if (T == 1) set_next(m, &L.w[3], 1, kNextBudgetAttn);
                if (!rc) rc = run_linears(m, 3, w3, T, y3, nullptr, st);
                set_next(m, nullptr, 0, 0);
            }
            if (rc) return rc;
        }
        if (T == 1 && c.head_dim % 32 == 0) {
            const float* q = m->q;
            const float* k = m->k;
            const float* v = m->v;
            float* kc = L.kc;
            float* vc = L.vc;
            const float* cs = m->rope_cos;
            const float* sn = m->rope_sin;
            const int32_t* pos = m->pos;
            int nh = (int)m->nh_l, nkv = (int)m->nkv_l, hd = (int)c.head_dim, ms = (int)c.max_seq;
            int8_t* planes = m->xq.planes;
            float4* stats = m->xq.stats;
            void* args[] = {&q, &k, &v, &kc, &vc, &cs, &sn, &pos, &nh, &nkv, &hd, &ms, &planes, &stats};
            rc = launch_simple((const void*)attn_decode_kernel, dim3((unsigned)nh), dim3(kAttnThreads),
                               (size_t)attn_smem_floats(c.max_seq, c.head_dim) * sizeof(float), st, args,
                               "attention kernel");
            if (rc) return rc;
        } else {
            float* q = m->q;
            const float* k = m->k;
            const float* v = m->v;
            float* kc = L.kc;
            float* vc = L.vc;
            const float* cs = m->rope_cos;
            const float* sn = m->rope_sin;
            const int32_t* pos = m->pos;
            int nh = (int)m->nh_l, nkv = (int)m->nkv_l, hd = (int)c.head_dim, ms = (int)c.max_seq;
            void* args[] = {&q, &k, &v, &kc, &vc, &cs, &sn, &pos, &nh, &nkv, &hd, &ms};
            rc = launch_simple((const void*)rope_append_kernel, dim3((unsigned)(nh + nkv), (unsigned)T),
                               dim3((unsigned)std::max(32, hd / 2)), 0, st, args, "rope kernel");
            if (rc) return rc;
            const float* qc = m->q;
            float* att = m->att;
            void* args2[] = {&qc, &kc, &vc, &pos, &nh, &nkv, &hd, &ms, &att};
            rc = launch_simple((const void*)attention_kernel, dim3((unsigned)nh, (unsigned)T), dim3(128),
                               (size_t)c.max_seq * sizeof(float), st, args2, "attention kernel");
            if (rc) return rc;
            if (!tc && i8_ok(&L.w[3], 1, T)) {
                // o on the int8 kernel: x (+)= att W^T, the residual in its epilogue
                const XQ2 q2 = i8_stage(m, T, nq);
                rc = launch_xq2_stage(m->att, T, nq, q2, st);
                float* y1[1] = {m->W == 1 ? m->x : m->part};
                const float* a1[1] = {m->R == 0 ? m->x : nullptr};
                if (!rc) rc = launch_mm_i8(&L.w[3], y1, 1, T, q2, m->ctx->sm_count, st, m->derr, a1);
                if (!rc && m->W > 1) rc = tp_allreduce(m->ctx, m->part, m->x, T * H, 0, 0, st);
                if (rc) return rc;
                goto mlp;
            }
            rc = tc ? launch_xh_stage(m->att, T, nq, m->xh, st) : launch_xquant(m->att, T, nq, m->xq, st);
            if (rc) return rc;
        }
        if (T == 1 && !tc) set_next(m, &L.w[4], 2, kNextBudget);
        {
            // o stages x * rms2 for gate/up in its epilogue where that is on
            const PipeRms rms_o{m->xqr, m->rss, m->rcnt, L.rms2};
            const bool ro = !tc && rms_in_epilogue(m, l, T);
            rc = tc ? row_parallel_mm(m, L.w[3], T, st) : row_parallel(m, L.w[3], T, st, nullptr, ro ? &rms_o : nullptr);
        }
        set_next(m, nullptr, 0, 0);
        if (rc) return rc;
    mlp:
        {
            const rq_weight* w2[2] = {L.w[4], L.w[5]};
            float* y2[2] = {m->g, m->u};
            if (tc) {
                rc = launch_xh_stage_rmsnorm(m->x, L.rms2, c.rms_eps, T, H, m->xh, st);
                if (!rc) rc = run_mm(m, 2, w2, T, y2, nullptr, st);
            } else if (i8_ok(w2, 2, T)) {
                const XQ2 q2 = i8_stage(m, T, H);
                rc = launch_xq2_stage(m->x, T, H, q2, st, L.rms2, c.rms_eps);
                if (!rc) rc = launch_mm_i8(w2, y2, 2, T, q2, m->ctx->sm_count, st, m->derr);
            } else if (swiglu_in_epilogue(m, L.w[4], L.w[5], T)) {
                // x * rms2 staged by o's epilogue, or the staging kernel
                const bool rin = rms_in_epilogue(m, l, T);
                if (!rin) rc = launch_xquant_rmsnorm(m->x, L.rms2, c.rms_eps, T, H, m->xq, st);
                const XQ src = rin ? m->xqr : m->xq;
                const XQ in2[2] = {src, src};
                const PipeSwiglu sw{m->xqd, m->swcnt, 0};
                const PipeRmsIn ri{m->rss, (int)(H / 32), (float)H, c.rms_eps};
                set_next(m, &L.w[6], 1, kNextBudget);
                if (!rc) rc = launch_matvec_pipe(w2, in2, y2, 2, m->ctx->sm_count, st, m->derr, nullptr, nullptr,
                                                 nullptr, &sw, nullptr, next_hint(m), nullptr, rin ? &ri : nullptr);
                // down prefetches the next layer's q/k/v and, where the next
                // layer reads it, stages x * rms1 of that layer
                if (l + 1 < c.n_layers) set_next(m, m->layers[l + 1].w, 3, kNextBudget);
                else set_next(m, nullptr, 0, 0);
                const bool rout = rin && rms_in_epilogue(m, l + 1, T);
                const PipeRms rms_d{m->xqr, m->rss, m->rcnt, rout ? m->layers[l + 1].rms1 : nullptr};
                if (!rc) rc = row_parallel(m, L.w[6], T, st, &m->xqd, rout ? &rms_d : nullptr);
                set_next(m, nullptr, 0, 0);
                if (rc) return rc;
                continue;
            } else {
                rc = launch_xquant_rmsnorm(m->x, L.rms2, c.rms_eps, T, H, m->xq, st);
                if (!rc) rc = run_linears(m, 2, w2, T, y2, nullptr, st);
            }
            if (rc) return rc;
        }
        if (tc) {
            rc = launch_xh_stage_swiglu(m->g, m->u, T, I, m->xh, st);
            if (!rc) rc = row_parallel_mm(m, L.w[6], T, st);
        } else if (i8_ok(&L.w[6], 1, T)) {
            // down on the int8 kernel (K split over four CTAs per row group)
            const XQ2 q2 = i8_stage(m, T, I);
            rc = launch_xq2_stage(m->g, T, I, q2, st, nullptr, 0.0f, m->u);
            float* y1[1] = {m->W == 1 ? m->x : m->part};
            const float* a1[1] = {m->R == 0 ? m->x : nullptr};
            if (!rc)
                rc = launch_mm_i8(&L.w[6], y1, 1, T, q2, m->ctx->sm_count, st, m->derr, a1, m->i8part, m->i8cnt);
            if (!rc && m->W > 1) rc = tp_allreduce(m->ctx, m->part, m->x, T * H, 0, 0, st);
        } else {
            rc = launch_xquant_swiglu(m->g, m->u, T, I, m->xq, st);
            if (!rc) rc = row_parallel(m, L.w[6], T, st);
        }
        if (rc) return rc;
    }
    (void)nk;
    unsigned long long* last_key = m->best;
    if (all_positions) {
        rc = head_all(m, T, want_logits, st);
        if (rc) return rc;
        last_key = m->keys + (T - 1);
    } else {
        {
            const float* xl = m->x + (T - 1) * H;
            const float* w = m->ln_f;
            float eps = c.rms_eps;
            int64_t hidden = H;
            float* hf = m->hf;
            void* args[] = {&xl, &w, &eps, &hidden, &hf};
            rc = launch_simple((const void*)rmsnorm_row_kernel, dim3(1), dim3(1024), 0, st, args,
                               "final norm kernel");
            if (rc) return rc;
        }
        const __half* W = m->lm_head;
        const float* hf = m->hf;
        int64_t vocab = m->vocab_l, hidden = H, roff = (int64_t)m->R * m->vocab_l;
        float* lg = want_logits ? m->logits : nullptr;
        unsigned long long* best = m->best;
        void* args[] = {&W, &hf, &vocab, &hidden, &roff, &lg, &best};
        const unsigned grid = (unsigned)std::min<int64_t>((vocab + 7) / 8, (int64_t)m->ctx->sm_count * 8);
        rc = launch_simple((const void*)lm_head_kernel, dim3(grid), dim3(256), (size_t)H * sizeof(float), st,
                           args, "lm_head kernel");
        if (rc) return rc;
        if (m->W > 1) {  // global argmax: max of the packed (value, index) keys
            rc = tp_allreduce(m->ctx, m->best, m->best, 1, 1, 1, st);
            if (rc) return rc;
        }
    }
    {
        unsigned long long* best = last_key;
        int32_t* tok = m->tokens;
        int32_t* pos = m->pos;
        int32_t* out = m->out;
        int32_t* nout = m->nout;
        int Ti = (int)T, mo = (int)c.max_seq;
        void* args[] = {&best, &tok, &pos, &out, &nout, &Ti, &mo};
        rc = launch_simple((const void*)finish_step_kernel, dim3(1), dim3(1), 0, st, args, "finish kernel");
    }
    return rc;
}

// Final norm and lm_head at every one of the T positions (the verify
// forward, forward_all of src/streaming_quantized.rs:611-620): per-position
// argmax tokens into m->amax (a MAX all-reduce of the keys under tensor
// parallelism) and, if wanted, logits into m->logits_all.  The lm_head
// matrix is read once per 6 positions.
int head_all(rq_llama* m, int64_t T, bool want_logits, cudaStream_t st) {
    const rq_llama_config& c = m->cfg;
    const int64_t H = c.hidden;
    int rc = cuda_error(cudaMemsetAsync(m->keys, 0, (size_t)T * 8, st), "memset");
    if (rc) return rc;
    {
        const float* x = m->x;
        const float* w = m->ln_f;
        float eps = c.rms_eps;
        int64_t hidden = H;
        float* y = m->part;  // [T][H], free at this point
        void* args[] = {&x, &w, &eps, &hidden, &y};
        rc = launch_simple((const void*)rmsnorm_rows_kernel, dim3((unsigned)T), dim3(1024), 0, st, args,
                           "final norm kernel");
        if (rc) return rc;
    }
    for (int64_t t0 = 0; t0 < T; t0 += 6) {
        const int nt = (int)std::min<int64_t>(6, T - t0);
        const __half* W = m->lm_head;
        const float* hf = m->part + t0 * H;
        int64_t vocab = m->vocab_l, hidden = H, roff = (int64_t)m->R * m->vocab_l;
        float* lg = want_logits ? m->logits_all + t0 * m->vocab_l : nullptr;
        unsigned long long* keys = m->keys + t0;
        void* args[] = {&W, &hf, &vocab, &hidden, &roff, &lg, &keys};
        const unsigned grid = (unsigned)std::min<int64_t>((vocab + 7) / 8, (int64_t)m->ctx->sm_count * 8);
        const size_t smem = (size_t)nt * H * sizeof(float);
        const void* fn = nt == 1   ? (const void*)lm_head_rows_kernel<1>
                         : nt == 2 ? (const void*)lm_head_rows_kernel<2>
                         : nt == 3 ? (const void*)lm_head_rows_kernel<3>
                         : nt == 4 ? (const void*)lm_head_rows_kernel<4>
                         : nt == 5 ? (const void*)lm_head_rows_kernel<5>
                                   : (const void*)lm_head_rows_kernel<6>;
        rc = launch_simple(fn, dim3(grid), dim3(256), smem, st, args, "lm_head kernel");
        if (rc) return rc;
    }
    if (m->W > 1) {
        rc = tp_allreduce(m->ctx, m->keys, m->keys, T, 1, 1, st);
        if (rc) return rc;
    }
    unsigned long long* keys = m->keys;
    int Ti = (int)T;
    int32_t* out = m->amax;
    void* args[] = {&keys, &Ti, &out};
    return launch_simple((const void*)unpack_argmax_kernel, dim3(1), dim3(256), 0, st, args, "argmax kernel");
}

template <typename T>
int dalloc(rq_llama* m, T** p, size_t n) {
    cudaError_t e = cudaMalloc((void**)p, n * sizeof(T));
    if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(llama)");
    m->allocs.push_back((void*)*p);
    return RQ_OK;
}

int copy_in(void* dst, const void* src, size_t bytes) {
    cudaPointerAttributes a;
    cudaMemcpyKind kind = cudaMemcpyHostToDevice;
    if (cudaPointerGetAttributes(&a, src) == cudaSuccess &&
        (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged))
        kind = cudaMemcpyDeviceToDevice;
    cudaGetLastError();
    return cuda_error(cudaMemcpy(dst, src, bytes, kind), "llama weight copy");
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

// The one-launch decode step applies with one GPU, every layer set, one
// weight type throughout and shapes the plan accepts.
bool fused_plan(rq_llama* m, DecParams& p, size_t* smem) {
    if (!m->fused || m->W != 1) return false;
    const rq_llama_config& c = m->cfg;
    int type = -1;
    for (int64_t l = 0; l < c.n_layers; l++) {
        if (!m->layer_set[(size_t)l]) return false;
        for (int i = 0; i < 7; i++) {
            const int t = m->layers[(size_t)l].w[i]->type;
            if (type < 0) type = t;
            if (t != type) return false;
        }
    }
    p = DecParams{};
    p.layers = m->dlayers;
    p.n_layers = (int)c.n_layers;
    p.type = type;
    p.H = c.hidden;
    p.I = m->I_l;
    p.nq = m->nh_l * c.head_dim;
    p.nk = m->nkv_l * c.head_dim;
    p.head_dim = c.head_dim;
    p.n_heads = m->nh_l;
    p.n_kv = m->nkv_l;
    p.max_seq = c.max_seq;
    p.vocab = m->vocab_l;
    p.eps = c.rms_eps;
    p.x = m->x;
    p.q = m->q;
    p.k = m->k;
    p.v = m->v;
    p.g = m->g;
    p.u = m->u;
    p.xq = m->xq;
    p.rope_cos = m->rope_cos;
    p.rope_sin = m->rope_sin;
    p.embed = m->embed;
    p.ln_f = m->ln_f;
    p.lm_head = m->lm_head;
    p.best = m->best;
    p.tokens = m->tokens;
    p.pos = m->pos;
    p.out = m->out;
    p.nout = m->nout;
    p.bar = m->bar;
    p.err = m->derr;
    return decode_plan(p, m->ctx->sm_count, smem);
}

}  // namespace
}  // namespace rq

using namespace rq;

extern "C" {

int rq_llama_create(rq_ctx* ctx, const rq_llama_config* cfg, rq_llama** out) {
    if (!ctx || !cfg || !out) return set_error(RQ_ERR_INVALID, "rq_llama_create: NULL argument");
    *out = nullptr;
    const rq_llama_config& c = *cfg;
    if (c.hidden <= 0 || c.intermediate <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 ||
        c.n_layers <= 0 || c.vocab <= 0 || c.max_seq <= 0 || c.max_batch_tokens <= 0)
        return set_error(RQ_ERR_INVALID, "rq_llama_create: every size must be positive");
    if (c.n_heads % c.n_kv_heads || c.head_dim % 2 || c.head_dim > 256 || c.hidden % 256 ||
        c.intermediate % 256 || (c.n_heads * c.head_dim) % 256)
        return set_error(RQ_ERR_INVALID,
                         "rq_llama_create: need n_heads %% n_kv_heads == 0, even head_dim <= 256, and "
                         "hidden, intermediate, n_heads*head_dim multiples of 256");
    if (attn_smem_floats(c.max_seq, c.head_dim) * (int64_t)sizeof(float) > 200 * 1024)
        return set_error(RQ_ERR_INVALID, "rq_llama_create: max_seq %lld too large for attention", (long long)c.max_seq);
    const int W = tp_world(ctx), R = tp_rank(ctx);
    if (c.n_kv_heads % W || c.intermediate % (256 * W) || (c.n_heads / W * c.head_dim) % 256 || c.vocab % W)
        return set_error(RQ_ERR_INVALID,
                         "rq_llama_create: %d-way tensor parallelism needs n_kv_heads %% W == 0, "
                         "intermediate/W and n_heads/W*head_dim multiples of 256, vocab %% W == 0", W);
    Guard g(ctx->device);
    rq_llama* m = new (std::nothrow) rq_llama();
    if (!m) return set_error(RQ_ERR_OOM, "host allocation failed");
    m->ctx = ctx;
    m->cfg = c;
    m->W = W;
    m->R = R;
    m->nh_l = c.n_heads / W;
    m->nkv_l = c.n_kv_heads / W;
    m->I_l = c.intermediate / W;
    m->vocab_l = c.vocab / W;
    m->layers.resize((size_t)c.n_layers);
    const int64_t T = c.max_batch_tokens, H = c.hidden, I = m->I_l;
    const int64_t nq = m->nh_l * c.head_dim, nk = m->nkv_l * c.head_dim, half = c.head_dim / 2;
    const int64_t maxin = std::max(std::max(H, I), nq);
    int rc = RQ_OK;
    for (auto& L : m->layers) {
        memset(L.w, 0, sizeof L.w);
        if (!rc) rc = dalloc(m, &L.rms1, (size_t)H);
        if (!rc) rc = dalloc(m, &L.rms2, (size_t)H);
        if (!rc) rc = dalloc(m, &L.kc, (size_t)(nk * c.max_seq));
        if (!rc) rc = dalloc(m, &L.vc, (size_t)(nk * c.max_seq));
    }
    if (!rc) rc = dalloc(m, &m->embed, (size_t)(c.vocab * H));
    if (!rc) rc = dalloc(m, &m->ln_f, (size_t)H);
    if (!rc) rc = dalloc(m, &m->lm_head, (size_t)(m->vocab_l * H));
    if (!rc) rc = dalloc(m, &m->rope_cos, (size_t)(c.max_seq * half));
    if (!rc) rc = dalloc(m, &m->rope_sin, (size_t)(c.max_seq * half));
    if (!rc) rc = dalloc(m, &m->x, (size_t)(T * H));
    if (!rc) rc = dalloc(m, &m->q, (size_t)(T * nq));
    if (!rc) rc = dalloc(m, &m->k, (size_t)(T * nk));
    if (!rc) rc = dalloc(m, &m->v, (size_t)(T * nk));
    if (!rc) rc = dalloc(m, &m->att, (size_t)(T * nq));
    if (!rc) rc = dalloc(m, &m->g, (size_t)(T * std::max(I, H)));
    if (!rc) rc = dalloc(m, &m->u, (size_t)(T * I));
    if (!rc) rc = dalloc(m, &m->hf, (size_t)H);
    if (!rc) rc = dalloc(m, &m->logits, (size_t)m->vocab_l);
    if (!rc) rc = dalloc(m, &m->part, (size_t)(T * H));
    uint8_t* xqbuf = nullptr;
    uint8_t* xhbuf = nullptr;
    uint8_t* xqdbuf = nullptr;
    if (!rc) rc = dalloc(m, &xqbuf, xq_bytes(T, maxin));
    if (!rc) rc = dalloc(m, &xqdbuf, xq_bytes(1, I));
    if (!rc) rc = dalloc(m, &m->i8part, (size_t)(4 * 8 * H));
    if (!rc) rc = dalloc(m, &m->i8cnt, 256);
    if (!rc) rc = cuda_error(cudaMemset(m->i8cnt, 0, 256 * sizeof(int)), "counter reset");
    if (!rc) rc = dalloc(m, &m->swcnt, (size_t)(I / 32 + 1));
    if (!rc) rc = cuda_error(cudaMemset(m->swcnt, 0, sizeof(int) * (size_t)(I / 32 + 1)), "counter reset");
    uint8_t* xqrbuf = nullptr;
    if (!rc) rc = dalloc(m, &xqrbuf, xq_bytes(1, H));
    if (!rc) rc = dalloc(m, &m->rss, (size_t)(H / 32 + 1));
    if (!rc) rc = dalloc(m, &m->rcnt, (size_t)(H / 32 + 1));
    if (!rc) rc = cuda_error(cudaMemset(m->rcnt, 0, sizeof(int) * (size_t)(H / 32 + 1)), "counter reset");
    if (!rc) rc = cuda_error(cudaDeviceSynchronize(), "counter reset");
    if (!rc && T >= kMinTensorM) rc = dalloc(m, &xhbuf, xh_bytes(T, maxin));
    if (!rc) rc = dalloc(m, &m->best, 1);
    if (!rc) rc = dalloc(m, &m->keys, (size_t)T);
    if (!rc) rc = dalloc(m, &m->amax, (size_t)T);
    if (!rc) rc = dalloc(m, &m->logits_all, (size_t)(T * m->vocab_l));
    if (!rc) rc = dalloc(m, &m->tokens, (size_t)T);
    if (!rc) rc = dalloc(m, &m->pos, 1);
    if (!rc) rc = dalloc(m, &m->out, (size_t)c.max_seq);
    if (!rc) rc = dalloc(m, &m->nout, 1);
    if (!rc) rc = dalloc(m, &m->dlayers, (size_t)c.n_layers);
    if (!rc) rc = dalloc(m, &m->bar, 1);
    if (!rc) rc = dalloc(m, &m->derr, 1);
    if (!rc) {
        m->hlayers.assign((size_t)c.n_layers, rq::DecLayer{});
        m->layer_set.assign((size_t)c.n_layers, false);
        m->xq.planes = (int8_t*)xqbuf;
        m->xq.stats = (float4*)(xqbuf + (((size_t)T * 3 * maxin + 255) & ~(size_t)255));
        m->xqd.planes = (int8_t*)xqdbuf;
        m->xqd.stats = (float4*)(xqdbuf + (((size_t)3 * I + 255) & ~(size_t)255));
        m->xqr.planes = (int8_t*)xqrbuf;
        m->xqr.stats = (float4*)(xqrbuf + (((size_t)3 * H + 255) & ~(size_t)255));
        m->xh = xhbuf ? xh_at(xhbuf, T, maxin) : XH{};
        // RoPE tables as QuantStreamCache::new computes them
        // (src/streaming_quantized.rs:104-118): inv_freq[i] =
        // 1 / theta^(2i / head_dim), angle = f32(position) * inv_freq[i].
        std::vector<float> cs((size_t)(c.max_seq * half)), sn(cs.size());
        for (int64_t i = 0; i < half; i++) {
            const float inv = 1.0f / powf(c.rope_theta, (float)(2 * i) / (float)c.head_dim);
            for (int64_t p = 0; p < c.max_seq; p++) {
                const float a = (float)p * inv;
                cs[(size_t)(p * half + i)] = cosf(a);
                sn[(size_t)(p * half + i)] = sinf(a);
            }
        }
        rc = cuda_error(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "rope copy");
        if (!rc) rc = cuda_error(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), "rope copy");
        if (!rc) rc = cuda_error(cudaMemset(m->best, 0, 8), "memset");
        if (!rc) rc = cuda_error(cudaMemset(m->pos, 0, 4), "memset");
        if (!rc) rc = cuda_error(cudaMemset(m->nout, 0, 4), "memset");
        if (!rc) rc = cuda_error(cudaMemset(m->tokens, 0, (size_t)T * 4), "memset");
        if (!rc) rc = cuda_error(cudaMemset(m->derr, 0, 4), "memset");
    }
    if (rc) {
        for (void* p : m->allocs) cudaFree(p);
        delete m;
        return rc;
    }
    *out = m;
    return RQ_OK;
}

int rq_llama_free(rq_llama* m) {
    if (!m) return RQ_OK;
    Guard g(m->ctx->device);
    for (void* p : m->allocs) cudaFree(p);
    for (rq_weight* w : m->owned) rq_weight_free(m->ctx, w);
    delete m;
    return RQ_OK;
}

int rq_llama_set_layer(rq_llama* m, int64_t layer, const rq_weight* const* w7, const float* rms1,
                       const float* rms2) {
    if (!m || !w7 || !rms1 || !rms2) return set_error(RQ_ERR_INVALID, "rq_llama_set_layer: NULL argument");
    const rq_llama_config& c = m->cfg;
    if (layer < 0 || layer >= c.n_layers) return set_error(RQ_ERR_INVALID, "rq_llama_set_layer: layer %lld", (long long)layer);
    const int64_t H = c.hidden, I = m->I_l, nq = m->nh_l * c.head_dim, nk = m->nkv_l * c.head_dim;
    const int64_t shp[7][2] = {{nq, H}, {nk, H}, {nk, H}, {H, nq}, {I, H}, {I, H}, {H, I}};  // (out, in)
    const char* names[7] = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"};
    for (int i = 0; i < 7; i++) {
        if (!w7[i]) return set_error(RQ_ERR_INVALID, "rq_llama_set_layer: %s is NULL", names[i]);
        if (w7[i]->out != shp[i][0] || w7[i]->in != shp[i][1] || w7[i]->device != m->ctx->device)
            return set_error(RQ_ERR_INVALID, "rq_llama_set_layer: %s is [%lld, %lld], expected [%lld, %lld]",
                             names[i], (long long)w7[i]->out, (long long)w7[i]->in, (long long)shp[i][0],
                             (long long)shp[i][1]);
    }
    if (w7[0]->type != w7[1]->type || w7[0]->type != w7[2]->type || w7[4]->type != w7[5]->type)
        return set_error(RQ_ERR_INVALID, "rq_llama_set_layer: q/k/v and gate/up must share a weight type");
    Guard g(m->ctx->device);
    rq_llama::Layer& L = m->layers[(size_t)layer];
    for (int i = 0; i < 7; i++) L.w[i] = w7[i];
    int rc = copy_in(L.rms1, rms1, (size_t)H * 4);
    if (!rc) rc = copy_in(L.rms2, rms2, (size_t)H * 4);
    if (rc) return rc;
    rq::DecLayer& D = m->hlayers[(size_t)layer];
    for (int i = 0; i < 7; i++) {
        D.qs[i] = w7[i]->qs;
        D.hdr[i] = w7[i]->hdr;
    }
    D.rms1 = L.rms1;
    D.rms2 = L.rms2;
    D.kc = L.kc;
    D.vc = L.vc;
    m->layer_set[(size_t)layer] = true;
    return cuda_error(cudaMemcpy(m->dlayers + layer, &D, sizeof D, cudaMemcpyHostToDevice), "layer table copy");
}

int rq_llama_load_gguf_dir(rq_llama* m, const char* dir) {
    if (!m || !dir) return set_error(RQ_ERR_INVALID, "rq_llama_load_gguf_dir: NULL argument");
    Guard g(m->ctx->device);
    const rq_llama_config& c = m->cfg;
    const int64_t H = c.hidden, nq = m->nh_l * c.head_dim, nk = m->nkv_l * c.head_dim, I = m->I_l;
    const int64_t out7[7] = {nq, nk, nk, H, I, I, H};
    const int64_t in7[7] = {H, H, H, nq, H, H, I};
    return llama_load_gguf_dir(m->ctx, m, dir, c.n_layers, c.vocab, H, m->W, m->R, out7, in7, m->owned);
}

int rq_llama_set_embedding(rq_llama* m, const uint16_t* embed_f16) {
    if (!m || !embed_f16) return set_error(RQ_ERR_INVALID, "rq_llama_set_embedding: NULL argument");
    Guard g(m->ctx->device);
    return copy_in(m->embed, embed_f16, (size_t)(m->cfg.vocab * m->cfg.hidden) * 2);
}

int rq_llama_set_head(rq_llama* m, const float* ln_f, const uint16_t* lm_head_f16) {
    if (!m || !ln_f || !lm_head_f16) return set_error(RQ_ERR_INVALID, "rq_llama_set_head: NULL argument");
    Guard g(m->ctx->device);
    int rc = copy_in(m->ln_f, ln_f, (size_t)m->cfg.hidden * 4);
    if (!rc) rc = copy_in(m->lm_head, lm_head_f16, (size_t)(m->vocab_l * m->cfg.hidden) * 2);
    return rc;
}

int rq_llama_forward(rq_llama* m, const int32_t* tokens, int64_t T, int64_t index_pos, float* logits,
                     int32_t* next_token, void* stream) {
    if (!m || !tokens) return set_error(RQ_ERR_INVALID, "rq_llama_forward: NULL argument");
    const rq_llama_config& c = m->cfg;
    if (T < 1 || T > c.max_batch_tokens)
        return set_error(RQ_ERR_INVALID, "rq_llama_forward: T = %lld (1..%lld)", (long long)T,
                         (long long)c.max_batch_tokens);
    if (index_pos < 0 || index_pos + T > c.max_seq)
        return set_error(RQ_ERR_INVALID, "rq_llama_forward: positions %lld..%lld exceed max_seq %lld",
                         (long long)index_pos, (long long)(index_pos + T), (long long)c.max_seq);
    for (auto& L : m->layers)
        if (!L.w[0]) return set_error(RQ_ERR_INVALID, "rq_llama_forward: a layer was not set");
    if (logits && m->W > 1)
        return set_error(RQ_ERR_UNSUPPORTED, "rq_llama_forward: logits are per-rank shards under tensor parallelism");
    Guard g(m->ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    int32_t p = (int32_t)index_pos;
    int rc = cuda_error(cudaMemcpyAsync(m->tokens, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, st), "token copy");
    if (!rc) rc = cuda_error(cudaMemcpyAsync(m->pos, &p, 4, cudaMemcpyHostToDevice, st), "pos copy");
    if (!rc) rc = forward_device(m, T, logits != nullptr, st);
    if (!rc && logits)
        rc = cuda_error(cudaMemcpyAsync(logits, m->logits, (size_t)c.vocab * 4, cudaMemcpyDefault, st), "logits copy");
    if (!rc && next_token)
        rc = cuda_error(cudaMemcpyAsync(next_token, m->tokens, 4, cudaMemcpyDeviceToHost, st), "token copy");
    if (!rc) rc = cuda_error(cudaStreamSynchronize(st), "rq_llama_forward sync");
    if (!rc) rc = rq_llama_status(m);  // a kernel wait that gave up
    return rc;
}

int rq_llama_forward_all(rq_llama* m, const int32_t* tokens, int64_t T, int64_t index_pos, float* logits,
                         int32_t* argmax, void* stream) {
    if (!m || !tokens || !argmax) return set_error(RQ_ERR_INVALID, "rq_llama_forward_all: NULL argument");
    const rq_llama_config& c = m->cfg;
    if (T < 1 || T > c.max_batch_tokens)
        return set_error(RQ_ERR_INVALID, "rq_llama_forward_all: T = %lld (1..%lld)", (long long)T,
                         (long long)c.max_batch_tokens);
    if (index_pos < 0 || index_pos + T > c.max_seq)
        return set_error(RQ_ERR_INVALID, "rq_llama_forward_all: positions %lld..%lld exceed max_seq %lld",
                         (long long)index_pos, (long long)(index_pos + T), (long long)c.max_seq);
    for (auto& L : m->layers)
        if (!L.w[0]) return set_error(RQ_ERR_INVALID, "rq_llama_forward_all: a layer was not set");
    if (logits && m->W > 1)
        return set_error(RQ_ERR_UNSUPPORTED, "rq_llama_forward_all: logits are per-rank shards under tensor parallelism");
    Guard g(m->ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    int32_t p = (int32_t)index_pos;
    int rc = cuda_error(cudaMemcpyAsync(m->tokens, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, st), "token copy");
    if (!rc) rc = cuda_error(cudaMemcpyAsync(m->pos, &p, 4, cudaMemcpyHostToDevice, st), "pos copy");
    if (!rc) rc = forward_device(m, T, logits != nullptr, st, true);
    if (!rc && logits)
        rc = cuda_error(cudaMemcpyAsync(logits, m->logits_all, (size_t)(T * c.vocab) * 4, cudaMemcpyDefault, st),
                        "logits copy");
    if (!rc) rc = cuda_error(cudaMemcpyAsync(argmax, m->amax, (size_t)T * 4, cudaMemcpyDefault, st), "argmax copy");
    if (!rc) rc = cuda_error(cudaStreamSynchronize(st), "rq_llama_forward_all sync");
    if (!rc) rc = rq_llama_status(m);
    return rc;
}

int rq_llama_decode_step(rq_llama* m, void* stream) {
    if (!m) return set_error(RQ_ERR_INVALID, "rq_llama_decode_step: NULL argument");
    Guard g(m->ctx->device);
    DecParams dp;
    size_t smem = 0;
    if (fused_plan(m, dp, &smem)) return launch_decode_step(dp, m->ctx->sm_count, smem, (cudaStream_t)stream);
    return forward_device(m, 1, false, (cudaStream_t)stream);
}

int rq_llama_set_fused(rq_llama* m, int enable) {
    if (!m) return set_error(RQ_ERR_INVALID, "rq_llama_set_fused: NULL argument");
    m->fused = enable != 0;
    return RQ_OK;
}

int rq_llama_status(rq_llama* m) {
    if (!m) return set_error(RQ_ERR_INVALID, "rq_llama_status: NULL argument");
    Guard g(m->ctx->device);
    int e = 0;
    int rc = cuda_error(cudaMemcpy(&e, m->derr, 4, cudaMemcpyDeviceToHost), "status copy");
    if (rc) return rc;
    if (e) {
        cudaMemset(m->derr, 0, 4);
        return set_error(RQ_ERR_TIMEOUT, "llama: a kernel's bounded wait gave up after ~1 s (the outputs since the "
                                         "last check are invalid)");
    }
    return RQ_OK;
}

int rq_llama_tokens(rq_llama* m, int32_t* out, int64_t cap, int64_t* count, int64_t* position) {
    if (!m) return set_error(RQ_ERR_INVALID, "rq_llama_tokens: NULL argument");
    Guard g(m->ctx->device);
    int32_t n = 0, p = 0;
    int rc = cuda_error(cudaMemcpy(&n, m->nout, 4, cudaMemcpyDeviceToHost), "count copy");
    if (!rc) rc = cuda_error(cudaMemcpy(&p, m->pos, 4, cudaMemcpyDeviceToHost), "pos copy");
    if (!rc && out && cap > 0) {
        const int64_t k = std::min<int64_t>(std::min<int64_t>(n, cap), m->cfg.max_seq);
        if (k > 0) rc = cuda_error(cudaMemcpy(out, m->out, (size_t)k * 4, cudaMemcpyDeviceToHost), "tokens copy");
    }
    if (count) *count = n;
    if (position) *position = p;
    return rc;
}

int rq_llama_truncate(rq_llama* m, int64_t new_len) {
    if (!m) return set_error(RQ_ERR_INVALID, "rq_llama_truncate: NULL argument");
    if (new_len < 0 || new_len > m->cfg.max_seq)
        return set_error(RQ_ERR_INVALID, "rq_llama_truncate: %lld", (long long)new_len);
    Guard g(m->ctx->device);
    int32_t p = (int32_t)new_len;
    // positions >= new_len are overwritten by later appends; only the
    // position moves (QuantStreamCache::truncate narrows the cache to new_len)
    return cuda_error(cudaMemcpy(m->pos, &p, 4, cudaMemcpyHostToDevice), "truncate");
}

int rq_llama_reset_tokens(rq_llama* m) {
    if (!m) return set_error(RQ_ERR_INVALID, "rq_llama_reset_tokens: NULL argument");
    Guard g(m->ctx->device);
    return cuda_error(cudaMemset(m->nout, 0, 4), "reset");
}

}  // extern "C"
