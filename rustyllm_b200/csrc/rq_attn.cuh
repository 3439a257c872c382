// rq_attn.cuh -- decode (T = 1) attention of one head, shared by the launch
// chain (attn_decode_kernel) and the one-launch decode step, so both compute
// the same bits.
#pragma once

#include "rq_async.cuh"
#include "rq_mv_common.cuh"

namespace rq {

constexpr int kAttnThreads = 480;  // threads that run one head

// Cached positions whose K and V rows the head copies into shared memory at
// its start (asynchronously, one round trip for all of them, while RoPE
// runs); later positions are read from the cache in place.
__host__ __device__ inline int attn_tile(int64_t hd) { return hd > 128 ? 16 : 32; }
__host__ __device__ inline int64_t attn_tile_off(int64_t max_seq, int64_t hd) {
    return (max_seq + 3 * hd + (kAttnThreads / hd) * hd + 3) & ~(int64_t)3;
}
// Shared floats the head needs: scores, roped q, new k, new v / output, the
// partial output sums of the position ranges, and the K / V tile.
__host__ __device__ inline int64_t attn_smem_floats(int64_t max_seq, int64_t hd) {
    return attn_tile_off(max_seq, hd) + 2 * (int64_t)attn_tile(hd) * hd;
}

// Head h of QAttn::forward (src/streaming_quantized.rs:201-257) for the one
// new token at position p = *pos: RoPE of q and of the new k (non-interleaved
// halves), KV-cache append by the first head of the kv group, scores q.k /
// sqrt(hd) over the p cached keys plus the new one, softmax, weighted values,
// and the staging of the head's hd outputs (hd / 32 blocks of row 0 of the
// o_proj input).  Run by kAttnThreads threads (tid 0..479) that synchronise
// with named barrier `bar`; `red` holds 32 floats.  No thread reads a cache
// slot written in this call.
__device__ __forceinline__ void attn_decode_head(const float* __restrict__ q, const float* __restrict__ k,
                                                 const float* __restrict__ v, float* __restrict__ kc,
                                                 float* __restrict__ vc, const float* __restrict__ cos_t,
                                                 const float* __restrict__ sin_t, const int32_t* __restrict__ pos,
                                                 int n_heads, int n_kv, int hd, int max_seq, int8_t* planes,
                                                 float4* stats, int h, int tid, int bar, float* sm, float* red) {
    constexpr int nthr = kAttnThreads, nw = kAttnThreads / 32;
    float* sc = sm;            // [max_seq] scores, then probabilities
    float* qs = sm + max_seq;  // [hd] roped q
    float* kn = qs + hd;       // [hd] roped new k
    float* vn = kn + hd;       // [hd] new v, then the head output
    float* part = vn + hd;     // [P][hd] partial outputs
    const int half = hd / 2, P = nthr / hd;
    const int pp = min(*pos, max_seq - 1);
    const int L = pp + 1;
    const int rep = n_heads / n_kv, kh = h / rep;
    const float* qh = q + (int64_t)h * hd;
    const float* ks = k + (int64_t)kh * hd;
    const float* vs = v + (int64_t)kh * hd;
    float* K = kc + (int64_t)kh * max_seq * hd;
    float* V = vc + (int64_t)kh * max_seq * hd;
    // K / V rows of the first np cached positions (written by earlier steps)
    // into the tile, in flight while RoPE runs
    const int np = min(pp, attn_tile(hd));
    float* kt = sm + attn_tile_off(max_seq, hd);
    float* vt = kt + (int64_t)attn_tile(hd) * hd;
    {
        const int chunks = np * hd / 4;  // 16-byte chunks per matrix (hd % 32 == 0)
        for (int i = tid; i < 2 * chunks; i += nthr) {
            const bool isv = i >= chunks;
            const int c = isv ? i - chunks : i;
            cp_async16((isv ? vt : kt) + 4 * c, (isv ? V : K) + 4 * c);
        }
        cp_async_commit();
    }
    for (int i = tid; i < half; i += nthr) {
        const float c = cos_t[(int64_t)pp * half + i], s = sin_t[(int64_t)pp * half + i];
        const float a = qh[i], b = qh[i + half];
        qs[i] = a * c - b * s;
        qs[i + half] = a * s + b * c;
        const float ka = ks[i], kb = ks[i + half];
        kn[i] = ka * c - kb * s;
        kn[i + half] = ka * s + kb * c;
    }
    for (int i = tid; i < hd; i += nthr) vn[i] = vs[i];
    cp_async_wait_all();
    named_bar_sync(bar, nthr);
    if (h % rep == 0)
        for (int i = tid; i < hd; i += nthr) {
            K[(int64_t)pp * hd + i] = kn[i];
            V[(int64_t)pp * hd + i] = vn[i];
        }
    const int warp = tid >> 5, lane = tid & 31;
    const float inv_sqrt = 1.0f / sqrtf((float)hd);
    for (int j = warp; j < L; j += nw) {
        const float* kj = j == pp ? kn : j < np ? kt + (int64_t)j * hd : K + (int64_t)j * hd;
        float acc = 0.0f;
        for (int d = lane; d < hd; d += 32) acc = fmaf(qs[d], kj[d], acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) sc[j] = acc * inv_sqrt;
    }
    named_bar_sync(bar, nthr);
    float mx = -INFINITY;
    for (int j = tid; j < L; j += nthr) mx = fmaxf(mx, sc[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    named_bar_sync(bar, nthr);
    mx = red[0];
    for (int w = 1; w < nw; w++) mx = fmaxf(mx, red[w]);
    named_bar_sync(bar, nthr);
    float sum = 0.0f;
    for (int j = tid; j < L; j += nthr) {
        const float e = expf(sc[j] - mx);
        sc[j] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[warp] = sum;
    named_bar_sync(bar, nthr);
    sum = 0.0f;
    for (int w = 0; w < nw; w++) sum += red[w];
    for (int j = tid; j < L; j += nthr) sc[j] = sc[j] / sum;
    named_bar_sync(bar, nthr);
    // P position ranges at once, summed in range order
    if (tid < P * hd) {
        const int d = tid % hd, r = tid / hd;
        const int j0 = r * L / P, j1 = (r + 1) * L / P;
        float acc = 0.0f;
#pragma unroll 4
        for (int j = j0; j < j1; j++)
            acc = fmaf(sc[j], j == pp ? vn[d] : j < np ? vt[(int64_t)j * hd + d] : V[(int64_t)j * hd + d], acc);
        part[r * hd + d] = acc;
    }
    named_bar_sync(bar, nthr);
    if (tid < hd) {
        float o = part[tid];
        for (int r = 1; r < P; r++) o += part[r * hd + tid];
        vn[tid] = o;
    }
    named_bar_sync(bar, nthr);
    const int nbh = hd / 32;
    if (tid < nbh) {
        float blk[32];
#pragma unroll
        for (int i = 0; i < 32; i++) blk[i] = vn[tid * 32 + i];
        stage_block(blk, 0, (int64_t)h * nbh + tid, (int64_t)n_heads * hd, planes, stats);
    }
}

}  // namespace rq
