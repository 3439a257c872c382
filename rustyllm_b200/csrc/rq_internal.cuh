// rq_internal.cuh -- shared definitions of librq (not part of the ABI).
#pragma once

#include <vector>

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/rq.h"

namespace rq {

// ------------------------------------------------------------ device layout
//
// A weight lives on the GPU split into two arrays, both row-major over
// [out][nblk] (nblk = in / block elements):
//   qs  : the quant bytes of each block, 16-byte aligned per block so that
//         128-bit loads are aligned and coalesced;
//   hdr : the per-block scale bytes.
//   Q4_K  qs 128 B (GGML bytes 16..143)     hdr 16 B (d, dmin, 12 scale bytes)
//   Q3_K  qs 128 B (q + 4 as nibbles)       hdr 20 B (16 int8 scales, d, 2 pad)
//   Q4_0  qs  16 B (GGML bytes 2..17)       hdr  2 B (d)
// Bytes keep their GGML order inside each part, so the total equals the GGML
// size -- except Q3_K, which is expanded at upload: its 3-bit values (2 low
// bits + hmask bit) become nibbles in Q4_K's arrangement (byte j of 64-element
// group c: element 64c + j low, 64c + 32 + j high) and its packed 6-bit
// scales become int8, so its matvec lane is a Q4_K lane (the 3-bit unpacking
// made it ALU-bound); 148 device bytes per 110 GGML bytes, and the layout
// kernels convert both ways exactly.
struct TypeInfo {
    int type;
    int block_elems;  // 32 or 256
    int block_bytes;  // GGML bytes per block
    int qs_bytes;     // device quant bytes per block
    int hdr_bytes;    // device header bytes per block
};

__host__ __device__ inline TypeInfo type_info(int t) {
    switch (t) {
    case RQ_Q4_K: return TypeInfo{RQ_Q4_K, 256, 144, 128, 16};
    case RQ_Q3_K: return TypeInfo{RQ_Q3_K, 256, 110, 128, 20};
    case RQ_Q4_0: return TypeInfo{RQ_Q4_0, 32, 18, 16, 2};
    case RQ_Q8_0: return TypeInfo{RQ_Q8_0, 32, 34, 32, 2};
    // Q6_K: quant part ql[128] qh[64]; header scales[16] d[2] + 2 bytes of
    // padding (4-byte aligned headers)
    case RQ_Q6_K: return TypeInfo{RQ_Q6_K, 256, 210, 192, 20};
    // Q5_K: quant part qh[32] qs[128]; header d dmin scales[12] (as Q4_K)
    case RQ_Q5_K: return TypeInfo{RQ_Q5_K, 256, 176, 160, 16};
    // Q2_K: quant part qs[64]; header scales[16] d[2] dmin[2]
    case RQ_Q2_K: return TypeInfo{RQ_Q2_K, 256, 84, 64, 20};
    default: return TypeInfo{0, 0, 0, 0, 0};
    }
}

// ------------------------------------------------------ activation staging
//
// The linear kernels consume activations pre-quantized per 32-element block
// into a 24-bit fixed-point value X = rint(x * 127*65536 / amax) split into
// three balanced signed bytes (X = 65536*x1 + 256*x2 + x3), stored as three
// int8 planes, plus per block: sx = amax / (127*65536), the f32 sum of the
// first 16, of the last 16 elements.  |x - X*sx| <= ~1.5*sx, i.e. about
// 2e-7 of the block's largest magnitude, so the integer dot products that
// follow lose nothing measurable against the f32 path.
constexpr float kXQScale = 8323072.0f;  // 127 * 65536

struct XQ {             // one activation matrix [M][in] in staged form
    int8_t* planes;     // [M][3][in]
    float4* stats;      // [M][in/32] : (sx, sum16a, sum16b, 0)
};

inline size_t xq_bytes(int64_t M, int64_t in) {
    size_t p = (size_t)M * 3 * (size_t)in;
    p = (p + 255) & ~(size_t)255;
    return p + (size_t)M * (size_t)(in / 32) * sizeof(float4);
}

}  // namespace rq

struct rq_weight {
    int type;
    int64_t out, in, nblk;
    uint8_t* qs;
    uint8_t* hdr;
    void* base;   // single allocation holding qs and hdr
    size_t bytes; // allocation size
    int device;
};

namespace rq {
struct TPComm;
}

struct rq_ctx {
    rq::TPComm* tp;  // tensor-parallel communicator (rq_tp_init), or NULL
    int device;
    cudaStream_t own_stream;  // used for host-pointer calls when stream == NULL
    void* ws;                 // workspace (activation staging, host-path buffers)
    size_t ws_bytes;
    int sm_count;
    float* sk_ws = nullptr;  // skinny matmul: split-K tile pieces
    size_t sk_ws_floats = 0;
    int* sk_cnt = nullptr;   // skinny matmul: arrivals per tile (kept at zero between launches)
    int sk_cnt_n = 0;
    // Error word of the context's kernels: a bounded wait (mbarrier, peer
    // flag) that gives up sets it to 1 and the kernel returns.  Synchronous
    // calls read it back (err_host, page-locked) before returning;
    // rq_ctx_status reads it for asynchronous ones.
    int* derr = nullptr;
    int* err_host = nullptr;
    int* i8_cnt = nullptr;   // int8 matmul split-K arrivals per row group (kept at zero between launches)
    // rq_linear_prefetch_hint: weights whose first rows the next M=1
    // pipeline launch of this context prefetches into L2 in its tail
    const rq_weight* hint_w[3] = {nullptr, nullptr, nullptr};
    int hint_n = 0;
};

namespace rq {

// tensor parallel (rq_tp.cu): world/rank are 1/0 without a communicator;
// dtype 0 = f32, 1 = u64; op 0 = sum, 1 = max
int tp_world(const rq_ctx* ctx);
int tp_rank(const rq_ctx* ctx);
int tp_allreduce(rq_ctx* ctx, const void* in, void* out, int64_t n, int dtype, int op, cudaStream_t st);
// the peer-memory exchange regions of the communicator, if it has them
struct P2PArgs;
bool tp_p2p_args(const rq_ctx* ctx, P2PArgs* a);
// Whether a row-parallel M=1 matvec does its all-reduce inside the matvec
// kernel (the fused epilogue; same bits as the separate kernel) at `world`
// ranks: the default at every world size; RQ_TP_FUSED=0 in the environment
// turns it off (the separate peer-memory kernel then runs).
bool tp_fused_enabled(int world);
void tp_destroy(rq_ctx* ctx);
// all-gather of nbytes from every rank into out[world][nbytes]
int tp_allgather_bytes(rq_ctx* ctx, const void* in, void* out, int64_t nbytes, cudaStream_t st);
// all-to-all with per-peer byte counts and offsets (ncclSend/ncclRecv in one
// group; the rank's own share is a device copy)
int tp_alltoallv_bytes(rq_ctx* ctx, const void* send, const int64_t* send_bytes, const int64_t* send_off, void* recv,
                       const int64_t* recv_bytes, const int64_t* recv_off, cudaStream_t st);

// GGUF shard directory -> a Llama model (rq_gguf.cu): per layer the 7
// linears (out x in of this rank's shard in dims7_out / dims7_in, q, k, v,
// o, gate, up, down) and the two norms, then embedding, final norm, head.
// The uploaded weights are appended to `owned`.
int llama_load_gguf_dir(rq_ctx* ctx, rq_llama* m, const char* dir, int64_t n_layers, int64_t vocab, int64_t hidden,
                        int world, int rank, const int64_t* dims7_out, const int64_t* dims7_in,
                        std::vector<rq_weight*>& owned);

// error handling (rq_api.cu)
int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
int ensure_workspace(rq_ctx* ctx, size_t bytes);
// Queue the copy of ctx's kernel error word to the host on st (before the
// call's final synchronisation) ...
int queue_error_readback(rq_ctx* ctx, cudaStream_t st);
// ... and after that synchronisation: RQ_ERR_TIMEOUT (word cleared) when a
// kernel's bounded wait gave up, else RQ_OK.
int take_kernel_error(rq_ctx* ctx, cudaStream_t st, const char* what);
// the error word of rq_linear_noalloc's kernels on device dev (rq_static.cu):
// 1 if set since the last call (and cleared), 0 if not, < 0 on a CUDA error
int static_error_take(int dev);

// layout kernels (rq_layout.cu)
int launch_repack(const rq_weight* w, const uint8_t* raw_dev, int64_t row0, int64_t rows,
                  cudaStream_t st);
int launch_unpack(const rq_weight* w, uint8_t* raw_dev, int64_t row0, int64_t rows,
                  cudaStream_t st);
int launch_dequant(const rq_weight* w, float* y, cudaStream_t st);
int launch_quantize(const rq_weight* w, const float* x, cudaStream_t st);

// bulk-copy pipelined matvec (rq_mv_pipe.cu): up to kMaxJobs independent
// M=1 matvecs with the same type and K in one launch; err may be NULL
constexpr int kMaxJobs = 8;
struct PipeJob {
    const uint8_t* qs;
    const uint8_t* hdr;
    XQ xq;             // the staged activation row of this job
    float* y;
    const float* add;  // optional residual: y = x W^T + add (may alias y)
    int64_t out;
};
// Jobs whose weight is chosen on the device (the sparse-MoE expert of a
// routing slot): job j's weight is (qs[kind[j]][e], hdr[kind[j]][e]) with e =
// slot_e[slot[j]] -- slot_e written by an earlier kernel in the stream, the
// tables device arrays of per-expert pointers (kind: gate, up, down).  The
// jobs' qs / hdr fields are then ignored; every table entry has the shape
// and type of the launch's representative weights.
struct PipeDevWeights {
    const int32_t* slot_e;        // [slots] expert of each routing slot (device)
    const uint8_t* const* qs[3];  // [kind] -> [E] (device)
    const uint8_t* const* hdr[3];
    int slot[kMaxJobs];           // routing slot of each job
    int kind[kMaxJobs];
};
bool pipe_supported(const rq_weight* w);
// With ar (one job, row-parallel under tensor parallelism): the partial y is
// all-reduced over the ranks' NVLink exchange regions inside the kernel and
// y receives the sum; returns kPipeNotFusable (no error set) when the launch
// cannot be fused.
struct P2PArgs;
constexpr int kPipeNotFusable = -1;
// SwiGLU staging epilogue: jobs come in pairs (2i gate, 2i+1 up) of one
// shape, out a multiple of 32.  Besides writing y, the kernel stages
// silu(gate) * up of pair i into row row0 + i of xq, with the arithmetic of
// launch_xquant_swiglu, for the down projection.  A 32-row block spans CTAs:
// each CTA adds the rows it wrote to the block's arrival counter
// cnt[(row0 + i) * out / 32 + block] and the CTA that completes the block
// (64 rows) stages it and zeroes the counter.  cnt starts zeroed.
struct PipeSwiglu {
    XQ xq;
    int* cnt;
    int row0;
};
// Sparse-MoE combine epilogue: the jobs are the down projections of routing
// slots slot0 .. slot0 + njobs - 1 in token-major order (slot t * k + r is
// the r-th pick of token t, njobs and slot0 multiples of k), so the k slots of
// a token share a CTA's rows.  Instead of writing y the kernel writes
// out[t][c] = sum over the token's slots in ascending expert order of
// wts[s] * o_s[c] (combine_kernel's arithmetic).
struct PipeCombine {
    const int32_t* ids;  // [slots] expert of each slot (device)
    const float* wts;    // [slots] routing weight of each slot (device)
    float* out;          // [tokens][out]
    int k, slot0;
};
// L2 prefetch of the weights the next launch in the stream will read: once
// the producer has issued its last copy, it prefetches into L2 (bulk
// prefetch, no shared memory) the first `budget` bytes of the rows its CTA
// index will own in that launch (grid = the SM count), so HBM keeps
// streaming through this launch's tail, the launch gap and the kernels in
// between (attention).  A hint only: nothing reads the prefetched lines
// except the next launch's ordinary copies.
constexpr int kMaxNext = 3;
struct PipeNext {
    const uint8_t* qs[kMaxNext];
    const uint8_t* hdr[kMaxNext];
    int64_t out[kMaxNext];  // rows of each weight
    uint32_t qrow, hrow;    // device bytes per row (quant part, header part)
    int n;                  // weights (0: no prefetch)
    uint32_t budget;        // bytes per CTA over all n weights
};
PipeNext pipe_next(const rq_weight* const* ws, int n, uint32_t budget);
// RMSNorm staging epilogue (one job whose y is the residual stream): the CTA
// that completes a 32-row block of y (arrival counters, as PipeSwiglu)
// stages v = y * w over the block into xq (the staging kernel's per-block
// arithmetic) and writes the block's sum of squares to ss[block].  The norm's
// 1 / sqrt(mean + eps) is not applied: the matvec that reads xq scales its
// outputs by it (PipeRmsIn), which is the same linear map.
struct PipeRms {
    XQ xq;
    float* ss;       // [out / 32] block sums of squares
    int* cnt;        // [out / 32] arrival counters (zero between launches)
    const float* w;  // RMSNorm weight [out]
};
// Outputs divided by sqrt(sum of ss[0..nb) / n + eps) (the sum in a fixed order).
struct PipeRmsIn {
    const float* ss;
    int nb;
    float n, eps;
};
int launch_matvec_pipe(const rq_weight* const* ws, const XQ* xqs, float* const* ys, int njobs,
                       int sm_count, cudaStream_t st, int* err = nullptr,
                       const float* const* adds = nullptr, const P2PArgs* ar = nullptr,
                       const PipeDevWeights* dw = nullptr, const PipeSwiglu* sw = nullptr,
                       const PipeCombine* cmb = nullptr, const PipeNext* next = nullptr,
                       const PipeRms* rms = nullptr, const PipeRmsIn* rsi = nullptr);

// small-M Q4_K matmul on the tensor cores (rq_mm_small.cu).  Activations are
// staged per row as x / s = hi + lo (two f16 values per element, s a power of
// two), quad-permuted, with f32 sums per 32-element block:
struct XH {
    __half* v;     // [rows][2][in]: hi plane, lo plane
    float* scale;  // [rows]
    float* bsum;   // [rows][in/32]
    __half* bs16;  // [rows][in/256][16]: the 8 block sums of a super-block as f16 hi, then f16 lo
};
size_t xh_bytes(int64_t rows, int64_t in);
XH xh_at(void* base, int64_t rows, int64_t in);

// Q4_K matmul for two activation rows on the int8 tensor cores
// (rq_mm_i8.cu).  Activations staged per token and 256-element super-block
// as X = rint(x * 127*65536 / amax) split into three balanced bytes with
// sx = amax / (127*65536), plus the f32 sum of every 32-element block.
struct XQ2 {
    int8_t* planes;  // [M][3][in]
    float* sx;       // [M][in/256]
    float* bsum;     // [M][in/32]
};
size_t xq2_bytes(int64_t M, int64_t in);
XQ2 xq2_at(void* base, int64_t M, int64_t in);
// stages x (M rows), with rms_w RMSNorm(x) * rms_w (eps), or with up
// silu(x) * up into q
int launch_xq2_stage(const float* x, int64_t M, int64_t in, XQ2 q, cudaStream_t st, const float* rms_w = nullptr,
                     float eps = 0.0f, const float* up = nullptr);
// whether weight w takes the int8 kernel for M rows (Q4_K, M = 2..4,
// in = 2048 .. 8192 in steps of 2048, or a multiple of 1024 up to 32768 with
// K split over four CTAs per row group)
bool mm_i8_supported(const rq_weight* w, int64_t M);
// scratch floats a launch on w needs for its split-K partial rows (0: none)
size_t mm_i8_scratch_floats(const rq_weight* w, int64_t M);
// y_j[M][out_j] = x W_j^T (+ add_j) for up to kMaxJobs weights of the same
// in; a split K (one job) needs part (mm_i8_scratch_floats) and cnt (256
// arrival counters, zero between launches, left zero)
int launch_mm_i8(const rq_weight* const* ws, float* const* ys, int njobs, int64_t M, XQ2 xq, int sm_count,
                 cudaStream_t st, int* err, const float* const* adds = nullptr, float* part = nullptr,
                 int* cnt = nullptr);
int launch_xh_stage(const float* x, int64_t M, int64_t in, XH xh, cudaStream_t st);
// the same staging of RMSNorm(x) * w, and of silu(gate) * up
int launch_xh_stage_rmsnorm(const float* x, const float* w, float eps, int64_t M, int64_t in, XH xh,
                            cudaStream_t st);
int launch_xh_stage_swiglu(const float* gate, const float* up, int64_t M, int64_t in, XH xh, cudaStream_t st);
// Up to kMaxJobs jobs with the same K, each y_j[M_j][out_j] = x[tok0_j ..
// tok0_j + M_j) W_j^T (+ add_j), M_j <= 8, all reading one staged matrix of
// `rows` rows; err may be NULL.
struct MMJobDesc {
    const rq_weight* w;
    int tok0, M;
    float* y;
    const float* add;
};
bool mm_small_supported(const rq_weight* w);
constexpr int64_t kMinTensorM = 4;  // smallest M routed to the tensor-core kernels
int launch_mm_small(const MMJobDesc* jobs, int njobs, XH xh, int64_t rows, int sm_count, cudaStream_t st,
                    int* err = nullptr);
// y[M][out] = x W^T (+ add) for M >= 2 staged rows, in tiles of 8 rows
int launch_matmul_small(const rq_weight* w, XH xh, int64_t M, float* y, const float* add, int sm_count,
                        cudaStream_t st, int* err = nullptr);
// Q4_K matmul on tcgen05 (rq_mm_tc.cu) for jobs of any M: 128 weight rows x
// up to 128 tokens per tile, f32 accumulators in TMEM; same staged matrix and
// job descriptors as launch_mm_small (no limit on M_j); err may be NULL.
constexpr int64_t kMinTcgenM = 24;  // smallest M routed to the tcgen05 kernel (measured crossover)
// M = 9..16 per job: tcgen05 with the raw quants as operands, per-sub-block
// accumulators and split-K over all SMs (rq_mm_skinny.cu); same job
// descriptors, every job M_j <= kSkinnyMaxM.  Below kSkinnyMinM the
// mma.sync kernel is faster (one tcgen05.mma of 128 x 16 x 16 issues only
// every ~60-100 cycles, which caps this kernel near 1.3 TB/s of weights at
// any M; mma.sync's 8-row tiles cost the same and M <= 8 needs one tile).
constexpr int kSkinnyMinM = 9;
constexpr int kSkinnyMaxM = 16;
int launch_mm_skinny(rq_ctx* ctx, const MMJobDesc* jobs, int njobs, XH xh, int64_t rows, cudaStream_t st,
                     int* err = nullptr);
// grow ctx's split-K scratch to floats / tiles (never during stream capture)
int ensure_skinny_scratch(rq_ctx* ctx, size_t floats, int tiles);
bool mm_tc_supported(const rq_weight* w);
// Q3_K rows from which one tcgen05 pass beats a pipeline pass per row (the
// int8 kernels take precedence where they take the shape)
constexpr int64_t kQ3TensorMinM = 6;
inline bool q3k_tensor_m(const rq_weight* w, int64_t M) {
    return M >= kQ3TensorMinM && w->type == RQ_Q3_K && mm_tc_supported(w) && !mm_i8_supported(w, M);
}
int launch_mm_tc(const MMJobDesc* jobs, int njobs, XH xh, int64_t rows, int sm_count, cudaStream_t st,
                 int* err = nullptr);

// linear kernels (rq_matvec.cu).  launch_linear runs y = x W^T for M staged
// activation rows (launch_xquant first).  launch_xquant_rows stages up to
// kMaxJobs separate rows (row j of `in` floats at xs[j]) into consecutive
// rows of xq in one launch.
int launch_xquant(const float* x, int64_t M, int64_t in, XQ xq, cudaStream_t st);
// Staging with a fused producer op (one CTA per row): RMSNorm
// (x / sqrt(mean(x^2) + eps) * w, candle_nn::ops::rms_norm order) or SwiGLU
// (silu(x) * up).
int launch_xquant_rmsnorm(const float* x, const float* w, float eps, int64_t M, int64_t in, XQ xq,
                          cudaStream_t st);
int launch_xquant_swiglu(const float* gate, const float* up, int64_t M, int64_t in, XQ xq,
                         cudaStream_t st);
int launch_xquant_rows(const float* const* xs, int n, int64_t in, XQ xq, cudaStream_t st);
struct PipeNext;
int launch_linear(const rq_weight* w, XQ xq, float* y, int64_t M, int sm_count, cudaStream_t st,
                  int* err = nullptr, const PipeNext* next = nullptr);
// The context's prefetch hint as a PipeNext (and the hint cleared), or n = 0.
PipeNext take_hint(rq_ctx* ctx);

}  // namespace rq
