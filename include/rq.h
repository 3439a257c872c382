/*
 * rq.h -- C ABI of librq, the B200 (sm_100a) quantized-linear and sparse-MoE
 * library behind rustyllm's q4_kernel / StreamingLlamaQuantized /
 * StreamingMixtral APIs.
 *
 * Conventions
 *   - Every entry point returns int: RQ_OK (0) on success, otherwise an
 *     RQ_ERR_* code; rq_last_error() then returns a thread-local message.
 *     This maps onto the reference's `Error::Msg(String)` (src/error.rs:4-29)
 *     the way q4_kernel.rs:90-107 builds its messages.  Nothing aborts.
 *   - Weights are GGML block bytes exactly as they sit in a GGUF tensor
 *     (Q4_0 = 18-byte blocks of 32, Q4_K = 144-byte super-blocks of 256,
 *     Q3_K = 110-byte super-blocks of 256; also Q8_0 = 34 / 32, Q6_K = 210,
 *     Q5_K = 176 and Q2_K = 84 bytes per 256), row-major [out][in/block].
 *     The library copies them to the GPU and owns the device copy.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 *   - Activation pointers (x, y) may be host or device memory.  Page-locked
 *     host memory (cudaHostAlloc / cudaHostRegister) is used in place: the
 *     kernels read x and write y over the bus.  Pageable host memory is
 *     staged through device memory.  With any host pointer the call returns
 *     with y filled and x no longer read; with device pointers only it is
 *     asynchronous on `stream`.
 *   - One rq_ctx per device; calls on one ctx are serialised by the caller
 *     (the reference's single-writer generate loop,
 *     src/streaming_quantized.rs:345-351).  Weight handles are read-only
 *     during forward calls and may be shared between threads.
 */
#ifndef RQ_H
#define RQ_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define RQ_API
#else
#define RQ_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct rq_ctx rq_ctx;
typedef struct rq_weight rq_weight;
typedef struct rq_moe rq_moe;

enum rq_status {
    RQ_OK = 0,
    RQ_ERR_INVALID = 1,     /* bad argument, shape or type */
    RQ_ERR_CUDA = 2,        /* CUDA runtime error */
    RQ_ERR_UNSUPPORTED = 3, /* valid request the library does not implement */
    RQ_ERR_OOM = 4,         /* device allocation failed */
    RQ_ERR_TIMEOUT = 5,     /* a bounded device or host wait gave up */
    RQ_ERR_NCCL = 6         /* collective failed */
};

/* GGML type ids (ggml_type / candle GgmlDType numbering). */
enum rq_ggml_type { RQ_Q4_0 = 2, RQ_Q8_0 = 8, RQ_Q2_K = 10, RQ_Q3_K = 11, RQ_Q4_K = 12, RQ_Q5_K = 13, RQ_Q6_K = 14 };

/* ---------------------------------------------------------------- context */

/* Create a context on CUDA device `device`.  Replaces the implicit candle
 * Device::Cuda(n) of src/inference.rs:56-70. */
RQ_API int rq_init(int device, rq_ctx** out);
RQ_API int rq_destroy(rq_ctx* ctx);

/* Copy the calling thread's last error message into buf (NUL-terminated,
 * truncated to n).  Returns the full message length. */
RQ_API int rq_last_error(char* buf, size_t n);

/* Synchronise the context's device and report whether a bounded wait
 * (mbarrier or peer flag, ~1 s) inside a kernel of an asynchronous call on
 * this context -- or of rq_linear_noalloc on this device -- gave up since the
 * last check: RQ_ERR_TIMEOUT (record cleared; the outputs of those calls are
 * incomplete), else RQ_OK.  Calls with host buffers check this themselves
 * before they return.  No reference counterpart (candle's CPU kernels cannot
 * time out). */
RQ_API int rq_ctx_status(rq_ctx* ctx);

/* "rq <version> sm_100a" */
RQ_API const char* rq_version(void);

/* Bytes / elements per GGML block; 0 for an unknown type. */
RQ_API size_t rq_block_bytes(int ggml_type);
RQ_API int rq_block_elems(int ggml_type);

/* ---------------------------------------------------------------- weights */

/* Upload GGML blocks [out][in/block] (host or device pointer, nbytes must be
 * exactly out*in/block*block_bytes).  Replaces QMatMul::from_arc over a
 * GgufLayer tensor (src/streaming_quantized.rs:63-70) and
 * ParallelQ4Linear::from_qtensor (src/q4_kernel.rs:89-171); in must be a
 * multiple of the block size (src/q4_kernel.rs:104-108). */
RQ_API int rq_weight_upload(rq_ctx* ctx, int ggml_type, const void* blocks, size_t nbytes,
                     int64_t out, int64_t in, rq_weight** w);

/* Quantize an f32 matrix [out][in] that is already on this device straight
 * into a device weight (no host round trip); the call returns once the
 * weight is written.  Q4_0 follows the rule of
 * src/q4_kernel.rs:137-163, Q8_0 GGML's rounding rule; the K-types use
 * librq's deterministic quantizers
 * (the counterpart of candle's QTensor::quantize, src/quantize.rs:131). */
RQ_API int rq_weight_quantize(rq_ctx* ctx, int ggml_type, const float* w_dev, int64_t out, int64_t in,
                       rq_weight** w, void* stream);

/* Copy a device weight back as GGML blocks into host memory. */
RQ_API int rq_weight_download(rq_ctx* ctx, const rq_weight* w, void* blocks_host, size_t nbytes);

RQ_API int rq_weight_free(rq_ctx* ctx, rq_weight* w);

/* Any of the out-pointers may be NULL.  device_bytes counts the library's
 * device copy: the GGML byte count, plus 2 pad bytes per Q6_K super-block;
 * Q3_K is held expanded (4-bit values and int8 scales, 148 bytes per
 * 110-byte super-block) so that its matvec is not bound by unpacking. */
RQ_API int rq_weight_info(const rq_weight* w, int* ggml_type, int64_t* out, int64_t* in,
                   size_t* device_bytes);

/* y[out][in] = dequantized weight in f32, bit-identical to GGML's dequant
 * (QTensor::dequantize, used at src/q4_kernel.rs:120-122). */
RQ_API int rq_dequantize(rq_ctx* ctx, const rq_weight* w, float* y, void* stream);

/* ----------------------------------------------------------------- linear */

/* y[M][out] = x[M][in] * W^T in f32.  Replaces QMatMul::forward
 * (src/streaming_quantized.rs:201-203,256,277-278) and
 * ParallelQ4Linear::forward (src/q4_kernel.rs:183-256).  M=1 is the decode
 * matvec; M=K+1 the speculative verify (examples/spec_decode_70b.rs:238);
 * larger M the prefill (src/streaming_quantized.rs:569-575). */
RQ_API int rq_linear(rq_ctx* ctx, const rq_weight* w, const float* x, float* y, int64_t M,
              void* stream);

/* n (1..8) independent decode matvecs y_i[1][out_i] = x_i[1][in] * W_i^T in
 * one launch, for weights of the same type and in_features -- the q/k/v
 * projections of QAttn::forward (src/streaming_quantized.rs:201-203) or the
 * gate/up projections of QMlp::forward (:277), which read the same x.  The
 * weights are streamed back to back without a pipeline drain between them;
 * x_i may alias one another.  x and y must be device memory on the context's
 * device.  Results equal n rq_linear calls with M = 1. */
RQ_API int rq_linear_batch(rq_ctx* ctx, int n, const rq_weight* const* w, const float* const* x,
                           float* const* y, void* stream);

/* A prefetch hint, no reference counterpart: the next M=1 pipeline launch
 * of rq_linear / rq_linear_batch / rq_linear_allreduce on this context
 * prefetches into L2, after its last weight copy, the first rows of these n
 * (<= 3, of one type and in_features) weights -- the weights the caller
 * multiplies next, as a layer loop knows them -- so HBM keeps streaming
 * through the launch gap.  Consumed by that launch; n = 0 clears it.  No
 * effect on results; captured into CUDA graphs like the launch itself. */
RQ_API int rq_linear_prefetch_hint(rq_ctx* ctx, int n, const rq_weight* const* w);

/* Row-parallel linear under tensor parallelism: y[M][out] = the sum over
 * the ranks of x_r[M][in] * W_r^T, where W_r is this rank's column slice of
 * the weight (the o_proj / down_proj shard) and x_r its slice of the input;
 * every rank calls with the same M and gets the same y bits.  At M = 1 the
 * all-reduce runs inside the matvec kernel: each CTA stores its rows of the
 * partial product straight into every peer's NVLink exchange buffer and sums
 * the W slots in rank order once the peers have flagged theirs; otherwise
 * (or with RQ_TP_FUSED=0) the partial product is all-reduced by a separate
 * kernel (NCCL above 512 K elements).  x and y are device memory;
 * asynchronous on `stream`; needs rq_tp_init.  No reference counterpart (the
 * reference runs on one device). */
RQ_API int rq_linear_allreduce(rq_ctx* ctx, const rq_weight* w, const float* x, float* y, int64_t M,
                               void* stream);

/* rq_linear for callers that cannot allocate device memory.  No counterpart
 * in the reference.
 *
 * rq_linear stages activations in a workspace it grows with cudaMalloc.
 * Callers whose device memory is owned by someone else (a serving engine
 * that reserves nearly all HBM up front, a framework allocator such as
 * candle's CUDA device) or whose decode loop cannot afford a cudaMalloc
 * that may synchronise the device use this entry point instead: it calls no
 * cudaMalloc, cudaFree or other allocating routine.  Its staging area is a
 * static 2 MiB device array that every GPU loading librq holds until exit.
 *
 *   - x [M][in] and y [M][out] must be device memory on w's device;
 *   - M * in is limited by the 2 MiB array at 3.5 bytes per element (plus
 *     alignment; e.g. M <= 20 at in = 28672, M <= 73 at in = 8192); larger
 *     requests fail with RQ_ERR_INVALID and a message;
 *   - every row runs the M=1 matvec kernels, so results match rq_linear's
 *     within the linear parity tolerance (relative L2 <= 1e-4; the same
 *     kernels at M = 1, while from M = 2 rq_linear takes its tensor-core
 *     kernels where the weight's type and shape allow); weights with no
 *     M=1 pipeline shape --
 *     Q8_0 / Q5_K with in not a multiple of 256, Q6_K / Q2_K with in not a
 *     multiple of 1024, any type with in > 30720 other than Q4_0 / Q4_K /
 *     Q3_K -- return RQ_ERR_UNSUPPORTED;
 *   - the first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress): make that first call before any stream
 *     capture;
 *   - all calls on a device share the one array, which keeps the last
 *     call's contents: calls that overlap on the GPU (other streams,
 *     threads) race on it, so serialise them;
 *   - the call is asynchronous on `stream`; a bounded kernel wait that gave
 *     up inside it is reported by rq_ctx_status on a context of that device. */
RQ_API int rq_linear_noalloc(const rq_weight* w, const float* x, float* y, int64_t M,
                             void* stream);

/* -------------------------------------------------------- tensor parallel */

/* One process per GPU.  Rank 0 creates an id (rq_tp_unique_id, >= 128
 * bytes), the host side distributes it (e.g. over torch.distributed), and
 * every rank calls rq_tp_init on its context.  Initialisation is bounded by
 * timeout_ms: a rank that never joins yields RQ_ERR_TIMEOUT on the others
 * (the communicator is aborted), never a hang.  No reference counterpart:
 * the reference is single-device (the build's TP splits the QAttn / QMlp
 * linears column- and row-parallel and joins them with all-reduces). */
RQ_API int rq_tp_unique_id(void* id_out, size_t n);
RQ_API int rq_tp_init(rq_ctx* ctx, int world, int rank, const void* id, int timeout_ms);
/* out[n] = sum over ranks of in[n] (f32), asynchronous on stream. */
RQ_API int rq_tp_allreduce_f32(rq_ctx* ctx, const float* in, float* out, int64_t n, void* stream);
/* RQ_OK while the communicator is healthy, RQ_ERR_NCCL after an async error. */
RQ_API int rq_tp_status(rq_ctx* ctx);
RQ_API int rq_tp_finalize(rq_ctx* ctx);

/* ------------------------------------------------------------- sparse MoE */

/* Mixtral SparseMoe (src/streaming_mixtral.rs:259-319) with quantized
 * experts: router weight f32 [E][hidden] (host or device; copied and rounded
 * to F16 as ParallelLinear::new does, src/parallel_linear.rs:128-131), expert
 * weights w1 = gate [ffn][hidden], w3 = up [ffn][hidden], w2 = down
 * [hidden][ffn] (borrowed: they must outlive the layer).  E <= 32.  Under a
 * communicator (rq_tp_init, world W > 1) the experts of other ranks (e % W
 * != rank) may be NULL: the layer then runs expert-parallel only. */
RQ_API int rq_moe_create(rq_ctx* ctx, int n_experts, int top_k, int64_t hidden, int64_t ffn,
                         const float* router_w, const rq_weight* const* w1,
                         const rq_weight* const* w3, const rq_weight* const* w2, rq_moe** out);
RQ_API int rq_moe_free(rq_moe* m);
/* y[T][hidden] = SparseMoe::forward(x[T][hidden]) (:280-319): router,
 * softmax, top-k with renormalised weights (ties to the lower expert index),
 * per-expert token buckets in ascending token order, SwiGLU experts, combine
 * in ascending expert order.  x, y host or device.  expert_ids_out [T][k]
 * (rank order) and perm_out [T*k] (tokens of expert 0, then expert 1, ...)
 * are optional host outputs.  With T < 4 (decode and speculative-verify
 * batches) no expert segment reaches the tensor-core kernels, so routing,
 * permutation and the expert products stay on the device: with device x /
 * y and no routing outputs the call is asynchronous on `stream` and can be
 * captured in a CUDA graph (after one call at that T outside capture, which
 * sizes the layer's buffers).  From T = 4 on, the per-expert token counts
 * are read back to the host once (the reference reads its whole routing
 * table there, :284-286) to pick each segment's kernel. */
/* Forwards of up to max_tokens tokens plan on the device (default and
 * minimum 3): every routing slot becomes one M=1 matvec job whose expert
 * the kernel reads from the routing table -- no host synchronisation,
 * asynchronous and graph-capturable at that T, slower than the host plan
 * from about 4 tokens (each slot streams its expert's weights). */
RQ_API int rq_moe_set_device_plan(rq_moe* m, int64_t max_tokens);

RQ_API int rq_moe_forward(rq_ctx* ctx, rq_moe* m, const float* x, float* y, int64_t T,
                          int32_t* expert_ids_out, int32_t* perm_out, void* stream);
/* Expert-parallel forward over the communicator of ctx: expert e lives on
 * rank e % W.  Each rank passes its own T tokens (T may differ per rank, 0
 * included; every rank must call).  Routing is local; the token rows go to
 * their experts' ranks and the expert outputs come back through NCCL
 * all-to-alls (ncclSend/ncclRecv), and each rank combines its own tokens in
 * ascending expert order.  y, expert_ids_out and perm_out as for
 * rq_moe_forward, for the local tokens; y equals rq_moe_forward on the same
 * tokens bit for bit. */
RQ_API int rq_moe_forward_ep(rq_ctx* ctx, rq_moe* m, const float* x, float* y, int64_t T,
                             int32_t* expert_ids_out, int32_t* perm_out, void* stream);

/* -------------------------------------------------------- Llama decode loop */

/* The quantized Llama forward of StreamingLlamaQuantized with every layer
 * resident on the GPU (src/streaming_quantized.rs:611-729, QBlock
 * :282-318), a per-layer f32 KV cache (QuantStreamCache :93-152) and the
 * greedy step of generate (:539-593).  Config mirrors candle's llama Config
 * fields the block uses (global sizes).  With a tensor-parallel communicator
 * on the context (world W, rank r), each rank holds shard r of every layer:
 * q/k/v/gate/up rows (heads r*n_heads/W.., kv heads r*n_kv_heads/W..,
 * intermediate rows r*intermediate/W..), the matching o/down columns, and
 * lm_head rows r*vocab/W..; the embedding and norms are replicated. */
typedef struct rq_llama rq_llama;
typedef struct rq_llama_config {
    int64_t hidden, intermediate, n_heads, n_kv_heads, head_dim, n_layers, vocab;
    int64_t max_seq;          /* KV cache capacity in positions */
    int64_t max_batch_tokens; /* most tokens per rq_llama_forward (prompt chunk) */
    float rms_eps, rope_theta;
} rq_llama_config;

RQ_API int rq_llama_create(rq_ctx* ctx, const rq_llama_config* cfg, rq_llama** out);
RQ_API int rq_llama_free(rq_llama* m);
/* Layer weights q,k,v,o,gate,up,down (this rank's shards; borrowed: they
 * must outlive m) and the two RmsNorm weights (f32 [hidden], host or device,
 * copied).  Replaces QBlock::load (src/streaming_quantized.rs:290-303). */
RQ_API int rq_llama_set_layer(rq_llama* m, int64_t layer, const rq_weight* const* w7,
                              const float* rms1, const float* rms2);
/* F16 [vocab][hidden] token embedding (model.embed_tokens.weight). */
RQ_API int rq_llama_set_embedding(rq_llama* m, const uint16_t* embed_f16);
/* Final RmsNorm weight (f32 [hidden]) and F16 lm_head rows of this rank
 * ([vocab/W][hidden]). */
RQ_API int rq_llama_set_head(rq_llama* m, const float* ln_f, const uint16_t* lm_head_f16);
/* forward(input_ids, index_pos) of src/streaming_quantized.rs:622-633 over T
 * host tokens at positions index_pos..index_pos+T-1: logits (host or device
 * [vocab], may be NULL; single rank only) of the last position and the
 * greedy next token (may be NULL).  Synchronous.  Leaves the next token and position on the device
 * for rq_llama_decode_step. */
RQ_API int rq_llama_forward(rq_llama* m, const int32_t* tokens, int64_t T, int64_t index_pos,
                            float* logits, int32_t* next_token, void* stream);
/* One greedy decode step entirely on the device (token and position read
 * from and written to device memory), so it can be captured in a CUDA graph
 * and replayed; each step appends its token to the device token list.  By
 * default a chain of per-layer kernels; rq_llama_set_fused(m, 1) makes the
 * step (one GPU, one weight type) a single persistent launch that streams the
 * weights through grid-wide phases and computes the same bits. */
/* The verify forward of speculative decoding (forward_all,
 * src/streaming_quantized.rs:611-620): T tokens at index_pos through every
 * layer, then the final norm and lm_head at EVERY position; argmax[T] (host
 * or device) receives each position's greedy token and logits[T][vocab]
 * (optional, one GPU only) the logits.  Like rq_llama_forward it leaves the
 * KV cache at index_pos + T and the last position's token as the next
 * input; rq_llama_truncate rolls back rejected positions. */
RQ_API int rq_llama_forward_all(rq_llama* m, const int32_t* tokens, int64_t T, int64_t index_pos, float* logits,
                                int32_t* argmax, void* stream);
RQ_API int rq_llama_decode_step(rq_llama* m, void* stream);
RQ_API int rq_llama_set_fused(rq_llama* m, int enable);
/* RQ_ERR_TIMEOUT (and clears it) when a bounded wait inside a kernel of the
 * model (a decode step, the one-launch step, a forward) gave up since the
 * last call; synchronous.  rq_llama_forward / _forward_all check it before
 * they return. */
RQ_API int rq_llama_status(rq_llama* m);
/* Tokens appended since the last reset (count may exceed cap), and the
 * current position.  Synchronous. */
RQ_API int rq_llama_tokens(rq_llama* m, int32_t* out, int64_t cap, int64_t* count,
                           int64_t* position);
RQ_API int rq_llama_reset_tokens(rq_llama* m);
/* QuantStreamCache::truncate / truncate_caches
 * (src/streaming_quantized.rs:131-141,603-609): roll the KV length back. */
RQ_API int rq_llama_truncate(rq_llama* m, int64_t new_len);

/* ------------------------------------------------------------------- GGUF */

/* A GGUF file read into host memory once (one sequential read, as
 * GgufLayer::open does, src/streaming_quantized.rs:42-61) and parsed:
 * versions 2 and 3, metadata skipped except general.alignment, tensor infos
 * bounds-checked against the file.  The format candle's gguf_file::write
 * emits for the reference's shards (src/quantize.rs:146-150). */
typedef struct rq_gguf rq_gguf;
RQ_API int rq_gguf_open(const char* path, rq_gguf** out);
/* the same from a caller-held buffer (copied), e.g. GgufLayer.buffer */
RQ_API int rq_gguf_open_memory(const void* data, size_t nbytes, rq_gguf** out);
RQ_API int rq_gguf_free(rq_gguf* f);
RQ_API int rq_gguf_tensor_count(const rq_gguf* f, int64_t* count);
/* index of a tensor by name (RQ_ERR_INVALID and index -1 when absent) */
RQ_API int rq_gguf_find(const rq_gguf* f, const char* name, int64_t* index);
/* name (NUL-terminated, truncated to name_cap), ggml type, n_dims, dims[4]
 * innermost first (a [out, in] matrix is {in, out, 1, 1}), offset of the
 * data in the file and its size (0 for an unknown type); NULL outputs are
 * skipped */
RQ_API int rq_gguf_tensor_info(const rq_gguf* f, int64_t index, char* name, size_t name_cap, int* ggml_type,
                               int* n_dims, int64_t* dims, uint64_t* file_offset, uint64_t* nbytes);
/* pointer to a tensor's bytes inside the file buffer (valid until free) */
RQ_API int rq_gguf_tensor_data(const rq_gguf* f, int64_t index, const void** data, uint64_t* nbytes);
/* the first `count` elements of an F32 / F16 / BF16 tensor as f32 (norms,
 * GgufLayer::tensor's dequantize, src/streaming_quantized.rs:74-83) */
RQ_API int rq_gguf_read_f32(const rq_gguf* f, const char* name, float* out, int64_t count);
/* Upload rows [row0, row0+rows) x columns [col0, col0+cols) of a 2-D Q4_0 /
 * Q4_K / Q3_K tensor (rows or cols < 0: to the end; columns on block
 * boundaries): GgufLayer::qmatmul (src/streaming_quantized.rs:63-70) with
 * the tensor-parallel shard taken on the host. */
RQ_API int rq_weight_upload_gguf(rq_ctx* ctx, const rq_gguf* f, const char* name, int64_t row0, int64_t rows,
                                 int64_t col0, int64_t cols, rq_weight** out);
/* Load a shard directory as StreamingLlamaQuantized::from_pretrained reads
 * it (src/streaming_quantized.rs:451-501): model.layers.<l>.gguf for every
 * layer (model.layers.<l>.self_attn.{q,k,v,o}_proj.weight,
 * .mlp.{gate,up,down}_proj.weight, .input_layernorm.weight,
 * .post_attention_layernorm.weight), model.embed_tokens.gguf,
 * model.norm.gguf and lm_head.gguf (absent: the head is the embedding).
 * Under tensor parallelism each rank uploads its own shards.  The model
 * owns the weights it uploads. */
RQ_API int rq_llama_load_gguf_dir(rq_llama* m, const char* dir);

#ifdef __cplusplus
}
#endif
#endif /* RQ_H */
