/*
 * rq_oracle.h -- CPU oracle for the quantized-linear / sparse-MoE path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: the tests, the
 * smoke check and the bench's CPU-baseline leg load it.  The product
 * (librq.so) never links or calls it.
 *
 * It restates, in plain C, the arithmetic rustyllm runs on the CPU:
 *   - Q4_0 repack quantizer            src/q4_kernel.rs:137-163
 *   - Q4_0 scalar dot                  src/q4_kernel.rs:274-293
 *   - Q4_0 AVX2 dot (lane order)       src/q4_kernel.rs:300-360
 *   - row-chunked threaded forward     src/q4_kernel.rs:207-243
 *   - GGML Q4_K / Q3_K dequantization  (candle-core 0.10.2 k-quants, reached
 *     through QMatMul at src/streaming_quantized.rs:63-70); pinned bit-for-bit
 *     against gguf-py 0.19.0 golden vectors in tests/golden/
 *   - GGML Q8_0 (quantizer and dequantization) and Q6_K / Q5_K / Q2_K
 *     dequantization, the other formats of src/quantize.rs:29-37; pinned
 *     against gguf-py 0.19.0 (Q8_0 quantize + dequantize, the K-types'
 *     dequantize) by tests/test_oracle.py
 *   - SparseMoe routing/permute/combine src/streaming_mixtral.rs:280-319
 *
 * Parity pins: Q4_0 follows the in-repo rule exactly.  Q4_K/Q3_K dequant is
 * pinned to gguf-py's published dequantizer.  The Q4_K/Q3_K *quantizer* here
 * is this project's own deterministic rule (candle's QTensor::quantize source
 * is not available); every parity test feeds identical block bytes to the
 * CPU and the GPU, so quantizer equality with candle is not needed for them.
 */
#ifndef RQ_ORACLE_H
#define RQ_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { RQO_F16 = 1, RQO_Q4_0 = 2, RQO_Q8_0 = 8, RQO_Q2_K = 10, RQO_Q3_K = 11, RQO_Q4_K = 12, RQO_Q5_K = 13, RQO_Q6_K = 14 };

uint16_t rqo_f32_to_f16(float f);
float rqo_f16_to_f32(uint16_t h);
void rqo_f32_to_f16_n(const float* x, uint16_t* h, int64_t n);
void rqo_f16_to_f32_n(const uint16_t* h, float* x, int64_t n);

/* bytes per block / elements per block of a GGML type; 0 if unknown */
int64_t rqo_block_bytes(int type);
int64_t rqo_block_elems(int type);

/* quantize rows x f32 [rows][in] -> GGML blocks (row-major) */
int rqo_quantize(int type, const float* x, int64_t rows, int64_t in, uint8_t* out);
/* dequantize GGML blocks -> f32 [rows][in] */
int rqo_dequantize(int type, const uint8_t* blocks, int64_t rows, int64_t in, float* out);

/* y[m][o] = sum_k x[m][k] * deq(W)[o][k], dequantize-then-dot.
 * acc64 = 0: f32 accumulation in ascending k; acc64 = 1: double accumulation. */
int rqo_matmul_ref(int type, const uint8_t* blocks, int64_t out, int64_t in,
                   const float* x, int64_t M, float* y, int acc64);

/* q4_kernel.rs dot restatements, one row */
float rqo_dot_q4_0_scalar(const uint8_t* w_row, const float* x_row, int64_t blocks_per_row);
float rqo_dot_q4_0_avx2order(const uint8_t* w_row, const float* x_row, int64_t blocks_per_row);

/* Threaded CPU forward, the CPU baseline.  Chunking follows
 * q4_kernel.rs:207-243.  Q4_0 uses the AVX2-order dot; Q4_K/Q3_K use a
 * dequant-fused f32 dot with 8 lanes.  nthreads <= 0 -> all cores. */
int rqo_linear_threaded(int type, const uint8_t* blocks, int64_t out, int64_t in,
                        const float* x, int64_t M, float* y, int nthreads);

/* The same products as rqo_linear_threaded (bit for bit), each weight row
 * dequantized once for all M activation rows (the oracle's fast path). */
int rqo_linear_rows(int type, const uint8_t* blocks, int64_t out, int64_t in, const float* x, int64_t M,
                    float* y, int nthreads);

/* ParallelLinear::forward (parallel_linear.rs:191-295): F16 weight w
 * [out][in] (IEEE half bits) times f32 x [n][in], chunked as :223-225.
 * avx2 = 1: the dot_f32_avx2_fma lane order (:64-94); 0: the scalar loop
 * (:48-55).  nthreads <= 0 -> all cores. */
int rqo_parallel_linear_f16(const uint16_t* w, int64_t out, int64_t in, const float* x, int64_t n,
                            float* y, int avx2, int nthreads);

/* ---- sparse MoE (streaming_mixtral.rs:280-319) ---- */
/* Router logits: the gate is a ParallelLinear with F16 weights wr16 [E][H]
 * (streaming_mixtral.rs:265,283), AVX2 lane order. */
void rqo_router_logits(const float* x, int64_t T, int64_t H, const uint16_t* wr16, int E, float* logits);
/* softmax + stable descending top-k with renormalised weights.
 * ids[T][k] in rank order, weights[T][k]. */
void rqo_route_topk(const float* logits, int64_t T, int E, int k, int32_t* ids, float* weights);
/* Bucket rows per expert in ascending token order.  offsets[E+1]; rows[T*k]
 * holds token ids; slot_w[T*k] the matching routing weights. */
void rqo_permute(const int32_t* ids, const float* weights, int64_t T, int E, int k,
                 int32_t* offsets, int32_t* rows, float* slot_w);
/* Full layer: route -> permute -> SwiGLU experts (w1=gate, w3=up, w2=down)
 * -> weighted combine in ascending expert order.  w1/w3: [E] pointers to
 * [F][H] weights; w2: [E] pointers to [H][F].  wtype = a GGML block type
 * (quantized experts) or RQO_F16 (F16 half bits: the reference's own
 * ParallelLinear experts, streaming_mixtral.rs:231-257).  wr16: F16 router
 * weight [E][H]. */
int rqo_moe_forward(const float* x, int64_t T, int64_t H, int64_t F, int E, int k,
                    const uint16_t* wr16, int wtype, const uint8_t* const* w1,
                    const uint8_t* const* w3, const uint8_t* const* w2, float* y,
                    int32_t* ids_out, int32_t* perm_out, int32_t* offsets_out,
                    int nthreads);

/* silu in f32: x / (1 + exp(-x)) (candle_nn::ops::silu) */
float rqo_silu(float x);

/* Quantized Llama forward (src/streaming_quantized.rs:193-317,611-633) with
 * its own KV cache; weights are borrowed (GGML blocks of type wtype for the
 * seven linears q,k,v,o,gate,up,down; F16 embedding and lm_head). */
typedef struct rqo_llama rqo_llama;
rqo_llama* rqo_llama_create(int64_t hidden, int64_t inter, int64_t n_heads, int64_t n_kv,
                            int64_t head_dim, int64_t n_layers, int64_t vocab, int64_t max_seq,
                            float eps, float theta, int wtype);
void rqo_llama_free(rqo_llama* m);
int rqo_llama_set_layer(rqo_llama* m, int64_t layer, const uint8_t* const* w7, const float* rms1,
                        const float* rms2);
void rqo_llama_set_embedding(rqo_llama* m, const uint16_t* emb);
void rqo_llama_set_head(rqo_llama* m, const float* ln_f, const uint16_t* lm_head);
int rqo_llama_forward(rqo_llama* m, const int32_t* tokens, int64_t T, int64_t index_pos,
                      float* logits_last, int32_t* next, int nthreads);
/* The forward in pieces, so a model too large for host memory can be run a
 * layer at a time (set_layer, layer, drop the blocks): x[T][H] = embedding
 * rows; one QBlock over x in place at positions pos..pos+T-1; final norm
 * and lm_head of every row of x (logits [T][vocab] may be NULL). */
void rqo_llama_embed(const rqo_llama* m, const int32_t* tokens, int64_t T, float* x);
int rqo_llama_layer(rqo_llama* m, int64_t layer, float* x, int64_t T, int64_t pos, int nthreads);
int rqo_llama_head(const rqo_llama* m, const float* x, int64_t T, float* logits, int32_t* argmax, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
