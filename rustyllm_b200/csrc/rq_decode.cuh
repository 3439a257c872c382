// rq_decode.cuh -- the one-launch decode step of the resident Llama loop
// (rq_decode.cu), shared with its host side (rq_llama.cu).
#pragma once

#include "rq_internal.cuh"

namespace rq {

// One layer's weights (device layout: quant part, header part) and state.
struct DecLayer {
    const uint8_t* qs[7];  // q, k, v, o, gate, up, down
    const uint8_t* hdr[7];
    const float* rms1;
    const float* rms2;
    float* kc;  // [n_kv][max_seq][head_dim]
    float* vc;
};

struct DecParams {
    const DecLayer* layers;  // device array [n_layers]
    int n_layers;
    int type;  // GGML type of every linear
    int64_t H, I, nq, nk, head_dim, n_heads, n_kv, max_seq, vocab;
    float eps;
    // activations (f32) and staged activations
    float* x;
    float* q;
    float* k;
    float* v;
    float* g;
    float* u;
    XQ xq;
    const float* rope_cos;
    const float* rope_sin;
    const __half* embed;
    const float* ln_f;
    const __half* lm_head;
    // device state of the generate loop
    unsigned long long* best;
    int32_t* tokens;
    int32_t* pos;
    int32_t* out;
    int32_t* nout;
    unsigned* bar;  // grid barrier arrivals, zeroed before every launch
    int* err;       // set on a timed-out wait
    // pipeline geometry per K (0: hidden, 1: intermediate)
    int S[2], G[2], RS[2];
    uint32_t qrow[2], hrow[2];
    int64_t nblk[2];
    uint32_t slot_bytes;
    int nslot;
    uint32_t red_off, scratch_off, ring_off;
};

// Shared-memory plan and pipeline geometry for the model; false when the
// shapes do not fit the one-launch step (the caller keeps the launch chain).
bool decode_plan(DecParams& p, int sm_count, size_t* smem);
int launch_decode_step(const DecParams& p, int grid, size_t smem, cudaStream_t st);

}  // namespace rq
