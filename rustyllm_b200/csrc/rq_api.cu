// rq_api.cu -- the extern "C" boundary of librq (declared in include/rq.h):
// contexts, error reporting, weight upload / download, dispatch.

#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>

#include "rq_internal.cuh"
#include "rq_p2p.cuh"

namespace rq {

static thread_local char g_err[1024] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return RQ_OK;
    return set_error(e == cudaErrorMemoryAllocation ? RQ_ERR_OOM : RQ_ERR_CUDA, "%s: %s (%s)", what,
                     cudaGetErrorString(e), cudaGetErrorName(e));
}

namespace {

// Makes ctx->device current for the duration of a call and restores the
// caller's device afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = (prev == dev) || cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

enum class Mem { Host, Device };

Mem mem_kind(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // clear the sticky-free error of an unknown pointer
        return Mem::Host;
    }
    return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) ? Mem::Device
                                                                                : Mem::Host;
}

// The address a kernel on this device can use for p: p itself in device
// memory, the mapped address of page-locked host memory (kernels then read
// and write it over the bus), or NULL for pageable host memory.
// *host tells whether p is host memory (page-locked or not).
void* device_alias(const void* p, bool* host) {
    cudaPointerAttributes a;
    *host = true;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
        *host = false;
        return const_cast<void*>(p);
    }
    if (a.type == cudaMemoryTypeHost && a.devicePointer) return a.devicePointer;
    return nullptr;
}

bool valid_type(int t) {
    return t == RQ_Q4_0 || t == RQ_Q4_K || t == RQ_Q3_K || t == RQ_Q8_0 || t == RQ_Q6_K || t == RQ_Q5_K ||
           t == RQ_Q2_K;
}

const char* type_name(int t) {
    switch (t) {
    case RQ_Q4_0: return "Q4_0";
    case RQ_Q4_K: return "Q4_K";
    case RQ_Q3_K: return "Q3_K";
    case RQ_Q8_0: return "Q8_0";
    case RQ_Q6_K: return "Q6_K";
    case RQ_Q5_K: return "Q5_K";
    case RQ_Q2_K: return "Q2_K";
    default: return "?";
    }
}

int check_shape(int type, int64_t out, int64_t in) {
    if (!valid_type(type))
        return set_error(RQ_ERR_UNSUPPORTED, "unsupported ggml type %d (Q4_0=2, Q8_0=8, Q2_K=10, Q3_K=11, Q4_K=12, Q5_K=13, Q6_K=14)",
                         type);
    TypeInfo ti = type_info(type);
    if (out <= 0 || in <= 0)
        return set_error(RQ_ERR_INVALID, "weight shape [%lld, %lld] must be positive", (long long)out,
                         (long long)in);
    if (in % ti.block_elems)
        return set_error(RQ_ERR_INVALID, "in_features %lld not divisible by %d (%s)", (long long)in,
                         ti.block_elems, type_name(type));
    return RQ_OK;
}

// A weight that views rows [r0, r0+n) of w.
rq_weight row_view(const rq_weight* w, int64_t r0, int64_t n) {
    TypeInfo ti = type_info(w->type);
    rq_weight v = *w;
    v.out = n;
    v.qs = w->qs + r0 * w->nblk * ti.qs_bytes;
    v.hdr = w->hdr + r0 * w->nblk * ti.hdr_bytes;
    return v;
}

int alloc_weight(rq_ctx* ctx, int type, int64_t out, int64_t in, rq_weight** res) {
    TypeInfo ti = type_info(type);
    rq_weight* w = new (std::nothrow) rq_weight();
    if (!w) return set_error(RQ_ERR_OOM, "host allocation failed");
    w->type = type;
    w->out = out;
    w->in = in;
    w->nblk = in / ti.block_elems;
    w->device = ctx->device;
    size_t qsz = (size_t)out * w->nblk * ti.qs_bytes;
    size_t hsz = (size_t)out * w->nblk * ti.hdr_bytes;
    size_t qpad = (qsz + 255) & ~(size_t)255;
    w->bytes = qpad + hsz;
    cudaError_t e = cudaMalloc(&w->base, w->bytes);
    if (e != cudaSuccess) {
        delete w;
        return cuda_error(e, "cudaMalloc(weight)");
    }
    w->qs = (uint8_t*)w->base;
    w->hdr = (uint8_t*)w->base + qpad;
    if (type == RQ_Q3_K || type == RQ_Q6_K) {  // pad bytes of the headers stay zero
        e = cudaMemset(w->hdr, 0, hsz);
        if (e != cudaSuccess) {
            cudaFree(w->base);
            delete w;
            return cuda_error(e, "cudaMemset(weight)");
        }
    }
    *res = w;
    return RQ_OK;
}

constexpr size_t kStageBytes = 64u << 20;  // host<->device staging chunk

}  // namespace

int ensure_workspace(rq_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->ws_bytes) return RQ_OK;
    if (ctx->ws) {
        cudaError_t e = cudaFree(ctx->ws);  // implicit device sync: no kernel still uses it
        ctx->ws = nullptr;
        ctx->ws_bytes = 0;
        if (e != cudaSuccess) return cuda_error(e, "cudaFree(workspace)");
    }
    size_t sz = std::max(bytes, (size_t)4 << 20);
    cudaError_t e = cudaMalloc(&ctx->ws, sz);
    if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(workspace)");
    ctx->ws_bytes = sz;
    return RQ_OK;
}

int ensure_skinny_scratch(rq_ctx* ctx, size_t floats, int tiles) {
    if (floats <= ctx->sk_ws_floats && tiles <= ctx->sk_cnt_n) return RQ_OK;
    // first use (or a larger launch): one allocation, outside any graph
    // capture (cudaMalloc fails inside one and the error is reported)
    if (floats > ctx->sk_ws_floats) {
        if (ctx->sk_ws) cudaFree(ctx->sk_ws);  // implicit device sync: no kernel still uses it
        ctx->sk_ws = nullptr;
        ctx->sk_ws_floats = 0;
        const size_t nf = std::max(floats, (size_t)4 << 20);
        cudaError_t e = cudaMalloc(&ctx->sk_ws, nf * sizeof(float));
        if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(skinny matmul pieces)");
        ctx->sk_ws_floats = nf;
    }
    if (tiles > ctx->sk_cnt_n) {
        if (ctx->sk_cnt) cudaFree(ctx->sk_cnt);
        ctx->sk_cnt = nullptr;
        ctx->sk_cnt_n = 0;
        const int n = std::max(tiles, 16384);
        cudaError_t e = cudaMalloc(&ctx->sk_cnt, (size_t)n * sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(ctx->sk_cnt, 0, (size_t)n * sizeof(int));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_error(e, "skinny matmul counters");
        ctx->sk_cnt_n = n;
    }
    return RQ_OK;
}

// Bytes of activation staging at the start of ctx->ws for rq_linear's
// kernel choice at M rows.
// Q4_0 from M = 5: launches of two to four rows on the int8 kernels over
// one staging (a weight pass per launch instead of per row)
bool q40_row_groups(const rq_weight* w, int64_t M) {
    return M > 8 && w->type == RQ_Q4_0 && mm_i8_supported(w, 8);
}

size_t small_m_staging_bytes(const rq_weight* w, int64_t M) {
    if (mm_i8_supported(w, M)) return xq2_bytes(M, w->in) + 256 + mm_i8_scratch_floats(w, M) * sizeof(float);
    if (q40_row_groups(w, M)) return xq2_bytes(M, w->in) + 256 + mm_i8_scratch_floats(w, 8) * sizeof(float);
    const bool small_m = (M >= kMinTensorM && mm_small_supported(w)) || q3k_tensor_m(w, M);
    return small_m ? xh_bytes(M, w->in) : xq_bytes(M, w->in);
}

// y = x W^T for device-resident x, y (M rows): stages x at the start of
// ctx->ws (small_m_staging_bytes) and runs the kernel rq_linear routes M to.
// M >= 24: tcgen05 tiles of 128 weight rows x up to 112 tokens; M = 9..16:
// the split-K tcgen05 kernel, one pass over the weights; M = 4..8 and
// 17..23: one mma.sync pass per 8 rows; M = 2..4 (Q4_K, in <= 8192): the
// int8 tensor-core kernel, one pass; the other M = 2, 3 shapes: the M=1
// pipeline once per row is faster (it streams at ~5 TB/s).  M = 2..8 of
// Q4_K, Q3_K and Q4_0 run the int8 kernels first; Q3_K from M = 9 the
// tcgen05 kernel; Q4_0 above eight rows one int8 launch per group of 5..8
// rows.
int linear_device(rq_ctx* ctx, const rq_weight* w, const float* xd, float* yd, int64_t M, cudaStream_t st) {
    uint8_t* ws = (uint8_t*)ctx->ws;
    int rc;
    if (q3k_tensor_m(w, M)) {
        const XH xh = xh_at(ws, M, w->in);
        rc = launch_xh_stage(xd, M, w->in, xh, st);
        const MMJobDesc job{w, 0, (int)M, yd, nullptr};
        if (!rc) rc = launch_mm_tc(&job, 1, xh, M, ctx->sm_count, st, ctx->derr);
        return rc;
    }
    if (mm_i8_supported(w, M)) {  // M = 2..4: one pass on the int8 tensor cores
        const XQ2 q = xq2_at(ws, M, w->in);
        float* part = (float*)(ws + ((xq2_bytes(M, w->in) + 255) & ~(size_t)255));
        rc = launch_xq2_stage(xd, M, w->in, q, st);
        if (!rc) rc = launch_mm_i8(&w, &yd, 1, M, q, ctx->sm_count, st, ctx->derr, nullptr, part, ctx->i8_cnt);
        return rc;
    }
    if (q40_row_groups(w, M)) {  // ceil(M / 8) groups of 5..8 rows, sizes as even as possible
        const XQ2 q = xq2_at(ws, M, w->in);
        float* part = (float*)(ws + ((xq2_bytes(M, w->in) + 255) & ~(size_t)255));
        rc = launch_xq2_stage(xd, M, w->in, q, st);
        const int64_t n = (M + 7) / 8, nsb = w->in / 256;
        for (int64_t g = 0, m0 = 0; g < n && !rc; g++) {
            const int64_t rows = M / n + (g < M % n ? 1 : 0);
            XQ2 qg = q;
            qg.planes += m0 * 3 * w->in;
            qg.sx += m0 * nsb;
            qg.bsum += m0 * (w->in / 32);
            float* yg = yd + m0 * w->out;
            rc = launch_mm_i8(&w, &yg, 1, rows, qg, ctx->sm_count, st, ctx->derr, nullptr, part, ctx->i8_cnt);
            m0 += rows;
        }
        return rc;
    }
    if (M >= kMinTensorM && mm_small_supported(w)) {
        const XH xh = xh_at(ws, M, w->in);
        rc = launch_xh_stage(xd, M, w->in, xh, st);
        if (!rc && M >= kMinTcgenM && mm_tc_supported(w)) {
            const MMJobDesc job{w, 0, (int)M, yd, nullptr};
            rc = launch_mm_tc(&job, 1, xh, M, ctx->sm_count, st, ctx->derr);
        } else if (!rc && M >= kSkinnyMinM && M <= kSkinnyMaxM) {
            const MMJobDesc job{w, 0, (int)M, yd, nullptr};
            rc = launch_mm_skinny(ctx, &job, 1, xh, M, st, ctx->derr);
        } else if (!rc) {
            rc = launch_matmul_small(w, xh, M, yd, nullptr, ctx->sm_count, st, ctx->derr);
        }
        return rc;
    }
    XQ xq;
    xq.planes = (int8_t*)ws;
    xq.stats = (float4*)(ws + (((size_t)M * 3 * w->in + 255) & ~(size_t)255));
    rc = launch_xquant(xd, M, w->in, xq, st);
    const PipeNext nx = take_hint(ctx);
    if (!rc) rc = launch_linear(w, xq, yd, M, ctx->sm_count, st, ctx->derr, &nx);
    return rc;
}

// bytes per CTA of the hinted weights' first rows (the decode loop's budget)
constexpr uint32_t kHintBudget = 128 * 1024;

PipeNext take_hint(rq_ctx* ctx) {
    const PipeNext nx = pipe_next(ctx->hint_w, ctx->hint_n, kHintBudget);
    ctx->hint_n = 0;
    return nx;
}

int queue_error_readback(rq_ctx* ctx, cudaStream_t st) {
    return cuda_error(cudaMemcpyAsync(ctx->err_host, ctx->derr, sizeof(int), cudaMemcpyDeviceToHost, st),
                      "error word copy");
}

int take_kernel_error(rq_ctx* ctx, cudaStream_t st, const char* what) {
    if (*(volatile int*)ctx->err_host == 0) return RQ_OK;
    *(volatile int*)ctx->err_host = 0;
    int rc = cuda_error(cudaMemsetAsync(ctx->derr, 0, sizeof(int), st), "error word reset");
    if (!rc) rc = cuda_error(cudaStreamSynchronize(st), "error word reset");
    if (rc) return rc;
    return set_error(RQ_ERR_TIMEOUT, "%s: a kernel's bounded wait gave up after ~1 s (its outputs are incomplete)",
                     what);
}

}  // namespace rq

using namespace rq;

extern "C" {

int rq_last_error(char* buf, size_t n) {
    size_t len = strlen(g_err);
    if (buf && n) {
        size_t c = std::min(len, n - 1);
        memcpy(buf, g_err, c);
        buf[c] = 0;
    }
    return (int)len;
}

const char* rq_version(void) { return "rq 0.1.0 sm_100a"; }

size_t rq_block_bytes(int t) { return valid_type(t) ? (size_t)type_info(t).block_bytes : 0; }
int rq_block_elems(int t) { return valid_type(t) ? type_info(t).block_elems : 0; }

int rq_init(int device, rq_ctx** out) {
    if (!out) return set_error(RQ_ERR_INVALID, "rq_init: out is NULL");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDeviceCount");
    if (device < 0 || device >= n)
        return set_error(RQ_ERR_INVALID, "device %d out of range (%d CUDA devices)", device, n);
    DeviceGuard g(device);
    if (!g.ok) return set_error(RQ_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDeviceProperties");
    if (prop.major != 10)
        return set_error(RQ_ERR_UNSUPPORTED, "device %d is sm_%d%d; librq is built for sm_100a only",
                         device, prop.major, prop.minor);
    rq_ctx* c = new (std::nothrow) rq_ctx();
    if (!c) return set_error(RQ_ERR_OOM, "host allocation failed");
    c->tp = nullptr;
    c->device = device;
    c->own_stream = nullptr;
    c->ws = nullptr;
    c->ws_bytes = 0;
    c->sm_count = prop.multiProcessorCount;
    e = cudaMalloc(&c->derr, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->derr, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&c->i8_cnt, 256 * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->i8_cnt, 0, 256 * sizeof(int));
    if (e == cudaSuccess) e = cudaHostAlloc(&c->err_host, sizeof(int), cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (c->derr) cudaFree(c->derr);
        if (c->i8_cnt) cudaFree(c->i8_cnt);
        delete c;
        return cuda_error(e, "rq_init: error word");
    }
    *c->err_host = 0;
    *out = c;
    return RQ_OK;
}

int rq_ctx_status(rq_ctx* ctx) {
    if (!ctx) return set_error(RQ_ERR_INVALID, "rq_ctx_status: NULL context");
    DeviceGuard g(ctx->device);
    int rc = cuda_error(cudaDeviceSynchronize(), "rq_ctx_status sync");
    if (!rc) rc = cuda_error(cudaMemcpy(ctx->err_host, ctx->derr, sizeof(int), cudaMemcpyDeviceToHost),
                             "error word copy");
    if (!rc) rc = take_kernel_error(ctx, nullptr, "rq_ctx_status");
    if (rc) return rc;
    const int s = static_error_take(ctx->device);
    if (s < 0) return s == -RQ_ERR_INVALID ? RQ_ERR_INVALID : RQ_ERR_CUDA;
    if (s > 0)
        return set_error(RQ_ERR_TIMEOUT,
                         "rq_ctx_status: a bounded wait inside an rq_linear_noalloc kernel on device %d gave up "
                         "after ~1 s (that call's y is incomplete)", ctx->device);
    return RQ_OK;
}

int rq_destroy(rq_ctx* ctx) {
    if (!ctx) return RQ_OK;
    DeviceGuard g(ctx->device);
    tp_destroy(ctx);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->sk_ws) cudaFree(ctx->sk_ws);
    if (ctx->sk_cnt) cudaFree(ctx->sk_cnt);
    if (ctx->derr) cudaFree(ctx->derr);
    if (ctx->i8_cnt) cudaFree(ctx->i8_cnt);
    if (ctx->err_host) cudaFreeHost(ctx->err_host);
    delete ctx;
    return RQ_OK;
}

int rq_weight_upload(rq_ctx* ctx, int type, const void* blocks, size_t nbytes, int64_t out,
                     int64_t in, rq_weight** res) {
    if (!ctx || !blocks || !res) return set_error(RQ_ERR_INVALID, "rq_weight_upload: NULL argument");
    *res = nullptr;
    int rc = check_shape(type, out, in);
    if (rc) return rc;
    TypeInfo ti = type_info(type);
    const int64_t row_bytes = in / ti.block_elems * ti.block_bytes;
    if ((int64_t)nbytes != out * row_bytes)
        return set_error(RQ_ERR_INVALID, "rq_weight_upload: %zu bytes given, %s [%lld, %lld] needs %lld",
                         nbytes, type_name(type), (long long)out, (long long)in,
                         (long long)(out * row_bytes));
    DeviceGuard g(ctx->device);
    rq_weight* w = nullptr;
    rc = alloc_weight(ctx, type, out, in, &w);
    if (rc) return rc;
    const uint8_t* src = (const uint8_t*)blocks;
    if (mem_kind(blocks) == Mem::Device) {
        rc = launch_repack(w, src, 0, out, 0);
        if (!rc) rc = cuda_error(cudaDeviceSynchronize(), "repack");
    } else {
        int64_t rows_per = std::max<int64_t>(1, (int64_t)kStageBytes / row_bytes);
        rows_per = std::min(rows_per, out);
        uint8_t* stage = nullptr;
        rc = cuda_error(cudaMalloc(&stage, (size_t)(rows_per * row_bytes)), "cudaMalloc(stage)");
        for (int64_t r0 = 0; !rc && r0 < out; r0 += rows_per) {
            int64_t n = std::min(rows_per, out - r0);
            rc = cuda_error(cudaMemcpy(stage, src + r0 * row_bytes, (size_t)(n * row_bytes),
                                       cudaMemcpyHostToDevice), "upload copy");
            if (!rc) {
                rq_weight v = row_view(w, r0, n);
                rc = launch_repack(&v, stage, 0, n, 0);
            }
            if (!rc) rc = cuda_error(cudaDeviceSynchronize(), "repack");
        }
        if (stage) cudaFree(stage);
    }
    if (rc) {
        cudaFree(w->base);
        delete w;
        return rc;
    }
    *res = w;
    return RQ_OK;
}

int rq_weight_quantize(rq_ctx* ctx, int type, const float* w_dev, int64_t out, int64_t in,
                       rq_weight** res, void* stream) {
    if (!ctx || !w_dev || !res) return set_error(RQ_ERR_INVALID, "rq_weight_quantize: NULL argument");
    *res = nullptr;
    int rc = check_shape(type, out, in);
    if (rc) return rc;
    if (mem_kind(w_dev) != Mem::Device)
        return set_error(RQ_ERR_INVALID, "rq_weight_quantize: w must be device memory");
    if ((reinterpret_cast<uintptr_t>(w_dev) & 15) != 0)
        return set_error(RQ_ERR_INVALID, "rq_weight_quantize: w must be 16-byte aligned");
    DeviceGuard g(ctx->device);
    rq_weight* w = nullptr;
    rc = alloc_weight(ctx, type, out, in, &w);
    if (rc) return rc;
    rc = launch_quantize(w, w_dev, (cudaStream_t)stream);
    // the weight is complete when the call returns (linear kernels start
    // streaming weights before they wait for the preceding kernel)
    if (!rc) rc = cuda_error(cudaStreamSynchronize((cudaStream_t)stream), "rq_weight_quantize sync");
    if (rc) {
        cudaFree(w->base);
        delete w;
        return rc;
    }
    *res = w;
    return RQ_OK;
}

int rq_weight_download(rq_ctx* ctx, const rq_weight* w, void* blocks_host, size_t nbytes) {
    if (!ctx || !w || !blocks_host) return set_error(RQ_ERR_INVALID, "rq_weight_download: NULL argument");
    TypeInfo ti = type_info(w->type);
    const int64_t row_bytes = w->nblk * ti.block_bytes;
    if ((int64_t)nbytes != w->out * row_bytes)
        return set_error(RQ_ERR_INVALID, "rq_weight_download: buffer is %zu bytes, weight has %lld",
                         nbytes, (long long)(w->out * row_bytes));
    DeviceGuard g(ctx->device);
    int64_t rows_per = std::min<int64_t>(w->out, std::max<int64_t>(1, (int64_t)kStageBytes / row_bytes));
    uint8_t* stage = nullptr;
    int rc = cuda_error(cudaMalloc(&stage, (size_t)(rows_per * row_bytes)), "cudaMalloc(stage)");
    for (int64_t r0 = 0; !rc && r0 < w->out; r0 += rows_per) {
        int64_t n = std::min(rows_per, w->out - r0);
        rq_weight v = row_view(w, r0, n);
        rc = launch_unpack(&v, stage, 0, n, 0);
        if (!rc)
            rc = cuda_error(cudaMemcpy((uint8_t*)blocks_host + r0 * row_bytes, stage,
                                       (size_t)(n * row_bytes), cudaMemcpyDeviceToHost),
                            "download copy");
    }
    if (stage) cudaFree(stage);
    return rc;
}

int rq_weight_free(rq_ctx* ctx, rq_weight* w) {
    if (!w) return RQ_OK;
    DeviceGuard g(ctx ? ctx->device : w->device);
    cudaError_t e = cudaFree(w->base);
    delete w;
    return cuda_error(e, "cudaFree(weight)");
}

int rq_weight_info(const rq_weight* w, int* type, int64_t* out, int64_t* in, size_t* device_bytes) {
    if (!w) return set_error(RQ_ERR_INVALID, "rq_weight_info: NULL weight");
    TypeInfo ti = type_info(w->type);
    if (type) *type = w->type;
    if (out) *out = w->out;
    if (in) *in = w->in;
    if (device_bytes) *device_bytes = (size_t)(w->out * w->nblk * (ti.qs_bytes + ti.hdr_bytes));
    return RQ_OK;
}

int rq_dequantize(rq_ctx* ctx, const rq_weight* w, float* y, void* stream) {
    if (!ctx || !w || !y) return set_error(RQ_ERR_INVALID, "rq_dequantize: NULL argument");
    DeviceGuard g(ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    if (mem_kind(y) == Mem::Device) {
        if ((reinterpret_cast<uintptr_t>(y) & 15) != 0)
            return set_error(RQ_ERR_INVALID, "rq_dequantize: device y must be 16-byte aligned");
        return launch_dequant(w, y, st);
    }
    const int64_t row_f = w->in * (int64_t)sizeof(float);
    int64_t rows_per = std::min<int64_t>(w->out, std::max<int64_t>(1, (int64_t)kStageBytes / row_f));
    int rc = ensure_workspace(ctx, (size_t)(rows_per * row_f));
    for (int64_t r0 = 0; !rc && r0 < w->out; r0 += rows_per) {
        int64_t n = std::min(rows_per, w->out - r0);
        rq_weight v = row_view(w, r0, n);
        rc = launch_dequant(&v, (float*)ctx->ws, st);
        if (!rc)
            rc = cuda_error(cudaMemcpyAsync(y + r0 * w->in, ctx->ws, (size_t)(n * row_f),
                                            cudaMemcpyDeviceToHost, st), "dequant copy");
        if (!rc) rc = cuda_error(cudaStreamSynchronize(st), "dequant sync");
    }
    return rc;
}

int rq_linear(rq_ctx* ctx, const rq_weight* w, const float* x, float* y, int64_t M, void* stream) {
    if (!ctx || !w || !x || !y) return set_error(RQ_ERR_INVALID, "rq_linear: NULL argument");
    if (M < 0) return set_error(RQ_ERR_INVALID, "rq_linear: M = %lld", (long long)M);
    if (M == 0) return RQ_OK;
    DeviceGuard g(ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    // device or page-locked host buffers are used in place (the kernels read
    // x and write y over the bus for the latter); pageable host buffers go
    // through the workspace with copies
    bool x_host = true, y_host = true;
    float* const x_alias = static_cast<float*>(device_alias(x, &x_host));
    float* const y_alias = static_cast<float*>(device_alias(y, &y_host));
    const bool x_dev = x_alias != nullptr, y_dev = y_alias != nullptr;
    const size_t xq_sz = small_m_staging_bytes(w, M);
    const size_t x_sz = x_dev ? 0 : (size_t)(M * w->in) * sizeof(float);
    const size_t y_sz = y_dev ? 0 : (size_t)(M * w->out) * sizeof(float);
    int rc = ensure_workspace(ctx, xq_sz + x_sz + y_sz + 512);
    if (rc) return rc;
    uint8_t* ws = (uint8_t*)ctx->ws;
    float* xd = x_dev ? x_alias : (float*)(ws + ((xq_sz + 255) & ~(size_t)255));
    float* yd = y_dev ? y_alias : (float*)((uint8_t*)xd + (x_dev ? 0 : ((x_sz + 255) & ~(size_t)255)));
    if (!y_dev && x_dev) yd = (float*)(ws + ((xq_sz + 255) & ~(size_t)255));
    if (!x_dev) {
        rc = cuda_error(cudaMemcpyAsync(xd, x, x_sz, cudaMemcpyHostToDevice, st), "x copy");
        if (rc) return rc;
    }
    rc = linear_device(ctx, w, xd, yd, M, st);
    if (rc) return rc;
    if (!y_dev) rc = cuda_error(cudaMemcpyAsync(y, yd, y_sz, cudaMemcpyDeviceToHost, st), "y copy");
    // host buffers: y is complete and x no longer read when the call returns,
    // and a kernel wait that gave up is reported here (device-only calls are
    // asynchronous: rq_ctx_status reports it)
    if (!rc && (x_host || y_host)) {
        rc = queue_error_readback(ctx, st);
        if (!rc) rc = cuda_error(cudaStreamSynchronize(st), "rq_linear sync");
        if (!rc) rc = take_kernel_error(ctx, st, "rq_linear");
    }
    return rc;
}

/* Row-parallel linear under tensor parallelism (no reference counterpart:
 * the reference runs on one device): y = sum over ranks of x_r W_r^T. */
int rq_linear_allreduce(rq_ctx* ctx, const rq_weight* w, const float* x, float* y, int64_t M, void* stream) {
    if (!ctx || !w || !x || !y) return set_error(RQ_ERR_INVALID, "rq_linear_allreduce: NULL argument");
    if (M < 0) return set_error(RQ_ERR_INVALID, "rq_linear_allreduce: M = %lld", (long long)M);
    if (!ctx->tp) return set_error(RQ_ERR_INVALID, "rq_linear_allreduce: no communicator (rq_tp_init)");
    if (M == 0) return RQ_OK;
    if (mem_kind(x) != Mem::Device || mem_kind(y) != Mem::Device)
        return set_error(RQ_ERR_INVALID, "rq_linear_allreduce: x and y must be device memory");
    DeviceGuard g(ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    P2PArgs ar;
    if (M == 1 && pipe_supported(w) && tp_fused_enabled(tp_world(ctx)) && tp_p2p_args(ctx, &ar)) {
        int rc = ensure_workspace(ctx, xq_bytes(1, w->in));
        if (rc) return rc;
        XQ xq;
        xq.planes = (int8_t*)ctx->ws;
        xq.stats = (float4*)((uint8_t*)ctx->ws + (((size_t)3 * w->in + 255) & ~(size_t)255));
        rc = launch_xquant(x, 1, w->in, xq, st);
        if (rc) return rc;
        const float* add = nullptr;
        const PipeNext nx = take_hint(ctx);
        rc = launch_matvec_pipe(&w, &xq, &y, 1, ctx->sm_count, st, ctx->derr, &add, &ar, nullptr, nullptr, nullptr,
                                &nx);
        if (rc != kPipeNotFusable) return rc;
    }
    // the partial product into the workspace's tail, then the all-reduce
    const size_t stage = small_m_staging_bytes(w, M);
    const size_t part_off = (stage + 255) & ~(size_t)255;
    int rc = ensure_workspace(ctx, part_off + (size_t)(M * w->out) * sizeof(float));
    if (rc) return rc;
    float* part = (float*)((uint8_t*)ctx->ws + part_off);
    rc = linear_device(ctx, w, x, part, M, st);
    if (!rc) rc = tp_allreduce(ctx, part, y, M * w->out, 0, 0, st);
    return rc;
}

int rq_linear_batch(rq_ctx* ctx, int n, const rq_weight* const* w, const float* const* x,
                    float* const* y, void* stream) {
    if (!ctx || !w || !x || !y) return set_error(RQ_ERR_INVALID, "rq_linear_batch: NULL argument");
    if (n < 1 || n > kMaxJobs)
        return set_error(RQ_ERR_INVALID, "rq_linear_batch: n = %d (1..%d)", n, kMaxJobs);
    for (int j = 0; j < n; j++) {
        if (!w[j] || !x[j] || !y[j]) return set_error(RQ_ERR_INVALID, "rq_linear_batch: NULL entry %d", j);
        if (w[j]->type != w[0]->type || w[j]->in != w[0]->in || w[j]->device != w[0]->device)
            return set_error(RQ_ERR_INVALID,
                             "rq_linear_batch: weight %d differs from weight 0 in type, in_features or device", j);
        if (mem_kind(x[j]) != Mem::Device || mem_kind(y[j]) != Mem::Device)
            return set_error(RQ_ERR_INVALID, "rq_linear_batch: x and y must be device memory");
    }
    DeviceGuard g(ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    if (!pipe_supported(w[0])) {  // shapes the pipeline does not take: one call each
        for (int j = 0; j < n; j++) {
            int rc = rq_linear(ctx, w[j], x[j], y[j], 1, stream);
            if (rc) return rc;
        }
        return RQ_OK;
    }
    // stage each distinct activation row once
    const float* rows[kMaxJobs];
    int row_of[kMaxJobs], nrows = 0;
    for (int j = 0; j < n; j++) {
        int r = 0;
        while (r < nrows && rows[r] != x[j]) r++;
        if (r == nrows) rows[nrows++] = x[j];
        row_of[j] = r;
    }
    const int64_t in = w[0]->in;
    int rc = ensure_workspace(ctx, xq_bytes(nrows, in));
    if (rc) return rc;
    XQ xq;
    xq.planes = (int8_t*)ctx->ws;
    xq.stats = (float4*)((uint8_t*)ctx->ws + (((size_t)nrows * 3 * in + 255) & ~(size_t)255));
    rc = launch_xquant_rows(rows, nrows, in, xq, st);
    if (rc) return rc;
    XQ xqs[kMaxJobs];
    for (int j = 0; j < n; j++)
        xqs[j] = XQ{xq.planes + (int64_t)row_of[j] * 3 * in, xq.stats + (int64_t)row_of[j] * (in / 32)};
    const PipeNext nx = take_hint(ctx);
    return launch_matvec_pipe(w, xqs, y, n, ctx->sm_count, st, ctx->derr, nullptr, nullptr, nullptr, nullptr, nullptr,
                              &nx);
}

/* A hint, no reference counterpart: the next M=1 pipeline launch of
 * rq_linear / rq_linear_batch / rq_linear_allreduce on this context
 * prefetches into L2, after its last weight copy, the first rows of these
 * n (<= 3) weights -- what the caller will multiply next (the decode loop
 * does the same between its own launches).  n = 0 clears it.  No effect on
 * results. */
int rq_linear_prefetch_hint(rq_ctx* ctx, int n, const rq_weight* const* w) {
    if (!ctx || n < 0 || n > 3 || (n > 0 && !w)) return set_error(RQ_ERR_INVALID, "rq_linear_prefetch_hint: bad argument");
    for (int i = 0; i < n; i++)
        if (!w[i]) return set_error(RQ_ERR_INVALID, "rq_linear_prefetch_hint: NULL weight %d", i);
    for (int i = 0; i < n; i++) ctx->hint_w[i] = w[i];
    ctx->hint_n = n;
    return RQ_OK;
}

}  // extern "C"
