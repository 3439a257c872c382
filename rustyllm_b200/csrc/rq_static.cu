// rq_static.cu -- rq_linear_noalloc: the quantized linear of rq_linear for
// callers that cannot allocate device memory.
//
// rq_linear stages the activations (three int8 planes plus per-block stats,
// 3.5 bytes per element) in a workspace that librq grows with cudaMalloc on
// demand.  Some callers cannot allow that: a serving engine that reserves
// nearly all HBM up front for its own pools (a cudaMalloc would fail or
// fragment its reservation), a host framework whose allocator owns every
// device buffer (candle's CUDA device in rustyllm), or a latency-critical
// decode loop where cudaMalloc/cudaFree may synchronise the device.  This
// entry point stages the activations the same way in a file-scope static
// __device__ array instead and runs the M=1 matvec kernels on every row
// (rq_linear moves to the tensor-core kernels from M = 4 on), and allocates
// nothing.
//
// The array is kStaticScratchBytes (2 MiB) on every GPU that loads librq,
// held until the process exits.

#include <mutex>

#include "rq_internal.cuh"

namespace rq {
namespace {

constexpr size_t kStaticScratchBytes = (size_t)2 << 20;

// Activation staging for rq_linear_noalloc.  Host code must not pass
// `g_static_scratch` itself to a kernel: on the host that name is only a
// stand-in; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
// The error word of rq_linear_noalloc's kernels (a bounded wait that gave up
// sets it); rq_ctx_status on a context of the same device reads and clears it.
// Resolved like the scratch array.
static __device__ int g_static_err;

constexpr int kMaxDevices = 64;

struct StaticDeviceState {
    bool ready = false;
    void* scratch = nullptr;  // device address of g_static_scratch on this device
    int* err = nullptr;       // device address of g_static_err on this device
    int sm_count = 0;
};

StaticDeviceState g_states[kMaxDevices];
std::mutex g_states_mu;

// Once per device, with that device current: resolve the scratch array's
// device address and the SM count.
int static_setup(int dev, StaticDeviceState** out) {
    if (dev < 0 || dev >= kMaxDevices)
        return set_error(RQ_ERR_INVALID, "rq_linear_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_states_mu);
    StaticDeviceState& s = g_states[dev];
    if (!s.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) return cuda_error(e, "rq_linear_noalloc: cudaGetSymbolAddress(scratch)");
        void* pe = nullptr;
        e = cudaGetSymbolAddress(&pe, g_static_err);
        if (e != cudaSuccess) return cuda_error(e, "rq_linear_noalloc: cudaGetSymbolAddress(error word)");
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_error(e, "rq_linear_noalloc: cudaDeviceGetAttribute");
        s.scratch = p;
        s.err = (int*)pe;
        s.sm_count = sms;
        s.ready = true;
    }
    *out = &s;
    return RQ_OK;
}

bool on_device(const void* p, int dev) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) && a.device == dev;
}

}  // namespace

// rq_ctx_status's view of the error word of device dev (the device is current):
// 1 = set since the last look (now cleared), 0 = not set or never used.
int static_error_take(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return -RQ_ERR_INVALID;
    StaticDeviceState* s = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_states_mu);
        if (!g_states[dev].ready) return 0;
        s = &g_states[dev];
    }
    int v = 0;
    if (cuda_error(cudaMemcpy(&v, s->err, sizeof(int), cudaMemcpyDeviceToHost), "noalloc error word copy"))
        return -RQ_ERR_CUDA;
    if (v && cuda_error(cudaMemset(s->err, 0, sizeof(int)), "noalloc error word reset")) return -RQ_ERR_CUDA;
    return v ? 1 : 0;
}

}  // namespace rq

using namespace rq;

extern "C" int rq_linear_noalloc(const rq_weight* w, const float* x, float* y, int64_t M,
                                 void* stream) {
    if (!w || !x || !y) return set_error(RQ_ERR_INVALID, "rq_linear_noalloc: NULL argument");
    if (M < 0) return set_error(RQ_ERR_INVALID, "rq_linear_noalloc: M = %lld", (long long)M);
    if (M == 0) return RQ_OK;
    const size_t need = xq_bytes(M, w->in);
    if (need > kStaticScratchBytes)
        return set_error(RQ_ERR_INVALID,
                         "rq_linear_noalloc: M=%lld x in=%lld needs %zu bytes of activation "
                         "staging; the static scratch holds %zu (3.5 bytes per element)",
                         (long long)M, (long long)w->in, need, kStaticScratchBytes);
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return set_error(RQ_ERR_CUDA, "cudaGetDevice failed");
    if (prev != w->device && cudaSetDevice(w->device) != cudaSuccess)
        return set_error(RQ_ERR_CUDA, "cudaSetDevice(%d) failed", w->device);
    int rc = RQ_OK;
    if (!on_device(x, w->device) || !on_device(y, w->device)) {
        rc = set_error(RQ_ERR_INVALID,
                       "rq_linear_noalloc: x and y must be device memory on device %d", w->device);
    }
    StaticDeviceState* s = nullptr;
    if (!rc) rc = static_setup(w->device, &s);
    if (!rc) {
        // xquant_kernel writes every plane byte and stats entry of the
        // M x in region before the matvec reads it, so nothing left over
        // from an earlier call is ever read and nothing needs clearing.
        uint8_t* base = (uint8_t*)s->scratch;
        XQ xq;
        xq.planes = (int8_t*)base;
        xq.stats = (float4*)(base + (((size_t)M * 3 * w->in + 255) & ~(size_t)255));
        cudaStream_t st = (cudaStream_t)stream;
        rc = launch_xquant(x, M, w->in, xq, st);
        if (!rc) rc = launch_linear(w, xq, y, M, s->sm_count, st, s->err);
    }
    if (prev >= 0 && prev != w->device) cudaSetDevice(prev);
    return rc;
}
