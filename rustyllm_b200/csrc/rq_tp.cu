// rq_tp.cu -- tensor-parallel communicator of a context: one NCCL
// communicator over NVLink / NVSwitch, one rank per GPU (one process per
// GPU).  Initialisation is non-blocking and bounded by a timeout, so a rank
// that never joins turns into RQ_ERR_TIMEOUT on the others instead of a hang;
// a communicator in error is aborted, never left waiting.
//
// Small all-reduces (the decode loop's two per layer: T x hidden f32, and the
// argmax's one u64) run as a one-shot all-reduce over NVLink peer memory
// instead of NCCL: every rank copies its input into its own exchange buffer
// (CUDA IPC, mapped by every peer), signals each peer with a release store
// into the peer's flag array, waits for the peers' flags (acquire, bounded)
// and sums the W buffers in rank order 0..W-1 -- the same bits on every rank.
// Each CTA owns a slice and its own flags, so no grid-wide barrier is needed;
// a rank reuses a buffer parity only after every peer has signalled the
// following call, which each peer does only after its previous call's kernel
// has finished reading.  RQ_TP_ALLREDUCE=nccl in the environment keeps NCCL.

#include <nccl.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <algorithm>
#include <vector>

#include "rq_async.cuh"
#include "rq_internal.cuh"
#include "rq_p2p.cuh"

namespace rq {

constexpr int kP2PMaxCTA = 32;  // CTAs of the standalone all-reduce kernel

struct TPComm {
    ncclComm_t comm = nullptr;
    int world = 1, rank = 0;
    bool p2p = false;  // one-shot peer-memory all-reduce available
    P2PArgs args{};
};

namespace {

double now_ms() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

int nccl_error(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return RQ_OK;
    return set_error(RQ_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
}

// Wait until a non-blocking NCCL call has been enqueued (or failed),
// bounded by timeout_ms; aborts the communicator on failure or timeout.
int settle(TPComm* c, ncclResult_t r, const char* what, double timeout_ms) {
    if (r != ncclSuccess && r != ncclInProgress) {
        ncclCommAbort(c->comm);
        c->comm = nullptr;
        return nccl_error(r, what);
    }
    const double t0 = now_ms();
    ncclResult_t st = r;
    while (st == ncclInProgress) {
        ncclResult_t q = ncclCommGetAsyncError(c->comm, &st);
        if (q != ncclSuccess) st = q;
        if (st == ncclInProgress && now_ms() - t0 > timeout_ms) {
            ncclCommAbort(c->comm);
            c->comm = nullptr;
            return set_error(RQ_ERR_TIMEOUT, "%s: no progress after %.0f ms (communicator aborted)", what,
                             timeout_ms);
        }
    }
    if (st != ncclSuccess) {
        ncclCommAbort(c->comm);
        c->comm = nullptr;
        return nccl_error(st, what);
    }
    return RQ_OK;
}

constexpr double kOpTimeoutMs = 60000.0;  // enqueue bound for collectives

template <typename T>
__device__ __forceinline__ T reduce_op(T a, T b) {
    return a + b;
}
template <>
__device__ __forceinline__ unsigned long long reduce_op(unsigned long long a, unsigned long long b) {
    return a > b ? a : b;
}

// One-shot all-reduce (sum of f32 / max of u64) of n elements over the
// ranks' exchange regions; grid = the same number of CTAs on every rank.
// Elements move in groups of V (4 floats = 16 bytes, or 1 u64); each thread
// issues the loads of all W ranks for a group before summing, so a group
// costs one NVLink round trip.
template <typename T, int V>
struct Vec {
    T v[V];
};

template <typename T, int V>
__global__ void __launch_bounds__(512) p2p_allreduce_kernel(const T* in, T* out, int64_t n, P2PArgs a) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    using G4 = Vec<T, V>;
    const int c = blockIdx.x, G = gridDim.x;
    uint8_t* own = a.base[a.rank];
    uint32_t* ctl = reinterpret_cast<uint32_t*>(own + kP2PCtlOff);  // epoch, done, err
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(ctl);
    const int par = (int)(e & 1u);
    const int64_t ng = n / V;  // n % V == 0 (checked by the host)
    const int64_t lo = (int64_t)c * ng / G, hi = (int64_t)(c + 1) * ng / G;
    G4* mine = reinterpret_cast<G4*>(own + par * kP2PCap);
    const G4* src = reinterpret_cast<const G4*>(in);
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) mine[i] = src[i];
    __syncthreads();
    const int t = threadIdx.x;
    const size_t fslot = ((size_t)par * kP2PFlagCTAs + (size_t)c) * kP2PMaxWorld;
    if (t < a.world && t != a.rank) {
        // this CTA's slice is in place: tell rank t
        __threadfence_system();
        uint32_t* pf = reinterpret_cast<uint32_t*>(a.base[t] + kP2PFlagsOff) + fslot + a.rank;
        st_release_sys(pf, e + 1u);
    }
    bool ok = true;
    if (t < a.world && t != a.rank) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(own + kP2PFlagsOff) + fslot + t;
        const long long t0 = clock64();
        while ((int)(ld_acquire_sys(f) - (e + 1u)) < 0)
            if (clock64() - t0 > kWaitCycles) {
                ok = false;
                atomicExch(ctl + 2, 1u);
                break;
            }
    }
    ok = __syncthreads_and(ok);
    if (ok) {
        G4* dst = reinterpret_cast<G4*>(out);
        for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            G4 v[kP2PMaxWorld];
#pragma unroll
            for (int r = 0; r < kP2PMaxWorld; r++)
                if (r < a.world) v[r] = reinterpret_cast<const G4*>(a.base[r] + par * kP2PCap)[i];
            G4 acc = v[0];
#pragma unroll
            for (int r = 1; r < kP2PMaxWorld; r++)
                if (r < a.world)
#pragma unroll
                    for (int k = 0; k < V; k++) acc.v[k] = reduce_op(acc.v[k], v[r].v[k]);
            dst[i] = acc;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(ctl + 1, 1u) == (unsigned)(G - 1)) {
            atomicExch(ctl + 1, 0u);
            atomicAdd(ctl, 1u);
        }
    }
}

template <typename T, int V>
int launch_p2p(TPComm* c, const T* in, T* out, int64_t n, cudaStream_t st) {
    // about one group per thread
    const int G = (int)std::min<int64_t>(kP2PMaxCTA, std::max<int64_t>(1, (n / V + 511) / 512));
    p2p_allreduce_kernel<T, V><<<G, 512, 0, st>>>(in, out, n, c->args);
    return cuda_error(cudaGetLastError(), "peer-memory all-reduce kernel");
}

void p2p_teardown(TPComm* c) {
    if (!c->args.base[c->rank]) return;
    for (int r = 0; r < c->world; r++)
        if (r != c->rank && c->args.base[r]) cudaIpcCloseMemHandle(c->args.base[r]);
    cudaFree(c->args.base[c->rank]);
    memset(&c->args, 0, sizeof c->args);
    c->p2p = false;
}

// Maps every rank's exchange region into this process (CUDA IPC handles
// exchanged with an NCCL all-gather); the ranks agree on the outcome.
int p2p_setup(TPComm* c) {
    const char* env = getenv("RQ_TP_ALLREDUCE");
    if (c->world < 2 || c->world > kP2PMaxWorld || (env && strcmp(env, "nccl") == 0)) return RQ_OK;
    c->args.world = c->world;
    c->args.rank = c->rank;
    int ok = 1;
    uint8_t* own = nullptr;
    if (cudaMalloc((void**)&own, kP2PBytes) != cudaSuccess || cudaMemset(own, 0, kP2PBytes) != cudaSuccess) ok = 0;
    c->args.base[c->rank] = own;
    cudaIpcMemHandle_t h;
    memset(&h, 0, sizeof h);
    if (ok && cudaIpcGetMemHandle(&h, own) != cudaSuccess) ok = 0;
    cudaGetLastError();
    // per rank: IPC handle, success flag, device UUID (ranks that share a
    // GPU must not spin on each other: they keep NCCL)
    const size_t hb = sizeof(cudaIpcMemHandle_t), rec = hb + 8 + 16;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceProp prop;
    memset(&prop, 0, sizeof prop);
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) ok = 0;
    uint8_t* dsend = nullptr;
    uint8_t* drecv = nullptr;
    int rc = cuda_error(cudaMalloc((void**)&dsend, rec), "cudaMalloc");
    if (!rc) rc = cuda_error(cudaMalloc((void**)&drecv, rec * (size_t)c->world), "cudaMalloc");
    std::vector<uint8_t> hsend(rec, 0), hrecv(rec * (size_t)c->world, 0);
    memcpy(hsend.data(), &h, hb);
    hsend[hb] = (uint8_t)ok;
    memcpy(hsend.data() + hb + 8, &prop.uuid, 16);
    if (!rc) rc = cuda_error(cudaMemcpy(dsend, hsend.data(), rec, cudaMemcpyHostToDevice), "handle copy");
    if (!rc) rc = settle(c, ncclAllGather(dsend, drecv, rec, ncclInt8, c->comm, 0), "ncclAllGather", kOpTimeoutMs);
    if (!rc) rc = cuda_error(cudaDeviceSynchronize(), "handle exchange");
    if (!rc) rc = cuda_error(cudaMemcpy(hrecv.data(), drecv, hrecv.size(), cudaMemcpyDeviceToHost), "handle copy");
    if (dsend) cudaFree(dsend);
    if (drecv) cudaFree(drecv);
    if (rc) {
        p2p_teardown(c);
        return rc;
    }
    for (int r = 0; r < c->world; r++) {
        ok &= hrecv[(size_t)r * rec + hb];
        for (int q = 0; q < r; q++)
            if (memcmp(hrecv.data() + (size_t)r * rec + hb + 8, hrecv.data() + (size_t)q * rec + hb + 8, 16) == 0)
                ok = 0;
    }
    for (int r = 0; r < c->world && ok; r++) {
        if (r == c->rank) continue;
        cudaIpcMemHandle_t hr;
        memcpy(&hr, hrecv.data() + (size_t)r * rec, hb);
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = 0;
        }
        c->args.base[r] = (uint8_t*)p;
    }
    // every rank must take the same path
    std::vector<uint8_t> flag(8, (uint8_t)ok), oks(8 * (size_t)c->world, 0);
    uint8_t* df = nullptr;
    rc = cuda_error(cudaMalloc((void**)&df, 8 * (size_t)(c->world + 1)), "cudaMalloc");
    if (!rc) rc = cuda_error(cudaMemcpy(df, flag.data(), 8, cudaMemcpyHostToDevice), "flag copy");
    if (!rc) rc = settle(c, ncclAllGather(df, df + 8, 8, ncclInt8, c->comm, 0), "ncclAllGather", kOpTimeoutMs);
    if (!rc) rc = cuda_error(cudaDeviceSynchronize(), "flag exchange");
    if (!rc) rc = cuda_error(cudaMemcpy(oks.data(), df + 8, oks.size(), cudaMemcpyDeviceToHost), "flag copy");
    if (df) cudaFree(df);
    for (int r = 0; r < c->world && !rc; r++) ok &= oks[(size_t)r * 8];
    if (rc || !ok) {
        p2p_teardown(c);
        return rc;
    }
    c->p2p = true;
    return RQ_OK;
}

}  // namespace

int tp_world(const rq_ctx* ctx) { return ctx->tp ? ctx->tp->world : 1; }
int tp_rank(const rq_ctx* ctx) { return ctx->tp ? ctx->tp->rank : 0; }

bool tp_fused_enabled(int world) {
    static const int mode = [] {
        const char* e = getenv("RQ_TP_FUSED");
        if (e && strcmp(e, "0") == 0) return 0;
        if (e && strcmp(e, "1") == 0) return 1;
        return 2;  // default
    }();
    return mode != 0 && (mode == 1 || world >= 2);
}

bool tp_p2p_args(const rq_ctx* ctx, P2PArgs* a) {
    const TPComm* c = ctx->tp;
    if (!c || !c->comm || !c->p2p) return false;
    *a = c->args;
    return true;
}

int tp_allreduce(rq_ctx* ctx, const void* in, void* out, int64_t n, int dtype, int op, cudaStream_t st) {
    TPComm* c = ctx->tp;
    if (!c || !c->comm) return set_error(RQ_ERR_INVALID, "tensor-parallel communicator not initialised");
    if (c->p2p && n > 0 && (size_t)n * 8 <= kP2PCap) {
        const bool a16 = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
        if (dtype == 0 && op == 0 && n % 4 == 0 && a16)
            return launch_p2p<float, 4>(c, (const float*)in, (float*)out, n, st);
        if (dtype == 0 && op == 0) return launch_p2p<float, 1>(c, (const float*)in, (float*)out, n, st);
        if (dtype == 1 && op == 1)
            return launch_p2p<unsigned long long, 1>(c, (const unsigned long long*)in, (unsigned long long*)out,
                                                     n, st);
    }
    const ncclDataType_t dt = dtype == 0 ? ncclFloat32 : ncclUint64;
    const ncclRedOp_t ro = op == 0 ? ncclSum : ncclMax;
    return settle(c, ncclAllReduce(in, out, (size_t)n, dt, ro, c->comm, st), "ncclAllReduce", kOpTimeoutMs);
}

int tp_allgather_bytes(rq_ctx* ctx, const void* in, void* out, int64_t nbytes, cudaStream_t st) {
    TPComm* c = ctx->tp;
    if (!c || !c->comm) return set_error(RQ_ERR_INVALID, "tensor-parallel communicator not initialised");
    return settle(c, ncclAllGather(in, out, (size_t)nbytes, ncclInt8, c->comm, st), "ncclAllGather", kOpTimeoutMs);
}

int tp_alltoallv_bytes(rq_ctx* ctx, const void* send, const int64_t* send_bytes, const int64_t* send_off, void* recv,
                       const int64_t* recv_bytes, const int64_t* recv_off, cudaStream_t st) {
    TPComm* c = ctx->tp;
    if (!c || !c->comm) return set_error(RQ_ERR_INVALID, "tensor-parallel communicator not initialised");
    // this rank's own share is a device copy
    if (send_bytes[c->rank] != recv_bytes[c->rank])
        return set_error(RQ_ERR_INVALID, "all-to-all: self send %lld != self receive %lld bytes",
                         (long long)send_bytes[c->rank], (long long)recv_bytes[c->rank]);
    if (send_bytes[c->rank] > 0) {
        int rc = cuda_error(cudaMemcpyAsync((uint8_t*)recv + recv_off[c->rank], (const uint8_t*)send + send_off[c->rank],
                                            (size_t)send_bytes[c->rank], cudaMemcpyDeviceToDevice, st),
                            "all-to-all self copy");
        if (rc) return rc;
    }
    ncclResult_t r = ncclGroupStart();
    for (int peer = 0; peer < c->world && (r == ncclSuccess || r == ncclInProgress); peer++) {
        if (peer == c->rank) continue;
        if (send_bytes[peer] > 0)
            r = ncclSend((const uint8_t*)send + send_off[peer], (size_t)send_bytes[peer], ncclInt8, peer, c->comm, st);
        if ((r == ncclSuccess || r == ncclInProgress) && recv_bytes[peer] > 0)
            r = ncclRecv((uint8_t*)recv + recv_off[peer], (size_t)recv_bytes[peer], ncclInt8, peer, c->comm, st);
    }
    const ncclResult_t r2 = ncclGroupEnd();
    if (r == ncclSuccess || r == ncclInProgress) r = r2;
    return settle(c, r, "all-to-all (ncclSend/ncclRecv)", kOpTimeoutMs);
}

void tp_destroy(rq_ctx* ctx) {
    if (!ctx->tp) return;
    cudaDeviceSynchronize();
    if (ctx->tp->p2p && ctx->tp->comm) {
        // no rank unmaps its region while a peer's last all-reduce may
        // still read it: every rank passes this collective after draining
        float* d = nullptr;
        if (cudaMalloc((void**)&d, 4) == cudaSuccess) {
            if (settle(ctx->tp, ncclAllReduce(d, d, 1, ncclFloat32, ncclSum, ctx->tp->comm, 0), "finalize barrier",
                       kOpTimeoutMs) == RQ_OK)
                cudaDeviceSynchronize();
            cudaFree(d);
        }
    }
    p2p_teardown(ctx->tp);
    if (ctx->tp->comm) {
        ncclResult_t st = ncclSuccess;
        ncclCommGetAsyncError(ctx->tp->comm, &st);
        if (st == ncclSuccess) ncclCommDestroy(ctx->tp->comm);
        else ncclCommAbort(ctx->tp->comm);
    }
    delete ctx->tp;
    ctx->tp = nullptr;
}

}  // namespace rq

using namespace rq;

extern "C" {

int rq_tp_unique_id(void* id_out, size_t n) {
    if (!id_out || n < sizeof(ncclUniqueId))
        return set_error(RQ_ERR_INVALID, "rq_tp_unique_id: buffer must hold %zu bytes", sizeof(ncclUniqueId));
    ncclUniqueId id;
    int rc = nccl_error(ncclGetUniqueId(&id), "ncclGetUniqueId");
    if (!rc) memcpy(id_out, &id, sizeof id);
    return rc;
}

int rq_tp_init(rq_ctx* ctx, int world, int rank, const void* id, int timeout_ms) {
    if (!ctx || !id) return set_error(RQ_ERR_INVALID, "rq_tp_init: NULL argument");
    if (world < 1 || rank < 0 || rank >= world)
        return set_error(RQ_ERR_INVALID, "rq_tp_init: rank %d of %d", rank, world);
    if (ctx->tp) return set_error(RQ_ERR_INVALID, "rq_tp_init: communicator already initialised");
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != ctx->device) cudaSetDevice(ctx->device);
    TPComm* c = new TPComm();
    c->world = world;
    c->rank = rank;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&c->comm, world, uid, rank, &cfg);
    int rc = settle(c, r, "ncclCommInitRankConfig", timeout_ms > 0 ? timeout_ms : 60000.0);
    if (!rc) rc = p2p_setup(c);
    if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
    if (rc) {
        if (c->comm) ncclCommAbort(c->comm);
        delete c;
        return rc;
    }
    ctx->tp = c;
    return RQ_OK;
}

int rq_tp_allreduce_f32(rq_ctx* ctx, const float* in, float* out, int64_t n, void* stream) {
    if (!ctx || !in || !out) return set_error(RQ_ERR_INVALID, "rq_tp_allreduce_f32: NULL argument");
    return tp_allreduce(ctx, in, out, n, 0, 0, (cudaStream_t)stream);
}

int rq_tp_status(rq_ctx* ctx) {
    if (!ctx || !ctx->tp || !ctx->tp->comm) return set_error(RQ_ERR_INVALID, "rq_tp_status: no communicator");
    if (ctx->tp->p2p) {
        uint32_t err = 0;
        int rc = cuda_error(cudaMemcpy(&err, ctx->tp->args.base[ctx->tp->rank] + kP2PCtlOff + 8, 4,
                                       cudaMemcpyDeviceToHost), "peer all-reduce status");
        if (rc) return rc;
        if (err) return set_error(RQ_ERR_TIMEOUT, "peer-memory all-reduce: a peer did not signal within ~1 s");
    }
    ncclResult_t st = ncclSuccess;
    ncclResult_t q = ncclCommGetAsyncError(ctx->tp->comm, &st);
    if (q != ncclSuccess) return nccl_error(q, "ncclCommGetAsyncError");
    if (st != ncclSuccess && st != ncclInProgress) return nccl_error(st, "communicator");
    return RQ_OK;
}

int rq_tp_finalize(rq_ctx* ctx) {
    if (!ctx) return set_error(RQ_ERR_INVALID, "rq_tp_finalize: NULL argument");
    tp_destroy(ctx);
    return RQ_OK;
}

}  // extern "C"
