// rq_tp.cu -- tensor-parallel communicator of a context: one NCCL
// communicator over NVLink / NVSwitch, one rank per GPU (one process per
// GPU).  Initialisation is non-blocking and bounded by a timeout, so a rank
// that never joins turns into RQ_ERR_TIMEOUT on the others instead of a hang;
// a communicator in error is aborted, never left waiting.

#include <nccl.h>
#include <string.h>
#include <time.h>

#include "rq_internal.cuh"

namespace rq {

struct TPComm {
    ncclComm_t comm = nullptr;
    int world = 1, rank = 0;
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

}  // namespace

int tp_world(const rq_ctx* ctx) { return ctx->tp ? ctx->tp->world : 1; }
int tp_rank(const rq_ctx* ctx) { return ctx->tp ? ctx->tp->rank : 0; }

int tp_allreduce(rq_ctx* ctx, const void* in, void* out, int64_t n, int dtype, int op, cudaStream_t st) {
    TPComm* c = ctx->tp;
    if (!c || !c->comm) return set_error(RQ_ERR_INVALID, "tensor-parallel communicator not initialised");
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
    if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
    if (rc) {
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
