// NCCL communicator of a row-sharded context: one process per GPU.
//
// Two collectives only: the all-reduce (MAX) of the fixpoint's 4-byte
// changed word once per sweep (fixpoint.zig:76-95 keeps this flag per
// sweep), and the all-gather of the per-node transform rows before message
// passing.  Tiles of other ranks reach a GPU only through these collectives
// into its own memory.  Host waits on a collective are bounded: a collective
// that does not finish within comm_timeout_ms aborts the communicator and
// returns TL_ERR_COMM instead of blocking forever.
#include <nccl.h>
#include <string.h>

#include <chrono>
#include <thread>

#include "tl_internal.h"

namespace tl {

static tl_status nccl_fail(tl_ctx* c, ncclResult_t r, const char* what) {
    return fail(c, TL_ERR_COMM, "%s: %s", what, ncclGetErrorString(r));
}

tl_status comm_init(tl_ctx* c) {
    ncclUniqueId id;
    static_assert(sizeof(id.internal) <= sizeof(c->opts.nccl_id), "ncclUniqueId size");
    memcpy(id.internal, c->opts.nccl_id, sizeof(id.internal));
    ncclComm_t comm = nullptr;
    ncclResult_t r = ncclCommInitRank(&comm, c->world, id, c->rank);
    if (r != ncclSuccess) return nccl_fail(c, r, "ncclCommInitRank");
    c->comm = comm;
    return TL_OK;
}

tl_status comm_destroy(tl_ctx* c) {
    if (!c->comm) return TL_OK;
    ncclCommDestroy((ncclComm_t)c->comm);
    c->comm = nullptr;
    return TL_OK;
}

// Wait for the stream with a bound, watching the communicator for errors.
static tl_status comm_wait(tl_ctx* c) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaStreamQuery(c->stream);
        if (e == cudaSuccess) return TL_OK;
        if (e != cudaErrorNotReady) return cuda_fail(c, e, "collective");
        ncclResult_t async = ncclSuccess;
        ncclCommGetAsyncError((ncclComm_t)c->comm, &async);
        if (async != ncclSuccess) {
            ncclCommAbort((ncclComm_t)c->comm);
            c->comm = nullptr;
            return nccl_fail(c, async, "collective");
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (ms > c->opts.comm_timeout_ms) {
            ncclCommAbort((ncclComm_t)c->comm);
            c->comm = nullptr;
            return fail(c, TL_ERR_COMM, "collective did not finish within %d ms", c->opts.comm_timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

tl_status comm_allreduce_max_int(tl_ctx* c, int* d_buf, int count) {
    if (!c->comm) return fail(c, TL_ERR_COMM, "no communicator");
    ncclResult_t r = ncclAllReduce(d_buf, d_buf, count, ncclInt32, ncclMax, (ncclComm_t)c->comm, c->stream);
    if (r != ncclSuccess) return nccl_fail(c, r, "ncclAllReduce");
    return comm_wait(c);
}

tl_status comm_allgather(tl_ctx* c, const void* d_send, void* d_recv, size_t bytes_per_rank) {
    if (!c->comm) return fail(c, TL_ERR_COMM, "no communicator");
    ncclResult_t r = ncclAllGather(d_send, d_recv, bytes_per_rank, ncclChar, (ncclComm_t)c->comm, c->stream);
    if (r != ncclSuccess) return nccl_fail(c, r, "ncclAllGather");
    return TL_OK;
}

}  // namespace tl

extern "C" tl_status tl_comm_unique_id(uint8_t id_out[128]) {
    if (!id_out) return TL_ERR_INVALID;
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return TL_ERR_COMM;
    memset(id_out, 0, 128);
    memcpy(id_out, id.internal, sizeof(id.internal));
    return TL_OK;
}
