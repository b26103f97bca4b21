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
#include <cstdlib>
#include <thread>
#include <vector>

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

// ----------------------------------------------------------------------------
// Fixpoint flags over peer memory.  Each rank allocates a slot array
// (kMaxPeers ranks x 2 sweep parities x 8 bytes), exports it with a CUDA IPC
// handle and maps every other rank's array, so the one-launch fixpoint can
// store its changed word straight into every peer's memory over NVLink.  The
// handles travel in one all-gather.  If any rank cannot take part (ranks
// sharing a GPU, more ranks than kMaxPeers, a handle that does not open),
// a second collective makes every rank fall back to the per-sweep all-reduce,
// so all ranks take the same path.
// ----------------------------------------------------------------------------
namespace {
struct PeerRecord {
    cudaIpcMemHandle_t handle;
    unsigned char uuid[16];
    int32_t ok;
    int32_t pad[3];
};
// a rank's slot array: words [2j, 2j + 1] for rank j's changed words (by sweep
// parity), then at 2 * kMaxPeers the count of sweeps this context exchanged
constexpr size_t kSlotBytes = 4096;
}  // namespace

void comm_peer_release(tl_ctx* c) {
    for (int j = 0; j < kMaxPeers; ++j) {
        if (c->peer_slots[j] && j != c->rank) cudaIpcCloseMemHandle(c->peer_slots[j]);
        c->peer_slots[j] = nullptr;
    }
    if (c->peer_own) cudaFree(c->peer_own);
    c->peer_own = nullptr;
    cudaGetLastError();
}

tl_status comm_peer_setup(tl_ctx* c) {
    if (c->peer_state != 0) return TL_OK;
    c->peer_state = -1;
    if (!c->comm) return fail(c, TL_ERR_COMM, "no communicator");
    const int world = c->world;
    PeerRecord mine{};
    mine.ok = world <= kMaxPeers && !getenv("TL_NO_PEER_FLAGS");
    if (mine.ok && cudaMalloc(&c->peer_own, kSlotBytes) != cudaSuccess) mine.ok = 0;
    if (mine.ok && cudaMemsetAsync(c->peer_own, 0, kSlotBytes, c->stream) != cudaSuccess) mine.ok = 0;
    if (mine.ok && cudaIpcGetMemHandle(&mine.handle, c->peer_own) != cudaSuccess) mine.ok = 0;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, c->device) == cudaSuccess) memcpy(mine.uuid, prop.uuid.bytes, 16);
    else mine.ok = 0;
    cudaGetLastError();

    std::vector<PeerRecord> all(world);
    PeerRecord* d = nullptr;
    TL_CK(c, cudaMalloc(&d, sizeof(PeerRecord) * (world + 1)));
    tl_status st = TL_OK;
    do {
        if (cudaMemcpyAsync(d + world, &mine, sizeof mine, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
            st = fail(c, TL_ERR_CUDA, "peer flag set-up: copy");
            break;
        }
        ncclResult_t r = ncclAllGather(d + world, d, sizeof(PeerRecord), ncclChar, (ncclComm_t)c->comm, c->stream);
        if (r != ncclSuccess) {
            st = nccl_fail(c, r, "ncclAllGather");
            break;
        }
        if ((st = comm_wait(c)) != TL_OK) break;
        if (cudaMemcpy(all.data(), d, sizeof(PeerRecord) * world, cudaMemcpyDeviceToHost) != cudaSuccess) {
            st = fail(c, TL_ERR_CUDA, "peer flag set-up: copy back");
            break;
        }
        int ok = 1;
        for (int j = 0; j < world; ++j) {
            ok = ok && all[j].ok;
            for (int i = 0; i < j; ++i) ok = ok && memcmp(all[i].uuid, all[j].uuid, 16) != 0;
        }
        for (int j = 0; ok && j < world; ++j) {
            if (j == c->rank) {
                c->peer_slots[j] = (unsigned long long*)c->peer_own;
                continue;
            }
            void* p = nullptr;
            if (cudaIpcOpenMemHandle(&p, all[j].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = 0;
                break;
            }
            c->peer_slots[j] = (unsigned long long*)p;
        }
        // every rank takes the peer path only if every rank can
        int* flag = reinterpret_cast<int*>(d + world);
        const int bad = ok ? 0 : 1;
        if (cudaMemcpyAsync(flag, &bad, sizeof bad, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
            st = fail(c, TL_ERR_CUDA, "peer flag set-up: copy");
            break;
        }
        if ((st = comm_allreduce_max_int(c, flag, 1)) != TL_OK) break;
        int any_bad = 1;
        if (cudaMemcpy(&any_bad, flag, sizeof any_bad, cudaMemcpyDeviceToHost) != cudaSuccess) {
            st = fail(c, TL_ERR_CUDA, "peer flag set-up: copy back");
            break;
        }
        c->peer_state = any_bad ? -1 : 1;
    } while (false);
    cudaFree(d);
    if (c->peer_state != 1) comm_peer_release(c);
    return st;
}

// ----------------------------------------------------------------------------
// The symmetric buffer of the sharded closure: every rank allocates `bytes`,
// zeroes it and exports it; the handles travel in one all-gather (which also
// orders every rank's zeroing before any peer can read), and every rank maps
// every other rank's buffer.  As with the flag slots, a second collective
// makes every rank agree on whether all of them could.  A larger size later
// unmaps the old buffers everywhere (a barrier between the unmapping and the
// frees) and sets up again.
// ----------------------------------------------------------------------------
tl_status comm_barrier(tl_ctx* c) {
    int* w = c->d_flags + 48;
    TL_CK(c, cudaMemsetAsync(w, 0, sizeof(int), c->stream));
    return comm_allreduce_max_int(c, w, 1);
}

void comm_sym_release(tl_ctx* c, int slot) {
    SymBuf& b = c->sym[slot];
    for (int j = 0; j < kMaxPeers; ++j) {
        if (b.peer[j] && j != c->rank) cudaIpcCloseMemHandle(b.peer[j]);
        b.peer[j] = nullptr;
    }
    if (b.own) cudaFree(b.own);
    b.own = nullptr;
    b.bytes = 0;
    cudaGetLastError();
}

tl_status comm_sym_setup(tl_ctx* c, int slot, size_t bytes) {
    SymBuf& b = c->sym[slot];
    if (b.state == -1 || (b.state == 1 && b.bytes >= bytes)) return TL_OK;
    if (!c->comm) return fail(c, TL_ERR_COMM, "no communicator");
    if (b.state == 1) {
        // every rank grows at the same call: unmap the peers' buffers, wait
        // until every rank has, then free this rank's
        for (int j = 0; j < kMaxPeers; ++j) {
            if (b.peer[j] && j != c->rank) cudaIpcCloseMemHandle(b.peer[j]);
            b.peer[j] = nullptr;
        }
        TL_TRY(comm_barrier(c));
        comm_sym_release(c, slot);
    }
    b.state = -1;
    const int world = c->world;
    PeerRecord mine{};
    mine.ok = world <= kMaxPeers && !getenv("TL_NO_PEER_ROWS");
    if (mine.ok && cudaMalloc(&b.own, bytes) != cudaSuccess) mine.ok = 0;
    if (mine.ok && cudaMemsetAsync(b.own, 0, bytes, c->stream) != cudaSuccess) mine.ok = 0;
    if (mine.ok && cudaIpcGetMemHandle(&mine.handle, b.own) != cudaSuccess) mine.ok = 0;
    cudaGetLastError();
    std::vector<PeerRecord> all(world);
    PeerRecord* d = nullptr;
    TL_CK(c, cudaMalloc(&d, sizeof(PeerRecord) * (world + 1)));
    tl_status st = TL_OK;
    int state = -1;
    do {
        if (cudaMemcpyAsync(d + world, &mine, sizeof mine, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
            st = fail(c, TL_ERR_CUDA, "peer buffer set-up: copy");
            break;
        }
        ncclResult_t r = ncclAllGather(d + world, d, sizeof(PeerRecord), ncclChar, (ncclComm_t)c->comm, c->stream);
        if (r != ncclSuccess) {
            st = nccl_fail(c, r, "ncclAllGather");
            break;
        }
        if ((st = comm_wait(c)) != TL_OK) break;
        if (cudaMemcpy(all.data(), d, sizeof(PeerRecord) * world, cudaMemcpyDeviceToHost) != cudaSuccess) {
            st = fail(c, TL_ERR_CUDA, "peer buffer set-up: copy back");
            break;
        }
        int ok = 1;
        for (int j = 0; j < world; ++j) ok = ok && all[j].ok;
        for (int j = 0; ok && j < world; ++j) {
            if (j == c->rank) {
                b.peer[j] = b.own;
                continue;
            }
            void* p = nullptr;
            if (cudaIpcOpenMemHandle(&p, all[j].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = 0;
                break;
            }
            b.peer[j] = p;
        }
        int* flag = reinterpret_cast<int*>(d + world);
        const int bad = ok ? 0 : 1;
        if (cudaMemcpyAsync(flag, &bad, sizeof bad, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
            st = fail(c, TL_ERR_CUDA, "peer buffer set-up: copy");
            break;
        }
        if ((st = comm_allreduce_max_int(c, flag, 1)) != TL_OK) break;
        int any_bad = 1;
        if (cudaMemcpy(&any_bad, flag, sizeof any_bad, cudaMemcpyDeviceToHost) != cudaSuccess) {
            st = fail(c, TL_ERR_CUDA, "peer buffer set-up: copy back");
            break;
        }
        state = any_bad ? -1 : 1;
    } while (false);
    cudaFree(d);
    if (state == 1) {
        b.bytes = bytes;
        if (slot == SYM_CLOSURE) c->sym_epoch = 0;
    } else {
        comm_sym_release(c, slot);
    }
    b.state = state;
    return st;
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
