// tl_closure_noalloc: the closure fixpoint on caller-owned device memory,
// with its scratch in a fixed array inside the library instead of cudaMalloc.
//
// Who needs it: a caller whose GPU memory is owned by its own pool or arena
// (a serving process with a fixed budget, a framework's caching allocator
// that must see every byte in use), which may not call cudaMalloc behind the
// pool's back.  Such a caller cannot create a tl_ctx (tl_init allocates), so
// this path takes no context at all.
//
// The call is synchronous: after every sweep it copies the changed word to
// the host and waits for the stream, so it returns with the result final.
// `stream` must belong to the current device (checked): the scratch address
// is the current device's.
//
// The scratch: one int32 "pending" word per row (the lowest 32-bit word of
// the row that may hold a bit not yet expanded) and the sweep's control
// words (changed flag, row counter), for at most TL_NOALLOC_MAX_ROWS rows.
// Every GPU that loads the library holds the array until the process exits.
// Host code cannot use the array's name as a device address; its address is
// looked up once per device with cudaGetSymbolAddress, with that device
// current, on the first call there; that first call should come before any
// stream capture.
#include <mutex>

#include "tl_internal.h"

namespace tl {
cudaError_t launch_closure_right_raw(uint32_t* R, int64_t rows, int64_t words, const int64_t* rowptr,
                                     const int32_t* colidx, int64_t e_rows, int* changed,
                                     unsigned long long* counter, int32_t* pending, int sweep,
                                     cudaStream_t stream);
}

namespace {

constexpr size_t kControlBytes = 256;   // changed word at 0, row counter at 64
constexpr size_t kScratchBytes = kControlBytes + (size_t)TL_NOALLOC_MAX_ROWS * sizeof(int32_t);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_lock;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (set-up once).
cudaError_t scratch_for_current_device(unsigned char** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> hold(g_lock);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
    return cudaSuccess;
}

}  // namespace

extern "C" tl_status tl_closure_noalloc(int64_t n, const int64_t* d_rowptr, const int32_t* d_colidx,
                                        uint32_t* d_reach, int32_t max_sweeps, void* stream,
                                        int32_t* sweeps_out) {
    if (sweeps_out) *sweeps_out = 0;
    if (n < 0) return TL_ERR_INVALID;
    if (n > TL_NOALLOC_MAX_ROWS) return TL_ERR_TOO_LARGE;   // before any device call
    if (n == 0) return TL_OK;
    if (!d_rowptr || !d_colidx || !d_reach) return TL_ERR_INVALID;
    if (max_sweeps <= 0) max_sweeps = 1000;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (s) {
        // the scratch address below is the current device's: a stream of
        // another device would hand a kernel there a foreign address
        int cur = 0, sdev = 0;
        if (cudaGetDevice(&cur) != cudaSuccess || cudaStreamGetDevice(s, &sdev) != cudaSuccess) return TL_ERR_CUDA;
        if (sdev != cur) return TL_ERR_INVALID;
    }
    unsigned char* scratch = nullptr;
    if (scratch_for_current_device(&scratch) != cudaSuccess) return TL_ERR_CUDA;
    int* changed = reinterpret_cast<int*>(scratch);
    unsigned long long* counter = reinterpret_cast<unsigned long long*>(scratch + 64);
    int32_t* pending = reinterpret_cast<int32_t*>(scratch + kControlBytes);
    const int64_t words = (n + 31) / 32;

    // every row starts with all of its bits unexpanded
    if (cudaMemsetAsync(pending, 0, (size_t)n * sizeof(int32_t), s) != cudaSuccess) return TL_ERR_CUDA;
    int sweeps = 0;
    int host_changed = 1;
    while (sweeps < max_sweeps && host_changed) {
        if (cudaMemsetAsync(scratch, 0, kControlBytes, s) != cudaSuccess) return TL_ERR_CUDA;
        if (tl::launch_closure_right_raw(d_reach, n, words, d_rowptr, d_colidx, n, changed, counter, pending, sweeps,
                                         s) != cudaSuccess)
            return TL_ERR_CUDA;
        // the changed word into a host stack variable (no pinned buffer needed)
        if (cudaMemcpyAsync(&host_changed, changed, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)
            return TL_ERR_CUDA;
        if (cudaStreamSynchronize(s) != cudaSuccess) return TL_ERR_CUDA;
        sweeps++;
    }
    if (sweeps_out) *sweeps_out = sweeps;
    return TL_OK;
}
