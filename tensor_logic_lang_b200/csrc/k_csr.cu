// CSR of a `sparse` tensor built on the GPU from its COO entries.
//
// The entries arrive in any order, may repeat a (row, column) pair (the last
// one counts) and, on a row-sharded context, cover every rank's rows.  The
// device build is a counting sort by row followed by one thread per row that
// sorts the row's entries by (column, input position) and keeps the last
// entry of each column: the same CSR (row pointers, ascending columns,
// values) as the host build in runtime.cpp, for rows of up to kCsrRowMax
// entries.  A longer row sends the whole upload back to the host build.
#include <stdio.h>

#include <algorithm>

#include "tl_internal.h"

namespace tl {
namespace {

constexpr int kCsrRowMax = 32;
constexpr int kScanThreads = 1024;

// stats[0]: an entry lies outside the tensor; stats[1]: longest local row;
// stats[2]: 1 while every value is >= 0, [3] > 0, [4] == 1
__global__ void k_coo_count(const int64_t* __restrict__ rows, const int64_t* __restrict__ cols, int64_t nnz,
                            int64_t n_rows, int64_t n_cols, int world, int rank, int* __restrict__ cnt,
                            int* __restrict__ stats) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nnz; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = rows[e], col = cols[e];
        if (r < 0 || r >= n_rows || col < 0 || col >= n_cols) {
            atomicOr(&stats[0], 1);
            continue;
        }
        if (world > 1 && r % world != rank) continue;
        atomicAdd(&cnt[world > 1 ? r / world : r], 1);
    }
}

// out[i] = sum of cnt[0 .. i) for i <= n (out[n] = the total), by one block,
// tile by tile: each thread loads 4 consecutive counts (one 16-byte load per
// lane, a warp reads 512 contiguous bytes), a warp scan and a scan of the 32
// warp totals give every thread its exclusive prefix, and a running carry
// links the tiles.  Also the largest count into *max_out (when given).
__global__ void __launch_bounds__(kScanThreads) k_scan_counts(const int* __restrict__ cnt, int64_t n,
                                                              int64_t* __restrict__ out, int* __restrict__ max_out) {
    static_assert(kScanThreads == 1024, "one warp scans the 32 warp totals");
    __shared__ int64_t wsum[32];
    __shared__ int wmax[32];
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    constexpr int PER = 4;
    int64_t carry = 0;
    int m = 0;
    for (int64_t base = 0; base < n; base += (int64_t)kScanThreads * PER) {
        const int64_t i0 = base + (int64_t)t * PER;
        int v[PER] = {0, 0, 0, 0};
        if (i0 + PER <= n && ((reinterpret_cast<uintptr_t>(cnt + i0) & 15) == 0)) {
            const int4 q = *reinterpret_cast<const int4*>(cnt + i0);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
#pragma unroll
            for (int k = 0; k < PER; ++k) v[k] = i0 + k < n ? cnt[i0 + k] : 0;
        }
        const int64_t s = (int64_t)v[0] + v[1] + v[2] + v[3];
        m = max(m, max(max(v[0], v[1]), max(v[2], v[3])));
        int64_t x = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[w] = x;
        __syncthreads();
        if (w == 0) {
            int64_t y = wsum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t z = __shfl_up_sync(0xffffffffu, y, o);
                if (lane >= o) y += z;
            }
            wsum[lane] = y;
        }
        __syncthreads();
        int64_t run = carry + (w > 0 ? wsum[w - 1] : 0) + (x - s);
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            if (i0 + k < n) out[i0 + k] = run;
            run += v[k];
        }
        carry += wsum[31];
        __syncthreads();   // wsum is rewritten by the next tile
    }
    if (t == 0) out[n] = carry;
    if (max_out) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) wmax[w] = m;
        __syncthreads();
        if (w == 0) {
            int v = wmax[lane];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0) *max_out = v;
        }
    }
}

// Entry e goes to its row's next free slot as the key (column << 32 | e).
__global__ void k_coo_scatter(const int64_t* __restrict__ rows, const int64_t* __restrict__ cols, int64_t nnz,
                              int world, int rank, const int64_t* __restrict__ start, int* __restrict__ fill,
                              unsigned long long* __restrict__ keys) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nnz; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = rows[e];
        if (world > 1 && r % world != rank) continue;
        const int64_t lr = world > 1 ? r / world : r;
        const int64_t at = start[lr] + atomicAdd(&fill[lr], 1);
        keys[at] = ((unsigned long long)cols[e] << 32) | (unsigned long long)(uint32_t)e;
    }
}

// One thread per row: sort the row's keys (column, then input position) and
// keep the last key of each column, compacted at the row's start; kept[r] =
// how many.
__global__ void k_row_dedupe(const int64_t* __restrict__ start, int64_t n_rows, unsigned long long* __restrict__ keys,
                             int* __restrict__ kept) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n_rows; r += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = start[r];
        const int len = (int)(start[r + 1] - b);
        unsigned long long k[kCsrRowMax];
        for (int i = 0; i < len && i < kCsrRowMax; ++i) k[i] = keys[b + i];
        for (int i = 1; i < len && i < kCsrRowMax; ++i) {
            const unsigned long long x = k[i];
            int j = i - 1;
            while (j >= 0 && k[j] > x) {
                k[j + 1] = k[j];
                --j;
            }
            k[j + 1] = x;
        }
        int n = 0;
        for (int i = 0; i < len && i < kCsrRowMax; ++i)
            if (i + 1 == len || (k[i + 1] >> 32) != (k[i] >> 32)) keys[b + n++] = k[i];
        kept[r] = n;
    }
}

// The CSR's columns and values from the kept keys; clears stats[2..4] for a
// value that breaks them.
__global__ void k_csr_fill(const int64_t* __restrict__ start, const int64_t* __restrict__ rowptr, int64_t n_rows,
                           const unsigned long long* __restrict__ keys, const double* __restrict__ vals,
                           int32_t* __restrict__ colidx, float* __restrict__ out_vals, int* __restrict__ stats) {
    bool nonneg = true, pos = true, ones = true;
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n_rows; r += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = start[r], o = rowptr[r], n = rowptr[r + 1] - o;
        for (int64_t j = 0; j < n; ++j) {
            const unsigned long long k = keys[b + j];
            const float v = vals ? (float)vals[(uint32_t)k] : 1.0f;
            colidx[o + j] = (int32_t)(k >> 32);
            out_vals[o + j] = v;
            nonneg = nonneg && v >= 0.0f;
            pos = pos && v > 0.0f;
            ones = ones && v == 1.0f;
        }
    }
    if (!__all_sync(0xffffffffu, nonneg) && (threadIdx.x & 31) == 0) atomicAnd(&stats[2], 0);
    if (!__all_sync(0xffffffffu, pos) && (threadIdx.x & 31) == 0) atomicAnd(&stats[3], 0);
    if (!__all_sync(0xffffffffu, ones) && (threadIdx.x & 31) == 0) atomicAnd(&stats[4], 0);
}

}  // namespace

// Builds t's CSR on the device from nnz COO entries in host (or device)
// memory.  *handled = false (nothing changed) when the device build does not
// apply: few entries, sizes past its 32-bit keys, or a local row longer than
// kCsrRowMax entries; the caller then builds on the host.  An entry outside
// the tensor fails with TL_ERR_INVALID.  Two small read-backs synchronise the
// stream (the row check, then the value flags).
tl_status csr_from_coo_gpu(tl_ctx* c, Tensor* t, int64_t nnz, const int64_t* rows, const int64_t* cols,
                           const double* vals, int64_t lrows, bool* handled) {
    *handled = false;
    if (nnz < 1024 || nnz >= (int64_t(1) << 32) || t->dims[1] >= (int64_t(1) << 31) || lrows < 1) return TL_OK;
    const int world = (t->shard == TL_SHARD_ROWS && c->world > 1) ? c->world : 1;
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    const size_t b_coo = al((size_t)nnz * 8), b_rows = al((size_t)lrows * 4), b_start = al((size_t)(lrows + 1) * 8);
    const size_t need = 3 * b_coo + (vals ? b_coo : 0) + 3 * b_rows + b_start + 256;
    void* ws = nullptr;
    TL_TRY(workspace(c, need, &ws, WS_GENERAL));
    char* p = static_cast<char*>(ws);
    int64_t* d_rows = reinterpret_cast<int64_t*>(p); p += b_coo;
    int64_t* d_cols = reinterpret_cast<int64_t*>(p); p += b_coo;
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(p); p += b_coo;
    double* d_vals = nullptr;
    if (vals) { d_vals = reinterpret_cast<double*>(p); p += b_coo; }
    int* cnt = reinterpret_cast<int*>(p); p += b_rows;
    int* fill = reinterpret_cast<int*>(p); p += b_rows;
    int* kept = reinterpret_cast<int*>(p); p += b_rows;
    int64_t* start = reinterpret_cast<int64_t*>(p); p += b_start;
    int* stats = reinterpret_cast<int*>(p);

    TL_CK(c, cudaMemcpyAsync(d_rows, rows, (size_t)nnz * 8, cudaMemcpyDefault, c->stream));
    TL_CK(c, cudaMemcpyAsync(d_cols, cols, (size_t)nnz * 8, cudaMemcpyDefault, c->stream));
    if (vals) TL_CK(c, cudaMemcpyAsync(d_vals, vals, (size_t)nnz * 8, cudaMemcpyDefault, c->stream));
    TL_CK(c, cudaMemsetAsync(cnt, 0, 2 * b_rows, c->stream));   // cnt and fill
    const int h_init[8] = {0, 0, 1, 1, 1, 0, 0, 0};
    memcpy(c->h_flags + 16, h_init, sizeof h_init);
    TL_CK(c, cudaMemcpyAsync(stats, c->h_flags + 16, sizeof h_init, cudaMemcpyHostToDevice, c->stream));
    const unsigned g_e = (unsigned)std::min<int64_t>((nnz + 255) / 256, (int64_t)c->sm_count * 8);
    const unsigned g_r = (unsigned)std::min<int64_t>((lrows + 255) / 256, (int64_t)c->sm_count * 8);
    {
        LaunchScope L(c, "csr_from_coo", (double)nnz * 16.0);
        k_coo_count<<<g_e, 256, 0, c->stream>>>(d_rows, d_cols, nnz, t->dims[0], t->dims[1], world, c->rank, cnt,
                                                stats);
        k_scan_counts<<<1, kScanThreads, 0, c->stream>>>(cnt, lrows, start, stats + 1);
        TL_TRY(L.done());
    }
    TL_CK(c, cudaMemcpyAsync(c->h_flags + 16, stats, 8 * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    TL_CK(c, cudaMemcpyAsync(c->h_flags + 24, start + lrows, sizeof(int64_t), cudaMemcpyDeviceToHost, c->stream));
    TL_CK(c, cudaStreamSynchronize(c->stream));
    if (c->h_flags[16]) {
        *handled = true;
        return fail(c, TL_ERR_INVALID, "a COO entry lies outside %s", t->name.c_str());
    }
    if (c->h_flags[17] > kCsrRowMax) return TL_OK;   // a long row: the host build takes it
    int64_t count = 0;
    memcpy(&count, c->h_flags + 24, sizeof count);
    *handled = true;
    if (count > t->csr_cap || !t->rowptr || t->csr_rows != lrows) {
        TL_CK(c, cudaStreamSynchronize(c->stream));
        cudaFree(t->rowptr); cudaFree(t->colidx); cudaFree(t->vals);
        t->rowptr = nullptr; t->colidx = nullptr; t->vals = nullptr;
        t->csr_cap = 0;
        const int64_t cap = std::max<int64_t>(count, 1);
        TL_CK(c, cudaMalloc(&t->rowptr, (lrows + 1) * sizeof(int64_t)));
        TL_CK(c, cudaMalloc(&t->colidx, cap * sizeof(int32_t)));
        TL_CK(c, cudaMalloc(&t->vals, cap * sizeof(float)));
        t->csr_cap = cap;
    }
    {
        LaunchScope L(c, "csr_from_coo", (double)count * 24.0);
        k_coo_scatter<<<g_e, 256, 0, c->stream>>>(d_rows, d_cols, nnz, world, c->rank, start, fill, keys);
        k_row_dedupe<<<g_r, 256, 0, c->stream>>>(start, lrows, keys, kept);
        k_scan_counts<<<1, kScanThreads, 0, c->stream>>>(kept, lrows, t->rowptr, nullptr);
        k_csr_fill<<<g_r, 256, 0, c->stream>>>(start, t->rowptr, lrows, keys, d_vals, t->colidx, t->vals, stats);
        TL_TRY(L.done());
    }
    TL_CK(c, cudaMemcpyAsync(c->h_flags + 16, stats, 8 * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    TL_CK(c, cudaMemcpyAsync(c->h_flags + 24, t->rowptr + lrows, sizeof(int64_t), cudaMemcpyDeviceToHost, c->stream));
    TL_CK(c, cudaStreamSynchronize(c->stream));
    int64_t n = 0;
    memcpy(&n, c->h_flags + 24, sizeof n);
    t->nnz = n;
    t->csr_nonneg = c->h_flags[18] != 0;
    t->csr_pos = c->h_flags[19] != 0;
    t->csr_ones = c->h_flags[20] != 0;
    return TL_OK;
}

}  // namespace tl
