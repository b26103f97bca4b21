// Sparse and Boolean storages: CSR of `sparse` tensors, bit rows of 0/1
// tensors, the Boolean closure sweeps of the fixpoint driver, and CSR SpMM
// for message passing.
//
// Reference semantics:
//   sparse decl dense view          src/codegen/llvm.zig:482-516
//   recursive max= step(...) sweep  src/codegen/fixpoint.zig:167-297
//     right form  R[x,z] max= step(R[x,y] E[y,z])   (C4 transitive closure)
//     left form   R[x,y] max= step(E[x,z] R[z,y])   (examples/ancestor.tl)
//   per-term relu message passing   src/codegen/einsum.zig:20-196, expr.zig:245-249
//
// Closure on bit rows.  With R in {0,1} and E >= 0, step(R[x,y] E[y,z]) is
// R[x,y] AND (E[y,z] > 0), and `max=` is OR, so the right form's update of
// row x is R[x] |= OR_{y in R[x]} succ(y); rows never read other rows.  A
// warp keeps row x (n bits) in shared memory and closes it within one sweep
// (see k_closure_right).  The reference's in-place z-ascending loop also
// closes every row in its first sweep when the edges run u < v, so both take
// two sweeps there (the second confirms); on any edge set the fixpoint is the
// least one above the start, bit for bit.  A device-side changed word
// records whether any row gained a bit.
#include <vector>

#include "tl_internal.h"

namespace tl {
namespace {

__global__ void k_csr_to_dense(const int64_t* rowptr, const int32_t* colidx, const float* vals, int64_t rows,
                               int64_t cols, float* out) {
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows;
         r += (int64_t)gridDim.x * (blockDim.x / 32)) {
        for (int64_t e = rowptr[r] + (threadIdx.x & 31); e < rowptr[r + 1]; e += 32)
            out[r * cols + colidx[e]] = vals[e];
    }
}

// Output row r takes source row r * stride + offset (a rank's cyclic rows of
// a replicated source; stride 1, offset 0 otherwise).
__global__ void k_csr_to_bits(const int64_t* rowptr, const int32_t* colidx, const float* vals, int64_t rows,
                              int64_t words, uint32_t* bits, int64_t stride, int64_t offset) {
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows;
         r += (int64_t)gridDim.x * (blockDim.x / 32)) {
        const int64_t s = r * stride + offset;
        for (int64_t e = rowptr[s] + (threadIdx.x & 31); e < rowptr[s + 1]; e += 32) {
            if (vals[e] > 0.f) {   // step(E)
                const int32_t c = colidx[e];
                atomicOr(&bits[r * words + (c >> 5)], 1u << (c & 31));
            }
        }
    }
}

__global__ void k_dense_to_bits(const float* in, int64_t rows, int64_t cols, int64_t words, uint32_t* bits) {
    const int64_t total = rows * words;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / words, w = i % words;
        uint32_t b = 0;
        for (int j = 0; j < 32; ++j) {
            const int64_t c = w * 32 + j;
            if (c < cols && in[r * cols + c] > 0.f) b |= 1u << j;
        }
        bits[i] = b;
    }
}

__global__ void k_bits_to_dense(const uint32_t* bits, int64_t rows, int64_t cols, int64_t words, float* out) {
    const int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = i % cols;
        out[i] = (bits[r * words + (c >> 5)] >> (c & 31)) & 1u ? 1.f : 0.f;
    }
}

// Right-form sweep on bit rows.
//
// Rows are independent under R[x] |= OR_{y in R[x]} succ(y).  A warp holds row
// x in shared memory and closes it within the sweep:
//  * rows are grabbed 32 at a time from a counter (heaviest rows, the low
//    indices of a u < v DAG, first); the 32 lanes check the rows' pending
//    words together and only rows with work are loaded;
//  * pending[r] is the lowest word of row r that may hold a bit whose
//    successors are not in the row yet (0 at the first sweep; none once the
//    row is closed);
//  * the set bits at or above that word go into a queue in shared memory;
//    each step the 32 lanes take one queued bit each and OR its successors
//    (CSR) into the row, queueing every bit that was new.
// The row is closed when the queue drains, so a row never needs a second
// sweep: on an edge set with u < v the first sweep closes every row (as the
// reference's in-place z-ascending loop does) and the second one finds no
// pending row, so the sweep counts match the reference's (2).  On edge sets
// with back edges the fixpoint is the same bit for bit, reached in at most as
// many sweeps.  If the queue overflows, the row falls back to a windowed scan
// that re-expands every set bit in ascending order (idempotent), and a bit
// that scan sets below its window is left pending for the next sweep.
constexpr int kClosureWarps = 4;
constexpr int kWindowWords = 32;
constexpr int kQueue = 1024;        // queued bit positions per warp (uint32)

// successors of y into the row; queue new bits (or flag an overflow)
__device__ __forceinline__ bool expand_into(uint32_t* row, int64_t y, const int64_t* __restrict__ rowptr,
                                            const int32_t* __restrict__ colidx, int64_t e_rows, uint32_t* q,
                                            int* qtail, int head, bool* overflow) {
    bool grew = false;
    if (y >= e_rows) return false;
    const int64_t e1 = rowptr[y + 1];
    for (int64_t e = rowptr[y]; e < e1; ++e) {
        const int32_t z = colidx[e];
        const uint32_t bit = 1u << (z & 31);
        if (row[z >> 5] & bit) continue;
        const uint32_t old = atomicOr(&row[z >> 5], bit);
        if (old & bit) continue;
        grew = true;
        const int pos = atomicAdd(qtail, 1);
        if (pos < head + kQueue) q[pos % kQueue] = (uint32_t)z;
        else *overflow = true;
    }
    return grew;
}

// Windowed ascending scan from word `from`: expands every set bit (again),
// re-reading each 1024-bit window until stable.  Returns the lowest word a
// successor landed in below its window (left pending), INT32_MAX if none.
__device__ int32_t expand_windows(uint32_t* row, int64_t words, int64_t from, const int64_t* __restrict__ rowptr,
                                  const int32_t* __restrict__ colidx, int64_t e_rows, uint16_t* wl, bool* grew) {
    const int lane = threadIdx.x & 31;
    int32_t low = INT32_MAX;
    for (int64_t c0 = (from / kWindowWords) * kWindowWords; c0 < words; c0 += kWindowWords) {
        const int64_t w = c0 + lane;
        uint32_t done = 0;
        for (;;) {
            const uint32_t pend = (w < words ? row[w] : 0u) & ~done;
            const int cnt = __popc(pend);
            int pre = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, pre, o);
                if (lane >= o) pre += v;
            }
            const int total = __shfl_sync(0xffffffffu, pre, 31);
            if (total == 0) break;
            int at = pre - cnt;
            for (uint32_t m = pend; m; m &= m - 1) wl[at++] = (uint16_t)(lane * 32 + __ffs(m) - 1);
            done |= pend;
            __syncwarp();
            for (int i = lane; i < total; i += 32) {
                const int64_t y = c0 * 32 + wl[i];
                if (y >= e_rows) continue;
                const int64_t e1 = rowptr[y + 1];
                for (int64_t e = rowptr[y]; e < e1; ++e) {
                    const int32_t z = colidx[e];
                    const uint32_t bit = 1u << (z & 31);
                    if (row[z >> 5] & bit) continue;
                    const uint32_t old = atomicOr(&row[z >> 5], bit);
                    if (!(old & bit)) {
                        *grew = true;
                        if ((z >> 5) < c0) low = min(low, (int32_t)(z >> 5));
                    }
                }
            }
            __syncwarp();
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) low = min(low, __shfl_xor_sync(0xffffffffu, low, o));
    return low;
}

__global__ void __launch_bounds__(32 * kClosureWarps)
    k_closure_right(uint32_t* R, int64_t local_rows, int64_t words, const int64_t* __restrict__ rowptr,
                    const int32_t* __restrict__ colidx, int64_t e_rows, int* changed, unsigned long long* next_row,
                    int32_t* pending) {
    extern __shared__ uint32_t smem_u[];
    __shared__ int qtail_s[kClosureWarps];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    uint32_t* row = smem_u + (int64_t)wib * (words + kQueue);
    uint32_t* q = row + words;
    uint16_t* wl = reinterpret_cast<uint16_t*>(q);       // the windowed fallback reuses the queue
    int* qtail = &qtail_s[wib];
    bool any_changed = false;
    for (;;) {
        unsigned long long base = 0;
        if (lane == 0) base = atomicAdd(next_row, 32ull);
        base = __shfl_sync(0xffffffffu, base, 0);
        if ((int64_t)base >= local_rows) break;
        const int64_t mine = (int64_t)base + lane;
        const int32_t my_pend = mine < local_rows ? pending[mine] : INT32_MAX;
        unsigned todo = __ballot_sync(0xffffffffu, my_pend < words);
        while (todo) {
            const int src = __ffs(todo) - 1;
            todo &= todo - 1;
            const int64_t r = (int64_t)base + src;
            const int64_t start_w = __shfl_sync(0xffffffffu, my_pend, src);
            uint32_t* grow = R + r * words;
            for (int64_t w = lane; w < words; w += 32) row[w] = grow[w];
            if (lane == 0) *qtail = 0;
            __syncwarp();
            // queue the row's set bits from its pending word on
            bool overflow = false;
            int stored = 0;
            for (int64_t w0 = start_w & ~int64_t(31); w0 < words && !overflow; w0 += 32) {
                const int64_t w = w0 + lane;
                const uint32_t bits = (w < words && w >= start_w) ? row[w] : 0u;
                const int cnt = __popc(bits);
                int pre = cnt;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int v = __shfl_up_sync(0xffffffffu, pre, o);
                    if (lane >= o) pre += v;
                }
                const int total = __shfl_sync(0xffffffffu, pre, 31);
                if (stored + total > kQueue) { overflow = true; break; }
                int at = stored + pre - cnt;
                for (uint32_t m = bits; m; m &= m - 1) q[at++] = (uint32_t)(w * 32 + __ffs(m) - 1);
                stored += total;
            }
            if (lane == 0) *qtail = stored;
            __syncwarp();
            bool grew = false;
            int head = 0;
            while (!overflow) {
                const int tail = *(volatile int*)qtail;
                if (head >= tail) break;
                const int take = min(32, tail - head);
                uint32_t y = 0;
                if (lane < take) y = q[(head + lane) % kQueue];
                __syncwarp();
                bool ovf = false;
                if (lane < take) grew |= expand_into(row, y, rowptr, colidx, e_rows, q, qtail, head + take, &ovf);
                head += take;
                overflow = __any_sync(0xffffffffu, ovf);
                __syncwarp();
            }
            int32_t low = INT32_MAX;
            if (overflow) low = expand_windows(row, words, 0, rowptr, colidx, e_rows, wl, &grew);
            const bool row_grew = __any_sync(0xffffffffu, grew);
            if (lane == 0) pending[r] = low;
            if (row_grew) {
                for (int64_t w = lane; w < words; w += 32) grow[w] = row[w];
                any_changed = true;
            }
            __syncwarp();
        }
    }
    if (lane == 0 && any_changed) *changed = 1;
}

// Left-form sweep Rnew[x] = R[x] | OR_{z in succ(x)} R[z] from the previous
// sweep's rows.  The reference sweeps x upward in place; on an edge set with
// u < v every row it reads (z > x) has not been updated yet in that sweep,
// so its sweep is exactly this Jacobi step and the sweep counts agree.
__global__ void __launch_bounds__(256) k_closure_left(const uint32_t* __restrict__ R, uint32_t* __restrict__ Rnew,
                                                      int64_t n, int64_t words, const int64_t* __restrict__ rowptr,
                                                      const int32_t* __restrict__ colidx, int64_t e_rows,
                                                      int* changed) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t x = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); x < n; x += warps) {
        bool grew = false;
        for (int64_t w = lane; w < words; w += 32) {
            const uint32_t cur = R[x * words + w];
            uint32_t acc = cur;
            if (x < e_rows)
                for (int64_t e = rowptr[x]; e < rowptr[x + 1]; ++e) acc |= R[(int64_t)colidx[e] * words + w];
            Rnew[x * words + w] = acc;
            grew = grew || (acc != cur);
        }
        if (__any_sync(0xffffffffu, grew) && lane == 0) *changed = 1;
    }
}

// out[v, :] (+)= sum_e vals[e] * P[col(e), :], one warp per row, 4 columns
// per lane per step (128-bit loads of P rows).
__global__ void __launch_bounds__(256) k_spmm(int64_t rows, const int64_t* __restrict__ rowptr,
                                              const int32_t* __restrict__ colidx, const float* __restrict__ vals,
                                              const float* __restrict__ P, int64_t ldp, int64_t f, float* out,
                                              int64_t ldo, int beta, int col_world, int64_t col_local) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const bool vec = (f % 4) == 0 && (ldp % 4) == 0 && (ldo % 4) == 0 && (((uintptr_t)P | (uintptr_t)out) & 15) == 0;
    for (int64_t v = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); v < rows; v += warps) {
        const int64_t e0 = rowptr[v], e1 = rowptr[v + 1];
        if (vec) {
            for (int64_t j = lane * 4; j < f; j += 128) {
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int64_t e = e0; e < e1; ++e) {
                    int64_t u = colidx[e];
                    if (col_world > 1) u = (u % col_world) * col_local + u / col_world;
                    const float a = vals[e];
                    const float4 pv = __ldg(reinterpret_cast<const float4*>(P + u * ldp + j));
                    acc.x = fmaf(a, pv.x, acc.x); acc.y = fmaf(a, pv.y, acc.y);
                    acc.z = fmaf(a, pv.z, acc.z); acc.w = fmaf(a, pv.w, acc.w);
                }
                float4* op = reinterpret_cast<float4*>(out + v * ldo + j);
                if (beta) { const float4 o = *op; acc.x += o.x; acc.y += o.y; acc.z += o.z; acc.w += o.w; }
                *op = acc;
            }
        } else {
            for (int64_t j = lane; j < f; j += 32) {
                float acc = 0.f;
                for (int64_t e = e0; e < e1; ++e) {
                    int64_t u = colidx[e];
                    if (col_world > 1) u = (u % col_world) * col_local + u / col_world;
                    acc = fmaf(vals[e], P[u * ldp + j], acc);
                }
                float* op = out + v * ldo + j;
                *op = beta ? *op + acc : acc;
            }
        }
    }
}

// Dense → CSR, pass 1: nonzeros per row, and flags for negative / non-unit values.
__global__ void k_dense_count(const float* in, int64_t rows, int64_t cols, int64_t* counts, int* flags) {
    const int lane = threadIdx.x & 31;
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
        int64_t cnt = 0;
        bool neg = false, nonunit = false;
        for (int64_t cc = lane; cc < cols; cc += 32) {
            const float v = in[r * cols + cc];
            if (v != 0.f) { cnt++; nonunit = nonunit || v != 1.f; }
            neg = neg || v < 0.f;
        }
        for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
        if (__any_sync(0xffffffffu, neg) && lane == 0) atomicExch(&flags[0], 1);
        if (__any_sync(0xffffffffu, nonunit) && lane == 0) atomicExch(&flags[1], 1);
        if (lane == 0) counts[r] = cnt;
    }
}

// Dense → CSR, pass 2: columns in ascending order per row (warp ballot compaction).
__global__ void k_dense_fill(const float* in, int64_t rows, int64_t cols, const int64_t* rowptr, int32_t* colidx,
                             float* vals) {
    const int lane = threadIdx.x & 31;
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
        int64_t pos = rowptr[r];
        for (int64_t c0 = 0; c0 < cols; c0 += 32) {
            const int64_t cc = c0 + lane;
            const float v = cc < cols ? in[r * cols + cc] : 0.f;
            const unsigned m = __ballot_sync(0xffffffffu, v != 0.f);
            if (v != 0.f) {
                const int64_t at = pos + __popc(m & ((1u << lane) - 1u));
                colidx[at] = (int32_t)cc;
                vals[at] = v;
            }
            pos += __popc(m);
        }
    }
}

unsigned grid_for(tl_ctx* c, int64_t items, int per_block) {
    int64_t b = (items + per_block - 1) / per_block;
    const int64_t cap = (int64_t)c->sm_count * 16;
    if (b > cap) b = cap;
    return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

tl_status launch_csr_to_dense(tl_ctx* c, Tensor* t) {
    const int64_t rows = t->csr_rows;
    TL_CK(c, cudaMemsetAsync(t->dense, 0, (size_t)rows * t->dims[1] * 4, c->stream));
    if (t->nnz == 0) return TL_OK;
    LaunchScope L(c, "csr_to_dense", (double)t->nnz * 12.0);
    k_csr_to_dense<<<grid_for(c, rows, 8), 256, 0, c->stream>>>(t->rowptr, t->colidx, t->vals, rows, t->dims[1], t->dense);
    return L.done();
}

tl_status launch_csr_to_bits(tl_ctx* c, Tensor* src, Tensor* dst) {
    TL_TRY(alloc_bits_public(c, dst));
    TL_CK(c, cudaMemsetAsync(dst->bits, 0, (size_t)dst->bits_rows * dst->bits_words * 4, c->stream));
    if (src->nnz == 0) return TL_OK;
    // a replicated source feeding a row-sharded destination: rank's cyclic rows
    int64_t stride = 1, offset = 0;
    if (src->csr_rows != dst->bits_rows) {
        const bool dst_sharded = dst->shard == TL_SHARD_ROWS && c->world > 1;
        if (!(dst_sharded && src->csr_rows == dst->dims[0]))
            return fail(c, TL_ERR_INVALID, "csr/bit row mismatch");
        stride = c->world;
        offset = c->rank;
    }
    if (dst->bits_rows > 0 && (dst->bits_rows - 1) * stride + offset >= src->csr_rows)
        return fail(c, TL_ERR_INVALID, "csr/bit row mapping out of range");
    LaunchScope L(c, "csr_to_bits", (double)src->nnz * 12.0);
    k_csr_to_bits<<<grid_for(c, dst->bits_rows, 8), 256, 0, c->stream>>>(src->rowptr, src->colidx, src->vals,
                                                                          dst->bits_rows, dst->bits_words, dst->bits,
                                                                          stride, offset);
    return L.done();
}

tl_status launch_dense_to_bits(tl_ctx* c, Tensor* t) {
    const int64_t rows = t->bits_rows;
    LaunchScope L(c, "dense_to_bits", (double)rows * t->dims[1] * 4.0);
    k_dense_to_bits<<<grid_for(c, rows * t->bits_words, 256), 256, 0, c->stream>>>(t->dense, rows, t->dims[1],
                                                                                     t->bits_words, t->bits);
    return L.done();
}

tl_status launch_bits_to_dense(tl_ctx* c, Tensor* t) {
    const int64_t rows = t->bits_rows;
    LaunchScope L(c, "bits_to_dense", (double)rows * t->dims[1] * 4.0);
    k_bits_to_dense<<<grid_for(c, rows * t->dims[1], 256), 256, 0, c->stream>>>(t->bits, rows, t->dims[1],
                                                                                  t->bits_words, t->dense);
    return L.done();
}

tl_status launch_dense_to_csr(tl_ctx* c, Tensor* t) {
    if (t->rank != 2) return fail(c, TL_ERR_UNSUPPORTED, "sparse storage needs rank 2");
    if (t->shard == TL_SHARD_ROWS && c->world > 1) return fail(c, TL_ERR_UNSUPPORTED, "CSR of a sharded dense tensor");
    TL_TRY(ensure_dense(c, t));
    const int64_t rows = t->dims[0], cols = t->dims[1];
    void* ws = nullptr;
    TL_TRY(workspace(c, (size_t)(rows + 1) * 8 + 64, &ws));
    int64_t* counts = (int64_t*)ws;
    int* flags = (int*)(counts + rows + 1);
    TL_CK(c, cudaMemsetAsync(flags, 0, 2 * sizeof(int), c->stream));
    {
        LaunchScope L(c, "dense_to_csr_count", (double)rows * cols * 4.0);
        k_dense_count<<<grid_for(c, rows, 8), 256, 0, c->stream>>>(t->dense, rows, cols, counts, flags);
        TL_TRY(L.done());
    }
    std::vector<int64_t> h(rows + 1, 0);
    int hf[2];
    TL_CK(c, cudaMemcpyAsync(h.data() + 1, counts, rows * 8, cudaMemcpyDeviceToHost, c->stream));
    TL_CK(c, cudaMemcpyAsync(hf, flags, 2 * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    TL_CK(c, cudaStreamSynchronize(c->stream));
    for (int64_t r = 0; r < rows; ++r) h[r + 1] += h[r];
    const int64_t nnz = h[rows];
    if (nnz > t->csr_cap || !t->rowptr || t->csr_rows != rows) {
        cudaFree(t->rowptr); cudaFree(t->colidx); cudaFree(t->vals);
        t->rowptr = nullptr; t->colidx = nullptr; t->vals = nullptr;
        const int64_t cap = nnz > 0 ? nnz : 1;
        TL_CK(c, cudaMalloc(&t->rowptr, (rows + 1) * 8));
        TL_CK(c, cudaMalloc(&t->colidx, cap * 4));
        TL_CK(c, cudaMalloc(&t->vals, cap * 4));
        t->csr_cap = cap;
    }
    TL_CK(c, cudaMemcpyAsync(t->rowptr, h.data(), (rows + 1) * 8, cudaMemcpyHostToDevice, c->stream));
    {
        LaunchScope L(c, "dense_to_csr_fill", (double)rows * cols * 4.0);
        k_dense_fill<<<grid_for(c, rows, 8), 256, 0, c->stream>>>(t->dense, rows, cols, t->rowptr, t->colidx, t->vals);
        TL_TRY(L.done());
    }
    TL_CK(c, cudaStreamSynchronize(c->stream));   // h dies here
    t->nnz = nnz;
    t->csr_rows = rows;
    t->csr_valid = true;
    t->csr_nonneg = hf[0] == 0;
    t->csr_ones = hf[1] == 0;
    return TL_OK;
}

tl_status launch_closure_right(tl_ctx* c, Tensor* R, Tensor* E, int* d_changed, int sweep) {
    const int64_t words = R->bits_words;
    const size_t smem = (size_t)kClosureWarps * (words + kQueue) * 4;
    if (smem > 200 * 1024)
        return fail(c, TL_ERR_UNSUPPORTED, "closure rows of %lld bits exceed shared memory", (long long)R->dims[1]);
    static size_t attr = 0;
    if (smem > 48 * 1024 && smem > attr) {
        TL_CK(c, cudaFuncSetAttribute(k_closure_right, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr = smem;
    }
    const int64_t rows = R->bits_rows;
    // fixpoint-long state: the per-row pending word (0 = expand everything)
    if ((size_t)rows * 4 > c->aux_cap) {
        TL_CK(c, cudaStreamSynchronize(c->stream));
        cudaFree(c->aux);
        c->aux = nullptr;
        c->aux_cap = 0;
        TL_CK(c, cudaMalloc(&c->aux, std::max<size_t>((size_t)rows * 4, 4096)));
        c->aux_cap = std::max<size_t>((size_t)rows * 4, 4096);
    }
    int32_t* pending = (int32_t*)c->aux;
    if (sweep == 0 && rows > 0) TL_CK(c, cudaMemsetAsync(pending, 0, (size_t)rows * 4, c->stream));
    unsigned long long* counter = reinterpret_cast<unsigned long long*>(c->d_flags + 16);
    TL_CK(c, cudaMemsetAsync(counter, 0, sizeof(unsigned long long), c->stream));
    // algorithmic bytes of one sweep: read and write the local bit rows, read the CSR
    const double bytes = (double)rows * words * 4.0 * 2.0 + (double)(E->csr_rows + 1) * 8.0 + (double)E->nnz * 4.0;
    LaunchScope L(c, "closure_sweep", bytes, 0);
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_closure_right, 32 * kClosureWarps, smem);
    if (per_sm < 1) per_sm = 1;
    int64_t grid = std::min<int64_t>((rows + kClosureWarps - 1) / kClosureWarps, (int64_t)c->sm_count * per_sm);
    if (grid < 1) grid = 1;
    k_closure_right<<<(unsigned)grid, 32 * kClosureWarps, smem, c->stream>>>(R->bits, rows, words, E->rowptr,
                                                                            E->colidx, E->csr_rows, d_changed,
                                                                            counter, pending);
    return L.done();
}

// The same right-form sweep with every buffer supplied by the caller and no
// context: for the allocation-free entry point (noalloc.cu).
cudaError_t launch_closure_right_raw(uint32_t* R, int64_t rows, int64_t words, const int64_t* rowptr,
                                     const int32_t* colidx, int64_t e_rows, int* changed,
                                     unsigned long long* counter, int32_t* pending, cudaStream_t stream) {
    const size_t smem = (size_t)kClosureWarps * (words + kQueue) * 4;
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    int dev = 0, sms = 148, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_closure_right, 32 * kClosureWarps, smem);
    if (per_sm < 1) per_sm = 1;
    int64_t grid = std::min<int64_t>((rows + kClosureWarps - 1) / kClosureWarps, (int64_t)sms * per_sm);
    if (grid < 1) grid = 1;
    k_closure_right<<<(unsigned)grid, 32 * kClosureWarps, smem, stream>>>(R, rows, words, rowptr, colidx, e_rows,
                                                                         changed, counter, pending);
    return cudaGetLastError();
}

tl_status launch_closure_left(tl_ctx* c, Tensor* R, Tensor* E, int* d_changed) {
    const int64_t n = R->dims[0], words = R->bits_words;
    const size_t bytes = (size_t)n * words * 4;
    void* ws = nullptr;
    TL_TRY(workspace(c, bytes, &ws, WS_FIXPOINT));
    {
        LaunchScope L(c, "closure_left_sweep", (double)E->nnz * words * 4.0 + (double)n * words * 8.0, 0);
        k_closure_left<<<grid_for(c, n, 8), 256, 0, c->stream>>>(R->bits, (uint32_t*)ws, n, words, E->rowptr,
                                                                 E->colidx, E->csr_rows, d_changed);
        TL_TRY(L.done());
    }
    TL_CK(c, cudaMemcpyAsync(R->bits, ws, bytes, cudaMemcpyDeviceToDevice, c->stream));
    return TL_OK;
}

tl_status launch_spmm(tl_ctx* c, int64_t rows, const int64_t* rowptr, const int32_t* colidx, const float* vals,
                      const float* P, int64_t ldp, int64_t f, float* out, int64_t ldo, int beta, int relu_out,
                      int col_world, int64_t col_local) {
    (void)relu_out;
    if (rows <= 0) return TL_OK;
    LaunchScope L(c, "spmm_csr", 0, 0);
    k_spmm<<<grid_for(c, rows, 8), 256, 0, c->stream>>>(rows, rowptr, colidx, vals, P, ldp, f, out, ldo, beta, col_world,
                                                       col_local);
    return L.done();
}

}  // namespace tl
