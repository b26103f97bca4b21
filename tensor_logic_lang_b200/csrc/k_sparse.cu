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

#include <algorithm>
#include <cstdlib>

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
// x in shared memory and closes it within the sweep (a breadth-first search
// from x over the successor lists):
//  * rows are taken from a counter, one at a time in the first sweep (every
//    row has work, and rows with large reach must not queue up behind one
//    another on a single warp) and 32 at a time afterwards, when the 32 lanes
//    check the rows' pending words together and load only rows with work;
//  * pending[r] is the lowest word of row r that may hold a bit whose
//    successors are not in the row yet (0 at the first sweep; none once the
//    row is closed);
//  * the row's set bits at or above that word start in the "spill" bit set;
//    the spill set feeds a circular queue of bit positions, and each step
//    every lane takes up to kItems queued bits, loads their successors
//    (kEdges per item per pass, all loads of a pass in flight together) and
//    ORs them into the row; every bit that was new joins the queue, or the
//    spill set when the queue is full.
// Every bit that enters the row is expanded exactly once, so the row is
// closed when queue and spill set are empty; a row never needs a second
// sweep.  On an edge set with u < v the first sweep closes every row (as the
// reference's in-place z-ascending loop does) and the second finds no pending
// row, so the sweep counts match the reference's (2).  On edge sets with back
// edges the fixpoint is the same bit for bit, reached in at most as many
// sweeps.
constexpr int kQueue = 1024;   // queued bit positions per warp (uint32)
constexpr int kItems = 4;      // queued bits one lane expands per step
constexpr int kEdges = 4;      // successors one lane loads per item per pass

__device__ __forceinline__ int warp_inclusive_scan(int v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    return v;
}

// Shared-memory words one warp of the sweep uses: row, spill set, queue.
__host__ __device__ __forceinline__ int64_t closure_warp_words(int64_t words) { return 2 * words + kQueue; }

// Moves up to `room` set bits of the spill set, lowest first from word `lo`,
// into the queue at position `tail`, clearing them.  Returns how many it
// moved and leaves in `lo` the lowest word that may still hold a bit (`words`
// when the set is empty).  Warp-uniform.
__device__ int harvest_spill(uint32_t* spill, int64_t words, int64_t& lo, uint32_t* q, int tail, int room,
                             int lane) {
    int stored = 0;
    for (int64_t w0 = lo & ~int64_t(31); w0 < words; w0 += 32) {
        const int64_t w = w0 + lane;
        const uint32_t bits = w < words ? spill[w] : 0u;
        const int cnt = __popc(bits);
        const int pre = warp_inclusive_scan(cnt, lane);
        const int total = __shfl_sync(0xffffffffu, pre, 31);
        const int start = stored + pre - cnt;
        const int allow = max(0, min(cnt, room - start));
        uint32_t take = bits;
        if (allow < cnt) {
            take = 0;
            uint32_t m = bits;
            for (int i = 0; i < allow; ++i) {
                take |= m & (0u - m);
                m &= m - 1;
            }
        }
        int at = tail + start;
        for (uint32_t m = take; m; m &= m - 1) q[(at++) % kQueue] = (uint32_t)(w * 32 + __ffs(m) - 1);
        if (take) spill[w] = bits & ~take;
        if (stored + total > room) {
            const unsigned left = __ballot_sync(0xffffffffu, (bits & ~take) != 0u);
            lo = w0 + (__ffs(left) - 1);
            return room;
        }
        stored += total;
    }
    lo = words;
    return stored;
}

__global__ void __launch_bounds__(128)
    k_closure_right(uint32_t* R, int64_t local_rows, int64_t words, const int64_t* __restrict__ rowptr,
                    const int32_t* __restrict__ colidx, int64_t e_rows, int* changed, unsigned long long* next_row,
                    int32_t* pending, int grab) {
    extern __shared__ uint32_t smem_u[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    uint32_t* row = smem_u + (int64_t)wib * closure_warp_words(words);
    uint32_t* spill = row + words;
    uint32_t* q = spill + words;
    bool any_changed = false;
    for (;;) {
        unsigned long long base = 0;
        if (lane == 0) base = atomicAdd(next_row, (unsigned long long)grab);
        base = __shfl_sync(0xffffffffu, base, 0);
        if ((int64_t)base >= local_rows) break;
        const int64_t mine = (int64_t)base + lane;
        const int32_t my_pend = (lane < grab && mine < local_rows) ? pending[mine] : INT32_MAX;
        unsigned todo = __ballot_sync(0xffffffffu, my_pend < words);
        while (todo) {
            const int src = __ffs(todo) - 1;
            todo &= todo - 1;
            const int64_t r = (int64_t)base + src;
            const int64_t start_w = __shfl_sync(0xffffffffu, my_pend, src);
            uint32_t* grow = R + r * words;
            for (int64_t w = lane; w < words; w += 32) {
                const uint32_t v = grow[w];
                row[w] = v;
                spill[w] = w >= start_w ? v : 0u;
            }
            __syncwarp();
            int64_t lo = start_w;   // lowest spill word that may hold a bit
            int head = 0, tail = 0;
            bool grew = false;
            for (;;) {
                if (head == tail) {
                    if (lo >= words) break;
                    const int got = harvest_spill(spill, words, lo, q, tail, kQueue, lane);
                    __syncwarp();
                    tail += got;
                    if (got == 0) break;
                    continue;
                }
                const int take = min(32 * kItems, tail - head);
                int64_t b[kItems], e[kItems];
#pragma unroll
                for (int k = 0; k < kItems; ++k) {
                    const int idx = k * 32 + lane;
                    const uint32_t y = idx < take ? q[(head + idx) % kQueue] : 0u;
                    b[k] = 0;
                    e[k] = 0;
                    if (idx < take && (int64_t)y < e_rows) {
                        b[k] = rowptr[y];
                        e[k] = rowptr[y + 1];
                    }
                }
                __syncwarp();   // the taken slots may be refilled from here on
                head += take;
                for (int64_t off = 0;; off += kEdges) {
                    int32_t z[kItems][kEdges];
#pragma unroll
                    for (int k = 0; k < kItems; ++k)
#pragma unroll
                        for (int j = 0; j < kEdges; ++j)
                            z[k][j] = b[k] + off + j < e[k] ? colidx[b[k] + off + j] : -1;
                    uint32_t fresh = 0;
#pragma unroll
                    for (int k = 0; k < kItems; ++k)
#pragma unroll
                        for (int j = 0; j < kEdges; ++j) {
                            const int32_t zz = z[k][j];
                            if (zz < 0) continue;
                            const uint32_t bit = 1u << (zz & 31);
                            if (row[zz >> 5] & bit) continue;
                            if (!(atomicOr(&row[zz >> 5], bit) & bit)) fresh |= 1u << (k * kEdges + j);
                        }
                    const int cnt = __popc(fresh);
                    const int pre = warp_inclusive_scan(cnt, lane);
                    const int total = __shfl_sync(0xffffffffu, pre, 31);
                    int at = tail + pre - cnt;
                    int64_t low = INT64_MAX;
#pragma unroll
                    for (int k = 0; k < kItems; ++k)
#pragma unroll
                        for (int j = 0; j < kEdges; ++j) {
                            if (!((fresh >> (k * kEdges + j)) & 1u)) continue;
                            const int32_t zz = z[k][j];
                            if (at < head + kQueue) {
                                q[at % kQueue] = (uint32_t)zz;
                            } else {
                                atomicOr(&spill[zz >> 5], 1u << (zz & 31));
                                low = min(low, (int64_t)(zz >> 5));
                            }
                            ++at;
                        }
                    if (total) {
                        grew = true;
                        tail = min(tail + total, head + kQueue);
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) low = min(low, __shfl_xor_sync(0xffffffffu, low, o));
                        lo = min(lo, low);
                    }
                    bool more = false;
#pragma unroll
                    for (int k = 0; k < kItems; ++k) more = more || (b[k] + off + kEdges < e[k]);
                    __syncwarp();
                    if (!__any_sync(0xffffffffu, more)) break;
                }
            }
            if (lane == 0) pending[r] = INT32_MAX;
            if (grew) {
                for (int64_t w = lane; w < words; w += 32) grow[w] = row[w];
                any_changed = true;
            }
            __syncwarp();
        }
    }
    if (lane == 0 && any_changed) *changed = 1;
}

// Warps per block and blocks per SM for a sweep over rows of `words` words
// with at most `smem_cap` bytes of shared memory per block: the split that
// keeps the most warps resident.
static void closure_shape(int64_t words, size_t smem_cap, int* wpb_out, int* per_sm_out, size_t* smem_out) {
    const size_t per_warp = (size_t)closure_warp_words(words) * 4;
    int best_wpb = 1, best_per_sm = 0;
    for (int wpb = 1; wpb <= 4; ++wpb) {
        const size_t smem = per_warp * wpb;
        if (smem > smem_cap) break;
        int per_sm = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_closure_right, 32 * wpb, smem);
        if (per_sm * wpb > best_per_sm * best_wpb) {
            best_wpb = wpb;
            best_per_sm = per_sm;
        }
    }
    *wpb_out = best_wpb;
    *per_sm_out = best_per_sm < 1 ? 1 : best_per_sm;
    *smem_out = per_warp * best_wpb;
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

// out[v, :] (+)= sum_e vals[e] * P[col(e), :], one warp per row, 128-bit
// loads of the gathered P rows (4 columns per lane and column half).
// A block waits until every other rank's fanned-out tiles of P have landed
// (their counters in this rank's array reach w.need), then the block's
// reads (plain or by the TMA) may start.  False if the wait ran out: the
// error word is set to 2 and the block does nothing.
__device__ __forceinline__ bool spmm_wait_peers(const SpWait& w, int* err) {
    __shared__ int ok_s;
    if (threadIdx.x == 0) {
        int ok = 1;
        if (w.cnt) {
            unsigned long long t0;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
            for (int j = 0; j < kMaxPeers && ok; ++j) {
                if (!w.need[j]) continue;
                for (;;) {
                    unsigned long long v;
                    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w.cnt + j) : "memory");
                    if (v >= w.need[j]) break;
                    unsigned long long now;
                    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
                    if (now - t0 > w.timeout_ns) {
                        atomicExch(err, 2);
                        ok = 0;
                        break;
                    }
                    __nanosleep(128);
                }
            }
            // the rows other ranks wrote are read next, also by the TMA
            asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

// The all-gather of a row-sharded GNN layer as peer stores: this rank's
// block of the gathered P (`len` floats at src, 16-byte aligned) is copied
// into the same place of every other rank's copy (dst[q], null for this
// rank), each block of threads storing a contiguous range with 128-bit
// stores over NVLink; then one thread per block adds 1 to every other
// rank's counter for this rank (release at system scope), after the
// block's stores (barrier, then a system-scope fence).
constexpr int kPushBlocks = 512;   // blocks of the push (every rank counts this many per layer)

struct PushArgs {
    const float* src;
    int64_t len;                           // floats, a multiple of 4
    float* dst[kMaxPeers];
    unsigned long long* cnt[kMaxPeers];
};

__global__ void __launch_bounds__(256) k_fan_push(const __grid_constant__ PushArgs a) {
    const int64_t n4 = a.len / 4;
    const int64_t per = (n4 + gridDim.x - 1) / gridDim.x;
    const int64_t b0 = (int64_t)blockIdx.x * per, b1 = min(n4, b0 + per);
    const float4* s4 = reinterpret_cast<const float4*>(a.src);
    for (int64_t i = b0 + threadIdx.x; i < b1; i += 4 * (int64_t)blockDim.x) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t j = i + (int64_t)u * blockDim.x;
            v[u] = j < b1 ? s4[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q = 0; q < kMaxPeers; ++q) {
            if (!a.dst[q]) continue;
            float4* d4 = reinterpret_cast<float4*>(a.dst[q]);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t j = i + (int64_t)u * blockDim.x;
                if (j < b1) d4[j] = v[u];
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int q = 0; q < kMaxPeers; ++q)
            if (a.cnt[q]) asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(a.cnt[q]), "l"(1ull) : "memory");
    }
}

template <int U>
__global__ void __launch_bounds__(256) k_spmm(int64_t rows, const int64_t* __restrict__ rowptr,
                                              const int32_t* __restrict__ colidx, const float* __restrict__ vals,
                                              const float* __restrict__ P, int64_t ldp, int64_t f, float* out,
                                              int64_t ldo, int beta, int col_world, int64_t col_local,
                                              const __grid_constant__ SpWait wait, int* err) {
    // rows other ranks wrote while this kernel may already run are read
    // through L2 (ld.cg), not the read-only path
    if (!spmm_wait_peers(wait, err)) return;
    const bool peer = wait.cnt != nullptr;
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const bool vec = (f % 4) == 0 && (ldp % 4) == 0 && (ldo % 4) == 0 && (((uintptr_t)P | (uintptr_t)out) & 15) == 0;
    for (int64_t v = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); v < rows; v += warps) {
        const int64_t e0 = rowptr[v], e1 = rowptr[v + 1];
        if (vec) {
            // the row's column indices and values 32 at a time, one per lane,
            // broadcast by shuffles; 4 nonzeros x 2 column halves (8 row
            // gathers) in flight per lane.  Each element still sums its terms
            // in nonzero order.
            for (int64_t jb = 0; jb < f; jb += 256) {
                const int64_t j0 = jb + lane * 4, j1 = j0 + 128;
                const bool h0 = j0 < f, h1 = j1 < f;
                float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
                for (int64_t eb = e0; eb < e1; eb += 32) {
                    const int ne = (int)(e1 - eb < 32 ? e1 - eb : 32);
                    long long u_l = 0;
                    float w_l = 0.f;
                    if (lane < ne) {
                        int64_t u = colidx[eb + lane];
                        if (col_world > 1) u = (u % col_world) * col_local + u / col_world;
                        u_l = (long long)u;
                        w_l = vals[eb + lane];
                    }
                    for (int k = 0; k < ne; k += U) {
                        float4 p0[U], p1[U];
                        float w[U];
#pragma unroll
                        for (int t = 0; t < U; ++t) {
                            const long long u = __shfl_sync(0xffffffffu, u_l, (k + t) & 31);
                            w[t] = __shfl_sync(0xffffffffu, w_l, (k + t) & 31);
                            const bool ok = k + t < ne;
                            const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
                            const float4* q0 = reinterpret_cast<const float4*>(P + u * ldp + j0);
                            const float4* q1 = reinterpret_cast<const float4*>(P + u * ldp + j1);
                            p0[t] = ok && h0 ? (peer ? __ldcg(q0) : __ldg(q0)) : z;
                            p1[t] = ok && h1 ? (peer ? __ldcg(q1) : __ldg(q1)) : z;
                        }
#pragma unroll
                        for (int t = 0; t < U; ++t) {
                            if (k + t >= ne) break;
                            a0.x = fmaf(w[t], p0[t].x, a0.x); a0.y = fmaf(w[t], p0[t].y, a0.y);
                            a0.z = fmaf(w[t], p0[t].z, a0.z); a0.w = fmaf(w[t], p0[t].w, a0.w);
                            a1.x = fmaf(w[t], p1[t].x, a1.x); a1.y = fmaf(w[t], p1[t].y, a1.y);
                            a1.z = fmaf(w[t], p1[t].z, a1.z); a1.w = fmaf(w[t], p1[t].w, a1.w);
                        }
                    }
                }
                if (h0) {
                    float4* op = reinterpret_cast<float4*>(out + v * ldo + j0);
                    if (beta) { const float4 o = *op; a0.x += o.x; a0.y += o.y; a0.z += o.z; a0.w += o.w; }
                    *op = a0;
                }
                if (h1) {
                    float4* op = reinterpret_cast<float4*>(out + v * ldo + j1);
                    if (beta) { const float4 o = *op; a1.x += o.x; a1.y += o.y; a1.z += o.z; a1.w += o.w; }
                    *op = a1;
                }
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

// ---------------------------------------------------------------------------
// SpMM with the row gathers done by the TMA (f = 128 or 256).  The kernel
// above is bound by the latency of its register-held gathers (each nonzero
// reads a 1 KB row of P from L2; 24 warps per SM at 80 registers).  Here
// every warp keeps a ring of slots of four P rows in shared memory: lane 0
// fills them with cp.async.bulk.tensor tile::gather4 copies (four nonzeros
// of one row per copy, completion counted on the slot's mbarrier) while the
// lanes sum the slots already landed, so no registers hold gathers in
// flight and 58 registers per thread leave room for 32 warps per SM.  Rows
// are taken cyclically (warp w: rows w, w + warps, ...); each element sums
// its terms in nonzero order with the same fmaf sequence as k_spmm, so the
// two kernels give identical results.
constexpr int kSpMaxSlots = 16;   // ring slots per warp (runtime count up to this)
constexpr int kSpMaxWarps = 8;    // warps per block (runtime count up to this)

__device__ __forceinline__ uint32_t sp_smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool sp_wait(uint64_t* bar, uint32_t parity, int* err) {
    const uint32_t addr = sp_smem_u32(bar);
    unsigned long long t0 = 0;
    for (unsigned it = 0;; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(addr), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((it & 1023u) == 0) {
            unsigned long long now;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (t0 == 0) t0 = now;
            else if (now - t0 > 2000000000ull) break;
        }
    }
    if (err) atomicExch(err, 1);
    return false;
}

template <int F>
__global__ void __launch_bounds__(32 * kSpMaxWarps) k_spmm_tma(const __grid_constant__ CUtensorMap tmP, int64_t rows,
                                                           const int64_t* __restrict__ rowptr,
                                                           const int32_t* __restrict__ colidx,
                                                           const float* __restrict__ vals, float* out, int64_t ldo,
                                                           int beta, int col_world, int64_t col_local, int* err,
                                                           int nslots, const __grid_constant__ SpWait wait) {
    if (!spmm_wait_peers(wait, err)) return;
    static_assert(F == 128 || F == 256, "row width");
    const int kSpWarps = blockDim.x >> 5;
    const int kSpSlots = nslots;
    constexpr int SLOT = 4 * F;   // floats
    extern __shared__ __align__(128) uint8_t sp_smem_raw[];
    // the TMA writes 128-byte aligned slots (the launch adds 128 bytes of slack)
    uint8_t* sp_smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sp_smem_raw) + 127) & ~uintptr_t(127));
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    float* ring = reinterpret_cast<float*>(sp_smem) + (size_t)wib * kSpSlots * SLOT;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sp_smem + (size_t)kSpWarps * kSpSlots * SLOT * 4) + wib * kSpSlots;
    if (lane == 0) {
        for (int k = 0; k < kSpSlots; ++k)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sp_smem_u32(&bars[k])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmP)) : "memory");
        if (wait.cnt) asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    __syncwarp();
    const int64_t warps = (int64_t)gridDim.x * kSpWarps;
    const int64_t first = (int64_t)blockIdx.x * kSpWarps + wib;
    // A row's nonzeros are taken 32 at a time: lane i holds the i-th column
    // (remapped to the gathered layout) and value, so a batch's four row
    // indices and weights come by shuffles, not by loads on the path to the
    // next copy.  Batches go into the ring in order; use u of the ring is
    // slot u % nslots, phase (u / nslots) & 1.
    uint32_t used = 0;
    int64_t nx0 = 0, nx1 = 0;   // the next row's nonzero range, loaded a row ahead
    if (first < rows) { nx0 = rowptr[first]; nx1 = rowptr[first + 1]; }
    for (int64_t v = first; v < rows; v += warps) {
        const int64_t e0 = nx0, e1 = nx1;
        if (v + warps < rows) { nx0 = rowptr[v + warps]; nx1 = rowptr[v + warps + 1]; }
        float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
        for (int64_t eb = e0; eb < e1; eb += 32) {
            const int ne = (int)(e1 - eb < 32 ? e1 - eb : 32);
            int32_t u_l = 0;
            float w_l = 0.f;
            if (lane < ne) {
                const int64_t u = colidx[eb + lane];
                u_l = (int32_t)(col_world > 1 ? (u % col_world) * col_local + u / col_world : u);
                w_l = vals[eb + lane];
            }
            const int nb = (ne + 3) >> 2;
            auto issue = [&](int b) {   // batch b of this chunk into the ring (uniform: every lane shuffles)
                int32_t u[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int k = 4 * b + t;
                    u[t] = __shfl_sync(0xffffffffu, u_l, k < ne ? k : 4 * b);
                }
                if (lane == 0) {
                    const int slot = (int)((used + (uint32_t)b) % (uint32_t)kSpSlots);
                    uint64_t* bar = &bars[slot];
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sp_smem_u32(bar)),
                                 "r"(SLOT * 4)
                                 : "memory");
                    asm volatile(
                        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes "
                        "[%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(sp_smem_u32(ring + (size_t)slot * SLOT)),
                        "l"(reinterpret_cast<uint64_t>(&tmP)), "r"(sp_smem_u32(bar)), "r"(0), "r"(u[0]), "r"(u[1]),
                        "r"(u[2]), "r"(u[3])
                        : "memory");
                }
            };
            const int ahead = nb < kSpSlots ? nb : kSpSlots;
            for (int b = 0; b < ahead; ++b) issue(b);
            for (int b = 0; b < nb; ++b) {
                const uint32_t use = used + (uint32_t)b;
                const int slot = (int)(use % (uint32_t)kSpSlots);
                if (!sp_wait(&bars[slot], (use / (uint32_t)kSpSlots) & 1u, err)) return;
                const float* rp = ring + (size_t)slot * SLOT;
                const int cnt = ne - 4 * b < 4 ? ne - 4 * b : 4;
                float w[4];
                float4 p0[4], p1[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    w[t] = __shfl_sync(0xffffffffu, w_l, (4 * b + t) & 31);
                    p0[t] = *reinterpret_cast<const float4*>(rp + t * F + lane * 4);
                    p1[t] = F == 256 ? *reinterpret_cast<const float4*>(rp + t * F + 128 + lane * 4) : p0[t];
                }
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    if (t >= cnt) break;
                    a0.x = fmaf(w[t], p0[t].x, a0.x); a0.y = fmaf(w[t], p0[t].y, a0.y);
                    a0.z = fmaf(w[t], p0[t].z, a0.z); a0.w = fmaf(w[t], p0[t].w, a0.w);
                    if (F == 256) {
                        a1.x = fmaf(w[t], p1[t].x, a1.x); a1.y = fmaf(w[t], p1[t].y, a1.y);
                        a1.z = fmaf(w[t], p1[t].z, a1.z); a1.w = fmaf(w[t], p1[t].w, a1.w);
                    }
                }
                __syncwarp();   // every lane has read the slot: it may be refilled
                if (b + kSpSlots < nb) issue(b + kSpSlots);
            }
            used += (uint32_t)nb;
        }
        float* op = out + v * ldo;
        float4* o0 = reinterpret_cast<float4*>(op + lane * 4);
        if (beta) { const float4 o = *o0; a0.x += o.x; a0.y += o.y; a0.z += o.z; a0.w += o.w; }
        *o0 = a0;
        if (F == 256) {
            float4* o1 = reinterpret_cast<float4*>(op + 128 + lane * 4);
            if (beta) { const float4 o = *o1; a1.x += o.x; a1.y += o.y; a1.z += o.z; a1.w += o.w; }
            *o1 = a1;
        }
    }
}

}  // namespace

int64_t fan_push_blocks() { return kPushBlocks; }

tl_status launch_fan_push(tl_ctx* c, const float* src, int64_t len, float* const* dst,
                          unsigned long long* const* cnt) {
    PushArgs a{};
    a.src = src;
    a.len = len;
    for (int q = 0; q < kMaxPeers; ++q) {
        a.dst[q] = dst[q];
        a.cnt[q] = cnt[q];
    }
    LaunchScope L(c, "gnn_fan_push", (double)len * 4.0, 0);
    k_fan_push<<<kPushBlocks, 256, 0, c->stream>>>(a);
    return L.done();
}

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
    t->csr_stamp = next_csr_stamp();
    t->csr_nonneg = hf[0] == 0;
    t->csr_pos = t->csr_nonneg;   // only nonzero values are stored
    t->csr_ones = hf[1] == 0;
    return TL_OK;
}

tl_status launch_closure_right(tl_ctx* c, Tensor* R, Tensor* E, int* d_changed, int sweep) {
    const int64_t words = R->bits_words;
    constexpr size_t kSmemCap = 200 * 1024;
    if ((size_t)closure_warp_words(words) * 4 > kSmemCap)
        return fail(c, TL_ERR_UNSUPPORTED, "closure rows of %lld bits exceed shared memory", (long long)R->dims[1]);
    TL_CK(c, cudaFuncSetAttribute(k_closure_right, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap));
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
    int wpb = 1, per_sm = 1;
    size_t smem = 0;
    closure_shape(words, kSmemCap, &wpb, &per_sm, &smem);
    int64_t grid = std::min<int64_t>((rows + wpb - 1) / wpb, (int64_t)c->sm_count * per_sm);
    if (grid < 1) grid = 1;
    k_closure_right<<<(unsigned)grid, 32 * wpb, smem, c->stream>>>(R->bits, rows, words, E->rowptr, E->colidx,
                                                                   E->csr_rows, d_changed, counter, pending,
                                                                   sweep == 0 ? 1 : 32);
    return L.done();
}

// The same right-form sweep with every buffer supplied by the caller and no
// context: for the allocation-free entry point (noalloc.cu).  Blocks stay
// within the default 48 KB of shared memory.
cudaError_t launch_closure_right_raw(uint32_t* R, int64_t rows, int64_t words, const int64_t* rowptr,
                                     const int32_t* colidx, int64_t e_rows, int* changed,
                                     unsigned long long* counter, int32_t* pending, int sweep,
                                     cudaStream_t stream) {
    constexpr size_t kSmemCap = 48 * 1024;
    if ((size_t)closure_warp_words(words) * 4 > kSmemCap) return cudaErrorInvalidValue;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int wpb = 1, per_sm = 1;
    size_t smem = 0;
    closure_shape(words, kSmemCap, &wpb, &per_sm, &smem);
    int64_t grid = std::min<int64_t>((rows + wpb - 1) / wpb, (int64_t)sms * per_sm);
    if (grid < 1) grid = 1;
    k_closure_right<<<(unsigned)grid, 32 * wpb, smem, stream>>>(R, rows, words, rowptr, colidx, e_rows, changed,
                                                                counter, pending, sweep == 0 ? 1 : 32);
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
                      const float* P, int64_t p_rows, int64_t ldp, int64_t f, float* out, int64_t ldo, int beta,
                      int relu_out, int col_world, int64_t col_local, const SpWait* wait) {
    (void)relu_out;
    if (rows <= 0) return TL_OK;
    SpWait w{};
    if (wait) {
        w = *wait;
        c->flags_armed = true;   // a wait that runs out sets the error word
    }
    const char* regs = getenv("TL_SPMM_REGS");
    CUtensorMap map;
    if ((f == 128 || f == 256) && ldo % 4 == 0 && ((uintptr_t)out & 15) == 0 && p_rows > 0 &&
        p_rows < INT32_MAX && !(regs && (regs[0] == '1' || regs[0] == '8')) &&
        make_gather_map(&map, P, f, p_rows, ldp)) {
        // gathers by the TMA: a persistent grid, three blocks of four warps per SM
        // ring slots per warp, warps per block and blocks per SM (TL_SPMM_SHAPE
        // = "slots,warps,blocks" overrides, for measurements)
        // (measured on the 2-layer GNN, n = 16384, f = 256, SpMM time per step:
        // one slot per warp, eight warps per block, four blocks per SM 0.055 ms;
        // two slots 0.059-0.061 ms; four slots 0.081-0.101 ms; eight slots
        // 0.130 ms; the register gathers 0.072 ms.  More copies in flight per
        // SM queue behind each other: the gathers' rate per SM, not the bytes
        // in flight, bounds the kernel)
        int kSpSlots = 1, kSpWarps = 8, bps = 4;
        if (const char* sh = getenv("TL_SPMM_SHAPE")) sscanf(sh, "%d,%d,%d", &kSpSlots, &kSpWarps, &bps);
        kSpSlots = std::max(1, std::min(kSpSlots, kSpMaxSlots));
        kSpWarps = std::max(1, std::min(kSpWarps, kSpMaxWarps));
        bps = std::max(1, bps);
        const size_t smem = (size_t)kSpWarps * kSpSlots * 4 * f * 4 + (size_t)kSpWarps * kSpSlots * 8 + 128;
        if (smem > 227 * 1024) return fail(c, TL_ERR_INVALID, "spmm ring of %zu bytes", smem);
        const int64_t grid = std::min<int64_t>((rows + kSpWarps - 1) / kSpWarps, (int64_t)c->sm_count * bps);
        LaunchScope L(c, "spmm_csr", 0, 0);
        c->flags_armed = true;
        if (f == 256) {
            TL_CK(c, cudaFuncSetAttribute(k_spmm_tma<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            k_spmm_tma<256><<<(unsigned)grid, 32 * kSpWarps, smem, c->stream>>>(map, rows, rowptr, colidx, vals, out,
                                                                             ldo, beta, col_world, col_local,
                                                                             c->d_flags + 8, kSpSlots, w);
        } else {
            TL_CK(c, cudaFuncSetAttribute(k_spmm_tma<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            k_spmm_tma<128><<<(unsigned)grid, 32 * kSpWarps, smem, c->stream>>>(map, rows, rowptr, colidx, vals, out,
                                                                             ldo, beta, col_world, col_local,
                                                                             c->d_flags + 8, kSpSlots, w);
        }
        return L.done();
    }
    LaunchScope L(c, "spmm_csr", 0, 0);
    if (regs && regs[0] == '8')   // eight nonzeros' gathers in flight per step
        k_spmm<8><<<grid_for(c, rows, 8), 256, 0, c->stream>>>(rows, rowptr, colidx, vals, P, ldp, f, out, ldo, beta,
                                                              col_world, col_local, w, c->d_flags + 8);
    else
        k_spmm<4><<<grid_for(c, rows, 8), 256, 0, c->stream>>>(rows, rowptr, colidx, vals, P, ldp, f, out, ldo, beta,
                                                              col_world, col_local, w, c->d_flags + 8);
    return L.done();
}

}  // namespace tl
