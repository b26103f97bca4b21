// The right-form closure fixpoint in one cooperative launch.
//
// Reference semantics (src/codegen/fixpoint.zig:46-98, 167-297): repeat
// sweeps of  R[x,z] max= step(R[x,y] E[y,z])  until a sweep changes nothing,
// at most max_sweeps times.  On bit rows one sweep is R[x] |= OR_{y in R[x]}
// succ(y) for every row x; rows never read other rows.
//
// One launch runs every sweep.  Blocks stay resident (cooperative launch) and
// take rows from a counter; after each sweep they meet at a grid barrier,
// where the last block to arrive settles the sweep: it reads the changed
// word, on a multi-GPU context exchanges it with every other rank through
// peer memory (one 8-byte store per peer over NVLink, then a wait for the
// peers' stores), and decides whether another sweep runs.  The block that
// settles the last sweep writes the control block (sweep count, error word)
// into the host's pinned mirror, which the host reads once, after the
// launch.  Every wait is bounded by %globaltimer; a wait that runs out
// records an error word and the kernel returns.
//
// With the columns split over ranks, a rank stores a slice of every row:
// the warp still builds the full row in shared memory, ORs in and writes
// back only the slice, and takes the first sweep's changed word from the
// graph (k_two_hop), so no rank waits for another.
//
// Per row, a warp keeps the row in shared memory and closes it with a
// breadth-first search over a successor table: node y's entry is one 32-byte
// sector holding up to 8 successors (unused slots hold a sentinel bit that is
// always set), so a queued bit costs one load.  Nodes with more than 8
// successors keep 7 in the table, mark slot 7, and the rest are read from the
// CSR.  Each step a lane takes up to kFixItems queued bits; every successor
// that was not in the row is set and queued, or put in the spill bit set
// when the queue is full.  Each bit that enters the row is expanded exactly
// once, so the row is closed when queue and spill set are empty and never
// needs a second sweep: on an edge set with u < v the first sweep closes
// every row, as the reference's in-place z-ascending loop does, and the
// second finds nothing pending (2 sweeps, as the reference).
//
// Rows of step(E) (the lazy start) take a shortcut: such a row, once closed,
// is exactly E+(y), the nodes reachable from y in one or more steps, and
// E+(y) is a subset of E+(x) for every y reached from x.  So when the search
// from x reaches a node y whose row is local and closed already, the warp ORs
// row y into row x instead of expanding y's successors, and queues none of
// the bits it brings: they are closed under succ.  The first sweep takes the
// rows in descending order, so on an edge set with u < v every successor's
// row is closed before its predecessors' rows start, and a row costs a few
// row ORs: R[x] = succ(x) | OR_{y in succ(x)} R[y].  A closed row publishes
// its nonzero word range and then its pending word (release at GPU scope);
// readers load the pending word, fence (acquire) and read the row through L2.
#include <stdio.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "tl_internal.h"

namespace tl {
namespace {

constexpr int kFixQueue = 1024;   // queued bit positions per warp
constexpr int kFixItems = 4;      // queued bits one lane expands per step (1 in the lazy sweep)
constexpr int kFixWarps = 8;      // most warps per block (the team of a heavy row)
constexpr int kHeavyBudget = 2048; // with teams on: queued bits a lone warp expands before handing the row over
static_assert((kFixQueue & (kFixQueue - 1)) == 0, "queue positions wrap with a mask");

struct FixState {
    unsigned long long next_row[2];   // row counters, by sweep parity
    int changed[2];                   // a row grew this sweep, by parity
    unsigned int bar_count;           // blocks arrived at the barrier
    unsigned int bar_gen;             // barriers completed
    int go;                           // another sweep runs
    int sweeps;                       // sweeps completed
    int last_changed;                 // the last sweep changed a row (all ranks)
    int err;                          // 1: barrier wait ran out, 2: peer wait ran out
    int n_heavy;                      // rows handed to teams this sweep
    int heavy_next;                   // next of them a team takes
    // %globaltimer marks of the first kFixMarks sweeps: launch, every block's
    // lone-warp rows done (latest), team rows done, sweep settled (after the
    // peer exchange)
    unsigned long long t_start;
    unsigned long long t_rows[2];
    unsigned long long t_team[2];
    unsigned long long t_settled[2];
    // the lazy sweep's work, summed over warps: closed rows ORed in (this
    // rank's, another rank's) and nodes whose successors were expanded
    uint32_t n_or_local, n_or_remote, n_expanded;
};
constexpr int kFixMarks = 2;
constexpr size_t kFixStateBytes = 128;   // one control block (two by launch parity; the pinned mirror)
static_assert(sizeof(FixState) <= kFixStateBytes && sizeof(FixState) % 8 == 0, "control block");

struct FixArgs {
    uint32_t* R;
    int64_t rows, words, wpad;
    const int4* succ;
    const int64_t* rowptr;
    const int32_t* colidx;
    int64_t e_rows;
    int32_t* pending;
    int32_t* heavy;            // rows handed to teams (one slot per local row)
    unsigned long long* closed;   // per row of the lazy sweep's row space: its closed word once closed
    uint32_t epoch;               // this launch's epoch in the closed words
    // the row space of the lazy sweep with shortcuts: dp_rows rows at dpR, row
    // r holding node r * dp_stride + dp_offset.  It is the relation itself
    // (the local rows); on a row-sharded multi-GPU context it is every row of
    // the relation in a scratch buffer (dp_copy), each rank closing all of
    // them and copying its own rows (global r = lr * row_stride + row_offset)
    // into the relation.
    uint32_t* dpR;
    int64_t dp_rows, dp_stride, dp_offset;
    int dp_copy;
    // peer rows: the row space is this rank's own rows (dp_stride = world,
    // dp_offset = rank), published for the other ranks in a buffer every
    // rank maps (prows/pclosed[rank]) and also written to the relation; a
    // successor y on rank y % world is read there at local row y / world
    // (closed word with acquire at system scope, the row with plain loads
    // over NVLink)
    int peer_dp;
    int64_t n_glob;                          // nodes of the relation (rows over all ranks)
    // stored rows: rw words per row at word rw0 of the full-width row the
    // warp builds in shared memory (rw = words, rw0 = 0 unless the columns
    // are sharded: then this rank keeps columns [32 rw0, 32 (rw0 + rw)) of
    // every row, and closed rows are read, ORed and published as such slices)
    int64_t rw, rw0;
    // columns sharded: whether the first sweep changes a row anywhere in the
    // relation (some node two steps from a row's node is not one step from
    // it), computed from the graph, so every rank sets the same changed word
    const int* two_hop;
    unsigned long long* pclosed[kMaxPeers];
    uint32_t* prows[kMaxPeers];
    int shortcut;              // lazy rows OR closed rows in (and run in descending order)
    FixState* st;
    FixState* st_next;     // the next launch's control block, emptied by this one
    // the pinned host mirror of the control block: written by the block that
    // settles the last sweep (no copy behind the launch)
    unsigned long long* host_out;
    int team;                  // warps per block
    unsigned team_qmask;       // team queue positions - 1 (a power of two)
    int team_budget;           // rows handed to teams after this many queued bits (0: no teams)
    int lazy;                  // rows not written yet: row r starts as succ(r * row_stride + row_offset)
    int64_t row_stride, row_offset;
    int max_sweeps;
    unsigned nblocks;
    int world, rank;
    // the changed word crosses GPUs after each sweep (0 when every rank's
    // word is the same by construction: the replicated lazy sweep closes
    // every row of the relation on every rank)
    int exchange;
    unsigned long long* slots[kMaxPeers];   // every rank's slot array, [rank][parity]
    // sweeps this context exchanged before: a device word beside this rank's
    // slots, advanced by the last sweep's settling thread
    unsigned long long* token_base;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void store_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long load_acquire_gpu(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void store_release_gpu(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// A closed row's word: bits 42..63 the launch's epoch (1 .. 2^22 - 1),
// bits 21..41 the end and bits 0..20 the first word of its nonzero 16-byte
// groups (0, 0 when the row is empty).  A word from another launch has
// another epoch and reads as not closed, so no launch clears the array.
constexpr int kClosedSpan = 21;                       // row widths below 2^21 words
constexpr uint32_t kEpochMax = (1u << 22) - 1;
__device__ __forceinline__ unsigned long long closed_word(uint32_t epoch, int lo, int hi) {
    return ((unsigned long long)epoch << 42) | ((unsigned long long)(unsigned)hi << kClosedSpan) | (unsigned)lo;
}

// Local row of global node y (row r holds node r * row_stride + row_offset), or -1.
__device__ __forceinline__ int32_t local_row(int64_t rows, int64_t stride, int64_t offset, int32_t y) {
    const int64_t d = (int64_t)y - offset;
    if (d < 0) return -1;
    int64_t l = d;
    if (stride != 1) {
        const uint32_t ud = (uint32_t)d, us = (uint32_t)stride;
        if (ud % us) return -1;
        l = ud / us;
    }
    return l < rows ? (int32_t)l : -1;
}

// Handle of node y's row in the lazy sweep's row space, or -1 when y has no
// row there: the local row index, or with peer rows the node itself.
template <bool PEER>
__device__ __forceinline__ int32_t dp_handle(const FixArgs& a, int32_t y) {
    if (PEER) return (y >= 0 && y < a.n_glob) ? y : -1;
    return local_row(a.dp_rows, a.dp_stride, a.dp_offset, y);
}

// The closed word of row handle h, read with acquire (system scope for
// another rank's word: its release was at system scope too).
template <bool PEER>
__device__ __forceinline__ unsigned long long dp_closed_load(const FixArgs& a, int32_t h) {
    if (!PEER) return load_acquire_gpu(&a.closed[h]);
    const uint32_t o = (uint32_t)h % (uint32_t)a.world, l = (uint32_t)h / (uint32_t)a.world;
    return (int)o == a.rank ? load_acquire_gpu(a.pclosed[o] + l) : load_acquire_sys(a.pclosed[o] + l);
}

// The row of handle h (this rank's, or another rank's through peer memory).
template <bool PEER>
__device__ __forceinline__ const uint32_t* dp_row(const FixArgs& a, int32_t h) {
    if (!PEER) return a.dpR + (int64_t)h * a.rw;
    const uint32_t o = (uint32_t)h % (uint32_t)a.world, l = (uint32_t)h / (uint32_t)a.world;
    return a.prows[o] + (int64_t)l * a.words;
}

__device__ __forceinline__ int scan_incl(int v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    return v;
}

__device__ __forceinline__ int64_t warp_min64(int64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v, o));
    return v;
}

// Queue slot `pos` if it lies below `limit`, else the spill set.
__device__ __forceinline__ void enqueue(uint32_t* q, unsigned qmask, uint32_t* spill, int pos, int limit, int32_t z,
                                        int64_t& low) {
    if (pos < limit) {
        q[(unsigned)pos & qmask] = (uint32_t)z;
    } else {
        atomicOr(&spill[z >> 5], 1u << (z & 31));
        low = min(low, (int64_t)(z >> 5));
    }
}

// Test-and-set of bit z of the row; true when it was not set before.
__device__ __forceinline__ bool set_new(uint32_t* row, int32_t z) {
    const uint32_t bit = 1u << (z & 31);
    if (row[z >> 5] & bit) return false;
    return !(atomicOr(&row[z >> 5], bit) & bit);
}

// Moves up to `room` bits of the spill set, lowest first from word `lo`, into
// the queue at `tail`, clearing them; leaves in `lo` the lowest word that may
// still hold a bit (`words` when none).  Warp-uniform.
__device__ __forceinline__ int harvest(uint32_t* spill, int64_t words, int64_t& lo, uint32_t* q, unsigned qmask,
                                      int tail, int room, int lane) {
    int stored = 0;
    for (int64_t w0 = lo & ~int64_t(31); w0 < words; w0 += 32) {
        const int64_t w = w0 + lane;
        const uint32_t bits = w < words ? spill[w] : 0u;
        const int cnt = __popc(bits);
        const int pre = scan_incl(cnt, lane);
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
        for (uint32_t m = take; m; m &= m - 1)
            q[(unsigned)(at++) & qmask] = (uint32_t)(w * 32 + __ffs(m) - 1);
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

// Columns sharded: row slice (at word rw0 of the shared row) |= the slices
// of the closed rows held by the lanes in m (local row ly, nonzero words
// [lo, hi) of the slice).  Each lane takes 16-byte group lane of every
// 128-word piece; KPR pieces per row, so 8 / KPR source rows' loads are in
// flight per round, with every index known at compile time.
template <bool PEER, int KPR>
__device__ __forceinline__ void or_slices(const FixArgs& a, unsigned m, int32_t ly, int lo, int hi, uint32_t* row,
                                          int lane) {
    constexpr int RPR = 8 / KPR;
    const int rw = (int)a.rw;
    uint32_t* dst = row + a.rw0;
    while (m) {
        int32_t sl[RPR];
        int sa[RPR], sb[RPR];
#pragma unroll
        for (int j = 0; j < RPR; ++j) {
            sl[j] = -1;
            sa[j] = 0;
            sb[j] = 0;
            if (m) {
                const int src = __ffs(m) - 1;
                m &= m - 1;
                sl[j] = __shfl_sync(0xffffffffu, ly, src);
                sa[j] = max(__shfl_sync(0xffffffffu, lo, src), 0);
                sb[j] = min(__shfl_sync(0xffffffffu, hi, src), rw);
            }
        }
        uint4 v[RPR][KPR];
#pragma unroll
        for (int j = 0; j < RPR; ++j)
#pragma unroll
            for (int i = 0; i < KPR; ++i) {
                const int w = i * 128 + lane * 4;
                v[j][i] = (sl[j] >= 0 && w < rw && w + 4 > sa[j] && w < sb[j])
                              ? __ldcg(reinterpret_cast<const uint4*>(dp_row<PEER>(a, sl[j])) + (w >> 2))
                              : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
        for (int i = 0; i < KPR; ++i) {
            uint4 o = v[0][i];
#pragma unroll
            for (int j = 1; j < RPR; ++j) {
                o.x |= v[j][i].x; o.y |= v[j][i].y; o.z |= v[j][i].z; o.w |= v[j][i].w;
            }
            const int w = i * 128 + lane * 4;
            if (w < rw && (o.x | o.y | o.z | o.w)) {
                uint4 t = *reinterpret_cast<uint4*>(dst + w);
                t.x |= o.x; t.y |= o.y; t.z |= o.z; t.w |= o.w;
                *reinterpret_cast<uint4*>(dst + w) = t;
            }
        }
        __syncwarp();
    }
}

// row |= the closed rows held by the lanes (at most one per lane: local row
// ly, nonzero words [lo, hi)).  Each lane ORs its own words (16-byte groups
// lane, lane + 32, ... of every 1024-word chunk) of the source rows into the
// shared row, two source rows' loads in flight at a time: no index search and
// no shared-memory atomics.
template <bool PEER, bool COLS = false>
__device__ __forceinline__ void or_closed_rows(const FixArgs& a, bool has, int32_t ly, int lo, int hi,
                                               uint32_t* row, bool vec, int lane) {
    unsigned m = __ballot_sync(0xffffffffu, has);
    if (COLS) {
        // a slice of rw <= 1024 words: KPR 128-word pieces per row (kpr rounded
        // up to a power of two), 8 / KPR rows' loads in flight per round
        const int kpr = ((int)a.rw + 127) >> 7;
        if (kpr == 1) or_slices<PEER, 1>(a, m, ly, lo, hi, row, lane);
        else if (kpr == 2) or_slices<PEER, 2>(a, m, ly, lo, hi, row, lane);
        else if (kpr <= 4) or_slices<PEER, 4>(a, m, ly, lo, hi, row, lane);
        else or_slices<PEER, 8>(a, m, ly, lo, hi, row, lane);
        return;
    }
    const int words = (int)a.words;
    if (!vec) {
        while (m) {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            const uint32_t* srow = dp_row<PEER>(a, __shfl_sync(0xffffffffu, ly, src));
            const int l = max(__shfl_sync(0xffffffffu, lo, src), 0);
            const int h = min(__shfl_sync(0xffffffffu, hi, src), words);
            for (int w = l + lane; w < h; w += 32) row[w] |= __ldcg(srow + w);
            __syncwarp();
        }
        return;
    }
    // source rows in pairs: (ly, lo, hi) of each
    int n = __popc(m);
    int32_t sl[2];
    int sa[2], sb[2];
    for (int base = 0; base < words; base += 1024) {
        unsigned mm = m;
        for (int done = 0; done < n; done += 2) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                sl[j] = -1;
                sa[j] = 0;
                sb[j] = 0;
                if (mm) {
                    const int src = __ffs(mm) - 1;
                    mm &= mm - 1;
                    sl[j] = __shfl_sync(0xffffffffu, ly, src);
                    sa[j] = max(__shfl_sync(0xffffffffu, lo, src), 0);
                    sb[j] = min(__shfl_sync(0xffffffffu, hi, src), words);
                }
            }
            uint4 v[2][8];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint4* srow = reinterpret_cast<const uint4*>(dp_row<PEER>(a, max(sl[j], 0)));
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int w = base + i * 128 + lane * 4;
                    v[j][i] = (sl[j] >= 0 && w + 4 > sa[j] && w < sb[j]) ? __ldcg(srow + (w >> 2))
                                                                        : make_uint4(0u, 0u, 0u, 0u);
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 o = make_uint4(v[0][i].x | v[1][i].x, v[0][i].y | v[1][i].y, v[0][i].z | v[1][i].z,
                                           v[0][i].w | v[1][i].w);
                const int w = base + i * 128 + lane * 4;
                if (o.x | o.y | o.z | o.w) {
                    uint4 t = *reinterpret_cast<uint4*>(row + w);
                    t.x |= o.x;
                    t.y |= o.y;
                    t.z |= o.z;
                    t.w |= o.w;
                    *reinterpret_cast<uint4*>(row + w) = t;
                }
            }
        }
    }
}

// The search state of one row.
struct RowSearch {
    int head, tail;   // queue positions (wrapping)
    int64_t lo;       // lowest spill-set word that may hold a bit (words: none)
    bool grew;        // a bit beyond the starting ones entered the row
    uint32_t n_or_local = 0, n_or_remote = 0, n_expanded = 0;   // this lane's counts (lazy sweep)
};

// Expands the row's queued bits (and spill set) until both are empty.
// own_first: queue slot 0 holds the row's own node (a lazy row), whose
// successors are the starting bits and do not count as growth.  dp: a queued
// node whose local row is closed (lazy sweep) is ORed in, not expanded.
// budget > 0: returns false once more than that many bits were expanded (the
// row goes to a team); true when the row is closed.
template <int ITEMS, bool PEER, bool COUNT = false, bool COLS = false>
__device__ __forceinline__ bool search_row(const FixArgs& a, RowSearch& S, bool own_first, bool dp, int budget,
                                           uint32_t* row, uint32_t* spill, uint32_t* q, int lane) {
    const int64_t words = a.words;
    const bool vec = (words & 3) == 0;
    for (;;) {
        if (budget && S.head > budget) return false;
        if (S.head == S.tail) {
            if (S.lo >= words) return true;
            const int got = harvest(spill, words, S.lo, q, kFixQueue - 1, S.tail, kFixQueue, lane);
            __syncwarp();
            S.tail += got;
            if (got == 0) return true;
            continue;
        }
        const bool counts = !own_first || S.head != 0;
        const int take = min(32 * ITEMS, S.tail - S.head);
        const int nk = (take + 31) >> 5;
        int4 A[ITEMS], B[ITEMS];
        int32_t Y[ITEMS], L[ITEMS];
        unsigned long long CW[ITEMS];
#pragma unroll
        for (int k = 0; k < ITEMS; ++k) {
            A[k] = make_int4(-1, -1, -1, -1);
            B[k] = make_int4(-1, -1, -1, -1);
            Y[k] = -1;
            L[k] = -1;
            CW[k] = 0;
            if (k < nk) {
                const int idx = k * 32 + lane;
                if (idx < take) {
                    const int32_t y = (int32_t)q[(unsigned)(S.head + idx) & (kFixQueue - 1)];
                    Y[k] = y;
                    // the table entry is loaded with the closed word, not
                    // after it: one round trip either way
                    A[k] = __ldg(&a.succ[2 * (int64_t)y]);
                    B[k] = __ldg(&a.succ[2 * (int64_t)y + 1]);
                    if (dp) L[k] = dp_handle<PEER>(a, y);
                }
            }
        }
        if (dp) {
            // closed words read with acquire: the reads of a closed row come
            // after it (for the other lanes, through the warp barrier below)
#pragma unroll
            for (int k = 0; k < ITEMS; ++k)
                if (L[k] >= 0) CW[k] = dp_closed_load<PEER>(a, L[k]);
#pragma unroll
            for (int k = 0; k < ITEMS; ++k) {
                if (L[k] >= 0 && (uint32_t)(CW[k] >> 42) == a.epoch) {
                    if (COUNT) {
                        if (PEER && (uint32_t)L[k] % (uint32_t)a.world != (uint32_t)a.rank) S.n_or_remote++;
                        else S.n_or_local++;
                    }
                    Y[k] = -1;   // closed: ORed in below
                } else {
                    L[k] = -1;
                }
            }
#pragma unroll
            for (int k = 0; k < ITEMS; ++k)
                if (COUNT && Y[k] >= 0) S.n_expanded++;
        }
        __syncwarp();   // the taken slots may be refilled from here on
        S.head += take;
        const int limit = S.head + kFixQueue;
        unsigned long long fresh = 0;
#pragma unroll
        for (int k = 0; k < ITEMS; ++k) {
            if (k < nk && Y[k] >= 0) {
                const int32_t s[8] = {A[k].x, A[k].y, A[k].z, A[k].w, B[k].x, B[k].y, B[k].z, B[k].w};
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if ((j < 7 || s[j] >= 0) && set_new(row, s[j])) fresh |= 1ull << (k * 8 + j);
            }
        }
        const int cnt = __popcll(fresh);
        const int pre = scan_incl(cnt, lane);
        const int total = __shfl_sync(0xffffffffu, pre, 31);
        int64_t slow = INT64_MAX;
        if (fresh) {
            int at = S.tail + pre - cnt;
#pragma unroll
            for (int k = 0; k < ITEMS; ++k) {
                if (!((fresh >> (k * 8)) & 0xffull)) continue;
                const int32_t s[8] = {A[k].x, A[k].y, A[k].z, A[k].w, B[k].x, B[k].y, B[k].z, B[k].w};
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if ((fresh >> (k * 8 + j)) & 1ull) enqueue(q, kFixQueue - 1, spill, at++, limit, s[j], slow);
            }
        }
        if (total) {
            S.grew = S.grew || counts;
            S.tail = min(S.tail + total, limit);
        }
        // successors past the table's 7 (slot 7 marked with -2), one per
        // lane per round, items of a lane taken in turn
        unsigned xm = 0;
#pragma unroll
        for (int k = 0; k < ITEMS; ++k)
            if (k < nk && Y[k] >= 0 && B[k].w == -2) xm |= 1u << k;
        if (__any_sync(0xffffffffu, xm)) {
            int64_t e = 0, e_end = 0;
            for (;;) {
                if (e >= e_end && xm) {
                    const int k = __ffs(xm) - 1;
                    xm &= xm - 1;
                    int32_t y = Y[0];
#pragma unroll
                    for (int kk = 1; kk < ITEMS; ++kk)
                        if (k == kk) y = Y[kk];
                    e = a.rowptr[y] + 7;
                    e_end = a.rowptr[y + 1];
                }
                if (!__any_sync(0xffffffffu, e < e_end)) break;
                bool f = false;
                int32_t z = 0;
                if (e < e_end) {
                    z = a.colidx[e++];
                    f = set_new(row, z);
                }
                const unsigned bal = __ballot_sync(0xffffffffu, f);
                if (f) enqueue(q, kFixQueue - 1, spill, S.tail + __popc(bal & ((1u << lane) - 1u)), limit, z, slow);
                if (bal) {
                    S.grew = S.grew || counts;
                    S.tail = min(S.tail + __popc(bal), limit);
                }
            }
        }
        S.lo = min(S.lo, warp_min64(slow));
        __syncwarp();
        if (dp) {
            // closed rows reached this step: OR them in (their bits are
            // closed under succ and are not queued); growth is judged by the
            // caller from the row's final popcount
#pragma unroll
            for (int k = 0; k < ITEMS; ++k) {
                const bool has = L[k] >= 0;
                if (__any_sync(0xffffffffu, has))
                    or_closed_rows<PEER, COLS>(a, has, L[k], (int)(CW[k] & ((1u << kClosedSpan) - 1u)),
                                   (int)((CW[k] >> kClosedSpan) & ((1u << kClosedSpan) - 1u)), row, vec, lane);
            }
            __syncwarp();
        }
    }
}

// Closes every pending row taken from `next_row` (grab rows per counter
// step, ascending); true if a row grew.  Lazy rows start empty with their own
// node queued.  budget > 0: a row still open after that many queued bits is
// handed to the block's team (the row stays unwritten and pending).
// split: the warps take 32 rows each in turn instead (warp g: rows 32 g, then
// 32 (g + warps), ...), with no counter: for the sweeps after a shortcut sweep,
// which find every row closed (or the few a team left) and only read the
// pending words, so the counter's atomics would be most of their time.
__device__ __forceinline__ bool close_rows(const FixArgs& a, unsigned long long* next_row, int grab, bool lazy,
                                           int budget, uint32_t* row, uint32_t* spill, uint32_t* q, int lane,
                                           bool split = false) {
    const int64_t words = a.words;
    const bool vec = (words & 3) == 0;
    bool any = false;
    const int64_t wg = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    if (split) grab = 32;
    for (int64_t it = 0;; ++it) {
        unsigned long long base = 0;
        if (split) {
            base = (unsigned long long)((wg + it * nw) * 32);
        } else {
            if (lane == 0) base = atomicAdd(next_row, (unsigned long long)grab);
            base = __shfl_sync(0xffffffffu, base, 0);
        }
        if ((int64_t)base >= a.rows) break;
        const int64_t mine = (int64_t)base + lane;
        const int32_t my_pend = (lane < grab && mine < a.rows) ? a.pending[mine] : INT32_MAX;
        unsigned todo = __ballot_sync(0xffffffffu, my_pend < words);
        while (todo) {
            const int src = __ffs(todo) - 1;
            todo &= todo - 1;
            const int64_t r = (int64_t)base + src;
            const int64_t start_w = __shfl_sync(0xffffffffu, my_pend, src);
            uint32_t* grow = a.R + r * words;

            RowSearch S{0, 0, words, false};
            if (lazy) {
                // the row is step(E)'s row: start empty with the row's own
                // node queued; its successors (the starting bits) do not
                // count as growth
                for (int64_t w = lane * 4; w < a.wpad; w += 128)
                    *reinterpret_cast<uint4*>(row + w) = make_uint4(0u, 0u, 0u, 0u);
                if (lane == 0) q[0] = (uint32_t)(r * a.row_stride + a.row_offset);
                S.tail = 1;
                __syncwarp();
            } else {
            // load the row; its set bits from the pending word on are the
            // first frontier (queue, then spill set)
            int stored = 0;
            int64_t low = INT64_MAX;
            for (int64_t w0 = 0; w0 < words; w0 += 128) {
                const int64_t w = w0 + lane * 4;
                uint32_t v[4] = {0u, 0u, 0u, 0u};
                if (vec) {
                    if (w < words) {
                        const uint4 t = *reinterpret_cast<const uint4*>(grow + w);
                        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
                        *reinterpret_cast<uint4*>(row + w) = t;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (w + i < words) {
                            v[i] = grow[w + i];
                            row[w + i] = v[i];
                        }
                }
                int cnt = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (w + i < start_w) v[i] = 0u;
                    cnt += __popc(v[i]);
                }
                if (!__any_sync(0xffffffffu, cnt)) continue;
                const int pre = scan_incl(cnt, lane);
                const int total = __shfl_sync(0xffffffffu, pre, 31);
                if (cnt) {
                    int at = stored + pre - cnt;
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        for (uint32_t m = v[i]; m; m &= m - 1, ++at) {
                            if (at < kFixQueue) {
                                q[at] = (uint32_t)((w + i) * 32 + __ffs(m) - 1);
                            } else {
                                spill[w + i] |= m & (0u - m);
                                low = min(low, w + i);
                            }
                        }
                }
                stored += total;
            }
            S.tail = min(stored, kFixQueue);
            S.lo = warp_min64(low);
            if (S.lo > words) S.lo = words;
            __syncwarp();
            }

            if (!search_row<kFixItems, false>(a, S, lazy, false, budget, row, spill, q, lane)) {
                // too much work for one warp: leave the row (unwritten, still
                // pending) to a team of warps after this phase
                if (lane == 0) a.heavy[atomicAdd(&a.st->n_heavy, 1)] = (int32_t)r;
                for (int64_t w = lane * 4; w < a.wpad; w += 128)
                    *reinterpret_cast<uint4*>(spill + w) = make_uint4(0u, 0u, 0u, 0u);
                __syncwarp();
                continue;
            }
            if (S.grew || lazy) {
                if (vec) {
                    for (int64_t w = lane * 4; w < words; w += 128)
                        *reinterpret_cast<uint4*>(grow + w) = *reinterpret_cast<const uint4*>(row + w);
                } else {
                    for (int64_t w = lane; w < words; w += 32) grow[w] = row[w];
                }
                any = any || S.grew;
            }
            if (lane == 0) a.pending[r] = INT32_MAX;
            __syncwarp();
        }
    }
    return any;
}

// The lazy sweep with shortcuts: rows of step(E) taken one at a time in
// descending order.  A row starts as succ(x) (from the successor table, the
// CSR for the rest of a long list); fresh successors whose rows are closed are
// ORed in, the others are queued and the search expands them (ORing in the
// closed rows it meets).  The rows are software-pipelined: while row r runs,
// the warp already takes the next row's index, its table entry and its
// successors' closed words, so a row starts with all of them in hand.  A
// closed word read early may say "not closed" for a row that closes later;
// that successor is then expanded instead, with the same result.  A row grew
// if it ends with more bits than succ(x) has.  Once written, the row publishes
// its closed word (release at GPU scope) and its pending word.
template <bool PEER, bool COUNT, bool COLS>
__device__ __forceinline__ bool close_rows_dp(const FixArgs& a, unsigned long long* next_row, int budget,
                                              uint32_t* row, uint32_t* spill, uint32_t* q, int lane) {
    const int64_t words = a.words;
    const bool vec = (words & 3) == 0;
    const int32_t sentinel = (int32_t)(a.wpad * 32);
    const int32_t* succ32 = reinterpret_cast<const int32_t*>(a.succ);
    const unsigned lanes_below = (1u << lane) - 1u;
    auto node_of = [&](unsigned long long i) { return (int64_t)(a.dp_rows - 1 - (int64_t)i) * a.dp_stride + a.dp_offset; };
    // successor slot `lane` (< 8) of row i's table entry, and its closed word
    auto slot_of = [&](unsigned long long i) {
        return ((int64_t)i < a.dp_rows && lane < 8) ? __ldg(succ32 + 8 * node_of(i) + lane) : -1;
    };
    auto closed_of = [&](int32_t sl) {
        const int32_t l = (sl >= 0 && sl < sentinel) ? dp_handle<PEER>(a, sl) : -1;
        return l >= 0 ? dp_closed_load<PEER>(a, l) : 0ull;
    };
    bool any = false;
    uint32_t c_orl = 0, c_orr = 0, c_exp = 0;   // this lane's work counts
    unsigned long long nb = 0;
    if (lane == 0) nb = atomicAdd(next_row, 1ull);
    nb = __shfl_sync(0xffffffffu, nb, 0);
    int32_t t_next = slot_of(nb);
    unsigned long long cw_next = closed_of(t_next);
    // the row space starts empty; each row's write-back empties it again
    for (int64_t w = lane * 4; w < a.wpad; w += 128)
        *reinterpret_cast<uint4*>(row + w) = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();
    // the written row's closed word, published once every lane's stores of
    // the row are done (warp barrier, then a release store at GPU scope)
    int64_t pub_r = -1, pub_p = -1;
    unsigned long long pub_w = 0;
    auto publish = [&]() {
        __syncwarp();
        if (lane == 0 && pub_r >= 0) {
            if (PEER) store_release_sys(&a.closed[pub_r], pub_w);
            else store_release_gpu(&a.closed[pub_r], pub_w);
            if (pub_p >= 0) a.pending[pub_p] = INT32_MAX;
        }
        pub_r = -1;
        __syncwarp();
    };
    while ((int64_t)nb < a.dp_rows) {
        const int64_t r = a.dp_rows - 1 - (int64_t)nb;
        const int64_t gx = node_of(nb);
        const int32_t tslot = t_next;
        const unsigned long long cw = cw_next;

        // the starting bits succ(x)
        RowSearch S{0, 0, words, false};
        const bool more = __shfl_sync(0xffffffffu, tslot, 7) == -2;
        const int32_t s0 = (lane < 8 && tslot >= 0 && tslot < sentinel) ? tslot : -1;
        const bool f = s0 >= 0 && set_new(row, s0);
        const int32_t l0 = f ? dp_handle<PEER>(a, s0) : -1;
        const unsigned fresh = __ballot_sync(0xffffffffu, f);
        int n_init = __popc(fresh);
        unsigned long long nb2 = 0;
        if (lane == 0) nb2 = atomicAdd(next_row, 1ull);   // the row after this one
        bool closed = f && l0 >= 0 && (uint32_t)(cw >> 42) == a.epoch;
        // a successor that read as open when its word was fetched (a row
        // earlier) has often closed since: read those words once more, so
        // fewer successors are expanded
        unsigned long long cw_now = cw;
        if (__any_sync(0xffffffffu, f && l0 >= 0 && !closed) && f && l0 >= 0 && !closed) {
            cw_now = dp_closed_load<PEER>(a, l0);
            closed = (uint32_t)(cw_now >> 42) == a.epoch;
        }
        const unsigned open = __ballot_sync(0xffffffffu, f && !closed);
        if (f && !closed) q[__popc(open & lanes_below)] = (uint32_t)s0;
        S.tail = __popc(open);
        if (more) {
            int64_t slow = INT64_MAX;
            const int64_t e_end = a.rowptr[gx + 1];
            for (int64_t e0 = a.rowptr[gx] + 7; e0 < e_end; e0 += 32) {
                const int64_t e = e0 + lane;
                const int32_t z = e < e_end ? a.colidx[e] : -1;
                const bool fz = z >= 0 && set_new(row, z);
                const unsigned bal = __ballot_sync(0xffffffffu, fz);
                if (fz) enqueue(q, kFixQueue - 1, spill, S.tail + __popc(bal & lanes_below), kFixQueue, z, slow);
                S.tail = min(S.tail + __popc(bal), kFixQueue);
                n_init += __popc(bal);
            }
            S.lo = min((int64_t)words, warp_min64(slow));
        }
        // the next row's index and table entry, in flight during the ORs
        nb = __shfl_sync(0xffffffffu, nb2, 0);
        t_next = slot_of(nb);
        __syncwarp();
        or_closed_rows<PEER, COLS>(a, closed, l0, (int)(cw_now & ((1u << kClosedSpan) - 1u)),
                       (int)((cw_now >> kClosedSpan) & ((1u << kClosedSpan) - 1u)), row, vec, lane);
        __syncwarp();
        // its successors' closed words, in flight during the search and write-back
        cw_next = closed_of(t_next);

        if (COUNT && closed) {
            if (PEER && (uint32_t)l0 % (uint32_t)a.world != (uint32_t)a.rank) c_orr++;
            else c_orl++;
        }
        const bool done = search_row<1, PEER, COUNT, COLS>(a, S, false, true, budget, row, spill, q, lane);
        c_orl += S.n_or_local;
        c_orr += S.n_or_remote;
        c_exp += S.n_expanded;
        if (!done) {
            if (lane == 0) a.heavy[atomicAdd(&a.st->n_heavy, 1)] = (int32_t)r;
            for (int64_t w = lane * 4; w < a.wpad; w += 128) {
                *reinterpret_cast<uint4*>(spill + w) = make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(row + w) = make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();
            continue;
        }
        // write the row back (emptying the row space); its nonzero range and
        // popcount.  A copied row space also gives this rank's own rows to the
        // relation (its pending word marks the local row closed).
        uint32_t* grow = a.dpR + r * a.rw;
        uint32_t* own = nullptr;
        int64_t lr = r;
        if (a.dp_copy) {
            const int64_t d = r - a.row_offset;
            lr = (d >= 0 && d % a.row_stride == 0 && d / a.row_stride < a.rows) ? d / a.row_stride : -1;
            if (lr >= 0) own = a.R + lr * words;
        } else if (PEER) {
            own = a.R + r * words;   // the published copy above, the relation here
        }
        int lo_w = INT32_MAX, hi_w = 0, pc = 0;
        if (COLS) {
            // the slice goes out; the whole row space is emptied
            const uint32_t* src = row + a.rw0;
            for (int64_t w = lane * 4; w < a.rw; w += 128) {
                const uint4 t = *reinterpret_cast<const uint4*>(src + w);
                *reinterpret_cast<uint4*>(grow + w) = t;
                const int c = __popc(t.x) + __popc(t.y) + __popc(t.z) + __popc(t.w);
                if (c) {
                    pc += c;
                    lo_w = min(lo_w, (int)w);
                    hi_w = (int)w + 4;
                }
            }
            __syncwarp();
            for (int64_t w = lane * 4; w < a.wpad; w += 128)
                *reinterpret_cast<uint4*>(row + w) = make_uint4(0u, 0u, 0u, 0u);
        } else if (vec) {
            for (int64_t w = lane * 4; w < words; w += 128) {
                const uint4 t = *reinterpret_cast<const uint4*>(row + w);
                *reinterpret_cast<uint4*>(row + w) = make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(grow + w) = t;
                if (own) *reinterpret_cast<uint4*>(own + w) = t;
                const int c = __popc(t.x) + __popc(t.y) + __popc(t.z) + __popc(t.w);
                if (c) {
                    pc += c;
                    lo_w = min(lo_w, (int)w);
                    hi_w = (int)w + 4;
                }
            }
        } else {
            for (int64_t w = lane; w < words; w += 32) {
                const uint32_t t = row[w];
                row[w] = 0u;
                grow[w] = t;
                if (own) own[w] = t;
                if (t) {
                    pc += __popc(t);
                    lo_w = min(lo_w, (int)w);
                    hi_w = (int)w + 1;
                }
            }
        }
        lo_w = __reduce_min_sync(0xffffffffu, lo_w);
        hi_w = __reduce_max_sync(0xffffffffu, hi_w);
        pc = __reduce_add_sync(0xffffffffu, pc);
        // with the columns sharded a row's growth may lie in another rank's
        // slice: the changed word comes from the graph (two_hop) instead
        if (!COLS) any = any || pc > n_init;
        pub_r = r;
        pub_p = lr;
        pub_w = lo_w < hi_w ? closed_word(a.epoch, lo_w, hi_w) : closed_word(a.epoch, 0, 0);
        publish();
    }
    if (COUNT) {
    c_orl = __reduce_add_sync(0xffffffffu, c_orl);
    c_orr = __reduce_add_sync(0xffffffffu, c_orr);
    c_exp = __reduce_add_sync(0xffffffffu, c_exp);
    if (lane == 0) {
        atomicAdd(&a.st->n_or_local, c_orl);
        atomicAdd(&a.st->n_or_remote, c_orr);
        atomicAdd(&a.st->n_expanded, c_exp);
    }
    }
    return any;
}

// Last block of a sweep on a multi-GPU context: publish this rank's changed
// word to every rank (slot [rank][parity] of each rank's array), then wait for
// every rank's word of this sweep.  The parity slots keep a rank that is one
// sweep ahead from overwriting a word not read yet.  Returns the OR.
__device__ int exchange_changed(const FixArgs& a, int s, int c, int* ok) {
    const unsigned long long token = *(volatile const unsigned long long*)a.token_base + (unsigned long long)s + 1;
    const unsigned long long v = (token << 1) | (c ? 1ull : 0ull);
    const int par = s & 1;
    for (int j = 0; j < a.world; ++j) store_release_sys(a.slots[j] + 2 * a.rank + par, v);
    int any = c;
    const unsigned long long t0 = global_ns();
    const unsigned long long* mine = a.slots[a.rank];
    for (int j = 0; j < a.world; ++j) {
        unsigned long long got = load_acquire_sys(mine + 2 * j + par);
        while ((got >> 1) < token) {
            if (global_ns() - t0 > a.timeout_ns) {
                atomicExch(&a.st->err, 2);
                *ok = 0;
                return 0;
            }
            __nanosleep(64);
            got = load_acquire_sys(mine + 2 * j + par);
        }
        any |= (int)(got & 1ull);
    }
    return any;
}

// One row closed by the whole block (a team of a.team warps): the row, its
// spill set and one large queue (every warp's queue space) are shared; each
// step every lane takes up to kFixItems queued bits, and new bits are placed
// with one shared-memory atomic per warp.  Returns true if the row grew.
static_assert(kFixItems == 4, "the team's extra-successor pass selects among 4 items");
__device__ bool team_close_row(const FixArgs& a, int64_t r, int64_t start_w, bool lazy, uint32_t* row,
                               uint32_t* spill, uint32_t* q) {
    __shared__ int s_head, s_tail, s_grew;
    __shared__ unsigned long long s_lo;
    const int lane = threadIdx.x & 31;
    const int T = blockDim.x;
    const unsigned qmask = a.team_qmask;
    const int QT = (int)qmask + 1;
    const int64_t words = a.words;
    const bool vec = (words & 3) == 0;
    uint32_t* grow = a.R + r * words;
    if (lazy) {
        for (int64_t w = threadIdx.x * 4; w < a.wpad; w += 4 * T)
            *reinterpret_cast<uint4*>(row + w) = make_uint4(0u, 0u, 0u, 0u);
        if (threadIdx.x == 0) {
            q[0] = (uint32_t)(r * a.row_stride + a.row_offset);
            s_head = 0;
            s_tail = 1;
            s_lo = (unsigned long long)words;
        }
    } else {
        // every set bit from the pending word on starts in the spill set
        for (int64_t w = threadIdx.x; w < words; w += T) {
            const uint32_t v = grow[w];
            row[w] = v;
            spill[w] = w >= start_w ? v : 0u;
        }
        if (threadIdx.x == 0) {
            s_head = 0;
            s_tail = 0;
            s_lo = (unsigned long long)start_w;
        }
    }
    if (threadIdx.x == 0) s_grew = 0;
    for (;;) {
        __syncthreads();
        const int h = s_head, t = s_tail;
        if (h == t) {
            if (s_lo >= (unsigned long long)words) break;
            if (threadIdx.x < 32) {
                int64_t lo = (int64_t)s_lo;
                const int got = harvest(spill, words, lo, q, qmask, t, QT, lane);
                if (lane == 0) {
                    s_tail = t + got;
                    s_lo = (unsigned long long)lo;
                }
            }
            continue;
        }
        const bool counts = !lazy || h != 0;
        const int take = min(T * kFixItems, t - h);
        int4 A[kFixItems], B[kFixItems];
        int32_t Y[kFixItems];
#pragma unroll
        for (int k = 0; k < kFixItems; ++k) {
            A[k] = make_int4(-1, -1, -1, -1);
            B[k] = make_int4(-1, -1, -1, -1);
            Y[k] = -1;
            const int idx = k * T + threadIdx.x;
            if (idx < take) {
                const int32_t y = (int32_t)q[(unsigned)(h + idx) & qmask];
                Y[k] = y;
                A[k] = __ldg(&a.succ[2 * (int64_t)y]);
                B[k] = __ldg(&a.succ[2 * (int64_t)y + 1]);
            }
        }
        __syncthreads();   // every taken slot is read: they may be refilled
        const int limit = h + take + QT;
        unsigned long long fresh = 0;
#pragma unroll
        for (int k = 0; k < kFixItems; ++k) {
            if (Y[k] >= 0) {
                const int32_t sv[8] = {A[k].x, A[k].y, A[k].z, A[k].w, B[k].x, B[k].y, B[k].z, B[k].w};
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if ((j < 7 || sv[j] >= 0) && set_new(row, sv[j])) fresh |= 1ull << (k * 8 + j);
            }
        }
        const int cnt = __popcll(fresh);
        const int pre = scan_incl(cnt, lane);
        const int total = __shfl_sync(0xffffffffu, pre, 31);
        int64_t slow = INT64_MAX;
        if (total) {
            int base = 0;
            if (lane == 31) base = atomicAdd(&s_tail, total);
            base = __shfl_sync(0xffffffffu, base, 31);
            int at = base + pre - cnt;
#pragma unroll
            for (int k = 0; k < kFixItems; ++k) {
                if (!((fresh >> (k * 8)) & 0xffull)) continue;
                const int32_t sv[8] = {A[k].x, A[k].y, A[k].z, A[k].w, B[k].x, B[k].y, B[k].z, B[k].w};
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if ((fresh >> (k * 8 + j)) & 1ull) enqueue(q, qmask, spill, at++, limit, sv[j], slow);
            }
            if (counts && lane == 0) s_grew = 1;
        }
        unsigned xm = 0;
#pragma unroll
        for (int k = 0; k < kFixItems; ++k)
            if (Y[k] >= 0 && B[k].w == -2) xm |= 1u << k;
        if (__any_sync(0xffffffffu, xm)) {
            int64_t e = 0, e_end = 0;
            for (;;) {
                if (e >= e_end && xm) {
                    const int k = __ffs(xm) - 1;
                    xm &= xm - 1;
                    const int32_t y = k == 0 ? Y[0] : k == 1 ? Y[1] : k == 2 ? Y[2] : Y[3];
                    e = a.rowptr[y] + 7;
                    e_end = a.rowptr[y + 1];
                }
                if (!__any_sync(0xffffffffu, e < e_end)) break;
                bool f = false;
                int32_t z = 0;
                if (e < e_end) {
                    z = a.colidx[e++];
                    f = set_new(row, z);
                }
                const unsigned bal = __ballot_sync(0xffffffffu, f);
                if (bal) {
                    int base = 0;
                    if (lane == 0) base = atomicAdd(&s_tail, __popc(bal));
                    base = __shfl_sync(0xffffffffu, base, 0);
                    if (f) enqueue(q, qmask, spill, base + __popc(bal & ((1u << lane) - 1u)), limit, z, slow);
                    if (counts && lane == 0) s_grew = 1;
                }
            }
        }
        slow = warp_min64(slow);
        if (lane == 0 && slow != INT64_MAX) atomicMin(&s_lo, (unsigned long long)slow);
        __syncthreads();
        if (threadIdx.x == 0) {
            s_head = h + take;
            if (s_tail > h + take + QT) s_tail = h + take + QT;   // the rest went to the spill set
        }
    }
    const bool grew = s_grew != 0;
    if (grew || lazy) {
        if (vec) {
            for (int64_t w = threadIdx.x * 4; w < words; w += 4 * T)
                *reinterpret_cast<uint4*>(grow + w) = *reinterpret_cast<const uint4*>(row + w);
        } else {
            for (int64_t w = threadIdx.x; w < words; w += T) grow[w] = row[w];
        }
    }
    if (threadIdx.x == 0) a.pending[r] = INT32_MAX;
    __syncthreads();
    return grew;
}

// Grid barrier number `gen` (1, 2, ...).  At the end of sweep s (settle) the
// last block to arrive settles the sweep: reads the changed word, exchanges it
// with the other ranks, decides whether another sweep runs.  False if a wait
// ran out.
__device__ bool grid_barrier(const FixArgs& a, unsigned gen, int s, bool settle) {
    __shared__ int ok_s;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        if (s < kFixMarks) atomicMax(settle ? &a.st->t_team[s] : &a.st->t_rows[s], global_ns());
        __threadfence();
        const unsigned prev = atomicAdd(&a.st->bar_count, 1u);
        if (prev == a.nblocks - 1) {
            __threadfence();
            if (settle) {
                int c = *(volatile int*)&a.st->changed[s & 1];
                if (a.exchange) c = exchange_changed(a, s, c, &ok);
                a.st->next_row[(s + 1) & 1] = 0;
                a.st->changed[(s + 1) & 1] = 0;
                a.st->n_heavy = 0;
                a.st->heavy_next = 0;
                a.st->sweeps = s + 1;
                a.st->last_changed = c;
                a.st->go = (ok && c && s + 1 < a.max_sweeps) ? 1 : 0;
                // the last sweep of the launch moves the token base past it
                if (a.exchange && !a.st->go) *a.token_base += (unsigned long long)(s + 1);
                if (s < kFixMarks) a.st->t_settled[s] = global_ns();
                if (!a.st->go) {
                    // the launch's result to the host's pinned mirror (visible
                    // to the host once the launch has completed)
                    __threadfence();
                    const volatile unsigned long long* src = reinterpret_cast<const volatile unsigned long long*>(a.st);
                    volatile unsigned long long* dst = a.host_out;
#pragma unroll
                    for (int i = 0; i < (int)(sizeof(FixState) / 8); ++i) dst[i] = src[i];
                }
            }
            a.st->bar_count = 0;
            __threadfence();
            atomicExch(&a.st->bar_gen, gen);
        } else {
            // the settling block may itself wait up to timeout_ns for the
            // other ranks: the blocks waiting for it allow twice that, so a
            // peer wait that runs out is the one reported
            const unsigned long long t0 = global_ns();
            const unsigned long long lim = a.world > 1 ? 2 * a.timeout_ns : a.timeout_ns;
            while (*(volatile unsigned*)&a.st->bar_gen < gen) {
                if (global_ns() - t0 > lim) {
                    atomicExch(&a.st->err, 1);
                    ok = 0;
                    break;
                }
                __nanosleep(128);
            }
        }
        __threadfence();
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

// COUNT: the lazy sweep counts its work (profiling runs that ask for it)
template <bool PEER, bool COUNT, bool COLS>
__global__ void __launch_bounds__(32 * kFixWarps, 2) k_closure_fix(const FixArgs a) {
    extern __shared__ __align__(16) uint32_t smem_fix[];
    __shared__ int s_idx;
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    uint32_t* row = smem_fix + (int64_t)wib * (2 * a.wpad + 4 + kFixQueue);
    uint32_t* spill = row + a.wpad + 4;
    uint32_t* q = spill + a.wpad;
    if (blockIdx.x == 0 && threadIdx.x == 0) a.st->t_start = global_ns();
    // the next launch's control block (the one the launch before this used,
    // whose result the host has read): emptied here, not by a host memset
    if (blockIdx.x == 0 && threadIdx.x < sizeof(FixState) / 8)
        reinterpret_cast<unsigned long long*>(a.st_next)[threadIdx.x] = 0ull;
    unsigned gen = 0;
    for (int s = 0; s < a.max_sweeps; ++s) {
        const bool lazy = a.lazy && s == 0;
        // each warp's own row space: the sentinel successor (bit 0 of word
        // wpad) reads as set; the spill set starts empty (a team row may have
        // used this space as queue)
        if (lane == 0) row[a.wpad] = 0xffffffffu;
        for (int64_t w = lane * 4; w < a.wpad; w += 128)
            *reinterpret_cast<uint4*>(spill + w) = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
        const int budget = a.team > 1 ? a.team_budget : 0;
        const bool grew = lazy && a.shortcut
                              ? close_rows_dp<PEER, COUNT, COLS>(a, &a.st->next_row[s & 1],
                                                                 a.dp_copy || PEER || COLS ? 0 : budget, row,
                                              spill, q, lane)
                              : close_rows(a, &a.st->next_row[s & 1], s == 0 ? 1 : 32, lazy, budget, row, spill, q,
                                           lane, s > 0 && a.lazy && a.shortcut);
        if (lane == 0 && grew) *(volatile int*)&a.st->changed[s & 1] = 1;
        if (COLS && lazy && blockIdx.x == 0 && threadIdx.x == 0 && *(volatile const int*)a.two_hop)
            *(volatile int*)&a.st->changed[s & 1] = 1;
        if (a.team > 1 && a.team_budget > 0) {
            if (!grid_barrier(a, ++gen, s, false)) return;
            // rows handed over in this sweep, one per block at a time
            const int n_heavy = *(volatile int*)&a.st->n_heavy;
            uint32_t* trow = smem_fix;
            for (;;) {
                if (threadIdx.x == 0) s_idx = atomicAdd(&a.st->heavy_next, 1);
                __syncthreads();
                const int idx = s_idx;
                __syncthreads();
                if (idx >= n_heavy) break;
                const int64_t r = a.heavy[idx];
                const bool tg = team_close_row(a, r, lazy ? 0 : a.pending[r], lazy, trow, trow + a.wpad + 4,
                                               trow + 2 * a.wpad + 4);
                if (threadIdx.x == 0 && tg) *(volatile int*)&a.st->changed[s & 1] = 1;
            }
        }
        if (!grid_barrier(a, ++gen, s, true)) return;
        if (!*(volatile int*)&a.st->go) return;
    }
}

// Successor table: entry y = 8 int32.  deg <= 8: the successors, unused
// slots the sentinel; deg > 8: the first 7, slot 7 = -2 (the rest from the
// CSR at rowptr[y] + 7).  Nodes without a CSR row have none.
__global__ void k_build_succ(const int64_t* __restrict__ rowptr, const int32_t* __restrict__ colidx, int64_t e_rows,
                             int64_t nodes, int32_t sentinel, int4* __restrict__ out) {
    for (int64_t y = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; y < nodes; y += (int64_t)gridDim.x * blockDim.x) {
        int32_t s[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] = sentinel;
        if (y < e_rows) {
            const int64_t b = rowptr[y], d = rowptr[y + 1] - b;
            const int inl = d > 8 ? 7 : (int)d;
            for (int j = 0; j < inl; ++j) s[j] = colidx[b + j];
            if (d > 8) s[7] = -2;
        }
        out[2 * y] = make_int4(s[0], s[1], s[2], s[3]);
        out[2 * y + 1] = make_int4(s[4], s[5], s[6], s[7]);
    }
}

// every instantiation the host launches (one launch shape fits all of them)
const void* const kFixVariants[] = {
    (const void*)k_closure_fix<false, false, false>, (const void*)k_closure_fix<true, false, false>,
    (const void*)k_closure_fix<false, true, false>,  (const void*)k_closure_fix<true, true, false>,
    (const void*)k_closure_fix<false, false, true>,  (const void*)k_closure_fix<false, true, true>};

// Sets *flag when some node z two steps from a node x (x -> y -> z) is not
// one step from it: exactly when a first sweep from step(E) adds a bit to
// some row (fixpoint.zig:256-273 on R = step(E)).  Column lists are sorted
// within a row (both CSR builds sort them).
__global__ void k_two_hop(const int64_t* __restrict__ rowptr, const int32_t* __restrict__ colidx, int64_t e_rows,
                          int* flag) {
    for (int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; x < e_rows; x += (int64_t)gridDim.x * blockDim.x) {
        if (*(volatile int*)flag) return;
        const int64_t b = rowptr[x], e = rowptr[x + 1];
        for (int64_t i = b; i < e; ++i) {
            const int32_t y = colidx[i];
            if (y < 0 || y >= e_rows) continue;
            for (int64_t j = rowptr[y]; j < rowptr[y + 1]; ++j) {
                const int32_t z = colidx[j];
                int64_t lo = b, hi = e;   // is z one of x's successors?
                while (lo < hi) {
                    const int64_t mid = (lo + hi) >> 1;
                    if (colidx[mid] < z) lo = mid + 1;
                    else hi = mid;
                }
                if (lo >= e || colidx[lo] != z) {
                    atomicExch(flag, 1);
                    return;
                }
            }
        }
    }
}

size_t fix_smem_per_warp(int64_t words) {
    const int64_t wpad = (words + 3) & ~int64_t(3);
    return (size_t)(2 * wpad + 4 + kFixQueue) * 4;
}

}  // namespace

// How a row-sharded relation runs its lazy sweep on several GPUs
// (TL_CLOSURE_SHARDED).  "replicate" (default): every rank closes every row
// in a scratch copy and keeps its own, with no changed word crossing GPUs.
// "peer": each rank closes its own rows and takes shortcuts through every
// rank's closed rows, read over NVLink from a buffer each rank publishes
// them in.  "local": each rank closes its own rows with shortcuts through
// its own closed rows only.  "bfs": each rank closes its own rows by a full
// breadth-first search, no shortcuts.  Measured at n = 32768 (first sweep,
// per launch): replicate 0.12-0.13 ms at every N; peer 0.24 / 0.27 / 0.29 ms
// at N = 2 / 4 / 8; bfs 0.24 / 0.23 ms at N = 4 / 8; local 0.25 ms at N = 2.
// Splitting the rows does not shorten the sweep: each row is a chain of
// dependent loads (longer when they cross NVLink), more rows in flight leave
// more successors open and expanded, and without shortcuts the deepest rows'
// searches alone take 0.2 ms.
enum ShardedSweep { SWEEP_PEER, SWEEP_REPLICATE, SWEEP_LOCAL, SWEEP_BFS };
static ShardedSweep sharded_sweep_mode() {
    const char* m = getenv("TL_CLOSURE_SHARDED");
    if (m && !strcmp(m, "local")) return SWEEP_LOCAL;
    if (m && !strcmp(m, "peer")) return SWEEP_PEER;
    if (m && !strcmp(m, "bfs")) return SWEEP_BFS;
    return SWEEP_REPLICATE;
}

tl_status launch_closure_fixpoint(tl_ctx* c, Tensor* R, Tensor* E, int max_sweeps, bool need_now, int* sweeps_out,
                                  bool* changed_out, bool* handled) {
    *handled = false;
    // the previous launch's result first (its control block shares the pinned slot)
    TL_TRY(fix_resolve(c));
    constexpr size_t kSmemCap = 200 * 1024;
    // columns sharded: this rank stores a slice of every row; the warps still
    // build full-width rows in shared memory (words is the full width)
    const bool cols = col_split(R);
    const int64_t words = cols ? (R->dims[1] + 31) / 32 : R->bits_words, rows = R->bits_rows;
    const int64_t wpad = (words + 3) & ~int64_t(3);
    // one table entry per bit position of a row (padding bits included)
    const int64_t nodes = words * 32;
    if (fix_smem_per_warp(words) > kSmemCap || wpad * 32 >= INT32_MAX || E->nnz >= INT32_MAX) {
        if (cols) return fail(c, TL_ERR_UNSUPPORTED, "column-sharded closure: relation too wide");
        return TL_OK;
    }
    if (getenv("TL_CLOSURE_PER_SWEEP") && !cols) return TL_OK;
    if (c->world > 1 && !cols) {
        TL_TRY(comm_peer_setup(c));
        if (c->peer_state != 1) return TL_OK;
    }
    if (c->fix_coop < 0) {
        int coop = 0;
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->device);
        c->fix_coop = coop ? 1 : 0;
    }
    if (!c->fix_coop) {
        if (cols) return fail(c, TL_ERR_UNSUPPORTED, "column-sharded closure needs a cooperative launch");
        return TL_OK;
    }
    *handled = true;

    // successor table, rebuilt when the CSR or the row width changed
    const int32_t sentinel = (int32_t)(wpad * 32);
    if (E->succ_stamp != E->csr_stamp || E->succ_nodes != nodes || E->succ_sentinel != sentinel || !E->succ) {
        // the table, then one int4 whose first word is the graph's two-step flag
        if (nodes * 2 + 1 > E->succ_cap) {
            TL_CK(c, cudaStreamSynchronize(c->stream));
            cudaFree(E->succ);
            E->succ = nullptr;
            E->succ_cap = 0;
            TL_CK(c, cudaMalloc(&E->succ, (size_t)(nodes * 2 + 1) * sizeof(int4)));
            E->succ_cap = nodes * 2 + 1;
        }
        LaunchScope L(c, "closure_successor_table", (double)nodes * 32.0 + (double)E->nnz * 4.0);
        const int64_t blocks = std::min<int64_t>((nodes + 255) / 256, (int64_t)c->sm_count * 8);
        k_build_succ<<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, c->stream>>>(E->rowptr, E->colidx, E->csr_rows,
                                                                                   nodes, sentinel, E->succ);
        TL_TRY(L.done());
        E->succ_stamp = E->csr_stamp;
        E->succ_nodes = nodes;
        E->succ_sentinel = sentinel;
        E->two_hop_stamp = 0;
    }
    if (cols && E->two_hop_stamp != E->csr_stamp) {
        // the graph's two-step flag (columns sharded only: on a graph that is
        // its own closure the search is quadratic in the degrees)
        LaunchScope L(c, "closure_two_hop", (double)E->nnz * 8.0);
        int* two_hop = reinterpret_cast<int*>(E->succ + nodes * 2);
        TL_CK(c, cudaMemsetAsync(two_hop, 0, sizeof(int), c->stream));
        const int64_t rb = std::min<int64_t>((E->csr_rows + 255) / 256, (int64_t)c->sm_count * 8);
        k_two_hop<<<(unsigned)std::max<int64_t>(rb, 1), 256, 0, c->stream>>>(E->rowptr, E->colidx, E->csr_rows,
                                                                            two_hop);
        TL_TRY(L.done());
        E->two_hop_stamp = E->csr_stamp;
    }

    // fixpoint-long state: pending word per row (0: expand everything), then
    // the list of rows handed to teams in a sweep
    const size_t aux_need = std::max<size_t>((size_t)rows * 8, 4096);
    if (aux_need > c->aux_cap) {
        TL_CK(c, cudaStreamSynchronize(c->stream));
        cudaFree(c->aux);
        c->aux = nullptr;
        c->aux_cap = 0;
        TL_CK(c, cudaMalloc(&c->aux, aux_need));
        c->aux_cap = aux_need;
    }
    static_assert(kFixWarps * 32 <= 1024, "block size");
    // two control blocks, by launch parity: each launch empties the other
    if (!c->fix_state) {
        TL_CK(c, cudaMalloc(&c->fix_state, 2 * kFixStateBytes));
        TL_CK(c, cudaMemsetAsync(c->fix_state, 0, 2 * kFixStateBytes, c->stream));
        c->fix_slot = 0;
    }
    // rows that step(E) left unwritten start from E's successor lists; their
    // sweep ORs in closed rows (closed words of this launch's epoch)
    const bool lazy = R->bits_valid && R->lazy_src == E && R->lazy_stamp == E->csr_stamp;
    if (cols && !(lazy && words < (int64_t(1) << kClosedSpan) && R->bits_words % 4 == 0 && R->bits_words <= 1024))
        return fail(c, TL_ERR_UNSUPPORTED,
                    "column-sharded closure: the relation must start as step(Edge) right before the fixpoint, "
                    "with slices of a multiple of 128 columns up to 32768");
    const bool sharded = R->shard == TL_SHARD_ROWS && c->world > 1;
    const ShardedSweep mode = sharded_sweep_mode();
    const bool shortcut = lazy && words < (int64_t(1) << kClosedSpan) && !(sharded && mode == SWEEP_BFS);
    // row-sharded on several GPUs, the lazy sweep runs one of two ways; only
    // the changed word crosses GPUs in either.  Replicated: every rank closes
    // every row of the relation in a scratch copy (a row's shortcuts read
    // rows of every rank's share) and keeps its own rows.  Local: each rank
    // closes only its own rows and takes shortcuts through its own closed
    // rows, expanding the successors other ranks hold.
    const bool replicate = shortcut && sharded && mode == SWEEP_REPLICATE;
    // peer rows: the published buffer holds, per rank, the closed words and
    // then the rows of the largest share (every rank asks for the same size)
    bool peer_rows = shortcut && sharded && mode == SWEEP_PEER;
    const int64_t rows_max = (R->dims[0] + c->world - 1) / c->world;
    const size_t sym_closed_bytes = ((size_t)rows_max * 8 + 255) & ~size_t(255);
    if (peer_rows) {
        TL_TRY(comm_sym_setup(c, SYM_CLOSURE, sym_closed_bytes + (size_t)rows_max * words * 4));
        peer_rows = c->sym[SYM_CLOSURE].state == 1;   // the same on every rank
    }
    const int64_t dp_rows = replicate ? R->dims[0] : rows;
    uint32_t* dpR = R->bits;
    if (replicate) {
        void* ws = nullptr;
        TL_TRY(workspace(c, (size_t)std::max<int64_t>(dp_rows, 1) * words * 4, &ws, WS_FIXPOINT));
        dpR = static_cast<uint32_t*>(ws);
    }
    if (peer_rows) {
        // one epoch count per context, advanced on every rank at the same
        // launch; at its wrap the closed words are cleared on every rank
        // before any rank reads them again
        if (++c->sym_epoch > kEpochMax) {
            TL_CK(c, cudaMemsetAsync(c->sym[SYM_CLOSURE].own, 0, sym_closed_bytes, c->stream));
            TL_TRY(comm_barrier(c));
            c->sym_epoch = 1;
        }
    } else if (shortcut) {
        const size_t need = std::max<size_t>((size_t)dp_rows * 8, 256);
        if (need > c->fix_closed_cap) {
            TL_CK(c, cudaStreamSynchronize(c->stream));
            cudaFree(c->fix_closed);
            c->fix_closed = nullptr;
            c->fix_closed_cap = 0;
            TL_CK(c, cudaMalloc(&c->fix_closed, need));
            c->fix_closed_cap = need;
            c->fix_epoch = kEpochMax;   // forces the clear below
        }
        if (++c->fix_epoch > kEpochMax) {
            TL_CK(c, cudaMemsetAsync(c->fix_closed, 0, c->fix_closed_cap, c->stream));
            c->fix_epoch = 1;
        }
    }
    // the lazy sweep with shortcuts writes every row's pending word before any
    // later sweep reads it; otherwise every row starts fully pending
    if (rows > 0 && !shortcut) TL_CK(c, cudaMemsetAsync(c->aux, 0, (size_t)rows * 4, c->stream));

    // shape: with teams (TL_CLOSURE_TEAMS) the largest block that fits, so a
    // heavy row gets the most warps; otherwise the split that keeps the most
    // warps resident
    const size_t per_warp = fix_smem_per_warp(words);
    const bool teams = getenv("TL_CLOSURE_TEAMS") != nullptr;
    if (c->fix_shape_words != words || c->fix_shape_teams != (int)teams) {
        for (const void* fn : kFixVariants)
            TL_CK(c, cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap));
        int wpb = 1, per_sm = 0;
        for (int w = kFixWarps; w >= 1; w >>= 1) {
            if (per_warp * w > kSmemCap) continue;
            int b = 0;
            // one shape for every variant (and every rank computes the same)
            b = INT32_MAX;
            for (const void* fn : kFixVariants) {
                int bb = 0;
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bb, fn, 32 * w, per_warp * w);
                b = std::min(b, bb);
            }
            if (b < 1) continue;
            if (teams) { wpb = w; per_sm = b; break; }
            if (b * w > per_sm * wpb) { wpb = w; per_sm = b; }
        }
        if (per_sm < 1) return fail(c, TL_ERR_UNSUPPORTED, "closure fixpoint: no resident block fits");
        c->fix_shape_words = words;
        c->fix_shape_teams = (int)teams;
        c->fix_wpb = wpb;
        c->fix_per_sm = per_sm;
    }
    const int wpb = c->fix_wpb, per_sm = c->fix_per_sm;
    // a team's queue: every warp's space except the row and spill set it works on
    const int64_t team_words = (int64_t)wpb * (int64_t)(per_warp / 4) - (2 * wpad + 4);
    int64_t qt = 1;
    while (qt * 2 <= team_words) qt *= 2;
    int64_t grid = std::min<int64_t>((int64_t)c->sm_count * per_sm,
                                     std::max<int64_t>((std::max(rows, dp_rows) + wpb - 1) / wpb, 1));

    FixArgs a{};
    a.R = R->bits;
    a.rows = rows;
    a.words = words;
    a.wpad = wpad;
    a.succ = E->succ;
    a.rowptr = E->rowptr;
    a.colidx = E->colidx;
    a.e_rows = E->csr_rows;
    a.pending = (int32_t*)c->aux;
    a.heavy = (int32_t*)c->aux + rows;
    a.team = wpb;
    a.team_qmask = (unsigned)(qt - 1);
    a.team_budget = teams ? kHeavyBudget : 0;
    // the pinned mirror reads "no result" until the launch writes it (the
    // previous launch is resolved above, so nothing writes it meanwhile)
    FixState* const mirror = reinterpret_cast<FixState*>(c->h_flags + 32);
    mirror->sweeps = -1;
    a.host_out = reinterpret_cast<unsigned long long*>(mirror);
    FixState* const slots = static_cast<FixState*>(c->fix_state);
    a.st = reinterpret_cast<FixState*>(reinterpret_cast<char*>(slots) + c->fix_slot * kFixStateBytes);
    a.st_next = reinterpret_cast<FixState*>(reinterpret_cast<char*>(slots) + (1 - c->fix_slot) * kFixStateBytes);
    a.lazy = lazy ? 1 : 0;
    a.shortcut = shortcut ? 1 : 0;
    a.closed = static_cast<unsigned long long*>(c->fix_closed);
    a.epoch = c->fix_epoch;
    a.peer_dp = peer_rows ? 1 : 0;
    a.rw = cols ? R->bits_words : words;
    a.rw0 = cols ? (int64_t)R->col_rank * R->bits_words : 0;
    a.two_hop = reinterpret_cast<const int*>(E->succ + nodes * 2);
    c->fix_mode = cols ? 5 : !sharded ? 0 : peer_rows ? 1 : replicate ? 2 : shortcut ? 3 : 4;
    a.n_glob = R->dims[0];
    if (peer_rows) {
        for (int j = 0; j < c->world; ++j) {
            a.pclosed[j] = static_cast<unsigned long long*>(c->sym[SYM_CLOSURE].peer[j]);
            a.prows[j] = reinterpret_cast<uint32_t*>(static_cast<char*>(c->sym[SYM_CLOSURE].peer[j]) + sym_closed_bytes);
        }
        a.closed = a.pclosed[c->rank];
        a.epoch = c->sym_epoch;
        dpR = a.prows[c->rank];
    }
    a.dpR = dpR;
    a.dp_rows = dp_rows;
    a.dp_copy = replicate ? 1 : 0;
    // local row r is global row r * world + rank of a row-sharded relation
    a.row_stride = 1;
    a.row_offset = 0;
    if (R->shard == TL_SHARD_ROWS && c->world > 1) {
        a.row_stride = c->world;
        a.row_offset = c->rank;
    }
    // the copied row space holds every node's row at its own index
    a.dp_stride = a.dp_copy ? 1 : a.row_stride;
    a.dp_offset = a.dp_copy ? 0 : a.row_offset;
    a.max_sweeps = max_sweeps;
    a.nblocks = (unsigned)grid;
    a.world = c->world;
    a.rank = c->rank;
    // Replicated, every rank closes every row in the lazy sweep, so every
    // rank's changed word of that sweep is the same, and every row is closed
    // after it (each row's search runs to the end), so no rank finds a row
    // pending in a later sweep: the words need not cross GPUs, and each rank
    // runs its fixpoint without waiting for the others.  A relation whose
    // lazy sweep does not run (rows written before, or another scheme)
    // exchanges them.
    a.exchange = c->world > 1 && !(replicate && lazy) && !cols ? 1 : 0;
    for (int j = 0; j < kMaxPeers; ++j) a.slots[j] = c->peer_slots[j];
    a.token_base = c->world > 1 ? static_cast<unsigned long long*>(c->peer_own) + 2 * kMaxPeers : nullptr;
    a.timeout_ns = (unsigned long long)std::max(c->opts.comm_timeout_ms, 1000) * 1000000ull;

    const double sweep_bytes = (double)rows * a.rw * 8.0 + (double)nodes * 32.0;
    {
        LaunchScope L(c, "closure_fixpoint", sweep_bytes);
        void* args[] = {&a};
        // the work counters only in profiling runs that ask for them
        // (TL_CLOSURE_COUNTS): they cost the sweep a few per cent
        const bool count = c->prof && getenv("TL_CLOSURE_COUNTS") != nullptr;
        const void* fn = cols ? (count ? (const void*)k_closure_fix<false, true, true>
                                       : (const void*)k_closure_fix<false, false, true>)
                         : peer_rows ? (count ? (const void*)k_closure_fix<true, true, false>
                                              : (const void*)k_closure_fix<true, false, false>)
                                     : (count ? (const void*)k_closure_fix<false, true, false>
                                              : (const void*)k_closure_fix<false, false, false>);
        c->fix_counted = count;
        TL_CK(c, cudaLaunchCooperativeKernel(fn, dim3((unsigned)grid), dim3(32 * wpb), args,
                                             per_warp * wpb, c->stream));
        c->fix_slot ^= 1;   // the launch empties the other block before it ends
        TL_TRY(L.done());
    }
    // the control block comes back to pinned memory from the kernel itself;
    // it is read at once only when the caller needs the sweep count or when
    // profiling (the phase marks); otherwise when the context next syncs,
    // asks for the sweep count or launches another fixpoint
    if (!c->fix_event) TL_CK(c, cudaEventCreateWithFlags(&c->fix_event, cudaEventDisableTiming));
    TL_CK(c, cudaEventRecord(c->fix_event, c->stream));
    c->fix_pending = true;
    c->fix_last_state = a.st;
    c->fix_prof = c->prof;
    c->fix_sweep_bytes = sweep_bytes;
    R->lazy_src = nullptr;   // every row is written now (or the status of the launch says why not)
    *sweeps_out = -1;
    *changed_out = false;
    if (!need_now && !c->prof) return TL_OK;
    TL_TRY(fix_resolve(c));
    *sweeps_out = c->last_sweeps;
    *changed_out = c->fix_last_changed;
    return TL_OK;
}

tl_status fix_resolve(tl_ctx* c) {
    if (!c->fix_pending) return TL_OK;
    c->fix_pending = false;
    TL_CK(c, cudaEventSynchronize(c->fix_event));
    FixState h{};
    memcpy(&h, c->h_flags + 32, sizeof(FixState));
    // a launch that ended without settling its last sweep (a wait that ran
    // out) did not write the mirror: its control block holds the error
    if (h.sweeps < 0) TL_CK(c, cudaMemcpy(&h, c->fix_last_state, sizeof(FixState), cudaMemcpyDeviceToHost));
    // algorithmic bytes of the launch: every sweep reads and writes the rows
    if (c->fix_prof && !c->pending.empty() && c->pending.back().name == "closure_fixpoint")
        c->pending.back().bytes = c->fix_sweep_bytes * std::max(h.sweeps, 1);
    if (c->fix_prof) {
        // phases of the launch from the device's own clock: each sweep's row
        // work (until the last block is done) and its settling (barrier and,
        // on several GPUs, the wait for the other ranks)
        unsigned long long prev = h.t_start;
        auto add = [&](const char* what, int s, unsigned long long from, unsigned long long to) {
            char nm[64];
            snprintf(nm, sizeof nm, "closure_fixpoint.sweep%d_%s", s + 1, what);
            KStat& k = c->stats[nm];
            k.launches++;
            k.total_ms += (double)(to - from) / 1e6;
        };
        for (int s = 0; s < std::min(h.sweeps, kFixMarks); ++s) {
            // lone-warp rows (ends at the phase barrier), team rows, settling
            const unsigned long long rows_end = h.t_rows[s] ? h.t_rows[s] : h.t_team[s];
            if (!h.t_team[s] || !h.t_settled[s] || rows_end < prev || h.t_team[s] < rows_end ||
                h.t_settled[s] < h.t_team[s])
                break;
            add("rows", s, prev, rows_end);
            if (h.t_rows[s]) add("teams", s, rows_end, h.t_team[s]);
            add("settle", s, h.t_team[s], h.t_settled[s]);
            prev = h.t_settled[s];
        }
    }
    if (c->fix_prof && c->fix_counted) {
        // the lazy sweep's work and the way its shortcuts were read
        auto count = [&](const char* what, double v) {
            KStat& k = c->stats[std::string("closure_fixpoint.n_") + what];
            k.launches++;
            k.total_ms += v;   // a count, summed over launches
        };
        count("orl", h.n_or_local);    // closed rows of this rank ORed in
        count("orr", h.n_or_remote);   // closed rows of other ranks ORed in
        count("exp", h.n_expanded);    // nodes expanded
        count(c->fix_mode == 1 ? "peer" : c->fix_mode == 2 ? "repl" : c->fix_mode == 3 ? "local" :
              c->fix_mode == 4 ? "bfs" : c->fix_mode == 5 ? "cols" : "1gpu", 1);   // the scheme
    }
    c->last_sweeps = h.sweeps;
    c->fix_last_changed = h.last_changed != 0;
    if (h.err) {
        if (c->world > 1) c->peer_state = -1;   // ranks may disagree on the token count now
        return fail(c, h.err == 2 ? TL_ERR_COMM : TL_ERR_CUDA,
                    "closure fixpoint: %s wait ran out after %d sweeps", h.err == 2 ? "peer" : "grid barrier",
                    h.sweeps);
    }
    if (c->fix_last_changed) fail(c, TL_OK, "fixpoint stopped at the %d-sweep cap", h.sweeps);
    return TL_OK;
}

}  // namespace tl
