// Internal declarations of libtl_cuda (not part of the ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/tl_cuda.h"

namespace tl {

constexpr int kMaxVars = 12;
constexpr int kMaxPeers = 8;   // ranks of one box that exchange fixpoint flags over NVLink
// a buffer of one size on every rank, every rank's copy mapped into this process
struct SymBuf {
    int state = 0;                 // 0 none, 1 ready, -1 unavailable
    size_t bytes = 0;
    void* own = nullptr;
    void* peer[kMaxPeers] = {};
};
enum SymSlot { SYM_CLOSURE = 0, SYM_GNN = 1 };

// ----------------------------------------------------------------------------
// Device tensor with several interchangeable storages.
// ----------------------------------------------------------------------------
struct Tensor {
    std::string name;
    void* owner = nullptr;  // tl_ctx that created the tensor
    int rank = 0;
    int64_t dims[TL_MAX_RANK] = {0};
    int64_t strides[TL_MAX_RANK] = {0};
    int64_t total = 0;

    // Reference state: present in the codegen's tensor map (defined) and
    // holding calloc zeros that have not been written yet (zero).
    bool defined = false;
    bool zero = true;
    bool boolean = false;   // every value is 0 or 1
    bool is_sparse = false; // declared `sparse`
    int shard = TL_SHARD_NONE;
    // every dense value is >= 0: set only by a writer that knows it (an upload
    // that saw the values, a message-passing chain with relu per term over a
    // non-negative sparse operand); any other write clears it
    bool nonneg = false;
    int col_rank = 0, col_world = 1;   // TL_SHARD_COLS: this rank's slice of the columns

    // fp32 dense row-major (local rows only when sharded)
    float* dense = nullptr;
    int64_t dense_elems = 0;
    bool dense_valid = false;

    // bit rows of a rank-2 0/1 tensor (local rows only when sharded)
    uint32_t* bits = nullptr;
    int64_t bits_words = 0;   // words per row
    int64_t bits_rows = 0;
    bool bits_valid = false;

    // CSR of a rank-2 tensor (local rows only when sharded)
    int64_t* rowptr = nullptr;
    int32_t* colidx = nullptr;
    float* vals = nullptr;
    int64_t nnz = 0, csr_cap = 0, csr_rows = 0;
    bool csr_valid = false;
    bool csr_nonneg = false;  // every stored value >= 0
    bool csr_pos = false;     // every stored value > 0 (each entry is an edge of step(E))
    bool csr_ones = false;    // every stored value == 1

    // CSC (predecessor lists) of a rank-2 tensor, global
    int64_t* colptr = nullptr;
    int32_t* rowidx = nullptr;
    int64_t csc_cap = 0;
    bool csc_valid = false;

    // bit rows not written yet: row r holds step(lazy_src) row r * world + rank
    // (row r when not sharded); ensure_bits writes them, the one-launch
    // closure fixpoint builds them in shared memory instead
    Tensor* lazy_src = nullptr;
    uint64_t lazy_stamp = 0;

    // CSR generation: changes whenever the CSR contents are rebuilt
    uint64_t csr_stamp = 0;
    // successor table of the one-launch closure fixpoint, built from the CSR
    int4* succ = nullptr;
    int64_t succ_cap = 0;       // int4 entries
    uint64_t succ_stamp = 0;    // csr_stamp it was built from (0: none)
    int64_t succ_nodes = 0;     // node count and sentinel it was built for
    int32_t succ_sentinel = 0;
    uint64_t two_hop_stamp = 0; // csr_stamp of the two-step flag after the table (0: none)

    int64_t local_rows(int rank_, int world) const {
        if (shard != TL_SHARD_ROWS || world <= 1 || this->rank < 1) return this->rank >= 1 ? dims[0] : 1;
        return dims[0] > rank_ ? (dims[0] - rank_ + world - 1) / world : 0;
    }
};

// the relation's columns are split over several slices (TL_SHARD_COLS with
// more than one slice); one slice behaves as an unsharded tensor
inline bool col_split(const Tensor* t) { return t->shard == TL_SHARD_COLS && t->col_world > 1; }

// A captured CUDA graph of one program run (tl_program_run): replayed while
// the statements and the context's host state at the start of a run (tensor
// storages, flags, workspaces) are the same as when it was captured.
struct GraphEntry {
    const void* stmts_at = nullptr;    // the caller's statement array
    std::vector<uint8_t> stmts;        // and its bytes when captured
    std::vector<uint8_t> begin, end;   // host state before / after the run
    std::vector<uint8_t> last_begin;   // state seen by the last eager run
    void* exec = nullptr;              // cudaGraphExec_t
    int64_t launches = 0;
    bool failed = false;               // capture not possible: always run eagerly
    uint64_t used = 0;
};

struct KStat {
    int64_t launches = 0;
    double total_ms = 0, bytes = 0, flops = 0;
};

struct PendingEvent {
    std::string name;
    cudaEvent_t a, b;
    double bytes, flops;
};

// A global of the backward-chaining queries (llvm.zig:222-264): a tensor named
// by a constant-index query (compute: it has a memo table and is evaluated by
// recursion) or an equation-defined tensor such a tensor's equations read.
struct BqHost {
    std::string name;
    int rank = 0;
    int64_t dims[TL_MAX_RANK] = {0};
    bool compute = false;
    std::vector<int> eqs;      // statement indices of its equations, program order
    bool detached = false;     // a `sparse` re-declaration replaced the forward tensor
    float* snap = nullptr;     // device copy of what it held then (nullptr: zeros)
};

}  // namespace tl

struct tl_tensor : tl::Tensor {};

struct tl_ctx {
    tl_init_opts opts{};
    int device = 0;
    int sm_count = 148;
    cudaStream_t stream = nullptr;
    std::unordered_map<std::string, int64_t> domains;
    std::unordered_map<std::string, std::vector<int64_t>> maxdims;
    std::map<std::string, std::unique_ptr<tl_tensor>> tensors;
    std::string err;
    std::string query_out;
    // tensors whose sign a later step / comparison / relu gradient tests: their
    // GEMMs run at fp32-class accuracy (3xTF32) so no sign flips against f64
    std::vector<std::string> sign_sensitive;
    int32_t last_sweeps = 0;
    int64_t launches = 0;
    int rank = 0, world = 1;
    void* comm = nullptr;  // ncclComm_t

    // device scratch
    void* ws[4] = {nullptr, nullptr, nullptr, nullptr};   // one buffer per tl::WsSlot
    size_t ws_cap[4] = {0, 0, 0, 0};
    int* d_flags = nullptr;     // [0..63] changed / error words
    void* aux = nullptr;        // state kept across the sweeps of one fixpoint
    size_t aux_cap = 0;
    int* h_flags = nullptr;     // pinned mirror
    void* fix_state = nullptr;  // control blocks of the one-launch closure fixpoint (two, by launch parity)
    int fix_slot = 0;           // the block the next launch uses
    void* fix_last_state = nullptr;   // the block the last launch used
    // closed words of the lazy closure sweep: one per local row, tagged with
    // the launch's epoch so no launch has to clear them
    void* fix_closed = nullptr;
    size_t fix_closed_cap = 0;
    uint32_t fix_epoch = 0;
    // launch shape of the closure fixpoint, computed once per row width
    int fix_coop = -1;
    int64_t fix_shape_words = -1;
    int fix_shape_teams = -1, fix_wpb = 0, fix_per_sm = 0;
    // a tensor-core GEMM was given the device error word since it was last read
    bool flags_armed = false;
    // a closure fixpoint whose control block has not been read yet (fix_resolve)
    bool fix_pending = false, fix_prof = false, fix_last_changed = false;
    double fix_sweep_bytes = 0;
    cudaEvent_t fix_event = nullptr;
    // globals of this run's constant-index queries
    std::vector<tl::BqHost> bq;
    // captured program runs (most recently used last)
    std::vector<tl::GraphEntry> graphs;
    uint64_t graph_clock = 0;
    // the equation of tl_program_run whose step(E) result may stay unwritten
    // until the closure fixpoint that reads it next
    const tl_equation* lazy_eq = nullptr;

    // multi-GPU fixpoint flags: every rank's slot array mapped into this
    // process (peer memory over NVLink), set up on first use
    int peer_state = 0;                              // 0 not tried, 1 ready, -1 unavailable
    unsigned long long* peer_slots[tl::kMaxPeers] = {};
    void* peer_own = nullptr;                        // this rank's slot array
    // buffers of one size on every rank, every rank's copy mapped into this
    // process (comm_sym_setup): [SYM_CLOSURE] the closed words and rows the
    // sharded closure publishes for the other ranks' peer loads,
    // [SYM_GNN] the gathered per-node transform the GNN layers fan out to
    tl::SymBuf sym[2];
    uint32_t sym_epoch = 0;                          // closed-word epoch of the sharded lazy sweep
    // fanned-out GNN layers: their count, and per writing rank the tiles it
    // has signalled into this rank's counters so far
    uint64_t gnn_layers = 0;
    unsigned long long gnn_expect[tl::kMaxPeers] = {};
    bool fix_counted = false;   // the last fixpoint launch counted its lazy sweep's work
    int fix_mode = 0;   // the last fixpoint's lazy sweep: 0 one GPU, 1 peer rows, 2 replicate, 3 local, 4 bfs

    // profiling
    bool prof = false;
    std::vector<tl::PendingEvent> pending;
    std::vector<cudaEvent_t> event_pool;
    std::map<std::string, tl::KStat> stats;
};

namespace tl {

// error helpers --------------------------------------------------------------
tl_status fail(tl_ctx* c, tl_status code, const char* fmt, ...)
    __attribute__((format(printf, 3, 4)));
tl_status cuda_fail(tl_ctx* c, cudaError_t e, const char* what);

#define TL_CK(ctx, call)                                                         \
    do {                                                                         \
        cudaError_t _e = (call);                                                 \
        if (_e != cudaSuccess) return ::tl::cuda_fail((ctx), _e, #call);         \
    } while (0)
#define TL_TRY(expr)                                                             \
    do {                                                                         \
        tl_status _s = (expr);                                                   \
        if (_s != TL_OK) return _s;                                              \
    } while (0)

// launch accounting: every kernel launch of the runtime goes through these
void launch_begin(tl_ctx* c, const char* name, double bytes, double flops, cudaEvent_t* ev);
tl_status launch_end(tl_ctx* c, cudaEvent_t* ev);
struct LaunchScope {
    tl_ctx* c;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    // own = false: timed like a kernel of this library but not counted as one
    // (a library collective)
    LaunchScope(tl_ctx* c_, const char* name, double bytes = 0, double flops = 0, bool own = true) : c(c_) {
        launch_begin(c, name, bytes, flops, ev);
        if (!own) c->launches--;
    }
    tl_status done() { return launch_end(c, ev); }
};

// device-side error words (pipeline timeouts); syncs the stream
tl_status check_device_flags(tl_ctx* c);

// scratch workspaces (grown on demand, never shrunk); users that can be
// nested (a message-passing step holding its transform while the GEMM that
// produces it stages operand copies) take different slots
enum WsSlot { WS_GENERAL = 0, WS_GEMM = 1, WS_CHAIN = 2, WS_FIXPOINT = 3 };
tl_status workspace(tl_ctx* c, size_t bytes, void** out, int slot = WS_GENERAL);
tl_status ensure_dense(tl_ctx* c, Tensor* t);
tl_status ensure_bits(tl_ctx* c, Tensor* t);
tl_status ensure_csr(tl_ctx* c, Tensor* t);
tl_status alloc_bits_public(tl_ctx* c, Tensor* t);
tl_status alloc_dense_public(tl_ctx* c, Tensor* t);
void mark_written_dense(Tensor* t);
void mark_written_bits(Tensor* t);
const float* read_ptr(tl_ctx* c, Tensor* t, tl_status* st);

// ----------------------------------------------------------------------------
// Kernel entry points (k_*.cu)
// ----------------------------------------------------------------------------
struct RefPlan {
    const float* ptr;     // nullptr → every element reads 0.0
    int64_t total;
    int32_t nidx;         // indices applied (min(rank, #indices))
    int32_t kind[TL_MAX_RANK];
    int32_t var[TL_MAX_RANK];
    int64_t val[TL_MAX_RANK];
    int64_t stride[TL_MAX_RANK];
    const float* virt[TL_MAX_RANK];
    int64_t virt_total[TL_MAX_RANK];
};

struct CodeOp {
    int32_t op, arg, arg2, _pad;
    double value;
};

struct GenericPlan {
    int32_t n_vars, n_free;
    int64_t sizes[kMaxVars];
    int64_t n_out;               // product of free sizes
    int64_t n_inner;             // product of contracted sizes
    int32_t n_refs, n_code;
    RefPlan refs[TL_MAX_REFS];
    CodeOp code[TL_MAX_CODE];
    float* lhs;
    int64_t lhs_total;
    int32_t n_lhs_terms;
    int32_t lhs_var[TL_MAX_RANK];
    int64_t lhs_div[TL_MAX_RANK];
    int64_t lhs_stride[TL_MAX_RANK];
    int32_t accum;
    int32_t has_contraction;
    int32_t old_zero;            // LHS holds logical zeros: start from 0.0
    int32_t atomic;              // several threads may hit one LHS element
    int32_t recursive;           // fixpoint sweep: report increases in *changed
    int32_t virt_pos_var;
    int32_t aligned;             // element-wise, every operand shaped and indexed like the LHS
};

tl_status launch_generic(tl_ctx* c, const GenericPlan& p, int* d_changed);

// rowwise softmax / lnorm over a strided row set
struct RowPlan {
    const float* in;
    float* out;
    int64_t in_total, out_total;
    int64_t rows, len;
    int32_t n_outer;
    int64_t outer_size[TL_MAX_RANK];
    int64_t outer_in_stride[TL_MAX_RANK];
    int64_t outer_out_stride[TL_MAX_RANK];
    int64_t in_sn, out_sn;
    int32_t lnorm;
};
tl_status launch_rowwise(tl_ctx* c, const RowPlan& p);

// dense GEMM C[m,n] (+)= sum_k f(A[m,k] B[k,n] * scale), arbitrary strides
struct GemmPlan {
    int64_t M, N, K;
    const float* A; int64_t sam, sak;
    const float* B; int64_t sbk, sbn;
    float* C; int64_t scm, scn;
    float scale;
    int32_t beta;        // 1: add into C, 0: overwrite
    int32_t relu_term;   // per-term relu
    int32_t a_nonneg, b_nonneg;   // per-term relu: A (B) has no negative value, so one K segment suffices
    int32_t epi_relu;    // additionally write relu(C) into D (fused next equation)
    int32_t precise;     // fp32-class accuracy (3xTF32) on the tensor cores
    float* D; int64_t sdm, sdn;
    // fan-out (an all-gather fused into the epilogue): every output tile is
    // also stored, with C's strides, at fan[q] in rank q's memory (peer
    // stores over NVLink; null for this rank), and each CTA then adds 1 to
    // fan_cnt[q] with release at system scope.  Needs the tensor-core path
    // with its TMA-store epilogue, no split K, beta = 0 and no fused relu
    // (gemm_fan_tiles counts its tiles).
    float* fan[kMaxPeers];
    unsigned long long* fan_cnt[kMaxPeers];
    int32_t fan_n;
};
tl_status launch_gemm(tl_ctx* c, const GemmPlan& p);
int64_t gemm_fan_tiles(int64_t M, int64_t N);
bool tcgen05_available(tl_ctx* c);
// S = scale Q K^T, A = softmax over the rows of S, O = A V: row-major fp32,
// Q, K, V and O with 64 columns, n_q and n_k multiples of 128 (k_gemm.cu)
struct AttnPlan {
    const float *Q, *K, *V;
    float *S, *A, *O;
    int64_t n_q, n_k;
    float scale;
};
tl_status launch_attention(tl_ctx* c, const AttnPlan& p);
// A small-batch head, H = [relu per term](s1 X W1), Z = s2 H W2, Y = softmax
// over the columns of Z: row-major fp32, b <= kHeadMaxRows rows, o <=
// kHeadMaxCols columns of Z (k_head.cu)
constexpr int kHeadMaxRows = 64, kHeadMaxCols = 32;
struct HeadPlan {
    const float *X, *W1, *W2;
    float *H, *Z, *Y;
    int64_t b, i, h, o;
    int relu_term;
    float sgn1, mag1;     // relu per term: relu(s1 t) = |s1| relu(sign(s1) t); else mag1 = s1
    float s2;
    // set by the launch: partial H of ks chunks of kc contracted indices
    float* hpart;
    int ks;
    int64_t kc;
};
tl_status launch_head(tl_ctx* c, HeadPlan p);

// Before a SpMM reads rows other ranks fanned out into P: per writing rank
// the count its tiles must have reached in this rank's counter array (0:
// no wait), read with acquire at system scope, bounded by timeout_ns.
struct SpWait {
    const unsigned long long* cnt;
    unsigned long long need[kMaxPeers];
    unsigned long long timeout_ns;
};
// Copies len floats at src (this rank's block of a gathered tensor) to
// dst[q] on every other rank q (peer memory; null for this rank), then adds
// fan_push_blocks() to each cnt[q] (release at system scope)
tl_status launch_fan_push(tl_ctx* c, const float* src, int64_t len, float* const* dst,
                          unsigned long long* const* cnt);
int64_t fan_push_blocks();
// CSR SpMM out[v, j] (+)= sum_e val[e] * P[col[e], j]; P has p_rows rows
tl_status launch_spmm(tl_ctx* c, int64_t rows, const int64_t* rowptr, const int32_t* colidx,
                      const float* vals, const float* P, int64_t p_rows, int64_t ldp, int64_t f, float* out,
                      int64_t ldo, int beta, int relu_out, int col_shard_world, int64_t col_local_rows,
                      const SpWait* wait = nullptr);

// closure
tl_status launch_csr_to_dense(tl_ctx* c, Tensor* t);
tl_status launch_csr_to_bits(tl_ctx* c, Tensor* t, Tensor* out);
tl_status launch_dense_to_bits(tl_ctx* c, Tensor* t);
tl_status launch_bits_to_dense(tl_ctx* c, Tensor* t);
tl_status launch_dense_to_csr(tl_ctx* c, Tensor* t);
tl_status launch_closure_right(tl_ctx* c, Tensor* R, Tensor* E, int* d_changed, int sweep);
// t's CSR built on the device from COO entries (k_csr.cu); *handled = false
// when the host build has to take it
tl_status csr_from_coo_gpu(tl_ctx* c, Tensor* t, int64_t nnz, const int64_t* rows, const int64_t* cols,
                           const double* vals, int64_t lrows, bool* handled);
tl_status launch_closure_left(tl_ctx* c, Tensor* R, Tensor* E, int* d_changed);
// every right-form sweep of a fixpoint in one cooperative launch; *handled is
// false when the shapes or the context do not allow it (the caller then runs
// one launch per sweep)
// One-launch closure fixpoint.  need_now: the sweep count is wanted at once;
// otherwise, on one GPU, it may stay pending (sweeps_out = -1) until
// fix_resolve, which the next sync, sweep-count query or fixpoint calls.
tl_status launch_closure_fixpoint(tl_ctx* c, Tensor* R, Tensor* E, int max_sweeps, bool need_now, int* sweeps_out,
                                  bool* changed_out, bool* handled);
tl_status fix_resolve(tl_ctx* c);
uint64_t next_csr_stamp();
// multi-GPU fixpoint flags over peer memory (comm.cpp); collective over all ranks
tl_status comm_peer_setup(tl_ctx* c);
// tensor map for tile::gather4 row gathers of a row-major fp32 matrix (k_gemm.cu)
bool make_gather_map(CUtensorMap* map, const float* base, int64_t cols, int64_t rows, int64_t row_stride);
void comm_peer_release(tl_ctx* c);
// the symmetric buffer (collective; every rank passes the same size): on
// return sym[slot].state is 1 on every rank or -1 on every rank
tl_status comm_sym_setup(tl_ctx* c, int slot, size_t bytes);
void comm_sym_release(tl_ctx* c, int slot);
tl_status comm_barrier(tl_ctx* c);
// captured program runs (lower.cpp)
void release_graphs(tl_ctx* c);

// elementwise gradient rules
// overwrite: out holds logical zeros that are not in memory yet (no memset
// needed when the rule covers every element, see grad_elem_covers)
tl_status launch_grad_elem(tl_ctx* c, int rule, float* out, int64_t out_total, const float* up,
                           int64_t up_total, const float* x, int64_t x_total, const float* y,
                           int64_t y_total, int overwrite = 0);
bool grad_elem_covers(int rule, int64_t out_total, int64_t up_total, int64_t x_total);
tl_status launch_grad_softmax(tl_ctx* c, float* out, int64_t out_total, const float* up,
                              int64_t up_total, const float* y, int64_t y_total);
tl_status launch_fill(tl_ctx* c, float* p, int64_t n, float v);
// out[0] = (old_zero ? 0 : out[0]) + sum a[i] b[i] (f64), one launch
tl_status launch_dot_scalar(tl_ctx* c, const float* a, const float* b, int64_t n, float* out, int old_zero);
tl_status launch_set1(tl_ctx* c, float* p, int64_t off, const GenericPlan& plan);

// communication (comm.cpp)
tl_status comm_init(tl_ctx* c);
tl_status comm_destroy(tl_ctx* c);
tl_status comm_allreduce_max_int(tl_ctx* c, int* d_buf, int count);
tl_status comm_allgather(tl_ctx* c, const void* d_send, void* d_recv, size_t bytes_per_rank);

// autodiff (autodiff.cpp)
tl_status run_backward(tl_ctx* c, const char* loss, const char (*params)[TL_NAME_LEN], int np,
                       const tl_equation* eqs, int n_eqs);

// equation lowering (runtime.cpp)
Tensor* find(tl_ctx* c, const std::string& name);
Tensor* find_defined(tl_ctx* c, const std::string& name);
tl_status allocate_tensor(tl_ctx* c, const char* name, const tl_index* idx, int n, Tensor** out);
tl_status new_tensor(tl_ctx* c, const std::string& name, int rank, const int64_t* dims, Tensor** out);
int64_t domain_size(tl_ctx* c, const char* name);
int64_t index_extent(tl_ctx* c, const tl_index* ix);

// backward-chaining queries (k_query.cu)
tl_status bq_prepare(tl_ctx* c, const tl_statement* s, int n);
tl_status bq_detach(tl_ctx* c, const char* name);
tl_status bq_run(tl_ctx* c, const tl_statement* s, int n, std::vector<double>* out);
void bq_release(tl_ctx* c);

}  // namespace tl
