// Backward-chaining queries: `T[0, 5]?` with any constant index.
//
// The reference compiles such a query into a recursive function per queried
// tensor with a memo table and a computed flag per element (backward.zig:
// 53-220): the function marks its element computed with value 0, then
// evaluates the tensor's equations in program order, each one either directly
// or as a sum over its contracted indices, folds each into the result with
// the equation's accumulation operator and stores the running result in the
// memo.  A reference to a queried tensor inside an equation is a recursive
// call (which returns the memo value at once for an element already computed,
// including one still in progress further up the stack); any other tensor is
// a load from the global the backward infrastructure allocated for it.
//
// That recursion is a chain of dependent scalar steps, so it runs as one GPU
// thread interpreting a compact plan of the program: every frame (the
// element, the equation, the loop counters, the partial sums and the
// expression stack) lives in an HBM frame array, so recursion depth is bounded
// by the plan's capacity and not by a thread stack.  All backward queries of a
// program run in one launch, in statement order, sharing the memo tables the
// way the reference's globals do.  The interpreter counts the steps it takes
// and stops with an error status past a step budget or a time limit on
// %globaltimer (defaults 2^31 steps and 4 s; TL_BQ_MAX_STEPS and TL_BQ_MAX_MS
// set them per run), so a deep query cannot hold the GPU for minutes; it has
// no waits.
//
// Arithmetic is f64 with the reference's operation order and no contraction
// (__dadd_rn and friends); forward tensors are read from their fp32 device
// storage.
#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

#include "tl_internal.h"

namespace tl {
namespace {

constexpr int kBqVars = 16;
constexpr int64_t kBqMaxFrames = int64_t(1) << 20;
constexpr int64_t kBqMaxSteps = int64_t(1) << 31;
constexpr int64_t kBqMaxMs = 4000;
constexpr int64_t kBqClockEvery = 1024;   // steps between reads of %globaltimer
constexpr double kBqMaxMemoBytes = 16.0 * (1 << 30);

// one index of a tensor reference: a constant, a parameter of the function
// (an LHS index name) or a loop variable of the contracted sum
enum : int32_t { SRC_CONST = 0, SRC_PARAM = 1, SRC_LOOP = 2 };

struct BqRef {
    int32_t global;   // plan global read or called; -1: a tensor the reference's map lacks (reads 0.0)
    int32_t nidx;
    int32_t src[TL_MAX_RANK];
    int64_t val[TL_MAX_RANK];
};

struct BqEq {
    int32_t accum, n_code, n_vars, _pad;
    int64_t n_iter;             // product of the loop extents (1 with no loops)
    int64_t size[kBqVars];      // loop extents, the first loop outermost
    BqRef ref[TL_MAX_REFS];
    int32_t op[TL_MAX_CODE];
    int32_t arg[TL_MAX_CODE];
    double value[TL_MAX_CODE];
};

struct BqGlobal {
    int32_t rank, compute, eq_first, eq_count;
    int64_t strides[TL_MAX_RANK];
    int64_t total;
    const float* data;          // forward values (compute == 0); nullptr reads zeros
    int64_t data_total;
    int64_t memo_base;          // compute == 1: first element in the memo tables
};

struct BqQuery {
    int32_t global, _pad;
    int64_t idx[TL_MAX_RANK];
};

struct BqFrame {
    int32_t g, e, pc, sp;
    int64_t off, it;
    int64_t idx[TL_MAX_RANK];
    int64_t lv[kBqVars];
    double result, accum;
    double vals[TL_MAX_CODE];
};

struct BqArgs {
    const BqGlobal* g;
    const BqEq* eq;
    const BqQuery* q;
    int32_t n_q;
    BqFrame* frames;
    int64_t max_frames;
    double* memo;
    uint8_t* done;
    double* out;
    int* status;                // 0 ok, 1 frame capacity, 2 step budget, 3 time limit
    int64_t max_steps;
    unsigned long long max_ns;  // time limit of the launch
};

__device__ __forceinline__ unsigned long long bq_now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// genBackwardExpr's nonlinearities (backward.zig:419-457): sigmoid has no
// temperature here, and every other function is the identity.
__device__ double bq_nl(int f, double x) {
    switch (f) {
    case TL_NL_STEP: return x > 0.0 ? 1.0 : 0.0;
    case TL_NL_RELU: return x > 0.0 ? x : 0.0;
    case TL_NL_SIGMOID: return __ddiv_rn(1.0, __dadd_rn(1.0, exp(-x)));
    case TL_NL_EXP: return exp(x);
    case TL_NL_LOG: return log(x);
    case TL_NL_SQRT: return sqrt(x);
    case TL_NL_ABS: return fabs(x);
    case TL_NL_SIN: return sin(x);
    case TL_NL_COS: return cos(x);
    case TL_NL_TANH: {
        const double e = exp(__dmul_rn(x, 2.0));
        return __ddiv_rn(__dsub_rn(e, 1.0), __dadd_rn(e, 1.0));
    }
    default: return __dadd_rn(0.0, x);
    }
}

__device__ void bq_frame_init(BqFrame* F, int g, int64_t off, const int64_t* iv, int rank) {
    F->g = g;
    F->e = 0;
    F->pc = 0;
    F->sp = 0;
    F->off = off;
    F->it = 0;
    for (int k = 0; k < rank; ++k) F->idx[k] = iv[k];
    for (int j = 0; j < kBqVars; ++j) F->lv[j] = 0;
    F->result = 0.0;
    F->accum = 0.0;
}

// Fold an equation's value into the running result (genComputeFunction,
// backward.zig:179-205), store it in the memo and move to the next equation.
__device__ void bq_finish(const BqArgs& a, BqFrame* F, const BqEq& E, double ev) {
    double r = F->result;
    switch (E.accum) {
    case TL_ACC_ADD: r = __dadd_rn(r, ev); break;
    case TL_ACC_MAX: r = ev > r ? ev : r; break;
    case TL_ACC_MIN: r = ev < r ? ev : r; break;
    case TL_ACC_MUL: r = __dmul_rn(r, ev); break;
    default: r = __dadd_rn(0.0, ev); break;
    }
    F->result = r;
    a.memo[a.g[F->g].memo_base + F->off] = r;
    F->e++;
    F->pc = 0;
    F->sp = 0;
    F->it = 0;
    F->accum = 0.0;
    for (int j = 0; j < kBqVars; ++j) F->lv[j] = 0;
}

__global__ void __launch_bounds__(32) k_backward_query(BqArgs a) {
    if (threadIdx.x != 0) return;
    int status = 0;
    int64_t steps = 0;
    const unsigned long long t0 = bq_now_ns();
    for (int q = 0; q < a.n_q && status == 0; ++q) {
        const BqQuery& Q = a.q[q];
        const BqGlobal& QG = a.g[Q.global];
        double ret = 0.0;
        int64_t depth = -1;
        {
            int64_t off = 0;
            for (int k = 0; k < QG.rank; ++k) off += Q.idx[k] * QG.strides[k];
            if (off >= 0 && off < QG.total) {
                if (a.done[QG.memo_base + off]) {
                    ret = a.memo[QG.memo_base + off];
                } else {
                    a.done[QG.memo_base + off] = 1;
                    a.memo[QG.memo_base + off] = 0.0;
                    depth = 0;
                    bq_frame_init(a.frames, Q.global, off, Q.idx, QG.rank);
                }
            }
        }
        while (depth >= 0) {
            BqFrame* F = a.frames + depth;
            const BqGlobal& G = a.g[F->g];
            if (F->e >= G.eq_count) {   // the function returns its result
                ret = F->result;
                if (--depth >= 0) {
                    BqFrame* C = a.frames + depth;
                    C->vals[C->sp++] = ret;
                }
                continue;
            }
            const BqEq& E = a.eq[G.eq_first + F->e];
            if (E.n_iter == 0) {        // an empty loop nest sums to 0
                bq_finish(a, F, E, 0.0);
                continue;
            }
            if (F->pc >= E.n_code) {    // one term evaluated
                const double v = F->sp > 0 ? F->vals[F->sp - 1] : 0.0;
                if (E.n_vars == 0) {
                    bq_finish(a, F, E, v);
                    continue;
                }
                F->accum = __dadd_rn(F->accum, v);
                if (++F->it < E.n_iter) {
                    int j = E.n_vars - 1;
                    while (j >= 0 && ++F->lv[j] >= E.size[j]) F->lv[j--] = 0;
                    F->pc = 0;
                    F->sp = 0;
                } else {
                    bq_finish(a, F, E, F->accum);
                }
                continue;
            }
            if (++steps > a.max_steps) { status = 2; break; }
            if (steps % kBqClockEvery == 0 && bq_now_ns() - t0 > a.max_ns) { status = 3; break; }
            const int pc = F->pc++;
            const int op = E.op[pc];
            switch (op) {
            case TL_OP_REF: {
                const BqRef& R = E.ref[E.arg[pc]];
                if (R.global < 0) { F->vals[F->sp++] = 0.0; break; }
                int64_t iv[TL_MAX_RANK];
                for (int k = 0; k < R.nidx; ++k)
                    iv[k] = R.src[k] == SRC_CONST ? R.val[k] : R.src[k] == SRC_PARAM ? F->idx[R.val[k]] : F->lv[R.val[k]];
                const BqGlobal& T = a.g[R.global];
                int64_t off = 0;
                const int nk = R.nidx < T.rank ? R.nidx : T.rank;
                for (int k = 0; k < nk; ++k) off += iv[k] * T.strides[k];
                if (off < 0 || off >= T.total) { F->vals[F->sp++] = 0.0; break; }
                if (!T.compute) {
                    F->vals[F->sp++] = (T.data && off < T.data_total) ? (double)T.data[off] : 0.0;
                    break;
                }
                uint8_t* d = a.done + T.memo_base + off;
                if (*d) { F->vals[F->sp++] = a.memo[T.memo_base + off]; break; }
                if (depth + 1 >= a.max_frames) { status = 1; break; }
                *d = 1;
                a.memo[T.memo_base + off] = 0.0;
                ++depth;
                bq_frame_init(a.frames + depth, R.global, off, iv, T.rank);
                break;
            }
            case TL_OP_LIT: F->vals[F->sp++] = E.value[pc]; break;
            case TL_OP_PROD: {
                const int n = E.arg[pc];
                double acc = F->vals[F->sp - n];
                for (int k = 1; k < n; ++k) acc = __dmul_rn(acc, F->vals[F->sp - n + k]);
                F->sp -= n;
                F->vals[F->sp++] = acc;
                break;
            }
            case TL_OP_NEG: F->vals[F->sp - 1] = -F->vals[F->sp - 1]; break;
            case TL_OP_NOT: F->vals[F->sp - 1] = F->vals[F->sp - 1] == 0.0 ? 1.0 : 0.0; break;
            case TL_OP_NL: F->vals[F->sp - 1] = bq_nl(E.arg[pc], F->vals[F->sp - 1]); break;
            default: {
                const double b = F->vals[--F->sp];
                const double x = F->vals[F->sp - 1];
                double r;
                switch (op) {
                case TL_OP_SUB: r = __dsub_rn(x, b); break;
                case TL_OP_MUL: r = __dmul_rn(x, b); break;
                case TL_OP_DIV: r = __ddiv_rn(x, b); break;
                default: r = __dadd_rn(x, b); break;   // add, and every other binary op
                }
                F->vals[F->sp - 1] = r;
            }
            }
            if (status) break;
        }
        a.out[q] = ret;
    }
    a.status[0] = status;
}

bool is_backward_query(const tl_ref& q) {
    for (int k = 0; k < q.rank; ++k)
        if (q.idx[k].kind == TL_IX_CONST) return true;
    return false;
}

BqHost* find_global(tl_ctx* c, const char* name) {
    for (BqHost& g : c->bq)
        if (g.name == name) return &g;
    return nullptr;
}

int64_t total_of(const BqHost& g) {
    int64_t s = 1;
    for (int k = 0; k < g.rank; ++k) s *= g.dims[k];
    return s;
}

}  // namespace

// The globals of llvm.zig:222-264: the tensors named by constant-index
// queries (each with its equations, in program order, from genBackwardInfra,
// backward.zig:78-97), then every equation-defined tensor their right-hand
// sides read.  Dims follow allocateTensorGlobal (tensor.zig:157-220), which
// is the forward allocation rule.
tl_status bq_prepare(tl_ctx* c, const tl_statement* s, int n) {
    bq_release(c);
    std::vector<std::string> queried, deps;
    auto has = [](const std::vector<std::string>& v, const char* x) {
        for (const std::string& y : v)
            if (y == x) return true;
        return false;
    };
    for (int i = 0; i < n; ++i)
        if (s[i].kind == TL_STMT_QUERY && is_backward_query(s[i].sparse) && !has(queried, s[i].name))
            queried.push_back(s[i].name);
    if (queried.empty()) return TL_OK;
    auto add = [&](const tl_ref& lhs) -> BqHost* {
        if (BqHost* g = find_global(c, lhs.tensor)) return g;
        BqHost g;
        g.name = lhs.tensor;
        auto it = c->maxdims.find(lhs.tensor);
        if (it != c->maxdims.end()) {
            g.rank = (int)it->second.size();
            for (int k = 0; k < g.rank && k < TL_MAX_RANK; ++k) g.dims[k] = it->second[k];
        } else {
            g.rank = lhs.rank;
            for (int k = 0; k < lhs.rank && k < TL_MAX_RANK; ++k)
                g.dims[k] = lhs.idx[k].kind == TL_IX_NORMALIZE ? 10 : index_extent(c, &lhs.idx[k]);
        }
        if (g.rank == 0) { g.rank = 1; g.dims[0] = 1; }
        c->bq.push_back(g);
        return &c->bq.back();
    };
    for (int i = 0; i < n; ++i) {
        if (s[i].kind != TL_STMT_EQUATION || !has(queried, s[i].eq.lhs.tensor)) continue;
        BqHost* g = add(s[i].eq.lhs);
        g->compute = true;
        g->eqs.push_back(i);
        for (int r = 0; r < s[i].eq.n_refs && r < TL_MAX_REFS; ++r)
            if (!has(deps, s[i].eq.refs[r].tensor)) deps.push_back(s[i].eq.refs[r].tensor);
    }
    for (int i = 0; i < n; ++i)
        if (s[i].kind == TL_STMT_EQUATION && has(deps, s[i].eq.lhs.tensor) && !has(queried, s[i].eq.lhs.tensor))
            add(s[i].eq.lhs);
    for (const BqHost& g : c->bq)
        if (g.rank > TL_MAX_RANK) return fail(c, TL_ERR_UNSUPPORTED, "%s: rank above %d", g.name.c_str(), TL_MAX_RANK);
    return TL_OK;
}

// genSparseDecl allocates unconditionally (llvm.zig:482-516): after a `sparse`
// declaration of a global, the forward program writes a new buffer and the
// compute functions keep reading the global with what it held at that point.
tl_status bq_detach(tl_ctx* c, const char* name) {
    BqHost* g = find_global(c, name);
    if (!g || g->compute || g->detached) return TL_OK;
    g->detached = true;
    Tensor* t = find_defined(c, name);
    if (!t || t->zero || t->total != total_of(*g)) return TL_OK;   // the global is still zeros
    if (t->shard == TL_SHARD_ROWS && c->world > 1)
        return fail(c, TL_ERR_UNSUPPORTED, "%s: backward query over a row-sharded tensor", name);
    TL_TRY(ensure_dense(c, t));
    TL_CK(c, cudaMalloc(&g->snap, (size_t)t->total * sizeof(float)));
    TL_CK(c, cudaMemcpyAsync(g->snap, t->dense, (size_t)t->total * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    return TL_OK;
}

void bq_release(tl_ctx* c) {
    for (BqHost& g : c->bq) cudaFree(g.snap);
    c->bq.clear();
}

namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Check a right-hand side's postfix program against the stack it needs, so
// the interpreter's stack accesses stay inside a frame.
bool code_is_valid(const tl_equation& eq) {
    int sp = 0;
    for (int i = 0; i < eq.n_code; ++i) {
        const tl_instr& in = eq.code[i];
        switch (in.op) {
        case TL_OP_REF:
            if (in.arg < 0 || in.arg >= eq.n_refs) return false;
            ++sp;
            break;
        case TL_OP_LIT: ++sp; break;
        case TL_OP_PROD:
            if (in.arg < 1 || in.arg > sp) return false;
            sp -= in.arg - 1;
            break;
        case TL_OP_NEG: case TL_OP_NOT: case TL_OP_NL:
            if (sp < 1) return false;
            break;
        default:
            if (in.op < TL_OP_ADD || in.op > TL_OP_OR || sp < 2) return false;
            --sp;
        }
    }
    return true;
}

}  // namespace

// Run every constant-index query of the program (genBackwardQuery,
// backward.zig:568-600) in one launch; out receives one value per such query,
// in statement order.
tl_status bq_run(tl_ctx* c, const tl_statement* s, int n, std::vector<double>* out) {
    out->clear();
    std::vector<BqQuery> queries;
    for (int i = 0; i < n; ++i) {
        if (s[i].kind != TL_STMT_QUERY || !is_backward_query(s[i].sparse)) continue;
        const BqHost* g = find_global(c, s[i].name);
        if (!g || !g->compute)
            return fail(c, TL_ERR_UNSUPPORTED, "%s: a constant-index query needs an equation defining it", s[i].name);
        if (s[i].sparse.rank != g->rank)
            return fail(c, TL_ERR_UNSUPPORTED, "%s: query has %d indices, tensor has %d", s[i].name, s[i].sparse.rank,
                        g->rank);
        BqQuery q{};
        q.global = (int32_t)(g - c->bq.data());
        for (int k = 0; k < g->rank; ++k)
            q.idx[k] = s[i].sparse.idx[k].kind == TL_IX_CONST ? s[i].sparse.idx[k].value : 0;
        queries.push_back(q);
    }
    if (queries.empty()) return TL_OK;

    std::vector<BqGlobal> gs(c->bq.size());
    std::vector<BqEq> eqs;
    int64_t memo_elems = 0;
    for (size_t gi = 0; gi < c->bq.size(); ++gi) {
        const BqHost& h = c->bq[gi];
        BqGlobal& g = gs[gi];
        memset(&g, 0, sizeof g);
        g.rank = h.rank;
        g.compute = h.compute ? 1 : 0;
        int64_t st = 1;
        for (int k = h.rank - 1; k >= 0; --k) { g.strides[k] = st; st *= h.dims[k]; }
        g.total = st;
        if (h.compute) {
            g.memo_base = memo_elems;
            memo_elems += g.total;
            continue;
        }
        if (h.detached) {
            g.data = h.snap;
            g.data_total = h.snap ? g.total : 0;
            continue;
        }
        Tensor* t = find_defined(c, h.name);
        if (!t || t->zero) continue;
        if (t->shard == TL_SHARD_ROWS && c->world > 1)
            return fail(c, TL_ERR_UNSUPPORTED, "%s: backward query over a row-sharded tensor", h.name.c_str());
        TL_TRY(ensure_dense(c, t));
        g.data = t->dense;
        g.data_total = t->total;
    }
    if ((double)memo_elems * 9.0 > kBqMaxMemoBytes)
        return fail(c, TL_ERR_TOO_LARGE, "backward-query memo tables of %lld elements", (long long)memo_elems);
    for (size_t gi = 0; gi < c->bq.size(); ++gi) {
        const BqHost& h = c->bq[gi];
        if (!h.compute) continue;
        gs[gi].eq_first = (int32_t)eqs.size();
        gs[gi].eq_count = (int32_t)h.eqs.size();
        for (int si : h.eqs) {
            const tl_equation& eq = s[si].eq;
            bool ok = eq.n_code >= 0 && eq.n_code <= TL_MAX_CODE && eq.n_refs >= 0 && eq.n_refs <= TL_MAX_REFS &&
                      eq.lhs.rank >= 0;
            for (int r = 0; ok && r < eq.n_refs; ++r) ok = eq.refs[r].rank >= 0 && eq.refs[r].rank <= TL_MAX_RANK;
            if (!ok || !code_is_valid(eq))
                return fail(c, TL_ERR_INVALID, "%s: malformed right-hand side", h.name.c_str());
            if (eq.lhs.rank > h.rank)
                return fail(c, TL_ERR_UNSUPPORTED, "%s: equation with %d indices on a rank-%d tensor", h.name.c_str(),
                            eq.lhs.rank, h.rank);
            BqEq E;
            memset(&E, 0, sizeof E);
            E.accum = eq.accum;
            E.n_code = eq.n_code;
            // genBackwardEquation (backward.zig:222-250): LHS names bind the
            // parameters (a repeated name binds its last position) ...
            auto param_of = [&](const char* nm) {
                int p = -1;
                for (int k = 0; k < eq.lhs.rank; ++k)
                    if (eq.lhs.idx[k].kind == TL_IX_NAME && !strcmp(eq.lhs.idx[k].name, nm)) p = k;
                return p;
            };
            // ... and every other right-hand-side name is a contracted loop
            std::vector<std::string> loops;
            for (int r = 0; r < eq.n_refs; ++r)
                for (int k = 0; k < eq.refs[r].rank; ++k) {
                    const tl_index& ix = eq.refs[r].idx[k];
                    if (ix.kind != TL_IX_NAME || param_of(ix.name) >= 0) continue;
                    bool seen = false;
                    for (const std::string& l : loops) seen = seen || l == ix.name;
                    if (seen) continue;
                    if ((int)loops.size() >= kBqVars)
                        return fail(c, TL_ERR_UNSUPPORTED, "%s: more than %d contracted indices", h.name.c_str(), kBqVars);
                    E.size[loops.size()] = domain_size(c, ix.name);
                    loops.push_back(ix.name);
                }
            E.n_vars = (int32_t)loops.size();
            double iters = 1.0;
            E.n_iter = 1;
            for (int j = 0; j < E.n_vars; ++j) {
                if (E.size[j] <= 0) { E.n_iter = 0; break; }
                iters *= (double)E.size[j];
                E.n_iter *= E.size[j];
            }
            if (iters > 1e12) return fail(c, TL_ERR_TOO_LARGE, "%s: contracted loop of %.3g terms", h.name.c_str(), iters);
            for (int r = 0; r < eq.n_refs; ++r) {
                const tl_ref& ref = eq.refs[r];
                BqRef& R = E.ref[r];
                const BqHost* tg = find_global(c, ref.tensor);
                R.global = tg ? (int32_t)(tg - c->bq.data()) : -1;
                R.nidx = ref.rank;
                if (tg && tg->compute && ref.rank != tg->rank)
                    return fail(c, TL_ERR_UNSUPPORTED, "%s: called with %d indices, has %d", ref.tensor, ref.rank, tg->rank);
                // genBackwardTensorAccess (backward.zig:505-525): names, then
                // constants; every other index form is 0
                for (int k = 0; k < ref.rank; ++k) {
                    const tl_index& ix = ref.idx[k];
                    R.src[k] = SRC_CONST;
                    R.val[k] = 0;
                    if (ix.kind == TL_IX_CONST) {
                        R.val[k] = ix.value;
                    } else if (ix.kind == TL_IX_NAME) {
                        const int p = param_of(ix.name);
                        if (p >= 0) {
                            R.src[k] = SRC_PARAM;
                            R.val[k] = p;
                        } else {
                            for (int j = 0; j < E.n_vars; ++j)
                                if (loops[j] == ix.name) { R.src[k] = SRC_LOOP; R.val[k] = j; }
                        }
                    }
                }
            }
            for (int i = 0; i < eq.n_code; ++i) {
                E.op[i] = eq.code[i].op;
                E.arg[i] = eq.code[i].arg;
                E.value[i] = eq.code[i].value;
            }
            eqs.push_back(E);
        }
    }

    const int64_t frames = std::min<int64_t>(memo_elems + 2, kBqMaxFrames);
    size_t off_g = 0;
    size_t off_e = align256(off_g + gs.size() * sizeof(BqGlobal));
    size_t off_q = align256(off_e + eqs.size() * sizeof(BqEq));
    size_t off_o = align256(off_q + queries.size() * sizeof(BqQuery));
    size_t off_st = align256(off_o + queries.size() * sizeof(double));
    size_t off_done = align256(off_st + 16);
    size_t off_memo = align256(off_done + (size_t)memo_elems);
    size_t off_f = align256(off_memo + (size_t)memo_elems * sizeof(double));
    size_t bytes = off_f + (size_t)frames * sizeof(BqFrame);
    void* ws = nullptr;
    TL_TRY(workspace(c, bytes, &ws));
    char* base = (char*)ws;
    std::vector<char> plan(off_q + queries.size() * sizeof(BqQuery));
    memcpy(plan.data() + off_g, gs.data(), gs.size() * sizeof(BqGlobal));
    memcpy(plan.data() + off_e, eqs.data(), eqs.size() * sizeof(BqEq));
    memcpy(plan.data() + off_q, queries.data(), queries.size() * sizeof(BqQuery));
    TL_CK(c, cudaMemcpyAsync(base, plan.data(), plan.size(), cudaMemcpyHostToDevice, c->stream));
    TL_CK(c, cudaMemsetAsync(base + off_st, 0, 16, c->stream));
    TL_CK(c, cudaMemsetAsync(base + off_done, 0, (size_t)memo_elems, c->stream));
    BqArgs a;
    a.g = (const BqGlobal*)(base + off_g);
    a.eq = (const BqEq*)(base + off_e);
    a.q = (const BqQuery*)(base + off_q);
    a.n_q = (int32_t)queries.size();
    a.frames = (BqFrame*)(base + off_f);
    a.max_frames = frames;
    a.memo = (double*)(base + off_memo);
    a.done = (uint8_t*)(base + off_done);
    a.out = (double*)(base + off_o);
    a.status = (int*)(base + off_st);
    // budgets of the launch (a test makes them tiny to see the error status)
    const char* ms_env = getenv("TL_BQ_MAX_STEPS");
    const char* mt_env = getenv("TL_BQ_MAX_MS");
    const long long max_steps = ms_env ? atoll(ms_env) : 0;
    const long long max_ms = mt_env ? atoll(mt_env) : 0;
    a.max_steps = max_steps > 0 ? (int64_t)max_steps : kBqMaxSteps;
    a.max_ns = (unsigned long long)(max_ms > 0 ? max_ms : kBqMaxMs) * 1000000ull;
    {
        LaunchScope L(c, "backward_query");
        k_backward_query<<<1, 32, 0, c->stream>>>(a);
        TL_TRY(L.done());
    }
    std::vector<char> back(off_st + sizeof(int) - off_o);
    TL_CK(c, cudaMemcpyAsync(back.data(), base + off_o, back.size(), cudaMemcpyDeviceToHost, c->stream));
    TL_CK(c, cudaStreamSynchronize(c->stream));
    int status = 0;
    memcpy(&status, back.data() + (off_st - off_o), sizeof(int));
    if (status == 1) return fail(c, TL_ERR_TOO_LARGE, "backward query deeper than %lld frames", (long long)frames);
    if (status == 2) return fail(c, TL_ERR_TOO_LARGE, "backward query above %lld steps", (long long)a.max_steps);
    if (status == 3)
        return fail(c, TL_ERR_TOO_LARGE, "backward query ran past %.0f ms", (double)a.max_ns / 1e6);
    out->resize(queries.size());
    memcpy(out->data(), back.data(), queries.size() * sizeof(double));
    return TL_OK;
}

}  // namespace tl
