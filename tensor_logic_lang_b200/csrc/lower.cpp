// Lowering of statements to kernels, the fixpoint driver and the program
// schedule.
//
// Reference anchors (Zollicoff/tensor_logic_lang):
//   LLVMCodegen.generate       src/codegen/llvm.zig:131-336
//   genEquation                src/codegen/llvm.zig:357-459
//   collectExprIndices         src/codegen/expr.zig:303-359
//   genEinsumLoops / accum     src/codegen/einsum.zig:20-278
//   genSoftmax / genLayerNorm  src/codegen/softmax.zig:19-267, layernorm.zig:25-348
//   genFixpointLoop            src/codegen/fixpoint.zig:21-297
//   genSparseDecl              src/codegen/llvm.zig:482-516
//   genSave / genLoad          src/codegen/llvm.zig:565-633 (paths without quotes)
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "tl_internal.h"

using namespace tl;

namespace {

// ----------------------------------------------------------------------------
// Index analysis (llvm.zig:383-455)
// ----------------------------------------------------------------------------
struct Var {
    std::string name;
    int64_t size;
    bool contracted;
};

struct Analysis {
    std::vector<Var> vars;       // free (LHS order) then contracted
    int n_free = 0;
    bool has_contraction = false;
    bool scalar = false;         // no index at all → genScalarAssign
    // LHS address terms: (var, divisor) paired with strides in emission order
    int n_lhs_terms = 0;
    int lhs_var[TL_MAX_RANK];
    int64_t lhs_div[TL_MAX_RANK];
    int64_t avg_div = 1;
};

std::string primed(const char* n) { return std::string(n) + "'"; }

int var_index(const std::vector<Var>& v, const std::string& n) {
    for (size_t i = 0; i < v.size(); ++i) if (v[i].name == n) return (int)i;
    return -1;
}

// collectExprIndices: RHS index variables in expression order.
void collect_rhs(tl_ctx* c, const tl_equation* eq, std::vector<Var>& all) {
    for (int r = 0; r < eq->n_refs; ++r) {
        const tl_ref* ref = &eq->refs[r];
        for (int k = 0; k < ref->rank; ++k) {
            const tl_index* ix = &ref->idx[k];
            std::string nm;
            int64_t size;
            switch (ix->kind) {
            case TL_IX_NAME: case TL_IX_ADD: case TL_IX_SUB: case TL_IX_DIV:
                nm = ix->name; size = domain_size(c, ix->name); break;
            case TL_IX_PRIMED: nm = primed(ix->name); size = domain_size(c, ix->name); break;
            case TL_IX_SLICE: {
                char b[64];
                snprintf(b, sizeof b, "_slice_%lld_%lld", (long long)ix->value, (long long)ix->value2);
                nm = b;
                size = ix->value2 > ix->value ? ix->value2 - ix->value : 1;
                break;
            }
            default: continue;
            }
            int at = var_index(all, nm);
            if (at < 0) all.push_back({nm, size, false});
            else all[at].size = size;
        }
    }
}

tl_status analyze(tl_ctx* c, const tl_equation* eq, bool recursive, Analysis* a) {
    std::vector<Var> all;
    std::vector<std::string> lhs_set;
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        std::string nm;
        bool ok = ix->kind == TL_IX_NAME || ix->kind == TL_IX_NORMALIZE;
        if (!recursive) ok = ok || ix->kind == TL_IX_DIV || ix->kind == TL_IX_PRIMED;
        if (!ok) continue;
        nm = ix->kind == TL_IX_PRIMED ? primed(ix->name) : std::string(ix->name);
        lhs_set.push_back(nm);
        int at = var_index(all, nm);
        if (at < 0) all.push_back({nm, domain_size(c, ix->name), false});
        else all[at].size = domain_size(c, ix->name);
    }
    collect_rhs(c, eq, all);
    if (all.empty()) { a->scalar = true; return TL_OK; }
    // free variables: LHS order (the fixpoint also loops the normalize index)
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        std::string nm;
        if (ix->kind == TL_IX_NAME || ix->kind == TL_IX_DIV) nm = ix->name;
        else if (ix->kind == TL_IX_PRIMED && !recursive) nm = primed(ix->name);
        else if (ix->kind == TL_IX_NORMALIZE && recursive) nm = ix->name;
        else continue;
        if (recursive && ix->kind == TL_IX_DIV) continue;
        if (var_index(a->vars, nm) >= 0 && recursive) continue;
        int at = var_index(all, nm);
        a->vars.push_back({nm, at >= 0 ? all[at].size : 10, false});
    }
    a->n_free = (int)a->vars.size();
    for (auto& v : all) {
        if (std::find(lhs_set.begin(), lhs_set.end(), v.name) != lhs_set.end()) continue;
        a->vars.push_back({v.name, v.size, true});
        a->has_contraction = true;
    }
    if ((int)a->vars.size() > kMaxVars)
        return fail(c, TL_ERR_UNSUPPORTED, "%s: more than %d index variables", eq->lhs.tensor, kMaxVars);
    // LHS address terms (einsum.zig:87-123; fixpoint.zig:212-225)
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        std::string nm;
        int64_t div = 1;
        if (recursive) {
            if (ix->kind != TL_IX_NAME && ix->kind != TL_IX_NORMALIZE) continue;
            nm = ix->name;
        } else if (ix->kind == TL_IX_NAME) nm = ix->name;
        else if (ix->kind == TL_IX_PRIMED) nm = primed(ix->name);
        else if (ix->kind == TL_IX_DIV) { nm = ix->name; div = ix->value; a->avg_div *= ix->value; }
        else continue;
        int at = var_index(a->vars, nm);
        if (at < 0) continue;
        if (div <= 0) return fail(c, TL_ERR_INVALID, "division index by %lld", (long long)div);
        a->lhs_var[a->n_lhs_terms] = at;
        a->lhs_div[a->n_lhs_terms++] = div;
    }
    return TL_OK;
}

// Every LHS element is addressed by exactly one free tuple.
bool lhs_bijective(const Analysis& a, const Tensor* lhs) {
    if (a.n_lhs_terms != lhs->rank || a.n_lhs_terms != a.n_free) return false;
    bool seen[kMaxVars] = {false};
    for (int t = 0; t < a.n_lhs_terms; ++t) {
        int v = a.lhs_var[t];
        if (seen[v] || a.lhs_div[t] != 1 || a.vars[v].size != lhs->dims[t]) return false;
        seen[v] = true;
    }
    return true;
}

// One thread per LHS element is safe (no two tuples share an element).
bool lhs_injective(const Analysis& a, const Tensor* lhs) {
    bool seen[kMaxVars] = {false};
    int covered = 0;
    for (int t = 0; t < a.n_lhs_terms && t < lhs->rank; ++t) {
        int v = a.lhs_var[t];
        if (seen[v] || a.lhs_div[t] != 1 || a.vars[v].size > lhs->dims[t]) return false;
        seen[v] = true;
        covered++;
    }
    return covered == a.n_free;
}

// ----------------------------------------------------------------------------
// Generic per-term loop nest on the GPU (einsum.zig:20-254 semantics)
// ----------------------------------------------------------------------------
tl_status build_refs(tl_ctx* c, const tl_equation* eq, const Analysis& a, GenericPlan* p) {
    p->n_refs = eq->n_refs;
    p->virt_pos_var = a.vars.empty() ? -1 : 0;
    for (int r = 0; r < eq->n_refs; ++r) {
        const tl_ref* ref = &eq->refs[r];
        RefPlan& rp = p->refs[r];
        memset(&rp, 0, sizeof rp);
        Tensor* t = find_defined(c, ref->tensor);
        tl_status st;
        if (t && t->shard == TL_SHARD_ROWS && c->world > 1)
            return fail(c, TL_ERR_UNSUPPORTED, "%s: row-sharded tensor in a generic equation", ref->tensor);
        rp.ptr = read_ptr(c, t, &st);
        TL_TRY(st);
        rp.total = t ? t->total : 0;
        int nidx = t ? std::min(ref->rank, t->rank) : 0;
        rp.nidx = nidx;
        for (int k = 0; k < nidx; ++k) {
            const tl_index* ix = &ref->idx[k];
            rp.kind[k] = ix->kind;
            rp.val[k] = ix->value;
            rp.stride[k] = t->strides[k];
            rp.var[k] = -1;
            switch (ix->kind) {
            case TL_IX_NAME: case TL_IX_ADD: case TL_IX_SUB: case TL_IX_DIV:
                rp.var[k] = var_index(a.vars, ix->name);
                if (ix->kind == TL_IX_DIV && ix->value <= 0) return fail(c, TL_ERR_INVALID, "division index by 0");
                break;
            case TL_IX_PRIMED: rp.var[k] = var_index(a.vars, primed(ix->name)); break;
            case TL_IX_VIRTUAL: {
                Tensor* vt = find_defined(c, ix->name);
                rp.virt[k] = read_ptr(c, vt, &st);
                TL_TRY(st);
                rp.virt_total[k] = vt ? vt->total : 0;
                break;
            }
            default: break;
            }
        }
    }
    p->n_code = eq->n_code;
    for (int i = 0; i < eq->n_code; ++i) {
        p->code[i].op = eq->code[i].op;
        p->code[i].arg = eq->code[i].arg;
        p->code[i].arg2 = eq->code[i].arg2;
        p->code[i].value = eq->code[i].value;
    }
    return TL_OK;
}

tl_status validate_code(tl_ctx* c, const tl_equation* eq) {
    if (eq->n_refs < 0 || eq->n_refs > TL_MAX_REFS || eq->n_code < 0 || eq->n_code > TL_MAX_CODE ||
        eq->lhs.rank < 0 || eq->lhs.rank > TL_MAX_RANK)
        return fail(c, TL_ERR_INVALID, "malformed equation descriptor");
    int sp = 0;
    for (int i = 0; i < eq->n_code; ++i) {
        const tl_instr* in = &eq->code[i];
        switch (in->op) {
        case TL_OP_REF:
            if (in->arg < 0 || in->arg >= eq->n_refs) return fail(c, TL_ERR_INVALID, "bad ref operand");
            sp++; break;
        case TL_OP_LIT: sp++; break;
        case TL_OP_PROD:
            if (in->arg < 1 || in->arg > sp) return fail(c, TL_ERR_INVALID, "bad product arity");
            sp -= in->arg - 1; break;
        case TL_OP_NEG: case TL_OP_NOT: case TL_OP_NL:
            if (sp < 1) return fail(c, TL_ERR_INVALID, "stack underflow");
            break;
        default:
            if (in->op < TL_OP_ADD || in->op > TL_OP_OR) return fail(c, TL_ERR_INVALID, "bad opcode %d", in->op);
            if (sp < 2) return fail(c, TL_ERR_INVALID, "stack underflow");
            sp--;
        }
        if (sp > 16) return fail(c, TL_ERR_UNSUPPORTED, "expression deeper than 16");
    }
    if (eq->n_code > 0 && sp != 1) return fail(c, TL_ERR_INVALID, "expression leaves %d values", sp);
    for (int r = 0; r < eq->n_refs; ++r)
        if (eq->refs[r].rank < 0 || eq->refs[r].rank > TL_MAX_RANK) return fail(c, TL_ERR_INVALID, "bad ref rank");
    return TL_OK;
}

bool root_is_boolean(const tl_equation* eq) {
    if (eq->n_code == 0) return false;
    const tl_instr* r = &eq->code[eq->n_code - 1];
    if (r->op == TL_OP_NL && r->arg == TL_NL_STEP) return true;
    if (r->op >= TL_OP_GT && r->op <= TL_OP_NE) return true;
    if (r->op == TL_OP_NOT) return true;
    if (r->op == TL_OP_LIT) return r->value == 0.0 || r->value == 1.0;
    return false;
}

// ----------------------------------------------------------------------------
// Pattern: C[m,n] (+)= [relu] (A[.,.] B[.,.] [* or / literal])  → GEMM
// ----------------------------------------------------------------------------
struct GemmMatch {
    int ref_a, ref_b;
    float scale;
    bool relu_term;
};

// Recognise REF a, REF b, [LIT s, MUL|DIV], PROD 2 [, NL relu] in any of the
// forms the parser produces for `A B`, `A B / s`, `A (B * s)`, `relu(A B)`.
bool match_product2(const tl_equation* eq, GemmMatch* m) {
    const tl_instr* c = eq->code;
    int n = eq->n_code;
    m->relu_term = false;
    m->scale = 1.0f;
    if (n >= 1 && c[n - 1].op == TL_OP_NL && c[n - 1].arg == TL_NL_RELU) { m->relu_term = true; n--; }
    if (eq->n_refs != 2) return false;
    // REF a REF b PROD
    if (n == 3 && c[0].op == TL_OP_REF && c[1].op == TL_OP_REF && c[2].op == TL_OP_PROD && c[2].arg == 2) {
        m->ref_a = c[0].arg; m->ref_b = c[1].arg; return true;
    }
    // REF a REF b LIT s (MUL|DIV) PROD     — A (B op s)
    if (n == 5 && c[0].op == TL_OP_REF && c[1].op == TL_OP_REF && c[2].op == TL_OP_LIT &&
        (c[3].op == TL_OP_MUL || c[3].op == TL_OP_DIV) && c[4].op == TL_OP_PROD && c[4].arg == 2) {
        if (c[3].op == TL_OP_DIV && c[2].value == 0.0) return false;
        m->ref_a = c[0].arg; m->ref_b = c[1].arg;
        m->scale = (float)(c[3].op == TL_OP_MUL ? c[2].value : 1.0 / c[2].value);
        // (B / s) with s a power of two is exact in fp32, else rounding differs ≤ 1 ulp
        return true;
    }
    // REF a LIT s (MUL|DIV) REF b PROD    — (A op s) B
    if (n == 5 && c[0].op == TL_OP_REF && c[1].op == TL_OP_LIT && (c[2].op == TL_OP_MUL || c[2].op == TL_OP_DIV) &&
        c[3].op == TL_OP_REF && c[4].op == TL_OP_PROD && c[4].arg == 2) {
        if (c[2].op == TL_OP_DIV && c[1].value == 0.0) return false;
        m->ref_a = c[0].arg; m->ref_b = c[3].arg;
        m->scale = (float)(c[2].op == TL_OP_MUL ? c[1].value : 1.0 / c[1].value);
        return true;
    }
    return false;
}

int ref_var(const tl_ref* r, int k, const Analysis& a) {
    if (k >= r->rank || r->idx[k].kind != TL_IX_NAME) return -2;
    return var_index(a.vars, r->idx[k].name);
}

// Tensor-shaped check: every index a plain name whose var size equals the dim.
bool plain_2d(const tl_ref* r, const Tensor* t, const Analysis& a) {
    if (!t || r->rank != 2 || t->rank != 2) return false;
    for (int k = 0; k < 2; ++k) {
        int v = ref_var(r, k, a);
        if (v < 0 || a.vars[v].size != t->dims[k]) return false;
    }
    return true;
}

// A full contraction of two same-shaped tensors into a scalar,
// `L = A[i,j] B[i,j]` (einsum.zig:20-254 with every index contracted): one
// f64 dot product over the contiguous elements.  `=` with a contraction adds
// into the old value, as `+=` does (einsum.zig:201-212).
tl_status try_dot(tl_ctx* c, const tl_equation* eq, const Analysis& a, Tensor* lhs, bool* done) {
    *done = false;
    if (eq->accum != TL_ACC_ASSIGN && eq->accum != TL_ACC_ADD) return TL_OK;
    if (a.n_free != 0 || !a.has_contraction || lhs->total != 1 || eq->n_refs != 2 || eq->n_code != 3) return TL_OK;
    if (eq->code[0].op != TL_OP_REF || eq->code[1].op != TL_OP_REF || eq->code[2].op != TL_OP_PROD ||
        eq->code[2].arg != 2 || eq->code[0].arg != 0 || eq->code[1].arg != 1)
        return TL_OK;
    Tensor* A = find_defined(c, eq->refs[0].tensor);
    Tensor* B = find_defined(c, eq->refs[1].tensor);
    if (!A || !B || A->rank < 1 || A->rank != B->rank || eq->refs[0].rank != A->rank || eq->refs[1].rank != B->rank)
        return TL_OK;
    if ((int)a.vars.size() != A->rank) return TL_OK;   // every variable is one of the tensors' axes
    for (int k = 0; k < A->rank; ++k) {
        const int v = ref_var(&eq->refs[0], k, a);
        if (v < 0 || v != ref_var(&eq->refs[1], k, a) || a.vars[v].size != A->dims[k] || A->dims[k] != B->dims[k])
            return TL_OK;
    }
    if ((A->shard == TL_SHARD_ROWS || B->shard == TL_SHARD_ROWS) && c->world > 1) return TL_OK;
    tl_status st;
    const float* ap = read_ptr(c, A, &st);
    TL_TRY(st);
    const float* bp = read_ptr(c, B, &st);
    TL_TRY(st);
    if (!ap || !bp) return TL_OK;   // an operand of zeros: the generic path keeps the old value
    const bool old_zero = lhs->zero;
    if (old_zero) TL_TRY(alloc_dense_public(c, lhs));
    else TL_TRY(ensure_dense(c, lhs));
    TL_TRY(launch_dot_scalar(c, ap, bp, A->total, lhs->dense, old_zero ? 1 : 0));
    mark_written_dense(lhs);
    lhs->boolean = false;
    *done = true;
    return TL_OK;
}

tl_status try_gemm(tl_ctx* c, const tl_equation* eq, const Analysis& a, Tensor* lhs, bool* done,
                   Tensor* fuse_relu = nullptr, bool* fused = nullptr) {
    *done = false;
    if (fused) *fused = false;
    if (eq->accum != TL_ACC_ASSIGN && eq->accum != TL_ACC_ADD) return TL_OK;
    if (a.n_free != 2 || (int)a.vars.size() != 3 || !a.has_contraction) return TL_OK;
    GemmMatch m;
    if (!match_product2(eq, &m)) return TL_OK;
    const tl_ref* ra = &eq->refs[m.ref_a];
    const tl_ref* rb = &eq->refs[m.ref_b];
    Tensor* ta = find_defined(c, ra->tensor);
    Tensor* tb = find_defined(c, rb->tensor);
    if (!lhs_bijective(a, lhs)) return TL_OK;
    if (!plain_2d(ra, ta, a) || !plain_2d(rb, tb, a) || !plain_2d(&eq->lhs, lhs, a)) {
        // an operand that was never defined reads 0.0: the product adds nothing
        if ((!ta || !tb) && lhs_bijective(a, lhs)) {
            // `=`/`+=` of zero terms leave the LHS as it was
            *done = true;
        }
        return TL_OK;
    }
    for (Tensor* t : {ta, tb, lhs})
        if (t->shard == TL_SHARD_ROWS && c->world > 1) return TL_OK;
    const int vm = a.lhs_var[0], vn = a.lhs_var[1], vk = a.n_free;  // contracted var is last
    // orient operands: A holds (m,k), B holds (k,n)
    auto holds = [&](const tl_ref* r, int v1, int v2) {
        int x = ref_var(r, 0, a), y = ref_var(r, 1, a);
        return (x == v1 && y == v2) || (x == v2 && y == v1);
    };
    const tl_ref *rA = ra, *rB = rb;
    Tensor *tA = ta, *tB = tb;
    if (!(holds(rA, vm, vk) && holds(rB, vk, vn))) {
        if (holds(rb, vm, vk) && holds(ra, vk, vn)) { std::swap(rA, rB); std::swap(tA, tB); }
        else return TL_OK;
    }
    GemmPlan g;
    memset(&g, 0, sizeof g);
    g.M = a.vars[vm].size; g.N = a.vars[vn].size; g.K = a.vars[vk].size;
    tl_status st;
    g.A = read_ptr(c, tA, &st); TL_TRY(st);
    g.B = read_ptr(c, tB, &st); TL_TRY(st);
    if (!g.A || !g.B) { *done = true; return TL_OK; }  // a zero operand adds 0.0 terms
    int am = ref_var(rA, 0, a) == vm ? 0 : 1;
    g.sam = tA->strides[am]; g.sak = tA->strides[1 - am];
    int bk = ref_var(rB, 0, a) == vk ? 0 : 1;
    g.sbk = tB->strides[bk]; g.sbn = tB->strides[1 - bk];
    g.scale = m.scale;
    g.relu_term = m.relu_term ? 1 : 0;
    g.precise = std::find(c->sign_sensitive.begin(), c->sign_sensitive.end(), lhs->name) != c->sign_sensitive.end();
    g.beta = lhs->zero ? 0 : 1;
    if (g.beta) TL_TRY(ensure_dense(c, lhs));
    else TL_TRY(alloc_dense_public(c, lhs));
    g.C = lhs->dense;
    // LHS [m,n] or [n,m]
    g.scm = lhs->strides[0]; g.scn = lhs->strides[1];
    if (a.lhs_var[0] != vm) std::swap(g.scm, g.scn);
    // the next statement `H = relu(LHS)` (same shape, same index order) is
    // written by this GEMM's epilogue; H must not be an operand being read
    if (fuse_relu && fuse_relu != tA && fuse_relu != tB && fuse_relu != lhs) {
        TL_TRY(alloc_dense_public(c, fuse_relu));
        g.epi_relu = 1;
        g.D = fuse_relu->dense;
        g.sdm = g.scm;
        g.sdn = g.scn;
    }
    TL_TRY(launch_gemm(c, g));
    mark_written_dense(lhs);
    lhs->boolean = false;
    if (g.epi_relu) {
        mark_written_dense(fuse_relu);
        fuse_relu->boolean = false;
        if (fused) *fused = true;
    }
    *done = true;
    return TL_OK;
}

// `next` is `H = relu(Z)` over the LHS Z of `eq`, element for element: same
// shape and the same index order on both sides.  Returns H (allocated) or null.
Tensor* relu_successor(tl_ctx* c, const tl_equation* eq, const tl_equation* next, Tensor* lhs) {
    if (!next || next->accum != TL_ACC_ASSIGN || next->n_refs != 1 || next->n_code != 2) return nullptr;
    if (!(next->code[0].op == TL_OP_REF && next->code[1].op == TL_OP_NL && next->code[1].arg == TL_NL_RELU)) return nullptr;
    const tl_ref* r = &next->refs[0];
    if (strcmp(r->tensor, eq->lhs.tensor) || !strcmp(next->lhs.tensor, eq->lhs.tensor)) return nullptr;
    if (r->rank != 2 || next->lhs.rank != 2 || lhs->rank != 2) return nullptr;
    for (int k = 0; k < 2; ++k) {
        if (r->idx[k].kind != TL_IX_NAME || next->lhs.idx[k].kind != TL_IX_NAME) return nullptr;
        if (strcmp(r->idx[k].name, next->lhs.idx[k].name)) return nullptr;
        if (domain_size(c, r->idx[k].name) != lhs->dims[k]) return nullptr;
    }
    if (!strcmp(r->idx[0].name, r->idx[1].name)) return nullptr;
    Tensor* h = find_defined(c, next->lhs.tensor);
    if (!h && allocate_tensor(c, next->lhs.tensor, next->lhs.idx, next->lhs.rank, &h) != TL_OK) return nullptr;
    if (h->rank != 2 || h->dims[0] != lhs->dims[0] || h->dims[1] != lhs->dims[1]) return nullptr;
    if (h->shard == TL_SHARD_ROWS && c->world > 1) return nullptr;
    return h;
}

// ----------------------------------------------------------------------------
// Row-sharded message passing with the all-gather done by this library over
// NVLink: each rank's P = [relu-per-term] X W for its rows goes into its
// block of the gathered P, and from there into the same block of every other
// rank's copy (a buffer every rank maps) by peer stores: the GEMM's own
// epilogue (default), or a push kernel after the GEMM (TL_GNN_FAN=push).  The
// storing blocks count themselves into every rank's counters; the SpMM of
// the rank's own output rows waits for every other rank's count and then
// reads the gathered P locally.  Gathered P alternates between two buffers
// by layer: a rank writes layer k's buffer only after its layer k - 1 SpMM
// saw every rank's layer k - 1 counts, so every rank has finished the SpMM
// of layer k - 2 (the last reader of that buffer).  The decision depends
// only on quantities every rank shares (sizes, the collective peer set-ups),
// so all ranks take the same path; otherwise the NCCL all-gather below runs.
// ----------------------------------------------------------------------------
constexpr int kGnnCounter = 64;   // word of the peer slot array where rank r's tile count is kept (+ r)

static tl_status sparse_chain_fanned(tl_ctx* c, Tensor* S, Tensor* lhs, const float* xp, const float* wp, int64_t nu,
                                     int64_t x_rows, int64_t g, int64_t f, bool relu, bool x_nonneg, bool w_nonneg,
                                     bool* handled) {
    *handled = false;
    const int world = c->world;
    const int64_t per = (nu + world - 1) / world;
    const int64_t min_rows = nu / world;            // the smallest share
    const char* env = getenv("TL_GNN_NCCL");
    if ((env && env[0] == '1') || world > kMaxPeers || f % 64 || f > 4096 || min_rows < 128 || g < 32 ||
        (double)min_rows * f * g < (double)(1 << 25) || c->opts.precision != TL_PREC_TF32 || !tcgen05_available(c) ||
        lhs->zero == false)
        return TL_OK;
    TL_TRY(comm_peer_setup(c));
    if (c->peer_state != 1) return TL_OK;
    const size_t half = (size_t)per * world * f * 4;
    TL_TRY(comm_sym_setup(c, SYM_GNN, 2 * half));
    if (c->sym[SYM_GNN].state != 1) return TL_OK;
    const int par = (int)(c->gnn_layers & 1);
    c->gnn_layers++;
    auto gathered = [&](int q) {
        return reinterpret_cast<float*>(static_cast<char*>(c->sym[SYM_GNN].peer[q]) + par * half);
    };
    GemmPlan gp;
    memset(&gp, 0, sizeof gp);
    gp.M = x_rows; gp.N = f; gp.K = g;   // this rank's rows of X: its block of P
    gp.A = xp; gp.sam = g; gp.sak = 1;
    gp.B = wp; gp.sbk = f; gp.sbn = 1;
    gp.C = gathered(c->rank) + (int64_t)c->rank * per * f; gp.scm = f; gp.scn = 1;
    gp.scale = 1.0f; gp.beta = 0; gp.relu_term = relu ? 1 : 0;
    gp.a_nonneg = x_nonneg ? 1 : 0; gp.b_nonneg = w_nonneg ? 1 : 0;
    float* dst[kMaxPeers] = {};
    unsigned long long* cnt[kMaxPeers] = {};
    for (int q = 0; q < world; ++q) {
        if (q == c->rank) continue;
        dst[q] = gathered(q) + (int64_t)c->rank * per * f;
        cnt[q] = c->peer_slots[q] + kGnnCounter + c->rank;
    }
    // the GEMM's epilogue stores each tile to the peers (default), or the
    // GEMM runs as usual and a push kernel of 512 blocks stores the block to
    // the peers afterwards (TL_GNN_FAN=push).  Measured at n = 16384, f = 256,
    // two layers: epilogue 0.138 / 0.152 ms per step at N = 2 / 4, push
    // 0.185 / 0.197 ms (its peer stores reach about 230 GB/s), NCCL
    // all-gather 0.231 / 0.279 ms.
    const char* how = getenv("TL_GNN_FAN");
    const bool epilogue = !(how && !strcmp(how, "push"));
    if (epilogue) {
        for (int q = 0; q < world; ++q) {
            gp.fan[q] = dst[q];
            gp.fan_cnt[q] = cnt[q];
        }
        gp.fan_n = world - 1;
    }
    TL_TRY(launch_gemm(c, gp));
    if (!epilogue) TL_TRY(launch_fan_push(c, gp.C, x_rows * f, dst, cnt));
    // every other rank's tiles of this layer, counted cumulatively
    SpWait w{};
    w.cnt = c->peer_slots[c->rank] + kGnnCounter;
    w.timeout_ns = (unsigned long long)std::max(c->opts.comm_timeout_ms, 1000) * 1000000ull;
    for (int r = 0; r < world; ++r) {
        if (r == c->rank) continue;
        const int64_t r_rows = nu > r ? (nu - r + world - 1) / world : 0;
        c->gnn_expect[r] += (unsigned long long)(epilogue ? gemm_fan_tiles(r_rows, f) : fan_push_blocks());
        w.need[r] = c->gnn_expect[r];
    }
    TL_TRY(alloc_dense_public(c, lhs));
    TL_TRY(launch_spmm(c, lhs->local_rows(c->rank, world), S->rowptr, S->colidx, S->vals, gathered(c->rank),
                       per * world, f, f, lhs->dense, f, 0, 0, world, per, &w));
    mark_written_dense(lhs);
    lhs->boolean = false;
    lhs->nonneg = relu && S->csr_nonneg;   // S >= 0 times P, a sum of relus
    *handled = true;
    return TL_OK;
}

// ----------------------------------------------------------------------------
// Pattern: H[v,f] (+)= [relu] (S[v,u] X[u,g] W[g,f]) with S sparse, S >= 0
//   → P = [relu-per-term] X·W  (dense GEMM), then H (+)= S · P  (CSR SpMM).
// relu(s·x·w) = s·relu(x·w) for s >= 0, so the per-term relu moves inside P.
// ----------------------------------------------------------------------------
tl_status try_sparse_chain(tl_ctx* c, const tl_equation* eq, const Analysis& a, Tensor* lhs, bool* done) {
    *done = false;
    if (eq->accum != TL_ACC_ASSIGN && eq->accum != TL_ACC_ADD) return TL_OK;
    if (eq->n_refs != 3 || a.n_free != 2 || (int)a.vars.size() != 4) return TL_OK;
    const tl_instr* k = eq->code;
    int n = eq->n_code;
    bool relu = false;
    if (n >= 1 && k[n - 1].op == TL_OP_NL && k[n - 1].arg == TL_NL_RELU) { relu = true; n--; }
    if (!(n == 5 && k[0].op == TL_OP_REF && k[1].op == TL_OP_REF && k[2].op == TL_OP_PROD && k[2].arg == 2 &&
          k[3].op == TL_OP_REF && k[4].op == TL_OP_PROD && k[4].arg == 2))
        return TL_OK;
    const tl_ref* rs = &eq->refs[k[0].arg];
    const tl_ref* rx = &eq->refs[k[1].arg];
    const tl_ref* rw = &eq->refs[k[3].arg];
    Tensor* S = find_defined(c, rs->tensor);
    Tensor* X = find_defined(c, rx->tensor);
    Tensor* W = find_defined(c, rw->tensor);
    if (!S || !X || !W || !S->csr_valid || !S->csr_nonneg) return TL_OK;
    if (!lhs_bijective(a, lhs) || S->rank != 2 || X->rank != 2 || W->rank != 2 || lhs->rank != 2) return TL_OK;
    int vv = a.lhs_var[0], vf = a.lhs_var[1];
    // S[v,u], X[u,g], W[g,f] as plain names with matching sizes
    int s0 = ref_var(rs, 0, a), s1 = ref_var(rs, 1, a);
    int x0 = ref_var(rx, 0, a), x1 = ref_var(rx, 1, a);
    int w0 = ref_var(rw, 0, a), w1 = ref_var(rw, 1, a);
    if (s0 != vv || x0 != s1 || w0 != x1 || w1 != vf) return TL_OK;
    if (s1 < a.n_free || x1 < a.n_free) return TL_OK;
    if (S->dims[0] != a.vars[vv].size || S->dims[1] != a.vars[s1].size || X->dims[0] != a.vars[s1].size ||
        X->dims[1] != a.vars[x1].size || W->dims[0] != a.vars[x1].size || W->dims[1] != a.vars[vf].size)
        return TL_OK;
    if (W->shard == TL_SHARD_ROWS && c->world > 1) return TL_OK;
    bool sharded = c->world > 1 && X->shard == TL_SHARD_ROWS;
    if (c->world > 1 && (S->shard == TL_SHARD_ROWS) != (lhs->shard == TL_SHARD_ROWS)) return TL_OK;
    if (c->world > 1 && S->shard != TL_SHARD_ROWS && sharded) return TL_OK;
    const int64_t nu = X->dims[0], g = X->dims[1], f = W->dims[1];
    tl_status st;
    const float* xp = read_ptr(c, X, &st); TL_TRY(st);
    const float* wp = read_ptr(c, W, &st); TL_TRY(st);
    int64_t lrows_x = X->local_rows(c->rank, c->world);
    // P rows for the local u rows (all rows when X is replicated)
    int64_t p_rows = sharded ? lrows_x : nu;
    int64_t gathered_rows_per_rank = sharded ? (nu + c->world - 1) / c->world : 0;
    if (sharded && xp && wp) {
        bool handled = false;
        TL_TRY(sparse_chain_fanned(c, S, lhs, xp, wp, nu, lrows_x, g, f, relu, X->nonneg, W->nonneg, &handled));
        if (handled) {
            *done = true;
            return TL_OK;
        }
    }
    size_t p_bytes = (size_t)p_rows * f * 4;
    size_t pg_bytes = sharded ? (size_t)gathered_rows_per_rank * c->world * f * 4 : 0;
    void* ws = nullptr;
    TL_TRY(workspace(c, p_bytes + pg_bytes + (sharded ? (size_t)gathered_rows_per_rank * f * 4 : 0) + 256, &ws,
                     WS_CHAIN));
    float* P = (float*)ws;
    if (!xp || !wp) {
        TL_CK(c, cudaMemsetAsync(P, 0, p_bytes, c->stream));
    } else {
        GemmPlan gp;
        memset(&gp, 0, sizeof gp);
        gp.M = p_rows; gp.N = f; gp.K = g;
        gp.A = xp; gp.sam = g; gp.sak = 1;
        gp.B = wp; gp.sbk = f; gp.sbn = 1;
        gp.C = P; gp.scm = f; gp.scn = 1;
        gp.scale = 1.0f; gp.beta = 0; gp.relu_term = relu ? 1 : 0;
        gp.a_nonneg = X->nonneg ? 1 : 0; gp.b_nonneg = W->nonneg ? 1 : 0;
        if (p_rows > 0) TL_TRY(launch_gemm(c, gp));
    }
    const float* Pfull = P;
    int col_world = 1;
    int64_t col_local = 0;
    if (sharded) {
        // pad the local block to the per-rank row count, then all-gather
        float* Ppad = (float*)((char*)ws + p_bytes);
        float* Pg = Ppad + gathered_rows_per_rank * f;
        if (p_rows > 0)
            TL_CK(c, cudaMemcpyAsync(Ppad, P, p_bytes, cudaMemcpyDeviceToDevice, c->stream));
        LaunchScope L(c, "nccl_allgather_P", (double)gathered_rows_per_rank * c->world * f * 4.0, 0, false);
        TL_TRY(comm_allgather(c, Ppad, Pg, (size_t)gathered_rows_per_rank * f * 4));
        TL_TRY(L.done());
        Pfull = Pg;
        col_world = c->world;
        col_local = gathered_rows_per_rank;
    }
    int beta = lhs->zero ? 0 : 1;
    const bool was_nonneg = lhs->nonneg;
    if (beta) TL_TRY(ensure_dense(c, lhs));
    else TL_TRY(alloc_dense_public(c, lhs));
    int64_t out_rows = lhs->local_rows(c->rank, c->world);
    const int64_t p_total = sharded ? gathered_rows_per_rank * c->world : nu;
    TL_TRY(launch_spmm(c, out_rows, S->rowptr, S->colidx, S->vals, Pfull, p_total, f, f, lhs->dense, f, beta, 0,
                       col_world, col_local));
    mark_written_dense(lhs);
    lhs->boolean = false;
    // S >= 0 times P, a sum of relus (plus what was there, if that was >= 0)
    lhs->nonneg = relu && S->csr_nonneg && (beta == 0 || was_nonneg);
    *done = true;
    return TL_OK;
}

// ----------------------------------------------------------------------------
// Pattern: R[x,y] = step(E[x,y]) with E sparse → bit rows of R
// ----------------------------------------------------------------------------
tl_status try_step_bits(tl_ctx* c, const tl_equation* eq, const Analysis& a, Tensor* lhs, bool* done) {
    *done = false;
    if (eq->accum != TL_ACC_ASSIGN || a.has_contraction || eq->n_refs != 1 || eq->n_code != 2) return TL_OK;
    if (!(eq->code[0].op == TL_OP_REF && eq->code[1].op == TL_OP_NL && eq->code[1].arg == TL_NL_STEP)) return TL_OK;
    Tensor* E = find_defined(c, eq->refs[0].tensor);
    if (!E || !E->csr_valid || lhs->rank != 2 || E->rank != 2) return TL_OK;
    if (!lhs_bijective(a, lhs) || !plain_2d(&eq->refs[0], E, a)) return TL_OK;
    if (ref_var(&eq->refs[0], 0, a) != a.lhs_var[0] || ref_var(&eq->refs[0], 1, a) != a.lhs_var[1]) return TL_OK;
    if (E->dims[0] != lhs->dims[0] || E->dims[1] != lhs->dims[1]) return TL_OK;
    // a sharded source needs a sharded destination; a replicated one feeds either
    if (c->world > 1 && E->shard == TL_SHARD_ROWS && lhs->shard != TL_SHARD_ROWS) return TL_OK;
    if (c->lazy_eq == eq && E->csr_pos && E->csr_rows == E->dims[0]) {
        // the closure fixpoint that runs next reads these rows: it builds
        // them from E's successor lists instead of reading them back
        TL_TRY(alloc_bits_public(c, lhs));
        mark_written_bits(lhs);
        lhs->lazy_src = E;
        lhs->lazy_stamp = E->csr_stamp;
        *done = true;
        return TL_OK;
    }
    if (col_split(lhs))
        return fail(c, TL_ERR_UNSUPPORTED, "%s: a column-sharded relation must start as step(Edge) right before "
                    "its fixpoint", lhs->name.c_str());
    TL_TRY(launch_csr_to_bits(c, E, lhs));
    mark_written_bits(lhs);
    *done = true;
    return TL_OK;
}

// ----------------------------------------------------------------------------
// Row-wise softmax / lnorm (softmax.zig:19-229, layernorm.zig:25-310)
// ----------------------------------------------------------------------------
tl_status run_rowwise(tl_ctx* c, const tl_equation* eq, bool lnorm) {
    if (eq->n_code != 2 || eq->code[0].op != TL_OP_REF) return TL_OK;  // F3: comment and return
    int norm_axis = -1;
    for (int k = 0; k < eq->lhs.rank; ++k)
        if (eq->lhs.idx[k].kind == TL_IX_NORMALIZE) { norm_axis = k; break; }
    if (norm_axis < 0 && eq->lhs.rank > 0) norm_axis = eq->lhs.rank - 1;
    Tensor* out = find_defined(c, eq->lhs.tensor);
    if (!out) TL_TRY(allocate_tensor(c, eq->lhs.tensor, eq->lhs.idx, eq->lhs.rank, &out));
    Tensor* in = find_defined(c, eq->refs[0].tensor);
    if (!in) return TL_OK;
    if ((in->shard == TL_SHARD_ROWS || out->shard == TL_SHARD_ROWS) && c->world > 1)
        return fail(c, TL_ERR_UNSUPPORTED, "row-wise op on a sharded tensor");
    RowPlan p;
    memset(&p, 0, sizeof p);
    std::vector<std::string> outer_names;
    int64_t norm_size = 1;
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        if (ix->kind != TL_IX_NAME && ix->kind != TL_IX_NORMALIZE) continue;
        int64_t s = domain_size(c, ix->name);
        if (k == norm_axis) norm_size = s;
        else {
            // repeated outer names share one loop variable
            if (std::find(outer_names.begin(), outer_names.end(), std::string(ix->name)) != outer_names.end()) continue;
            outer_names.push_back(ix->name);
            p.outer_size[p.n_outer++] = s;
        }
    }
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        if (ix->kind != TL_IX_NAME && ix->kind != TL_IX_NORMALIZE) continue;
        int64_t si = k < in->rank ? in->strides[k] : 0;
        int64_t so = k < out->rank ? out->strides[k] : 0;
        if (k == norm_axis) { p.in_sn += si; p.out_sn += so; continue; }
        int o = (int)(std::find(outer_names.begin(), outer_names.end(), std::string(ix->name)) - outer_names.begin());
        p.outer_in_stride[o] += si;
        p.outer_out_stride[o] += so;
    }
    p.rows = 1;
    for (int o = 0; o < p.n_outer; ++o) p.rows *= p.outer_size[o];
    p.len = norm_size;
    tl_status st;
    (void)st;
    TL_TRY(ensure_dense(c, in));
    p.in = in->dense;
    // every output element is written exactly once when the row set tiles it
    TL_TRY(ensure_dense(c, out));
    p.out = out->dense;
    p.in_total = in->total;
    p.out_total = out->total;
    p.lnorm = lnorm ? 1 : 0;
    if (p.rows > 0 && p.len > 0) TL_TRY(launch_rowwise(c, p));
    mark_written_dense(out);
    out->boolean = false;
    return TL_OK;
}

}  // namespace

namespace tl {
static tl_status alloc_dense_impl(tl_ctx* c, Tensor* t);
tl_status alloc_dense_public(tl_ctx* c, Tensor* t) { return alloc_dense_impl(c, t); }
static tl_status alloc_dense_impl(tl_ctx* c, Tensor* t) {
    // dense storage without defining its contents (the caller writes all of it)
    int64_t need = t->local_rows(c->rank, c->world) * (t->rank >= 1 && t->dims[0] > 0 ? t->total / t->dims[0] : 1);
    if (t->shard != TL_SHARD_ROWS || c->world <= 1) need = t->total;
    if (t->dense && t->dense_elems >= need) return TL_OK;
    cudaFree(t->dense);
    t->dense = nullptr;
    TL_CK(c, cudaMalloc(&t->dense, std::max<int64_t>(need, 1) * sizeof(float)));
    t->dense_elems = need;
    return TL_OK;
}
}  // namespace tl

// ============================================================================
// genEquation (llvm.zig:357-459)
// ============================================================================
static tl_status run_equation(tl_ctx* c, const tl_equation* eq, const tl_equation* next = nullptr,
                              bool* consumed_next = nullptr) {
    if (consumed_next) *consumed_next = false;
    TL_TRY(validate_code(c, eq));
    if (eq->n_code > 0 && eq->code[eq->n_code - 1].op == TL_OP_NL) {
        int f = eq->code[eq->n_code - 1].arg;
        if (f == TL_NL_SOFTMAX) return run_rowwise(c, eq, false);
        if (f == TL_NL_LNORM) return run_rowwise(c, eq, true);
        if (f == TL_NL_CONCAT) return fail(c, TL_ERR_UNSUPPORTED, "concat is not lowered");
    }
    Tensor* lhs = find_defined(c, eq->lhs.tensor);
    if (!lhs) TL_TRY(allocate_tensor(c, eq->lhs.tensor, eq->lhs.idx, eq->lhs.rank, &lhs));
    Analysis a;
    TL_TRY(analyze(c, eq, false, &a));

    GenericPlan* p = new GenericPlan();
    std::unique_ptr<GenericPlan> hold(p);
    memset(p, 0, sizeof *p);
    if (a.scalar) {
        // genScalarAssign (einsum.zig:257-278): constant indices only
        if (lhs->shard == TL_SHARD_ROWS && c->world > 1) return fail(c, TL_ERR_UNSUPPORTED, "scalar store into a sharded tensor");
        int64_t off = 0;
        for (int k = 0; k < eq->lhs.rank && k < lhs->rank; ++k)
            off += (eq->lhs.idx[k].kind == TL_IX_CONST ? eq->lhs.idx[k].value : 0) * lhs->strides[k];
        TL_TRY(build_refs(c, eq, a, p));
        TL_TRY(ensure_dense(c, lhs));
        bool was_bool = lhs->boolean;
        if (off >= 0 && off < lhs->total) TL_TRY(launch_set1(c, lhs->dense, off, *p));
        mark_written_dense(lhs);
        lhs->boolean = was_bool && root_is_boolean(eq);
        return TL_OK;
    }
    if (lhs->shard == TL_SHARD_ROWS && c->world > 1) {
        bool done = false;
        TL_TRY(try_sparse_chain(c, eq, a, lhs, &done));
        if (!done) TL_TRY(try_step_bits(c, eq, a, lhs, &done));
        if (!done) {
            // fill of a sharded input before its load: `X[u,g] = 0`
            if (eq->n_code == 1 && eq->code[0].op == TL_OP_LIT && eq->code[0].value == 0.0 && !a.has_contraction &&
                eq->accum == TL_ACC_ASSIGN) {
                lhs->zero = true;
                lhs->dense_valid = lhs->bits_valid = lhs->csr_valid = false;
                return TL_OK;
            }
            return fail(c, TL_ERR_UNSUPPORTED, "%s: equation on a row-sharded tensor is not lowered", eq->lhs.tensor);
        }
        return TL_OK;
    }
    // constant fill of the whole tensor: `X[b,i] = 0` (kept lazy when zero)
    if (eq->n_code == 1 && eq->code[0].op == TL_OP_LIT && !a.has_contraction && eq->accum == TL_ACC_ASSIGN &&
        lhs_bijective(a, lhs)) {
        double v = eq->code[0].value;
        if (v == 0.0) {
            lhs->zero = true;
            lhs->boolean = true;
            lhs->dense_valid = lhs->bits_valid = lhs->csr_valid = lhs->csc_valid = false;
            return TL_OK;
        }
        TL_TRY(alloc_dense_public(c, lhs));
        TL_TRY(launch_fill(c, lhs->dense, lhs->total, (float)v));
        mark_written_dense(lhs);
        lhs->boolean = v == 1.0;
        return TL_OK;
    }
    bool done = false;
    Tensor* fuse = nullptr;
    if (next && consumed_next && validate_code(c, next) == TL_OK) fuse = relu_successor(c, eq, next, lhs);
    bool fused = false;
    TL_TRY(try_gemm(c, eq, a, lhs, &done, fuse, &fused));
    if (done && fused && consumed_next) *consumed_next = true;
    if (!done) TL_TRY(try_sparse_chain(c, eq, a, lhs, &done));
    if (!done) TL_TRY(try_step_bits(c, eq, a, lhs, &done));
    if (!done) TL_TRY(try_dot(c, eq, a, lhs, &done));
    if (done) return TL_OK;

    // generic loop nest
    TL_TRY(build_refs(c, eq, a, p));
    p->n_vars = (int)a.vars.size();
    p->n_free = a.n_free;
    p->n_out = 1;
    p->n_inner = 1;
    for (int i = 0; i < p->n_vars; ++i) {
        p->sizes[i] = a.vars[i].size;
        if (i < a.n_free) p->n_out *= a.vars[i].size;
        else p->n_inner *= a.vars[i].size;
    }
    bool bij = lhs_bijective(a, lhs);
    bool inj = lhs_injective(a, lhs);
    bool was_zero = lhs->zero;
    bool was_bool = lhs->boolean;
    if (bij && was_zero) {
        TL_TRY(alloc_dense_public(c, lhs));
        p->old_zero = 1;
    } else {
        TL_TRY(ensure_dense(c, lhs));
        p->old_zero = 0;
    }
    p->lhs = lhs->dense;
    p->lhs_total = lhs->total;
    p->n_lhs_terms = std::min(a.n_lhs_terms, lhs->rank);
    for (int t = 0; t < p->n_lhs_terms; ++t) {
        p->lhs_var[t] = a.lhs_var[t];
        p->lhs_div[t] = a.lhs_div[t];
        p->lhs_stride[t] = lhs->strides[t];
    }
    p->accum = eq->accum;
    p->has_contraction = a.has_contraction ? 1 : 0;
    p->atomic = inj ? 0 : 1;
    p->recursive = 0;
    // element-wise with every operand indexed exactly like the LHS
    p->aligned = (!a.has_contraction && bij) ? 1 : 0;
    for (int r = 0; r < eq->n_refs && p->aligned; ++r) {
        const tl_ref* ref = &eq->refs[r];
        Tensor* t = find_defined(c, ref->tensor);
        if (ref->rank != lhs->rank || (t && t->rank != lhs->rank)) { p->aligned = 0; break; }
        for (int k = 0; k < ref->rank; ++k) {
            if (ref->idx[k].kind != TL_IX_NAME || var_index(a.vars, ref->idx[k].name) != a.lhs_var[k] ||
                (t && t->dims[k] != lhs->dims[k])) {
                p->aligned = 0;
                break;
            }
        }
    }
    if (p->n_out > 0 && p->n_inner > 0) TL_TRY(launch_generic(c, *p, nullptr));
    // avg= divides the whole LHS by the product of its divisors (einsum.zig:151-195)
    if (eq->accum == TL_ACC_AVG && a.avg_div > 1) {
        GenericPlan* d = new GenericPlan();
        std::unique_ptr<GenericPlan> hd(d);
        memset(d, 0, sizeof *d);
        d->n_vars = 1; d->n_free = 1; d->sizes[0] = lhs->total; d->n_out = lhs->total; d->n_inner = 1;
        d->n_refs = 1;
        d->refs[0].ptr = lhs->dense; d->refs[0].total = lhs->total; d->refs[0].nidx = 1;
        d->refs[0].kind[0] = TL_IX_NAME; d->refs[0].var[0] = 0; d->refs[0].stride[0] = 1;
        d->n_code = 3;
        d->code[0] = {TL_OP_REF, 0, 0, 0, 0.0};
        d->code[1] = {TL_OP_LIT, 0, 0, 0, (double)a.avg_div};
        d->code[2] = {TL_OP_DIV, 0, 0, 0, 0.0};
        d->lhs = lhs->dense; d->lhs_total = lhs->total; d->n_lhs_terms = 1;
        d->lhs_var[0] = 0; d->lhs_div[0] = 1; d->lhs_stride[0] = 1;
        d->accum = TL_ACC_ASSIGN;
        if (lhs->total > 0) TL_TRY(launch_generic(c, *d, nullptr));
    }
    mark_written_dense(lhs);
    bool b = root_is_boolean(eq);
    if (eq->accum == TL_ACC_MAX || eq->accum == TL_ACC_MIN) b = b && (was_bool || was_zero);
    else if (eq->accum != TL_ACC_ASSIGN || a.has_contraction) b = false;
    else if (!bij) b = b && was_bool;
    lhs->boolean = b;
    return TL_OK;
}

extern "C" tl_status tl_equation_run(tl_ctx* c, const tl_equation* eq) {
    if (!c || !eq) return TL_ERR_INVALID;
    TL_CK(c, cudaSetDevice(c->device));
    return run_equation(c, eq);
}

// ============================================================================
// Fixpoint (fixpoint.zig:46-297)
// ============================================================================
static bool is_recursive(const tl_equation* eq) {
    for (int r = 0; r < eq->n_refs; ++r)
        if (strcmp(eq->refs[r].tensor, eq->lhs.tensor) == 0) return true;
    return false;
}

enum ClosureForm { NOT_CLOSURE = 0, CLOSURE_RIGHT, CLOSURE_LEFT };

// R[x,z] max= step(R[x,y] E[y,z])   → right form (rows of R are independent)
// R[x,y] max= step(E[x,z] R[z,y])   → left form  (row x reads rows z of R)
static ClosureForm match_closure(tl_ctx* c, const tl_equation* eq, Tensor** Rout, Tensor** Eout) {
    if (eq->accum != TL_ACC_MAX || eq->n_refs != 2 || eq->n_code != 4) return NOT_CLOSURE;
    const tl_instr* k = eq->code;
    if (!(k[0].op == TL_OP_REF && k[1].op == TL_OP_REF && k[2].op == TL_OP_PROD && k[2].arg == 2 &&
          k[3].op == TL_OP_NL && k[3].arg == TL_NL_STEP))
        return NOT_CLOSURE;
    const tl_ref* r0 = &eq->refs[k[0].arg];
    const tl_ref* r1 = &eq->refs[k[1].arg];
    const tl_ref* L = &eq->lhs;
    if (L->rank != 2 || r0->rank != 2 || r1->rank != 2) return NOT_CLOSURE;
    for (const tl_ref* r : {L, r0, r1})
        for (int i = 0; i < 2; ++i) if (r->idx[i].kind != TL_IX_NAME) return NOT_CLOSURE;
    auto nm = [](const tl_ref* r, int i) { return std::string(r->idx[i].name); };
    std::string x = nm(L, 0), z = nm(L, 1);
    if (x == z) return NOT_CLOSURE;
    ClosureForm form = NOT_CLOSURE;
    const tl_ref* er = nullptr;
    // right: R[x,y] E[y,z]
    if (!strcmp(r0->tensor, L->tensor) && strcmp(r1->tensor, L->tensor) && nm(r0, 0) == x && nm(r1, 1) == z &&
        nm(r0, 1) == nm(r1, 0) && nm(r0, 1) != x && nm(r0, 1) != z) {
        form = CLOSURE_RIGHT; er = r1;
    }
    // left: E[x,y] R[y,z]
    if (!strcmp(r1->tensor, L->tensor) && strcmp(r0->tensor, L->tensor) && nm(r0, 0) == x && nm(r1, 1) == z &&
        nm(r0, 1) == nm(r1, 0) && nm(r0, 1) != x && nm(r0, 1) != z) {
        form = CLOSURE_LEFT; er = r0;
    }
    if (form == NOT_CLOSURE) return NOT_CLOSURE;
    Tensor* R = find_defined(c, L->tensor);
    Tensor* E = find_defined(c, er->tensor);
    if (!R || !E || R->rank != 2 || E->rank != 2) return NOT_CLOSURE;
    int64_t n = R->dims[0];
    std::string y = nm(r0, 1);
    // E may have fewer rows than n (its max dims come from constant-index
    // assignments); the missing rows read as 0.0, i.e. have no successors
    if (R->dims[1] != n || E->dims[0] > n || E->dims[1] != n) return NOT_CLOSURE;
    if (domain_size(c, x.c_str()) != n || domain_size(c, z.c_str()) != n || domain_size(c, y.c_str()) != n)
        return NOT_CLOSURE;
    if (!R->boolean) return NOT_CLOSURE;
    // step(r * e) == (r > 0) && (e > 0) needs e >= 0 (r is 0/1)
    // the bit-row sweeps treat every stored entry as an edge: values must be > 0
    if (!(E->csr_valid ? E->csr_pos : E->boolean)) return NOT_CLOSURE;
    // the sweeps read successor lists of every row: the relation is replicated
    if (E->csr_valid && E->csr_rows != E->dims[0]) return NOT_CLOSURE;
    if (form == CLOSURE_LEFT && R->shard == TL_SHARD_ROWS && c->world > 1) return NOT_CLOSURE;
    *Rout = R;
    *Eout = E;
    return form;
}

static tl_status generic_recursive(tl_ctx* c, const tl_equation* eq, int* d_changed) {
    Tensor* lhs = find_defined(c, eq->lhs.tensor);
    if (!lhs) TL_TRY(allocate_tensor(c, eq->lhs.tensor, eq->lhs.idx, eq->lhs.rank, &lhs));
    if (lhs->shard == TL_SHARD_ROWS && c->world > 1)
        return fail(c, TL_ERR_UNSUPPORTED, "%s: recursive equation on a sharded tensor", eq->lhs.tensor);
    Analysis a;
    TL_TRY(analyze(c, eq, true, &a));
    if (a.scalar) return TL_OK;
    GenericPlan* p = new GenericPlan();
    std::unique_ptr<GenericPlan> hold(p);
    memset(p, 0, sizeof *p);
    TL_TRY(ensure_dense(c, lhs));
    mark_written_dense(lhs);
    TL_TRY(build_refs(c, eq, a, p));
    p->n_vars = (int)a.vars.size();
    p->n_free = a.n_free;
    p->n_out = 1; p->n_inner = 1;
    for (int i = 0; i < p->n_vars; ++i) {
        p->sizes[i] = a.vars[i].size;
        if (i < a.n_free) p->n_out *= a.vars[i].size; else p->n_inner *= a.vars[i].size;
    }
    p->lhs = lhs->dense;
    p->lhs_total = lhs->total;
    p->n_lhs_terms = std::min(a.n_lhs_terms, lhs->rank);
    for (int t = 0; t < p->n_lhs_terms; ++t) {
        p->lhs_var[t] = a.lhs_var[t]; p->lhs_div[t] = 1; p->lhs_stride[t] = lhs->strides[t];
    }
    p->accum = eq->accum;
    p->has_contraction = a.has_contraction;
    p->atomic = lhs_injective(a, lhs) ? 0 : 1;
    p->recursive = 1;
    bool was_bool = lhs->boolean;
    lhs->nonneg = false;   // written in place below
    if (p->n_out > 0 && p->n_inner > 0) TL_TRY(launch_generic(c, *p, d_changed));
    lhs->boolean = was_bool && eq->accum == TL_ACC_MAX && root_is_boolean(eq);
    return TL_OK;
}

static tl_status run_fixpoint(tl_ctx* c, const tl_equation* eqs, int n, int32_t* sweeps_out) {
    for (int i = 0; i < n; ++i) TL_TRY(validate_code(c, &eqs[i]));
    // allocate every recursive LHS first (genRecursiveEquation, fixpoint.zig:103-106)
    for (int i = 0; i < n; ++i) {
        Tensor* t = find_defined(c, eqs[i].lhs.tensor);
        if (!t) TL_TRY(allocate_tensor(c, eqs[i].lhs.tensor, eqs[i].lhs.idx, eqs[i].lhs.rank, &t));
    }
    int max_sweeps = c->opts.max_sweeps > 0 ? c->opts.max_sweeps : 1000;
    int* d_changed = c->d_flags;   // word 0: changed this sweep
    int sweeps = 0;
    bool changed = true;
    // a single closure equation runs on bit rows
    Tensor *R = nullptr, *E = nullptr;
    ClosureForm form = n == 1 ? match_closure(c, &eqs[0], &R, &E) : NOT_CLOSURE;
    // the bit-row sweeps read the relation's successor lists (CSR)
    if (form != NOT_CLOSURE && !E->csr_valid) {
        // a dense 0/1 relation (element assignments): build its successor lists
        if (E->shard == TL_SHARD_ROWS && c->world > 1) form = NOT_CLOSURE;
        else {
            TL_TRY(launch_dense_to_csr(c, E));
            if (!E->csr_pos) form = NOT_CLOSURE;
        }
    }
    if (form == CLOSURE_RIGHT) {
        // rows left unwritten by step(E) are built by the one-launch fixpoint
        if (!(R->bits_valid && R->lazy_src == E)) TL_TRY(ensure_bits(c, R));
        bool handled = false;
        // the sweep count (and the note at the cap) is set when the launch's
        // result is read: now if the caller wants it, else at the next sync
        TL_TRY(launch_closure_fixpoint(c, R, E, max_sweeps, sweeps_out != nullptr, &sweeps, &changed, &handled));
        if (handled) {
            mark_written_bits(R);
            if (sweeps_out) *sweeps_out = sweeps;
            return TL_OK;
        }
    }
    if (form != NOT_CLOSURE) TL_TRY(ensure_bits(c, R));
    while (sweeps < max_sweeps && changed) {
        TL_CK(c, cudaMemsetAsync(d_changed, 0, sizeof(int), c->stream));
        if (form == CLOSURE_RIGHT) TL_TRY(launch_closure_right(c, R, E, d_changed, sweeps));
        else if (form == CLOSURE_LEFT) TL_TRY(launch_closure_left(c, R, E, d_changed));
        else for (int i = 0; i < n; ++i) TL_TRY(generic_recursive(c, &eqs[i], d_changed));
        if (c->world > 1) TL_TRY(comm_allreduce_max_int(c, d_changed, 1));
        TL_CK(c, cudaMemcpyAsync(c->h_flags, d_changed, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
        TL_CK(c, cudaStreamSynchronize(c->stream));
        changed = c->h_flags[0] != 0;
        sweeps++;
    }
    if (form != NOT_CLOSURE) mark_written_bits(R);
    c->last_sweeps = sweeps;
    if (sweeps_out) *sweeps_out = sweeps;
    if (changed) fail(c, TL_OK, "fixpoint stopped at the %d-sweep cap", sweeps);
    return TL_OK;
}

extern "C" tl_status tl_fixpoint(tl_ctx* c, const tl_equation* eqs, int32_t n, int32_t* sweeps_out) {
    if (!c || (n > 0 && !eqs)) return TL_ERR_INVALID;
    TL_CK(c, cudaSetDevice(c->device));
    return run_fixpoint(c, eqs, n, sweeps_out);
}

// ============================================================================
// sparse declaration, save / load, program schedule
// ============================================================================
extern "C" tl_status tl_sparse_decl(tl_ctx* c, const tl_ref* decl) {
    if (!c || !decl || decl->rank < 0 || decl->rank > TL_MAX_RANK) return TL_ERR_INVALID;
    tl_index idx[TL_MAX_RANK];
    for (int k = 0; k < decl->rank; ++k) {
        memset(&idx[k], 0, sizeof idx[k]);
        idx[k].kind = TL_IX_NAME;
        snprintf(idx[k].name, TL_NAME_LEN, "%s", decl->idx[k].name);
    }
    TL_TRY(bq_detach(c, decl->tensor));
    Tensor* t;
    TL_TRY(allocate_tensor(c, decl->tensor, idx, decl->rank, &t));
    t->is_sparse = true;
    return TL_OK;
}

static tl_status run_save(tl_ctx* c, const tl_statement* st) {
    Tensor* t = find_defined(c, st->name);
    if (!t) return TL_OK;   // the reference emits a comment
    std::vector<double> v(std::max<int64_t>(t->total, 1));
    TL_TRY(tl_tensor_download(static_cast<tl_tensor*>(t), v.data()));
    FILE* f = fopen(st->path, "wb");
    if (!f) return fail(c, TL_ERR_IO, "cannot open %s", st->path);
    size_t w = fwrite(v.data(), 8, (size_t)t->total, f);
    fclose(f);
    return w == (size_t)t->total ? TL_OK : fail(c, TL_ERR_IO, "short write to %s", st->path);
}

static tl_status run_load(tl_ctx* c, const tl_statement* st) {
    Tensor* t = find_defined(c, st->name);
    if (!t) return TL_OK;
    if (st->host_data) return tl_tensor_upload(static_cast<tl_tensor*>(t), st->host_data);
    if (st->path[0] == 0) {
        // resident input: the device storage already holds this run's values
        if (!t->dense) return fail(c, TL_ERR_INVALID, "%s: resident load without device data", st->name);
        t->zero = false;
        t->nonneg = false;   // values unknown to the host
        t->dense_valid = true;
        t->bits_valid = t->csr_valid = t->csc_valid = false;
        return TL_OK;
    }
    std::vector<double> v(std::max<int64_t>(t->total, 1), 0.0);
    FILE* f = fopen(st->path, "rb");
    if (!f) return fail(c, TL_ERR_IO, "cannot open %s", st->path);
    size_t r = fread(v.data(), 8, (size_t)t->total, f);
    fclose(f);
    (void)r;
    return tl_tensor_upload(static_cast<tl_tensor*>(t), v.data());
}

static tl_status run_sparse_load(tl_ctx* c, const tl_statement* st) {
    Tensor* t = find_defined(c, st->name);
    if (!t) return fail(c, TL_ERR_NOT_FOUND, "sparse tensor %s not declared", st->name);
    if (!st->coo_rows) {
        // resident: keep the CSR uploaded earlier
        if (!t->rowptr) return fail(c, TL_ERR_INVALID, "%s: resident sparse load without device data", st->name);
        t->zero = false;
        t->csr_valid = true;
        t->boolean = t->csr_ones;
        t->nonneg = t->csr_nonneg;
        t->dense_valid = t->bits_valid = false;
        t->csc_valid = t->colptr != nullptr;
        return TL_OK;
    }
    return tl_sparse_upload(static_cast<tl_tensor*>(t), st->size, st->coo_rows, st->coo_cols, st->host_data);
}

// True if statement st names tensor t (a backward pass counts as naming every tensor).
static bool names_tensor(const tl_statement* st, const char* t) {
    switch (st->kind) {
    case TL_STMT_EQUATION:
        if (!strcmp(st->eq.lhs.tensor, t)) return true;
        for (int k = 0; k < st->eq.n_refs && k < TL_MAX_REFS; ++k)
            if (!strcmp(st->eq.refs[k].tensor, t)) return true;
        return false;
    case TL_STMT_SPARSE: return !strcmp(st->sparse.tensor, t);
    case TL_STMT_SPARSE_LOAD: case TL_STMT_LOAD: case TL_STMT_SAVE: return !strcmp(st->name, t);
    case TL_STMT_BACKWARD: return true;
    default: return false;
    }
}

// The equation R[..] = step(E[..]) whose bit rows may stay unwritten until the
// fixpoint: the program's only recursive equation reads R and E, and no
// statement after it touches R or E before the fixpoint runs.
static const tl_equation* lazy_step_equation(const tl_statement* s, int n) {
    const tl_equation* rec = nullptr;
    int n_rec = 0;
    for (int i = 0; i < n; ++i)
        if (s[i].kind == TL_STMT_EQUATION && is_recursive(&s[i].eq)) { ++n_rec; rec = &s[i].eq; }
    if (n_rec != 1 || rec->accum != TL_ACC_MAX || rec->n_refs != 2 || getenv("TL_NO_LAZY_STEP")) return nullptr;
    const char* R = rec->lhs.tensor;
    const char* E = !strcmp(rec->refs[0].tensor, R) ? rec->refs[1].tensor : rec->refs[0].tensor;
    if (!strcmp(E, R)) return nullptr;
    for (int i = n - 1; i >= 0; --i) {
        const tl_statement* st = &s[i];
        if (st->kind == TL_STMT_EQUATION && &st->eq == rec) continue;
        if (!names_tensor(st, R) && !names_tensor(st, E)) continue;
        const tl_equation* eq = &st->eq;
        if (st->kind == TL_STMT_EQUATION && !strcmp(eq->lhs.tensor, R) && eq->n_refs == 1 &&
            !strcmp(eq->refs[0].tensor, E) && eq->n_code == 2 && eq->code[1].op == TL_OP_NL &&
            eq->code[1].arg == TL_NL_STEP && !is_recursive(eq))
            return eq;
        return nullptr;
    }
    return nullptr;
}

// An attention block, three equations in a row (softmax.zig:19-229 between
// two contractions, einsum.zig:20-254):
//   S[q,k] = Q[q,d] K[k,d] (times or divided by a literal)
//   A[q,k.] = softmax(S[q,k])
//   O[q,d] = A[q,k] V[k,d]
// on row-major fp32 tensors with d = 64 and q, k multiples of 128, S and O
// written for the first time in this run and no sign test on S or O: run as
// the tiled kernel and the combine kernel (launch_attention), which write S,
// A and O in full.  Anything else takes the three equations one by one.
static tl_status try_attention(tl_ctx* c, const tl_equation* e1, const tl_equation* e2, const tl_equation* e3,
                               bool* done) {
    *done = false;
    if (getenv("TL_NO_FUSED_ATTENTION") || c->opts.precision != TL_PREC_TF32 || !tcgen05_available(c)) return TL_OK;
    if (e1->accum != TL_ACC_ASSIGN || e2->accum != TL_ACC_ASSIGN || e3->accum != TL_ACC_ASSIGN) return TL_OK;
    auto name_is = [](const tl_index& ix, const char* n) { return !strcmp(ix.name, n); };
    auto plain = [](const tl_ref& r) {
        if (r.rank != 2) return false;
        for (int k = 0; k < 2; ++k)
            if (r.idx[k].kind != TL_IX_NAME) return false;
        return true;
    };
    // e2: A[q, k.] = softmax(S[q, k])
    if (e2->n_refs != 1 || e2->n_code != 2 || e2->code[0].op != TL_OP_REF || e2->code[0].arg != 0 ||
        e2->code[1].op != TL_OP_NL || e2->code[1].arg != TL_NL_SOFTMAX)
        return TL_OK;
    const tl_ref& rs2 = e2->refs[0];
    if (!plain(rs2) || e2->lhs.rank != 2 || e2->lhs.idx[0].kind != TL_IX_NAME ||
        (e2->lhs.idx[1].kind != TL_IX_NAME && e2->lhs.idx[1].kind != TL_IX_NORMALIZE))
        return TL_OK;
    const char* qn = rs2.idx[0].name;
    const char* kn = rs2.idx[1].name;
    if (!strcmp(qn, kn) || !name_is(e2->lhs.idx[0], qn) || !name_is(e2->lhs.idx[1], kn)) return TL_OK;
    // e1: S[q, k] = Q[q, d] K[k, d] scale
    GemmMatch m1, m3;
    if (!match_product2(e1, &m1) || m1.relu_term || !plain(e1->lhs) || strcmp(e1->lhs.tensor, rs2.tensor) ||
        !name_is(e1->lhs.idx[0], qn) || !name_is(e1->lhs.idx[1], kn))
        return TL_OK;
    const tl_ref* rq = &e1->refs[m1.ref_a];
    const tl_ref* rk = &e1->refs[m1.ref_b];
    if (!plain(*rq) || !plain(*rk)) return TL_OK;
    if (name_is(rq->idx[0], kn)) std::swap(rq, rk);
    if (!name_is(rq->idx[0], qn) || !name_is(rk->idx[0], kn)) return TL_OK;
    const char* dn = rq->idx[1].name;
    if (!name_is(rk->idx[1], dn) || !strcmp(dn, qn) || !strcmp(dn, kn)) return TL_OK;
    // e3: O[q, d] = A[q, k] V[k, d]
    if (!match_product2(e3, &m3) || m3.relu_term || m3.scale != 1.0f || !plain(e3->lhs) ||
        !name_is(e3->lhs.idx[0], qn) || !name_is(e3->lhs.idx[1], dn))
        return TL_OK;
    const tl_ref* ra = &e3->refs[m3.ref_a];
    const tl_ref* rv = &e3->refs[m3.ref_b];
    if (strcmp(ra->tensor, e2->lhs.tensor)) std::swap(ra, rv);
    if (!plain(*ra) || !plain(*rv) || strcmp(ra->tensor, e2->lhs.tensor) || !name_is(ra->idx[0], qn) ||
        !name_is(ra->idx[1], kn) || !name_is(rv->idx[0], kn) || !name_is(rv->idx[1], dn))
        return TL_OK;
    // the tensors: inputs defined and dense, outputs distinct and fresh
    const int64_t nq = domain_size(c, qn), nk = domain_size(c, kn), nd = domain_size(c, dn);
    if (nd != 64 || nq < 128 || nk < 128 || nq % 128 || nk % 128 || nq >= INT32_MAX || nk >= INT32_MAX) return TL_OK;
    const char* outs[3] = {e1->lhs.tensor, e2->lhs.tensor, e3->lhs.tensor};
    const char* ins[3] = {rq->tensor, rk->tensor, rv->tensor};
    for (int i = 0; i < 3; ++i) {
        for (int j = 0; j < 3; ++j)
            if (!strcmp(outs[i], ins[j]) || (i != j && !strcmp(outs[i], outs[j]))) return TL_OK;
        if (std::find(c->sign_sensitive.begin(), c->sign_sensitive.end(), std::string(outs[i])) !=
            c->sign_sensitive.end())
            return TL_OK;
    }
    Tensor* tq = find_defined(c, rq->tensor);
    Tensor* tk = find_defined(c, rk->tensor);
    Tensor* tv = find_defined(c, rv->tensor);
    auto shape_ok = [](const Tensor* t, int64_t r, int64_t cl) {
        return t && t->rank == 2 && t->dims[0] == r && t->dims[1] == cl && t->shard != TL_SHARD_ROWS;
    };
    if (!shape_ok(tq, nq, 64) || !shape_ok(tk, nk, 64) || !shape_ok(tv, nk, 64)) return TL_OK;
    Tensor* out[3];
    for (int i = 0; i < 3; ++i) {
        const tl_equation* e = i == 0 ? e1 : i == 1 ? e2 : e3;
        out[i] = find_defined(c, outs[i]);
        if (!out[i]) TL_TRY(allocate_tensor(c, e->lhs.tensor, e->lhs.idx, e->lhs.rank, &out[i]));
    }
    if (!shape_ok(out[0], nq, nk) || !shape_ok(out[1], nq, nk) || !shape_ok(out[2], nq, 64) || !out[0]->zero ||
        !out[2]->zero)
        return TL_OK;
    tl_status st;
    AttnPlan p;
    p.Q = read_ptr(c, tq, &st); TL_TRY(st);
    p.K = read_ptr(c, tk, &st); TL_TRY(st);
    p.V = read_ptr(c, tv, &st); TL_TRY(st);
    if (!p.Q || !p.K || !p.V) return TL_OK;   // a zero operand: the one-by-one path keeps its meaning
    for (int i = 0; i < 3; ++i) TL_TRY(alloc_dense_public(c, out[i]));
    p.S = out[0]->dense;
    p.A = out[1]->dense;
    p.O = out[2]->dense;
    p.n_q = nq;
    p.n_k = nk;
    p.scale = m1.scale;
    for (const void* ptr : {(const void*)p.Q, (const void*)p.K, (const void*)p.V, (const void*)p.S, (const void*)p.A,
                            (const void*)p.O})
        if ((uintptr_t)ptr & 15) return TL_OK;
    TL_TRY(launch_attention(c, p));
    for (int i = 0; i < 3; ++i) {
        mark_written_dense(out[i]);
        out[i]->boolean = false;
    }
    *done = true;
    return TL_OK;
}

// A small-batch head: H[b, h] = [relu](X[b, i] W1[i, h] s1), Z[b, o] =
// H[b, h] W2[h, o] s2, Y[b, o.] = softmax(Z[b, o]) (either operand order in
// each product), b <= 64 and o <= 32, H and Z defined fresh by these
// statements: two launches (k_head.cu) instead of three latency-bound ones.
static tl_status try_head(tl_ctx* c, const tl_equation* e1, const tl_equation* e2, const tl_equation* e3,
                          bool* done) {
    *done = false;
    if (getenv("TL_NO_FUSED_HEAD")) return TL_OK;
    if (e1->accum != TL_ACC_ASSIGN || e2->accum != TL_ACC_ASSIGN || e3->accum != TL_ACC_ASSIGN) return TL_OK;
    auto name_is = [](const tl_index& ix, const char* n) { return !strcmp(ix.name, n); };
    auto plain = [](const tl_ref& r) {
        if (r.rank != 2) return false;
        for (int k = 0; k < 2; ++k)
            if (r.idx[k].kind != TL_IX_NAME) return false;
        return true;
    };
    // e3: Y[b, o.] = softmax(Z[b, o])
    if (e3->n_refs != 1 || e3->n_code != 2 || e3->code[0].op != TL_OP_REF || e3->code[0].arg != 0 ||
        e3->code[1].op != TL_OP_NL || e3->code[1].arg != TL_NL_SOFTMAX)
        return TL_OK;
    const tl_ref& rz = e3->refs[0];
    if (!plain(rz) || e3->lhs.rank != 2 || e3->lhs.idx[0].kind != TL_IX_NAME ||
        (e3->lhs.idx[1].kind != TL_IX_NAME && e3->lhs.idx[1].kind != TL_IX_NORMALIZE))
        return TL_OK;
    const char* bn = rz.idx[0].name;
    const char* on = rz.idx[1].name;
    if (!strcmp(bn, on) || !name_is(e3->lhs.idx[0], bn) || !name_is(e3->lhs.idx[1], on)) return TL_OK;
    // e2: Z[b, o] = H[b, h] W2[h, o] s2
    GemmMatch m1, m2;
    if (!match_product2(e2, &m2) || m2.relu_term || !plain(e2->lhs) || strcmp(e2->lhs.tensor, rz.tensor) ||
        !name_is(e2->lhs.idx[0], bn) || !name_is(e2->lhs.idx[1], on))
        return TL_OK;
    const tl_ref* rh = &e2->refs[m2.ref_a];
    const tl_ref* rw2 = &e2->refs[m2.ref_b];
    if (strcmp(rh->tensor, e1->lhs.tensor)) std::swap(rh, rw2);
    if (!plain(*rh) || !plain(*rw2) || strcmp(rh->tensor, e1->lhs.tensor) || !name_is(rh->idx[0], bn)) return TL_OK;
    const char* hn = rh->idx[1].name;
    if (!name_is(rw2->idx[0], hn) || !name_is(rw2->idx[1], on) || !strcmp(hn, bn) || !strcmp(hn, on)) return TL_OK;
    // e1: H[b, h] = [relu](X[b, i] W1[i, h] s1)
    if (!match_product2(e1, &m1) || !plain(e1->lhs) || !name_is(e1->lhs.idx[0], bn) || !name_is(e1->lhs.idx[1], hn))
        return TL_OK;
    const tl_ref* rx = &e1->refs[m1.ref_a];
    const tl_ref* rw1 = &e1->refs[m1.ref_b];
    if (!plain(*rx) || !plain(*rw1)) return TL_OK;
    if (!name_is(rx->idx[0], bn)) std::swap(rx, rw1);
    if (!name_is(rx->idx[0], bn)) return TL_OK;
    const char* in = rx->idx[1].name;
    if (!name_is(rw1->idx[0], in) || !name_is(rw1->idx[1], hn) || !strcmp(in, bn) || !strcmp(in, hn) ||
        !strcmp(in, on))
        return TL_OK;
    const int64_t nb = domain_size(c, bn), ni = domain_size(c, in), nh = domain_size(c, hn), no = domain_size(c, on);
    // (X's chunk of a block, at most 64 rows x 192 contracted indices, fits
    // 48 KB of shared memory; a row of H fits 200 KB)
    if (nb < 1 || nb > kHeadMaxRows || no < 1 || no > kHeadMaxCols || ni < 1 || ni > 12288 || nh < 1 ||
        nh > 50 * 1024)
        return TL_OK;
    // inputs defined, outputs distinct, fresh and not read by these statements
    const char* outs[3] = {e1->lhs.tensor, e2->lhs.tensor, e3->lhs.tensor};
    const char* ins[3] = {rx->tensor, rw1->tensor, rw2->tensor};
    for (int i = 0; i < 3; ++i) {
        for (int j = 0; j < 3; ++j)
            if (!strcmp(outs[i], ins[j]) || (i != j && !strcmp(outs[i], outs[j]))) return TL_OK;
        if (std::find(c->sign_sensitive.begin(), c->sign_sensitive.end(), std::string(outs[i])) !=
            c->sign_sensitive.end())
            return TL_OK;
    }
    Tensor* tx = find_defined(c, rx->tensor);
    Tensor* tw1 = find_defined(c, rw1->tensor);
    Tensor* tw2 = find_defined(c, rw2->tensor);
    auto shape_ok = [](const Tensor* t, int64_t r, int64_t cl) {
        return t && t->rank == 2 && t->dims[0] == r && t->dims[1] == cl && t->shard != TL_SHARD_ROWS;
    };
    if (!shape_ok(tx, nb, ni) || !shape_ok(tw1, ni, nh) || !shape_ok(tw2, nh, no)) return TL_OK;
    Tensor* out[3];
    for (int i = 0; i < 3; ++i) {
        const tl_equation* e = i == 0 ? e1 : i == 1 ? e2 : e3;
        out[i] = find_defined(c, outs[i]);
        if (!out[i]) TL_TRY(allocate_tensor(c, e->lhs.tensor, e->lhs.idx, e->lhs.rank, &out[i]));
    }
    if (!shape_ok(out[0], nb, nh) || !shape_ok(out[1], nb, no) || !shape_ok(out[2], nb, no) || !out[0]->zero ||
        !out[1]->zero)
        return TL_OK;
    tl_status st;
    HeadPlan p{};
    p.X = read_ptr(c, tx, &st); TL_TRY(st);
    p.W1 = read_ptr(c, tw1, &st); TL_TRY(st);
    p.W2 = read_ptr(c, tw2, &st); TL_TRY(st);
    if (!p.X || !p.W1 || !p.W2) return TL_OK;   // a zero operand: the one-by-one path keeps its meaning
    for (int i = 0; i < 3; ++i) TL_TRY(alloc_dense_public(c, out[i]));
    p.H = out[0]->dense;
    p.Z = out[1]->dense;
    p.Y = out[2]->dense;
    p.b = nb; p.i = ni; p.h = nh; p.o = no;
    p.relu_term = m1.relu_term ? 1 : 0;
    p.sgn1 = m1.relu_term && m1.scale < 0.f ? -1.f : 1.f;
    p.mag1 = m1.relu_term ? fabsf(m1.scale) : m1.scale;
    p.s2 = m2.scale;
    TL_TRY(launch_head(c, p));
    for (int i = 0; i < 3; ++i) {
        mark_written_dense(out[i]);
        out[i]->boolean = false;
    }
    out[0]->nonneg = m1.relu_term;   // a sum of relus times |s1|
    out[2]->nonneg = true;           // a softmax
    *done = true;
    return TL_OK;
}

// The statements of a run in order (non-recursive equations, declarations,
// loads, backward); recursive equations are collected into `rec`.
static tl_status run_statements(tl_ctx* c, const tl_statement* s, int n, const std::vector<tl_equation>& eqs,
                                std::vector<tl_equation>* rec) {
    for (int i = 0; i < n; ++i) {
        const tl_statement* st = &s[i];
        switch (st->kind) {
        case TL_STMT_DOMAIN: case TL_STMT_QUERY: break;
        case TL_STMT_EQUATION:
            if (is_recursive(&st->eq)) rec->push_back(st->eq);
            else {
                // an attention block runs as one tiled pipeline
                if (i + 2 < n && s[i + 1].kind == TL_STMT_EQUATION && s[i + 2].kind == TL_STMT_EQUATION &&
                    !is_recursive(&s[i + 1].eq) && !is_recursive(&s[i + 2].eq)) {
                    bool fused = false;
                    TL_TRY(validate_code(c, &st->eq));
                    TL_TRY(validate_code(c, &s[i + 1].eq));
                    TL_TRY(validate_code(c, &s[i + 2].eq));
                    TL_TRY(try_attention(c, &st->eq, &s[i + 1].eq, &s[i + 2].eq, &fused));
                    if (!fused) TL_TRY(try_head(c, &st->eq, &s[i + 1].eq, &s[i + 2].eq, &fused));
                    if (fused) {
                        i += 2;
                        break;
                    }
                }
                // an element-wise relu right after a GEMM is written by its epilogue
                const tl_equation* next = (i + 1 < n && s[i + 1].kind == TL_STMT_EQUATION &&
                                           !is_recursive(&s[i + 1].eq)) ? &s[i + 1].eq : nullptr;
                bool consumed = false;
                TL_TRY(run_equation(c, &st->eq, next, &consumed));
                if (consumed) ++i;
            }
            break;
        case TL_STMT_SPARSE: TL_TRY(tl_sparse_decl(c, &st->sparse)); break;
        case TL_STMT_SPARSE_LOAD: TL_TRY(run_sparse_load(c, st)); break;
        case TL_STMT_BACKWARD:
            TL_TRY(run_backward(c, st->name, st->params, st->n_params, eqs.data(), (int)eqs.size()));
            break;
        case TL_STMT_SAVE: TL_TRY(run_save(c, st)); break;
        case TL_STMT_LOAD: TL_TRY(run_load(c, st)); break;
        default: return fail(c, TL_ERR_INVALID, "unknown statement kind %d", st->kind);
        }
    }
    return TL_OK;
}

// ----------------------------------------------------------------------------
// Program runs as CUDA graphs.  A run whose statements only launch work on
// the stream (no host data, files, queries, fixpoint or collectives) is
// captured once its host state has repeated (the same tensors, storages and
// flags at the start of two eager runs), and later runs with that state replay
// the graph: one launch instead of the host work and launches of every
// statement.  The host-visible state after a replay is the one the captured
// run ended with.
// ----------------------------------------------------------------------------
namespace {

struct TensorSnap {
    char name[64];
    int32_t rank, shard, succ_sentinel;
    int64_t dims[TL_MAX_RANK];
    int64_t total, dense_elems, bits_words, bits_rows, nnz, csr_cap, csr_rows, csc_cap, succ_cap, succ_nodes;
    uint8_t defined, zero, boolean, is_sparse, dense_valid, bits_valid, csr_valid, csc_valid, csr_nonneg, csr_ones,
        csr_pos, nonneg, pad[4];
    const void *dense, *bits, *rowptr, *colidx, *vals, *colptr, *rowidx, *succ, *lazy_src;
    uint64_t csr_stamp, succ_stamp, lazy_stamp;
};

struct CtxSnap {
    const void* ws[4];
    size_t ws_cap[4];
    const void* aux;
    size_t aux_cap;
};

std::vector<uint8_t> snapshot(tl_ctx* c) {
    std::vector<uint8_t> out;
    CtxSnap cs;
    memset(&cs, 0, sizeof cs);
    for (int i = 0; i < 4; ++i) { cs.ws[i] = c->ws[i]; cs.ws_cap[i] = c->ws_cap[i]; }
    cs.aux = c->aux;
    cs.aux_cap = c->aux_cap;
    out.insert(out.end(), (const uint8_t*)&cs, (const uint8_t*)&cs + sizeof cs);
    for (auto& kv : c->tensors) {
        const Tensor* t = kv.second.get();
        TensorSnap z;
        memset(&z, 0, sizeof z);
        snprintf(z.name, sizeof z.name, "%s", kv.first.c_str());
        z.rank = t->rank; z.shard = t->shard; z.succ_sentinel = t->succ_sentinel;
        for (int k = 0; k < TL_MAX_RANK; ++k) z.dims[k] = t->dims[k];
        z.total = t->total; z.dense_elems = t->dense_elems; z.bits_words = t->bits_words; z.bits_rows = t->bits_rows;
        z.nnz = t->nnz; z.csr_cap = t->csr_cap; z.csr_rows = t->csr_rows; z.csc_cap = t->csc_cap;
        z.succ_cap = t->succ_cap; z.succ_nodes = t->succ_nodes;
        z.defined = t->defined; z.zero = t->zero; z.boolean = t->boolean; z.is_sparse = t->is_sparse;
        z.dense_valid = t->dense_valid; z.bits_valid = t->bits_valid; z.csr_valid = t->csr_valid;
        z.csc_valid = t->csc_valid; z.csr_nonneg = t->csr_nonneg; z.csr_ones = t->csr_ones; z.csr_pos = t->csr_pos;
        z.nonneg = t->nonneg;
        z.dense = t->dense; z.bits = t->bits; z.rowptr = t->rowptr; z.colidx = t->colidx; z.vals = t->vals;
        z.colptr = t->colptr; z.rowidx = t->rowidx; z.succ = t->succ; z.lazy_src = t->lazy_src;
        z.csr_stamp = t->csr_stamp; z.succ_stamp = t->succ_stamp; z.lazy_stamp = t->lazy_stamp;
        out.insert(out.end(), (const uint8_t*)&z, (const uint8_t*)&z + sizeof z);
    }
    return out;
}

// Puts the flags of a snapshot back (storages are the same by construction);
// tensors the snapshot does not know become absent logical zeros.
void apply_snapshot(tl_ctx* c, const std::vector<uint8_t>& snap) {
    // the usual case: the same tensors in the same (name) order
    const size_t n_snap = snap.size() >= sizeof(CtxSnap) ? (snap.size() - sizeof(CtxSnap)) / sizeof(TensorSnap) : 0;
    std::vector<const TensorSnap*> pos;
    if (n_snap == c->tensors.size()) {
        size_t i = 0;
        for (auto& kv : c->tensors) {
            const TensorSnap* z = reinterpret_cast<const TensorSnap*>(snap.data() + sizeof(CtxSnap) + i * sizeof(TensorSnap));
            if (strncmp(z->name, kv.first.c_str(), sizeof z->name) != 0) break;
            pos.push_back(z);
            ++i;
        }
        if (pos.size() != n_snap) pos.clear();
    }
    std::map<std::string, const TensorSnap*> by;
    if (pos.empty())
        for (size_t off = sizeof(CtxSnap); off + sizeof(TensorSnap) <= snap.size(); off += sizeof(TensorSnap)) {
            const TensorSnap* z = reinterpret_cast<const TensorSnap*>(snap.data() + off);
            by[z->name] = z;
        }
    size_t i = 0;
    for (auto& kv : c->tensors) {
        Tensor* t = kv.second.get();
        const TensorSnap* found = nullptr;
        if (!pos.empty()) {
            found = pos[i++];
        } else {
            auto it = by.find(kv.first);
            if (it != by.end()) found = it->second;
        }
        if (!found) {
            t->defined = false; t->zero = true;
            t->dense_valid = t->bits_valid = t->csr_valid = t->csc_valid = false;
            t->lazy_src = nullptr;
            continue;
        }
        const TensorSnap* z = found;
        t->defined = z->defined; t->zero = z->zero; t->boolean = z->boolean; t->is_sparse = z->is_sparse;
        t->dense_valid = z->dense_valid; t->bits_valid = z->bits_valid; t->csr_valid = z->csr_valid;
        t->csc_valid = z->csc_valid; t->csr_nonneg = z->csr_nonneg; t->csr_ones = z->csr_ones; t->csr_pos = z->csr_pos;
        t->nonneg = z->nonneg;
        t->nnz = z->nnz; t->csr_rows = z->csr_rows; t->csr_stamp = z->csr_stamp; t->succ_stamp = z->succ_stamp;
        t->succ_nodes = z->succ_nodes; t->succ_sentinel = z->succ_sentinel;
        t->lazy_src = const_cast<Tensor*>(static_cast<const Tensor*>(z->lazy_src));
        t->lazy_stamp = z->lazy_stamp;
    }
}

bool graphable(tl_ctx* c, const tl_statement* s, int n) {
    if (c->prof || c->world > 1 || getenv("TL_NO_GRAPHS")) return false;
    for (int i = 0; i < n; ++i) {
        const tl_statement* st = &s[i];
        switch (st->kind) {
        case TL_STMT_QUERY: case TL_STMT_SAVE: return false;
        case TL_STMT_LOAD: if (st->host_data || st->path[0]) return false; break;
        case TL_STMT_SPARSE_LOAD: if (st->coo_rows || st->coo_cols) return false; break;
        case TL_STMT_EQUATION: if (is_recursive(&st->eq)) return false; break;
        default: break;
        }
    }
    return true;
}

}  // namespace

void tl::release_graphs(tl_ctx* c) {
    for (auto& g : c->graphs)
        if (g.exec) cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(g.exec));
    c->graphs.clear();
}

// Replays or captures this run; *done when the run's work is on the stream.
// Replays the graph of a program seen before with the same statement bytes
// from the same host state; *done when it did.  Called before the run's host
// bookkeeping, which then overlaps the graph's work on the GPU.
static tl_status replay_graph(tl_ctx* c, const tl_statement* s, int n, bool* done) {
    *done = false;
    const size_t bytes = (size_t)n * sizeof(tl_statement);
    GraphEntry* e = nullptr;
    for (auto& g : c->graphs)
        if (g.exec && !g.failed && g.stmts_at == s && g.stmts.size() == bytes && memcmp(g.stmts.data(), s, bytes) == 0) {
            e = &g;
            break;
        }
    if (!e || e->begin != snapshot(c)) return TL_OK;
    e->used = ++c->graph_clock;
    TL_CK(c, cudaGraphLaunch(static_cast<cudaGraphExec_t>(e->exec), c->stream));
    c->flags_armed = true;   // the graph may hold tensor-core GEMMs
    apply_snapshot(c, e->end);
    c->launches += e->launches;
    c->stats["program_graph_replay"].launches++;   // visible through tl_profile_read
    *done = true;
    return TL_OK;
}

static tl_status run_as_graph(tl_ctx* c, const tl_statement* s, int n, const std::vector<tl_equation>& eqs,
                              bool* done) {
    *done = false;
    // the same statement array with the same bytes (a memcmp, not a hash: the
    // statements are several KB each)
    const size_t bytes = (size_t)n * sizeof(tl_statement);
    std::vector<uint8_t> begin = snapshot(c);
    GraphEntry* e = nullptr;
    for (auto& g : c->graphs)
        if (g.stmts_at == s && g.stmts.size() == bytes && memcmp(g.stmts.data(), s, bytes) == 0) e = &g;
    if (!e) {
        if (c->graphs.size() >= 8) {   // drop the least recently used
            auto old = std::min_element(c->graphs.begin(), c->graphs.end(),
                                        [](const GraphEntry& a, const GraphEntry& b) { return a.used < b.used; });
            if (old->exec) cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(old->exec));
            c->graphs.erase(old);
        }
        c->graphs.emplace_back();
        e = &c->graphs.back();
        e->stmts_at = s;
        e->stmts.assign(reinterpret_cast<const uint8_t*>(s), reinterpret_cast<const uint8_t*>(s) + bytes);
    }
    e->used = ++c->graph_clock;
    if (e->failed) return TL_OK;
    if (e->exec && e->begin == begin) {
        TL_CK(c, cudaGraphLaunch(static_cast<cudaGraphExec_t>(e->exec), c->stream));
        c->flags_armed = true;   // the graph may hold tensor-core GEMMs
        apply_snapshot(c, e->end);
        c->launches += e->launches;
        c->stats["program_graph_replay"].launches++;   // visible through tl_profile_read
        *done = true;
        return TL_OK;
    }
    if (e->last_begin != begin) {   // not repeated yet: run eagerly, remember the state
        if (getenv("TL_GRAPH_DEBUG") && !e->last_begin.empty()) {
            size_t i = 0;
            while (i < begin.size() && i < e->last_begin.size() && begin[i] == e->last_begin[i]) ++i;
            const size_t t = i < sizeof(CtxSnap) ? (size_t)-1 : (i - sizeof(CtxSnap)) / sizeof(TensorSnap);
            fprintf(stderr, "tl graph: host state differs at byte %zu (%s %s), sizes %zu/%zu\n", i,
                    t == (size_t)-1 ? "context" : "tensor",
                    t == (size_t)-1 ? "" : reinterpret_cast<const TensorSnap*>(begin.data() + sizeof(CtxSnap) +
                                                                           t * sizeof(TensorSnap))->name,
                    begin.size(), e->last_begin.size());
        }
        e->last_begin = begin;
        return TL_OK;
    }
    if (e->exec) {
        cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(e->exec));
        e->exec = nullptr;
    }
    const int64_t launches0 = c->launches;
    if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed) != cudaSuccess) {
        cudaGetLastError();
        e->failed = true;
        return TL_OK;
    }
    std::vector<tl_equation> rec;
    const tl_status st = run_statements(c, s, n, eqs, &rec);
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(c->stream, &g);
    cudaGraphExec_t x = nullptr;
    bool ok = st == TL_OK && ce == cudaSuccess && g && rec.empty();
    if (ok && cudaGraphInstantiate(&x, g, 0) != cudaSuccess) ok = false;
    if (g) cudaGraphDestroy(g);
    if (!ok) {
        // nothing ran: put the state back and run this program eagerly from now on
        if (getenv("TL_GRAPH_DEBUG"))
            fprintf(stderr, "tl graph: capture failed (status %d, %s, %zu recursive): %s\n", (int)st,
                    cudaGetErrorString(ce), rec.size(), c->err.c_str());
        cudaGetLastError();
        if (x) cudaGraphExecDestroy(x);
        apply_snapshot(c, begin);
        c->launches = launches0;
        c->err.clear();
        e->failed = true;
        return TL_OK;
    }
    e->exec = x;
    e->begin = begin;
    e->end = snapshot(c);
    e->launches = c->launches - launches0;
    TL_CK(c, cudaGraphLaunch(x, c->stream));
    c->flags_armed = true;
    *done = true;
    return TL_OK;
}

static bool is_constant_query(const tl_ref& q) {
    for (int k = 0; k < q.rank; ++k)
        if (q.idx[k].kind == TL_IX_CONST) return true;
    return false;
}

extern "C" tl_status tl_program_run(tl_ctx* c, const tl_statement* s, int32_t n) {
    if (!c || (n > 0 && !s)) return TL_ERR_INVALID;
    TL_CK(c, cudaSetDevice(c->device));
    TL_TRY(fix_resolve(c));   // an earlier run's fixpoint result, before last_sweeps is reset
    c->err.clear();
    c->query_out.clear();
    // a fresh run: every tensor is absent until its first definition
    for (auto& kv : c->tensors) kv.second->defined = false;
    // a repeating program replays its graph first; the bookkeeping below then
    // runs while the graph works
    const bool can_graph = graphable(c, s, n);
    bool replayed = false;
    if (can_graph) TL_TRY(replay_graph(c, s, n, &replayed));
    c->domains.clear();   // a program's domains are its own (llvm.zig:133-140)
    c->maxdims.clear();
    for (int i = 0; i < n; ++i)
        if (s[i].kind == TL_STMT_DOMAIN) TL_TRY(tl_domain(c, s[i].name, s[i].size));
    std::vector<tl_equation> eqs, rec;
    for (int i = 0; i < n; ++i)
        if (s[i].kind == TL_STMT_EQUATION) eqs.push_back(s[i].eq);
    TL_TRY(tl_declare_dims(c, eqs.data(), (int)eqs.size()));
    // the globals of constant-index queries exist before the program runs
    struct BqReset {
        tl_ctx* c;
        ~BqReset() { bq_release(c); }
    } bq_reset{c};
    TL_TRY(bq_prepare(c, s, n));
    // sign-sensitive tensors: step / comparison arguments, and relu arguments
    // when a backward pass will take relu's gradient step(x)
    bool has_backward = false;
    for (int i = 0; i < n; ++i) has_backward = has_backward || s[i].kind == TL_STMT_BACKWARD;
    c->sign_sensitive.clear();
    for (const tl_equation& e : eqs) {
        for (int i = 1; i < e.n_code && i < TL_MAX_CODE; ++i) {
            const tl_instr& in = e.code[i];
            const bool tests_sign = (in.op == TL_OP_NL && (in.arg == TL_NL_STEP || (in.arg == TL_NL_RELU && has_backward))) ||
                                    (in.op >= TL_OP_GT && in.op <= TL_OP_NE);
            if (!tests_sign) continue;
            for (int back = 1; back <= 2 && i - back >= 0; ++back) {
                const tl_instr& prev = e.code[i - back];
                if (prev.op == TL_OP_REF && prev.arg >= 0 && prev.arg < e.n_refs)
                    c->sign_sensitive.push_back(e.refs[prev.arg].tensor);
                if (in.op == TL_OP_NL) break;   // unary: only the direct operand
            }
        }
    }
    struct LazyReset {
        tl_ctx* c;
        ~LazyReset() { c->lazy_eq = nullptr; }
    } lazy_reset{c};
    c->lazy_eq = lazy_step_equation(s, n);
    if (can_graph && !replayed) TL_TRY(run_as_graph(c, s, n, eqs, &replayed));
    if (!replayed) TL_TRY(run_statements(c, s, n, eqs, &rec));
    c->lazy_eq = nullptr;
    c->last_sweeps = 0;
    if (!rec.empty()) TL_TRY(run_fixpoint(c, rec.data(), (int)rec.size(), nullptr));
    // queries in statement order (llvm.zig:309-318): a constant-index query
    // prints the backward-chaining value (backward.zig:568-600)
    std::vector<double> backward_values;
    TL_TRY(bq_run(c, s, n, &backward_values));
    size_t next_backward = 0;
    for (int i = 0; i < n; ++i) {
        if (s[i].kind != TL_STMT_QUERY) continue;
        if (next_backward < backward_values.size() && is_constant_query(s[i].sparse)) {
            char line[64 + TL_NAME_LEN];
            snprintf(line, sizeof line, "%s = %.6g\n", s[i].name, backward_values[next_backward++]);
            c->query_out += line;
            if (c->opts.verbose) fputs(line, stdout);
            continue;
        }
        Tensor* t = find_defined(c, s[i].name);
        if (!t) continue;
        std::vector<char> buf(64 + 20 * 32 + strlen(s[i].name));
        TL_TRY(tl_query_format(static_cast<tl_tensor*>(t), buf.data(), (int64_t)buf.size()));
        c->query_out += buf.data();
        if (c->opts.verbose) fputs(buf.data(), stdout);
    }
    // the device error word of a tensor-core pipeline stays set until read:
    // the next call that waits for the device anyway (tl_sync, a download)
    // reports it, so the run returns as soon as its work is queued
    return TL_OK;
}
