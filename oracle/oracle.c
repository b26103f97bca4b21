/*
 * oracle.c — f64 CPU restatement of the Tensor Logic reference's hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA backend's parity tests
 * and the timed CPU baseline.  The product never links or calls this file.
 *
 * Every routine restates a reference codegen routine (path:line inside the
 * Zollicoff/tensor_logic_lang project) as a direct f64 loop nest, so the
 * values it computes are the values the reference's emitted program computes.
 * Where the reference has undefined behaviour (reads or writes outside a
 * tensor's allocation) the oracle reads 0.0 and skips the write.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define MAX_TENSORS 512
#define MAX_DOMAINS 128
#define MAX_VARS 16

typedef struct {
    char name[TL_NAME_LEN];
    int32_t rank;
    int64_t dims[TL_MAX_RANK];
    int64_t strides[TL_MAX_RANK];
    int64_t total;
    double* data;
} or_tensor;

typedef struct {
    char name[TL_NAME_LEN];
    int32_t rank;
    int64_t dims[TL_MAX_RANK];
} or_maxdims;

/* A global the backward-chaining infrastructure allocates before main
 * (llvm.zig:231-260, tensor.zig:157-220): the queried tensors and the
 * left-hand sides their equations read. */
#define MAX_BW 64
#define BW_MAX_DEPTH 4096
typedef struct {
    char name[TL_NAME_LEN];
    int32_t rank;
    int64_t dims[TL_MAX_RANK];
    int64_t strides[TL_MAX_RANK];
    int64_t total;
    int32_t compute;          /* queried with a constant index: @compute_T */
    int32_t n_eq;
    int32_t* eq_stmt;         /* statement indices of T's equations, program order */
    double* memo;             /* @memo_T */
    unsigned char* done;      /* @memo_T_computed */
    int32_t detached;         /* a `sparse` re-declaration replaced the forward tensor */
    double* snap;             /* what the global held at that point */
} bw_global;

struct or_ctx {
    int32_t max_sweeps;
    int32_t last_sweeps;
    int32_t n_tensors;
    or_tensor tensors[MAX_TENSORS];
    int32_t n_domains;
    char dom_names[MAX_DOMAINS][TL_NAME_LEN];
    int64_t dom_sizes[MAX_DOMAINS];
    int32_t n_maxdims;
    or_maxdims maxdims[MAX_TENSORS];
    char* qout;
    size_t qlen, qcap;
    char err[256];
    int32_t n_bw;
    bw_global bw[MAX_BW];
    const tl_statement* bw_stmts;
    int32_t bw_depth;
    int32_t bw_err;
};

/* ------------------------------------------------------------------------ */
/* Registry                                                                   */
/* ------------------------------------------------------------------------ */
static or_tensor* find_tensor(or_ctx* c, const char* name) {
    for (int i = 0; i < c->n_tensors; ++i)
        if (strcmp(c->tensors[i].name, name) == 0) return &c->tensors[i];
    return NULL;
}

/* domains.get(name) orelse 10 (llvm.zig:407,435; expr.zig:309). */
static int64_t domain_size(or_ctx* c, const char* name) {
    for (int i = 0; i < c->n_domains; ++i)
        if (strcmp(c->dom_names[i], name) == 0) return c->dom_sizes[i];
    return 10;
}

static void put_domain(or_ctx* c, const char* name, int64_t size) {
    for (int i = 0; i < c->n_domains; ++i)
        if (strcmp(c->dom_names[i], name) == 0) { c->dom_sizes[i] = size; return; }
    if (c->n_domains < MAX_DOMAINS) {
        snprintf(c->dom_names[c->n_domains], TL_NAME_LEN, "%s", name);
        c->dom_sizes[c->n_domains++] = size;
    }
}

/* Size an index contributes to a tensor's dims (tensor.zig:93-126). */
static int64_t index_extent(or_ctx* c, const tl_index* ix) {
    switch (ix->kind) {
    case TL_IX_NAME: case TL_IX_NORMALIZE: case TL_IX_PRIMED: case TL_IX_ADD: case TL_IX_SUB:
        return domain_size(c, ix->name);
    case TL_IX_CONST: return ix->value + 1;
    case TL_IX_DIV: { int64_t b = domain_size(c, ix->name); return (b + ix->value - 1) / ix->value; }
    case TL_IX_SLICE: return ix->value2 > ix->value ? ix->value2 - ix->value : 1;
    default: return 10;
    }
}

/* updateTensorMaxDims (tensor.zig:84-129). */
static void update_max_dims(or_ctx* c, const tl_ref* lhs) {
    if (lhs->rank == 0) return;
    for (int i = 0; i < c->n_maxdims; ++i) {
        or_maxdims* m = &c->maxdims[i];
        if (strcmp(m->name, lhs->tensor) == 0) {
            for (int k = 0; k < lhs->rank && k < m->rank; ++k) {
                int64_t s = index_extent(c, &lhs->idx[k]);
                if (s > m->dims[k]) m->dims[k] = s;
            }
            return;
        }
    }
    if (c->n_maxdims >= MAX_TENSORS) return;
    or_maxdims* m = &c->maxdims[c->n_maxdims++];
    snprintf(m->name, TL_NAME_LEN, "%s", lhs->tensor);
    m->rank = lhs->rank;
    for (int k = 0; k < lhs->rank; ++k) m->dims[k] = index_extent(c, &lhs->idx[k]);
}

static or_tensor* new_tensor(or_ctx* c, const char* name, int32_t rank, const int64_t* dims) {
    or_tensor* t = find_tensor(c, name);
    if (!t) {
        if (c->n_tensors >= MAX_TENSORS) return NULL;
        t = &c->tensors[c->n_tensors++];
        snprintf(t->name, TL_NAME_LEN, "%s", name);
    } else {
        free(t->data);
    }
    if (rank == 0) { rank = 1; t->dims[0] = 1; }
    else for (int k = 0; k < rank; ++k) t->dims[k] = dims[k];
    t->rank = rank;
    int64_t s = 1;
    for (int k = rank - 1; k >= 0; --k) { t->strides[k] = s; s *= t->dims[k]; }
    t->total = s;
    t->data = (double*)calloc((size_t)(s > 0 ? s : 1), sizeof(double));
    return t;
}

/* allocateTensor (tensor.zig:14-81): max dims when known, else per index. */
static or_tensor* allocate_tensor(or_ctx* c, const char* name, const tl_index* idx, int32_t n) {
    int64_t dims[TL_MAX_RANK];
    for (int i = 0; i < c->n_maxdims; ++i) {
        if (strcmp(c->maxdims[i].name, name) == 0)
            return new_tensor(c, name, c->maxdims[i].rank, c->maxdims[i].dims);
    }
    for (int k = 0; k < n; ++k) {
        /* the fallback path has no .normalize case (tensor.zig:25-47) */
        dims[k] = idx[k].kind == TL_IX_NORMALIZE ? 10 : index_extent(c, &idx[k]);
    }
    return new_tensor(c, name, n, dims);
}

static double tread(const or_tensor* t, int64_t off) {
    return (off >= 0 && off < t->total) ? t->data[off] : 0.0;
}

/* ------------------------------------------------------------------------ */
/* Expression evaluation (expr.zig:14-300)                                   */
/* ------------------------------------------------------------------------ */
typedef struct {
    int32_t n;
    char names[MAX_VARS][TL_NAME_LEN + 2];
    int64_t sizes[MAX_VARS];
    int32_t contracted[MAX_VARS];
} var_list;

static int var_find(const var_list* v, const char* name) {
    for (int i = 0; i < v->n; ++i) if (strcmp(v->names[i], name) == 0) return i;
    return -1;
}

static void primed_name(char* out, const char* base) { snprintf(out, TL_NAME_LEN + 2, "%s'", base); }

typedef struct {
    const or_tensor* t[TL_MAX_REFS];        /* NULL: not allocated → reads 0.0 */
    int32_t nix[TL_MAX_REFS];
    /* per ref, per index: kind, var id or -1, value */
    int32_t kind[TL_MAX_REFS][TL_MAX_RANK];
    int32_t var[TL_MAX_REFS][TL_MAX_RANK];
    int64_t val[TL_MAX_REFS][TL_MAX_RANK];
    const or_tensor* virt[TL_MAX_REFS][TL_MAX_RANK];
    int32_t virt_pos_var;                    /* loop var used as gather position */
} access_plan;

static void plan_access(or_ctx* c, const tl_equation* eq, const var_list* v, access_plan* p) {
    p->virt_pos_var = v->n > 0 ? 0 : -1;
    for (int r = 0; r < eq->n_refs; ++r) {
        const tl_ref* ref = &eq->refs[r];
        p->t[r] = find_tensor(c, ref->tensor);
        p->nix[r] = ref->rank;
        for (int k = 0; k < ref->rank; ++k) {
            const tl_index* ix = &ref->idx[k];
            char pn[TL_NAME_LEN + 2];
            p->kind[r][k] = ix->kind;
            p->val[r][k] = ix->value;
            p->var[r][k] = -1;
            p->virt[r][k] = NULL;
            switch (ix->kind) {
            case TL_IX_NAME: case TL_IX_ADD: case TL_IX_SUB: case TL_IX_DIV:
                p->var[r][k] = var_find(v, ix->name); break;
            case TL_IX_PRIMED:
                primed_name(pn, ix->name); p->var[r][k] = var_find(v, pn); break;
            case TL_IX_VIRTUAL:
                p->virt[r][k] = find_tensor(c, ix->name); break;
            default: break;
            }
        }
    }
}

/* genTensorAccess (expr.zig:48-157): one index value per position. */
static double load_ref(const access_plan* p, int r, const int64_t* iv) {
    const or_tensor* t = p->t[r];
    if (!t) return 0.0;
    int64_t off = 0;
    int n = p->nix[r] < t->rank ? p->nix[r] : t->rank;
    for (int k = 0; k < n; ++k) {
        int64_t x = 0;
        int var = p->var[r][k];
        switch (p->kind[r][k]) {
        case TL_IX_NAME: case TL_IX_PRIMED: x = var >= 0 ? iv[var] : 0; break;
        case TL_IX_CONST: x = p->val[r][k]; break;
        case TL_IX_ADD: x = var >= 0 ? iv[var] + p->val[r][k] : p->val[r][k]; break;
        case TL_IX_SUB: x = var >= 0 ? iv[var] - p->val[r][k] : p->val[r][k]; break;
        case TL_IX_DIV: x = var >= 0 ? iv[var] / p->val[r][k] : 0; break;
        case TL_IX_SLICE: x = p->val[r][k]; break;
        case TL_IX_VIRTUAL: {
            const or_tensor* vt = p->virt[r][k];
            if (vt && p->virt_pos_var >= 0) x = (int64_t)tread(vt, iv[p->virt_pos_var]);
            else x = 0;
            break;
        }
        default: x = 0; break;
        }
        off += x * t->strides[k];
    }
    return tread(t, off);
}

/* genNonlinearity (expr.zig:240-300). */
static double apply_nl(int32_t f, double x, int has_temp, double temp) {
    switch (f) {
    case TL_NL_RELU: return x > 0.0 ? x : 0.0;
    case TL_NL_SIGMOID: {
        double s = has_temp ? -(x / temp) : -x;
        return 1.0 / (1.0 + exp(s));
    }
    case TL_NL_TANH: { double e = exp(x * 2.0); return (e - 1.0) / (e + 1.0); }
    case TL_NL_STEP: return x > 0.0 ? 1.0 : 0.0;
    case TL_NL_EXP: return exp(x);
    case TL_NL_LOG: return log(x);
    case TL_NL_SQRT: return sqrt(x);
    case TL_NL_ABS: return fabs(x);
    case TL_NL_SIN: return sin(x);
    case TL_NL_COS: return cos(x);
    default: return x + 0.0;     /* norm / unknown: identity (expr.zig:297) */
    }
}

/* genExpr over the postfix program (expr.zig:14-25, 160-237). */
static double eval_rhs(const tl_equation* eq, const access_plan* p, const int64_t* iv) {
    double st[TL_MAX_CODE];
    int sp = 0;
    for (int i = 0; i < eq->n_code; ++i) {
        const tl_instr* in = &eq->code[i];
        switch (in->op) {
        case TL_OP_REF: st[sp++] = load_ref(p, in->arg, iv); break;
        case TL_OP_LIT: st[sp++] = in->value; break;
        case TL_OP_PROD: {
            int n = in->arg;
            double acc = st[sp - n];
            for (int k = 1; k < n; ++k) acc = acc * st[sp - n + k];
            sp -= n;
            st[sp++] = acc;
            break;
        }
        case TL_OP_NEG: st[sp - 1] = -st[sp - 1]; break;
        case TL_OP_NOT: st[sp - 1] = (st[sp - 1] == 0.0) ? 1.0 : 0.0; break;
        case TL_OP_NL: st[sp - 1] = apply_nl(in->arg, st[sp - 1], in->arg2, in->value); break;
        default: {
            double b = st[--sp];
            double a = st[sp - 1];
            double r;
            switch (in->op) {
            case TL_OP_ADD: r = a + b; break;
            case TL_OP_SUB: r = a - b; break;
            case TL_OP_MUL: r = a * b; break;
            case TL_OP_DIV: r = a / b; break;
            case TL_OP_POW: r = pow(a, b); break;
            case TL_OP_GT: r = a > b; break;
            case TL_OP_LT: r = a < b; break;
            case TL_OP_GE: r = a >= b; break;
            case TL_OP_LE: r = a <= b; break;
            case TL_OP_EQ: r = a == b; break;
            case TL_OP_NE: r = (a < b) || (a > b); break;  /* fcmp one */
            default: r = a + b; break;                      /* & | → fadd */
            }
            st[sp - 1] = r;
        }
        }
    }
    return sp > 0 ? st[sp - 1] : 0.0;
}

/* collectExprIndices (expr.zig:303-359), in expression order. */
static void collect_rhs_vars(or_ctx* c, const tl_equation* eq, var_list* all) {
    for (int r = 0; r < eq->n_refs; ++r) {
        const tl_ref* ref = &eq->refs[r];
        for (int k = 0; k < ref->rank; ++k) {
            const tl_index* ix = &ref->idx[k];
            char nm[TL_NAME_LEN + 2];
            int64_t size;
            switch (ix->kind) {
            case TL_IX_NAME: case TL_IX_ADD: case TL_IX_SUB: case TL_IX_DIV:
                snprintf(nm, sizeof nm, "%s", ix->name); size = domain_size(c, ix->name); break;
            case TL_IX_PRIMED:
                primed_name(nm, ix->name); size = domain_size(c, ix->name); break;
            case TL_IX_SLICE:
                snprintf(nm, sizeof nm, "_slice_%lld_%lld", (long long)ix->value, (long long)ix->value2);
                size = ix->value2 > ix->value ? ix->value2 - ix->value : 1; break;
            default: continue;
            }
            int at = var_find(all, nm);
            if (at < 0 && all->n < MAX_VARS) {
                at = all->n++;
                snprintf(all->names[at], TL_NAME_LEN + 2, "%s", nm);
            }
            if (at >= 0) all->sizes[at] = size;     /* put overwrites */
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Equations (llvm.zig:357-459, einsum.zig:20-278)                           */
/* ------------------------------------------------------------------------ */
static int rowwise(or_ctx* c, const tl_equation* eq, int is_lnorm);

static int rhs_root_is(const tl_equation* eq, int nl) {
    return eq->n_code > 0 && eq->code[eq->n_code - 1].op == TL_OP_NL && eq->code[eq->n_code - 1].arg == nl;
}

static int gen_equation(or_ctx* c, const tl_equation* eq) {
    if (rhs_root_is(eq, TL_NL_SOFTMAX)) return rowwise(c, eq, 0);
    if (rhs_root_is(eq, TL_NL_LNORM)) return rowwise(c, eq, 1);
    if (rhs_root_is(eq, TL_NL_CONCAT)) {
        snprintf(c->err, sizeof c->err, "concat is not lowered");
        return TL_ERR_UNSUPPORTED;
    }
    or_tensor* lhs = find_tensor(c, eq->lhs.tensor);
    if (!lhs) lhs = allocate_tensor(c, eq->lhs.tensor, eq->lhs.idx, eq->lhs.rank);
    if (!lhs) return TL_ERR_OOM;

    /* index analysis (llvm.zig:383-455) */
    var_list all; memset(&all, 0, sizeof all);
    char lhs_set[TL_MAX_RANK][TL_NAME_LEN + 2];
    int n_lhs_set = 0;
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        char nm[TL_NAME_LEN + 2];
        if (ix->kind == TL_IX_NAME || ix->kind == TL_IX_NORMALIZE || ix->kind == TL_IX_DIV)
            snprintf(nm, sizeof nm, "%s", ix->name);
        else if (ix->kind == TL_IX_PRIMED) primed_name(nm, ix->name);
        else continue;
        snprintf(lhs_set[n_lhs_set++], TL_NAME_LEN + 2, "%s", nm);
        int at = var_find(&all, nm);
        if (at < 0) { at = all.n++; snprintf(all.names[at], TL_NAME_LEN + 2, "%s", nm); }
        all.sizes[at] = domain_size(c, ix->name);
    }
    collect_rhs_vars(c, eq, &all);

    access_plan plan;
    if (all.n == 0) {
        /* genScalarAssign (einsum.zig:257-278) */
        var_list none; memset(&none, 0, sizeof none);
        plan_access(c, eq, &none, &plan);
        double v = eval_rhs(eq, &plan, NULL);
        int64_t off = 0;
        for (int k = 0; k < eq->lhs.rank && k < lhs->rank; ++k)
            off += (eq->lhs.idx[k].kind == TL_IX_CONST ? eq->lhs.idx[k].value : 0) * lhs->strides[k];
        if (off >= 0 && off < lhs->total) lhs->data[off] = v;
        return TL_OK;
    }

    /* loop variables: free (LHS order) then contracted (first appearance) */
    var_list v; memset(&v, 0, sizeof v);
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        char nm[TL_NAME_LEN + 2];
        if (ix->kind == TL_IX_NAME || ix->kind == TL_IX_DIV) snprintf(nm, sizeof nm, "%s", ix->name);
        else if (ix->kind == TL_IX_PRIMED) primed_name(nm, ix->name);
        else continue;
        int at = var_find(&all, nm);
        snprintf(v.names[v.n], TL_NAME_LEN + 2, "%s", nm);
        v.sizes[v.n] = at >= 0 ? all.sizes[at] : 10;
        v.contracted[v.n++] = 0;
    }
    int has_contraction = 0;
    for (int i = 0; i < all.n; ++i) {
        int in_lhs = 0;
        for (int k = 0; k < n_lhs_set; ++k) if (strcmp(lhs_set[k], all.names[i]) == 0) in_lhs = 1;
        if (in_lhs) continue;
        snprintf(v.names[v.n], TL_NAME_LEN + 2, "%s", all.names[i]);
        v.sizes[v.n] = all.sizes[i];
        v.contracted[v.n++] = 1;
        has_contraction = 1;
    }

    /* LHS address terms (einsum.zig:87-123): one value per name/primed/div
     * index, paired with strides in order of emission. */
    int lhs_var[TL_MAX_RANK]; int64_t lhs_div[TL_MAX_RANK]; int n_lhs_terms = 0;
    int64_t avg_div = 1;
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        char nm[TL_NAME_LEN + 2];
        if (ix->kind == TL_IX_NAME) snprintf(nm, sizeof nm, "%s", ix->name);
        else if (ix->kind == TL_IX_PRIMED) primed_name(nm, ix->name);
        else if (ix->kind == TL_IX_DIV) { snprintf(nm, sizeof nm, "%s", ix->name); avg_div *= ix->value; }
        else continue;
        int at = var_find(&v, nm);
        if (at < 0) continue;
        lhs_var[n_lhs_terms] = at;
        lhs_div[n_lhs_terms++] = ix->kind == TL_IX_DIV ? ix->value : 1;
    }
    plan_access(c, eq, &v, &plan);

    int64_t iv[MAX_VARS];
    for (int i = 0; i < v.n; ++i) { iv[i] = 0; if (v.sizes[i] <= 0) goto avg_pass; }
    for (;;) {
        int64_t off = 0;
        for (int t = 0; t < n_lhs_terms && t < lhs->rank; ++t)
            off += (iv[lhs_var[t]] / lhs_div[t]) * lhs->strides[t];
        double rhs = eval_rhs(eq, &plan, iv);
        if (off >= 0 && off < lhs->total) {
            double* d = &lhs->data[off];
            switch (eq->accum) {
            case TL_ACC_ASSIGN: *d = has_contraction ? *d + rhs : rhs; break;
            case TL_ACC_ADD: case TL_ACC_AVG: *d = *d + rhs; break;
            case TL_ACC_MAX: *d = (rhs > *d) ? rhs : *d; break;
            case TL_ACC_MIN: *d = (rhs < *d) ? rhs : *d; break;
            case TL_ACC_MUL: *d = *d * rhs; break;
            }
        }
        int k = v.n - 1;
        while (k >= 0) {
            if (++iv[k] < v.sizes[k]) break;
            iv[k] = 0;
            --k;
        }
        if (k < 0) break;
    }
avg_pass:
    if (eq->accum == TL_ACC_AVG && avg_div > 1)
        for (int64_t i = 0; i < lhs->total; ++i) lhs->data[i] = lhs->data[i] / (double)avg_div;
    return TL_OK;
}

/* genSoftmax (softmax.zig:19-229) and genLayerNorm (layernorm.zig:25-310):
 * the input is indexed with the LHS's index positions. */
static int rowwise(or_ctx* c, const tl_equation* eq, int is_lnorm) {
    if (eq->n_code != 2 || eq->code[0].op != TL_OP_REF) return TL_OK;   /* F3: comment + return */
    int norm_axis = -1;
    for (int k = 0; k < eq->lhs.rank; ++k)
        if (eq->lhs.idx[k].kind == TL_IX_NORMALIZE) { norm_axis = k; break; }
    if (norm_axis < 0 && eq->lhs.rank > 0) norm_axis = eq->lhs.rank - 1;
    or_tensor* out = find_tensor(c, eq->lhs.tensor);
    if (!out) out = allocate_tensor(c, eq->lhs.tensor, eq->lhs.idx, eq->lhs.rank);
    or_tensor* in = find_tensor(c, eq->refs[0].tensor);
    if (!in || !out) return TL_OK;

    /* outer dims: LHS name/normalize indices other than the norm axis */
    int pos[TL_MAX_RANK]; int64_t size[TL_MAX_RANK]; int n_outer = 0;
    int64_t norm_size = 1;
    char names[TL_MAX_RANK][TL_NAME_LEN];
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        if (ix->kind != TL_IX_NAME && ix->kind != TL_IX_NORMALIZE) continue;
        int64_t s = domain_size(c, ix->name);
        if (k == norm_axis) norm_size = s;
        else { pos[n_outer] = k; size[n_outer] = s; snprintf(names[n_outer], TL_NAME_LEN, "%s", ix->name); n_outer++; }
    }
    /* per LHS position: which loop value feeds it (computeSoftmaxOffset) */
    int src[TL_MAX_RANK];   /* -2: skip, -1: norm var, >=0: outer var */
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        src[k] = -2;
        if (ix->kind != TL_IX_NAME && ix->kind != TL_IX_NORMALIZE) continue;
        if (k == norm_axis) { src[k] = -1; continue; }
        for (int o = 0; o < n_outer; ++o) if (strcmp(names[o], ix->name) == 0) { src[k] = o; break; }
    }
    int64_t ov[TL_MAX_RANK] = {0};
    for (int o = 0; o < n_outer; ++o) if (size[o] <= 0) return TL_OK;
    (void)pos;
    for (;;) {
        #define OFFSET(T, J) ({ int64_t _o = 0; \
            for (int _k = 0; _k < eq->lhs.rank && _k < (T)->rank; ++_k) { \
                if (src[_k] == -2) continue; \
                _o += (src[_k] == -1 ? (J) : ov[src[_k]]) * (T)->strides[_k]; } _o; })
        if (!is_lnorm) {
            double sum = 0.0;
            for (int64_t j = 0; j < norm_size; ++j) sum = sum + exp(tread(in, OFFSET(in, j)));
            for (int64_t j = 0; j < norm_size; ++j) {
                double y = exp(tread(in, OFFSET(in, j))) / sum;
                int64_t o = OFFSET(out, j);
                if (o >= 0 && o < out->total) out->data[o] = y;
            }
        } else {
            double mean = 0.0;
            for (int64_t j = 0; j < norm_size; ++j) mean = mean + tread(in, OFFSET(in, j));
            mean = mean / (double)norm_size;
            double var = 0.0;
            for (int64_t j = 0; j < norm_size; ++j) { double d = tread(in, OFFSET(in, j)) - mean; var = var + d * d; }
            var = var / (double)norm_size;
            double sd = sqrt(var + 1.0e-5);
            for (int64_t j = 0; j < norm_size; ++j) {
                double y = (tread(in, OFFSET(in, j)) - mean) / sd;
                int64_t o = OFFSET(out, j);
                if (o >= 0 && o < out->total) out->data[o] = y;
            }
        }
        #undef OFFSET
        int k = n_outer - 1;
        while (k >= 0) { if (++ov[k] < size[k]) break; ov[k] = 0; --k; }
        if (k < 0) break;
    }
    return TL_OK;
}

/* ------------------------------------------------------------------------ */
/* Fixpoint (fixpoint.zig:21-297)                                            */
/* ------------------------------------------------------------------------ */
static int is_recursive(const tl_equation* eq) {
    for (int r = 0; r < eq->n_refs; ++r)
        if (strcmp(eq->refs[r].tensor, eq->lhs.tensor) == 0) return 1;
    return 0;
}

/* genRecursiveEquation + genRecursiveEinsumLoops (fixpoint.zig:101-297). */
static int recursive_sweep(or_ctx* c, const tl_equation* eq, int* changed) {
    or_tensor* lhs = find_tensor(c, eq->lhs.tensor);
    if (!lhs) lhs = allocate_tensor(c, eq->lhs.tensor, eq->lhs.idx, eq->lhs.rank);
    if (!lhs) return TL_ERR_OOM;
    var_list all; memset(&all, 0, sizeof all);
    char lhs_set[TL_MAX_RANK][TL_NAME_LEN + 2]; int n_lhs_set = 0;
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        if (ix->kind != TL_IX_NAME && ix->kind != TL_IX_NORMALIZE) continue;
        snprintf(lhs_set[n_lhs_set++], TL_NAME_LEN + 2, "%s", ix->name);
        int at = var_find(&all, ix->name);
        if (at < 0) { at = all.n++; snprintf(all.names[at], TL_NAME_LEN + 2, "%s", ix->name); }
        all.sizes[at] = domain_size(c, ix->name);
    }
    collect_rhs_vars(c, eq, &all);
    var_list v; memset(&v, 0, sizeof v);
    int lhs_var[TL_MAX_RANK]; int n_lhs_terms = 0;
    for (int k = 0; k < eq->lhs.rank; ++k) {
        const tl_index* ix = &eq->lhs.idx[k];
        if (ix->kind != TL_IX_NAME && ix->kind != TL_IX_NORMALIZE) continue;
        int at = var_find(&all, ix->name);
        int vi = var_find(&v, ix->name);
        if (vi < 0) {
            vi = v.n++;
            snprintf(v.names[vi], TL_NAME_LEN + 2, "%s", ix->name);
            v.sizes[vi] = at >= 0 ? all.sizes[at] : 10;
        }
        lhs_var[n_lhs_terms++] = vi;
    }
    for (int i = 0; i < all.n; ++i) {
        int in_lhs = 0;
        for (int k = 0; k < n_lhs_set; ++k) if (strcmp(lhs_set[k], all.names[i]) == 0) in_lhs = 1;
        if (in_lhs) continue;
        snprintf(v.names[v.n], TL_NAME_LEN + 2, "%s", all.names[i]);
        v.sizes[v.n] = all.sizes[i];
        v.contracted[v.n++] = 1;
    }
    access_plan plan;
    plan_access(c, eq, &v, &plan);
    int64_t iv[MAX_VARS];
    for (int i = 0; i < v.n; ++i) { iv[i] = 0; if (v.sizes[i] <= 0) return TL_OK; }
    for (;;) {
        int64_t off = 0;
        for (int t = 0; t < n_lhs_terms && t < lhs->rank; ++t) off += iv[lhs_var[t]] * lhs->strides[t];
        double old = tread(lhs, off);
        double rhs = eval_rhs(eq, &plan, iv);
        double nv;
        if (eq->accum == TL_ACC_ADD) { nv = old + rhs; if (nv > old) *changed = 1; }
        else if (eq->accum == TL_ACC_MAX) { nv = (rhs > old) ? rhs : old; if (rhs > old) *changed = 1; }
        else { nv = rhs; *changed = 1; }
        if (off >= 0 && off < lhs->total) lhs->data[off] = nv;
        int k = v.n - 1;
        while (k >= 0) { if (++iv[k] < v.sizes[k]) break; iv[k] = 0; --k; }
        if (k < 0) break;
    }
    return TL_OK;
}

/* ------------------------------------------------------------------------ */
/* Autodiff (autodiff.zig:87-1082, llvm.zig:635-693)                          */
/* ------------------------------------------------------------------------ */
enum { AD_IDENTITY, AD_SCALAR, AD_MATMUL, AD_ADD, AD_MUL, AD_RELU, AD_SIGMOID, AD_TANH,
       AD_SOFTMAX, AD_LNORM, AD_EXP, AD_LOG };
enum { R_PASS, R_MM_LEFT, R_MM_RIGHT, R_MM_SELF, R_RELU, R_SIGMOID, R_SOFTMAX, R_TANH, R_EXP, R_LOG };

typedef struct {
    char out[TL_NAME_LEN];
    int op;
    int n_in;
    char in[TL_MAX_REFS][TL_NAME_LEN];
} ad_node;

typedef struct {
    int rule;
    char out[TL_NAME_LEN + 8];       /* dL_dX */
    char up[TL_NAME_LEN + 8];        /* dL_dY */
    char ops[3][TL_NAME_LEN];
} ad_grad;

/* analyzeExpr (autodiff.zig:116-158): the root decides the op. */
static int root_op(const tl_equation* eq) {
    if (eq->n_code == 0) return AD_IDENTITY;
    const tl_instr* r = &eq->code[eq->n_code - 1];
    switch (r->op) {
    case TL_OP_REF: return AD_IDENTITY;
    case TL_OP_LIT: return AD_SCALAR;
    case TL_OP_PROD: return AD_MATMUL;
    case TL_OP_ADD: return AD_ADD;
    case TL_OP_MUL: return AD_MUL;
    case TL_OP_NL:
        switch (r->arg) {
        case TL_NL_RELU: return AD_RELU; case TL_NL_SIGMOID: return AD_SIGMOID;
        case TL_NL_TANH: return AD_TANH; case TL_NL_SOFTMAX: return AD_SOFTMAX;
        case TL_NL_LNORM: return AD_LNORM; case TL_NL_EXP: return AD_EXP;
        case TL_NL_LOG: return AD_LOG; default: return AD_IDENTITY;
        }
    default: return AD_IDENTITY;
    }
}

typedef struct {
    int n_nodes;
    ad_node nodes[MAX_TENSORS];
    int n_topo;
    char topo[MAX_TENSORS][TL_NAME_LEN];
    int n_grads;
    ad_grad grads[MAX_TENSORS * 2];
} ad_graph;

static ad_node* ad_find(ad_graph* g, const char* name) {
    for (int i = 0; i < g->n_nodes; ++i) if (strcmp(g->nodes[i].out, name) == 0) return &g->nodes[i];
    return NULL;
}

static int is_param(const char* name, const char (*params)[TL_NAME_LEN], int np) {
    for (int i = 0; i < np; ++i) if (strcmp(name, params[i]) == 0) return 1;
    return 0;
}

/* hasPathToParam (autodiff.zig:408-420), with a depth guard: a recursive
 * equation's node lists itself, where the reference recurses without end. */
static int has_path(ad_graph* g, const char* name, const char (*params)[TL_NAME_LEN], int np, int depth) {
    if (is_param(name, params, np)) return 1;
    if (depth > 64) return 0;
    ad_node* n = ad_find(g, name);
    if (!n) return 0;
    for (int i = 0; i < n->n_in; ++i) if (has_path(g, n->in[i], params, np, depth + 1)) return 1;
    return 0;
}

static void topo_visit(ad_graph* g, const char* name, char (*visited)[TL_NAME_LEN], int* nv) {
    for (int i = 0; i < *nv; ++i) if (strcmp(visited[i], name) == 0) return;
    snprintf(visited[(*nv)++], TL_NAME_LEN, "%s", name);
    ad_node* n = ad_find(g, name);
    if (n) for (int i = 0; i < n->n_in; ++i) topo_visit(g, n->in[i], visited, nv);
    snprintf(g->topo[g->n_topo++], TL_NAME_LEN, "%s", name);
}

static void add_grad(ad_graph* g, int rule, const char* input, const char* output,
                     const char* a, const char* b, const char* cc) {
    ad_grad* gr = &g->grads[g->n_grads++];
    gr->rule = rule;
    snprintf(gr->out, sizeof gr->out, "dL_d%s", input);
    snprintf(gr->up, sizeof gr->up, "dL_d%s", output);
    snprintf(gr->ops[0], TL_NAME_LEN, "%s", a ? a : "");
    snprintf(gr->ops[1], TL_NAME_LEN, "%s", b ? b : "");
    snprintf(gr->ops[2], TL_NAME_LEN, "%s", cc ? cc : "");
}

/* genGradients (autodiff.zig:202-390). */
static void gen_gradients(ad_graph* g, const ad_node* n, const char (*params)[TL_NAME_LEN], int np) {
    switch (n->op) {
    case AD_MATMUL:
        if (n->n_in == 2 && strcmp(n->in[0], n->in[1]) == 0) {
            if (has_path(g, n->in[0], params, np, 0)) add_grad(g, R_MM_SELF, n->in[0], n->out, n->in[0], NULL, NULL);
        } else if (n->n_in >= 2) {
            if (has_path(g, n->in[0], params, np, 0)) add_grad(g, R_MM_LEFT, n->in[0], n->out, n->in[0], n->in[1], n->out);
            if (has_path(g, n->in[1], params, np, 0)) add_grad(g, R_MM_RIGHT, n->in[1], n->out, n->in[0], n->in[1], n->out);
        } else {
            for (int i = 0; i < n->n_in; ++i) {
                int dup = 0;
                for (int j = 0; j < i; ++j) if (strcmp(n->in[i], n->in[j]) == 0) dup = 1;
                if (!dup && has_path(g, n->in[i], params, np, 0)) add_grad(g, R_PASS, n->in[i], n->out, n->in[i], NULL, NULL);
            }
        }
        break;
    case AD_ADD: case AD_IDENTITY:
        for (int i = 0; i < n->n_in; ++i)
            if (has_path(g, n->in[i], params, np, 0)) add_grad(g, R_PASS, n->in[i], n->out, n->in[i], NULL, NULL);
        break;
    case AD_RELU: if (n->n_in >= 1 && has_path(g, n->in[0], params, np, 0)) add_grad(g, R_RELU, n->in[0], n->out, n->in[0], NULL, NULL); break;
    case AD_SIGMOID: if (n->n_in >= 1 && has_path(g, n->in[0], params, np, 0)) add_grad(g, R_SIGMOID, n->in[0], n->out, n->in[0], n->out, NULL); break;
    case AD_SOFTMAX: if (n->n_in >= 1 && has_path(g, n->in[0], params, np, 0)) add_grad(g, R_SOFTMAX, n->in[0], n->out, n->in[0], n->out, NULL); break;
    case AD_TANH: if (n->n_in >= 1 && has_path(g, n->in[0], params, np, 0)) add_grad(g, R_TANH, n->in[0], n->out, n->in[0], n->out, NULL); break;
    case AD_EXP: if (n->n_in >= 1 && has_path(g, n->in[0], params, np, 0)) add_grad(g, R_EXP, n->in[0], n->out, n->in[0], n->out, NULL); break;
    case AD_LOG: if (n->n_in >= 1 && has_path(g, n->in[0], params, np, 0)) add_grad(g, R_LOG, n->in[0], n->out, n->in[0], NULL, NULL); break;
    default: break;   /* scalar, mul, lnorm: no rule */
    }
}

/* genGradEquation and the per-rule loops (autodiff.zig:459-1082). */
static void gen_grad_equation(or_ctx* c, const ad_grad* gr) {
    or_tensor* out = find_tensor(c, gr->out);
    if (!out) {
        or_tensor* base = find_tensor(c, gr->out + 4);
        if (base) out = new_tensor(c, gr->out, base->rank, base->dims);
    }
    if (!out) return;
    or_tensor* up = find_tensor(c, gr->up);
    switch (gr->rule) {
    case R_PASS:
        if (!up) return;
        for (int64_t i = 0; i < up->total; ++i) if (i < out->total) out->data[i] += up->data[i];
        return;
    case R_RELU: {
        or_tensor* x = find_tensor(c, gr->ops[0]);
        if (!up || !x) return;
        for (int64_t i = 0; i < up->total; ++i)
            if (i < out->total) out->data[i] += up->data[i] * (tread(x, i) > 0.0 ? 1.0 : 0.0);
        return;
    }
    case R_SIGMOID: case R_TANH: case R_EXP: {
        or_tensor* y = find_tensor(c, gr->ops[1]);
        if (!up || !y) return;
        for (int64_t i = 0; i < up->total; ++i) {
            double yv = tread(y, i), d;
            if (gr->rule == R_SIGMOID) d = yv * (1.0 - yv);
            else if (gr->rule == R_TANH) d = 1.0 - yv * yv;
            else d = yv;
            if (i < out->total) out->data[i] += up->data[i] * d;
        }
        return;
    }
    case R_LOG: {
        or_tensor* x = find_tensor(c, gr->ops[0]);
        if (!up || !x) return;
        for (int64_t i = 0; i < up->total; ++i) if (i < out->total) out->data[i] += up->data[i] / tread(x, i);
        return;
    }
    case R_SOFTMAX: {
        or_tensor* y = find_tensor(c, gr->ops[1]);
        if (!up || !y) return;
        double s = 0.0;
        for (int64_t i = 0; i < up->total; ++i) s = s + up->data[i] * tread(y, i);
        for (int64_t i = 0; i < up->total; ++i)
            if (i < out->total) out->data[i] += tread(y, i) * (up->data[i] - s);
        return;
    }
    case R_MM_SELF: {
        or_tensor* x = find_tensor(c, gr->ops[0]);
        if (!x) return;
        for (int64_t i = 0; i < x->total; ++i) if (i < out->total) out->data[i] += x->data[i] * 2.0;
        return;
    }
    case R_MM_LEFT: {
        or_tensor* b = find_tensor(c, gr->ops[1]);
        if (!up || !b) return;
        if (up->total == 1 && out->rank == 1) {
            double dy = up->data[0];
            for (int64_t i = 0; i < out->dims[0]; ++i) out->data[i] += dy * tread(b, i);
            return;
        }
        int64_t di = out->rank > 0 ? out->dims[0] : 1, dj = out->rank > 1 ? out->dims[1] : 1;
        int64_t dk = up->rank > 1 ? up->dims[1] : 1;
        #pragma omp parallel for schedule(static) if (di * dj * dk > 1000000)
        for (int64_t i = 0; i < di; ++i)
            for (int64_t j = 0; j < dj; ++j) {
                double acc = out->data[i * dj + j];
                for (int64_t k = 0; k < dk; ++k) acc = acc + tread(up, i * dk + k) * tread(b, j * dk + k);
                if (i * dj + j < out->total) out->data[i * dj + j] = acc;
            }
        return;
    }
    case R_MM_RIGHT: {
        or_tensor* a = find_tensor(c, gr->ops[0]);
        if (!up || !a) return;
        if (up->total == 1 && out->rank == 1) {
            double dy = up->data[0];
            for (int64_t i = 0; i < out->dims[0]; ++i) out->data[i] += dy * tread(a, i);
            return;
        }
        int64_t di = a->rank > 0 ? a->dims[0] : 1;
        int64_t dj = out->rank > 0 ? out->dims[0] : 1, dk = out->rank > 1 ? out->dims[1] : 1;
        #pragma omp parallel for schedule(static) if (di * dj * dk > 1000000)
        for (int64_t j = 0; j < dj; ++j)
            for (int64_t k = 0; k < dk; ++k) {
                double acc = out->data[j * dk + k];
                for (int64_t i = 0; i < di; ++i) acc = acc + tread(a, i * dj + j) * tread(up, i * dk + k);
                if (j * dk + k < out->total) out->data[j * dk + k] = acc;
            }
        return;
    }
    }
}

/* genBackward (llvm.zig:635-693). */
static int gen_backward(or_ctx* c, const tl_statement* st, const tl_statement* all, int n_all) {
    ad_graph* g = (ad_graph*)calloc(1, sizeof(ad_graph));
    if (!g) return TL_ERR_OOM;
    for (int s = 0; s < n_all; ++s) {
        if (all[s].kind != TL_STMT_EQUATION) continue;
        const tl_equation* eq = &all[s].eq;
        ad_node* n = ad_find(g, eq->lhs.tensor);
        if (!n) n = &g->nodes[g->n_nodes++];
        memset(n, 0, sizeof *n);
        snprintf(n->out, TL_NAME_LEN, "%s", eq->lhs.tensor);
        n->op = root_op(eq);
        n->n_in = eq->n_refs;
        for (int r = 0; r < eq->n_refs; ++r) snprintf(n->in[r], TL_NAME_LEN, "%s", eq->refs[r].tensor);
    }
    char (*visited)[TL_NAME_LEN] = calloc(MAX_TENSORS, TL_NAME_LEN);
    int nv = 0;
    topo_visit(g, st->name, visited, &nv);
    free(visited);
    for (int a = 0, b = g->n_topo - 1; a < b; ++a, --b) {
        char tmp[TL_NAME_LEN];
        memcpy(tmp, g->topo[a], TL_NAME_LEN); memcpy(g->topo[a], g->topo[b], TL_NAME_LEN); memcpy(g->topo[b], tmp, TL_NAME_LEN);
    }
    for (int i = 0; i < g->n_topo; ++i) {
        ad_node* n = ad_find(g, g->topo[i]);
        if (n) gen_gradients(g, n, st->params, st->n_params);
    }
    for (int p = 0; p < st->n_params; ++p) {
        or_tensor* base = find_tensor(c, st->params[p]);
        char gname[TL_NAME_LEN + 8];
        snprintf(gname, sizeof gname, "dL_d%s", st->params[p]);
        if (base) new_tensor(c, gname, base->rank, base->dims);
    }
    or_tensor* loss = find_tensor(c, st->name);
    if (loss) {
        char gname[TL_NAME_LEN + 8];
        snprintf(gname, sizeof gname, "dL_d%s", st->name);
        or_tensor* dl = new_tensor(c, gname, loss->rank, loss->dims);
        if (dl) dl->data[0] = 1.0;
    }
    for (int i = 0; i < g->n_grads; ++i) gen_grad_equation(c, &g->grads[i]);
    free(g);
    return TL_OK;
}

/* ------------------------------------------------------------------------ */
/* Backward chaining: constant-index queries (backward.zig:37-600)            */
/* ------------------------------------------------------------------------ */

/* isBackwardQuery (backward.zig:37-46): any constant index. */
static int bw_is_query(const tl_ref* q) {
    for (int k = 0; k < q->rank; ++k) if (q->idx[k].kind == TL_IX_CONST) return 1;
    return 0;
}

static bw_global* bw_find(or_ctx* c, const char* name) {
    for (int i = 0; i < c->n_bw; ++i) if (strcmp(c->bw[i].name, name) == 0) return &c->bw[i];
    return NULL;
}

static void bw_reset(or_ctx* c) {
    for (int i = 0; i < c->n_bw; ++i) {
        free(c->bw[i].eq_stmt); free(c->bw[i].memo); free(c->bw[i].done); free(c->bw[i].snap);
    }
    memset(c->bw, 0, sizeof c->bw);
    c->n_bw = 0;
    c->bw_stmts = NULL;
    c->bw_depth = 0;
    c->bw_err = 0;
}

/* allocateTensorGlobal (tensor.zig:157-220): max dims when known, else per index. */
static bw_global* bw_add(or_ctx* c, const tl_ref* lhs) {
    bw_global* g = bw_find(c, lhs->tensor);
    if (g) return g;
    if (c->n_bw >= MAX_BW) return NULL;
    g = &c->bw[c->n_bw++];
    snprintf(g->name, TL_NAME_LEN, "%s", lhs->tensor);
    const or_maxdims* m = NULL;
    for (int i = 0; i < c->n_maxdims; ++i) if (strcmp(c->maxdims[i].name, lhs->tensor) == 0) m = &c->maxdims[i];
    if (m) { g->rank = m->rank; for (int k = 0; k < m->rank; ++k) g->dims[k] = m->dims[k]; }
    else {
        g->rank = lhs->rank;
        for (int k = 0; k < lhs->rank; ++k)
            g->dims[k] = lhs->idx[k].kind == TL_IX_NORMALIZE ? 10 : index_extent(c, &lhs->idx[k]);
    }
    if (g->rank == 0) { g->rank = 1; g->dims[0] = 1; }
    int64_t s = 1;
    for (int k = g->rank - 1; k >= 0; --k) { g->strides[k] = s; s *= g->dims[k]; }
    g->total = s;
    return g;
}

static int name_in(const char (*names)[TL_NAME_LEN], int n, const char* name) {
    for (int i = 0; i < n; ++i) if (strcmp(names[i], name) == 0) return 1;
    return 0;
}

/* The globals and memo tables of llvm.zig:222-264 and genBackwardInfra
 * (backward.zig:53-118): queried tensors' equations in program order, then
 * the equation-defined tensors their right-hand sides read. */
static int bw_prepare(or_ctx* c, const tl_statement* stmts, int n) {
    static char queried[MAX_BW][TL_NAME_LEN], deps[MAX_BW * TL_MAX_REFS][TL_NAME_LEN];
    int nq = 0, nd = 0;
    bw_reset(c);
    c->bw_stmts = stmts;
    for (int s = 0; s < n; ++s)
        if (stmts[s].kind == TL_STMT_QUERY && bw_is_query(&stmts[s].sparse) &&
            !name_in(queried, nq, stmts[s].name) && nq < MAX_BW)
            snprintf(queried[nq++], TL_NAME_LEN, "%s", stmts[s].name);
    if (nq == 0) return TL_OK;
    for (int s = 0; s < n; ++s) {
        if (stmts[s].kind != TL_STMT_EQUATION || !name_in(queried, nq, stmts[s].eq.lhs.tensor)) continue;
        bw_global* g = bw_add(c, &stmts[s].eq.lhs);
        if (!g) return TL_ERR_TOO_LARGE;
        g->compute = 1;
        g->eq_stmt = (int32_t*)realloc(g->eq_stmt, sizeof(int32_t) * (size_t)(g->n_eq + 1));
        g->eq_stmt[g->n_eq++] = s;
        for (int r = 0; r < stmts[s].eq.n_refs; ++r)
            if (!name_in(deps, nd, stmts[s].eq.refs[r].tensor) && nd < MAX_BW * TL_MAX_REFS)
                snprintf(deps[nd++], TL_NAME_LEN, "%s", stmts[s].eq.refs[r].tensor);
    }
    for (int s = 0; s < n; ++s) {
        if (stmts[s].kind != TL_STMT_EQUATION) continue;
        const char* lhs = stmts[s].eq.lhs.tensor;
        if (name_in(deps, nd, lhs) && !name_in(queried, nq, lhs) && !bw_add(c, &stmts[s].eq.lhs))
            return TL_ERR_TOO_LARGE;
    }
    for (int i = 0; i < c->n_bw; ++i) {
        bw_global* g = &c->bw[i];
        if (!g->compute) continue;
        g->memo = (double*)calloc((size_t)g->total, sizeof(double));
        g->done = (unsigned char*)calloc((size_t)g->total, 1);
        if (!g->memo || !g->done) return TL_ERR_OOM;
    }
    return TL_OK;
}

/* genSparseDecl re-allocates unconditionally (llvm.zig:482-516), so after a
 * `sparse` declaration of a global the forward code writes a new buffer and
 * the compute functions keep reading the global as it was. */
static void bw_detach(or_ctx* c, const char* name) {
    bw_global* g = bw_find(c, name);
    if (!g || g->detached) return;
    g->detached = 1;
    g->snap = (double*)calloc((size_t)g->total, sizeof(double));
    const or_tensor* t = find_tensor(c, name);
    if (g->snap && t && t->total == g->total) memcpy(g->snap, t->data, (size_t)g->total * sizeof(double));
}

static double bw_call(or_ctx* c, bw_global* g, const int64_t* iv);

/* A contracted equation's loop variables (collectContracted,
 * backward.zig:253-282), in order of first appearance. */
typedef struct {
    int32_t n;
    char names[MAX_VARS][TL_NAME_LEN];
    int64_t sizes[MAX_VARS];
    int64_t cur[MAX_VARS];
} bw_loops;

/* genBackwardTensorAccess (backward.zig:493-548). */
static double bw_access(or_ctx* c, const tl_equation* eq, int r, const int64_t* params,
                        const tl_ref* lhs, const bw_loops* lv) {
    const tl_ref* ref = &eq->refs[r];
    bw_global* g = bw_find(c, ref->tensor);
    if (!g) return 0.0;                        /* not in the codegen's tensor map */
    int64_t iv[TL_MAX_RANK];
    for (int k = 0; k < ref->rank; ++k) {
        const tl_index* ix = &ref->idx[k];
        iv[k] = 0;
        if (ix->kind == TL_IX_CONST) { iv[k] = ix->value; continue; }
        if (ix->kind != TL_IX_NAME) continue;
        int bound = -1;
        for (int j = 0; j < lhs->rank; ++j)
            if (lhs->idx[j].kind == TL_IX_NAME && strcmp(lhs->idx[j].name, ix->name) == 0) bound = j;
        if (bound >= 0) { iv[k] = params[bound]; continue; }
        for (int j = 0; j < lv->n; ++j)
            if (strcmp(lv->names[j], ix->name) == 0) { iv[k] = lv->cur[j]; break; }
    }
    if (g->compute) {
        if (ref->rank != g->rank) { c->bw_err = TL_ERR_UNSUPPORTED; return 0.0; }
        return bw_call(c, g, iv);
    }
    /* computeLinearOffset (tensor.zig:131-154) over the global's strides */
    int64_t off = 0;
    int nk = ref->rank < g->rank ? ref->rank : g->rank;
    for (int k = 0; k < nk; ++k) off += iv[k] * g->strides[k];
    if (off < 0 || off >= g->total) return 0.0;
    if (g->detached) return g->snap ? g->snap[off] : 0.0;
    const or_tensor* t = find_tensor(c, g->name);
    return (t && off < t->total) ? t->data[off] : 0.0;
}

/* genBackwardExpr (backward.zig:375-488) over the postfix program. */
static double bw_eval(or_ctx* c, const tl_equation* eq, const int64_t* params, const bw_loops* lv) {
    double st[TL_MAX_CODE];
    int sp = 0;
    for (int i = 0; i < eq->n_code && !c->bw_err; ++i) {
        const tl_instr* in = &eq->code[i];
        switch (in->op) {
        case TL_OP_REF: st[sp++] = bw_access(c, eq, in->arg, params, &eq->lhs, lv); break;
        case TL_OP_LIT: st[sp++] = in->value; break;
        case TL_OP_PROD: {
            int n = in->arg;
            double acc = st[sp - n];
            for (int k = 1; k < n; ++k) acc = acc * st[sp - n + k];
            sp -= n;
            st[sp++] = acc;
            break;
        }
        case TL_OP_NEG: st[sp - 1] = -st[sp - 1]; break;
        case TL_OP_NOT: st[sp - 1] = (st[sp - 1] == 0.0) ? 1.0 : 0.0; break;
        case TL_OP_NL: {
            double x = st[sp - 1], r;
            switch (in->arg) {
            case TL_NL_STEP: r = x > 0.0 ? 1.0 : 0.0; break;
            case TL_NL_RELU: r = x > 0.0 ? x : 0.0; break;
            case TL_NL_SIGMOID: r = 1.0 / (1.0 + exp(-x)); break;   /* no temperature */
            case TL_NL_EXP: r = exp(x); break;
            case TL_NL_LOG: r = log(x); break;
            case TL_NL_SQRT: r = sqrt(x); break;
            case TL_NL_ABS: r = fabs(x); break;
            case TL_NL_SIN: r = sin(x); break;
            case TL_NL_COS: r = cos(x); break;
            case TL_NL_TANH: { double e = x * 2.0; e = exp(e); r = (e - 1.0) / (e + 1.0); break; }
            default: r = 0.0 + x; break;
            }
            st[sp - 1] = r;
            break;
        }
        default: {
            double b = st[--sp];
            double a = st[sp - 1];
            switch (in->op) {
            case TL_OP_SUB: st[sp - 1] = a - b; break;
            case TL_OP_MUL: st[sp - 1] = a * b; break;
            case TL_OP_DIV: st[sp - 1] = a / b; break;
            default: st[sp - 1] = a + b; break;     /* add, and every other binary op */
            }
        }
        }
    }
    return sp > 0 ? st[sp - 1] : 0.0;
}

/* genBackwardEquation + genContractedSum (backward.zig:222-371). */
static double bw_equation(or_ctx* c, const tl_equation* eq, const int64_t* params) {
    bw_loops lv;
    lv.n = 0;
    for (int r = 0; r < eq->n_refs; ++r)
        for (int k = 0; k < eq->refs[r].rank; ++k) {
            const tl_index* ix = &eq->refs[r].idx[k];
            if (ix->kind != TL_IX_NAME) continue;
            int bound = 0;
            for (int j = 0; j < eq->lhs.rank; ++j)
                if (eq->lhs.idx[j].kind == TL_IX_NAME && strcmp(eq->lhs.idx[j].name, ix->name) == 0) bound = 1;
            if (bound) continue;
            int at = -1;
            for (int j = 0; j < lv.n; ++j) if (strcmp(lv.names[j], ix->name) == 0) at = j;
            if (at < 0 && lv.n < MAX_VARS) {
                at = lv.n++;
                snprintf(lv.names[at], TL_NAME_LEN, "%s", ix->name);
                lv.sizes[at] = domain_size(c, ix->name);
            }
        }
    if (lv.n == 0) return bw_eval(c, eq, params, &lv);
    double acc = 0.0;
    for (int j = 0; j < lv.n; ++j) { lv.cur[j] = 0; if (lv.sizes[j] <= 0) return acc; }
    for (;;) {
        acc = acc + bw_eval(c, eq, params, &lv);
        if (c->bw_err) return 0.0;
        int j = lv.n - 1;                      /* the first loop is the outermost */
        while (j >= 0 && ++lv.cur[j] >= lv.sizes[j]) lv.cur[j--] = 0;
        if (j < 0) return acc;
    }
}

/* @compute_T (genComputeFunction, backward.zig:119-220). */
static double bw_call(or_ctx* c, bw_global* g, const int64_t* iv) {
    int64_t off = 0;
    for (int k = 0; k < g->rank; ++k) off += iv[k] * g->strides[k];
    if (off < 0 || off >= g->total) return 0.0;   /* outside the memo table */
    if (g->done[off]) return g->memo[off];
    if (c->bw_depth >= BW_MAX_DEPTH) { c->bw_err = TL_ERR_TOO_LARGE; return 0.0; }
    c->bw_depth++;
    g->done[off] = 1;
    g->memo[off] = 0.0;
    double result = 0.0;
    for (int e = 0; e < g->n_eq && !c->bw_err; ++e) {
        const tl_equation* eq = &c->bw_stmts[g->eq_stmt[e]].eq;
        double v = bw_equation(c, eq, iv);
        switch (eq->accum) {
        case TL_ACC_ADD: result = result + v; break;
        case TL_ACC_MAX: result = (v > result) ? v : result; break;
        case TL_ACC_MIN: result = (v < result) ? v : result; break;
        case TL_ACC_MUL: result = result * v; break;
        default: result = 0.0 + v; break;
        }
        g->memo[off] = result;
    }
    c->bw_depth--;
    return result;
}

/* genBackwardQuery (backward.zig:568-600): "%s = %.6g\n". */
static int bw_query(or_ctx* c, const tl_statement* st, double* out) {
    bw_global* g = bw_find(c, st->name);
    if (!g || !g->compute) {
        snprintf(c->err, sizeof c->err, "%s: a constant-index query needs an equation defining it", st->name);
        return TL_ERR_UNSUPPORTED;
    }
    if (st->sparse.rank != g->rank) {
        snprintf(c->err, sizeof c->err, "%s: query has %d indices, tensor has %d", st->name, st->sparse.rank, g->rank);
        return TL_ERR_UNSUPPORTED;
    }
    int64_t iv[TL_MAX_RANK];
    for (int k = 0; k < st->sparse.rank; ++k)
        iv[k] = st->sparse.idx[k].kind == TL_IX_CONST ? st->sparse.idx[k].value : 0;
    c->bw_depth = 0;
    *out = bw_call(c, g, iv);
    if (c->bw_err) {
        snprintf(c->err, sizeof c->err, "%s: backward query failed (%d)", st->name, c->bw_err);
        return c->bw_err;
    }
    return TL_OK;
}

/* ------------------------------------------------------------------------ */
/* Program (llvm.zig:131-336)                                                 */
/* ------------------------------------------------------------------------ */
static void qprintf(or_ctx* c, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
#include <stdarg.h>
static void qprintf(or_ctx* c, const char* fmt, ...) {
    char buf[512];
    va_list ap; va_start(ap, fmt);
    int n = vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (n < 0) return;
    if (c->qlen + (size_t)n + 1 > c->qcap) {
        size_t cap = c->qcap ? c->qcap * 2 : 4096;
        while (cap < c->qlen + (size_t)n + 1) cap *= 2;
        c->qout = (char*)realloc(c->qout, cap);
        c->qcap = cap;
    }
    memcpy(c->qout + c->qlen, buf, (size_t)n + 1);
    c->qlen += (size_t)n;
}

or_ctx* or_create(int32_t max_sweeps) {
    or_ctx* c = (or_ctx*)calloc(1, sizeof(or_ctx));
    if (c) c->max_sweeps = max_sweeps > 0 ? max_sweeps : 1000;
    return c;
}

void or_destroy(or_ctx* c) {
    if (!c) return;
    for (int i = 0; i < c->n_tensors; ++i) free(c->tensors[i].data);
    bw_reset(c);
    free(c->qout);
    free(c);
}

static int run_statement(or_ctx* c, const tl_statement* st, const tl_statement* all, int n_all) {
    switch (st->kind) {
    case TL_STMT_EQUATION: return gen_equation(c, &st->eq);
    case TL_STMT_SPARSE: {
        /* genSparseDecl (llvm.zig:482-516): the dense view */
        tl_index idx[TL_MAX_RANK];
        for (int k = 0; k < st->sparse.rank; ++k) {
            memset(&idx[k], 0, sizeof idx[k]);
            idx[k].kind = TL_IX_NAME;
            snprintf(idx[k].name, TL_NAME_LEN, "%s", st->sparse.idx[k].name);
        }
        bw_detach(c, st->sparse.tensor);
        return allocate_tensor(c, st->sparse.tensor, idx, st->sparse.rank) ? TL_OK : TL_ERR_OOM;
    }
    case TL_STMT_SPARSE_LOAD: {
        or_tensor* t = find_tensor(c, st->name);
        if (!t || t->rank != 2) return TL_ERR_NOT_FOUND;
        for (int64_t e = 0; e < st->size; ++e) {
            int64_t off = st->coo_rows[e] * t->strides[0] + st->coo_cols[e];
            if (off >= 0 && off < t->total) t->data[off] = st->host_data ? st->host_data[e] : 1.0;
        }
        return TL_OK;
    }
    case TL_STMT_BACKWARD: return gen_backward(c, st, all, n_all);
    case TL_STMT_SAVE: {
        or_tensor* t = find_tensor(c, st->name);
        if (!t) return TL_OK;
        FILE* f = fopen(st->path, "wb");
        if (!f) return TL_ERR_IO;
        size_t w = fwrite(t->data, 8, (size_t)t->total, f);
        fclose(f);
        return w == (size_t)t->total ? TL_OK : TL_ERR_IO;
    }
    case TL_STMT_LOAD: {
        or_tensor* t = find_tensor(c, st->name);
        if (!t) return TL_OK;
        if (st->host_data) { memcpy(t->data, st->host_data, (size_t)t->total * 8); return TL_OK; }
        FILE* f = fopen(st->path, "rb");
        if (!f) return TL_ERR_IO;
        size_t r = fread(t->data, 8, (size_t)t->total, f);
        fclose(f);
        (void)r;
        return TL_OK;
    }
    default: return TL_OK;
    }
}

int32_t or_program_run(or_ctx* c, const tl_statement* stmts, int32_t n) {
    c->qlen = 0;
    if (c->qout) c->qout[0] = 0;
    c->err[0] = 0;
    for (int s = 0; s < n; ++s)
        if (stmts[s].kind == TL_STMT_DOMAIN && stmts[s].size >= 0) put_domain(c, stmts[s].name, stmts[s].size);
    for (int s = 0; s < n; ++s)
        if (stmts[s].kind == TL_STMT_EQUATION) update_max_dims(c, &stmts[s].eq.lhs);
    int brc = bw_prepare(c, stmts, n);
    if (brc != TL_OK) return brc;
    /* non-recursive statements in source order (llvm.zig:287-301) */
    int n_rec = 0;
    for (int s = 0; s < n; ++s) {
        if (stmts[s].kind == TL_STMT_QUERY || stmts[s].kind == TL_STMT_DOMAIN) continue;
        if (stmts[s].kind == TL_STMT_EQUATION && is_recursive(&stmts[s].eq)) { n_rec++; continue; }
        int rc = run_statement(c, &stmts[s], stmts, n);
        if (rc != TL_OK) return rc;
    }
    /* fixpoint (fixpoint.zig:46-98) */
    c->last_sweeps = 0;
    if (n_rec > 0) {
        int iter = 0, changed = 1;
        while (iter < c->max_sweeps && changed) {
            changed = 0;
            for (int s = 0; s < n; ++s)
                if (stmts[s].kind == TL_STMT_EQUATION && is_recursive(&stmts[s].eq)) {
                    int rc = recursive_sweep(c, &stmts[s].eq, &changed);
                    if (rc != TL_OK) return rc;
                }
            iter++;
        }
        c->last_sweeps = iter;
    }
    /* queries (llvm.zig:310-318, 461-480) */
    for (int s = 0; s < n; ++s) {
        if (stmts[s].kind != TL_STMT_QUERY) continue;
        if (bw_is_query(&stmts[s].sparse)) {
            double v;
            int rc = bw_query(c, &stmts[s], &v);
            if (rc != TL_OK) return rc;
            qprintf(c, "%s = %.6g\n", stmts[s].name, v);
            continue;
        }
        or_tensor* t = find_tensor(c, stmts[s].name);
        if (!t) continue;
        qprintf(c, "%s[%zu] = [", t->name, (size_t)t->total);
        int64_t np = t->total < 20 ? t->total : 20;
        for (int64_t i = 0; i < np; ++i) qprintf(c, "%.4g ", t->data[i]);
        qprintf(c, "]\n");
    }
    return TL_OK;
}

int32_t or_tensor_info(or_ctx* c, const char* name, int32_t* rank, int64_t* dims) {
    or_tensor* t = find_tensor(c, name);
    if (!t) return -1;
    if (rank) *rank = t->rank;
    if (dims) for (int k = 0; k < t->rank; ++k) dims[k] = t->dims[k];
    return 0;
}

const double* or_tensor_data(or_ctx* c, const char* name) {
    or_tensor* t = find_tensor(c, name);
    return t ? t->data : NULL;
}

int32_t or_last_sweeps(or_ctx* c) { return c->last_sweeps; }
const char* or_query_output(or_ctx* c) { return c->qout ? c->qout : ""; }
const char* or_last_error(or_ctx* c) { return c->err; }

/* ------------------------------------------------------------------------ */
/* Full-size restatements                                                    */
/* ------------------------------------------------------------------------ */

/* Right-form closure in the reference's in-place loop order: for each row x,
 * z ascending, R[x,z] = max(R[x,z], step(R[x,y] E[y,z])) over y (fixpoint.zig
 * :167-297 with the max= branch :256-273).  E[y,z] != 0 only for y in the
 * predecessor list of z, so the inner y loop visits exactly those; every
 * other y contributes step(0) = 0, which never raises R.  Rows never read
 * other rows, so each row's sweep sequence is independent and the sweep
 * count of the whole tensor is the maximum over rows. */
int32_t or_closure_right(int64_t n, const int64_t* colptr, const int32_t* rowidx,
                         uint32_t* R, int64_t row_begin, int64_t row_end, int32_t max_sweeps,
                         int32_t n_threads) {
    int64_t W = (n + 31) / 32;
    int32_t worst = 0;
    (void)n_threads;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
    #pragma omp parallel for schedule(dynamic, 16) reduction(max : worst)
    for (int64_t x = row_begin; x < row_end; ++x) {
        uint32_t* row = R + (x - row_begin) * W;
        int32_t sweeps = 0;
        int changed = 1;
        while (sweeps < max_sweeps && changed) {
            changed = 0;
            for (int64_t z = 0; z < n; ++z) {
                if (row[z >> 5] >> (z & 31) & 1u) continue;
                for (int64_t e = colptr[z]; e < colptr[z + 1]; ++e) {
                    int32_t y = rowidx[e];
                    if (row[y >> 5] >> (y & 31) & 1u) {
                        row[z >> 5] |= 1u << (z & 31);
                        changed = 1;
                        break;
                    }
                }
            }
            sweeps++;
        }
        if (sweeps > worst) worst = sweeps;
    }
    return worst;
}

void or_gnn_layer(int64_t n, int64_t g, int64_t f, const int64_t* rowptr, const int32_t* colidx,
                  const double* adj_vals, const double* H, const double* W, double* out,
                  int32_t n_threads) {
    double* P = (double*)calloc((size_t)(n * f), sizeof(double));
    (void)n_threads;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
    /* P[u,f] = sum_g relu(H[u,g] W[g,f]) */
    #pragma omp parallel for schedule(static)
    for (int64_t u = 0; u < n; ++u)
        for (int64_t j = 0; j < f; ++j) {
            double acc = 0.0;
            for (int64_t k = 0; k < g; ++k) {
                double t = H[u * g + k] * W[k * f + j];
                acc = acc + (t > 0.0 ? t : 0.0);
            }
            P[u * f + j] = acc;
        }
    /* out[v,f] = sum_u Adj[v,u] P[u,f]; relu(a*t) = a*relu(t) for a in {0,1} */
    #pragma omp parallel for schedule(static)
    for (int64_t v = 0; v < n; ++v)
        for (int64_t j = 0; j < f; ++j) {
            double acc = 0.0;
            for (int64_t e = rowptr[v]; e < rowptr[v + 1]; ++e) {
                double a = adj_vals ? adj_vals[e] : 1.0;
                acc = acc + a * P[(int64_t)colidx[e] * f + j];
            }
            out[v * f + j] = acc;
        }
    free(P);
}

void or_gemm(int64_t M, int64_t N, int64_t K, const double* A, int64_t sam, int64_t sak,
             const double* B, int64_t sbk, int64_t sbn, double* Cout, int64_t scm, int64_t scn,
             int32_t relu_per_term, double scale, int32_t n_threads) {
    (void)n_threads;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
    #pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m)
        for (int64_t nn = 0; nn < N; ++nn) {
            double acc = Cout[m * scm + nn * scn];
            for (int64_t k = 0; k < K; ++k) {
                double t = A[m * sam + k * sak] * (B[k * sbk + nn * sbn] * scale);
                if (relu_per_term) t = t > 0.0 ? t : 0.0;
                acc = acc + t;
            }
            Cout[m * scm + nn * scn] = acc;
        }
}

/* The literal loop nest of one right-form sweep (fixpoint.zig:167-297) over
 * rows [x0, x0 + nrows): for x, for z, for y: old = R[x,z]; rhs =
 * step(R[x,y] * E[y,z]); if rhs > old store rhs.  R rows are f64 as in the
 * reference; Edge is read from a bit matrix (its dense f64 view would need
 * n*n*8 bytes).  Used as the timed CPU sample of the reference algorithm. */
int64_t or_closure_literal_rows(int64_t n, const uint32_t* Ebits, int64_t x0, int64_t nrows, double* Rrows) {
    return or_closure_literal_rows_mt(n, Ebits, x0, nrows, Rrows, 1);
}

/* The same literal sweep with the rows spread over n_threads host threads
   (rows are independent within the right-form sweep). */
int64_t or_closure_literal_rows_mt(int64_t n, const uint32_t* Ebits, int64_t x0, int64_t nrows, double* Rrows,
                                   int32_t n_threads) {
    int64_t W = (n + 31) / 32;
    int64_t changed = 0;
    (void)n_threads;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#endif
    #pragma omp parallel for schedule(dynamic, 1) reduction(+ : changed)
    for (int64_t x = 0; x < nrows; ++x) {
        double* row = Rrows + x * n;
        for (int64_t z = 0; z < n; ++z) {
            for (int64_t y = 0; y < n; ++y) {
                double old = row[z];
                double e = (Ebits[y * W + (z >> 5)] >> (z & 31)) & 1u ? 1.0 : 0.0;
                double t = row[y] * e;
                double rhs = t > 0.0 ? 1.0 : 0.0;
                if (rhs > old) { row[z] = rhs; changed++; }
            }
        }
    }
    (void)x0;
    return changed;
}
