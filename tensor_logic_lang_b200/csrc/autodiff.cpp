// `backward L wrt P1, ...` lowering.
//
// The rule set and its order follow the reference exactly:
//   graph over every equation (a later equation for the same LHS replaces
//   the earlier node)                          src/codegen/autodiff.zig:87-158
//   DFS topological order from the loss, reversed   :161-198
//   per-node rules, inputs needing a gradient only  :202-420
//   gradient buffers calloc'd with the base dims    :459-481, llvm.zig:647-669
//   dL/dL = 1 in a fresh buffer                     llvm.zig:671-687
// Each rule becomes one kernel: element-wise rules go to k_grad.cu, the
// matmul rules (autodiff.zig:774-1014, which read every operand as a
// row-major 2-D [rows x cols] array regardless of its index names) become
// transposed-operand GEMMs on the tensor cores.
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "tl_internal.h"

namespace tl {

enum GradRule { G_PASS = 0, G_RELU, G_SIGMOID, G_TANH, G_EXP, G_LOG, G_SELF };
tl_status alloc_dense_public(tl_ctx* c, Tensor* t);

namespace {

enum Op { AD_IDENTITY, AD_SCALAR, AD_MATMUL, AD_ADD, AD_MUL, AD_RELU, AD_SIGMOID, AD_TANH, AD_SOFTMAX, AD_LNORM,
          AD_EXP, AD_LOG };
enum Rule { R_PASS, R_MM_LEFT, R_MM_RIGHT, R_MM_SELF, R_RELU, R_SIGMOID, R_SOFTMAX, R_TANH, R_EXP, R_LOG };

struct Node {
    std::string out;
    Op op;
    std::vector<std::string> in;
};

struct Grad {
    Rule rule;
    std::string out, up;
    std::string ops[3];
};

Op root_op(const tl_equation* eq) {
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
        case TL_NL_RELU: return AD_RELU;
        case TL_NL_SIGMOID: return AD_SIGMOID;
        case TL_NL_TANH: return AD_TANH;
        case TL_NL_SOFTMAX: return AD_SOFTMAX;
        case TL_NL_LNORM: return AD_LNORM;
        case TL_NL_EXP: return AD_EXP;
        case TL_NL_LOG: return AD_LOG;
        default: return AD_IDENTITY;
        }
    default: return AD_IDENTITY;
    }
}

struct Graph {
    std::vector<Node> nodes;
    std::vector<std::string> topo;
    std::vector<Grad> grads;
    const char (*params)[TL_NAME_LEN] = nullptr;
    int np = 0;

    Node* find(const std::string& n) {
        for (auto& x : nodes) if (x.out == n) return &x;
        return nullptr;
    }
    bool is_param(const std::string& n) const {
        for (int i = 0; i < np; ++i) if (n == params[i]) return true;
        return false;
    }
    // hasPathToParam (autodiff.zig:408-420); the depth bound stops the
    // self-reference of a recursive equation, where the reference recurses
    // without end.
    bool has_path(const std::string& n, int depth = 0) {
        if (is_param(n)) return true;
        if (depth > 64) return false;
        Node* x = find(n);
        if (!x) return false;
        for (auto& i : x->in) if (has_path(i, depth + 1)) return true;
        return false;
    }
    void visit(const std::string& n, std::vector<std::string>& seen) {
        if (std::find(seen.begin(), seen.end(), n) != seen.end()) return;
        seen.push_back(n);
        if (Node* x = find(n)) {
            const std::vector<std::string> ins = x->in;
            for (auto& i : ins) visit(i, seen);
        }
        topo.push_back(n);
    }
    void add(Rule r, const std::string& input, const std::string& output, const std::string& a = "",
             const std::string& b = "", const std::string& cc = "") {
        grads.push_back({r, "dL_d" + input, "dL_d" + output, {a, b, cc}});
    }
    // genGradients (autodiff.zig:202-390)
    void rules(const Node& n) {
        switch (n.op) {
        case AD_MATMUL:
            if (n.in.size() == 2 && n.in[0] == n.in[1]) {
                if (has_path(n.in[0])) add(R_MM_SELF, n.in[0], n.out, n.in[0]);
            } else if (n.in.size() >= 2) {
                if (has_path(n.in[0])) add(R_MM_LEFT, n.in[0], n.out, n.in[0], n.in[1], n.out);
                if (has_path(n.in[1])) add(R_MM_RIGHT, n.in[1], n.out, n.in[0], n.in[1], n.out);
            } else {
                for (size_t i = 0; i < n.in.size(); ++i) {
                    bool dup = false;
                    for (size_t j = 0; j < i; ++j) dup = dup || n.in[i] == n.in[j];
                    if (!dup && has_path(n.in[i])) add(R_PASS, n.in[i], n.out, n.in[i]);
                }
            }
            break;
        case AD_ADD: case AD_IDENTITY:
            for (auto& i : n.in) if (has_path(i)) add(R_PASS, i, n.out, i);
            break;
        case AD_RELU: if (!n.in.empty() && has_path(n.in[0])) add(R_RELU, n.in[0], n.out, n.in[0]); break;
        case AD_SIGMOID: if (!n.in.empty() && has_path(n.in[0])) add(R_SIGMOID, n.in[0], n.out, n.in[0], n.out); break;
        case AD_SOFTMAX: if (!n.in.empty() && has_path(n.in[0])) add(R_SOFTMAX, n.in[0], n.out, n.in[0], n.out); break;
        case AD_TANH: if (!n.in.empty() && has_path(n.in[0])) add(R_TANH, n.in[0], n.out, n.in[0], n.out); break;
        case AD_EXP: if (!n.in.empty() && has_path(n.in[0])) add(R_EXP, n.in[0], n.out, n.in[0], n.out); break;
        case AD_LOG: if (!n.in.empty() && has_path(n.in[0])) add(R_LOG, n.in[0], n.out, n.in[0]); break;
        default: break;  // scalar, `*` and lnorm have no rule
        }
    }
};

// Dense fp32 view of a tensor for reading (nullptr when absent or zero).
tl_status rd(tl_ctx* c, const std::string& name, Tensor** t, const float** p) {
    *t = find_defined(c, name);
    tl_status st;
    *p = read_ptr(c, *t, &st);
    if (*t && (*t)->shard == TL_SHARD_ROWS && c->world > 1)
        return fail(c, TL_ERR_UNSUPPORTED, "%s: backward over a sharded tensor", name.c_str());
    return st;
}

int64_t dim_or1(const Tensor* t, int k) { return t && t->rank > k ? t->dims[k] : 1; }

// genGradEquation (autodiff.zig:459-498) and the rule loops.
tl_status run_grad(tl_ctx* c, const Grad& g) {
    Tensor* out = find_defined(c, g.out);
    if (!out) {
        Tensor* base = find_defined(c, g.out.substr(4));
        if (!base) return TL_OK;
        TL_TRY(new_tensor(c, g.out, base->rank, base->dims, &out));
    }
    Tensor* up;
    const float* upp;
    TL_TRY(rd(c, g.up, &up, &upp));
    switch (g.rule) {
    case R_PASS: case R_RELU: case R_SIGMOID: case R_TANH: case R_EXP: case R_LOG: {
        if (!up) return TL_OK;
        Tensor *x = nullptr, *y = nullptr;
        const float *xp = nullptr, *yp = nullptr;
        if (g.rule == R_RELU || g.rule == R_LOG) {
            TL_TRY(rd(c, g.ops[0], &x, &xp));
            if (!x) return TL_OK;
        }
        if (g.rule == R_SIGMOID || g.rule == R_TANH || g.rule == R_EXP) {
            TL_TRY(rd(c, g.ops[1], &y, &yp));
            if (!y) return TL_OK;
        }
        if (!upp && g.rule != R_LOG) return TL_OK;     // zero upstream adds zeros
        const int rule = g.rule == R_PASS ? G_PASS : g.rule == R_RELU ? G_RELU : g.rule == R_SIGMOID ? G_SIGMOID
                         : g.rule == R_TANH ? G_TANH : g.rule == R_EXP ? G_EXP : G_LOG;
        // a fresh (calloc) gradient buffer that the rule covers is written, not zeroed and added to
        const bool fresh = out->zero && !out->dense_valid && upp &&
                           grad_elem_covers(rule, out->total, up->total, x ? x->total : 0);
        if (fresh) TL_TRY(alloc_dense_public(c, out));
        else TL_TRY(ensure_dense(c, out));
        TL_TRY(launch_grad_elem(c, rule, out->dense, out->total, upp, up->total, xp, x ? x->total : 0, yp,
                                y ? y->total : 0, fresh ? 1 : 0));
        mark_written_dense(out);
        out->boolean = false;
        return TL_OK;
    }
    case R_SOFTMAX: {
        Tensor* y;
        const float* yp;
        TL_TRY(rd(c, g.ops[1], &y, &yp));
        if (!up || !y || !upp) return TL_OK;
        TL_TRY(ensure_dense(c, out));
        TL_TRY(launch_grad_softmax(c, out->dense, out->total, upp, up->total, yp, y->total));
        mark_written_dense(out);
        out->boolean = false;
        return TL_OK;
    }
    case R_MM_SELF: {
        Tensor* x;
        const float* xp;
        TL_TRY(rd(c, g.ops[0], &x, &xp));
        if (!x || !xp) return TL_OK;
        TL_TRY(ensure_dense(c, out));
        TL_TRY(launch_grad_elem(c, G_SELF, out->dense, out->total, nullptr, 0, xp, x->total, nullptr, 0));
        mark_written_dense(out);
        out->boolean = false;
        return TL_OK;
    }
    case R_MM_LEFT: case R_MM_RIGHT: {
        if (!up) return TL_OK;
        const bool left = g.rule == R_MM_LEFT;
        Tensor* op;
        const float* opp;
        TL_TRY(rd(c, left ? g.ops[1] : g.ops[0], &op, &opp));
        if (!op) return TL_OK;
        GemmPlan p;
        memset(&p, 0, sizeof p);
        p.scale = 1.0f;
        if (up->total == 1 && out->rank == 1) {
            // dot-product form (autodiff.zig:1016-1082): out[i] += dy * op[i]
            const int64_t n = out->dims[0];
            if (op->total < n) return fail(c, TL_ERR_UNSUPPORTED, "%s: gradient operand shorter than the output", g.out.c_str());
            p.M = n; p.N = 1; p.K = 1;
            p.A = opp; p.sam = 1; p.sak = 1;
            p.B = upp; p.sbk = 1; p.sbn = 1;
        } else if (left) {
            // dA[i,j] += sum_k dC[i,k] * B[j,k]   (autodiff.zig:774-893)
            const int64_t di = dim_or1(out, 0), dj = dim_or1(out, 1), dk = dim_or1(up, 1);
            if (di * dj != out->total || di * dk != up->total || dj * dk != op->total)
                return fail(c, TL_ERR_UNSUPPORTED, "%s: matmul gradient over mismatched shapes", g.out.c_str());
            p.M = di; p.N = dj; p.K = dk;
            p.A = upp; p.sam = dk; p.sak = 1;
            p.B = opp; p.sbk = 1; p.sbn = dk;
        } else {
            // dB[j,k] += sum_i A[i,j] * dC[i,k]   (autodiff.zig:895-1014)
            const int64_t di = dim_or1(op, 0), dj = dim_or1(out, 0), dk = dim_or1(out, 1);
            if (dj * dk != out->total || di * dk != up->total || di * dj != op->total)
                return fail(c, TL_ERR_UNSUPPORTED, "%s: matmul gradient over mismatched shapes", g.out.c_str());
            p.M = dj; p.N = dk; p.K = di;
            p.A = opp; p.sam = 1; p.sak = dj;
            p.B = upp; p.sbk = dk; p.sbn = 1;
        }
        if (!p.A || !p.B) return TL_OK;   // a zero operand adds zeros
        p.scm = p.N; p.scn = 1;
        p.beta = out->zero ? 0 : 1;
        if (p.beta) TL_TRY(ensure_dense(c, out));
        else TL_TRY(alloc_dense_public(c, out));
        p.C = out->dense;
        TL_TRY(launch_gemm(c, p));
        mark_written_dense(out);
        out->boolean = false;
        return TL_OK;
    }
    }
    return TL_OK;
}

}  // namespace

tl_status run_backward(tl_ctx* c, const char* loss, const char (*params)[TL_NAME_LEN], int np, const tl_equation* eqs,
                       int n_eqs) {
    if (np < 0 || np > TL_MAX_PARAMS) return fail(c, TL_ERR_INVALID, "bad parameter count");
    Graph g;
    g.params = params;
    g.np = np;
    for (int e = 0; e < n_eqs; ++e) {
        const tl_equation* eq = &eqs[e];
        Node n{eq->lhs.tensor, root_op(eq), {}};
        for (int r = 0; r < eq->n_refs; ++r) n.in.push_back(eq->refs[r].tensor);
        if (Node* old = g.find(n.out)) *old = n;
        else g.nodes.push_back(n);
    }
    std::vector<std::string> seen;
    g.visit(loss, seen);
    std::reverse(g.topo.begin(), g.topo.end());
    for (auto& name : g.topo) {
        if (Node* n = g.find(name)) {
            const Node copy = *n;
            g.rules(copy);
        }
    }
    // fresh gradient buffers for the parameters, then dL/dL = 1
    for (int i = 0; i < np; ++i) {
        Tensor* base = find_defined(c, params[i]);
        if (!base) continue;
        Tensor* t;
        TL_TRY(new_tensor(c, std::string("dL_d") + params[i], base->rank, base->dims, &t));
    }
    if (Tensor* L = find_defined(c, loss)) {
        Tensor* t;
        TL_TRY(new_tensor(c, std::string("dL_d") + loss, L->rank, L->dims, &t));
        TL_TRY(ensure_dense(c, t));
        // dL/dL = 1 (a device fill: no host memory, no synchronisation)
        TL_TRY(launch_fill(c, t->dense, 1, 1.0f));
        mark_written_dense(t);
    }
    for (auto& gr : g.grads) TL_TRY(run_grad(c, gr));
    return TL_OK;
}

}  // namespace tl

extern "C" tl_status tl_backward(tl_ctx* c, const char* loss, const char (*params)[TL_NAME_LEN], int32_t n_params,
                                 const tl_equation* eqs, int32_t n_eqs) {
    if (!c || !loss || (n_params > 0 && !params) || (n_eqs > 0 && !eqs)) return TL_ERR_INVALID;
    TL_CK(c, cudaSetDevice(c->device));
    return tl::run_backward(c, loss, params, n_params, eqs, n_eqs);
}
