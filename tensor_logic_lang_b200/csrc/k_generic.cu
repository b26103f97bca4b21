// Generic per-term tensor equation on CUDA cores.
//
// One thread per free-index tuple (LHS element); the thread walks the
// contracted index space in the reference's loop order and folds every term
// with the equation's accumulation operator, exactly like the innermost body
// of the emitted loop nest: src/codegen/einsum.zig:20-254 (loops and
// genAccumulation), src/codegen/expr.zig:14-300 (per-term expression),
// src/codegen/fixpoint.zig:227-280 (recursive change detection).
// Terms are evaluated in f64 from fp32 operands, so per-term nonlinearities
// (exp, sigmoid, tanh, log, ...) and mixed expressions keep f64 rounding.
#include <math.h>

#include "tl_internal.h"

namespace tl {
namespace {

__device__ __forceinline__ double load_ref(const RefPlan& r, const int64_t* iv, int pos_var) {
    if (!r.ptr) return 0.0;
    int64_t off = 0;
    for (int k = 0; k < r.nidx; ++k) {
        int64_t x;
        const int v = r.var[k];
        switch (r.kind[k]) {
        case TL_IX_NAME: case TL_IX_PRIMED: x = v >= 0 ? iv[v] : 0; break;
        case TL_IX_CONST: x = r.val[k]; break;
        case TL_IX_ADD: x = v >= 0 ? iv[v] + r.val[k] : r.val[k]; break;
        case TL_IX_SUB: x = v >= 0 ? iv[v] - r.val[k] : r.val[k]; break;
        case TL_IX_DIV: x = v >= 0 ? iv[v] / r.val[k] : 0; break;
        case TL_IX_SLICE: x = r.val[k]; break;
        case TL_IX_VIRTUAL: {
            x = 0;
            if (r.virt[k] && pos_var >= 0) {
                int64_t p = iv[pos_var];
                if (p >= 0 && p < r.virt_total[k]) x = (int64_t)(double)r.virt[k][p];
            }
            break;
        }
        default: x = 0; break;
        }
        off += x * r.stride[k];
    }
    return (off >= 0 && off < r.total) ? (double)r.ptr[off] : 0.0;
}

__device__ __forceinline__ double nonlin(int f, double x, int has_t, double t) {
    switch (f) {
    case TL_NL_RELU: return x > 0.0 ? x : 0.0;
    case TL_NL_SIGMOID: return 1.0 / (1.0 + exp(has_t ? -(x / t) : -x));
    case TL_NL_TANH: { double e = exp(x * 2.0); return (e - 1.0) / (e + 1.0); }
    case TL_NL_STEP: return x > 0.0 ? 1.0 : 0.0;
    case TL_NL_EXP: return exp(x);
    case TL_NL_LOG: return log(x);
    case TL_NL_SQRT: return sqrt(x);
    case TL_NL_ABS: return fabs(x);
    case TL_NL_SIN: return sin(x);
    case TL_NL_COS: return cos(x);
    default: return x;
    }
}

__device__ double eval(const GenericPlan& p, const int64_t* iv) {
    double st[16];
    int sp = 0;
    for (int i = 0; i < p.n_code; ++i) {
        const CodeOp& in = p.code[i];
        switch (in.op) {
        case TL_OP_REF: st[sp++] = load_ref(p.refs[in.arg], iv, p.virt_pos_var); break;
        case TL_OP_LIT: st[sp++] = in.value; break;
        case TL_OP_PROD: {
            const int n = in.arg;
            double acc = st[sp - n];
            for (int k = 1; k < n; ++k) acc = acc * st[sp - n + k];
            sp -= n;
            st[sp++] = acc;
            break;
        }
        case TL_OP_NEG: st[sp - 1] = -st[sp - 1]; break;
        case TL_OP_NOT: st[sp - 1] = st[sp - 1] == 0.0 ? 1.0 : 0.0; break;
        case TL_OP_NL: st[sp - 1] = nonlin(in.arg, st[sp - 1], in.arg2, in.value); break;
        default: {
            const double b = st[--sp];
            const double a = st[sp - 1];
            double r;
            switch (in.op) {
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
            case TL_OP_NE: r = (a < b) || (a > b); break;   // fcmp one
            default: r = a + b; break;                       // & and | lower to fadd
            }
            st[sp - 1] = r;
        }
        }
    }
    return sp > 0 ? st[sp - 1] : 0.0;
}

__device__ __forceinline__ void atomic_fold(float* addr, int accum, float v) {
    if (accum == TL_ACC_MAX || accum == TL_ACC_MIN || accum == TL_ACC_MUL) {
        unsigned int* a = reinterpret_cast<unsigned int*>(addr);
        unsigned int old = *a, assumed;
        do {
            assumed = old;
            float cur = __uint_as_float(assumed);
            float nv = accum == TL_ACC_MAX ? (v > cur ? v : cur)
                     : accum == TL_ACC_MIN ? (v < cur ? v : cur) : cur * v;
            if (__float_as_uint(nv) == assumed) return;
            old = atomicCAS(a, assumed, __float_as_uint(nv));
        } while (old != assumed);
    } else {
        atomicAdd(addr, v);
    }
}

// One thread per free tuple.  `serial` folds every tuple in one thread, for
// plain stores into elements several tuples share (the last one wins, as in
// the sequential loop nest).
__global__ void k_generic(const __grid_constant__ GenericPlan p, int* changed, int serial) {
    const int64_t n_threads = serial ? 1 : p.n_out;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n_threads;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n_tuples = serial ? p.n_out : 1;
        for (int64_t s = 0; s < n_tuples; ++s) {
            int64_t iv[kMaxVars];
            int64_t rem = serial ? s : t;
            for (int v = p.n_free - 1; v >= 0; --v) {
                iv[v] = rem % p.sizes[v];
                rem /= p.sizes[v];
            }
            for (int v = p.n_free; v < p.n_vars; ++v) iv[v] = 0;
            int64_t off = 0;
            for (int k = 0; k < p.n_lhs_terms; ++k) off += (iv[p.lhs_var[k]] / p.lhs_div[k]) * p.lhs_stride[k];
            const bool in_range = off >= 0 && off < p.lhs_total;
            const bool atomic = p.atomic && !serial;
            double acc;
            if (atomic) {
                // partial fold from the operator's identity, merged atomically
                acc = (p.accum == TL_ACC_MAX) ? -INFINITY : (p.accum == TL_ACC_MIN) ? INFINITY
                    : (p.accum == TL_ACC_MUL) ? 1.0 : 0.0;
            } else {
                acc = (p.old_zero || !in_range) ? 0.0 : (double)p.lhs[off];
            }
            bool inc = false;
            for (int64_t j = 0; j < p.n_inner; ++j) {
                const double rhs = eval(p, iv);
                if (p.recursive) {
                    // fixpoint.zig:236-280: += and max= detect increases, every
                    // other operator stores the term and counts as a change
                    if (p.accum == TL_ACC_ADD) {
                        const double nv = acc + rhs;
                        if (nv > acc) inc = true;
                        acc = nv;
                    } else if (p.accum == TL_ACC_MAX) {
                        if (rhs > acc) { acc = rhs; inc = true; }
                    } else {
                        acc = rhs;
                        inc = true;
                    }
                } else {
                    switch (p.accum) {
                    case TL_ACC_ASSIGN: acc = p.has_contraction ? acc + rhs : rhs; break;
                    case TL_ACC_ADD: case TL_ACC_AVG: acc = acc + rhs; break;
                    case TL_ACC_MAX: acc = rhs > acc ? rhs : acc; break;
                    case TL_ACC_MIN: acc = rhs < acc ? rhs : acc; break;
                    case TL_ACC_MUL: acc = acc * rhs; break;
                    }
                }
                // odometer over the contracted variables
                for (int v = p.n_vars - 1; v >= p.n_free; --v) {
                    if (++iv[v] < p.sizes[v]) break;
                    iv[v] = 0;
                }
            }
            if (!in_range) continue;
            if (atomic) {
                if (p.n_inner > 0) atomic_fold(&p.lhs[off], p.accum, (float)acc);
            } else {
                p.lhs[off] = (float)acc;
            }
            if (p.recursive && inc && changed) *changed = 1;
        }
    }
}

// Small outputs with long contractions: block (o, s) folds slice s of LHS
// element o's contracted range with its 256 threads and a tree in f64, and
// a second pass folds the slices in order and merges the LHS's old value.
// The operator must be associative (sum, max, min, product); the order of
// the partial folds differs from the reference's sequential loop only in
// f64 rounding of sums.
__device__ __forceinline__ double fold_op(int accum, double a, double b) {
    switch (accum) {
    case TL_ACC_MAX: return b > a ? b : a;
    case TL_ACC_MIN: return b < a ? b : a;
    case TL_ACC_MUL: return a * b;
    default: return a + b;
    }
}

__device__ __forceinline__ double fold_ident(int accum) {
    return accum == TL_ACC_MAX ? -INFINITY : accum == TL_ACC_MIN ? INFINITY : accum == TL_ACC_MUL ? 1.0 : 0.0;
}

__global__ void __launch_bounds__(256) k_generic_reduce(const __grid_constant__ GenericPlan p, double* partial,
                                                        int64_t chunk) {
    __shared__ double sh[256];
    const int64_t o = blockIdx.x, s = blockIdx.y;
    int64_t iv[kMaxVars];
    int64_t rem = o;
    for (int v = p.n_free - 1; v >= 0; --v) {
        iv[v] = rem % p.sizes[v];
        rem /= p.sizes[v];
    }
    double acc = fold_ident(p.accum);
    const int64_t j1 = (s + 1) * chunk < p.n_inner ? (s + 1) * chunk : p.n_inner;
    for (int64_t j = s * chunk + threadIdx.x; j < j1; j += blockDim.x) {
        int64_t r = j;
        for (int v = p.n_vars - 1; v >= p.n_free; --v) {
            iv[v] = r % p.sizes[v];
            r /= p.sizes[v];
        }
        acc = fold_op(p.accum, acc, eval(p, iv));
    }
    sh[threadIdx.x] = acc;
    __syncthreads();
    for (int h = blockDim.x / 2; h > 0; h >>= 1) {
        if (threadIdx.x < h) sh[threadIdx.x] = fold_op(p.accum, sh[threadIdx.x], sh[threadIdx.x + h]);
        __syncthreads();
    }
    if (threadIdx.x == 0) partial[o * gridDim.y + s] = sh[0];
}

__global__ void k_generic_reduce_finish(const __grid_constant__ GenericPlan p, const double* partial, int nsplit) {
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < p.n_out; o += (int64_t)gridDim.x * blockDim.x) {
        int64_t iv[kMaxVars];
        int64_t rem = o;
        for (int v = p.n_free - 1; v >= 0; --v) {
            iv[v] = rem % p.sizes[v];
            rem /= p.sizes[v];
        }
        double part = fold_ident(p.accum);
        for (int s = 0; s < nsplit; ++s) part = fold_op(p.accum, part, partial[o * nsplit + s]);
        int64_t off = 0;
        for (int k = 0; k < p.n_lhs_terms; ++k) off += (iv[p.lhs_var[k]] / p.lhs_div[k]) * p.lhs_stride[k];
        if (off >= 0 && off < p.lhs_total) {
            const double old = p.old_zero ? 0.0 : (double)p.lhs[off];
            p.lhs[off] = (float)fold_op(p.accum, old, part);
        }
    }
}

// Element-wise equations whose operands share the LHS's shape and index
// order: the flat index addresses every operand, no index decoding.
__global__ void k_generic_aligned(const __grid_constant__ GenericPlan p) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < p.n_out; t += (int64_t)gridDim.x * blockDim.x) {
        double st[16];
        int sp = 0;
        for (int i = 0; i < p.n_code; ++i) {
            const CodeOp& in = p.code[i];
            switch (in.op) {
            case TL_OP_REF: { const float* q = p.refs[in.arg].ptr; st[sp++] = q ? (double)q[t] : 0.0; break; }
            case TL_OP_LIT: st[sp++] = in.value; break;
            case TL_OP_PROD: {
                const int n = in.arg;
                double a = st[sp - n];
                for (int k = 1; k < n; ++k) a = a * st[sp - n + k];
                sp -= n;
                st[sp++] = a;
                break;
            }
            case TL_OP_NEG: st[sp - 1] = -st[sp - 1]; break;
            case TL_OP_NOT: st[sp - 1] = st[sp - 1] == 0.0 ? 1.0 : 0.0; break;
            case TL_OP_NL: st[sp - 1] = nonlin(in.arg, st[sp - 1], in.arg2, in.value); break;
            default: {
                const double b = st[--sp], a = st[sp - 1];
                double r;
                switch (in.op) {
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
                case TL_OP_NE: r = (a < b) || (a > b); break;
                default: r = a + b; break;
                }
                st[sp - 1] = r;
            }
            }
        }
        const double rhs = sp > 0 ? st[sp - 1] : 0.0;
        const double old = p.old_zero ? 0.0 : (double)p.lhs[t];
        double nv;
        switch (p.accum) {
        case TL_ACC_ASSIGN: nv = rhs; break;
        case TL_ACC_ADD: case TL_ACC_AVG: nv = old + rhs; break;
        case TL_ACC_MAX: nv = rhs > old ? rhs : old; break;
        case TL_ACC_MIN: nv = rhs < old ? rhs : old; break;
        default: nv = old * rhs; break;
        }
        p.lhs[t] = (float)nv;
    }
}

__global__ void k_set1(const __grid_constant__ GenericPlan p, float* dst, int64_t off) {
    if (threadIdx.x == 0 && blockIdx.x == 0) dst[off] = (float)eval(p, nullptr);
}

__global__ void k_fill(float* p, int64_t n, float v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = v;
}

}  // namespace

tl_status launch_generic(tl_ctx* c, const GenericPlan& p, int* d_changed) {
    const bool serial = p.atomic && p.accum == TL_ACC_ASSIGN && !p.has_contraction;
    const double terms = (double)p.n_out * (double)p.n_inner;
    if (p.aligned && !p.recursive && !p.has_contraction) {
        int64_t blocks = (p.n_out + 255) / 256;
        const int64_t cap = (int64_t)c->sm_count * 16;
        if (blocks > cap) blocks = cap;
        LaunchScope L(c, "elementwise", (double)p.n_out * 4.0 * (p.n_refs + 1), (double)p.n_out);
        k_generic_aligned<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, c->stream>>>(p);
        return L.done();
    }
    // few outputs, long contraction, associative operator: split the contraction
    const bool assoc = p.has_contraction && (p.accum == TL_ACC_ASSIGN || p.accum == TL_ACC_ADD ||
                                             p.accum == TL_ACC_AVG || p.accum == TL_ACC_MAX ||
                                             p.accum == TL_ACC_MIN || p.accum == TL_ACC_MUL);
    if (assoc && !p.recursive && !p.atomic && p.n_inner >= 512 && p.n_out < (int64_t)c->sm_count * 64) {
        // slices of >= 1024 terms, enough blocks to cover the SMs four times
        int64_t nsplit = ((int64_t)c->sm_count * 4 + p.n_out - 1) / p.n_out;
        const int64_t max_split = (p.n_inner + 1023) / 1024;
        if (nsplit > max_split) nsplit = max_split;
        if (nsplit > 65535) nsplit = 65535;
        if (nsplit < 1) nsplit = 1;
        const int64_t chunk = (p.n_inner + nsplit - 1) / nsplit;
        void* ws = nullptr;
        TL_TRY(workspace(c, (size_t)p.n_out * nsplit * sizeof(double) + 64, &ws));
        {
            LaunchScope L(c, "generic_reduce", terms * 4.0 * p.n_refs, terms * 2.0);
            k_generic_reduce<<<dim3((unsigned)p.n_out, (unsigned)nsplit), 256, 0, c->stream>>>(p, (double*)ws, chunk);
            TL_TRY(L.done());
        }
        LaunchScope L(c, "generic_reduce_finish", (double)p.n_out * nsplit * 8.0, 0);
        k_generic_reduce_finish<<<(unsigned)((p.n_out + 127) / 128), 128, 0, c->stream>>>(p, (const double*)ws,
                                                                                          (int)nsplit);
        return L.done();
    }
    const int threads = 128;
    int64_t blocks = serial ? 1 : (p.n_out + threads - 1) / threads;
    blocks = blocks < 1 ? 1 : (blocks > 65535LL * 8 ? 65535LL * 8 : blocks);
    LaunchScope L(c, "generic_einsum", terms * 4.0 * (p.n_refs + 0.0) / (p.n_inner > 0 ? p.n_inner : 1) + p.n_out * 4.0,
                  terms * 2.0);
    k_generic<<<(unsigned)blocks, serial ? 1 : threads, 0, c->stream>>>(p, d_changed, serial ? 1 : 0);
    return L.done();
}

tl_status launch_set1(tl_ctx* c, float* dst, int64_t off, const GenericPlan& p) {
    LaunchScope L(c, "scalar_assign");
    k_set1<<<1, 32, 0, c->stream>>>(p, dst, off);
    return L.done();
}

tl_status launch_fill(tl_ctx* c, float* p, int64_t n, float v) {
    if (n <= 0) return TL_OK;
    LaunchScope L(c, "fill", n * 4.0, 0);
    int64_t blocks = (n + 255) / 256;
    if (blocks > c->sm_count * 16) blocks = c->sm_count * 16;
    k_fill<<<(unsigned)blocks, 256, 0, c->stream>>>(p, n, v);
    return L.done();
}

}  // namespace tl
