// Element-wise gradient rules of the `backward L wrt ...` lowering.
//
// Reference rules (src/codegen/autodiff.zig), all accumulating into the
// gradient buffer (`+=`) over the upstream gradient's element count:
//   pass_through  dX += dY                       :500-519
//   relu_grad     dX += dY * step(X)             :521-554
//   sigmoid_grad  dX += dY * Y * (1 - Y)         :556-584
//   tanh_grad     dX += dY * (1 - Y^2)           :586-612
//   exp_grad      dX += dY * Y                   :614-638
//   log_grad      dX += dY / X                   :640-664
//   matmul_self   dX += 2 X   (upstream unused)  :749-772
//   softmax_grad  dX += Y * (dY - sum_all(dY*Y)) :686-747  (one sum over the
//                 whole tensor, not per row)
// Out-of-range elements read 0.0 and are not written.
#include "tl_internal.h"

namespace tl {

enum GradRule { G_PASS = 0, G_RELU, G_SIGMOID, G_TANH, G_EXP, G_LOG, G_SELF };

namespace {

__device__ __forceinline__ float at(const float* p, int64_t n, int64_t i) {
    return (p && i < n) ? p[i] : 0.f;
}

__global__ void k_grad_elem(int rule, float* out, int64_t out_n, const float* up, int64_t up_n, const float* x,
                            int64_t x_n, const float* y, int64_t y_n, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if (i >= out_n) continue;
        const float dy = at(up, up_n, i);
        float g;
        switch (rule) {
        case G_PASS: g = dy; break;
        case G_RELU: g = dy * (at(x, x_n, i) > 0.f ? 1.f : 0.f); break;
        case G_SIGMOID: { const float v = at(y, y_n, i); g = dy * (v * (1.f - v)); break; }
        case G_TANH: { const float v = at(y, y_n, i); g = dy * (1.f - v * v); break; }
        case G_EXP: g = dy * at(y, y_n, i); break;
        case G_LOG: g = dy / at(x, x_n, i); break;
        default: g = at(x, x_n, i) * 2.f; break;   // matmul_self
        }
        out[i] += g;
    }
}

__device__ __forceinline__ float grad_rule(int rule, float dy, float xv, float yv) {
    switch (rule) {
    case G_PASS: return dy;
    case G_RELU: return dy * (xv > 0.f ? 1.f : 0.f);
    case G_SIGMOID: return dy * (yv * (1.f - yv));
    case G_TANH: return dy * (1.f - yv * yv);
    case G_EXP: return dy * yv;
    case G_LOG: return dy / xv;
    default: return xv * 2.f;   // matmul_self
    }
}

// The same rules when every operand covers all n elements (n a multiple of
// 4, 16-byte aligned): 128-bit loads and stores.  overwrite: the gradient
// buffer holds logical zeros, so it is written instead of read and added to.
__global__ void k_grad_elem4(int rule, float* __restrict__ out, const float* __restrict__ up,
                             const float* __restrict__ x, const float* __restrict__ y, int64_t n4, int overwrite) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 d = up ? reinterpret_cast<const float4*>(up)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 xv = x ? reinterpret_cast<const float4*>(x)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 yv = y ? reinterpret_cast<const float4*>(y)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 g = make_float4(grad_rule(rule, d.x, xv.x, yv.x), grad_rule(rule, d.y, xv.y, yv.y),
                               grad_rule(rule, d.z, xv.z, yv.z), grad_rule(rule, d.w, xv.w, yv.w));
        float4* o = reinterpret_cast<float4*>(out) + i;
        if (!overwrite) {
            const float4 v = *o;
            g.x += v.x; g.y += v.y; g.z += v.z; g.w += v.w;
        }
        *o = g;
    }
}

// s = sum_i a[i] * b[i] in f64 in one launch: every block adds its partial
// sum into acc; the last block to finish writes out[0] = old + s (old = 0 for
// a logically zero output) and puts acc and the counter back to zero.
__global__ void __launch_bounds__(256) k_dot_scalar(const float* __restrict__ a, const float* __restrict__ b,
                                                    int64_t n, float* out, int old_zero, double* acc,
                                                    unsigned* done) {
    double s = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        s += (double)a[i] * (double)b[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __shared__ double sh[8];
    __shared__ bool last;
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += sh[w];
        atomicAdd(acc, t);
        __threadfence();
        last = atomicAdd(done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        const double total = *(volatile double*)acc;
        out[0] = (float)((old_zero ? 0.0 : (double)out[0]) + total);
        *acc = 0.0;
        *done = 0u;
    }
}

// sum_i dY[i] * Y[i] over the whole tensor, in f64
__global__ void k_dot(const float* up, int64_t up_n, const float* y, int64_t y_n, double* acc) {
    double s = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < up_n; i += (int64_t)gridDim.x * blockDim.x)
        s += (double)up[i] * (double)at(y, y_n, i);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __shared__ double sh[32];
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) atomicAdd(acc, v);
    }
}

__global__ void k_softmax_grad(float* out, int64_t out_n, const float* up, int64_t up_n, const float* y, int64_t y_n,
                               const double* dot) {
    const double s = *dot;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < up_n; i += (int64_t)gridDim.x * blockDim.x) {
        if (i >= out_n) continue;
        const double v = at(y, y_n, i);
        out[i] += (float)(v * ((double)up[i] - s));
    }
}

unsigned blocks_for(tl_ctx* c, int64_t n) {
    int64_t b = (n + 255) / 256;
    const int64_t cap = (int64_t)c->sm_count * 16;
    if (b > cap) b = cap;
    return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

bool grad_elem_covers(int rule, int64_t out_total, int64_t up_total, int64_t x_total) {
    const int64_t n = rule == G_SELF ? x_total : up_total;
    return n >= out_total;
}

tl_status launch_grad_elem(tl_ctx* c, int rule, float* out, int64_t out_total, const float* up, int64_t up_total,
                           const float* x, int64_t x_total, const float* y, int64_t y_total, int overwrite) {
    const int64_t n = rule == G_SELF ? x_total : up_total;
    if (n <= 0) return TL_OK;
    auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    const bool vec = (n & 3) == 0 && out_total >= n && (rule == G_SELF || up_total >= n) && (!x || x_total >= n) &&
                     (!y || y_total >= n) && al(out) && al(up) && al(x) && al(y);
    if (vec) {
        LaunchScope L(c, "grad_elementwise", (double)n * 4.0 * (2 + (up ? 1 : 0) + (x ? 1 : 0) + (y ? 1 : 0) -
                                                                 (overwrite ? 1 : 0)),
                      (double)n * 2.0);
        k_grad_elem4<<<blocks_for(c, n / 4), 256, 0, c->stream>>>(rule, out, rule == G_SELF ? nullptr : up, x, y,
                                                                   n / 4, overwrite);
        return L.done();
    }
    if (overwrite) TL_CK(c, cudaMemsetAsync(out, 0, (size_t)out_total * sizeof(float), c->stream));
    LaunchScope L(c, "grad_elementwise", (double)n * 12.0, (double)n * 2.0);
    k_grad_elem<<<blocks_for(c, n), 256, 0, c->stream>>>(rule, out, out_total, up, up_total, x, x_total, y, y_total, n);
    return L.done();
}

tl_status launch_dot_scalar(tl_ctx* c, const float* a, const float* b, int64_t n, float* out, int old_zero) {
    if (n <= 0) return TL_OK;
    // accumulator (double) and block counter live in the context's flag words
    double* acc = reinterpret_cast<double*>(c->d_flags + 40);
    unsigned* done = reinterpret_cast<unsigned*>(c->d_flags + 44);
    int64_t blocks = (n + 2047) / 2048;
    if (blocks > c->sm_count) blocks = c->sm_count;
    LaunchScope L(c, "dot_scalar", (double)n * 8.0, (double)n * 2.0);
    k_dot_scalar<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, c->stream>>>(a, b, n, out, old_zero, acc, done);
    return L.done();
}

tl_status launch_grad_softmax(tl_ctx* c, float* out, int64_t out_total, const float* up, int64_t up_total,
                              const float* y, int64_t y_total) {
    if (up_total <= 0) return TL_OK;
    void* ws = nullptr;
    TL_TRY(workspace(c, 64, &ws));
    double* dot = (double*)ws;
    TL_CK(c, cudaMemsetAsync(dot, 0, sizeof(double), c->stream));
    {
        LaunchScope L(c, "softmax_grad_dot", (double)up_total * 8.0);
        k_dot<<<blocks_for(c, up_total), 256, 0, c->stream>>>(up, up_total, y, y_total, dot);
        TL_TRY(L.done());
    }
    LaunchScope L(c, "softmax_grad", (double)up_total * 16.0);
    k_softmax_grad<<<blocks_for(c, up_total), 256, 0, c->stream>>>(out, out_total, up, up_total, y, y_total, dot);
    return L.done();
}

}  // namespace tl
