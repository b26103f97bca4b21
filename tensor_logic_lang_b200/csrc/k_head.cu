// A small-batch two-layer head in two launches:
//   H[b, h]  = Σ_i  [relu](s1 · X[b, i] W1[i, h])    (relu per term, or none)
//   Z[b, o]  = s2 · Σ_h H[b, h] W2[h, o]
//   Y[b, o.] = softmax over o of Z[b, o]
// Reference semantics: the three statements one by one (einsum.zig:20-278
// with the per-term nonlinearity of expr.zig:14-300, then softmax.zig:19-229);
// H, Z and Y are all written, as the reference keeps them.
//
// B200 mapping: at a batch of at most 64 rows the first contraction is too
// small for the tensor cores (a 128-row MMA tile would be mostly empty) and
// one-statement kernels are latency-bound, three launches of a few
// microseconds each.  k_head_h splits H's columns (32 per block, a lane each)
// and the contracted range (ks chunks) over the grid, so enough blocks run at
// once; each block stages its chunk of X in shared memory and writes a partial
// H.  k_head_zy, a block per batch row, adds the partials in chunk order (no
// atomics: the result does not depend on scheduling), writes the row of H,
// contracts it with W2 and takes the softmax of the row of Z in registers.
// fp32 throughout, as the one-statement SIMT and skinny kernels compute these
// shapes.
#include <math.h>

#include <algorithm>

#include "tl_internal.h"

namespace tl {
namespace {

constexpr int HD_THREADS = 256;
constexpr int HD_COLS = 32;              // H columns per k_head_h block
constexpr int HD_RPW = kHeadMaxRows / 8; // batch rows per warp (8 warps)
constexpr int HD_KB = 32;                // contracted indices whose loads are in flight at once
constexpr int HD_XPT = 8;                // X elements a thread stages per round

// The inputs are cold (read once per run), so the kernels issue every load of
// a round before using any: a round costs one memory round trip.

// Partial H of one block: columns [32 bx, 32 bx + 32), contracted indices
// [ky kc, ky kc + kc), every batch row (warp w takes rows w, w + 8, ...).
__global__ void __launch_bounds__(HD_THREADS) k_head_h(const HeadPlan p) {
    extern __shared__ float xs[];   // X[b, k0 .. k0 + kn) row by row
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t col = (int64_t)blockIdx.x * HD_COLS + lane;
    const int64_t k0 = (int64_t)blockIdx.y * p.kc;
    const int kn = (int)std::min<int64_t>(p.kc, p.i - k0);
    const int nx = (int)p.b * kn;
    const bool in = col < p.h;
    const float* w1 = p.W1 + k0 * p.h + col;
    // the first round of W1 is in flight while X is staged
    float wv[HD_KB];
#pragma unroll
    for (int u = 0; u < HD_KB; ++u) wv[u] = (in && u < kn) ? w1[(int64_t)u * p.h] : 0.f;
    for (int t0 = 0; t0 < nx; t0 += HD_THREADS * HD_XPT) {
        float v[HD_XPT];
#pragma unroll
        for (int u = 0; u < HD_XPT; ++u) {
            const int t = t0 + u * HD_THREADS + threadIdx.x;
            const int r = t / kn, kk = t - r * kn;
            v[u] = t < nx ? p.X[(int64_t)r * p.i + k0 + kk] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < HD_XPT; ++u) {
            const int t = t0 + u * HD_THREADS + threadIdx.x;
            if (t < nx) xs[t] = v[u];
        }
    }
    __syncthreads();
    float acc[HD_RPW];
#pragma unroll
    for (int j = 0; j < HD_RPW; ++j) acc[j] = 0.f;
    for (int ks0 = 0; ks0 < kn; ks0 += HD_KB) {
        if (ks0 > 0) {
#pragma unroll
            for (int u = 0; u < HD_KB; ++u) wv[u] = (in && ks0 + u < kn) ? w1[(int64_t)(ks0 + u) * p.h] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < HD_RPW; ++j) {
            const int r = w + 8 * j;
            if (r >= p.b) break;
            const float* xr = xs + r * kn + ks0;
            float a = acc[j];
            if (p.relu_term) {
#pragma unroll
                for (int u = 0; u < HD_KB; ++u)
                    if (ks0 + u < kn) a += fmaxf(p.sgn1 * (xr[u] * wv[u]), 0.f);
            } else {
#pragma unroll
                for (int u = 0; u < HD_KB; ++u)
                    if (ks0 + u < kn) a += xr[u] * wv[u];
            }
            acc[j] = a;
        }
    }
    if (!in) return;
#pragma unroll
    for (int j = 0; j < HD_RPW; ++j) {
        const int r = w + 8 * j;
        if (r < p.b) p.hpart[((int64_t)blockIdx.y * p.b + r) * p.h + col] = acc[j];
    }
}

// Row r of H (the partials in chunk order, times s1's magnitude or s1), of
// Z = s2 H W2 (warp w takes columns w, w + 8, ... of Z; lanes split h) and of
// Y = softmax(Z) (warp 0, a lane per column), as the row-wise kernel takes it:
// the row maximum subtracted, a maximum of -inf or NaN taken as 0.
__global__ void __launch_bounds__(HD_THREADS) k_head_zy(const HeadPlan p) {
    extern __shared__ float hs[];   // the row of H
    __shared__ float zs[kHeadMaxCols];
    const int64_t r = blockIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t stride = p.b * p.h;   // between the chunks' partials of one element
    // this warp's columns of Z are o = w, w + 8, w + 16, w + 24: their first
    // 256 rows of W2 are in flight while the partials are added
    constexpr int OPW = kHeadMaxCols / 8;
    float w2[OPW][8];
#pragma unroll
    for (int q = 0; q < OPW; ++q)
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int o = w + 8 * q;
            const int64_t c = u * 32 + lane;
            w2[q][u] = (o < p.o && c < p.h) ? p.W2[c * p.o + o] : 0.f;
        }
    for (int64_t c = threadIdx.x; c < p.h; c += HD_THREADS) {
        const float* src = p.hpart + r * p.h + c;
        float v = 0.f;
        for (int k0 = 0; k0 < p.ks; k0 += HD_KB) {
            float t[HD_KB];
#pragma unroll
            for (int u = 0; u < HD_KB; ++u) t[u] = k0 + u < p.ks ? src[(int64_t)(k0 + u) * stride] : 0.f;
#pragma unroll
            for (int u = 0; u < HD_KB; ++u) v += t[u];   // in chunk order (the padding adds zeros)
        }
        v *= p.mag1;
        hs[c] = v;
        p.H[r * p.h + c] = v;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < OPW; ++q) {
        const int o = w + 8 * q;
        if (o >= p.o) break;
        float s = 0.f;
        for (int64_t c0 = 0; c0 < p.h; c0 += 32 * 8) {
            float wv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int64_t c = c0 + u * 32 + lane;
                wv[u] = c0 == 0 ? w2[q][u] : (c < p.h ? p.W2[c * p.o + o] : 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int64_t c = c0 + u * 32 + lane;
                if (c < p.h) s = fmaf(hs[c], wv[u], s);
            }
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
        if (lane == 0) zs[o] = s * p.s2;
    }
    __syncthreads();
    if (w != 0) return;
    const bool in = lane < p.o;
    const float z = in ? zs[lane] : -INFINITY;
    if (in) p.Z[r * p.o + lane] = z;
    float m = z;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    if (m == -INFINITY || m != m) m = 0.f;
    const float e = in ? __expf(z - m) : 0.f;
    float s = e;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
    if (in) p.Y[r * p.o + lane] = e * (1.0f / s);
}

}  // namespace

tl_status launch_head(tl_ctx* c, HeadPlan p) {
    if (p.b < 1 || p.b > kHeadMaxRows || p.o < 1 || p.o > kHeadMaxCols || p.h < 1 || p.i < 1)
        return fail(c, TL_ERR_INVALID, "head: shape outside the fused kernel's range");
    if ((size_t)p.h * 4 > 200 * 1024) return fail(c, TL_ERR_UNSUPPORTED, "head: hidden row too long");
    const int64_t col_blocks = (p.h + HD_COLS - 1) / HD_COLS;
    // chunks of 32 contracted indices (one round of loads), more per chunk
    // when that would leave over 64 partials per element of H; X's chunk
    // within 48 KB of shared memory
    int64_t kc = HD_KB * std::max<int64_t>(1, (p.i + 64 * HD_KB - 1) / (64 * HD_KB));
    if (p.b * kc * 4 > 48 * 1024) return fail(c, TL_ERR_UNSUPPORTED, "head: contracted range too long");
    const int64_t ks = (p.i + kc - 1) / kc;
    p.ks = (int)ks;
    p.kc = kc;
    void* ws = nullptr;
    TL_TRY(workspace(c, (size_t)ks * p.b * p.h * sizeof(float), &ws, WS_GEMM));
    p.hpart = static_cast<float*>(ws);
    {
        LaunchScope L(c, "head_hidden", (double)(p.b * p.i + p.i * p.h + ks * p.b * p.h) * 4.0,
                      2.0 * p.b * p.i * p.h);
        k_head_h<<<dim3((unsigned)col_blocks, (unsigned)ks), HD_THREADS, (size_t)p.b * kc * 4, c->stream>>>(p);
        TL_TRY(L.done());
    }
    if ((size_t)p.h * 4 > 48 * 1024)
        TL_CK(c, cudaFuncSetAttribute(k_head_zy, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(p.h * 4)));
    {
        LaunchScope L(c, "head_output_softmax",
                      (double)(ks * p.b * p.h + p.b * p.h + p.h * p.o + 2 * p.b * p.o) * 4.0, 2.0 * p.b * p.h * p.o);
        k_head_zy<<<(unsigned)p.b, HD_THREADS, (size_t)p.h * 4, c->stream>>>(p);
        TL_TRY(L.done());
    }
    return TL_OK;
}

}  // namespace tl
