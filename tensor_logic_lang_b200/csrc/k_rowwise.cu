// Row-wise softmax and layer norm.
//
// Reference semantics: src/codegen/softmax.zig:19-229 (y = exp(x) / sum exp(x)
// along the `.`-marked axis, input indexed with the LHS index positions) and
// src/codegen/layernorm.zig:25-310 (biased variance, (x - mean) /
// sqrt(var + 1e-5), no affine parameters).
//
// B200 mapping: one warp per row with the row held in registers (128-bit
// loads when the row is contiguous and 16-byte aligned), so each element is
// read once and written once: the kernel is HBM-bound.  Softmax subtracts the
// row maximum before exponentiating; exp(x - m) / sum exp(x - m) equals the
// reference's unshifted quotient wherever its f64 sum is finite, and keeps
// fp32 from overflowing for inputs above 88.  Contiguous rows of 2049 to 8192
// values are held in a block's registers instead (one HBM read per value);
// longer or strided rows use a block per row and re-read the row from L2.
#include <math.h>

#include <algorithm>

#include "tl_internal.h"

namespace tl {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ void row_bases(const RowPlan& p, int64_t r, int64_t* ib, int64_t* ob) {
    int64_t in_b = 0, out_b = 0, rem = r;
    for (int o = p.n_outer - 1; o >= 0; --o) {
        const int64_t v = rem % p.outer_size[o];
        rem /= p.outer_size[o];
        in_b += v * p.outer_in_stride[o];
        out_b += v * p.outer_out_stride[o];
    }
    *ib = in_b;
    *ob = out_b;
}

// Contiguous rows, VEC values per 128-bit access, VPL values per lane.
template <int VPL, bool VEC>
__global__ void __launch_bounds__(256) k_row_warp(const __grid_constant__ RowPlan p) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < p.rows; r += n_warps) {
        int64_t ib, ob;
        row_bases(p, r, &ib, &ob);
        float v[VPL];
        const int64_t L = p.len;
        if (VEC) {
#pragma unroll
            for (int i = 0; i < VPL / 4; ++i) {
                const int64_t e = ((int64_t)i * 32 + lane) * 4;
                float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                if (e < L) x = __ldg(reinterpret_cast<const float4*>(p.in + ib + e));
                v[4 * i + 0] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const int64_t e = (int64_t)i * 32 + lane;
                const int64_t off = ib + e * p.in_sn;
                v[i] = (e < L && off >= 0 && off < p.in_total) ? __ldg(p.in + off) : 0.f;
            }
        }
        auto valid = [&](int i) -> bool {
            const int64_t e = VEC ? (((int64_t)(i / 4) * 32 + lane) * 4 + (i % 4)) : ((int64_t)i * 32 + lane);
            return e < L;
        };
        if (!p.lnorm) {
            float m = -INFINITY;
#pragma unroll
            for (int i = 0; i < VPL; ++i) if (valid(i)) m = fmaxf(m, v[i]);
            m = warp_max(m);
            if (m == -INFINITY || m != m) m = 0.f;
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                v[i] = valid(i) ? __expf(v[i] - m) : 0.f;
                s += v[i];
            }
            s = warp_sum(s);
            const float inv = 1.0f / s;
#pragma unroll
            for (int i = 0; i < VPL; ++i) v[i] *= inv;
        } else {
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < VPL; ++i) s += valid(i) ? v[i] : 0.f;
            const float mean = warp_sum(s) / (float)L;
            float q = 0.f;
#pragma unroll
            for (int i = 0; i < VPL; ++i) { const float d = valid(i) ? v[i] - mean : 0.f; q += d * d; }
            const float var = warp_sum(q) / (float)L;
            const float rs = rsqrtf(var + 1.0e-5f);
#pragma unroll
            for (int i = 0; i < VPL; ++i) v[i] = (v[i] - mean) * rs;
        }
        if (VEC) {
#pragma unroll
            for (int i = 0; i < VPL / 4; ++i) {
                const int64_t e = ((int64_t)i * 32 + lane) * 4;
                if (e < L)
                    *reinterpret_cast<float4*>(p.out + ob + e) = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const int64_t e = (int64_t)i * 32 + lane;
                const int64_t off = ob + e * p.out_sn;
                if (e < L && off >= 0 && off < p.out_total) p.out[off] = v[i];
            }
        }
    }
}

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* sh) {
    v = is_max ? warp_max(v) : warp_sum(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    float r = lane < nw ? sh[lane] : (is_max ? -INFINITY : 0.f);
    r = is_max ? warp_max(r) : warp_sum(r);
    return r;
}

// Contiguous, 16-byte aligned rows of 2049 .. 8192 values: a block per row,
// the row held in registers (VPT values per thread, 128-bit loads), so each
// value is read from HBM once and written once; two block reductions.
template <int VPT>
__global__ void __launch_bounds__(256) k_row_cta(const __grid_constant__ RowPlan p) {
    __shared__ float sh[32];
    constexpr int NV = VPT / 4;
    const int64_t L = p.len;
    for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
        int64_t ib, ob;
        row_bases(p, r, &ib, &ob);
        float4 v[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int64_t e = ((int64_t)i * blockDim.x + threadIdx.x) * 4;
            v[i] = e < L ? __ldg(reinterpret_cast<const float4*>(p.in + ib + e)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        auto valid = [&](int i) { return ((int64_t)i * blockDim.x + threadIdx.x) * 4 < L; };
        if (!p.lnorm) {
            float m = -INFINITY;
#pragma unroll
            for (int i = 0; i < NV; ++i)
                if (valid(i)) m = fmaxf(fmaxf(m, fmaxf(v[i].x, v[i].y)), fmaxf(v[i].z, v[i].w));
            m = block_reduce(m, true, sh);
            if (m == -INFINITY || m != m) m = 0.f;
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                if (valid(i)) {
                    v[i] = make_float4(__expf(v[i].x - m), __expf(v[i].y - m), __expf(v[i].z - m), __expf(v[i].w - m));
                    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
                }
            }
            const float inv = 1.0f / block_reduce(s, false, sh);
#pragma unroll
            for (int i = 0; i < NV; ++i) v[i] = make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv);
        } else {
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < NV; ++i)
                if (valid(i)) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
            const float mean = block_reduce(s, false, sh) / (float)L;
            float q = 0.f;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                if (valid(i)) {
                    const float a = v[i].x - mean, b = v[i].y - mean, c2 = v[i].z - mean, d = v[i].w - mean;
                    q += (a * a + b * b) + (c2 * c2 + d * d);
                }
            }
            const float rs = rsqrtf(block_reduce(q, false, sh) / (float)L + 1.0e-5f);
#pragma unroll
            for (int i = 0; i < NV; ++i)
                v[i] = make_float4((v[i].x - mean) * rs, (v[i].y - mean) * rs, (v[i].z - mean) * rs, (v[i].w - mean) * rs);
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int64_t e = ((int64_t)i * blockDim.x + threadIdx.x) * 4;
            if (e < L) *reinterpret_cast<float4*>(p.out + ob + e) = v[i];
        }
        __syncthreads();   // sh is reused by the next row's reductions
    }
}

// Any row length or stride: a block per row, several passes over the row.
__global__ void __launch_bounds__(256) k_row_block(const __grid_constant__ RowPlan p) {
    __shared__ float sh[32];
    for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
        int64_t ib, ob;
        row_bases(p, r, &ib, &ob);
        auto ld = [&](int64_t e) -> float {
            const int64_t off = ib + e * p.in_sn;
            return (off >= 0 && off < p.in_total) ? __ldg(p.in + off) : 0.f;
        };
        if (!p.lnorm) {
            float m = -INFINITY;
            for (int64_t e = threadIdx.x; e < p.len; e += blockDim.x) m = fmaxf(m, ld(e));
            m = block_reduce(m, true, sh);
            if (m == -INFINITY || m != m) m = 0.f;
            float s = 0.f;
            for (int64_t e = threadIdx.x; e < p.len; e += blockDim.x) s += __expf(ld(e) - m);
            s = block_reduce(s, false, sh);
            const float inv = 1.0f / s;
            for (int64_t e = threadIdx.x; e < p.len; e += blockDim.x) {
                const int64_t off = ob + e * p.out_sn;
                if (off >= 0 && off < p.out_total) p.out[off] = __expf(ld(e) - m) * inv;
            }
        } else {
            float s = 0.f;
            for (int64_t e = threadIdx.x; e < p.len; e += blockDim.x) s += ld(e);
            const float mean = block_reduce(s, false, sh) / (float)p.len;
            float q = 0.f;
            for (int64_t e = threadIdx.x; e < p.len; e += blockDim.x) { const float d = ld(e) - mean; q += d * d; }
            const float var = block_reduce(q, false, sh) / (float)p.len;
            const float rs = rsqrtf(var + 1.0e-5f);
            for (int64_t e = threadIdx.x; e < p.len; e += blockDim.x) {
                const int64_t off = ob + e * p.out_sn;
                if (off >= 0 && off < p.out_total) p.out[off] = (ld(e) - mean) * rs;
            }
        }
        __syncthreads();
    }
}

template <int VPL>
tl_status launch_warp(tl_ctx* c, const RowPlan& p, bool vec) {
    const int threads = 256;
    int64_t blocks = (p.rows + 7) / 8;
    const int64_t cap = (int64_t)c->sm_count * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    if (vec) k_row_warp<VPL, true><<<(unsigned)blocks, threads, 0, c->stream>>>(p);
    else k_row_warp<VPL, false><<<(unsigned)blocks, threads, 0, c->stream>>>(p);
    return TL_OK;
}

}  // namespace

tl_status launch_rowwise(tl_ctx* c, const RowPlan& p) {
    // bounds: the fast paths are used only when every access stays inside
    int64_t max_in = 0, max_out = 0, min_in = 0, min_out = 0;
    for (int o = 0; o < p.n_outer; ++o) {
        const int64_t a = (p.outer_size[o] - 1) * p.outer_in_stride[o];
        const int64_t b = (p.outer_size[o] - 1) * p.outer_out_stride[o];
        if (a > 0) max_in += a; else min_in += a;
        if (b > 0) max_out += b; else min_out += b;
    }
    const int64_t lin = (p.len - 1) * p.in_sn, lout = (p.len - 1) * p.out_sn;
    if (lin > 0) max_in += lin; else min_in += lin;
    if (lout > 0) max_out += lout; else min_out += lout;
    const bool inside = p.in != nullptr && min_in >= 0 && max_in < p.in_total && min_out >= 0 && max_out < p.out_total;
    bool vec = inside && p.in_sn == 1 && p.out_sn == 1 && (p.len % 4) == 0 &&
               ((uintptr_t)p.in % 16) == 0 && ((uintptr_t)p.out % 16) == 0;
    for (int o = 0; o < p.n_outer && vec; ++o)
        vec = (p.outer_in_stride[o] % 4) == 0 && (p.outer_out_stride[o] % 4) == 0;
    RowPlan q = p;
    if (!q.in) {
        // an undefined input reads 0.0 everywhere: point at a zero row
        return fail(c, TL_ERR_INVALID, "row-wise input without storage");
    }
    const double bytes = (double)p.rows * p.len * 8.0;
    LaunchScope L(c, p.lnorm ? "lnorm_rows" : "softmax_rows", bytes, (double)p.rows * p.len * 4.0);
    if (vec && p.len > 2048 && p.len <= 8192) {
        const int64_t blocks = std::min<int64_t>(std::max<int64_t>(p.rows, 1), (int64_t)c->sm_count * 8);
        if (p.len <= 4096) k_row_cta<16><<<(unsigned)blocks, 256, 0, c->stream>>>(q);
        else k_row_cta<32><<<(unsigned)blocks, 256, 0, c->stream>>>(q);
    } else if (!inside || p.len > 2048) {
        int64_t blocks = p.rows < (int64_t)c->sm_count * 16 ? p.rows : (int64_t)c->sm_count * 16;
        k_row_block<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, c->stream>>>(q);
    } else if (p.len <= 32) launch_warp<1>(c, q, false);
    else if (p.len <= 128) { if (vec) launch_warp<4>(c, q, true); else launch_warp<4>(c, q, false); }
    else if (p.len <= 256) { if (vec) launch_warp<8>(c, q, true); else launch_warp<8>(c, q, false); }
    else if (p.len <= 512) { if (vec) launch_warp<16>(c, q, true); else launch_warp<16>(c, q, false); }
    else if (p.len <= 1024) { if (vec) launch_warp<32>(c, q, true); else launch_warp<32>(c, q, false); }
    else { if (vec) launch_warp<64>(c, q, true); else launch_warp<64>(c, q, false); }
    return L.done();
}

}  // namespace tl
