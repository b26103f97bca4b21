// Dense contractions C[m,n] (+)= sum_k f(A[m,k] B[k,n] s): the GEMM-shaped
// equations of src/codegen/einsum.zig:20-254 (free indices m,n; one
// contracted index k; per-term relu from src/codegen/expr.zig:245-249).
//
// Two kernels:
//  * k_gemm_tc  — sm_100a tensor cores: TMA (cp.async.bulk.tensor, 128-byte
//    swizzle) stages fp32 tiles in shared memory, one elected thread issues
//    tcgen05.mma kind::tf32 into a TMEM accumulator, four epilogue warps
//    read it back with tcgen05.ld.  Warp-specialised, 4-6 stage mbarrier
//    pipeline, one 128 x BN tile per CTA.  Operands may be K-major or
//    MN-major (UMMA descriptors of both majors), so transposed operands of
//    the backward pass need no transpose copies.
//  * k_gemm_simt — fp32 FFMA tiles for small, skinny or unaligned shapes and
//    for TL_PREC_FP32.
// A per-term relu is exact on tensor cores through the sign split
// relu(a b) = a+ b+ + a- b- (K doubles): a prep kernel writes [A+|A-] and
// [B+;B-] as K-major copies.
#include <cuda.h>
#include <stdint.h>

#include <algorithm>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tl_internal.h"

namespace tl {
namespace {

// ============================================================================
// SIMT fp32 GEMM
// ============================================================================
constexpr int SB_M = 64, SB_K = 16;

// 64 x BN tile per block of 256 threads, each thread 4 rows x BN/16 columns.
// With gridDim.z > 1 the K range is split and partial tiles are added with
// atomics (C already holds its starting values).
template <int BN>
__global__ void __launch_bounds__(256) k_gemm_simt(const __grid_constant__ GemmPlan p, float sgn, float mag,
                                                   int64_t k_chunk) {
    constexpr int TN = BN / 16;
    __shared__ float As[SB_K][SB_M + 4];
    __shared__ float Bs[SB_K][BN + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int64_t m0 = (int64_t)blockIdx.y * SB_M, n0 = (int64_t)blockIdx.x * BN;
    const int64_t kb = (int64_t)blockIdx.z * k_chunk;
    const int64_t ke = kb + k_chunk < p.K ? kb + k_chunk : p.K;
    const bool a_kmajor = p.sak == 1, b_nmajor = p.sbn == 1;
    constexpr int A_PER = SB_M * SB_K / 256, B_PER = (BN * SB_K + 255) / 256;
    // the next tile's loads are issued into registers before this tile's FMAs
    float ra[A_PER], rb[B_PER];
    auto load = [&](int64_t k0) {
#pragma unroll
        for (int t = 0; t < A_PER; ++t) {
            const int i = threadIdx.x + t * 256;
            // walk the contiguous dimension of A across consecutive threads
            const int mm = a_kmajor ? i / SB_K : i % SB_M;
            const int kk = a_kmajor ? i % SB_K : i / SB_M;
            const int64_t gm = m0 + mm, gk = k0 + kk;
            ra[t] = (gm < p.M && gk < ke) ? p.A[gm * p.sam + gk * p.sak] : 0.f;
        }
#pragma unroll
        for (int t = 0; t < B_PER; ++t) {
            const int i = threadIdx.x + t * 256;
            const int nn = b_nmajor ? i % BN : i / SB_K;
            const int kk = b_nmajor ? i / BN : i % SB_K;
            const int64_t gn = n0 + nn, gk = k0 + kk;
            rb[t] = (i < BN * SB_K && gn < p.N && gk < ke) ? p.B[gk * p.sbk + gn * p.sbn] * sgn : 0.f;
        }
    };
    float acc[4][TN] = {};
    if (kb < ke) load(kb);
    for (int64_t k0 = kb; k0 < ke; k0 += SB_K) {
#pragma unroll
        for (int t = 0; t < A_PER; ++t) {
            const int i = threadIdx.x + t * 256;
            As[a_kmajor ? i % SB_K : i / SB_M][a_kmajor ? i / SB_K : i % SB_M] = ra[t];
        }
#pragma unroll
        for (int t = 0; t < B_PER; ++t) {
            const int i = threadIdx.x + t * 256;
            if (i < BN * SB_K) Bs[b_nmajor ? i / BN : i % SB_K][b_nmajor ? i % BN : i / SB_K] = rb[t];
        }
        __syncthreads();
        if (k0 + SB_K < ke) load(k0 + SB_K);
#pragma unroll
        for (int kk = 0; kk < SB_K; ++kk) {
            float a[4], b[TN];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tx * TN + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) {
                    if (p.relu_term) acc[i][j] += fmaxf(a[i] * b[j], 0.f);
                    else acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
                }
        }
        __syncthreads();
    }
    const bool split = gridDim.z > 1;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t gm = m0 + ty * 4 + i;
        if (gm >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int64_t gn = n0 + tx * TN + j;
            if (gn >= p.N) continue;
            float v = acc[i][j] * mag;
            float* cp = p.C + gm * p.scm + gn * p.scn;
            if (split) { atomicAdd(cp, v); continue; }
            if (p.beta) v += *cp;
            *cp = v;
            if (p.epi_relu) p.D[gm * p.sdm + gn * p.sdn] = fmaxf(v, 0.f);
        }
    }
}

// ============================================================================
// Skinny shapes (no per-term nonlinearity), fp32 FFMA, bandwidth-bound
// ============================================================================
// C[M, N <= 16] = scale * A[M, K] B[K, N] with a long K (the output layer and
// its weight gradient).  Both kernels keep many loads of A in flight (the
// cost is streaming A once) and add partial sums with atomics when K is split
// over blockIdx.y (C zeroed first unless it accumulates).
//
// k_skinny_kcont, A's k contiguous: a block owns 32 rows (4 per warp) and a
// 512-wide K range.  B's slice is staged n-major, so lane l reads column n at
// k = 4l .. 4l+3 with one 128-bit load shared by the warp's 4 rows (rows of
// the slice padded by 4 floats, so the staging stores spread over the banks);
// each lane keeps 8 128-bit loads of A in flight, and the warp reduces its 64
// sums (4 rows x 16 columns) with a transpose-reduction: 5 shuffle levels
// that each halve the values a lane keeps (62 shuffles), after which lane l
// holds sums 2l and 2l + 1.
constexpr int SKC_RPW = 4, SKC_ROWS = 8 * SKC_RPW, SKC_K = 512, SKC_PAD = 4;
// k_skinny_mcont, A's rows contiguous (a transposed activation): lane = row,
// a block owns 32 rows and a 256-wide K range, warp w takes k = w, w + 8, ...
// (32 loads in flight per lane), B's slice is staged k-major (broadcast
// reads), and the 8 warps' sums are added in shared memory.
constexpr int SKM_ROWS = 32, SKM_K = 256;

__device__ __forceinline__ void skinny_put(const GemmPlan& p, int64_t m, int n, float v, bool atomic) {
    if (m >= p.M || n >= p.N) return;
    float* cp = p.C + m * p.scm + n * p.scn;
    v *= p.scale;
    if (atomic) atomicAdd(cp, v);
    else *cp = p.beta ? *cp + v : v;
}

// B[k0 + kk, nn] for kk < KMAX, nn < 16 (zero past kn and N) into dst(kk, nn),
// walking whichever of k / n is contiguous in memory.  Each of the 256
// threads issues all of its KMAX * 16 / 256 loads before any store, so the
// slice costs one memory round trip.
template <int KMAX, typename F>
__device__ __forceinline__ void stage_b(const GemmPlan& p, int64_t k0, int kn, F dst) {
    constexpr int PER = KMAX * 16 / 256;
    static_assert(KMAX * 16 % 256 == 0, "256 threads stage the slice");
    float v[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
        const int i = threadIdx.x + u * 256;
        const int kk = p.sbn == 1 ? (i >> 4) : (i % KMAX);
        const int nn = p.sbn == 1 ? (i & 15) : (i / KMAX);
        v[u] = (kk < kn && nn < p.N) ? p.B[(k0 + kk) * p.sbk + nn * p.sbn] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < PER; ++u) {
        const int i = threadIdx.x + u * 256;
        dst(p.sbn == 1 ? (i >> 4) : (i % KMAX), p.sbn == 1 ? (i & 15) : (i / KMAX), v[u]);
    }
}

__global__ void __launch_bounds__(256) k_skinny_kcont(const __grid_constant__ GemmPlan p, int vec) {
    __shared__ __align__(16) float Bt[16][SKC_K + SKC_PAD];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t m0 = (int64_t)blockIdx.x * SKC_ROWS + w * SKC_RPW;
    const int64_t kc = (int64_t)blockIdx.y * SKC_K;
    const int kn = (int)(p.K - kc < SKC_K ? p.K - kc : SKC_K);
    stage_b<SKC_K>(p, kc, kn, [&](int kk, int nn, float v) { Bt[nn][kk] = v; });
    __syncthreads();
    float acc[SKC_RPW][16];
#pragma unroll
    for (int r = 0; r < SKC_RPW; ++r)
#pragma unroll
        for (int nn = 0; nn < 16; ++nn) acc[r][nn] = 0.f;
    // the warp's rows at 4 consecutive k per lane, two 128-wide k groups per
    // round (8 loads of A in flight), each column of B read once per group
    // and used by all the warp's rows
    for (int g0 = 0; g0 < SKC_K / 128; g0 += 2) {
        float a[2][SKC_RPW][4];
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int r = 0; r < SKC_RPW; ++r) {
                const int kk = lane * 4 + 128 * (g0 + u);
                const int64_t m = m0 + r;
                const float* ap = p.A + m * p.sam + kc + kk;
                if (m < p.M && vec && kk + 3 < kn) {
                    const float4 t = *reinterpret_cast<const float4*>(ap);
                    a[u][r][0] = t.x; a[u][r][1] = t.y; a[u][r][2] = t.z; a[u][r][3] = t.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) a[u][r][j] = (m < p.M && kk + j < kn) ? ap[j] : 0.f;
                }
            }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int kk = lane * 4 + 128 * (g0 + u);
#pragma unroll
            for (int nn = 0; nn < 16; ++nn) {
                if (nn >= p.N) break;
                const float4 b = *reinterpret_cast<const float4*>(&Bt[nn][kk]);
#pragma unroll
                for (int r = 0; r < SKC_RPW; ++r) {
                    float t = fmaf(a[u][r][0], b.x, acc[r][nn]);
                    t = fmaf(a[u][r][1], b.y, t);
                    t = fmaf(a[u][r][2], b.z, t);
                    acc[r][nn] = fmaf(a[u][r][3], b.w, t);
                }
            }
        }
    }
    static_assert(SKC_RPW * 16 == 64, "the transpose-reduction takes 64 sums per lane");
    float v[64];
#pragma unroll
    for (int r = 0; r < SKC_RPW; ++r)
#pragma unroll
        for (int nn = 0; nn < 16; ++nn) v[r * 16 + nn] = acc[r][nn];
#pragma unroll
    for (int o = 16, cnt = 32; o >= 1; o >>= 1, cnt >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < cnt; ++i) {
            const float send = upper ? v[i] : v[i + cnt];
            const float keep = upper ? v[i + cnt] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    // lane l: sums 2l and 2l + 1 of the flattened (row, column) order
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int idx = 2 * lane + j;
        skinny_put(p, m0 + idx / 16, idx % 16, v[j], gridDim.y > 1);
    }
}

__global__ void __launch_bounds__(256) k_skinny_mcont(const __grid_constant__ GemmPlan p) {
    __shared__ __align__(16) float Bs[SKM_K][16];
    __shared__ float red[8][SKM_ROWS][17];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t m = (int64_t)blockIdx.x * SKM_ROWS + lane;
    const int64_t kc = (int64_t)blockIdx.y * SKM_K;
    const int kn = (int)(p.K - kc < SKM_K ? p.K - kc : SKM_K);
    stage_b<SKM_K>(p, kc, kn, [&](int kk, int nn, float v) { Bs[kk][nn] = v; });
    constexpr int U = SKM_K / 8;
    float a[U];
    const float* ap = p.A + m * p.sam + kc * p.sak;
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int kk = w + 8 * u;
        a[u] = (m < p.M && kk < kn) ? ap[kk * p.sak] : 0.f;
    }
    __syncthreads();
    float acc[16];
#pragma unroll
    for (int nn = 0; nn < 16; ++nn) acc[nn] = 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const float4* b4 = reinterpret_cast<const float4*>(Bs[w + 8 * u]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 b = b4[q];
            acc[4 * q + 0] = fmaf(a[u], b.x, acc[4 * q + 0]);
            acc[4 * q + 1] = fmaf(a[u], b.y, acc[4 * q + 1]);
            acc[4 * q + 2] = fmaf(a[u], b.z, acc[4 * q + 2]);
            acc[4 * q + 3] = fmaf(a[u], b.w, acc[4 * q + 3]);
        }
    }
#pragma unroll
    for (int nn = 0; nn < 16; ++nn) red[w][lane][nn] = acc[nn];
    __syncthreads();
    for (int i = threadIdx.x; i < SKM_ROWS * 16; i += 256) {
        const int r = i >> 4, nn = i & 15;
        float v = 0.f;
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) v += red[ww][r][nn];
        skinny_put(p, (int64_t)blockIdx.x * SKM_ROWS + r, nn, v, gridDim.y > 1);
    }
}

// C[M, N] = scale * A[M, K <= 16] B[K, N] (an outer-product-like GEMM whose
// cost is writing C): thread t of block x loads B[:, 4t .. 4t+3] of the
// block's TK_COLS columns into registers (K padded to 16 with zeros), the
// block's rows of A (at most TK_ROWS) are staged in shared memory, and each
// row costs the thread four broadcast shared loads, 64 FMAs and one 128-bit
// store.
constexpr int TK_ROWS = 16, TK_THREADS = 128, TK_COLS = 4 * TK_THREADS;

__global__ void __launch_bounds__(TK_THREADS) k_gemm_thin_k(const __grid_constant__ GemmPlan p, int64_t rows_per_block,
                                                     int vec) {
    __shared__ __align__(16) float As[TK_ROWS][16];
    const int64_t n = ((int64_t)blockIdx.x * TK_THREADS + threadIdx.x) * 4;
    // this thread's 4 columns of B: up to 64 independent loads, all in flight
    float b[16][4];
#pragma unroll
    for (int k = 0; k < 16; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) b[k][j] = (k < p.K && n + j < p.N) ? p.B[k * p.sbk + (n + j) * p.sbn] : 0.f;
    const int64_t mb = (int64_t)blockIdx.y * rows_per_block;
    const int64_t me = mb + rows_per_block < p.M ? mb + rows_per_block : p.M;
    for (int i = threadIdx.x; i < TK_ROWS * 16; i += blockDim.x) {
        const int r = i >> 4, k = i & 15;
        As[r][k] = (mb + r < me && k < p.K) ? p.A[(mb + r) * p.sam + k * p.sak] : 0.f;
    }
    __syncthreads();
    if (n >= p.N) return;
    for (int64_t m = mb; m < me; ++m) {
        const float4* a4 = reinterpret_cast<const float4*>(As[m - mb]);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 a = a4[q];
            const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[j] = fmaf(av[i], b[4 * q + i][j], acc[j]);
        }
        float* cp = p.C + m * p.scm + n * p.scn;
        if (vec && n + 3 < p.N) {
            float4 v = make_float4(acc[0] * p.scale, acc[1] * p.scale, acc[2] * p.scale, acc[3] * p.scale);
            if (p.beta) {
                const float4 o = *reinterpret_cast<const float4*>(cp);
                v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
            }
            *reinterpret_cast<float4*>(cp) = v;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (n + j < p.N) {
                    const float v = acc[j] * p.scale;
                    float* q = cp + j * p.scn;
                    *q = p.beta ? *q + v : v;
                }
        }
    }
}

// ============================================================================
// tcgen05 TF32 GEMM
// ============================================================================
constexpr int TC_BM = 128;
constexpr int TC_BK = 32;               // 32 fp32 = 128 bytes = one swizzle row
constexpr int TC_THREADS = 192;         // warp0 TMA, warp1 MMA, warps 2-5 epilogue
constexpr uint64_t kWaitLimitNs = 2000000000ull;

struct TcEpi {
    float* C; int64_t scm, scn;
    float* D; int64_t sdm, sdn;
    int64_t M, N;
    float mag;
    int beta, epi_relu;
    int* err;
    float* fan[kMaxPeers];                  // peer copies of C (GemmPlan::fan)
    unsigned long long* fan_cnt[kMaxPeers];
    int fan_n;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: gives up after ~2 s of device time, flags *err and returns
// false, so a pipeline that never completes ends the kernel instead of
// hanging the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (unsigned it = 0;; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(addr), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((it & 1023u) == 0) {
            const uint64_t now = globaltimer_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > kWaitLimitNs) break;
        }
    }
    if (err) atomicExch(err, 1);
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// UMMA shared-memory descriptor (sm_100 version 1).  Layout type 2 is the
// 128-byte swizzle of K-major tiles; type 1 is the 128-byte swizzle with a
// 32-byte atom, the one shared-memory layout MN-major tf32 operands have.
constexpr uint64_t kLayoutSW128 = 2, kLayoutSW128Base32B = 1;
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint64_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;                 // descriptor version (Blackwell)
    d |= layout << 61;
    return d;
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Epilogue stores through the TMA: a 32 x 32 fp32 tile in shared memory (rows
// of 128 bytes, 16-byte chunk j of row r at position j ^ (r & 7): the 128-byte
// swizzle) written to the tensor map's box at {x, y}, plainly or added
// element-wise in L2 (accumulation and split K).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// NSEG = 2 (3xTF32 as hi/lo pairs): a stage holds the hi and lo tiles of A
// and of B for one k-block, and the MMA warp issues hi*hi, hi*lo and lo*hi.
template <int BN, int NSEG = 1>
struct TcCfg {
    static constexpr int A_BYTES = TC_BM * TC_BK * 4;      // 16 KB per segment
    static constexpr int B_BYTES = BN * TC_BK * 4;
    static constexpr int STAGE = NSEG * (A_BYTES + B_BYTES);
    static constexpr int STAGES = (196 * 1024) / STAGE > 8 ? 8 : (196 * 1024) / STAGE;
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
    static constexpr int SMEM = STAGES * STAGE + 1024 /*align*/ + 256 /*barriers*/;
};

// A_MN / B_MN: operand stored MN-major (M or N is the contiguous dim).
// P3 (3xTF32): tmA / tmB map the hi copies and tmA1 / tmB1 the lo copies,
// each K long (zeros past it); every k-block of K takes three products.
template <int BN, bool A_MN, bool B_MN, bool P3>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
              const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
              const __grid_constant__ TcEpi epi, int num_kb, int kb_per_split, int tma_store) {
    constexpr int NSEG = P3 ? 2 : 1;
    using Cfg = TcCfg<BN, NSEG>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE);
    uint64_t* empty = full + Cfg::STAGES;
    uint64_t* accum_full = empty + Cfg::STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_full + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int m0 = blockIdx.y * TC_BM, n0 = blockIdx.x * BN;
    // this CTA's K range: k-blocks [kb_first, kb_first + n_kb) of num_kb
    const int kb_first = blockIdx.z * kb_per_split;
    const int n_kb = min(kb_per_split, num_kb - kb_first);
    const bool split_k = gridDim.z > 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(accum_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(Cfg::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            for (int kb = 0; kb < n_kb; ++kb) {
                const int s = kb % Cfg::STAGES;
                const uint32_t ph = (kb / Cfg::STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, epi.err)) break;
                uint8_t* stage = smem + s * Cfg::STAGE;
                mbar_expect_tx(&full[s], Cfg::STAGE);
                const int k0 = (kb_first + kb) * TC_BK;
#pragma unroll
                for (int g = 0; g < NSEG; ++g) {
                    uint8_t* sa = stage + g * Cfg::A_BYTES;
                    uint8_t* sb = stage + NSEG * Cfg::A_BYTES + g * Cfg::B_BYTES;
                    const CUtensorMap* ma = g ? &tmA1 : &tmA;
                    const CUtensorMap* mb = g ? &tmB1 : &tmB;
                    if (!A_MN) {
                        tma_load_2d(sa, ma, &full[s], k0, m0);
                    } else {
#pragma unroll
                        for (int j = 0; j < TC_BM / 32; ++j) tma_load_2d(sa + j * 4096, ma, &full[s], m0 + 32 * j, k0);
                    }
                    if (!B_MN) {
                        tma_load_2d(sb, mb, &full[s], k0, n0);
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / 32; ++j) tma_load_2d(sb + j * 4096, mb, &full[s], n0 + 32 * j, k0);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc = (1u << 4)                        // D = F32
                                   | (2u << 7) | (2u << 10)          // A, B = TF32
                                   | ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16)
                                   | ((uint32_t)(BN >> 3) << 17)     // N
                                   | ((uint32_t)(TC_BM >> 4) << 24); // M
        bool ok = true;
        for (int kb = 0; kb < n_kb && ok; ++kb) {
            const int s = kb % Cfg::STAGES;
            const uint32_t ph = (kb / Cfg::STAGES) & 1;
            ok = mbar_wait(&full[s], ph, epi.err);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (lane == 0) {
                const uint32_t stage = smem_u32(smem + s * Cfg::STAGE);
                // (A segment, B segment) products: one, or hi*hi, hi*lo, lo*hi
                constexpr int NP = P3 ? 3 : 1;
#pragma unroll
                for (int pr = 0; pr < NP; ++pr) {
                    const int ga = pr == 2 ? 1 : 0, gb = pr == 1 ? 1 : 0;
                    const uint32_t sa = stage + ga * Cfg::A_BYTES;
                    const uint32_t sb = stage + NSEG * Cfg::A_BYTES + gb * Cfg::B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 8; ++kk) {
                        // K-major: advance 32 bytes inside the swizzled 128-byte row; SBO = 8 rows.
                        // MN-major: 8 K rows of 128 bytes per MMA (two 4-row 32B-atom groups,
                        // SBO = 512 bytes); LBO = the next 32-wide MN chunk (one 4 KB box).
                        const uint64_t ad = A_MN ? umma_desc(sa + kk * 1024, 4096, 512, kLayoutSW128Base32B)
                                                 : umma_desc(sa + kk * 32, 16, 1024, kLayoutSW128);
                        const uint64_t bd = B_MN ? umma_desc(sb + kk * 1024, 4096, 512, kLayoutSW128Base32B)
                                                 : umma_desc(sb + kk * 32, 16, 1024, kLayoutSW128);
                        umma_tf32(tmem, ad, bd, idesc, (kb > 0 || pr > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                umma_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (lane == 0) umma_commit(accum_full);
        __syncwarp();
    } else {
        // ---------------- epilogue: TMEM -> registers -> global ----------------
        const int q = warp & 3;                      // TMEM lane quarter of this warp
        const bool ok = mbar_wait(accum_full, 0, epi.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int64_t row = (int64_t)m0 + q * 32 + lane;
        if (ok && tma_store && (n_kb > 0 || !split_k)) {
            // coalesced stores by the TMA: per 32-column chunk, this warp's 32
            // rows go through a swizzled shared tile (the pipeline's stage
            // memory is free now), two tiles in flight per warp
            const bool add = split_k || epi.beta;
            uint8_t* ebase = smem + (size_t)q * 16384;
#pragma unroll 1
            for (int ch = 0; ch < BN / 32; ++ch) {
                uint8_t* sc = ebase + (ch & 1) * 8192;
                uint8_t* sd = sc + 4096;
                if (ch >= 2) {
                    if (lane == 0) bulk_wait_read_1();   // the store of chunk ch - 2 has read this tile
                    __syncwarp();
                }
                float v[32];
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + ch * 32, v);
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + ch * 32 + 16, v + 16);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 o = make_float4(v[4 * j] * epi.mag, v[4 * j + 1] * epi.mag, v[4 * j + 2] * epi.mag,
                                                 v[4 * j + 3] * epi.mag);
                    const int off = lane * 128 + ((j ^ (lane & 7)) << 4);
                    *reinterpret_cast<float4*>(sc + off) = o;
                    if (epi.epi_relu)
                        *reinterpret_cast<float4*>(sd + off) =
                            make_float4(fmaxf(o.x, 0.f), fmaxf(o.y, 0.f), fmaxf(o.z, 0.f), fmaxf(o.w, 0.f));
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    const int x = n0 + ch * 32, y = m0 + q * 32;
                    if (add) tma_reduce_add_2d(&tmC, sc, x, y);
                    else tma_store_2d(&tmC, sc, x, y);
                    if (epi.epi_relu) tma_store_2d(&tmD, sd, x, y);
                    bulk_commit();
                }
                if (epi.fan_n) {
                    // the same 32 x 32 chunk into every peer's copy: the warp
                    // reads the staged tile back four rows at a time, so each
                    // store instruction writes four 128-byte row pieces
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int r = i * 4 + (lane >> 3), c4 = lane & 7;
                        const int64_t grow = (int64_t)m0 + q * 32 + r;
                        const int64_t gcol = (int64_t)n0 + ch * 32 + c4 * 4;   // N is a multiple of 4
                        if (grow >= epi.M || gcol >= epi.N) continue;
                        const float4 v = *reinterpret_cast<const float4*>(sc + r * 128 + ((c4 ^ (r & 7)) << 4));
                        const int64_t off = grow * epi.scm + gcol;
#pragma unroll
                        for (int j = 0; j < kMaxPeers; ++j)
                            if (epi.fan[j]) *reinterpret_cast<float4*>(epi.fan[j] + off) = v;
                    }
                }
            }
            if (lane == 0) bulk_wait_all();
            __syncwarp();
        } else if (ok && n_kb > 0 && split_k) {
            // partial tile of a split K range: add into C
#pragma unroll 1
            for (int ch = 0; ch < BN / 16; ++ch) {
                float v[16];
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + ch * 16, v);
                if (row >= epi.M) continue;
                const int64_t col0 = (int64_t)n0 + ch * 16;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (col0 + j < epi.N) atomicAdd(epi.C + row * epi.scm + (col0 + j) * epi.scn, v[j] * epi.mag);
            }
        } else if (ok && !split_k) {
#pragma unroll 1
            for (int ch = 0; ch < BN / 16; ++ch) {
                float v[16];
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + ch * 16, v);
                if (row >= epi.M) continue;
                const int64_t col0 = (int64_t)n0 + ch * 16;
                float* crow = epi.C + row * epi.scm;
                const bool vec = epi.scn == 1 && col0 + 16 <= epi.N && (((uintptr_t)(crow + col0)) & 15) == 0;
                if (vec) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        float4* cp = reinterpret_cast<float4*>(crow + col0 + j);
                        float4 o = make_float4(v[j] * epi.mag, v[j + 1] * epi.mag, v[j + 2] * epi.mag, v[j + 3] * epi.mag);
                        if (epi.beta) { const float4 old = *cp; o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w; }
                        *cp = o;
                        if (epi.epi_relu) {
                            float* dp = epi.D + row * epi.sdm + (col0 + j) * epi.sdn;
                            dp[0] = fmaxf(o.x, 0.f); dp[epi.sdn] = fmaxf(o.y, 0.f);
                            dp[2 * epi.sdn] = fmaxf(o.z, 0.f); dp[3 * epi.sdn] = fmaxf(o.w, 0.f);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int64_t col = col0 + j;
                        if (col >= epi.N) break;
                        float* cp = crow + col * epi.scn;
                        float o = v[j] * epi.mag;
                        if (epi.beta) o += *cp;
                        *cp = o;
                        if (epi.epi_relu) epi.D[row * epi.sdm + col * epi.sdn] = fmaxf(o, 0.f);
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::TMEM_COLS));
    }
    if (epi.fan_n && threadIdx.x == 0) {
        // every warp's peer stores of this tile happen before the barrier
        // above; the fence and the release make them visible to a rank that
        // reads its counter with acquire at system scope
        __threadfence_system();
#pragma unroll 1
        for (int j = 0; j < kMaxPeers; ++j)
            if (epi.fan_cnt[j])
                asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(epi.fan_cnt[j]), "l"(1ull) : "memory");
    }
}

// Round an fp32 value to TF32 (10-bit mantissa), nearest with ties away from
// zero.  The tensor cores would otherwise drop the low 13 bits (truncation),
// which biases sums of same-sign terms such as the sign-split products.
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Tensor-core operand copies.  An operand is viewed as R rows (M or N) by K;
// the copy holds nseg segments of K values each, segment s transformed by
// op s (4 bits each in `ops`), applied to x = sgn * source:
//   OP_RN   round(x)                      plain TF32 operand
//   OP_LO   round(x - round(x))           low part (3xTF32: hi*hi + hi*lo + lo*hi)
//   OP_POS  round(max(x, 0))              relu sign split: a+ b+ + a- b-
//   OP_NEG  round(max(-x, 0))
enum { OP_RN = 0, OP_LO = 1, OP_POS = 2, OP_NEG = 3 };

__device__ __forceinline__ float seg_op(int op, float x) {
    switch (op) {
    case OP_LO: { const float h = tf32_rna(x); return tf32_rna(x - h); }
    case OP_POS: return tf32_rna(fmaxf(x, 0.f));
    case OP_NEG: return tf32_rna(fmaxf(-x, 0.f));
    default: return tf32_rna(x);
    }
}

// One operand's row-wise copy (k_prep_rows below): its grid is gx x gy blocks.
struct PrepRows {
    const float* S;
    int64_t src_rs, rows, len;
    int nseg;
    unsigned ops;
    float sgn;
    float* D;
    int64_t dst_rs, dst_ss;
    int vec, tpr_log2;
    unsigned gx, gy;
};

// Row-wise segment copy: for each source row i (stride src_rs, len elements,
// contiguous) and segment s, dst[i * dst_rs + s * dst_ss + j] = op_s(x[j]).
// Serves both orientations: K-major copies of K-contiguous sources (rows = R)
// and MN-major copies of MN-contiguous sources (rows = K).  A block's 256
// threads cover 256 / tpr rows of tpr threads each (tpr a power of two sized
// to the row, so short rows do not leave most threads idle); a 2-D grid (row
// chunks x row groups) needs no index division; 128-bit loads and stores when
// every stride and base is 16-byte aligned.
// Both operands of a GEMM go in one launch: blockIdx.z picks the operand,
// and blocks past that operand's own gx x gy grid return.
__global__ void __launch_bounds__(256) k_prep_rows(const __grid_constant__ PrepRows pr0,
                                                   const __grid_constant__ PrepRows pr1) {
    const PrepRows& a = blockIdx.z ? pr1 : pr0;
    if (blockIdx.x >= a.gx || blockIdx.y >= a.gy) return;
    const float* __restrict__ S = a.S;
    float* __restrict__ D = a.D;
    const int64_t src_rs = a.src_rs, rows = a.rows, len = a.len, dst_rs = a.dst_rs, dst_ss = a.dst_ss;
    const int nseg = a.nseg;
    const unsigned ops = a.ops;
    const float sgn = a.sgn;
    const int tpr_log2 = a.tpr_log2;
    const int tpr = 1 << tpr_log2, rpb = 256 >> tpr_log2;
    const int t = threadIdx.x & (tpr - 1);
    const int64_t row_step = (int64_t)a.gy * rpb;
    if (a.vec) {
        // up to four rows per thread (as the grid leaves them), their loads
        // issued before any store
        for (int64_t i0 = (int64_t)blockIdx.y * rpb + (threadIdx.x >> tpr_log2); i0 < rows; i0 += 4 * row_step) {
            for (int64_t j = ((int64_t)blockIdx.x * tpr + t) * 4; j < len; j += (int64_t)a.gx * tpr * 4) {
                float4 x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int64_t i = i0 + u * row_step;
                    x[u] = i < rows ? *reinterpret_cast<const float4*>(S + i * src_rs + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int64_t i = i0 + u * row_step;
                    if (i >= rows) break;
                    float4 y = x[u];
                    y.x *= sgn; y.y *= sgn; y.z *= sgn; y.w *= sgn;
                    float* dst = D + i * dst_rs;
                    for (int sg = 0; sg < nseg; ++sg) {
                        const int op = (ops >> (4 * sg)) & 15;
                        *reinterpret_cast<float4*>(dst + sg * dst_ss + j) =
                            make_float4(seg_op(op, y.x), seg_op(op, y.y), seg_op(op, y.z), seg_op(op, y.w));
                    }
                }
            }
        }
        return;
    }
    for (int64_t i = (int64_t)blockIdx.y * rpb + (threadIdx.x >> tpr_log2); i < rows; i += row_step) {
        const float* src = S + i * src_rs;
        float* dst = D + i * dst_rs;
        for (int64_t j = (int64_t)blockIdx.x * tpr + t; j < len; j += (int64_t)a.gx * tpr) {
            const float x = src[j] * sgn;
            for (int sg = 0; sg < nseg; ++sg) dst[sg * dst_ss + j] = seg_op((ops >> (4 * sg)) & 15, x);
        }
    }
}

// K-major copy of a source with any strides, through 32 x 33 shared-memory
// tiles so both the reads (along the source's fastest dim) and the writes
// (along k) coalesce.
__global__ void k_prep_transpose(const float* __restrict__ S, int64_t s_r, int64_t s_k, int64_t R, int64_t K,
                                 int nseg, unsigned ops, float sgn, float* __restrict__ D, int64_t ld) {
    __shared__ float tile[32][33];
    const int64_t r0 = (int64_t)blockIdx.x * 32, k0 = (int64_t)blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t k = k0 + i, r = r0 + threadIdx.x;   // read along r
        tile[i][threadIdx.x] = (r < R && k < K) ? S[r * s_r + k * s_k] * sgn : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t r = r0 + i, k = k0 + threadIdx.x;   // write along k
        if (r < R && k < K) {
            const float x = tile[threadIdx.x][i];
            for (int s = 0; s < nseg; ++s) D[r * ld + s * K + k] = seg_op((ops >> (4 * s)) & 15, x);
        }
    }
}

// ============================================================================
// Attention block: S = scale Q K^T, A = softmax over keys, O = A V (d = 64)
// ============================================================================
// The three equations of an attention block (softmax.zig:19-229 between two
// einsum contractions, einsum.zig:20-254) as two kernels, Scores and Attn
// still written in full:
//  * k_attn_tile, one CTA per (128 queries, 128 keys) tile: TMA brings the
//    Q, K and V tiles into shared memory, where they are rounded to TF32
//    (nearest) in place; one elected thread issues S = Q K^T with
//    tcgen05.mma into TMEM; the four softmax warps read S back (a row per
//    thread), store scale * S through the TMA, take the row maximum m and
//    sum l of exp(S - m) over the tile's keys, and write P = exp(S - m)
//    (TF32) into shared memory in the 128-byte-swizzled K-major layout the
//    tensor cores read (over Q and K, done with by then); O_tile = P V goes
//    into TMEM with a second tcgen05.mma and is stored unnormalised with m and
//    l.  97 KB of shared memory: two CTAs per SM.
//  * k_attn_rows, a warp per query row: m* = max of the tiles' m, l* = sum
//    of exp(m - m*) l, O = sum of exp(m - m*) O_tile / l*, and the row of A =
//    exp(S - m*) / l* from the stored scores.
// The softmax subtracts the row maximum, as the row-wise kernel does; the
// quotient equals the reference's exp(x) / sum exp(x) wherever its sum is
// finite.
constexpr int AT_ROWS = 128, AT_KEYS = 128, AT_D = 64, AT_THREADS = 192;
constexpr int AT_Q = 0, AT_K = 32768, AT_V = 65536, AT_P = 0, AT_BAR = 98304;   // P over Q and K
constexpr int AT_SMEM = AT_BAR + 256 + 1024;   // + barriers, + alignment slack
constexpr uint32_t AT_TMEM_COLS = 256;          // S in columns 0..127, O in 128..191

struct AttnArgs {
    float* S;             // scores, row-major with row stride ls
    int64_t ls;
    int64_t n_q;          // queries (rows of Q, S, O)
    float scale;          // the equation's literal factor on Q K^T
    float* opart;         // [key tiles][n_q][64]: P V of each key tile, unnormalised
    float* mpart;         // [key tiles][n_q]: row maximum of scale * S over the tile
    float* lpart;         // [key tiles][n_q]: row sum of exp(scale * S - m) over the tile
    int* err;             // a bounded pipeline wait ran out
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Every fp32 of [base, base + bytes) rounded to TF32 in place by nthreads threads.
__device__ __forceinline__ void round_tf32_inplace(uint8_t* base, int bytes, int t, int nthreads) {
    for (int off = t * 16; off < bytes; off += nthreads * 16) {
        float4 v = *reinterpret_cast<float4*>(base + off);
        v.x = tf32_rna(v.x); v.y = tf32_rna(v.y); v.z = tf32_rna(v.z); v.w = tf32_rna(v.w);
        *reinterpret_cast<float4*>(base + off) = v;
    }
}

__global__ void __launch_bounds__(AT_THREADS, 2)
    k_attn_tile(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmS,
                const __grid_constant__ AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // 0: Q, K landed  1: V landed  2: Q, K rounded  3: V rounded  4: S done  5: P written  6: O done
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + AT_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 8);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int m0 = blockIdx.x * AT_ROWS, n0 = blockIdx.y * AT_KEYS;

    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1); mbar_init(&bar[1], 1);
        mbar_init(&bar[2], 160); mbar_init(&bar[3], 32);
        mbar_init(&bar[4], 1); mbar_init(&bar[5], 128); mbar_init(&bar[6], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmK)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmV)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(AT_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA: Q and K as two 32-wide K-major blocks each, V
        // as four 32-key blocks of two 32 x 32 MN-major boxes; then this warp
        // helps round Q and K, and rounds V alone (V is needed only by the
        // second MMA, so its rounding stays off the softmax warps' path) -------
        if (lane == 0) {
            mbar_expect_tx(&bar[0], 4 * 16384);
            tma_load_2d(smem + AT_Q, &tmQ, &bar[0], 0, m0);
            tma_load_2d(smem + AT_Q + 16384, &tmQ, &bar[0], 32, m0);
            tma_load_2d(smem + AT_K, &tmK, &bar[0], 0, n0);
            tma_load_2d(smem + AT_K + 16384, &tmK, &bar[0], 32, n0);
            mbar_expect_tx(&bar[1], 8 * 4096);
#pragma unroll
            for (int kb = 0; kb < 4; ++kb)
#pragma unroll
                for (int j = 0; j < 2; ++j)
                    tma_load_2d(smem + AT_V + kb * 8192 + j * 4096, &tmV, &bar[1], 32 * j, n0 + 32 * kb);
        }
        __syncwarp();
        bool ok = mbar_wait(&bar[0], 0, a.err);
        if (ok) round_tf32_inplace(smem + AT_Q, 4 * 16384, 128 + lane, 160);
        fence_proxy_async_smem();
        mbar_arrive(&bar[2]);
        ok = ok && mbar_wait(&bar[1], 0, a.err);
        if (ok) round_tf32_inplace(smem + AT_V, 8 * 4096, lane, 32);
        fence_proxy_async_smem();
        mbar_arrive(&bar[3]);
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc_s = (1u << 4) | (2u << 7) | (2u << 10)           // D f32, A, B tf32
                                     | ((uint32_t)(AT_KEYS >> 3) << 17) | ((uint32_t)(AT_ROWS >> 4) << 24);
        constexpr uint32_t idesc_o = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 16)   // B MN-major
                                     | ((uint32_t)(AT_D >> 3) << 17) | ((uint32_t)(AT_ROWS >> 4) << 24);
        bool ok = mbar_wait(&bar[2], 0, a.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok && lane == 0) {
#pragma unroll
            for (int kb = 0; kb < 2; ++kb)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t ad = umma_desc(smem_u32(smem + AT_Q + kb * 16384) + kk * 32, 16, 1024, kLayoutSW128);
                    const uint64_t bd = umma_desc(smem_u32(smem + AT_K + kb * 16384) + kk * 32, 16, 1024, kLayoutSW128);
                    umma_tf32(tmem, ad, bd, idesc_s, (kb > 0 || kk > 0) ? 1u : 0u);
                }
            umma_commit(&bar[4]);
        }
        __syncwarp();
        ok = ok && mbar_wait(&bar[3], 0, a.err) && mbar_wait(&bar[5], 0, a.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok && lane == 0) {
#pragma unroll
            for (int kb = 0; kb < 4; ++kb)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t ad = umma_desc(smem_u32(smem + AT_P + kb * 16384) + kk * 32, 16, 1024, kLayoutSW128);
                    const uint64_t bd =
                        umma_desc(smem_u32(smem + AT_V + kb * 8192) + kk * 1024, 4096, 512, kLayoutSW128Base32B);
                    umma_tf32(tmem + AT_KEYS, ad, bd, idesc_o, (kb > 0 || kk > 0) ? 1u : 0u);
                }
            umma_commit(&bar[6]);
        }
        __syncwarp();
    } else {
        // ---------------- softmax warps: a row per thread ----------------
        const int t = threadIdx.x - 64;
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        const int row = q * 32 + lane;          // row of the tile = TMEM lane
        bool ok = mbar_wait(&bar[0], 0, a.err);
        if (ok) round_tf32_inplace(smem + AT_Q, 4 * 16384, t, 160);
        fence_proxy_async_smem();
        mbar_arrive(&bar[2]);
        ok = ok && mbar_wait(&bar[4], 0, a.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float s[AT_KEYS];
#pragma unroll
        for (int ch = 0; ch < AT_KEYS / 16; ++ch) tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + ch * 16, s + 16 * ch);
#pragma unroll
        for (int i = 0; i < AT_KEYS; ++i) s[i] *= a.scale;
        // the Scores tile through the TMA: this warp's 32 rows staged, 32
        // columns per swizzled 4 KB tile, in the warp's own 16 KB of the P
        // space (over Q and K, free once S is done); P goes there after the
        // stores have read it
        uint8_t* stage = smem + AT_P + q * 16384;
#pragma unroll
        for (int ch = 0; ch < AT_KEYS / 32; ++ch) {
            uint8_t* sc = stage + ch * 4096;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                *reinterpret_cast<float4*>(sc + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                    make_float4(s[32 * ch + 4 * j], s[32 * ch + 4 * j + 1], s[32 * ch + 4 * j + 2], s[32 * ch + 4 * j + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && ok) {
#pragma unroll
            for (int ch = 0; ch < AT_KEYS / 32; ++ch) tma_store_2d(&tmS, stage + ch * 4096, n0 + ch * 32, m0 + q * 32);
            bulk_commit();
        }
        // the tile's row statistics and P = exp(S - m), TF32, into the
        // K-major swizzled operand layout: 32-key block kb, 16-byte chunk j
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < AT_KEYS; ++i) mx = fmaxf(mx, s[i]);
        if (mx == -INFINITY || mx != mx) mx = 0.f;
        float l = 0.f;
#pragma unroll
        for (int i = 0; i < AT_KEYS; ++i) {
            s[i] = __expf(s[i] - mx);
            l += s[i];
        }
        // every warp's Scores stores have read their staging tiles (a warp's
        // staging space is one whole 32-key block of P, which holds P rows of
        // all four warps)
        if (lane == 0) bulk_wait_read_0();
        asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
        for (int kb = 0; kb < AT_KEYS / 32; ++kb)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float* v = s + 32 * kb + 4 * j;
                *reinterpret_cast<float4*>(smem + AT_P + kb * 16384 + row * 128 + ((j ^ (row & 7)) << 4)) =
                    make_float4(tf32_rna(v[0]), tf32_rna(v[1]), tf32_rna(v[2]), tf32_rna(v[3]));
            }
        fence_proxy_async_smem();
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&bar[5]);
        const int64_t prow = (int64_t)blockIdx.y * a.n_q + m0 + row;
        a.mpart[prow] = mx;
        a.lpart[prow] = l;
        ok = ok && mbar_wait(&bar[6], 0, a.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (lane == 0) bulk_wait_all();   // the Scores stores are done before the CTA exits
        __syncwarp();
        if (ok) {
            float* op = a.opart + prow * AT_D;
#pragma unroll
            for (int ch = 0; ch < AT_D / 16; ++ch) {
                float o[16];
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + AT_KEYS + ch * 16, o);
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                    *reinterpret_cast<float4*>(op + ch * 16 + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AT_TMEM_COLS));
    }
}

// A warp per query row: the key tiles' statistics combined (m*, l*), the row
// of O (lane l: columns 2l, 2l + 1), then the row of A = exp(S - m*) / l*
// from the scores the tile kernel stored (n_k a multiple of 4; 128-bit loads
// and stores).  The row's first 1024 scores and first 16 tiles' partials are
// loaded with its statistics, in one memory round trip; the rest 8 loads per
// lane at a time.
__global__ void __launch_bounds__(256)
    k_attn_rows(const float* __restrict__ opart, const float* __restrict__ mpart, const float* __restrict__ lpart,
                int n_kt, int64_t n_q, float* __restrict__ O, int64_t lo, const float* __restrict__ S,
                float* __restrict__ A, int64_t n_k) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t q4 = n_k / 4;
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n_q; r += warps) {
        const float4* Sr = reinterpret_cast<const float4*>(S + r * n_k);
        float4* Ar = reinterpret_cast<float4*>(A + r * n_k);
        // the row's first 1024 scores and its first 16 tiles' O and maxima are
        // loaded together with the statistics below: one memory round trip
        float4 sv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int64_t j = lane + 32 * u;
            sv[u] = j < q4 ? Sr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float w0[16];
        float2 v0[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            w0[u] = u < n_kt ? mpart[u * n_q + r] : -INFINITY;
            v0[u] = u < n_kt ? *reinterpret_cast<const float2*>(opart + (u * n_q + r) * AT_D + 2 * lane)
                             : make_float2(0.f, 0.f);
        }
        float m = -INFINITY, lt = 0.f;
        for (int t = lane; t < n_kt; t += 32) {
            const float mt = mpart[t * n_q + r];
            const float l1 = lpart[t * n_q + r];
            // running (m, l) of this lane's tiles
            const float mn = fmaxf(m, mt);
            lt = lt * __expf(m - mn) + l1 * __expf(mt - mn);
            m = mn;
        }
        float mstar = m;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mstar = fmaxf(mstar, __shfl_xor_sync(0xffffffffu, mstar, o));
        float l = m == -INFINITY ? 0.f : lt * __expf(m - mstar);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        const float inv = 1.0f / l;
        float o0 = 0.f, o1 = 0.f;
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            const float e = __expf(w0[u] - mstar);
            o0 = fmaf(e, v0[u].x, o0);
            o1 = fmaf(e, v0[u].y, o1);
        }
        // tiles past the first 16, 8 tiles' loads in flight at a time
        for (int t0 = 16; t0 < n_kt; t0 += 8) {
            float w[8];
            float2 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int t = t0 + u;
                w[u] = t < n_kt ? mpart[t * n_q + r] : -INFINITY;
                v[u] = t < n_kt ? *reinterpret_cast<const float2*>(opart + (t * n_q + r) * AT_D + 2 * lane)
                                : make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float e = __expf(w[u] - mstar);
                o0 = fmaf(e, v[u].x, o0);
                o1 = fmaf(e, v[u].y, o1);
            }
        }
        *reinterpret_cast<float2*>(O + r * lo + 2 * lane) = make_float2(o0 * inv, o1 * inv);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int64_t j = lane + 32 * u;
            if (j < q4)
                Ar[j] = make_float4(__expf(sv[u].x - mstar) * inv, __expf(sv[u].y - mstar) * inv,
                                    __expf(sv[u].z - mstar) * inv, __expf(sv[u].w - mstar) * inv);
        }
        for (int64_t j0 = lane + 32 * 8; j0 < q4; j0 += 32 * 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int64_t j = j0 + 32 * u;
                v[u] = j < q4 ? Sr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int64_t j = j0 + 32 * u;
                if (j < q4)
                    Ar[j] = make_float4(__expf(v[u].x - mstar) * inv, __expf(v[u].y - mstar) * inv,
                                        __expf(v[u].z - mstar) * inv, __expf(v[u].w - mstar) * inv);
            }
        }
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D fp32 map: inner (contiguous) extent x, outer extent y, row stride in
// elements; box 32 x box_y.  K-major tiles use the 128-byte swizzle;
// MN-major tiles (mn = true) the 128-byte swizzle with 32-byte atoms that
// the MN-major tf32 UMMA layout expects.
bool make_map(CUtensorMap* map, const float* base, int64_t x, int64_t y, int64_t row_stride, int box_y, bool mn) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)x, (cuuint64_t)y};
    cuuint64_t strides[1] = {(cuuint64_t)(row_stride * 4)};
    cuuint32_t box[2] = {32, (cuuint32_t)box_y};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     mn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Store map of a row-major fp32 matrix (rows of `row_stride` floats): 32 x 32
// boxes, 128-byte swizzle (the epilogue's shared tile layout).
bool make_store_map(CUtensorMap* map, const float* base, int64_t cols, int64_t rows, int64_t row_stride) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(row_stride * 4)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, bool AM, bool BM, bool P3>
tl_status launch_tc_inst(tl_ctx* c, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                         const CUtensorMap& md, const CUtensorMap& ma1, const CUtensorMap& mb1, int tma_store,
                         const TcEpi& e, int64_t M, int64_t N, int num_kb, int kb_per_split, int splits) {
    using Cfg = TcCfg<BN, P3 ? 2 : 1>;
    static_assert(Cfg::STAGES >= 2, "two stages in flight");
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(k_gemm_tc<BN, AM, BM, P3>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) !=
            cudaSuccess)
            return fail(c, TL_ERR_CUDA, "cannot reserve %d bytes of shared memory", Cfg::SMEM);
        attr_set = true;
    }
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + TC_BM - 1) / TC_BM), (unsigned)splits);
    static_assert(Cfg::STAGES * Cfg::STAGE >= 4 * 16384, "epilogue tiles fit in the stage memory");
    k_gemm_tc<BN, AM, BM, P3><<<grid, TC_THREADS, Cfg::SMEM, c->stream>>>(ma, mb, mc, md, ma1, mb1, e, num_kb,
                                                                          kb_per_split, tma_store);
    return TL_OK;
}

template <int BN>
tl_status launch_tc_bn(tl_ctx* c, bool am, bool bm, bool p3, const CUtensorMap& ma, const CUtensorMap& mb,
                       const CUtensorMap& mc, const CUtensorMap& md, const CUtensorMap& ma1, const CUtensorMap& mb1,
                       int ts, const TcEpi& e, int64_t M, int64_t N, int num_kb, int kb_per_split, int splits) {
#define TL_TC_INST(AMV, BMV, P3V) \
    launch_tc_inst<BN, AMV, BMV, P3V>(c, ma, mb, mc, md, ma1, mb1, ts, e, M, N, num_kb, kb_per_split, splits)
    if (p3) {
        if (!am && !bm) return TL_TC_INST(false, false, true);
        if (am && !bm) return TL_TC_INST(true, false, true);
        if (!am && bm) return TL_TC_INST(false, true, true);
        return TL_TC_INST(true, true, true);
    }
    if (!am && !bm) return TL_TC_INST(false, false, false);
    if (am && !bm) return TL_TC_INST(true, false, false);
    if (!am && bm) return TL_TC_INST(false, true, false);
    return TL_TC_INST(true, true, false);
#undef TL_TC_INST
}

// Tile width of the tensor-core GEMM for N output columns.
int tc_tile_n(int64_t N) { return N >= 256 && (N % 256 == 0 || N >= 1024) ? 256 : (N >= 128 ? 128 : 64); }

bool env_flag(const char* name) {
    const char* v = getenv(name);
    return v && v[0] && v[0] != '0';
}

}  // namespace

// Map for row gathers of a row-major fp32 matrix (`rows` rows of `cols`
// floats, rows `row_stride` floats apart): a box of one row of `cols`
// floats, no swizzle, for cp.async.bulk.tensor ... tile::gather4 (four rows
// of given indices per copy).
bool make_gather_map(CUtensorMap* map, const float* base, int64_t cols, int64_t rows, int64_t row_stride) {
    EncodeTiledFn enc = get_encode();
    if (!enc || cols > 256 || (cols * 4) % 16 || (row_stride * 4) % 16 || ((uintptr_t)base & 15)) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(row_stride * 4)};
    cuuint32_t box[2] = {(cuuint32_t)cols, 1};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int64_t gemm_fan_tiles(int64_t M, int64_t N) {
    const int bn = tc_tile_n(N);
    return ((M + TC_BM - 1) / TC_BM) * ((N + bn - 1) / bn);
}

bool tcgen05_available(tl_ctx* c) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, c->device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, c->device);
    return major == 10 && minor == 0 && get_encode() != nullptr && !env_flag("TL_GEMM_SIMT");
}

static tl_status launch_simt(tl_ctx* c, const GemmPlan& p);

// Skinny shapes without a per-term nonlinearity; false if the shape is not one.
static bool launch_skinny(tl_ctx* c, const GemmPlan& p, tl_status* st) {
    if (p.relu_term || p.epi_relu || p.K <= 0) return false;
    if (p.N <= 16 && p.K >= 128 && (p.sam == 1 || p.sak == 1)) {
        const bool mcont = p.sam == 1 && p.sak != 1;
        const int64_t rows = mcont ? SKM_ROWS : SKC_ROWS, kw = mcont ? SKM_K : SKC_K;
        dim3 g((unsigned)((p.M + rows - 1) / rows), (unsigned)((p.K + kw - 1) / kw));
        if (g.x > 2147483647u || g.y > 65535u) return false;
        if (g.y > 1 && !p.beta) {
            // zero C (a memset when dense, else a K = 0 pass), then add the partial sums
            if (p.scn == 1 && p.scm == p.N) {
                const cudaError_t e = cudaMemsetAsync(p.C, 0, (size_t)p.M * p.N * sizeof(float), c->stream);
                if (e != cudaSuccess) {
                    *st = cuda_fail(c, e, "cudaMemsetAsync");
                    return true;
                }
            } else {
                GemmPlan z = p;
                z.K = 0;
                *st = launch_simt(c, z);
                if (*st != TL_OK) return true;
            }
        }
        const int vec = !mcont && (p.sam & 3) == 0 && ((uintptr_t)p.A & 15) == 0 ? 1 : 0;
        LaunchScope L(c, "gemm_skinny_fp32", (double)(p.M * p.K + p.K * p.N + p.M * p.N * (1 + p.beta)) * 4.0,
                      2.0 * p.M * p.N * p.K);
        if (mcont) k_skinny_mcont<<<g, 256, 0, c->stream>>>(p);
        else k_skinny_kcont<<<g, 256, 0, c->stream>>>(p, vec);
        *st = L.done();
        return true;
    }
    if (p.K <= 16 && p.N >= 64 && p.M >= 64) {
        const int vec = p.scn == 1 && (p.scm & 3) == 0 && ((uintptr_t)p.C & 15) == 0 ? 1 : 0;
        const int64_t nblocks = (p.N + TK_COLS - 1) / TK_COLS;
        // about four blocks per SM over the rows, at most TK_ROWS rows a block
        int64_t rows = std::max<int64_t>(1, (p.M * nblocks + (int64_t)c->sm_count * 4 - 1) / ((int64_t)c->sm_count * 4));
        if (rows > TK_ROWS) rows = TK_ROWS;
        const int64_t mblocks = (p.M + rows - 1) / rows;
        LaunchScope L(c, "gemm_thin_k_fp32", (double)(p.M * p.K + p.K * p.N + p.M * p.N * (1 + p.beta)) * 4.0,
                      2.0 * p.M * p.N * p.K);
        k_gemm_thin_k<<<dim3((unsigned)nblocks, (unsigned)mblocks), TK_THREADS, 0, c->stream>>>(p, rows, vec);
        *st = L.done();
        return true;
    }
    return false;
}

static tl_status launch_simt(tl_ctx* c, const GemmPlan& p) {
    if (p.K > 0 && !env_flag("TL_GEMM_NO_SKINNY")) {
        tl_status st = TL_OK;
        if (launch_skinny(c, p, &st)) return st;
    }
    const float sgn = p.scale < 0.f ? -1.f : 1.f;
    const float mag = fabsf(p.scale);
    const int bn = p.N <= 16 ? 16 : 64;
    const int64_t tiles = ((p.N + bn - 1) / bn) * ((p.M + SB_M - 1) / SB_M);
    // split K when the output has too few tiles to fill the GPU
    int64_t splits = 1;
    if (!p.epi_relu && p.K >= 64) {
        // about two blocks per SM, each at least two 16-deep k-steps
        const int64_t want = (int64_t)c->sm_count * 2;
        if (tiles < want) splits = (want + tiles - 1) / tiles;
        const int64_t max_splits = (p.K + 31) / 32;
        if (splits > max_splits) splits = max_splits;
    }
    int64_t chunk = (p.K + splits - 1) / splits;
    chunk = (chunk + SB_K - 1) / SB_K * SB_K;
    splits = chunk > 0 ? (p.K + chunk - 1) / chunk : 1;
    if (splits < 1) splits = 1;
    LaunchScope L(c, "gemm_simt_fp32", (double)(p.M * p.K + p.K * p.N + p.M * p.N * (1 + p.beta)) * 4.0,
                  2.0 * p.M * p.N * p.K);
    dim3 grid((unsigned)((p.N + bn - 1) / bn), (unsigned)((p.M + SB_M - 1) / SB_M), (unsigned)splits);
    if (splits > 1 && !p.beta) {
        // zero C first (a memset when dense, else a K = 0 pass), then add the partial tiles
        if (p.scn == 1 && p.scm == p.N) {
            TL_CK(c, cudaMemsetAsync(p.C, 0, (size_t)p.M * p.N * sizeof(float), c->stream));
        } else {
            GemmPlan z = p;
            z.K = 0;
            dim3 g1(grid.x, grid.y, 1);
            if (bn == 16) k_gemm_simt<16><<<g1, 256, 0, c->stream>>>(z, sgn, mag, 0);
            else k_gemm_simt<64><<<g1, 256, 0, c->stream>>>(z, sgn, mag, 0);
        }
    }
    if (bn == 16) k_gemm_simt<16><<<grid, 256, 0, c->stream>>>(p, sgn, mag, splits > 1 ? chunk : p.K);
    else k_gemm_simt<64><<<grid, 256, 0, c->stream>>>(p, sgn, mag, splits > 1 ? chunk : p.K);
    return L.done();
}

// The attention block S = scale Q K^T, A = softmax over keys (the rows of S),
// O = A V on row-major fp32 tensors with d = 64 and query / key counts that are
// multiples of 128 (the caller checks the shapes); see k_attn_tile.
tl_status launch_attention(tl_ctx* c, const AttnPlan& p) {
    CUtensorMap mq, mk, mv, ms;
    memset(&mq, 0, sizeof mq); memset(&mk, 0, sizeof mk); memset(&mv, 0, sizeof mv); memset(&ms, 0, sizeof ms);
    bool ok = make_map(&mq, p.Q, AT_D, p.n_q, AT_D, AT_ROWS, false) && make_map(&mk, p.K, AT_D, p.n_k, AT_D, AT_KEYS, false) &&
              make_map(&mv, p.V, AT_D, p.n_k, AT_D, 32, true) && make_store_map(&ms, p.S, p.n_k, p.n_q, p.n_k);
    if (!ok) return fail(c, TL_ERR_CUDA, "attention: tensor maps");
    const int n_kt = (int)(p.n_k / AT_KEYS);
    const size_t part = (size_t)n_kt * p.n_q;
    void* ws = nullptr;
    TL_TRY(workspace(c, part * (AT_D + 2) * sizeof(float), &ws, WS_GEMM));
    AttnArgs a;
    a.S = p.S;
    a.ls = p.n_k;
    a.n_q = p.n_q;
    a.scale = p.scale;
    a.opart = static_cast<float*>(ws);
    a.mpart = a.opart + part * AT_D;
    a.lpart = a.mpart + part;
    a.err = c->d_flags + 8;
    c->flags_armed = true;
    static int attr_dev[64] = {0};
    if (c->device >= 0 && c->device < 64 && !attr_dev[c->device]) {
        TL_CK(c, cudaFuncSetAttribute(k_attn_tile, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM));
        attr_dev[c->device] = 1;
    }
    {
        LaunchScope L(c, "attention_tile", (double)(3 * p.n_k * AT_D + p.n_q * AT_D) * 4.0 + (double)p.n_q * p.n_k * 4.0,
                      4.0 * (double)p.n_q * p.n_k * AT_D);
        k_attn_tile<<<dim3((unsigned)(p.n_q / AT_ROWS), (unsigned)n_kt), AT_THREADS, AT_SMEM, c->stream>>>(mq, mk, mv, ms, a);
        TL_TRY(L.done());
    }
    {
        LaunchScope L(c, "attention_combine",
                      (double)part * (AT_D + 2) * 4.0 + (double)p.n_q * AT_D * 4.0 + (double)p.n_q * p.n_k * 8.0);
        const int64_t blocks = std::min<int64_t>((p.n_q + 7) / 8, (int64_t)c->sm_count * 8);
        k_attn_rows<<<(unsigned)blocks, 256, 0, c->stream>>>(a.opart, a.mpart, a.lpart, n_kt, p.n_q, p.O, AT_D, p.S,
                                                             p.A, p.n_k);
        TL_TRY(L.done());
    }
    return TL_OK;
}

tl_status launch_gemm(tl_ctx* c, const GemmPlan& p) {
    if (p.M <= 0 || p.N <= 0) return TL_OK;
    if (p.K <= 0) {
        if (!p.beta) {
            // sum over an empty range: zeros
            GemmPlan q = p;
            q.K = 0;
            return launch_simt(c, q);
        }
        return TL_OK;
    }
    const double macs = (double)p.M * p.N * p.K;
    bool tc = c->opts.precision == TL_PREC_TF32 && tcgen05_available(c) && p.M >= 128 && p.N >= 64 && p.K >= 32 &&
              macs >= (double)(1 << 25);
    if (p.fan_n && (!tc || p.beta || p.epi_relu || p.N % 4 || p.scn != 1))
        return fail(c, TL_ERR_UNSUPPORTED, "fanned-out GEMM needs the tensor-core path (M %lld, N %lld)",
                    (long long)p.M, (long long)p.N);
    if (!tc) return launch_simt(c, p);

    // Every tensor-core operand is copied once into the workspace, rounded to
    // TF32 (nearest; the hardware would truncate), with the K segments of the
    // chosen precision: plain, relu sign split (2K), or 3xTF32 (3K, fp32-class
    // accuracy for tensors whose sign a later step / relu gradient tests).
    // A copy keeps its source's orientation when that is K- or MN-contiguous
    // (a streaming copy; MN-major tiles feed the tensor cores directly) and
    // becomes K-major through shared-memory tiles otherwise.
    const bool use_mn = !env_flag("TL_GEMM_NO_MN");
    const bool split = p.relu_term != 0;
    const bool precise = !split && p.precise != 0;
    const float sgn = p.scale < 0.f ? -1.f : 1.f;
    // relu(s a b) = a+ (s b)+ + a- (s b)-; with a >= 0 it is a (s b)+, and
    // with b >= 0 it is (s a)+ b: one K segment instead of two
    const bool one_a = split && p.a_nonneg, one_b = split && !one_a && p.b_nonneg;
    const bool split2 = split && !one_a && !one_b;
    // 3xTF32 as hi/lo copies of A and B, K each (the stage pairs them:
    // hi*hi + hi*lo + lo*hi), when every segment starts on a 16-byte boundary;
    // else three concatenated segments [hi, hi, lo] x [hi, lo, hi]
    const bool p3 = precise && p.K % 4 == 0 && !env_flag("TL_GEMM_NO_PAIRS");
    const int nseg = split2 ? 2 : p3 ? 2 : precise ? 3 : 1;
    const unsigned ops_a = split2 ? (OP_POS | OP_NEG << 4) : one_b ? OP_POS : p3 ? (OP_RN | OP_LO << 4)
                           : precise ? (OP_RN | OP_RN << 4 | OP_LO << 8) : OP_RN;
    const unsigned ops_b = split2 ? (OP_POS | OP_NEG << 4) : one_a ? OP_POS : p3 ? (OP_RN | OP_LO << 4)
                           : precise ? (OP_RN | OP_LO << 4 | OP_RN << 8) : OP_RN;
    const int64_t Ke = nseg * p.K;
    struct Prep { int64_t R, s_r, s_k; unsigned ops; float sgn; bool mn; int64_t ld; float* dst; const char* name; };
    Prep pa{p.M, p.sam, p.sak, ops_a, one_b ? sgn : 1.f, use_mn && p.sak != 1 && p.sam == 1, 0, nullptr, "gemm_prep_a"};
    Prep pb{p.N, p.sbn, p.sbk, ops_b, split2 || one_a ? sgn : 1.f, use_mn && p.sbk != 1 && p.sbn == 1, 0, nullptr,
            "gemm_prep_b"};
    size_t need = 0;
    for (Prep* q : {&pa, &pb}) {
        q->ld = q->mn ? ((q->R + 3) & ~int64_t(3)) : ((Ke + 3) & ~int64_t(3));   // 16-byte row strides
        need += (((size_t)(q->mn ? Ke : q->R) * q->ld * 4) + 255) & ~size_t(255);
    }
    void* ws = nullptr;
    TL_TRY(workspace(c, need, &ws, WS_GEMM));
    uint8_t* wp = (uint8_t*)ws;
    // the row-wise copies of both operands go in one launch; a source with
    // neither K nor MN contiguous is copied through shared-memory tiles
    PrepRows rw[2] = {};
    int n_rows = 0;
    double rows_bytes = 0;
    for (Prep* q : {&pa, &pb}) {
        q->dst = (float*)wp;
        wp += (((size_t)(q->mn ? Ke : q->R) * q->ld * 4) + 255) & ~size_t(255);
        const float* src = q == &pa ? p.A : p.B;
        if (q->mn || q->s_k == 1) {
            // rows of the contiguous dim: R rows of K (K-major) or K rows of R (MN-major)
            const int64_t rows = q->mn ? p.K : q->R, len = q->mn ? q->R : p.K;
            const int64_t src_rs = q->mn ? q->s_k : q->s_r;
            const int64_t dst_ss = q->mn ? p.K * q->ld : p.K;
            const bool vec = (len & 3) == 0 && (src_rs & 3) == 0 && (q->ld & 3) == 0 && (dst_ss & 3) == 0 &&
                             ((uintptr_t)src & 15) == 0 && ((uintptr_t)q->dst & 15) == 0;
            const int64_t per_row = vec ? (len + 3) / 4 : len;
            int tl = 0;   // threads per row: the power of two that covers the row, at most 256
            while ((1 << tl) < per_row && tl < 8) ++tl;
            const int64_t rpb = 256 >> tl;
            // the vector path takes four rows per thread when one row each
            // would give at least four blocks per SM (a small operand keeps
            // one row per thread, so enough blocks stay in flight)
            const int64_t gx = std::min<int64_t>((per_row + 255) / 256, 64);
            int64_t row_groups = (rows + rpb - 1) / rpb;
            if (vec && gx * row_groups >= 4 * (int64_t)c->sm_count) row_groups = (rows + 4 * rpb - 1) / (4 * rpb);
            PrepRows& r = rw[n_rows++];
            r.S = src; r.src_rs = src_rs; r.rows = rows; r.len = len; r.nseg = nseg; r.ops = q->ops; r.sgn = q->sgn;
            r.D = q->dst; r.dst_rs = q->ld; r.dst_ss = dst_ss; r.vec = vec ? 1 : 0; r.tpr_log2 = tl;
            r.gx = (unsigned)gx;
            r.gy = (unsigned)std::min<int64_t>(row_groups, 65535);
            rows_bytes += (double)q->R * p.K * 4.0 * (1 + nseg);
        } else {
            LaunchScope L(c, q->name, (double)q->R * p.K * 4.0 * (1 + nseg));
            dim3 g((unsigned)((q->R + 31) / 32), (unsigned)((p.K + 31) / 32));
            k_prep_transpose<<<g, dim3(32, 8), 0, c->stream>>>(src, q->s_r, q->s_k, q->R, p.K, nseg, q->ops, q->sgn,
                                                              q->dst, q->ld);
            TL_TRY(L.done());
        }
    }
    if (n_rows) {
        LaunchScope L(c, "gemm_prep", rows_bytes);
        dim3 g(std::max(rw[0].gx, rw[1].gx), std::max(rw[0].gy, rw[1].gy), (unsigned)n_rows);
        k_prep_rows<<<g, 256, 0, c->stream>>>(rw[0], rw[1]);
        TL_TRY(L.done());
    }
    // the maps span Ke; TMA reads zeros past it (the K tail of the last block)
    CUtensorMap ma, mb, ma1, mb1;
    memset(&ma1, 0, sizeof ma1);
    memset(&mb1, 0, sizeof mb1);
    // the tile width depends on N alone, so every rank can count another
    // rank's fanned-out tiles (gemm_fan_tiles)
    const int BN = tc_tile_n(p.N);
    // p3: one map per copy, K long, so a k-block past K reads zeros instead
    // of the next copy; the lo copy starts K (K-major: columns, MN-major: rows) on
    const int64_t kx = p3 ? p.K : Ke;
    auto seg = [&](const Prep& q, int g) { return q.dst + (int64_t)g * p.K * (q.mn ? q.ld : 1); };
    bool ok = pa.mn ? make_map(&ma, pa.dst, p.M, kx, pa.ld, 32, true) : make_map(&ma, pa.dst, kx, p.M, pa.ld, TC_BM, false);
    ok = ok && (pb.mn ? make_map(&mb, pb.dst, p.N, kx, pb.ld, 32, true) : make_map(&mb, pb.dst, kx, p.N, pb.ld, BN, false));
    if (p3) {
        ok = ok && (pa.mn ? make_map(&ma1, seg(pa, 1), p.M, p.K, pa.ld, 32, true)
                          : make_map(&ma1, seg(pa, 1), p.K, p.M, pa.ld, TC_BM, false));
        ok = ok && (pb.mn ? make_map(&mb1, seg(pb, 1), p.N, p.K, pb.ld, 32, true)
                          : make_map(&mb1, seg(pb, 1), p.K, p.N, pb.ld, BN, false));
    }
    if (!ok) return launch_simt(c, p);
    const int num_kb = (int)((kx + TC_BK - 1) / TC_BK);
    // split K only when the output tiles fill less than half of the SMs (each
    // split >= 4 k-blocks): the atomic epilogue of a split costs more than the
    // idle SMs of a grid that is already half a wave or more
    const int64_t tiles = ((p.N + BN - 1) / BN) * ((p.M + TC_BM - 1) / TC_BM);
    int splits = 1;
    if (!p.epi_relu && !p.fan_n && tiles * 2 <= c->sm_count && num_kb >= 8) {
        splits = (int)std::min<int64_t>((c->sm_count + tiles - 1) / tiles, num_kb / 4);
        if (splits < 1) splits = 1;
    }
    const int kb_per_split = (num_kb + splits - 1) / splits;
    splits = (num_kb + kb_per_split - 1) / kb_per_split;
    if (splits > 1 && !p.beta) {
        // zero C, then add the partial tiles: a memset when C is one dense
        // block, else a K = 0 pass (it honours C's strides)
        if (p.scn == 1 && p.scm == p.N) {
            TL_CK(c, cudaMemsetAsync(p.C, 0, (size_t)p.M * p.N * sizeof(float), c->stream));
        } else {
            GemmPlan z = p;
            z.K = 0;
            TL_TRY(launch_simt(c, z));
        }
    }
    TcEpi e;
    e.C = p.C; e.scm = p.scm; e.scn = p.scn;
    e.D = p.D; e.sdm = p.sdm; e.sdn = p.sdn;
    e.M = p.M; e.N = p.N;
    e.mag = split ? fabsf(p.scale) : p.scale;
    e.beta = p.beta; e.epi_relu = p.epi_relu;
    e.err = c->d_flags + 8;
    c->flags_armed = true;
    for (int j = 0; j < kMaxPeers; ++j) {
        e.fan[j] = p.fan_n ? p.fan[j] : nullptr;
        e.fan_cnt[j] = p.fan_n ? p.fan_cnt[j] : nullptr;
    }
    e.fan_n = p.fan_n;
    // epilogue through the TMA when C (and the fused relu output D) are row-major
    // with 16-byte aligned rows; a fused relu needs the plain store (it reads
    // the final sum, which an accumulating reduce does not return)
    CUtensorMap mc, md;
    memset(&mc, 0, sizeof mc);
    memset(&md, 0, sizeof md);
    auto tma_ok = [](const float* base, int64_t sm, int64_t sn) {
        return base && sn == 1 && sm > 0 && (sm * 4) % 16 == 0 && ((uintptr_t)base & 15) == 0;
    };
    int ts = !env_flag("TL_GEMM_NO_TMA_STORE") && tma_ok(p.C, p.scm, p.scn) &&
             (!p.epi_relu || (tma_ok(p.D, p.sdm, p.sdn) && !p.beta && splits == 1));
    if (ts) ts = make_store_map(&mc, p.C, p.N, p.M, p.scm) && (!p.epi_relu || make_store_map(&md, p.D, p.N, p.M, p.sdm));
    if (p.fan_n && !ts) return fail(c, TL_ERR_UNSUPPORTED, "fanned-out GEMM needs the TMA-store epilogue");
    LaunchScope L(c, "gemm_tcgen05_tf32", (double)(p.M * p.K + p.K * p.N + p.M * p.N * (1 + p.beta)) * 4.0,
                  2.0 * p.M * p.N * p.K);
    if (BN == 256) TL_TRY(launch_tc_bn<256>(c, pa.mn, pb.mn, p3, ma, mb, mc, md, ma1, mb1, ts, e, p.M, p.N, num_kb, kb_per_split, splits));
    else if (BN == 128) TL_TRY(launch_tc_bn<128>(c, pa.mn, pb.mn, p3, ma, mb, mc, md, ma1, mb1, ts, e, p.M, p.N, num_kb, kb_per_split, splits));
    else TL_TRY(launch_tc_bn<64>(c, pa.mn, pb.mn, p3, ma, mb, mc, md, ma1, mb1, ts, e, p.M, p.N, num_kb, kb_per_split, splits));
    return L.done();
}

}  // namespace tl
