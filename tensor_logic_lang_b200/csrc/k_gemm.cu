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
    const bool a_kmajor = p.sak == 1;
    float acc[4][TN] = {};
    for (int64_t k0 = kb; k0 < ke; k0 += SB_K) {
        for (int i = threadIdx.x; i < SB_M * SB_K; i += 256) {
            // walk the contiguous dimension of A across consecutive threads
            const int mm = a_kmajor ? i / SB_K : i % SB_M;
            const int kk = a_kmajor ? i % SB_K : i / SB_M;
            const int64_t gm = m0 + mm, gk = k0 + kk;
            As[kk][mm] = (gm < p.M && gk < ke) ? p.A[gm * p.sam + gk * p.sak] : 0.f;
        }
        for (int i = threadIdx.x; i < BN * SB_K; i += 256) {
            const bool b_nmajor = p.sbn == 1;
            const int nn = b_nmajor ? i % BN : i / SB_K;
            const int kk = b_nmajor ? i / BN : i % SB_K;
            const int64_t gn = n0 + nn, gk = k0 + kk;
            Bs[kk][nn] = (gn < p.N && gk < ke) ? p.B[gk * p.sbk + gn * p.sbn] * sgn : 0.f;
        }
        __syncthreads();
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

template <int BN>
struct TcCfg {
    static constexpr int A_BYTES = TC_BM * TC_BK * 4;      // 16 KB
    static constexpr int B_BYTES = BN * TC_BK * 4;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int STAGES = (196 * 1024) / STAGE > 8 ? 8 : (196 * 1024) / STAGE;
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
    static constexpr int SMEM = STAGES * STAGE + 1024 /*align*/ + 256 /*barriers*/;
};

// A_MN / B_MN: operand stored MN-major (M or N is the contiguous dim).
template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ TcEpi epi, int num_kb) {
    using Cfg = TcCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE);
    uint64_t* empty = full + Cfg::STAGES;
    uint64_t* accum_full = empty + Cfg::STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_full + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int m0 = blockIdx.y * TC_BM, n0 = blockIdx.x * BN;

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
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % Cfg::STAGES;
                const uint32_t ph = (kb / Cfg::STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, epi.err)) break;
                uint8_t* sa = smem + s * Cfg::STAGE;
                uint8_t* sb = sa + Cfg::A_BYTES;
                mbar_expect_tx(&full[s], Cfg::STAGE);
                const int k0 = kb * TC_BK;
                if (!A_MN) {
                    tma_load_2d(sa, &tmA, &full[s], k0, m0);
                } else {
#pragma unroll
                    for (int j = 0; j < TC_BM / 32; ++j) tma_load_2d(sa + j * 4096, &tmA, &full[s], m0 + 32 * j, k0);
                }
                if (!B_MN) {
                    tma_load_2d(sb, &tmB, &full[s], k0, n0);
                } else {
#pragma unroll
                    for (int j = 0; j < BN / 32; ++j) tma_load_2d(sb + j * 4096, &tmB, &full[s], n0 + 32 * j, k0);
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
        for (int kb = 0; kb < num_kb && ok; ++kb) {
            const int s = kb % Cfg::STAGES;
            const uint32_t ph = (kb / Cfg::STAGES) & 1;
            ok = mbar_wait(&full[s], ph, epi.err);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (lane == 0) {
                const uint32_t sa = smem_u32(smem + s * Cfg::STAGE);
                const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
                for (int kk = 0; kk < TC_BK / 8; ++kk) {
                    // K-major: advance 32 bytes inside the swizzled 128-byte row; SBO = 8 rows.
                    // MN-major: 8 K rows of 128 bytes per MMA (two 4-row 32B-atom groups,
                    // SBO = 512 bytes); LBO = the next 32-wide MN chunk (one 4 KB box).
                    const uint64_t ad = A_MN ? umma_desc(sa + kk * 1024, 4096, 512, kLayoutSW128Base32B)
                                             : umma_desc(sa + kk * 32, 16, 1024, kLayoutSW128);
                    const uint64_t bd = B_MN ? umma_desc(sb + kk * 1024, 4096, 512, kLayoutSW128Base32B)
                                             : umma_desc(sb + kk * 32, 16, 1024, kLayoutSW128);
                    umma_tf32(tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
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
        if (ok) {
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
}

// Round an fp32 value to TF32 (10-bit mantissa), nearest with ties away from
// zero.  The tensor cores would otherwise drop the low 13 bits (truncation),
// which biases sums of same-sign terms such as the sign-split products.
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// relu sign split into K-major copies: Ap[m, 0:K] = max(A,0), Ap[m, K:2K] = max(-A,0);
// Bp[n, 0:K] = max(sB,0), Bp[n, K:2K] = max(-sB,0) with s the sign of the scale.
__global__ void k_split_a(const float* __restrict__ A, int64_t sam, int64_t sak, int64_t M, int64_t K, int64_t ldp,
                          float* __restrict__ Ap, int split) {
    const int64_t total = M * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / K, k = i % K;
        const float a = A[m * sam + k * sak];
        if (split) {
            Ap[m * ldp + k] = tf32_rna(fmaxf(a, 0.f));
            Ap[m * ldp + K + k] = tf32_rna(fmaxf(-a, 0.f));
        } else {
            Ap[m * ldp + k] = tf32_rna(a);
        }
    }
}

// Transposing copy through shared memory (coalesced both ways) of a [R x C]
// view with arbitrary strides into a row-major [C x ld] block, optional split.
__global__ void k_transpose_split(const float* __restrict__ S, int64_t s_r, int64_t s_c, int64_t R, int64_t Cn,
                                  float* __restrict__ D, int64_t ld, float sgn, int split) {
    __shared__ float tile[32][33];
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t r = r0 + i, cc = c0 + threadIdx.x;
        tile[i][threadIdx.x] = (r < R && cc < Cn) ? S[r * s_r + cc * s_c] * sgn : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t cc = c0 + i, r = r0 + threadIdx.x;
        if (cc < Cn && r < R) {
            const float v = tile[threadIdx.x][i];
            if (split) {
                D[cc * ld + r] = tf32_rna(fmaxf(v, 0.f));
                D[cc * ld + R + r] = tf32_rna(fmaxf(-v, 0.f));
            } else {
                D[cc * ld + r] = tf32_rna(v);
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

struct Operand {
    const float* ptr;
    int64_t rows_stride;   // stride of the non-contiguous dim (elements)
    bool mn_major;         // contiguous along M (or N)
};

template <int BN, bool AM, bool BM>
tl_status launch_tc_inst(tl_ctx* c, const CUtensorMap& ma, const CUtensorMap& mb, const TcEpi& e, int64_t M, int64_t N,
                         int num_kb) {
    using Cfg = TcCfg<BN>;
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(k_gemm_tc<BN, AM, BM>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) !=
            cudaSuccess)
            return fail(c, TL_ERR_CUDA, "cannot reserve %d bytes of shared memory", Cfg::SMEM);
        attr_set = true;
    }
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + TC_BM - 1) / TC_BM));
    k_gemm_tc<BN, AM, BM><<<grid, TC_THREADS, Cfg::SMEM, c->stream>>>(ma, mb, e, num_kb);
    return TL_OK;
}

template <int BN>
tl_status launch_tc_bn(tl_ctx* c, bool am, bool bm, const CUtensorMap& ma, const CUtensorMap& mb, const TcEpi& e,
                       int64_t M, int64_t N, int num_kb) {
    if (!am && !bm) return launch_tc_inst<BN, false, false>(c, ma, mb, e, M, N, num_kb);
    if (am && !bm) return launch_tc_inst<BN, true, false>(c, ma, mb, e, M, N, num_kb);
    if (!am && bm) return launch_tc_inst<BN, false, true>(c, ma, mb, e, M, N, num_kb);
    return launch_tc_inst<BN, true, true>(c, ma, mb, e, M, N, num_kb);
}

bool env_flag(const char* name) {
    const char* v = getenv(name);
    return v && v[0] && v[0] != '0';
}

}  // namespace

bool tcgen05_available(tl_ctx* c) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, c->device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, c->device);
    return major == 10 && minor == 0 && get_encode() != nullptr && !env_flag("TL_GEMM_SIMT");
}

static tl_status launch_simt(tl_ctx* c, const GemmPlan& p) {
    const float sgn = p.scale < 0.f ? -1.f : 1.f;
    const float mag = fabsf(p.scale);
    const int bn = p.N <= 16 ? 16 : 64;
    const int64_t tiles = ((p.N + bn - 1) / bn) * ((p.M + SB_M - 1) / SB_M);
    // split K when the output has too few tiles to fill the GPU
    int64_t splits = 1;
    if (!p.epi_relu && p.K >= 256) {
        const int64_t want = (int64_t)c->sm_count * 2;
        if (tiles < want) splits = (want + tiles - 1) / tiles;
        const int64_t max_splits = (p.K + 127) / 128;
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
        // zero C first (a K = 0 pass), then add the partial tiles
        GemmPlan z = p;
        z.K = 0;
        dim3 g1(grid.x, grid.y, 1);
        if (bn == 16) k_gemm_simt<16><<<g1, 256, 0, c->stream>>>(z, sgn, mag, 0);
        else k_gemm_simt<64><<<g1, 256, 0, c->stream>>>(z, sgn, mag, 0);
    }
    if (bn == 16) k_gemm_simt<16><<<grid, 256, 0, c->stream>>>(p, sgn, mag, splits > 1 ? chunk : p.K);
    else k_gemm_simt<64><<<grid, 256, 0, c->stream>>>(p, sgn, mag, splits > 1 ? chunk : p.K);
    return L.done();
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
    if (!tc) return launch_simt(c, p);

    // Operand layouts.  A[m,k]: K-major when sak == 1, MN-major when sam == 1.
    // B[k,n] as the UMMA "B" (N x K): K-major when sbk == 1, MN-major when sbn == 1.
    // MN-major operand descriptors are opt-in (TL_GEMM_MN=1) until validated;
    // by default MN-major operands go through a K-major transposing copy.
    const bool no_mn = !env_flag("TL_GEMM_MN");
    const bool split = p.relu_term != 0;
    const float sgn = p.scale < 0.f ? -1.f : 1.f;
    const int64_t Ke = split ? 2 * p.K : p.K;
    const int64_t Kpad = (Ke + 3) & ~int64_t(3);   // 16-byte row strides for TMA
    Operand A{p.A, 0, false}, B{p.B, 0, false};
    bool a_ok = false, b_ok = false;
    if (!split && p.sak == 1 && (p.sam % 4) == 0 && ((uintptr_t)p.A % 16) == 0) { A.rows_stride = p.sam; a_ok = true; }
    else if (!split && !no_mn && p.sam == 1 && (p.sak % 4) == 0 && ((uintptr_t)p.A % 16) == 0) {
        A.rows_stride = p.sak; A.mn_major = true; a_ok = true;
    }
    if (!split && p.sbk == 1 && (p.sbn % 4) == 0 && ((uintptr_t)p.B % 16) == 0) { B.rows_stride = p.sbn; b_ok = true; }
    else if (!split && !no_mn && p.sbn == 1 && (p.sbk % 4) == 0 && ((uintptr_t)p.B % 16) == 0) {
        B.rows_stride = p.sbk; B.mn_major = true; b_ok = true;
    }
    // prep copies (sign split, transposes) live in the workspace
    size_t need = 0;
    if (!a_ok) need += (size_t)p.M * Kpad * 4 + 256;
    if (!b_ok) need += (size_t)p.N * Kpad * 4 + 256;
    void* ws = nullptr;
    if (need) TL_TRY(workspace(c, need, &ws));
    uint8_t* wp = (uint8_t*)ws;
    if (!a_ok) {
        float* Ap = (float*)wp;
        wp += ((size_t)p.M * Kpad * 4 + 255) & ~size_t(255);
        if (Kpad != Ke) TL_CK(c, cudaMemsetAsync(Ap, 0, (size_t)p.M * Kpad * 4, c->stream));
        LaunchScope L(c, "gemm_prep_a", (double)p.M * p.K * 4.0 + (double)p.M * Ke * 4.0);
        if (p.sak == 1 || p.sam != 1) {
            int64_t blocks = (p.M * p.K + 255) / 256;
            if (blocks > (int64_t)c->sm_count * 32) blocks = (int64_t)c->sm_count * 32;
            k_split_a<<<(unsigned)blocks, 256, 0, c->stream>>>(p.A, p.sam, p.sak, p.M, p.K, Kpad, Ap, split ? 1 : 0);
        } else {
            // A is M-contiguous: view it as [K x M] and transpose
            dim3 g((unsigned)((p.M + 31) / 32), (unsigned)((p.K + 31) / 32));
            k_transpose_split<<<g, dim3(32, 8), 0, c->stream>>>(p.A, p.sak, p.sam, p.K, p.M, Ap, Kpad, 1.f, split ? 1 : 0);
        }
        TL_TRY(L.done());
        A = {Ap, Kpad, false};
    }
    if (!b_ok) {
        float* Bp = (float*)wp;
        if (Kpad != Ke) TL_CK(c, cudaMemsetAsync(Bp, 0, (size_t)p.N * Kpad * 4, c->stream));
        LaunchScope L(c, "gemm_prep_b", (double)p.N * p.K * 4.0 + (double)p.N * Ke * 4.0);
        // B[k,n] → Bp[n, k] (K-major), times the scale's sign, optional split
        dim3 g((unsigned)((p.N + 31) / 32), (unsigned)((p.K + 31) / 32));
        k_transpose_split<<<g, dim3(32, 8), 0, c->stream>>>(p.B, p.sbk, p.sbn, p.K, p.N, Bp, Kpad, split ? sgn : 1.f,
                                                            split ? 1 : 0);
        TL_TRY(L.done());
        B = {Bp, Kpad, false};
    }
    // each map spans only its own operand's K extent; TMA reads zeros past it
    const int64_t Ka = a_ok ? p.K : Kpad, Kb = b_ok ? p.K : Kpad;
    const int64_t Kx = Ka > Kb ? Ka : Kb;
    CUtensorMap ma, mb;
    bool ok = A.mn_major ? make_map(&ma, A.ptr, p.M, Ka, A.rows_stride, 32, true)
                         : make_map(&ma, A.ptr, Ka, p.M, A.rows_stride, TC_BM, false);
    const int BN = p.N >= 256 && (p.N % 256 == 0 || p.N >= 1024) ? 256 : (p.N >= 128 ? 128 : 64);
    ok = ok && (B.mn_major ? make_map(&mb, B.ptr, p.N, Kb, B.rows_stride, 32, true)
                           : make_map(&mb, B.ptr, Kb, p.N, B.rows_stride, BN, false));
    if (!ok) return launch_simt(c, p);
    TcEpi e;
    e.C = p.C; e.scm = p.scm; e.scn = p.scn;
    e.D = p.D; e.sdm = p.sdm; e.sdn = p.sdn;
    e.M = p.M; e.N = p.N;
    e.mag = split ? fabsf(p.scale) : p.scale;
    e.beta = p.beta; e.epi_relu = p.epi_relu;
    e.err = c->d_flags + 8;
    const int num_kb = (int)((Kx + TC_BK - 1) / TC_BK);
    LaunchScope L(c, "gemm_tcgen05_tf32", (double)(p.M * p.K + p.K * p.N + p.M * p.N * (1 + p.beta)) * 4.0,
                  2.0 * p.M * p.N * p.K);
    if (BN == 256) TL_TRY(launch_tc_bn<256>(c, A.mn_major, B.mn_major, ma, mb, e, p.M, p.N, num_kb));
    else if (BN == 128) TL_TRY(launch_tc_bn<128>(c, A.mn_major, B.mn_major, ma, mb, e, p.M, p.N, num_kb));
    else TL_TRY(launch_tc_bn<64>(c, A.mn_major, B.mn_major, ma, mb, e, p.M, p.N, num_kb));
    return L.done();
}

}  // namespace tl
