/*
 * oracle.h — f64 CPU restatement of the Tensor Logic reference's hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (libtl_cuda) links,
 * loads or calls this code; it is the checker the parity tests compare the
 * CUDA backend against, and the CPU baseline the benchmark times.
 *
 * It executes the same tl_statement arrays the runtime consumes
 * (include/tl_cuda.h) with the reference's semantics: f64 tensors, calloc on
 * first sight, loop nests with free indices outer in LHS order and
 * contracted indices inner, per-term nonlinearities, the accumulation rules,
 * Gauss-Seidel fixpoint sweeps and the rule-based autodiff.  Each function in
 * oracle.c names the reference file:line it follows.
 *
 * Parity pinning: the reference ships no golden vectors or numeric tests for
 * this path (tests/integration_test.zig:12-23 checks exit codes only), and its
 * toolchain (zig 0.15, clang) is absent here.  The oracle is pinned by the
 * hand-derived known answers of the reference's examples/ .tl programs (see
 * tests/golden/), which is the strongest pin available.
 */
#ifndef TL_ORACLE_H
#define TL_ORACLE_H

#include <stdint.h>
#include "../include/tl_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct or_ctx or_ctx;

or_ctx* or_create(int32_t max_sweeps);
void or_destroy(or_ctx* ctx);
/* Run a whole program (LLVMCodegen.generate order).  Returns TL_OK or an error. */
int32_t or_program_run(or_ctx* ctx, const tl_statement* stmts, int32_t n);
/* Tensor access after a run; returns 0 when the tensor exists. */
int32_t or_tensor_info(or_ctx* ctx, const char* name, int32_t* rank, int64_t* dims);
const double* or_tensor_data(or_ctx* ctx, const char* name);
int32_t or_last_sweeps(or_ctx* ctx);
/* Text printed by the program's queries (llvm.zig:461-480 format). */
const char* or_query_output(or_ctx* ctx);
const char* or_last_error(or_ctx* ctx);

/* Full-size restatements with identical results, for configs whose literal
 * loop nests are infeasible on a CPU. */

/* Reach[x,z] max= step(Reach[x,y] Edge[y,z]) swept in place in the
 * reference's loop order (x, z outer; y inner), rows [row_begin, row_end) of
 * an n x n bit matrix R (n_words = ceil(n/32) words per row).  Edge is given
 * as CSC (colptr[n+1], rowidx: predecessors y of each column z).  Sweeps until
 * no change or max_sweeps; returns the sweep count of the slowest row. */
int32_t or_closure_right(int64_t n, const int64_t* colptr, const int32_t* rowidx,
                         uint32_t* R, int64_t row_begin, int64_t row_end, int32_t max_sweeps,
                         int32_t n_threads);

/* H_out[v,f] = sum_u Adj[v,u] * sum_g relu(H_in[u,g] W[g,f]) — the per-term
 * relu einsum relu(Adj[v,u] H[u,g] W[g,f]) for Adj in {0,1} (einsum.zig:20-196
 * with expr.zig:245-249), with Adj as CSR. */
void or_gnn_layer(int64_t n, int64_t g, int64_t f, const int64_t* rowptr, const int32_t* colidx,
                  const double* adj_vals, const double* H, const double* W, double* out,
                  int32_t n_threads);

/* Reference-order dense contraction C[m,n] += sum_k A[m,k] B[k,n] (f64) with
 * arbitrary strides; used for full-size parity of GEMM-shaped equations. */
void or_gemm(int64_t M, int64_t N, int64_t K, const double* A, int64_t sam, int64_t sak,
             const double* B, int64_t sbk, int64_t sbn, double* Cout, int64_t scm, int64_t scn,
             int32_t relu_per_term, double scale, int32_t n_threads);

/* One literal right-form sweep over rows [x0, x0+nrows) (timed CPU sample). */
int64_t or_closure_literal_rows(int64_t n, const uint32_t* Ebits, int64_t x0, int64_t nrows, double* Rrows);
int64_t or_closure_literal_rows_mt(int64_t n, const uint32_t* Ebits, int64_t x0, int64_t nrows, double* Rrows,
                                   int32_t n_threads);

#ifdef __cplusplus
}
#endif
#endif
