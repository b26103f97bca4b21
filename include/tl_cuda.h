/*
 * tl_cuda.h — C ABI of libtl_cuda, the B200 (sm_100a) execution backend for
 * Tensor Logic programs.
 *
 * The reference compiler (Zollicoff/tensor_logic_lang, Zig) lowers every
 * tensor equation to single-threaded f64 LLVM-IR loop nests.  This ABI is the
 * drop-in boundary that replaces that loop-nest emission: a CUDA target of the
 * codegen emits `declare i32 @tl_...` plus calls (the pattern sketched by the
 * unused FFI declarations in src/codegen/gpu.zig:293-310), and links against
 * libtl_cuda.so.  Every entry point below names the reference function it
 * replaces.
 *
 * Plain C: no C++ or torch types, fixed-size structs (no pointer ownership
 * questions across the FFI), every call returns a tl_status and never aborts.
 *
 * Data model (mirrors src/codegen/tensor.zig:14-81): a tensor is a row-major
 * array named by the program; it is created zero-filled (calloc semantics) on
 * first sight and keeps its dims for the life of the context.  On the host the
 * element type is f64 (the reference type); on the device the runtime keeps
 * fp32 dense storage, a bit-packed storage for 0/1-valued rank-2 tensors, and
 * CSR for `sparse` declarations, converting between them on demand.
 */
#ifndef TL_CUDA_H
#define TL_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Limits of the fixed-size descriptors                                      */
/* ------------------------------------------------------------------------ */
#define TL_MAX_RANK 8      /* indices per tensor reference                   */
#define TL_MAX_REFS 8      /* tensor references in one right-hand side       */
#define TL_MAX_CODE 48     /* postfix instructions in one right-hand side    */
#define TL_MAX_PARAMS 8    /* parameters of one `backward ... wrt ...`       */
#define TL_NAME_LEN 32     /* tensor / index names incl. the NUL             */
#define TL_PATH_LEN 256

/* ------------------------------------------------------------------------ */
/* Status codes.  The reference has no run-time errors (its codegen reports  */
/* through Zig error unions, src/main.zig:140-246); the backend reports every */
/* failure through these codes and tl_last_error().                          */
/* ------------------------------------------------------------------------ */
typedef int32_t tl_status;
#define TL_OK                 0
#define TL_ERR_INVALID        1  /* malformed descriptor or argument          */
#define TL_ERR_OOM            2  /* device or host allocation failed          */
#define TL_ERR_CUDA           3  /* a CUDA call or kernel failed              */
#define TL_ERR_COMM           4  /* an NCCL call failed or timed out          */
#define TL_ERR_NOT_CONVERGED  5  /* reserved: a fixpoint that reaches its     */
                                 /* sweep cap returns TL_OK with the cap as   */
                                 /* its sweep count, as the reference stops   */
                                 /* silently (fixpoint.zig:67-72)             */
#define TL_ERR_UNSUPPORTED    6  /* form the backend does not lower           */
#define TL_ERR_NOT_FOUND      7  /* unknown tensor name                       */
#define TL_ERR_IO             8  /* save/load file error                      */
#define TL_ERR_TOO_LARGE      9  /* size above a fixed capacity (see below)   */

/* ------------------------------------------------------------------------ */
/* Index forms: src/frontend/ast.zig:17-59 (Index union)                     */
/* ------------------------------------------------------------------------ */
#define TL_IX_NAME       0  /* i            name = "i"                        */
#define TL_IX_CONST      1  /* 3            value = 3                         */
#define TL_IX_ADD        2  /* i+1          name = "i", value = 1             */
#define TL_IX_SUB        3  /* i-1          name = "i", value = 1             */
#define TL_IX_PRIMED     4  /* i'           name = "i" (loop var "i'")        */
#define TL_IX_DIV        5  /* i/2          name = "i", value = 2             */
#define TL_IX_NORMALIZE  6  /* i.           softmax / lnorm axis marker       */
#define TL_IX_SLICE      7  /* 4:8          value = start, value2 = end       */
#define TL_IX_VIRTUAL    8  /* *t           name = tensor t (gather)          */

typedef struct tl_index {
    int32_t kind;
    int32_t _pad;
    int64_t value;
    int64_t value2;
    char name[TL_NAME_LEN];
} tl_index;

/* A tensor reference T[i, j, ...]: src/frontend/ast.zig TensorRef. */
typedef struct tl_ref {
    char tensor[TL_NAME_LEN];
    int32_t rank;
    int32_t _pad;
    tl_index idx[TL_MAX_RANK];
} tl_ref;

/* ------------------------------------------------------------------------ */
/* Right-hand sides are postfix programs over the expression tree of         */
/* src/frontend/ast.zig Expr (evaluated per term by src/codegen/expr.zig).   */
/* ------------------------------------------------------------------------ */
#define TL_OP_REF   0   /* push refs[arg]                                      */
#define TL_OP_LIT   1   /* push value                                          */
#define TL_OP_PROD  2   /* implicit product of the top `arg` values, left to   */
                        /* right (expr.zig:207-220)                            */
#define TL_OP_ADD   3   /* binary ops pop right then left (expr.zig:160-204)  */
#define TL_OP_SUB   4
#define TL_OP_MUL   5   /* explicit `*`: same value as PROD, no gradient      */
#define TL_OP_DIV   6
#define TL_OP_POW   7
#define TL_OP_GT    8
#define TL_OP_LT    9
#define TL_OP_GE    10
#define TL_OP_LE    11
#define TL_OP_EQ    12
#define TL_OP_NE    13
#define TL_OP_AND   14  /* `&` and `|` evaluate as fadd in the reference       */
#define TL_OP_OR    15
#define TL_OP_NEG   16  /* unary -                                             */
#define TL_OP_NOT   17  /* unary !                                             */
#define TL_OP_NL    18  /* nonlinearity `arg` (TL_NL_*); value = temperature   */
                        /* when arg2 != 0 (sigmoid(x, T), expr.zig:250-273)    */

#define TL_NL_STEP     0
#define TL_NL_SOFTMAX  1
#define TL_NL_RELU     2
#define TL_NL_SIGMOID  3
#define TL_NL_TANH     4
#define TL_NL_EXP      5
#define TL_NL_LOG      6
#define TL_NL_ABS      7
#define TL_NL_SQRT     8
#define TL_NL_SIN      9
#define TL_NL_COS      10
#define TL_NL_NORM     11  /* identity in the reference (expr.zig:297)        */
#define TL_NL_LNORM    12
#define TL_NL_CONCAT   13

typedef struct tl_instr {
    int32_t op;
    int32_t arg;
    int32_t arg2;
    int32_t _pad;
    double value;
} tl_instr;

/* Accumulation operators: src/frontend/ast.zig AccumulationOp,
 * semantics src/codegen/einsum.zig:199-254. */
#define TL_ACC_ASSIGN 0   /* `=`    (with a contraction: load + add + store)  */
#define TL_ACC_ADD    1   /* `+=`                                              */
#define TL_ACC_MUL    2   /* `*=`                                              */
#define TL_ACC_MAX    3   /* `max=`                                            */
#define TL_ACC_MIN    4   /* `min=`                                            */
#define TL_ACC_AVG    5   /* `avg=` (sum, then divide by the LHS divisors)     */

/* One tensor equation LHS[...] op= RHS: src/frontend/ast.zig Equation. */
typedef struct tl_equation {
    tl_ref lhs;
    int32_t accum;
    int32_t n_refs;
    int32_t n_code;
    int32_t _pad;
    tl_ref refs[TL_MAX_REFS];
    tl_instr code[TL_MAX_CODE];
} tl_equation;

/* ------------------------------------------------------------------------ */
/* Statements of a program: src/frontend/ast.zig Statement.                  */
/* ------------------------------------------------------------------------ */
#define TL_STMT_DOMAIN    0  /* domain name: size                             */
#define TL_STMT_EQUATION  1
#define TL_STMT_SPARSE    2  /* sparse Name[i, j] (dense view sized by the    */
                             /* index names as domains, llvm.zig:482-516)     */
#define TL_STMT_BACKWARD  3  /* backward L wrt P1, P2, ...                    */
#define TL_STMT_QUERY     4  /* T?   (prints first 20 values, llvm.zig:461)   */
#define TL_STMT_SAVE      5  /* save T "path"  (raw f64, quotes stripped)     */
#define TL_STMT_LOAD      6  /* load T "path"  (raw f64); when host_data is   */
                             /* non-NULL the values come from that host array */
                             /* instead of a file (the harness input path)    */
#define TL_STMT_SPARSE_LOAD 7 /* fill a sparse tensor from host COO arrays    */

typedef struct tl_statement {
    int32_t kind;
    int32_t n_params;
    int64_t size;                       /* DOMAIN size; SPARSE_LOAD nnz        */
    char name[TL_NAME_LEN];             /* DOMAIN / BACKWARD loss / tensor     */
    char params[TL_MAX_PARAMS][TL_NAME_LEN];
    char path[TL_PATH_LEN];
    const double* host_data;            /* LOAD: dense f64 values, row-major   */
                                        /* SPARSE_LOAD: nnz values (NULL = 1)  */
    const int64_t* coo_rows;            /* SPARSE_LOAD: nnz row indices        */
    const int64_t* coo_cols;            /* SPARSE_LOAD: nnz column indices     */
    tl_ref sparse;                      /* SPARSE declaration                  */
    tl_equation eq;                     /* EQUATION                            */
} tl_statement;

/* ------------------------------------------------------------------------ */
/* Context                                                                    */
/* ------------------------------------------------------------------------ */
#define TL_PREC_TF32   0   /* fp32 storage, TF32 tensor cores (default)        */
#define TL_PREC_FP32   1   /* fp32 storage, CUDA-core fp32 contractions        */

typedef struct tl_init_opts {
    int32_t device;          /* CUDA ordinal; -1 = current device              */
    int32_t precision;       /* TL_PREC_*                                      */
    int32_t rank;            /* row-sharding: this process's rank             */
    int32_t world_size;      /* 1 = single GPU                                */
    uint8_t nccl_id[128];    /* ncclUniqueId from rank 0 when world_size > 1  */
    int32_t max_sweeps;      /* fixpoint cap; 0 = 1000 (fixpoint.zig:67-72)   */
    int32_t verbose;         /* 1 = queries print to stdout                   */
    int32_t comm_timeout_ms; /* host wait bound on a collective; 0 = 30000    */
    int32_t _pad;
} tl_init_opts;

typedef struct tl_ctx tl_ctx;

/* Fill opts with defaults (device -1, TF32, single GPU, 1000 sweeps). */
void tl_default_opts(tl_init_opts* opts);

/* Create a context on one GPU (replaces the emitted module prologue,
 * llvm.zig:131-270).  With world_size > 1 it also joins an NCCL communicator
 * of world_size ranks, one process per GPU. */
tl_status tl_init(const tl_init_opts* opts, tl_ctx** out);

/* Destroy the context and every tensor (llvm.zig:321-327 frees). */
tl_status tl_shutdown(tl_ctx* ctx);

/* Text of the last error on this context ("" when none). */
const char* tl_last_error(const tl_ctx* ctx);

/* Wait for all queued device work; returns the first deferred error. */
tl_status tl_sync(tl_ctx* ctx);

/* Generate a fresh ncclUniqueId (rank 0) into id[128]. */
tl_status tl_comm_unique_id(uint8_t id[128]);

/* ------------------------------------------------------------------------ */
/* Program execution: replaces LLVMCodegen.generate (llvm.zig:131-336).      */
/* Runs domains first, then every non-recursive statement in source order   */
/* (llvm.zig:287-301), then one fixpoint over all recursive equations        */
/* (llvm.zig:304-306, fixpoint.zig:46-98), then queries (llvm.zig:310-318). */
/* Tensors persist in the context; each run starts from calloc semantics    */
/* (every tensor defined by an equation reads as zero until written), so    */
/* repeated runs of one program give the same results.                       */
/* ------------------------------------------------------------------------ */
tl_status tl_program_run(tl_ctx* ctx, const tl_statement* stmts, int32_t n_stmts);

/* Sweeps the last fixpoint of tl_program_run took (the reference's `iter`). */
/* tl_program_run does not wait for a one-launch closure fixpoint on one     */
/* GPU; this call (like tl_sync) waits for it and reads its sweep count.     */
/* A failure of that launch (a bounded device wait that ran out) is          */
/* reported by the next tl_sync or tl_program_run.                           */
int32_t tl_last_sweeps(const tl_ctx* ctx);

/* ------------------------------------------------------------------------ */
/* Per-statement entry points (what a CUDA codegen target emits one call    */
/* per statement for).                                                       */
/* ------------------------------------------------------------------------ */

/* domain decl: llvm.zig:131-140. */
tl_status tl_domain(tl_ctx* ctx, const char* name, int64_t size);

/* Pre-compute max dims of every tensor from all equation LHS uses
 * (updateTensorMaxDims, tensor.zig:84-129; llvm.zig:142-148). */
tl_status tl_declare_dims(tl_ctx* ctx, const tl_equation* eqs, int32_t n_eqs);

/* One non-recursive equation: genEquation (llvm.zig:357-459) and its
 * softmax / lnorm dispatch (llvm.zig:361-375) → einsum.zig / softmax.zig /
 * layernorm.zig loop nests. */
tl_status tl_equation_run(tl_ctx* ctx, const tl_equation* eq);

/* The fixpoint over the recursive equations: genFixpointLoop
 * (fixpoint.zig:46-98).  *sweeps_out receives the sweep count. */
tl_status tl_fixpoint(tl_ctx* ctx, const tl_equation* eqs, int32_t n_eqs,
                      int32_t* sweeps_out);

/* backward L wrt params: genBackward (llvm.zig:635-693) with the rule set
 * of autodiff.zig:87-1082; `eqs` are all equations of the program (the
 * graph covers every equation, autodiff.zig:87-94). */
tl_status tl_backward(tl_ctx* ctx, const char* loss, const char (*params)[TL_NAME_LEN],
                      int32_t n_params, const tl_equation* eqs, int32_t n_eqs);

/* sparse decl (llvm.zig:482-516): dense view sized from the index names. */
tl_status tl_sparse_decl(tl_ctx* ctx, const tl_ref* decl);

/* ------------------------------------------------------------------------ */
/* Tensors: allocateTensor (tensor.zig:14-81) and the host side of          */
/* save / load / query (llvm.zig:461-480, 565-633).                          */
/* ------------------------------------------------------------------------ */
typedef struct tl_tensor tl_tensor;

/* Create (zero-filled) or look up a tensor; an existing tensor keeps its dims. */
tl_status tl_tensor_create(tl_ctx* ctx, const char* name, int32_t rank,
                           const int64_t* dims, tl_tensor** out);
tl_status tl_tensor_lookup(tl_ctx* ctx, const char* name, tl_tensor** out);
int32_t   tl_tensor_rank(const tl_tensor* t);
int64_t   tl_tensor_dim(const tl_tensor* t, int32_t axis);
int64_t   tl_tensor_numel(const tl_tensor* t);

/* Host f64 row-major <-> device (load / save / query data paths). */
tl_status tl_tensor_upload(tl_tensor* t, const double* host);
tl_status tl_tensor_download(tl_tensor* t, double* host);
/* fp32 variants (no f64 conversion on the host). */
tl_status tl_tensor_upload_f32(tl_tensor* t, const float* host);
tl_status tl_tensor_download_f32(tl_tensor* t, float* host);
/* Bit-packed download of a 0/1 rank-2 tensor: rows of ceil(cols/32) words,
 * bit (c & 31) of word c >> 5 is element [r, c]. */
tl_status tl_tensor_download_bits(tl_tensor* t, uint32_t* host);
/* Raw device address of the fp32 dense storage (materialised on demand). */
tl_status tl_tensor_device_ptr(tl_tensor* t, float** dptr);
/* Element store with constant indices (genScalarAssign, einsum.zig:257-278). */
tl_status tl_tensor_set(tl_tensor* t, const int64_t* idx, double v);
/* Fill a sparse tensor from COO triples (vals NULL = all 1.0). */
tl_status tl_sparse_upload(tl_tensor* t, int64_t nnz, const int64_t* rows,
                           const int64_t* cols, const double* vals);
/* Query print: "Name[total] = [v0 ... v19 ]\n" with %.4g (llvm.zig:461-480). */
tl_status tl_query_format(tl_tensor* t, char* buf, int64_t buf_len);
/* The text the last tl_program_run's queries printed, in statement order:
 * what the reference's program writes to stdout (llvm.zig:309-318).  A query
 * with a constant index prints "Name = %.6g\n", the backward-chaining value
 * (backward.zig:568-600); any other query prints as tl_query_format.
 * Copies at most buf_len - 1 bytes and a terminating 0; *needed (optional)
 * receives the full length. */
tl_status tl_program_output(tl_ctx* ctx, char* buf, int64_t buf_len, int64_t* needed);

/* ------------------------------------------------------------------------ */
/* Row sharding (closure and GNN message passing across the GPUs of a box). */
/* A sharded rank-2 tensor keeps rows r with r % world_size == rank on this  */
/* rank (cyclic rows balance the skewed reach sets of a DAG).               */
/* Column sharding (TL_SHARD_COLS, a closure relation only): this rank keeps */
/* columns [rank * c / world_size, (rank + 1) * c / world_size) of every     */
/* row of an r x c relation (c a multiple of 128 * world_size), as bit rows; */
/* the relation must start as step(Edge) right before its fixpoint, and it   */
/* is downloaded with tl_tensor_download_bits.  No extension of the          */
/* reference: its fixpoint (fixpoint.zig:46-98) has no distribution at all.  */
/* ------------------------------------------------------------------------ */
#define TL_SHARD_NONE 0
#define TL_SHARD_ROWS 1
#define TL_SHARD_COLS 2
tl_status tl_set_sharding(tl_ctx* ctx, const char* name, int32_t mode);

/* ------------------------------------------------------------------------ */
/* Timing hooks for the benchmark: device time of the last fixpoint and of   */
/* the dominant kernel launches, measured with CUDA events on the context's */
/* stream.                                                                    */
/* ------------------------------------------------------------------------ */
typedef struct tl_kernel_stats {
    char name[TL_NAME_LEN];
    int64_t launches;
    double total_ms;
    double algo_bytes;   /* algorithmic bytes moved, summed over launches */
    double algo_flops;   /* algorithmic flops, summed over launches        */
} tl_kernel_stats;

/* Enable per-launch event timing (adds an event pair per kernel launch). */
tl_status tl_profile_enable(tl_ctx* ctx, int32_t on);
/* Copy up to max entries of the accumulated per-kernel stats; returns count. */
int32_t tl_profile_read(tl_ctx* ctx, tl_kernel_stats* out, int32_t max);
tl_status tl_profile_reset(tl_ctx* ctx);
/* Count of kernel launches issued by the runtime since the context was made. */
int64_t tl_launch_count(const tl_ctx* ctx);
/* The context's CUDA stream (a cudaStream_t) for event timing by the caller. */
void* tl_stream(const tl_ctx* ctx);

/* ------------------------------------------------------------------------ */
/* Allocation-free closure fixpoint.                                         */
/*                                                                           */
/* No counterpart in the reference.  For callers that must not allocate GPU */
/* memory: a host application whose device memory belongs to its own pool   */
/* or arena (a serving process under a fixed memory budget, a framework     */
/* whose caching allocator must account for every byte on the device), so   */
/* that a cudaMalloc behind the pool's back is not allowed.  Such a caller   */
/* cannot create a tl_ctx (tl_init allocates), so this entry point takes no */
/* context: every input and output is caller-owned device memory, and the   */
/* fixpoint's scratch (one word per row plus control words) lives in a fixed */
/* array inside the library, sized for at most TL_NOALLOC_MAX_ROWS rows      */
/* (about 256 KiB, held by every GPU that loads the library until the        */
/* process exits).                                                           */
/*                                                                           */
/* Computes Reach[x,z] max= step(Reach[x,y] Edge[y,z]) to its fixpoint, the  */
/* same sweeps tl_fixpoint runs for this equation:                           */
/*   n         rows and columns of Reach and Edge (0..TL_NOALLOC_MAX_ROWS;   */
/*             a larger n returns TL_ERR_TOO_LARGE before touching the GPU)  */
/*   d_rowptr  Edge as CSR on the device: n+1 int64 row offsets             */
/*   d_colidx  column indices (int32, each in [0, n)); every stored entry    */
/*             counts as a positive value                                    */
/*   d_reach   in: the initial 0/1 relation, out: the fixpoint; n rows of    */
/*             ceil(n/32) uint32 words, bit (z & 31) of word z >> 5 = [x,z]  */
/*   max_sweeps  the sweep cap (0 = 1000, as fixpoint.zig:67-72)            */
/*   stream    the cudaStream_t to run on (NULL = the default stream); it    */
/*             must belong to the current device (else TL_ERR_INVALID),      */
/*             whose copy of the scratch array the call uses                 */
/*   sweeps_out  receives the sweep count (may be NULL)                      */
/* The call is synchronous: after every sweep it copies the changed word to  */
/* the host and waits for the stream, so it returns with d_reach final.  It   */
/* returns TL_OK when a sweep changed nothing or when the cap was reached     */
/* (then *sweeps_out == max_sweeps and the relation may not be closed, as    */
/* the reference stops silently at its cap).  The first call on a device     */
/* looks up the scratch array's device address (cudaGetSymbolAddress); make  */
/* that first call before any stream capture.  Every call shares the one     */
/* array, so calls that overlap on the GPU (other streams, other host        */
/* threads) race; serialise them.                                            */
/* ------------------------------------------------------------------------ */
#define TL_NOALLOC_MAX_ROWS 65536
tl_status tl_closure_noalloc(int64_t n, const int64_t* d_rowptr, const int32_t* d_colidx,
                             uint32_t* d_reach, int32_t max_sweeps, void* stream,
                             int32_t* sweeps_out);

#ifdef __cplusplus
}
#endif

#endif /* TL_CUDA_H */
