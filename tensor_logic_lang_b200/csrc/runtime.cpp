// libtl_cuda host runtime: context, tensor storages, program schedule and the
// lowering of each tensor equation to a kernel.
//
// Reference anchors (Zollicoff/tensor_logic_lang):
//   program schedule      src/codegen/llvm.zig:131-336 (LLVMCodegen.generate)
//   equation analysis     src/codegen/llvm.zig:357-459, src/codegen/expr.zig:303-359
//   loop-nest semantics   src/codegen/einsum.zig:20-278, src/codegen/expr.zig:14-300
//   softmax / lnorm       src/codegen/softmax.zig:19-267, src/codegen/layernorm.zig:25-348
//   fixpoint              src/codegen/fixpoint.zig:21-297
//   tensors               src/codegen/tensor.zig:14-153
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstring>

#include "tl_internal.h"

using namespace tl;

// ============================================================================
// errors and launch accounting
// ============================================================================
namespace tl {

tl_status fail(tl_ctx* c, tl_status code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (c) c->err = buf;
    return code;
}

tl_status cuda_fail(tl_ctx* c, cudaError_t e, const char* what) {
    return fail(c, e == cudaErrorMemoryAllocation ? TL_ERR_OOM : TL_ERR_CUDA, "%s: %s", what,
                cudaGetErrorString(e));
}

void launch_begin(tl_ctx* c, const char* name, double bytes, double flops, cudaEvent_t* ev) {
    c->launches++;
    ev[0] = ev[1] = nullptr;
    if (!c->prof) return;
    for (int i = 0; i < 2; ++i) {
        if (!c->event_pool.empty()) {
            ev[i] = c->event_pool.back();
            c->event_pool.pop_back();
        } else {
            cudaEventCreate(&ev[i]);
        }
    }
    cudaEventRecord(ev[0], c->stream);
    c->pending.push_back({name, ev[0], ev[1], bytes, flops});
}

tl_status launch_end(tl_ctx* c, cudaEvent_t* ev) {
    cudaError_t e = cudaGetLastError();
    if (ev[1]) cudaEventRecord(ev[1], c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "kernel launch");
    return TL_OK;
}

tl_status workspace(tl_ctx* c, size_t bytes, void** out, int slot) {
    if (slot < 0 || slot > 3) return fail(c, TL_ERR_INVALID, "bad workspace slot");
    if (bytes > c->ws_cap[slot]) {
        if (c->ws[slot]) {
            TL_CK(c, cudaStreamSynchronize(c->stream));
            cudaFree(c->ws[slot]);
            c->ws[slot] = nullptr;
            c->ws_cap[slot] = 0;
        }
        size_t cap = std::max(bytes, (size_t)16 << 20);
        TL_CK(c, cudaMalloc(&c->ws[slot], cap));
        c->ws_cap[slot] = cap;
    }
    *out = c->ws[slot];
    return TL_OK;
}

int64_t domain_size(tl_ctx* c, const char* name) {
    auto it = c->domains.find(name);
    return it == c->domains.end() ? 10 : it->second;
}

Tensor* find(tl_ctx* c, const std::string& name) {
    auto it = c->tensors.find(name);
    return it == c->tensors.end() ? nullptr : it->second.get();
}

Tensor* find_defined(tl_ctx* c, const std::string& name) {
    Tensor* t = find(c, name);
    return (t && t->defined) ? t : nullptr;
}

// ============================================================================
// tensor storages
// ============================================================================
uint64_t next_csr_stamp() {
    static std::atomic<uint64_t> stamp{0};
    return ++stamp;
}

static void free_storage(Tensor* t) {
    cudaFree(t->dense); t->dense = nullptr; t->dense_elems = 0;
    cudaFree(t->bits); t->bits = nullptr; t->bits_words = t->bits_rows = 0;
    cudaFree(t->rowptr); cudaFree(t->colidx); cudaFree(t->vals);
    t->rowptr = nullptr; t->colidx = nullptr; t->vals = nullptr; t->csr_cap = 0;
    cudaFree(t->colptr); cudaFree(t->rowidx);
    t->colptr = nullptr; t->rowidx = nullptr; t->csc_cap = 0;
    cudaFree(t->succ); t->succ = nullptr; t->succ_cap = 0; t->succ_stamp = 0;
    t->lazy_src = nullptr;
    t->dense_valid = t->bits_valid = t->csr_valid = t->csc_valid = false;
}

// (Re)create a tensor with calloc semantics (tensor.zig:14-81).  Storage is
// reused when the dims are unchanged; the values become logical zeros.
tl_status new_tensor(tl_ctx* c, const std::string& name, int rank, const int64_t* dims, Tensor** out) {
    if (rank > TL_MAX_RANK) return fail(c, TL_ERR_INVALID, "%s: rank %d > %d", name.c_str(), rank, TL_MAX_RANK);
    int64_t d[TL_MAX_RANK];
    if (rank == 0) { rank = 1; d[0] = 1; }
    else for (int k = 0; k < rank; ++k) d[k] = dims[k];
    for (int k = 0; k < rank; ++k)
        if (d[k] < 0) return fail(c, TL_ERR_INVALID, "%s: negative dim", name.c_str());
    auto& slot = c->tensors[name];
    if (!slot) { slot.reset(new tl_tensor()); slot->name = name; }
    Tensor* t = slot.get();
    t->owner = c;
    bool same = t->rank == rank;
    for (int k = 0; same && k < rank; ++k) same = t->dims[k] == d[k];
    if (!same) free_storage(t);
    t->rank = rank;
    int64_t s = 1;
    for (int k = rank - 1; k >= 0; --k) { t->dims[k] = d[k]; t->strides[k] = s; s *= d[k]; }
    t->total = s;
    t->defined = true;
    t->zero = true;
    t->boolean = true;  // zeros are 0/1 valued
    t->is_sparse = false;
    t->dense_valid = t->bits_valid = t->csr_valid = t->csc_valid = false;
    *out = t;
    return TL_OK;
}

int64_t index_extent(tl_ctx* c, const tl_index* ix) {
    switch (ix->kind) {
    case TL_IX_NAME: case TL_IX_NORMALIZE: case TL_IX_PRIMED: case TL_IX_ADD: case TL_IX_SUB:
        return domain_size(c, ix->name);
    case TL_IX_CONST: return ix->value + 1;
    case TL_IX_DIV: { int64_t b = domain_size(c, ix->name); return ix->value > 0 ? (b + ix->value - 1) / ix->value : b; }
    case TL_IX_SLICE: return ix->value2 > ix->value ? ix->value2 - ix->value : 1;
    default: return 10;
    }
}

// allocateTensor (tensor.zig:14-81): the precomputed max dims when known.
tl_status allocate_tensor(tl_ctx* c, const char* name, const tl_index* idx, int n, Tensor** out) {
    auto it = c->maxdims.find(name);
    if (it != c->maxdims.end())
        return new_tensor(c, name, (int)it->second.size(), it->second.data(), out);
    int64_t dims[TL_MAX_RANK];
    for (int k = 0; k < n; ++k) dims[k] = idx[k].kind == TL_IX_NORMALIZE ? 10 : index_extent(c, &idx[k]);
    return new_tensor(c, name, n, dims, out);
}

static int64_t dense_rows(tl_ctx* c, Tensor* t) {
    return t->local_rows(c->rank, c->world);
}

static int64_t dense_local_elems(tl_ctx* c, Tensor* t) {
    if (t->shard == TL_SHARD_ROWS && c->world > 1 && t->rank >= 1)
        return dense_rows(c, t) * (t->total / std::max<int64_t>(1, t->dims[0]));
    return t->total;
}

static tl_status alloc_dense(tl_ctx* c, Tensor* t) {
    int64_t need = dense_local_elems(c, t);
    if (t->dense && t->dense_elems >= need) return TL_OK;
    cudaFree(t->dense);
    t->dense = nullptr;
    TL_CK(c, cudaMalloc(&t->dense, std::max<int64_t>(need, 1) * sizeof(float)));
    t->dense_elems = need;
    return TL_OK;
}

static tl_status alloc_bits(tl_ctx* c, Tensor* t) {
    if (t->rank != 2) return fail(c, TL_ERR_UNSUPPORTED, "%s: bit storage needs rank 2", t->name.c_str());
    int64_t words = (t->dims[1] + 31) / 32;
    int64_t rows = dense_rows(c, t);
    if (col_split(t)) {
        // this rank's slice of the columns of every row
        if (t->dims[1] % (128 * (int64_t)t->col_world))
            return fail(c, TL_ERR_UNSUPPORTED, "%s: column sharding needs a multiple of %d columns", t->name.c_str(),
                        128 * t->col_world);
        words = t->dims[1] / 32 / t->col_world;
        rows = t->dims[0];
    }
    if (t->bits && t->bits_words == words && t->bits_rows == rows) return TL_OK;
    cudaFree(t->bits);
    t->bits = nullptr;
    TL_CK(c, cudaMalloc(&t->bits, std::max<int64_t>(rows * words, 1) * sizeof(uint32_t)));
    t->bits_words = words;
    t->bits_rows = rows;
    return TL_OK;
}

tl_status ensure_dense(tl_ctx* c, Tensor* t) {
    if (col_split(t))
        return fail(c, TL_ERR_UNSUPPORTED, "%s: a column-sharded relation is read only as bit rows",
                    t->name.c_str());
    TL_TRY(alloc_dense(c, t));
    if (t->dense_valid) return TL_OK;
    if (t->zero) {
        TL_CK(c, cudaMemsetAsync(t->dense, 0, dense_local_elems(c, t) * sizeof(float), c->stream));
    } else if (t->bits_valid) {
        TL_TRY(ensure_bits(c, t));   // writes lazy bit rows first
        TL_TRY(launch_bits_to_dense(c, t));
    } else if (t->csr_valid) {
        TL_TRY(launch_csr_to_dense(c, t));
    } else {
        TL_CK(c, cudaMemsetAsync(t->dense, 0, dense_local_elems(c, t) * sizeof(float), c->stream));
    }
    t->dense_valid = true;
    return TL_OK;
}

tl_status ensure_bits(tl_ctx* c, Tensor* t) {
    // a column-sharded relation is written only by its closure fixpoint
    if (col_split(t) && !(t->bits_valid && !t->lazy_src))
        return fail(c, TL_ERR_UNSUPPORTED, "%s: a column-sharded relation must start as step(Edge) right before "
                    "its fixpoint", t->name.c_str());
    TL_TRY(alloc_bits(c, t));
    if (t->bits_valid && t->lazy_src) {
        Tensor* src = t->lazy_src;
        t->lazy_src = nullptr;
        if (!src->csr_valid || src->csr_stamp != t->lazy_stamp)
            return fail(c, TL_ERR_INVALID, "%s: the relation its rows were defined from changed", t->name.c_str());
        return launch_csr_to_bits(c, src, t);
    }
    if (t->bits_valid) return TL_OK;
    if (t->zero) {
        TL_CK(c, cudaMemsetAsync(t->bits, 0, t->bits_rows * t->bits_words * 4, c->stream));
    } else if (t->csr_valid) {
        TL_TRY(launch_csr_to_bits(c, t, t));
    } else {
        TL_TRY(ensure_dense(c, t));
        TL_TRY(launch_dense_to_bits(c, t));
    }
    t->bits_valid = true;
    t->lazy_src = nullptr;
    return TL_OK;
}

tl_status ensure_csr(tl_ctx* c, Tensor* t) {
    if (t->csr_valid) return TL_OK;
    return fail(c, TL_ERR_UNSUPPORTED, "%s: no sparse storage", t->name.c_str());
}

tl_status alloc_bits_public(tl_ctx* c, Tensor* t) { return alloc_bits(c, t); }

void mark_written_dense(Tensor* t) {
    t->lazy_src = nullptr;
    t->nonneg = false;
    t->dense_valid = true;
    t->zero = false;
    t->bits_valid = t->csr_valid = t->csc_valid = false;
}

void mark_written_bits(Tensor* t) {
    t->lazy_src = nullptr;
    t->nonneg = true;   // 0/1 values
    t->bits_valid = true;
    t->zero = false;
    t->boolean = true;
    t->dense_valid = t->csr_valid = t->csc_valid = false;
}

// Device pointer to read a tensor through (nullptr reads as zeros).
const float* read_ptr(tl_ctx* c, Tensor* t, tl_status* st) {
    *st = TL_OK;
    if (!t || !t->defined || t->zero) return nullptr;
    *st = ensure_dense(c, t);
    return *st == TL_OK ? t->dense : nullptr;
}

}  // namespace tl

// ============================================================================
// ABI: context
// ============================================================================
extern "C" void tl_default_opts(tl_init_opts* o) {
    if (!o) return;
    memset(o, 0, sizeof *o);
    o->device = -1;
    o->precision = TL_PREC_TF32;
    o->rank = 0;
    o->world_size = 1;
    o->max_sweeps = 1000;
    o->verbose = 0;
    o->comm_timeout_ms = 30000;
}

extern "C" tl_status tl_init(const tl_init_opts* opts, tl_ctx** out) {
    if (!out) return TL_ERR_INVALID;
    *out = nullptr;
    std::unique_ptr<tl_ctx> c(new tl_ctx());
    if (opts) c->opts = *opts; else tl_default_opts(&c->opts);
    if (c->opts.max_sweeps <= 0) c->opts.max_sweeps = 1000;
    if (c->opts.comm_timeout_ms <= 0) c->opts.comm_timeout_ms = 30000;
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return TL_ERR_CUDA;
    }
    int dev = c->opts.device;
    if (dev < 0) cudaGetDevice(&dev);
    if (dev >= ndev) return TL_ERR_INVALID;
    if (cudaSetDevice(dev) != cudaSuccess) return TL_ERR_CUDA;
    c->device = dev;
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) return TL_ERR_CUDA;
    if (cudaMalloc(&c->d_flags, 64 * sizeof(int)) != cudaSuccess) return TL_ERR_OOM;
    if (cudaMallocHost(&c->h_flags, 64 * sizeof(int)) != cudaSuccess) return TL_ERR_OOM;
    cudaMemset(c->d_flags, 0, 64 * sizeof(int));
    c->rank = c->opts.rank;
    c->world = c->opts.world_size > 0 ? c->opts.world_size : 1;
    if (c->world > 1) {
        tl_status s = comm_init(c.get());
        if (s != TL_OK) return s;
    }
    *out = c.release();
    return TL_OK;
}

extern "C" tl_status tl_shutdown(tl_ctx* c) {
    if (!c) return TL_OK;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (auto& kv : c->tensors) free_storage(kv.second.get());
    c->tensors.clear();
    for (auto& p : c->pending) { cudaEventDestroy(p.a); cudaEventDestroy(p.b); }
    for (auto e : c->event_pool) cudaEventDestroy(e);
    release_graphs(c);
    comm_peer_release(c);
    comm_sym_release(c, SYM_CLOSURE);
    comm_sym_release(c, SYM_GNN);
    if (c->comm) comm_destroy(c);
    for (int i = 0; i < 4; ++i) cudaFree(c->ws[i]);
    cudaFree(c->aux);
    cudaFree(c->fix_state);
    cudaFree(c->fix_closed);
    if (c->fix_event) cudaEventDestroy(c->fix_event);
    bq_release(c);
    cudaFree(c->d_flags);
    cudaFreeHost(c->h_flags);
    cudaStreamDestroy(c->stream);
    delete c;
    return TL_OK;
}

extern "C" const char* tl_last_error(const tl_ctx* c) { return c ? c->err.c_str() : "no context"; }

namespace tl {
// Device-side error words: [8] a tensor-core pipeline wait gave up.
tl_status check_device_flags(tl_ctx* c) {
    // only the tensor-core GEMM and the message-passing SpMM write the error
    // word (1: a pipeline wait ran out, 2: a wait for another rank's tiles
    // ran out): without one since the last read there is nothing to read
    // (and no reason to wait for the stream)
    if (!c->flags_armed) return TL_OK;
    c->flags_armed = false;
    TL_CK(c, cudaMemcpyAsync(c->h_flags + 8, c->d_flags + 8, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    TL_CK(c, cudaStreamSynchronize(c->stream));
    if (c->h_flags[8] != 0) {
        const int what = c->h_flags[8];
        c->h_flags[8] = 0;
        TL_CK(c, cudaMemsetAsync(c->d_flags + 8, 0, sizeof(int), c->stream));
        if (what == 2) {
            if (c->world > 1) c->peer_state = -1;   // the ranks' tile counts may disagree now
            return fail(c, TL_ERR_COMM, "a wait for another rank's fanned-out tiles timed out; results are invalid");
        }
        return fail(c, TL_ERR_CUDA, "a tensor-core pipeline wait timed out; results are invalid");
    }
    return TL_OK;
}
}  // namespace tl

extern "C" tl_status tl_sync(tl_ctx* c) {
    if (!c) return TL_ERR_INVALID;
    TL_CK(c, cudaStreamSynchronize(c->stream));
    TL_CK(c, cudaGetLastError());
    TL_TRY(fix_resolve(c));
    return check_device_flags(c);
}

extern "C" int32_t tl_last_sweeps(const tl_ctx* c) {
    if (!c) return 0;
    // a fixpoint result still in flight is read here (cached state of the context)
    tl_ctx* m = const_cast<tl_ctx*>(c);
    fix_resolve(m);
    return m->last_sweeps;
}
extern "C" int64_t tl_launch_count(const tl_ctx* c) { return c ? c->launches : 0; }
extern "C" void* tl_stream(const tl_ctx* c) { return c ? (void*)c->stream : nullptr; }

extern "C" tl_status tl_domain(tl_ctx* c, const char* name, int64_t size) {
    if (!c || !name) return TL_ERR_INVALID;
    if (size >= 0) c->domains[name] = size;
    return TL_OK;
}

// updateTensorMaxDims (tensor.zig:84-129) over every equation's LHS.
extern "C" tl_status tl_declare_dims(tl_ctx* c, const tl_equation* eqs, int32_t n) {
    if (!c || (n > 0 && !eqs)) return TL_ERR_INVALID;
    for (int e = 0; e < n; ++e) {
        const tl_ref* lhs = &eqs[e].lhs;
        if (lhs->rank <= 0) continue;
        if (lhs->rank > TL_MAX_RANK) return fail(c, TL_ERR_INVALID, "LHS rank too large");
        auto it = c->maxdims.find(lhs->tensor);
        if (it == c->maxdims.end()) {
            std::vector<int64_t> d(lhs->rank);
            for (int k = 0; k < lhs->rank; ++k) d[k] = index_extent(c, &lhs->idx[k]);
            c->maxdims[lhs->tensor] = d;
        } else {
            for (int k = 0; k < lhs->rank && k < (int)it->second.size(); ++k)
                it->second[k] = std::max(it->second[k], index_extent(c, &lhs->idx[k]));
        }
    }
    return TL_OK;
}

// ============================================================================
// ABI: tensors
// ============================================================================
extern "C" tl_status tl_tensor_create(tl_ctx* c, const char* name, int32_t rank, const int64_t* dims,
                                      tl_tensor** out) {
    if (!c || !name || !out || rank < 0 || (rank > 0 && !dims)) return TL_ERR_INVALID;
    Tensor* t = find(c, name);
    if (t && t->defined) { *out = static_cast<tl_tensor*>(t); return TL_OK; }
    TL_TRY(new_tensor(c, name, rank, dims, &t));
    *out = static_cast<tl_tensor*>(t);
    return TL_OK;
}

extern "C" tl_status tl_tensor_lookup(tl_ctx* c, const char* name, tl_tensor** out) {
    if (!c || !name || !out) return TL_ERR_INVALID;
    Tensor* t = find_defined(c, name);
    if (!t) return fail(c, TL_ERR_NOT_FOUND, "tensor %s not found", name);
    *out = static_cast<tl_tensor*>(t);
    return TL_OK;
}

extern "C" int32_t tl_tensor_rank(const tl_tensor* t) { return t ? t->rank : -1; }
extern "C" int64_t tl_tensor_dim(const tl_tensor* t, int32_t a) {
    return (t && a >= 0 && a < t->rank) ? t->dims[a] : -1;
}
extern "C" int64_t tl_tensor_numel(const tl_tensor* t) { return t ? t->total : -1; }

// Owner context of a tensor (tensors never move between contexts).
static tl_ctx* owner_of(const Tensor* t) { return t ? (tl_ctx*)t->owner : nullptr; }

// Host staging buffer (pinned) for f64 <-> f32 conversion.
static tl_status staging(tl_ctx* c, size_t bytes, float** out) {
    static thread_local float* buf = nullptr;
    static thread_local size_t cap = 0;
    if (bytes > cap) {
        if (buf) cudaFreeHost(buf);
        buf = nullptr;
        size_t n = std::max(bytes, (size_t)1 << 20);
        TL_CK(c, cudaMallocHost(&buf, n));
        cap = n;
    }
    *out = buf;
    return TL_OK;
}

static tl_status upload_common(tl_ctx* c, Tensor* t, const double* h64, const float* h32) {
    TL_TRY(alloc_dense(c, t));
    int64_t rows = t->rank >= 1 ? t->dims[0] : 1;
    int64_t row_elems = rows > 0 ? t->total / rows : 0;
    bool sharded = t->shard == TL_SHARD_ROWS && c->world > 1;
    int64_t lrows = sharded ? dense_rows(c, t) : rows;
    int64_t n = sharded ? lrows * row_elems : t->total;
    float* st = nullptr;
    TL_TRY(staging(c, n * sizeof(float) + 16, &st));
    // the staging buffer is reused: wait for earlier copies out of it
    TL_CK(c, cudaStreamSynchronize(c->stream));
    bool boolean = true, nonneg = true;
    for (int64_t lr = 0; lr < lrows; ++lr) {
        int64_t gr = sharded ? lr * c->world + c->rank : lr;
        const int64_t src = gr * row_elems, dst = lr * row_elems;
        for (int64_t j = 0; j < row_elems; ++j) {
            float v = h64 ? (float)h64[src + j] : h32[src + j];
            st[dst + j] = v;
            boolean = boolean && (v == 0.0f || v == 1.0f);
            nonneg = nonneg && v >= 0.0f;
        }
    }
    if (t->rank == 0 || rows == 0) { /* scalar / empty */ }
    TL_CK(c, cudaMemcpyAsync(t->dense, st, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    mark_written_dense(t);
    t->boolean = boolean;
    t->nonneg = nonneg;
    return TL_OK;
}

extern "C" tl_status tl_tensor_upload(tl_tensor* t, const double* host) {
    tl_ctx* c = owner_of(t);
    if (!c || !host) return TL_ERR_INVALID;
    return upload_common(c, t, host, nullptr);
}

extern "C" tl_status tl_tensor_upload_f32(tl_tensor* t, const float* host) {
    tl_ctx* c = owner_of(t);
    if (!c || !host) return TL_ERR_INVALID;
    return upload_common(c, t, nullptr, host);
}

static tl_status download_f32(tl_ctx* c, Tensor* t, float** st_out, int64_t* n_out) {
    int64_t n = dense_local_elems(c, t);
    float* st = nullptr;
    TL_TRY(staging(c, n * sizeof(float) + 16, &st));
    if (!t->defined || t->zero) {
        memset(st, 0, n * sizeof(float));
    } else {
        TL_TRY(ensure_dense(c, t));
        TL_CK(c, cudaMemcpyAsync(st, t->dense, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
        TL_CK(c, cudaStreamSynchronize(c->stream));
        TL_TRY(check_device_flags(c));   // values a timed-out pipeline left are not returned as valid
    }
    *st_out = st;
    *n_out = n;
    return TL_OK;
}

// A row-sharded tensor downloads its local rows (rank, rank+world, ...) packed.
extern "C" tl_status tl_tensor_download(tl_tensor* t, double* host) {
    tl_ctx* c = owner_of(t);
    if (!c || !host) return TL_ERR_INVALID;
    float* st; int64_t n;
    TL_TRY(download_f32(c, t, &st, &n));
    for (int64_t i = 0; i < n; ++i) host[i] = st[i];
    return TL_OK;
}

extern "C" tl_status tl_tensor_download_f32(tl_tensor* t, float* host) {
    tl_ctx* c = owner_of(t);
    if (!c || !host) return TL_ERR_INVALID;
    float* st; int64_t n;
    TL_TRY(download_f32(c, t, &st, &n));
    memcpy(host, st, n * sizeof(float));
    return TL_OK;
}

extern "C" tl_status tl_tensor_download_bits(tl_tensor* t, uint32_t* host) {
    tl_ctx* c = owner_of(t);
    if (!c || !host) return TL_ERR_INVALID;
    if (t->rank != 2) return fail(c, TL_ERR_UNSUPPORTED, "bit download needs rank 2");
    if (!t->boolean && !t->bits_valid) return fail(c, TL_ERR_UNSUPPORTED, "%s is not 0/1 valued", t->name.c_str());
    TL_TRY(ensure_bits(c, t));
    TL_CK(c, cudaMemcpyAsync(host, t->bits, t->bits_rows * t->bits_words * 4, cudaMemcpyDeviceToHost, c->stream));
    TL_CK(c, cudaStreamSynchronize(c->stream));
    return check_device_flags(c);
}

extern "C" tl_status tl_tensor_device_ptr(tl_tensor* t, float** dptr) {
    tl_ctx* c = owner_of(t);
    if (!c || !dptr) return TL_ERR_INVALID;
    TL_TRY(ensure_dense(c, t));
    mark_written_dense(t);   // the caller may write through the pointer
    *dptr = t->dense;
    return TL_OK;
}

extern "C" tl_status tl_tensor_set(tl_tensor* t, const int64_t* idx, double v) {
    tl_ctx* c = owner_of(t);
    if (!c || !idx) return TL_ERR_INVALID;
    int64_t off = 0;
    for (int k = 0; k < t->rank; ++k) {
        if (idx[k] < 0 || idx[k] >= t->dims[k]) return fail(c, TL_ERR_INVALID, "index out of range");
        off += idx[k] * t->strides[k];
    }
    if (t->shard == TL_SHARD_ROWS && c->world > 1) return fail(c, TL_ERR_UNSUPPORTED, "set on a sharded tensor");
    TL_TRY(ensure_dense(c, t));
    float f = (float)v;
    TL_CK(c, cudaMemcpyAsync(t->dense + off, &f, 4, cudaMemcpyHostToDevice, c->stream));
    TL_CK(c, cudaStreamSynchronize(c->stream));
    bool b = t->boolean && (f == 0.0f || f == 1.0f);
    const bool nn = t->nonneg && f >= 0.0f;
    mark_written_dense(t);
    t->boolean = b;
    t->nonneg = nn;
    return TL_OK;
}

// COO upload into CSR (rows of this rank when sharded).  The CSR is built on
// the host (counting sort by row, columns ascending within a row); a
// repeated (row, col) keeps the last value, as repeated element assignments
// would.
extern "C" tl_status tl_sparse_upload(tl_tensor* t, int64_t nnz, const int64_t* rows, const int64_t* cols,
                                      const double* vals) {
    tl_ctx* c = owner_of(t);
    if (!c || nnz < 0 || (nnz > 0 && (!rows || !cols))) return TL_ERR_INVALID;
    if (t->rank != 2) return fail(c, TL_ERR_UNSUPPORTED, "sparse storage needs rank 2");
    if (t->dims[1] > INT32_MAX) return fail(c, TL_ERR_UNSUPPORTED, "sparse column count exceeds int32");
    const bool sharded = t->shard == TL_SHARD_ROWS && c->world > 1;
    const int64_t lrows = dense_rows(c, t);
    // large uploads build the CSR on the device; the host build below takes
    // the rest (few entries, or a local row of more than 32 entries)
    bool on_device = false;
    TL_TRY(csr_from_coo_gpu(c, t, nnz, rows, cols, vals, lrows, &on_device));
    if (on_device) {
        t->csr_rows = lrows;
        t->zero = false;
        t->defined = true;
        t->csr_valid = true;
        t->csr_stamp = next_csr_stamp();
        t->boolean = t->csr_nonneg && t->csr_ones;
        t->nonneg = t->csr_nonneg;
        t->dense_valid = t->bits_valid = t->csc_valid = false;
        return TL_OK;
    }
    // counting sort of the entries by (local) row, stable in input order
    std::vector<int64_t> rowptr(lrows + 2, 0);
    for (int64_t e = 0; e < nnz; ++e) {
        if (rows[e] < 0 || rows[e] >= t->dims[0] || cols[e] < 0 || cols[e] >= t->dims[1])
            return fail(c, TL_ERR_INVALID, "COO entry %lld out of range", (long long)e);
        if (sharded && rows[e] % c->world != c->rank) continue;
        rowptr[(sharded ? rows[e] / c->world : rows[e]) + 1]++;
    }
    for (int64_t r = 0; r < lrows; ++r) rowptr[r + 1] += rowptr[r];
    const int64_t count = rowptr[lrows];
    // the columns (and values) scattered to their rows in input order, so the
    // per-row pass below reads contiguous memory
    std::vector<int32_t> gcol(std::max<int64_t>(count, 1));
    std::vector<float> gval(vals ? std::max<int64_t>(count, 1) : 0);
    {
        std::vector<int64_t> fillp(rowptr.begin(), rowptr.end() - 1);
        for (int64_t e = 0; e < nnz; ++e) {
            if (sharded && rows[e] % c->world != c->rank) continue;
            const int64_t at = fillp[sharded ? rows[e] / c->world : rows[e]]++;
            gcol[at] = (int32_t)cols[e];
            if (vals) gval[at] = (float)vals[e];
        }
    }
    // the CSR is assembled in the pinned staging buffer and copied from there:
    // row pointers, then columns, then values (16-byte aligned sections)
    const size_t ptr_b = ((size_t)(lrows + 1) * 8 + 15) & ~size_t(15);
    const size_t col_b = ((size_t)count * 4 + 15) & ~size_t(15);
    float* stage = nullptr;
    TL_TRY(staging(c, ptr_b + col_b + (size_t)count * 4 + 16, &stage));
    TL_CK(c, cudaStreamSynchronize(c->stream));   // earlier copies out of the staging buffer
    int64_t* out_ptr = reinterpret_cast<int64_t*>(stage);
    int32_t* out_col = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(stage) + ptr_b);
    float* out_val = reinterpret_cast<float*>(reinterpret_cast<char*>(stage) + ptr_b + col_b);
    // each row sorted by column (stable, so among repeats of a column the last
    // entry of the input comes last and is the one kept)
    bool nonneg = true, ones = true, pos = true;
    int64_t n = 0;
    out_ptr[0] = 0;
    std::vector<std::pair<int32_t, float>> longrow;
    for (int64_t r = 0; r < lrows; ++r) {
        int32_t* bc = gcol.data() + rowptr[r];
        float* bv = vals ? gval.data() + rowptr[r] : nullptr;
        const int64_t len = rowptr[r + 1] - rowptr[r];
        if (len <= 32) {
            for (int64_t i = 1; i < len; ++i) {
                const int32_t kc = bc[i];
                const float kv = bv ? bv[i] : 1.0f;
                int64_t j = i - 1;
                while (j >= 0 && bc[j] > kc) {
                    bc[j + 1] = bc[j];
                    if (bv) bv[j + 1] = bv[j];
                    --j;
                }
                bc[j + 1] = kc;
                if (bv) bv[j + 1] = kv;
            }
        } else {
            longrow.resize(len);
            for (int64_t i = 0; i < len; ++i) longrow[i] = {bc[i], bv ? bv[i] : 1.0f};
            std::stable_sort(longrow.begin(), longrow.end(),
                             [](const std::pair<int32_t, float>& x, const std::pair<int32_t, float>& y) {
                                 return x.first < y.first;
                             });
            for (int64_t i = 0; i < len; ++i) {
                bc[i] = longrow[i].first;
                if (bv) bv[i] = longrow[i].second;
            }
        }
        for (int64_t i = 0; i < len; ++i) {
            if (i + 1 < len && bc[i + 1] == bc[i]) continue;
            const float v = bv ? bv[i] : 1.0f;
            nonneg = nonneg && v >= 0.0f;
            pos = pos && v > 0.0f;
            ones = ones && v == 1.0f;
            out_col[n] = bc[i];
            out_val[n] = v;
            ++n;
        }
        out_ptr[r + 1] = n;
    }
    if (n > t->csr_cap || !t->rowptr || t->csr_rows != lrows) {
        cudaFree(t->rowptr); cudaFree(t->colidx); cudaFree(t->vals);
        t->rowptr = nullptr; t->colidx = nullptr; t->vals = nullptr;
        const int64_t cap = std::max<int64_t>(n, 1);
        TL_CK(c, cudaMalloc(&t->rowptr, (lrows + 1) * sizeof(int64_t)));
        TL_CK(c, cudaMalloc(&t->colidx, cap * sizeof(int32_t)));
        TL_CK(c, cudaMalloc(&t->vals, cap * sizeof(float)));
        t->csr_cap = cap;
    }
    // copies from pinned memory; waited for here, since the staging buffer is
    // shared by every context of this host thread
    TL_CK(c, cudaMemcpyAsync(t->rowptr, out_ptr, (lrows + 1) * 8, cudaMemcpyHostToDevice, c->stream));
    if (n) {
        TL_CK(c, cudaMemcpyAsync(t->colidx, out_col, n * 4, cudaMemcpyHostToDevice, c->stream));
        TL_CK(c, cudaMemcpyAsync(t->vals, out_val, n * 4, cudaMemcpyHostToDevice, c->stream));
    }
    TL_CK(c, cudaStreamSynchronize(c->stream));
    t->nnz = n;
    t->csr_rows = lrows;
    t->zero = false;
    t->defined = true;
    t->csr_valid = true;
    t->csr_stamp = next_csr_stamp();
    t->csr_nonneg = nonneg;
    t->csr_pos = pos;
    t->csr_ones = ones;
    t->boolean = nonneg && ones;
    t->nonneg = nonneg;
    t->dense_valid = t->bits_valid = t->csc_valid = false;
    return TL_OK;
}

extern "C" tl_status tl_query_format(tl_tensor* t, char* buf, int64_t len) {
    tl_ctx* c = owner_of(t);
    if (!c || !buf || len <= 0) return TL_ERR_INVALID;
    int64_t np = std::min<int64_t>(t->total, 20);
    std::vector<double> v(std::max<int64_t>(t->total, 1));
    if (t->shard == TL_SHARD_ROWS && c->world > 1) return fail(c, TL_ERR_UNSUPPORTED, "query of a sharded tensor");
    TL_TRY(tl_tensor_download(t, v.data()));
    std::string s;
    char tmp[64];
    snprintf(tmp, sizeof tmp, "%s[%zu] = [", t->name.c_str(), (size_t)t->total);
    s += tmp;
    for (int64_t i = 0; i < np; ++i) { snprintf(tmp, sizeof tmp, "%.4g ", v[i]); s += tmp; }
    s += "]\n";
    snprintf(buf, (size_t)len, "%s", s.c_str());
    return TL_OK;
}

extern "C" tl_status tl_program_output(tl_ctx* c, char* buf, int64_t len, int64_t* needed) {
    if (!c || (len > 0 && !buf) || len < 0) return TL_ERR_INVALID;
    if (needed) *needed = (int64_t)c->query_out.size();
    if (len > 0) snprintf(buf, (size_t)len, "%s", c->query_out.c_str());
    return TL_OK;
}

extern "C" tl_status tl_set_sharding(tl_ctx* c, const char* name, int32_t mode) {
    if (!c || !name || (mode != TL_SHARD_NONE && mode != TL_SHARD_ROWS && mode != TL_SHARD_COLS)) return TL_ERR_INVALID;
    auto& slot = c->tensors[name];
    if (!slot) { slot.reset(new tl_tensor()); slot->name = name; slot->defined = false; slot->owner = c; }
    // columns: slice rank of world; TL_SHARD_COLS_OF="r/n" makes it slice r
    // of n on a one-GPU context (tests check the slices one by one against
    // the whole relation)
    int col_rank = 0, col_world = 1;
    if (mode == TL_SHARD_COLS) {
        col_rank = c->rank;
        col_world = c->world;
        const char* of = getenv("TL_SHARD_COLS_OF");
        if (of && c->world == 1) {
            int r = -1, w = 0;
            if (sscanf(of, "%d/%d", &r, &w) != 2 || w < 1 || r < 0 || r >= w) return TL_ERR_INVALID;
            col_rank = r;
            col_world = w;
        }
    }
    if (slot->shard != mode || slot->col_rank != col_rank || slot->col_world != col_world) {
        free_storage(slot.get());
        slot->shard = mode;
        slot->col_rank = col_rank;
        slot->col_world = col_world;
        slot->zero = true;
    }
    return TL_OK;
}

extern "C" tl_status tl_profile_enable(tl_ctx* c, int32_t on) {
    if (!c) return TL_ERR_INVALID;
    c->prof = on != 0;
    return TL_OK;
}

static tl_status drain_profile(tl_ctx* c) {
    if (c->pending.empty()) return TL_OK;
    TL_CK(c, cudaStreamSynchronize(c->stream));
    for (auto& p : c->pending) {
        float ms = 0;
        cudaEventElapsedTime(&ms, p.a, p.b);
        auto& s = c->stats[p.name];
        s.launches++;
        s.total_ms += ms;
        s.bytes += p.bytes;
        s.flops += p.flops;
        c->event_pool.push_back(p.a);
        c->event_pool.push_back(p.b);
    }
    c->pending.clear();
    return TL_OK;
}

extern "C" int32_t tl_profile_read(tl_ctx* c, tl_kernel_stats* out, int32_t max) {
    if (!c) return 0;
    if (drain_profile(c) != TL_OK) return 0;
    int n = 0;
    for (auto& kv : c->stats) {
        if (n >= max || !out) break;
        tl_kernel_stats& s = out[n++];
        memset(&s, 0, sizeof s);
        snprintf(s.name, TL_NAME_LEN, "%s", kv.first.c_str());
        s.launches = kv.second.launches;
        s.total_ms = kv.second.total_ms;
        s.algo_bytes = kv.second.bytes;
        s.algo_flops = kv.second.flops;
    }
    return n;
}

extern "C" tl_status tl_profile_reset(tl_ctx* c) {
    if (!c) return TL_ERR_INVALID;
    TL_TRY(drain_profile(c));
    c->stats.clear();
    return TL_OK;
}

