"""ctypes mirror of include/tl_cuda.h.

The structures here have the exact layout of the C ABI; both the CUDA runtime
(libtl_cuda.so) and the f64 oracle (oracle/liboracle.so) consume them.
"""
import ctypes as C
import os

TL_MAX_RANK = 8
TL_MAX_REFS = 8
TL_MAX_CODE = 48
TL_MAX_PARAMS = 8
TL_NAME_LEN = 32
TL_PATH_LEN = 256

# status codes
TL_OK = 0
TL_ERR_INVALID = 1
TL_ERR_OOM = 2
TL_ERR_CUDA = 3
TL_ERR_COMM = 4
TL_ERR_NOT_CONVERGED = 5
TL_ERR_UNSUPPORTED = 6
TL_ERR_NOT_FOUND = 7
TL_ERR_IO = 8
TL_ERR_TOO_LARGE = 9
STATUS_NAMES = {
    0: "TL_OK", 1: "TL_ERR_INVALID", 2: "TL_ERR_OOM", 3: "TL_ERR_CUDA",
    4: "TL_ERR_COMM", 5: "TL_ERR_NOT_CONVERGED", 6: "TL_ERR_UNSUPPORTED",
    7: "TL_ERR_NOT_FOUND", 8: "TL_ERR_IO", 9: "TL_ERR_TOO_LARGE",
}
TL_NOALLOC_MAX_ROWS = 65536

# index kinds
IX_NAME, IX_CONST, IX_ADD, IX_SUB, IX_PRIMED, IX_DIV, IX_NORMALIZE, IX_SLICE, IX_VIRTUAL = range(9)

# postfix ops
(OP_REF, OP_LIT, OP_PROD, OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_POW, OP_GT, OP_LT, OP_GE,
 OP_LE, OP_EQ, OP_NE, OP_AND, OP_OR, OP_NEG, OP_NOT, OP_NL) = range(19)

# nonlinearities
NL = {
    "step": 0, "softmax": 1, "relu": 2, "sigmoid": 3, "tanh": 4, "exp": 5, "log": 6,
    "abs": 7, "sqrt": 8, "sin": 9, "cos": 10, "norm": 11, "lnorm": 12, "concat": 13,
}

# accumulation ops
ACC = {"=": 0, "+=": 1, "*=": 2, "max=": 3, "min=": 4, "avg=": 5}

# statements
(STMT_DOMAIN, STMT_EQUATION, STMT_SPARSE, STMT_BACKWARD, STMT_QUERY, STMT_SAVE, STMT_LOAD,
 STMT_SPARSE_LOAD) = range(8)

PREC_TF32 = 0
PREC_FP32 = 1
SHARD_NONE = 0
SHARD_ROWS = 1
SHARD_COLS = 2


class Index(C.Structure):
    _fields_ = [("kind", C.c_int32), ("_pad", C.c_int32), ("value", C.c_int64),
                ("value2", C.c_int64), ("name", C.c_char * TL_NAME_LEN)]


class Ref(C.Structure):
    _fields_ = [("tensor", C.c_char * TL_NAME_LEN), ("rank", C.c_int32), ("_pad", C.c_int32),
                ("idx", Index * TL_MAX_RANK)]


class Instr(C.Structure):
    _fields_ = [("op", C.c_int32), ("arg", C.c_int32), ("arg2", C.c_int32), ("_pad", C.c_int32),
                ("value", C.c_double)]


class Equation(C.Structure):
    _fields_ = [("lhs", Ref), ("accum", C.c_int32), ("n_refs", C.c_int32), ("n_code", C.c_int32),
                ("_pad", C.c_int32), ("refs", Ref * TL_MAX_REFS), ("code", Instr * TL_MAX_CODE)]


class Statement(C.Structure):
    _fields_ = [("kind", C.c_int32), ("n_params", C.c_int32), ("size", C.c_int64),
                ("name", C.c_char * TL_NAME_LEN),
                ("params", (C.c_char * TL_NAME_LEN) * TL_MAX_PARAMS),
                ("path", C.c_char * TL_PATH_LEN),
                ("host_data", C.POINTER(C.c_double)),
                ("coo_rows", C.POINTER(C.c_int64)),
                ("coo_cols", C.POINTER(C.c_int64)),
                ("sparse", Ref), ("eq", Equation)]


class InitOpts(C.Structure):
    _fields_ = [("device", C.c_int32), ("precision", C.c_int32), ("rank", C.c_int32),
                ("world_size", C.c_int32), ("nccl_id", C.c_uint8 * 128), ("max_sweeps", C.c_int32),
                ("verbose", C.c_int32), ("comm_timeout_ms", C.c_int32), ("_pad", C.c_int32)]


class KernelStats(C.Structure):
    _fields_ = [("name", C.c_char * TL_NAME_LEN), ("launches", C.c_int64), ("total_ms", C.c_double),
                ("algo_bytes", C.c_double), ("algo_flops", C.c_double)]


PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(PKG_DIR, "libtl_cuda.so")

# Every symbol include/tl_cuda.h declares (checked by the CPU test suite).
EXPORTS = [
    "tl_default_opts", "tl_init", "tl_shutdown", "tl_last_error", "tl_sync", "tl_comm_unique_id",
    "tl_program_run", "tl_last_sweeps", "tl_domain", "tl_declare_dims", "tl_equation_run",
    "tl_fixpoint", "tl_backward", "tl_sparse_decl", "tl_tensor_create", "tl_tensor_lookup",
    "tl_tensor_rank", "tl_tensor_dim", "tl_tensor_numel", "tl_tensor_upload",
    "tl_tensor_download", "tl_tensor_upload_f32", "tl_tensor_download_f32",
    "tl_tensor_download_bits", "tl_tensor_device_ptr", "tl_tensor_set", "tl_sparse_upload",
    "tl_query_format", "tl_program_output", "tl_set_sharding", "tl_profile_enable", "tl_profile_read",
    "tl_profile_reset", "tl_launch_count", "tl_stream", "tl_closure_noalloc",
]


def _declare(lib):
    P = C.POINTER
    vp = C.c_void_p
    sigs = {
        "tl_default_opts": (None, [P(InitOpts)]),
        "tl_init": (C.c_int32, [P(InitOpts), P(vp)]),
        "tl_shutdown": (C.c_int32, [vp]),
        "tl_last_error": (C.c_char_p, [vp]),
        "tl_sync": (C.c_int32, [vp]),
        "tl_comm_unique_id": (C.c_int32, [P(C.c_uint8)]),
        "tl_program_run": (C.c_int32, [vp, P(Statement), C.c_int32]),
        "tl_last_sweeps": (C.c_int32, [vp]),
        "tl_domain": (C.c_int32, [vp, C.c_char_p, C.c_int64]),
        "tl_declare_dims": (C.c_int32, [vp, P(Equation), C.c_int32]),
        "tl_equation_run": (C.c_int32, [vp, P(Equation)]),
        "tl_fixpoint": (C.c_int32, [vp, P(Equation), C.c_int32, P(C.c_int32)]),
        "tl_backward": (C.c_int32, [vp, C.c_char_p, vp, C.c_int32, P(Equation), C.c_int32]),
        "tl_sparse_decl": (C.c_int32, [vp, P(Ref)]),
        "tl_tensor_create": (C.c_int32, [vp, C.c_char_p, C.c_int32, P(C.c_int64), P(vp)]),
        "tl_tensor_lookup": (C.c_int32, [vp, C.c_char_p, P(vp)]),
        "tl_tensor_rank": (C.c_int32, [vp]),
        "tl_tensor_dim": (C.c_int64, [vp, C.c_int32]),
        "tl_tensor_numel": (C.c_int64, [vp]),
        "tl_tensor_upload": (C.c_int32, [vp, P(C.c_double)]),
        "tl_tensor_download": (C.c_int32, [vp, P(C.c_double)]),
        "tl_tensor_upload_f32": (C.c_int32, [vp, P(C.c_float)]),
        "tl_tensor_download_f32": (C.c_int32, [vp, P(C.c_float)]),
        "tl_tensor_download_bits": (C.c_int32, [vp, P(C.c_uint32)]),
        "tl_tensor_device_ptr": (C.c_int32, [vp, P(P(C.c_float))]),
        "tl_tensor_set": (C.c_int32, [vp, P(C.c_int64), C.c_double]),
        "tl_sparse_upload": (C.c_int32, [vp, C.c_int64, P(C.c_int64), P(C.c_int64), P(C.c_double)]),
        "tl_query_format": (C.c_int32, [vp, C.c_char_p, C.c_int64]),
        "tl_program_output": (C.c_int32, [vp, C.c_char_p, C.c_int64, P(C.c_int64)]),
        "tl_set_sharding": (C.c_int32, [vp, C.c_char_p, C.c_int32]),
        "tl_profile_enable": (C.c_int32, [vp, C.c_int32]),
        "tl_profile_read": (C.c_int32, [vp, P(KernelStats), C.c_int32]),
        "tl_profile_reset": (C.c_int32, [vp]),
        "tl_launch_count": (C.c_int64, [vp]),
        "tl_stream": (C.c_void_p, [vp]),
        "tl_closure_noalloc": (C.c_int32, [C.c_int64, vp, vp, vp, C.c_int32, vp, P(C.c_int32)]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = None


def load_library(path=None):
    """Load libtl_cuda.so from the package directory.

    There is no fallback: a missing or unloadable library raises, so no test
    or benchmark can silently run anything but the CUDA backend.
    """
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(
            f"libtl_cuda.so not built at {p}; run `python -m tensor_logic_lang_b200.build`")
    # NCCL: load the same libnccl.so.2 torch uses before our library resolves it.
    try:
        import nvidia.nccl  # noqa: F401
        nccl_dir = os.path.join(list(nvidia.nccl.__path__)[0], "lib")
        cand = os.path.join(nccl_dir, "libnccl.so.2")
        if os.path.exists(cand):
            C.CDLL(cand, mode=C.RTLD_GLOBAL)
    except Exception:
        pass
    lib = _declare(C.CDLL(p, mode=C.RTLD_GLOBAL))
    if path is None:
        _LIB = lib
    return lib


class TLError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status
