"""ctypes binding of the f64 oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the product package.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def build():
    subprocess.run(["make", "-C", HERE, "-s"], check=True)


def _load(name="liboracle.so"):
    path = os.path.join(HERE, name)
    if not os.path.exists(path):
        build()
    lib = C.CDLL(path)
    vp = C.c_void_p
    lib.or_create.restype = vp
    lib.or_create.argtypes = [C.c_int32]
    lib.or_destroy.argtypes = [vp]
    lib.or_program_run.restype = C.c_int32
    lib.or_program_run.argtypes = [vp, vp, C.c_int32]
    lib.or_tensor_info.restype = C.c_int32
    lib.or_tensor_info.argtypes = [vp, C.c_char_p, C.POINTER(C.c_int32), C.POINTER(C.c_int64)]
    lib.or_tensor_data.restype = C.POINTER(C.c_double)
    lib.or_tensor_data.argtypes = [vp, C.c_char_p]
    lib.or_last_sweeps.restype = C.c_int32
    lib.or_last_sweeps.argtypes = [vp]
    lib.or_query_output.restype = C.c_char_p
    lib.or_query_output.argtypes = [vp]
    lib.or_last_error.restype = C.c_char_p
    lib.or_last_error.argtypes = [vp]
    lib.or_closure_right.restype = C.c_int32
    lib.or_closure_right.argtypes = [C.c_int64, C.POINTER(C.c_int64), C.POINTER(C.c_int32),
                                     C.POINTER(C.c_uint32), C.c_int64, C.c_int64, C.c_int32, C.c_int32]
    lib.or_gnn_layer.restype = None
    lib.or_gnn_layer.argtypes = [C.c_int64, C.c_int64, C.c_int64, C.POINTER(C.c_int64),
                                 C.POINTER(C.c_int32), C.POINTER(C.c_double), C.POINTER(C.c_double),
                                 C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_int32]
    lib.or_gemm.restype = None
    lib.or_gemm.argtypes = [C.c_int64, C.c_int64, C.c_int64, C.POINTER(C.c_double), C.c_int64,
                            C.c_int64, C.POINTER(C.c_double), C.c_int64, C.c_int64,
                            C.POINTER(C.c_double), C.c_int64, C.c_int64, C.c_int32, C.c_double,
                            C.c_int32]
    lib.or_closure_literal_rows.restype = C.c_int64
    lib.or_closure_literal_rows.argtypes = [C.c_int64, C.POINTER(C.c_uint32), C.c_int64, C.c_int64,
                                            C.POINTER(C.c_double)]
    lib.or_closure_literal_rows_mt.restype = C.c_int64
    lib.or_closure_literal_rows_mt.argtypes = [C.c_int64, C.POINTER(C.c_uint32), C.c_int64, C.c_int64,
                                               C.POINTER(C.c_double), C.c_int32]
    return lib


_LIBS = {}


def lib(name="liboracle.so"):
    if name not in _LIBS:
        _LIBS[name] = _load(name)
    return _LIBS[name]


class OracleRun:
    """Run one program on a fresh oracle context; read tensors back as numpy."""

    def __init__(self, program, max_sweeps=1000, libname="liboracle.so"):
        self.lib = lib(libname)
        self.ctx = self.lib.or_create(max_sweeps)
        self.program = program
        self.status = self.lib.or_program_run(self.ctx, C.addressof(program.stmts), program.n)

    def __del__(self):
        if getattr(self, "ctx", None):
            self.lib.or_destroy(self.ctx)
            self.ctx = None

    def tensor(self, name):
        rank = C.c_int32()
        dims = (C.c_int64 * 8)()
        if self.lib.or_tensor_info(self.ctx, name.encode(), C.byref(rank), dims) != 0:
            raise KeyError(name)
        shape = tuple(dims[k] for k in range(rank.value))
        n = int(np.prod(shape))
        ptr = self.lib.or_tensor_data(self.ctx, name.encode())
        return np.ctypeslib.as_array(ptr, shape=(n,)).copy().reshape(shape)

    def has(self, name):
        return self.lib.or_tensor_info(self.ctx, name.encode(), None, None) == 0

    @property
    def sweeps(self):
        return self.lib.or_last_sweeps(self.ctx)

    @property
    def queries(self):
        return self.lib.or_query_output(self.ctx).decode()


def closure_right(n, colptr, rowidx, R, row_begin=0, row_end=None, max_sweeps=1000, threads=0):
    """In-place right-form closure over bit rows R[(row_end-row_begin), ceil(n/32)] (uint32)."""
    row_end = n if row_end is None else row_end
    colptr = np.ascontiguousarray(colptr, dtype=np.int64)
    rowidx = np.ascontiguousarray(rowidx, dtype=np.int32)
    assert R.dtype == np.uint32 and R.flags.c_contiguous
    return lib().or_closure_right(n, colptr.ctypes.data_as(C.POINTER(C.c_int64)),
                                  rowidx.ctypes.data_as(C.POINTER(C.c_int32)),
                                  R.ctypes.data_as(C.POINTER(C.c_uint32)), row_begin, row_end,
                                  max_sweeps, threads)


def gnn_layer(rowptr, colidx, H, W, vals=None, threads=0):
    n, g = H.shape
    f = W.shape[1]
    rowptr = np.ascontiguousarray(rowptr, dtype=np.int64)
    colidx = np.ascontiguousarray(colidx, dtype=np.int32)
    H = np.ascontiguousarray(H, dtype=np.float64)
    W = np.ascontiguousarray(W, dtype=np.float64)
    out = np.zeros((n, f), dtype=np.float64)
    vp = None
    if vals is not None:
        vals = np.ascontiguousarray(vals, dtype=np.float64)
        vp = vals.ctypes.data_as(C.POINTER(C.c_double))
    D = C.POINTER(C.c_double)
    lib().or_gnn_layer(n, g, f, rowptr.ctypes.data_as(C.POINTER(C.c_int64)),
                       colidx.ctypes.data_as(C.POINTER(C.c_int32)), vp, H.ctypes.data_as(D),
                       W.ctypes.data_as(D), out.ctypes.data_as(D), threads)
    return out


def gemm(A, B, C_init=None, relu_per_term=False, scale=1.0, threads=0):
    """C[m,n] (+)= sum_k term(A[m,k], B[k,n]) in the reference's loop order (f64)."""
    A = np.asarray(A, dtype=np.float64)
    B = np.asarray(B, dtype=np.float64)
    M, K = A.shape
    N = B.shape[1]
    out = np.zeros((M, N)) if C_init is None else np.array(C_init, dtype=np.float64, copy=True)
    A = np.ascontiguousarray(A)
    Bt = np.ascontiguousarray(B.T)          # k contiguous for both operands in the inner loop
    D = C.POINTER(C.c_double)
    lib().or_gemm(M, N, K, A.ctypes.data_as(D), K, 1, Bt.ctypes.data_as(D), 1, K,
                  out.ctypes.data_as(D), N, 1, int(relu_per_term), scale, threads)
    return out


def closure_literal_rows(n, Ebits, R_rows, x0=0, threads=1, libname="liboracle.so"):
    """One literal reference-order sweep over the given f64 rows (in place),
    rows spread over `threads` host threads."""
    Ebits = np.ascontiguousarray(Ebits, dtype=np.uint32)
    assert R_rows.dtype == np.float64 and R_rows.flags.c_contiguous
    return lib(libname).or_closure_literal_rows_mt(n, Ebits.ctypes.data_as(C.POINTER(C.c_uint32)), x0,
                                                   R_rows.shape[0], R_rows.ctypes.data_as(C.POINTER(C.c_double)),
                                                   int(threads))
