"""Drive libtl_cuda through its C ABI (include/tl_cuda.h).

`Context` owns one tl_ctx on one GPU; `Context.run(program)` executes a
lowered `.tl` program the way the reference's emitted `main()` does
(LLVMCodegen.generate order: statements, fixpoint, queries), and
`Context.tensor(name)` reads a result back as f64 numpy.  There is no CPU
fallback: without the built library or a GPU, construction raises.
"""
import ctypes as C

import numpy as np

from . import abi


class Context:
    def __init__(self, device=-1, precision=abi.PREC_TF32, rank=0, world_size=1, nccl_id=None,
                 max_sweeps=1000, verbose=False, comm_timeout_ms=30000, lib=None):
        self.lib = lib or abi.load_library()
        opts = abi.InitOpts()
        self.lib.tl_default_opts(C.byref(opts))
        opts.device = device
        opts.precision = precision
        opts.rank = rank
        opts.world_size = world_size
        opts.max_sweeps = max_sweeps
        opts.verbose = 1 if verbose else 0
        opts.comm_timeout_ms = comm_timeout_ms
        if nccl_id is not None:
            for i, b in enumerate(bytes(nccl_id)[:128]):
                opts.nccl_id[i] = b
        h = C.c_void_p()
        st = self.lib.tl_init(C.byref(opts), C.byref(h))
        if st != abi.TL_OK:
            raise abi.TLError(st, "tl_init failed (no CUDA device or bad options)")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.tl_shutdown(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def check(self, st, what=""):
        if st != abi.TL_OK:
            msg = self.lib.tl_last_error(self.h).decode(errors="replace")
            raise abi.TLError(st, f"{what}: {msg}")

    # ------------------------------------------------------------------ program
    def run(self, program):
        self.check(self.lib.tl_program_run(self.h, C.cast(program.stmts, C.POINTER(abi.Statement)), program.n),
                   "tl_program_run")
        return self

    def sync(self):
        self.check(self.lib.tl_sync(self.h), "tl_sync")

    @property
    def sweeps(self):
        return self.lib.tl_last_sweeps(self.h)

    def last_error(self):
        """tl_last_error: the text of the last failure or note (the sweep cap)."""
        return self.lib.tl_last_error(self.h).decode(errors="replace")

    @property
    def launches(self):
        return self.lib.tl_launch_count(self.h)

    @property
    def stream_ptr(self):
        return self.lib.tl_stream(self.h)

    def set_sharding(self, name, mode=abi.SHARD_ROWS):
        self.check(self.lib.tl_set_sharding(self.h, name.encode(), mode), "tl_set_sharding")

    # ------------------------------------------------------------------ tensors
    def _lookup(self, name):
        t = C.c_void_p()
        self.check(self.lib.tl_tensor_lookup(self.h, name.encode(), C.byref(t)), f"lookup {name}")
        return t

    def shape(self, name):
        t = self._lookup(name)
        return tuple(self.lib.tl_tensor_dim(t, k) for k in range(self.lib.tl_tensor_rank(t)))

    def tensor(self, name, rows=None):
        """f64 copy of a tensor (a row-sharded one gives its local rows)."""
        t = self._lookup(name)
        shape = self.shape(name)
        if rows is not None:
            shape = (rows,) + shape[1:]
        out = np.empty(shape, dtype=np.float64)
        self.check(self.lib.tl_tensor_download(t, out.ctypes.data_as(C.POINTER(C.c_double))), f"download {name}")
        return out

    def tensor_f32(self, name, rows=None):
        t = self._lookup(name)
        shape = self.shape(name)
        if rows is not None:
            shape = (rows,) + shape[1:]
        out = np.empty(shape, dtype=np.float32)
        self.check(self.lib.tl_tensor_download_f32(t, out.ctypes.data_as(C.POINTER(C.c_float))), f"download {name}")
        return out

    def bits(self, name, rows=None, out=None, words=None):
        """Bit rows (uint32 words) of a 0/1 rank-2 tensor (into `out` when given,
        e.g. a pinned host buffer).  A row-sharded tensor gives its `rows`
        local rows; a column-sharded one its slice of `words` words per row."""
        t = self._lookup(name)
        r, cols = self.shape(name)
        if rows is not None:
            r = rows
        w = (cols + 31) // 32 if words is None else words
        if out is None:
            out = np.empty((r, w), dtype=np.uint32)
        assert out.dtype == np.uint32 and out.flags.c_contiguous and out.shape == (r, w)
        self.check(self.lib.tl_tensor_download_bits(t, out.ctypes.data_as(C.POINTER(C.c_uint32))), f"bits {name}")
        return out

    def upload(self, name, arr):
        t = self._lookup(name)
        a = np.ascontiguousarray(arr, dtype=np.float64)
        self.check(self.lib.tl_tensor_upload(t, a.ctypes.data_as(C.POINTER(C.c_double))), f"upload {name}")

    def upload_f32(self, name, arr):
        t = self._lookup(name)
        a = np.ascontiguousarray(arr, dtype=np.float32)
        self.check(self.lib.tl_tensor_upload_f32(t, a.ctypes.data_as(C.POINTER(C.c_float))), f"upload {name}")

    def create(self, name, shape):
        t = C.c_void_p()
        dims = (C.c_int64 * max(1, len(shape)))(*shape)
        self.check(self.lib.tl_tensor_create(self.h, name.encode(), len(shape), dims, C.byref(t)), f"create {name}")
        return t

    def query(self, name):
        t = self._lookup(name)
        buf = C.create_string_buffer(4096)
        self.check(self.lib.tl_query_format(t, buf, len(buf)), f"query {name}")
        return buf.value.decode()

    def output(self):
        """What the last program's queries printed (the reference's stdout)."""
        need = C.c_int64()
        self.check(self.lib.tl_program_output(self.h, None, 0, C.byref(need)), "program output")
        buf = C.create_string_buffer(need.value + 1)
        self.check(self.lib.tl_program_output(self.h, buf, len(buf), None), "program output")
        return buf.value.decode()

    # ------------------------------------------------------------------ profiling
    def profile(self, on=True):
        self.check(self.lib.tl_profile_enable(self.h, 1 if on else 0), "profile")

    def profile_reset(self):
        self.check(self.lib.tl_profile_reset(self.h), "profile_reset")

    def profile_read(self):
        arr = (abi.KernelStats * 64)()
        n = self.lib.tl_profile_read(self.h, arr, 64)
        return {arr[i].name.decode(): dict(launches=arr[i].launches, total_ms=arr[i].total_ms,
                                           bytes=arr[i].algo_bytes, flops=arr[i].algo_flops)
                for i in range(n)}


def unique_id(lib=None):
    lib = lib or abi.load_library()
    buf = (C.c_uint8 * 128)()
    st = lib.tl_comm_unique_id(buf)
    if st != abi.TL_OK:
        raise abi.TLError(st, "tl_comm_unique_id")
    return bytes(buf)
