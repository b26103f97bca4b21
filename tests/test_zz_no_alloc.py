"""The allocation-free closure entry point against the oracle and the regular one.

tl_closure_noalloc exists for callers that must not allocate GPU memory (a
host whose device memory belongs to its own pool or arena, which may not
call cudaMalloc behind it): they pass every buffer in, and the library keeps
the fixpoint's scratch in a fixed array of its own.  This test, run last,
makes the caller-side allocations itself (with torch), calls the entry point
through the C ABI on several relations in a row (the last one exactly
TL_NOALLOC_MAX_ROWS rows, which fills the whole scratch array), and checks
each result and sweep count against the oracle's closure and against
tl_program_run on the same relation.  Boolean results: bit-exact.
"""
import ctypes as C
import os

import numpy as np
import pytest

from tensor_logic_lang_b200 import abi, lang
from tensor_logic_lang_b200 import inputs as gen
from tensor_logic_lang_b200.runtime import Context

pytestmark = pytest.mark.gpu


def _program(n, rows, cols):
    src = (f"domain x: {n}\ndomain y: {n}\ndomain z: {n}\nsparse Edge[x, y]\n"
           "Reach[x,y] = step(Edge[x,y])\nReach[x,z] max= step(Reach[x,y] Edge[y,z])\n")
    return lang.Program(src, sparse_inputs={"Edge": (rows, cols, None)})


def _cyclic(n, m, seed):
    rng = np.random.default_rng(seed)
    pairs = np.unique(rng.integers(0, n, size=(m, 2)), axis=0)
    pairs = pairs[pairs[:, 0] != pairs[:, 1]]
    return pairs[:, 0].copy(), pairs[:, 1].copy()


def _oracle(oracle_lib, n, rows, cols):
    colptr, rowidx = gen.csr_from_coo(n, cols, rows)
    R = np.zeros((n, (n + 31) // 32), dtype=np.uint32)
    np.bitwise_or.at(R, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
    sweeps = oracle_lib.closure_right(n, colptr, rowidx, R, threads=os.cpu_count() or 1)
    return R, sweeps


def _noalloc(lib, torch, n, rows, cols, device=0, stream=None):
    rowptr, colidx = gen.csr_from_coo(n, rows, cols)
    words = (n + 31) // 32
    R0 = np.zeros((n, words), dtype=np.uint32)
    np.bitwise_or.at(R0, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
    # caller-owned device buffers
    with torch.cuda.device(device):             # the current device for the call
        d_rowptr = torch.from_numpy(rowptr).cuda()
        d_colidx = torch.from_numpy(colidx).cuda()
        d_reach = torch.from_numpy(R0.view(np.int32)).cuda()
        torch.cuda.synchronize()
        sweeps = C.c_int32(0)
        st = lib.tl_closure_noalloc(n, d_rowptr.data_ptr(), d_colidx.data_ptr(), d_reach.data_ptr(), 0, stream,
                                    C.byref(sweeps))
        assert st == abi.TL_OK, abi.STATUS_NAMES.get(st, st)
        return d_reach.cpu().numpy().view(np.uint32), sweeps.value


def test_noalloc_matches_oracle_and_program_run(oracle_lib):
    import torch
    lib = abi.load_library()
    big = abi.TL_NOALLOC_MAX_ROWS
    cases = [(4096,) + gen.random_dag(4096, 4, 31), (3000,) + _cyclic(3000, 7000, 32),
             (big,) + gen.random_dag(big, 2, 33)]
    ctx = Context(device=0)
    try:
        for n, rows, cols in cases:          # calls in a row, different relations
            got, sweeps = _noalloc(lib, torch, n, rows, cols)
            want, want_sweeps = _oracle(oracle_lib, n, rows, cols)
            np.testing.assert_array_equal(got, want)
            if np.all(rows < cols):
                assert sweeps == want_sweeps == 2
            else:
                # with cycles every row still closes in its first sweep, so
                # the count can be below the reference's in-place order
                assert 2 <= sweeps <= want_sweeps
            ctx.run(_program(n, rows, cols))
            np.testing.assert_array_equal(got, ctx.bits("Reach"))
            assert sweeps == ctx.sweeps
    finally:
        ctx.close()


def test_noalloc_on_a_second_device(oracle_lib):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    lib = abi.load_library()
    n = 4096
    rows, cols = gen.random_dag(n, 4, 34)
    want, want_sweeps = _oracle(oracle_lib, n, rows, cols)
    got, sweeps = _noalloc(lib, torch, n, rows, cols, device=1)   # its own scratch address
    np.testing.assert_array_equal(got, want)
    assert sweeps == want_sweeps
    # a stream of device 1 while device 0 is current is refused before any work
    other = torch.cuda.Stream(device=1)
    with torch.cuda.device(0):
        st = lib.tl_closure_noalloc(n, 1, 1, 1, 0, other.cuda_stream, None)
    assert st == abi.TL_ERR_INVALID


def test_noalloc_rejects_oversized_relation():
    lib = abi.load_library()
    sweeps = C.c_int32(-1)
    st = lib.tl_closure_noalloc(abi.TL_NOALLOC_MAX_ROWS + 1, None, None, None, 0, None, C.byref(sweeps))
    assert st == abi.TL_ERR_TOO_LARGE and sweeps.value == 0
