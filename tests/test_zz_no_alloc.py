"""The allocation-free closure entry point against the regular one.

tl_closure_noalloc exists for callers that must not allocate GPU memory (a
host whose device memory belongs to its own pool, or work prepared around
stream capture): they pass every buffer in, and the library keeps the
fixpoint's scratch in a fixed array of its own.  This test, run last, makes
the caller-side allocations itself (with torch), calls the entry point through
the C ABI twice in a row, and checks each result and sweep count against
tl_program_run on the same relation.  Boolean results: bit-exact.
"""
import ctypes as C

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


def _noalloc(lib, torch, n, rows, cols):
    rowptr, colidx = gen.csr_from_coo(n, rows, cols)
    words = (n + 31) // 32
    R0 = np.zeros((n, words), dtype=np.uint32)
    np.bitwise_or.at(R0, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
    # caller-owned device buffers
    d_rowptr = torch.from_numpy(rowptr).cuda()
    d_colidx = torch.from_numpy(colidx).cuda()
    d_reach = torch.from_numpy(R0.view(np.int32)).cuda()
    torch.cuda.synchronize()
    sweeps = C.c_int32(0)
    st = lib.tl_closure_noalloc(n, d_rowptr.data_ptr(), d_colidx.data_ptr(), d_reach.data_ptr(), 0, None,
                                C.byref(sweeps))
    assert st == abi.TL_OK, abi.STATUS_NAMES.get(st, st)
    return d_reach.cpu().numpy().view(np.uint32), sweeps.value


def test_noalloc_matches_program_run():
    import torch
    lib = abi.load_library()
    cases = [(4096,) + gen.random_dag(4096, 4, 31), (3000,) + _cyclic(3000, 7000, 32)]
    ctx = Context(device=0)
    try:
        for n, rows, cols in cases:          # two calls in a row, different relations
            got, sweeps = _noalloc(lib, torch, n, rows, cols)
            ctx.run(_program(n, rows, cols))
            np.testing.assert_array_equal(got, ctx.bits("Reach"))
            assert sweeps == ctx.sweeps
    finally:
        ctx.close()


def test_noalloc_rejects_oversized_relation():
    lib = abi.load_library()
    sweeps = C.c_int32(-1)
    st = lib.tl_closure_noalloc(abi.TL_NOALLOC_MAX_ROWS + 1, None, None, None, 0, None, C.byref(sweeps))
    assert st == abi.TL_ERR_TOO_LARGE and sweeps.value == 0
