"""Failure detection on one GPU, in the forms that fault nothing.

The reference stops a fixpoint silently after its sweep cap
(fixpoint.zig:67-72).  The backend does the same: the run returns TL_OK, the
sweep count equals the cap, tl_last_error carries a note, and the relation
holds exactly the state the reference's capped loop leaves (checked against
the oracle run with the same cap).  Both closure paths are covered: the
left form (one launch per sweep) and the right form (every sweep inside one
cooperative launch, whose cap is read from the device's control block).
"""
import numpy as np
import pytest

from tensor_logic_lang_b200 import lang
from tensor_logic_lang_b200 import inputs as gen

pytestmark = pytest.mark.gpu


def _chain_left(n):
    edges = "\n".join(f"Par[{a},{a + 1}] = 1" for a in range(n - 1))
    return (f"domain p: {n}\ndomain x: {n}\ndomain y: {n}\ndomain z: {n}\nsparse Par[p, p]\n{edges}\n"
            "Anc[x,y] = step(Par[x,y])\nAnc[x,y] max= step(Par[x,z] Anc[z,y])\n")


@pytest.mark.parametrize("cap", [1, 3, 7])
def test_left_form_stops_at_the_cap(gpu_ctx_factory, oracle_lib, cap):
    p = lang.Program(_chain_left(20))      # needs 19 sweeps to converge
    ctx = gpu_ctx_factory(max_sweeps=cap)
    try:
        ctx.run(p)
        assert ctx.sweeps == cap
        assert "cap" in ctx.last_error()
        ref = oracle_lib.OracleRun(p, max_sweeps=cap)
        assert ref.sweeps == cap
        np.testing.assert_array_equal(ctx.tensor("Anc"), ref.tensor("Anc"))
    finally:
        ctx.close()


def test_right_form_one_launch_stops_at_the_cap(gpu_ctx_factory, oracle_lib):
    # on a DAG the first sweep closes every row and changes them, so a cap of
    # one stops before the sweep that would find nothing left
    n = 2048
    rows, cols = gen.random_dag(n, 4, 11)
    src = (f"domain x: {n}\ndomain y: {n}\ndomain z: {n}\nsparse Edge[x, y]\n"
           "Reach[x,y] = step(Edge[x,y])\nReach[x,z] max= step(Reach[x,y] Edge[y,z])\n")
    p = lang.Program(src, sparse_inputs={"Edge": (rows, cols, None)})
    ctx = gpu_ctx_factory(max_sweeps=1)
    try:
        ctx.run(p)
        assert ctx.sweeps == 1
        assert "cap" in ctx.last_error()
        colptr, rowidx = gen.csr_from_coo(n, cols, rows)
        R = np.zeros((n, n // 32), dtype=np.uint32)
        np.bitwise_or.at(R, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
        assert oracle_lib.closure_right(n, colptr, rowidx, R, max_sweeps=1) == 1
        np.testing.assert_array_equal(ctx.bits("Reach"), R)
        # the context is usable afterwards: the uncapped run converges in two
        ctx2 = gpu_ctx_factory()
        try:
            ctx2.run(p)
            assert ctx2.sweeps == 2
        finally:
            ctx2.close()
    finally:
        ctx.close()
