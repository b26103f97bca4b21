"""Program runs replayed as CUDA graphs: a program whose inputs stay on the
device is captured once its host state repeats, and later runs replay the
graph.  Every replayed run must give the oracle's results, also after new
input values are written into the same device storage."""
import numpy as np
import pytest

from tensor_logic_lang_b200 import configs
from tensor_logic_lang_b200 import inputs as gen

from gpu_helpers import TOL_TF32, assert_close

pytestmark = pytest.mark.gpu


def resident(builder, **kw):
    """The config's program, and a copy whose loads keep the device contents."""
    p, data, sparse, _ = configs.program(builder, **kw)
    p_res = configs.program(builder, **kw)[0]
    for k in range(p_res.n):
        s = p_res.stmts[k]
        if s.kind == 6:        # load: no host data, no file
            s.host_data = None
            s.path = b""
        if s.kind == 7:        # sparse load: keep the CSR on the device
            s.coo_rows = None
            s.coo_cols = None
    return p, p_res, data, sparse


def replays(ctx):
    return ctx.profile_read().get("program_graph_replay", {}).get("launches", 0)


def test_replayed_gnn_runs_match_oracle(gpu_ctx_factory, oracle_lib):
    ctx = gpu_ctx_factory()
    try:
        n, f = 512, 32
        p, p_res, d, sp = resident(configs.gnn, n=n, f=f)
        ctx.run(p)
        rows, cols, _ = sp["Adj"]
        rowptr, colidx = gen.csr_from_coo(n, rows, cols)
        h1 = oracle_lib.gnn_layer(rowptr, colidx, d["H0"], d["W1"])
        h2 = oracle_lib.gnn_layer(rowptr, colidx, h1, d["W2"])
        per_run = None
        for _ in range(5):
            before = ctx.launches
            ctx.run(p_res)
            launched = ctx.launches - before
            per_run = per_run or launched
            assert launched == per_run
            assert_close(ctx.tensor("H1"), h1, TOL_TF32, "H1")
            assert_close(ctx.tensor("H2"), h2, TOL_TF32, "H2")
        assert replays(ctx) >= 2

        # new input values in the same storage: a replay reads them
        H0b = gen.normal(77, "H0b", (n, f))
        ctx.upload("H0", H0b)
        for _ in range(3):
            ctx.run(p_res)
        h1b = oracle_lib.gnn_layer(rowptr, colidx, H0b, d["W1"])
        h2b = oracle_lib.gnn_layer(rowptr, colidx, h1b, d["W2"])
        assert_close(ctx.tensor("H1"), h1b, TOL_TF32, "H1 after upload")
        assert_close(ctx.tensor("H2"), h2b, TOL_TF32, "H2 after upload")
    finally:
        ctx.close()


def test_replayed_training_steps_match_oracle(gpu_ctx_factory, oracle_lib):
    ctx = gpu_ctx_factory()
    try:
        p, p_res, d, _ = resident(configs.mlp_train, b=256, i=784, h=512, o=10)
        ctx.run(p)
        ref = oracle_lib.OracleRun(p)
        for _ in range(5):
            ctx.run(p_res)
            for name in ("Z1", "Y", "dL_dW2"):
                assert_close(ctx.tensor(name), ref.tensor(name), TOL_TF32, name)
        assert replays(ctx) >= 2
    finally:
        ctx.close()
