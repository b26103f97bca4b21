"""Constant-index (backward-chaining) queries on the GPU against the oracle
and the hand-traced answers: the printed text of the whole program."""
import numpy as np
import pytest

from tensor_logic_lang_b200 import abi, lang

import backward_cases as bc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx(gpu_ctx_factory):
    c = gpu_ctx_factory()
    yield c
    c.close()


def run_both(ctx, oracle_lib, src, data=None):
    p = lang.Program(src, inputs=data)
    ctx.run(p)
    ref = oracle_lib.OracleRun(p)
    assert ref.status == 0
    return ctx.output(), ref.queries


def parse(text):
    out = []
    for line in text.splitlines():
        name, value = line.split(" = ")
        out.append((name, float(value)))
    return out


@pytest.mark.parametrize("name,src,want", bc.KNOWN, ids=[k[0] for k in bc.KNOWN])
def test_known_answers(ctx, oracle_lib, name, src, want):
    got, ref = run_both(ctx, oracle_lib, src)
    assert got == want == ref


def test_forward_and_backward_queries_interleave(ctx, oracle_lib):
    got, ref = run_both(ctx, oracle_lib, bc.MIXED)
    assert got == ref


def test_out_of_range_constant(ctx, oracle_lib):
    got, ref = run_both(ctx, oracle_lib, bc.OUT_OF_RANGE)
    assert got == ref


def test_query_without_equation_is_an_error(ctx):
    with pytest.raises(abi.TLError) as e:
        ctx.run(lang.Program(bc.NO_EQUATION))
    assert e.value.status == abi.TL_ERR_UNSUPPORTED


def test_memo_starts_empty_each_run(ctx, oracle_lib):
    p = lang.Program(bc.CYCLE_LATE)
    ctx.run(p)
    first = ctx.output()
    ctx.run(lang.Program(bc.CYCLE_EARLY))
    assert ctx.output() == bc.CYCLE_EARLY_OUT
    ctx.run(p)
    assert ctx.output() == first == bc.CYCLE_LATE_OUT


GRAPHS = [(12, 20, False), (12, 20, True), (24, 50, True), (40, 90, True), (40, 70, False)]


@pytest.mark.parametrize("form", ["right", "left"])
@pytest.mark.parametrize("n,m,cyclic", GRAPHS, ids=[f"n{g[0]}-m{g[1]}-{'cyc' if g[2] else 'dag'}" for g in GRAPHS])
def test_random_graphs(ctx, oracle_lib, n, m, cyclic, form):
    edges, queries = bc.random_graph(n, m, 12, seed=n * 7 + m, cyclic=cyclic)
    got, ref = run_both(ctx, oracle_lib, bc.graph_program(n, edges, queries, form))
    assert got == ref
    assert len(got.splitlines()) == len(queries)


def test_long_chain_recursion(ctx, oracle_lib):
    # the left form on a 400-node chain: the query's row is computed through
    # a stack about 400 frames deep, and the elements it reads while they are
    # still in progress make the far pairs 0 (the forward fixpoint converges
    # in two sweeps, so the oracle stays quick)
    n = 400
    edges = [(i, i + 1) for i in range(n - 1)]
    src = bc.graph_program(n, edges, [(0, n - 1), (n - 1, 0), (5, 300), (0, 2)], "left")
    got, ref = run_both(ctx, oracle_lib, src)
    assert got == ref == "R = 0\nR = 0\nR = 0\nR = 1\n"


@pytest.mark.parametrize("n,seed", [(6, 1), (17, 2)])
def test_float_equations(ctx, oracle_lib, n, seed):
    src, data = bc.float_program(n, seed)
    # inputs on a 1/64 grid are exact in the fp32 device storage, so the
    # values differ from the f64 oracle only by the device's exp
    data = {k: np.round(v * 64) / 64 for k, v in data.items()}
    got, ref = run_both(ctx, oracle_lib, src, data)
    g, r = parse(got), parse(ref)
    assert [a for a, _ in g] == [a for a, _ in r]
    for (name, x), (_, y) in zip(g, r):
        assert abs(x - y) <= 1e-5 * abs(y) + 1e-6, (name, x, y)


@pytest.mark.parametrize("env", [{"TL_BQ_MAX_STEPS": "50"}, {"TL_BQ_MAX_MS": "1", "TL_BQ_MAX_STEPS": "0"}],
                         ids=["step_budget", "time_limit"])
def test_budget_ends_the_interpreter_with_an_error(ctx, monkeypatch, env):
    # the device interpreter stops at its step budget, or at its time limit
    # on %globaltimer (read every 1024 steps), and the run reports
    # TL_ERR_TOO_LARGE; the context stays usable afterwards.  The 400-node
    # chain takes far more than 50 steps, and far more than 1 ms.
    n = 400
    edges = [(i, i + 1) for i in range(n - 1)]
    src = bc.graph_program(n, edges, [(0, n - 1)] * 1 + [(k, n - 1) for k in range(0, 200, 10)], "left")
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    with pytest.raises(abi.TLError) as e:
        ctx.run(lang.Program(src))
    assert e.value.status == abi.TL_ERR_TOO_LARGE
    for k in env:
        monkeypatch.delenv(k)
    ctx.run(lang.Program(bc.CHAIN))
    assert ctx.output() == bc.CHAIN_OUT
