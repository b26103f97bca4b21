"""CUDA backend against the known answers and the f64 oracle (small programs)."""
import json
import os

import numpy as np
import pytest

from tensor_logic_lang_b200 import lang

from gpu_helpers import TOL_FP32, assert_close

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "known_answers.json")))


@pytest.fixture(scope="module")
def ctx(gpu_ctx_factory):
    c = gpu_ctx_factory()
    yield c
    c.close()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_known_answer(ctx, oracle_lib, case):
    p = lang.Program(case["src"])
    ctx.run(p)
    ref = oracle_lib.OracleRun(p)
    for name, want in case["expect"].items():
        got = ctx.tensor(name)
        want = np.asarray(want, dtype=float).reshape(got.shape)
        if name in ("R", "Anc"):
            np.testing.assert_array_equal(got, want)          # Boolean: bit-exact
        else:
            assert_close(got, want, TOL_FP32, name)
        assert_close(got, ref.tensor(name), TOL_FP32, name + " vs oracle")
    if "sweeps" in case:
        assert ctx.sweeps == case["sweeps"] == ref.sweeps


def test_query_text_matches_oracle(ctx, oracle_lib):
    case = next(c for c in CASES if c["name"] == "matmul")
    p = lang.Program(case["src"])
    ctx.run(p)
    ref = oracle_lib.OracleRun(p)
    assert ctx.query("C") == ref.queries


def test_repeated_runs_start_from_calloc(ctx):
    # `=` with a contraction accumulates into the LHS; a second run of the
    # same program must start from zeros again (calloc on first sight)
    case = next(c for c in CASES if c["name"] == "matmul")
    p = lang.Program(case["src"])
    ctx.run(p)
    first = ctx.tensor("C")
    ctx.run(p)
    np.testing.assert_array_equal(ctx.tensor("C"), first)


def test_unsupported_forms_report_errors(ctx):
    from tensor_logic_lang_b200 import abi
    p = lang.Program("domain i: 4\nA[i] = 1\nB[i] = concat(A[i])\n")
    with pytest.raises(abi.TLError) as e:
        ctx.run(p)
    assert e.value.status == abi.TL_ERR_UNSUPPORTED
