"""The CUDA backend on the reference's own example programs.

Every tensor each example defines is compared with the f64 oracle's value
recorded in tests/golden/reference_examples.json (the oracle itself is held
to answers derived by hand in tests/test_reference_examples.py): Boolean
relations bit-exact, float tensors within the fp32 tolerance; the printed
query text byte for byte; fixpoint sweep counts exactly; and the raw f64
files fileio.tl saves.
"""
import json
import os

import numpy as np
import pytest

from tensor_logic_lang_b200 import lang

from gpu_helpers import TOL_FP32, assert_close

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "reference_examples.json")))
BOOLEAN = {"Ancestor", "Reach"}


@pytest.fixture(scope="module")
def ctx(gpu_ctx_factory):
    c = gpu_ctx_factory()
    yield c
    c.close()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_example_matches_oracle(ctx, case, tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    p = lang.Program(case["src"])
    ctx.run(p)
    rec = case["oracle"]
    for name, want in rec["tensors"].items():
        got = ctx.tensor(name)
        assert list(got.shape) == want["shape"], name
        want = np.asarray(want["values"], dtype=np.float64).reshape(got.shape)
        if name in BOOLEAN:
            np.testing.assert_array_equal(got, want, err_msg=name)
        else:
            assert_close(got, want, TOL_FP32, name)
    assert ctx.output() == rec["queries"]
    if rec["sweeps"]:
        assert ctx.sweeps == rec["sweeps"]
    for path, want in case.get("expect_files", {}).items():
        got = np.fromfile(tmp_path / path, dtype=np.float64)
        assert got.shape == (len(want),), path
        assert_close(got, want, TOL_FP32, path)


def test_saved_files_load_back(ctx, oracle_lib, tmp_path, monkeypatch):
    # fileio.tl saves W1; a second program loads the raw f64 file
    # (llvm.zig:565-633 layout) into a fresh tensor and uses it
    monkeypatch.chdir(tmp_path)
    case = next(c for c in CASES if c["name"] == "fileio")
    ctx.run(lang.Program(case["src"]))
    src = ("domain i: 4\ndomain h: 3\nV[i,h] = 0\nload V \"w1.bin\"\nS[i] = V[i,h]\nT[h,i] = V[i,h]\nS?\n")
    p = lang.Program(src)
    ctx.run(p)
    ref = oracle_lib.OracleRun(p)
    want = np.asarray(case["expect_files"]["w1.bin"]).reshape(4, 3)
    assert_close(ctx.tensor("V"), want, TOL_FP32, "V")
    assert_close(ctx.tensor("S"), want.sum(axis=1), TOL_FP32, "S")
    assert_close(ctx.tensor("T"), want.T, TOL_FP32, "T")
    assert_close(ctx.tensor("S"), ref.tensor("S"), TOL_FP32, "S vs oracle")
    assert ctx.output() == ref.queries
