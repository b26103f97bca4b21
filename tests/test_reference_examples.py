"""The f64 oracle against the reference's own example programs.

tests/golden/reference_examples.json holds the nine programs of the
reference's examples/ folder with answers derived independently of the
oracle (tests/golden/make_reference_examples.py): C = A B of matmul.tl, the
strict upper triangle of ancestor.tl with its 9 sweeps, zero gradients
through explicit `*` in training.tl, the temperature sigmoids, the three
zero answers of backward_query.tl, and the files fileio.tl saves.  The
oracle must reproduce every one of them; the GPU tests then compare the
CUDA backend with the oracle's values recorded in the same file.
"""
import json
import os

import numpy as np
import pytest

from tensor_logic_lang_b200 import lang

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "reference_examples.json")))
REF_CHECKOUT = os.environ.get("TL_REFERENCE_CHECKOUT", "/root/reference")


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_hand_answers(oracle_lib, case, tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)                 # fileio.tl saves to relative paths
    r = oracle_lib.OracleRun(lang.Program(case["src"]))
    assert r.status == 0
    for name, want in case["expect"].items():
        got = r.tensor(name)
        assert list(got.shape) == want["shape"], name
        np.testing.assert_allclose(got.ravel(), want["values"], rtol=0, atol=1e-12, err_msg=name)
    assert r.queries == case["expect_queries"]
    if "expect_sweeps" in case:
        assert r.sweeps == case["expect_sweeps"]
    for path, want in case.get("expect_files", {}).items():
        got = np.fromfile(tmp_path / path, dtype=np.float64)
        np.testing.assert_array_equal(got, want, err_msg=path)
    # the recorded oracle values are the ones the GPU tests compare with
    for name, rec in case["oracle"]["tensors"].items():
        np.testing.assert_array_equal(r.tensor(name).ravel(), rec["values"], err_msg=name)
    assert r.queries == case["oracle"]["queries"] and r.sweeps == case["oracle"]["sweeps"]


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF_CHECKOUT, "examples")),
                    reason="no reference checkout on this machine")
@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_fixture_text_is_the_reference_example(case):
    with open(os.path.join(REF_CHECKOUT, case["source"])) as f:
        assert f.read() == case["src"]
