"""The f64 oracle against the known answers and against its own literal loop nests.

CPU only.  The known answers (tests/golden/known_answers.json) are derived
independently of the oracle by tests/golden/make_known_answers.py.
"""
import json
import os

import numpy as np
import pytest

from tensor_logic_lang_b200 import configs, inputs, lang

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "known_answers.json")))


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_known_answers(oracle_lib, case):
    r = oracle_lib.OracleRun(lang.Program(case["src"]))
    assert r.status == 0
    for name, want in case["expect"].items():
        got = r.tensor(name)
        np.testing.assert_allclose(got.ravel(), np.asarray(want, dtype=float).ravel(), rtol=1e-12, atol=1e-12)
    if "sweeps" in case:
        assert r.sweeps == case["sweeps"]


def test_query_format(oracle_lib):
    case = next(c for c in CASES if c["name"] == "matmul")
    r = oracle_lib.OracleRun(lang.Program(case["src"]))
    C = np.asarray(case["expect"]["C"]).ravel()
    assert r.queries == "C[6] = [" + "".join("%.4g " % v for v in C) + "]\n"


def _closure_src(n):
    return (f"domain x: {n}\ndomain y: {n}\ndomain z: {n}\nsparse Edge[x, y]\n"
            "Reach[x,y] = step(Edge[x,y])\nReach[x,z] max= step(Reach[x,y] Edge[y,z])\n")


@pytest.mark.parametrize("n,deg", [(64, 2), (200, 4)])
def test_closure_restatement_matches_literal(oracle_lib, n, deg):
    """or_closure_right (CSC, row-wise) equals the literal Gauss-Seidel loop nest."""
    rows, cols = inputs.random_dag(n, deg, 11)
    p = lang.Program(_closure_src(n), sparse_inputs={"Edge": (rows, cols, None)})
    lit = oracle_lib.OracleRun(p)
    want = lit.tensor("Reach")
    colptr, rowidx = inputs.csr_from_coo(n, cols, rows)   # CSC = CSR of the transpose
    W = (n + 31) // 32
    R = np.zeros((n, W), dtype=np.uint32)
    for u, v in zip(rows, cols):
        R[u, v >> 5] |= np.uint32(1 << (v & 31))
    sweeps = oracle_lib.closure_right(n, colptr, rowidx, R)
    got = np.unpackbits(R.view(np.uint8), bitorder="little").reshape(n, W * 32)[:, :n]
    np.testing.assert_array_equal(got, want.astype(np.uint8))
    assert sweeps == lit.sweeps == 2


def test_closure_restatement_cycles(oracle_lib):
    """A graph with back edges: same fixpoint and sweep count as the literal loops."""
    n = 80
    rng = np.random.default_rng(3)
    rows = rng.integers(0, n, 300)
    cols = rng.integers(0, n, 300)
    keep = rows != cols
    rows, cols = rows[keep], cols[keep]
    pairs = np.unique(np.stack([rows, cols], 1), axis=0)
    rows, cols = pairs[:, 0], pairs[:, 1]
    lit = oracle_lib.OracleRun(lang.Program(_closure_src(n), sparse_inputs={"Edge": (rows, cols, None)}))
    colptr, rowidx = inputs.csr_from_coo(n, cols, rows)
    W = (n + 31) // 32
    R = np.zeros((n, W), dtype=np.uint32)
    for u, v in zip(rows, cols):
        R[u, v >> 5] |= np.uint32(1 << (v & 31))
    sweeps = oracle_lib.closure_right(n, colptr, rowidx, R)
    got = np.unpackbits(R.view(np.uint8), bitorder="little").reshape(n, W * 32)[:, :n]
    np.testing.assert_array_equal(got, lit.tensor("Reach").astype(np.uint8))
    assert sweeps == lit.sweeps


def test_gnn_restatement_matches_literal(oracle_lib):
    """H = relu(Adj H0 W) per term over (u, g) equals Adj @ P with P = sum_g relu(H0 W)."""
    src, data, sparse, _ = configs.gnn(n=48, f=8, degree=3)
    p = lang.Program(src, inputs=data, sparse_inputs=sparse)
    lit = oracle_lib.OracleRun(p)
    rows, cols, _ = sparse["Adj"]
    rowptr, colidx = inputs.csr_from_coo(48, rows, cols)
    h1 = oracle_lib.gnn_layer(rowptr, colidx, data["H0"], data["W1"])
    np.testing.assert_allclose(h1, lit.tensor("H1"), rtol=1e-12, atol=1e-12)
    h2 = oracle_lib.gnn_layer(rowptr, colidx, h1, data["W2"])
    np.testing.assert_allclose(h2, lit.tensor("H2"), rtol=1e-12, atol=1e-12)


def test_gemm_restatement(oracle_lib):
    rng = np.random.default_rng(0)
    A = rng.normal(size=(5, 7))
    B = rng.normal(size=(7, 3))
    np.testing.assert_allclose(oracle_lib.gemm(A, B), A @ B, rtol=1e-12)
    relu = np.maximum(A[:, :, None] * B[None], 0).sum(1)
    np.testing.assert_allclose(oracle_lib.gemm(A, B, relu_per_term=True), relu, rtol=1e-12)


def test_configs_small_run(oracle_lib):
    for builder, kw in [(configs.mlp_forward, dict(b=4, i=16, h=8, o=3)),
                        (configs.attention, dict(s=8, d=4)),
                        (configs.mlp_train, dict(b=4, i=6, h=5, o=3))]:
        p, data, sparse, _ = configs.program(builder, **kw)
        r = oracle_lib.OracleRun(p)
        assert r.status == 0
    # C2: check the gradient chain against numpy
    p, d, _, _ = configs.program(configs.mlp_train, b=4, i=6, h=5, o=3)
    r = oracle_lib.OracleRun(p)
    Z1 = d["X"] @ d["W1"]
    H = np.maximum(Z1, 0)
    Z2 = H @ d["W2"]
    Y = np.exp(Z2) / np.exp(Z2).sum(1, keepdims=True)
    dY = 2 * (Y - d["Target"])
    dZ2 = Y * (dY - (dY * Y).sum())
    dW2 = H.T @ dZ2
    dZ1 = (dZ2 @ d["W2"].T) * (Z1 > 0)
    np.testing.assert_allclose(r.tensor("dL_dW2"), dW2, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(r.tensor("dL_dW1"), d["X"].T @ dZ1, rtol=1e-10, atol=1e-12)
