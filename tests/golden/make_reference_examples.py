"""Fixtures from the reference's own example programs (reference_examples.json).

The reference's integration tests compile and run the programs in its
`examples/` folder (tests/integration_test.zig:12-23); they are the only
programs the reference itself holds for this path, but it checks no values.
This script reads each example from a checkout of the reference and records:

  * the program text, with the file it came from;
  * `expect`: answers derived here with plain numpy and pure-Python loops
    from the reference's rules, independently of the oracle:
      - an index letter without a `domain` of the same name has size 10
        (llvm.zig:407, 435; domain names are case-sensitive), so `i` in
        matmul.tl is 10 wide although `domain I: 3` is declared;
      - a tensor's extent is the largest over its left-hand uses
        (tensor.zig:84-129); reads past it are undefined in the reference
        and 0.0 here (gnn.tl and temperature.tl read past their tensors);
      - softmax is exp(x)/sum exp(x) over the last axis (softmax.zig:128-211);
      - sigmoid(x, T) = 1/(1+exp(-x/T)) (expr.zig:250-273);
      - the fixpoint is the in-place loop nest of fixpoint.zig:167-297,
        free indices outer, the contracted index inner, a sweep counted
        until one changes nothing (fixpoint.zig:46-98);
      - explicit `*` has no gradient rule (autodiff.zig:202-390), so
        training.tl's gradients are zero;
      - a `sparse` declaration re-allocates the relation the recursion
        reads (llvm.zig:482-516), so backward_query.tl's queries print 0;
      - a query prints `Name[total] = [` and the first 20 values as
        `%.4g ` (llvm.zig:461-480); a constant-index query prints
        `Name = %.6g` (backward.zig:568-600);
      - `save` writes the tensor as raw row-major f64 (llvm.zig:565-633);
  * `oracle`: every tensor the program defines, the printed queries and the
    sweep count, as the f64 oracle (oracle/) computes them — the values the
    GPU tests compare against on a machine without the reference checkout.

Run:  python tests/golden/make_reference_examples.py [reference checkout]
(default /root/reference); rewrites reference_examples.json next to this file.
"""
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

EXAMPLES = ["matmul", "ancestor", "backward_query", "attention", "gnn", "mlp", "temperature", "training", "fileio"]


def lit(shape, entries, fill=0.0):
    a = np.full(shape, fill)
    for idx, v in entries.items():
        a[idx] = v
    return a


def softmax_rows(z):
    e = np.exp(z)
    return e / e.sum(axis=-1, keepdims=True)


def sigmoid(x, t=1.0):
    return 1.0 / (1.0 + np.exp(-x / t))


def fixpoint_left(E, R):
    """R[x,y] max= step(E[x,z] R[z,y]) in place, x, y outer and z inner,
    rows past E's or R's extent reading 0; returns (R, sweeps)."""
    R = R.copy()
    nx, ny = R.shape
    nz = 10
    def e(x, z): return E[x, z] if x < E.shape[0] and z < E.shape[1] else 0.0
    def r(z, y): return R[z, y] if z < R.shape[0] and y < R.shape[1] else 0.0
    sweeps = 0
    while sweeps < 1000:
        changed = False
        for x in range(nx):
            for y in range(ny):
                for z in range(nz):
                    rhs = 1.0 if e(x, z) * r(z, y) > 0 else 0.0
                    if rhs > R[x, y]:
                        R[x, y] = rhs
                        changed = True
        sweeps += 1
        if not changed:
            break
    return R, sweeps


def query_text(name, arr):
    flat = np.asarray(arr, dtype=np.float64).ravel()
    return f"{name}[{flat.size}] = [" + "".join("%.4g " % v for v in flat[:20]) + "]\n"


def expected(name):
    """(tensors, queries or None, sweeps or None, files or None) derived by hand."""
    if name == "matmul":
        A = lit((10, 10), {(i, j): float(4 * i + j + 1) for i in range(3) for j in range(4)})
        B = lit((10, 10), {(j, k): float(2 * j + k + 1) for j in range(4) for k in range(2)})
        return {"A": A, "B": B, "C": A @ B}, "", None, None
    if name in ("ancestor", "backward_query"):
        P = lit((10, 10), {(a, a + 1): 1.0 for a in range(9)})
        R, sweeps = fixpoint_left(P, (P > 0).astype(float))
        assert np.array_equal(R, np.triu(np.ones((10, 10)), 1))
        q = "" if name == "ancestor" else "Ancestor = 0\n" * 3
        return {"Ancestor": R}, q, sweeps, None
    if name == "attention":
        Q = lit((10, 3), {(0, 0): 1, (0, 2): 1, (1, 0): .5, (1, 1): .5, (2, 1): 1, (2, 2): .5,
                          (3, 0): 1, (3, 1): 1, (3, 2): 1})
        K = lit((10, 3), {(0, 0): 1, (1, 1): 1, (2, 2): 1, (3, 0): .5, (3, 1): .5, (3, 2): .5})
        V = lit((10, 3), {(0, 0): 1, (1, 1): 1, (2, 2): 1, (3, 0): 1, (3, 1): 1, (3, 2): 1})
        S = Q @ K.T
        A = softmax_rows(S)
        return {"Q": Q, "K": K, "V": V, "Scores": S, "Attn": A, "Out": A @ V}, "", None, None
    if name == "gnn":
        A = lit((5, 10), {(a, a): 1.0 for a in range(5)})
        for a in range(4):
            A[a, a + 1] = 1.0
        X = lit((5, 4), {(0, 0): 1, (1, 1): 1, (2, 2): 1, (3, 3): 1, (4, 0): 1, (4, 1): 1, (4, 2): 1, (4, 3): 1})
        A5 = A[:, :5]                     # columns m >= 5 read rows past X / H*: 0.0
        H1 = A5 @ X
        H1r = np.maximum(H1, 0)
        H2 = A5 @ H1r
        H2r = np.maximum(H2, 0)
        H3 = A5 @ H2r
        R, sweeps = fixpoint_left(A, (A > 0).astype(float))
        return {"A": A, "X": X, "H1": H1, "H1r": H1r, "H2": H2, "H2r": H2r, "H3": H3, "Out": sigmoid(H3),
                "Reach": R}, "", sweeps, None
    if name == "mlp":
        X = np.array([[1.0, 0.5, -0.5], [-1.0, 2.0, 0.0]])
        W1 = np.array([[0.1, 0.2, 0.3], [-0.1, 0.4, 0.1], [0.2, -0.2, 0.5], [0.3, 0.1, -0.1]])
        W2 = np.array([[0.5, -0.3, 0.2, 0.1], [-0.4, 0.6, -0.1, 0.3]])
        Z1 = X @ W1.T
        H = np.maximum(Z1, 0)
        Z2 = H @ W2.T
        return {"Z1": Z1, "H": H, "Z2": Z2, "Y": softmax_rows(Z2)}, "", None, None
    if name == "temperature":
        E = lit((4, 3), {(0, 0): 1.0, (1, 1): 1.0, (2, 2): 1.0, (3, 0): 0.7, (3, 1): 0.7})
        Rel = lit((3, 3), {(0, 0): 2.0, (1, 1): 2.0, (2, 2): 2.0})
        E10 = np.zeros((10, 3))
        E10[:4] = E                       # rows i, j >= 4 read past Emb: 0.0
        S = E10 @ Rel @ E10.T
        t = {"Emb": E, "RelEmb": Rel, "Score": S, "Sharp": sigmoid(S, 0.1), "Medium": sigmoid(S, 1.0),
             "Soft": sigmoid(S, 5.0)}
        q = "".join(query_text(k, t[k]) for k in ("Score", "Sharp", "Medium", "Soft"))
        return t, q, None, None
    if name == "training":
        X = np.array([[1.0, 0.5, 0.2, 0.1], [0.3, 0.8, 0.4, 0.2]])
        W = np.full((4, 1), 0.5)
        b = np.full((1,), 0.1)
        T = np.array([[3.35], [2.7]])
        Lin = X @ W
        Y = Lin + b
        D = Y - T
        return {"W": W, "b": b, "Linear": Lin, "Y": Y, "Diff": D, "Loss": D * D,
                "dL_dW": np.zeros((4, 1)), "dL_db": np.zeros((1,))}, "", None, None
    if name == "fileio":
        W1 = lit((4, 3), {(0, 0): 0.1, (1, 1): 0.2, (2, 2): 0.3, (3, 0): 0.4}, fill=0.5)
        W2 = lit((3, 2), {(0, 0): 0.6, (1, 1): 0.7, (2, 0): 0.8}, fill=0.5)
        b1 = np.full((3,), 0.1)
        b2 = np.full((2,), 0.2)
        t = {"W1": W1, "W2": W2, "b1": b1, "b2": b2}
        q = query_text("W1", W1) + query_text("W2", W2)
        files = {"w1.bin": W1, "w2.bin": W2, "b1.bin": b1, "b2.bin": b2}
        return t, q, None, files
    raise KeyError(name)


def defined_tensors(program):
    names = []
    for st in program.parsed:
        if st[0] == "eq" and st[1][1] not in names:
            names.append(st[1][1])
        if st[0] == "backward":
            for p in st[2]:
                names.append("dL_d" + p)
    return names


def oracle_outputs(src, workdir):
    from oracle.oracle import OracleRun
    from tensor_logic_lang_b200 import lang
    cwd = os.getcwd()
    os.chdir(workdir)                     # `save` writes relative paths
    try:
        p = lang.Program(src)
        r = OracleRun(p)
        assert r.status == 0, r.status
        tensors = {}
        for nm in defined_tensors(p):
            if r.has(nm):
                a = r.tensor(nm)
                tensors[nm] = {"shape": list(a.shape), "values": a.ravel().tolist()}
        return tensors, r.queries, r.sweeps
    finally:
        os.chdir(cwd)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    out = []
    for name in EXAMPLES:
        rel = f"examples/{name}.tl"
        with open(os.path.join(ref, rel)) as f:
            src = f.read()
        t, q, sweeps, files = expected(name)
        with tempfile.TemporaryDirectory() as d:
            tensors, queries, osw = oracle_outputs(src, d)
        case = {"name": name, "source": rel, "src": src,
                "expect": {k: {"shape": list(np.shape(v)), "values": np.ravel(v).tolist()} for k, v in t.items()},
                "expect_queries": q,
                "oracle": {"tensors": tensors, "queries": queries, "sweeps": osw}}
        if sweeps is not None:
            case["expect_sweeps"] = sweeps
        if files:
            case["expect_files"] = {k: np.ravel(v).tolist() for k, v in files.items()}
        out.append(case)
    with open(os.path.join(HERE, "reference_examples.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", len(out), "examples")


if __name__ == "__main__":
    main()
