"""Derive the known-answer fixtures in known_answers.json.

The reference ships no numeric tests or golden vectors for its codegen
(tests/integration_test.zig:12-23 only checks exit codes), so each fixture is
a small program written for this repository together with its answer derived
here from the reference's documented semantics with plain numpy, independent
of the oracle:

  * implicit products sum over contracted indices (einsum.zig:20-196);
  * an index letter without a `domain` has size 10 (llvm.zig:407,435);
  * a nonlinearity around a product applies per term (expr.zig:240-300);
  * softmax is exp(x)/sum exp(x) on the `.` axis (softmax.zig:128-211);
  * lnorm is (x - mean)/sqrt(biased var + 1e-5) (layernorm.zig:134-292);
  * avg= divides by the product of the LHS divisors (einsum.zig:151-195);
  * max= step recursion reaches the transitive closure (fixpoint.zig:46-98);
    the sweep counts follow from the in-place loop order;
  * backward: `L = D D` gives dD = 2 D, explicit `*` gives no gradient,
    softmax's gradient uses one sum over the whole tensor (autodiff.zig).

Run: python tests/golden/make_known_answers.py  (rewrites the JSON).
"""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def lit(name, arr):
    lines = []
    arr = np.asarray(arr, dtype=float)
    for idx in np.ndindex(arr.shape):
        if arr[idx] != 0.0:
            lines.append(f"{name}[{','.join(map(str, idx))}] = {float(arr[idx])!r}")
    return "\n".join(lines)


def softmax_rows(z):
    e = np.exp(z)
    return e / e.sum(axis=-1, keepdims=True)


def cases():
    out = []
    rng = np.random.default_rng(7)

    # 1. matmul with declared domains
    A = np.arange(1.0, 13.0).reshape(3, 4)
    B = np.array([[1.0, -2.0], [0.5, 3.0], [-1.0, 0.0], [2.0, 1.0]])
    src = "domain i: 3\ndomain j: 4\ndomain k: 2\nA[i,j] = 0\nB[j,k] = 0\n" + lit("A", A) + "\n" + lit("B", B) + \
        "\nC[i,k] = A[i,j] B[j,k]\nC?\n"
    out.append(dict(name="matmul", src=src, expect={"C": (A @ B).tolist()}))

    # 2. undeclared index letters default to 10: C is 10 x 10, the product sits top-left
    src = "domain I: 3\ndomain J: 4\ndomain K: 2\nA[i,j] = 0\nB[j,k] = 0\n" + lit("A", A) + "\n" + lit("B", B) + \
        "\nC[i,k] = A[i,j] B[j,k]\n"
    C10 = np.zeros((10, 10))
    C10[:3, :2] = A @ B
    out.append(dict(name="undeclared_domain_10", src=src, expect={"C": C10.tolist()}))

    # 3. per-term relu: sum_i relu(X[b,i] W[i,h]), not relu of the sum
    X = np.array([[1.0, -2.0, 0.5], [-1.0, 1.5, 2.0]])
    W = np.array([[0.5, -1.0], [1.0, 2.0], [-2.0, 0.25]])
    H = np.maximum(X[:, :, None] * W[None, :, :], 0.0).sum(axis=1)
    src = "domain b: 2\ndomain i: 3\ndomain h: 2\nX[b,i] = 0\nW[i,h] = 0\n" + lit("X", X) + "\n" + lit("W", W) + \
        "\nH[b,h] = relu(X[b,i] W[i,h])\n"
    out.append(dict(name="relu_per_term", src=src, expect={"H": H.tolist()}))

    # 4. softmax on the last axis and on a marked first axis
    Z = np.array([[0.1, 2.0, -1.0, 0.5], [1.0, 1.0, 1.0, 1.0], [-3.0, 0.0, 3.0, 0.25]])
    src = "domain r: 3\ndomain c: 4\nZ[r,c] = 0\n" + lit("Z", Z) + \
        "\nY[r,c.] = softmax(Z[r,c])\nYc[r.,c] = softmax(Z[r,c])\n"
    out.append(dict(name="softmax_axes", src=src,
                    expect={"Y": softmax_rows(Z).tolist(), "Yc": softmax_rows(Z.T).T.tolist()}))

    # 5. layer norm
    Xl = rng.normal(size=(4, 6)).round(3)
    mu = Xl.mean(axis=1, keepdims=True)
    var = ((Xl - mu) ** 2).mean(axis=1, keepdims=True)
    src = "domain r: 4\ndomain c: 6\nX[r,c] = 0\n" + lit("X", Xl) + "\nN[r,c.] = lnorm(X[r,c])\n"
    out.append(dict(name="lnorm", src=src, expect={"N": ((Xl - mu) / np.sqrt(var + 1e-5)).tolist()}))

    # 6. avg pooling over i/2
    x = np.array([1.0, 3.0, 2.0, 6.0, -1.0, 5.0, 4.0, 0.0])
    src = "domain i: 8\nX[i] = 0\n" + lit("X", x) + "\nP[i/2] avg= X[i]\n"
    out.append(dict(name="avg_pool", src=src, expect={"P": (x.reshape(4, 2).sum(axis=1) / 2.0).tolist()}))

    # 7. chain closure, left form (R[x] reads later rows): n-1 edges → n-1 sweeps
    n = 7
    E = np.zeros((n, n))
    for a in range(n - 1):
        E[a, a + 1] = 1.0
    reach = np.triu(np.ones((n, n)), 1)
    src = f"domain p: {n}\ndomain x: {n}\ndomain y: {n}\ndomain z: {n}\nsparse Par[p, p]\n" + lit("Par", E) + \
        "\nAnc[x,y] = step(Par[x,y])\nAnc[x,y] max= step(Par[x,z] Anc[z,y])\n"
    out.append(dict(name="closure_left_chain", src=src, expect={"Anc": reach.tolist()}, sweeps=n - 1))

    # 8. chain closure, right form (z ascending in place): closes in 1 sweep + 1 check
    src = f"domain p: {n}\ndomain x: {n}\ndomain y: {n}\ndomain z: {n}\nsparse Par[p, p]\n" + lit("Par", E) + \
        "\nR[x,y] = step(Par[x,y])\nR[x,z] max= step(R[x,y] Par[y,z])\n"
    out.append(dict(name="closure_right_chain", src=src, expect={"R": reach.tolist()}, sweeps=2))

    # 9. sigmoid with temperature, elementwise
    S = np.array([[2.0, -1.0], [0.0, 0.7]])
    src = "domain i: 2\ndomain j: 2\nS[i,j] = 0\n" + lit("S", S) + \
        "\nA[i,j] = sigmoid(S[i,j], 0.5)\nB[i,j] = tanh(S[i,j])\n"
    out.append(dict(name="sigmoid_temperature", src=src,
                    expect={"A": (1 / (1 + np.exp(-S / 0.5))).tolist(), "B": np.tanh(S).tolist()}))

    # 10. backward: explicit `*` has no gradient; implicit product L = D D gives 2 D
    Xn = np.array([[1.0, 0.5], [0.3, 0.8]])
    Wt = np.array([[0.5], [-0.25]])
    T = np.array([[1.0], [0.0]])
    base = "domain n: 2\ndomain f: 2\ndomain o: 1\nX[n,f] = 0\nW[f,o] = 0\nT[n,o] = 0\n" + lit("X", Xn) + "\n" + \
        lit("W", Wt) + "\n" + lit("T", T) + "\nY[n,o] = X[n,f] W[f,o]\nD[n,o] = Y[n,o] - T[n,o]\n"
    src = base + "L[n,o] = D[n,o] * D[n,o]\nbackward L wrt W\n"
    out.append(dict(name="backward_explicit_mul", src=src, expect={"dL_dW": np.zeros((2, 1)).tolist()}))
    D = Xn @ Wt - T
    dD = 2 * D
    dW = Xn.T @ dD
    src = base + "L = D[n,o] D[n,o]\nbackward L wrt W\n"
    out.append(dict(name="backward_implicit_square", src=src,
                    expect={"dL_dW": dW.tolist(), "L": [float((D * D).sum())]}))

    # 11. softmax gradient sums over the whole tensor
    Zs = np.array([[0.2, -0.4, 1.0], [0.5, 0.1, -0.3]])
    Tg = np.array([[0.0, 1.0, 0.0], [1.0, 0.0, 0.0]])
    Ws = np.array([[1.0, 0.0, 0.5], [0.0, 1.0, -0.5], [0.25, 0.25, 1.0]])
    src = "domain b: 2\ndomain h: 3\ndomain o: 3\nZ[b,h] = 0\nW[h,o] = 0\nT[b,o] = 0\n" + lit("Z", Zs) + "\n" + \
        lit("W", Ws) + "\n" + lit("T", Tg) + \
        "\nZ2[b,o] = Z[b,h] W[h,o]\nY[b,o.] = softmax(Z2[b,o])\nD[b,o] = Y[b,o] - T[b,o]\nL = D[b,o] D[b,o]\n" \
        "backward L wrt W\n"
    Z2 = Zs @ Ws
    Y = softmax_rows(Z2)
    dY = 2 * (Y - Tg)
    s = (dY * Y).sum()
    dZ2 = Y * (dY - s)
    out.append(dict(name="backward_softmax_global_sum", src=src, expect={"dL_dW": (Zs.T @ dZ2).tolist()}))
    return out


if __name__ == "__main__":
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(cases(), f, indent=1)
    print("wrote", len(cases()), "cases")
