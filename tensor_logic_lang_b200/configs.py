"""The benchmark configurations as Tensor Logic programs.

Each program declares a domain for every index letter it uses (an undeclared
index silently gets size 10 in the reference, src/codegen/llvm.zig:407,435),
writes softmax over a bare tensor reference (src/codegen/softmax.zig:23-27),
and defines its inputs as zero tensors followed by `load` (the harness feeds
the values; the reference's `load` path is broken by quoted paths,
src/codegen/llvm.zig:585-586).  Sizes are parameters so the parity tests can
run the same programs at sizes the f64 oracle finishes in seconds.
"""
import numpy as np

from . import inputs as gen
from .lang import Program

SEED = 0


def mlp_forward(b=32, i=784, h=256, o=10, seed=SEED):
    """C0: H = relu(X W1) per term, Z2 = H W2, Y = softmax(Z2)."""
    src = f"""
domain b: {b}
domain i: {i}
domain h: {h}
domain o: {o}
X[b,i] = 0
load X "x.bin"
W1[i,h] = 0
load W1 "w1.bin"
W2[h,o] = 0
load W2 "w2.bin"
H[b,h] = relu(X[b,i] W1[i,h])
Z2[b,o] = H[b,h] W2[h,o]
Y[b,o.] = softmax(Z2[b,o])
"""
    data = {
        "X": gen.uniform(seed, "C0.X", (b, i)),
        "W1": gen.normal(seed, "C0.W1", (i, h), np.sqrt(2.0 / i)),
        "W2": gen.normal(seed, "C0.W2", (h, o), np.sqrt(2.0 / h)),
    }
    flops = 2 * b * h * i + 2 * b * o * h
    return src, data, {}, flops


def attention(s=2048, d=64, seed=SEED):
    """C1: Scores = Q K^T / 8, Attn = softmax over k, Out = Attn V."""
    src = f"""
domain q: {s}
domain k: {s}
domain d: {d}
Q[q,d] = 0
load Q "q.bin"
K[k,d] = 0
load K "k.bin"
V[k,d] = 0
load V "v.bin"
Scores[q,k] = Q[q,d] K[k,d] / 8.0
Attn[q,k.] = softmax(Scores[q,k])
Out[q,d] = Attn[q,k] V[k,d]
"""
    data = {n: gen.normal(seed, f"C1.{n}", (s, d)) for n in ("Q", "K", "V")}
    flops = 2 * (2 * s * s * d)
    return src, data, {}, flops


def mlp_train(b=1024, i=784, h=4096, o=10, seed=SEED):
    """C2: split-form MLP forward, squared-error loss, backward L wrt W1, W2."""
    src = f"""
domain b: {b}
domain i: {i}
domain h: {h}
domain o: {o}
X[b,i] = 0
load X "x.bin"
W1[i,h] = 0
load W1 "w1.bin"
W2[h,o] = 0
load W2 "w2.bin"
Target[b,o] = 0
load Target "t.bin"
Z1[b,h] = X[b,i] W1[i,h]
H[b,h] = relu(Z1[b,h])
Z2[b,o] = H[b,h] W2[h,o]
Y[b,o.] = softmax(Z2[b,o])
Diff[b,o] = Y[b,o] - Target[b,o]
L = Diff[b,o] Diff[b,o]
backward L wrt W1, W2
"""
    data = {
        "X": gen.uniform(seed, "C2.X", (b, i)),
        "W1": gen.normal(seed, "C2.W1", (i, h), np.sqrt(2.0 / i)),
        "W2": gen.normal(seed, "C2.W2", (h, o), np.sqrt(2.0 / h)),
        "Target": gen.labels_onehot(seed, "C2.T", b, o),
    }
    fwd = 2 * b * i * h + 2 * b * h * o
    bwd = 2 * i * b * h + 2 * b * o * h + 2 * h * b * o
    return src, data, {}, fwd + bwd


def gnn(n=16384, f=256, degree=16, seed=SEED):
    """C3: two per-term relu message-passing layers over a sparse ER graph."""
    src = f"""
domain v: {n}
domain u: {n}
domain f: {f}
domain g: {f}
sparse Adj[v, u]
H0[u,g] = 0
load H0 "h0.bin"
W1[g,f] = 0
load W1 "w1.bin"
W2[g,f] = 0
load W2 "w2.bin"
H1[v,f] = relu(Adj[v,u] H0[u,g] W1[g,f])
H2[v,f] = relu(Adj[v,u] H1[u,g] W2[g,f])
"""
    rows, cols = gen.er_graph(n, degree, seed + 3)
    data = {
        "H0": gen.normal(seed, "C3.H0", (n, f)),
        "W1": gen.normal(seed, "C3.W1", (f, f), np.sqrt(2.0 / f)),
        "W2": gen.normal(seed, "C3.W2", (f, f), np.sqrt(2.0 / f)),
    }
    nnz = len(rows)
    flops = 2 * (2 * n * f * f + 2 * nnz * f)
    return src, data, {"Adj": (rows, cols, None)}, flops


def closure(n=32768, degree=4, seed=SEED):
    """C4: Reach = step(Edge); Reach max= step(Reach Edge) to the fixpoint."""
    src = f"""
domain x: {n}
domain y: {n}
domain z: {n}
sparse Edge[x, y]
Reach[x,y] = step(Edge[x,y])
Reach[x,z] max= step(Reach[x,y] Edge[y,z])
"""
    rows, cols = gen.random_dag(n, degree, seed + 4)
    return src, {}, {"Edge": (rows, cols, None)}, 0


def rowwise(rows=65536, cols=1024, op="softmax", seed=SEED):
    """Row-wise softmax or layer norm over the last axis of an r x c matrix
    (src/codegen/softmax.zig:19-229, src/codegen/layernorm.zig:25-310); sized
    well past L2 so the kernel streams from HBM.  The last element is the
    algorithmic bytes (one read and one write of every element), not flops."""
    src = f"""
domain r: {rows}
domain c: {cols}
X[r,c] = 0
load X "x.bin"
Y[r,c.] = {op}(X[r,c])
"""
    data = {"X": gen.normal(seed, f"R.{op}.X", (rows, cols))}
    return src, data, {}, 8 * rows * cols


def program(builder, **kw):
    src, data, sparse, flops = builder(**kw)
    return Program(src, inputs=data, sparse_inputs=sparse), data, sparse, flops
