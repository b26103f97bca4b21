"""Programs with constant-index queries and their known answers.

The reference compiles a query with a constant index into a memoised
recursive function per queried tensor (src/codegen/backward.zig).  Each
answer below was traced by hand through that function's rules:

  * the function marks its element computed with value 0, then evaluates the
    tensor's equations in program order, folding each into the result with
    the equation's operator (`=` replaces, `+=` adds, `max=`/`min=` compare,
    `*=` multiplies) and storing the running result in the memo;
  * a contracted index sums the whole right-hand side per term, so a
    nonlinearity applies to each term before the sum (`step` per path);
  * a reference to a queried tensor is a recursive call, which returns the
    memo at once for an element already computed or still in progress;
  * any other tensor reads the global allocated before `main`; a `sparse`
    declaration re-allocates its tensor in `main`, so the recursion keeps
    reading the zeros of the global (llvm.zig:231-260, 482-516);
  * binary operators other than + - * / evaluate as + (backward.zig:404-410).
"""

# A chain 0 -> 1 -> 2 -> 3; `Parent[9,9] = 0` sizes Parent 10x10 so that
# every read stays inside the tensor.
CHAIN = """
Parent[0,1] = 1
Parent[1,2] = 1
Parent[2,3] = 1
Parent[9,9] = 0
Ancestor[x,y] = step(Parent[x,y])
Ancestor[x,z] max= step(Parent[x,y] Ancestor[y,z])
Ancestor[0,3]?
Ancestor[3,0]?
Ancestor[1,3]?
"""
CHAIN_OUT = "Ancestor = 1\nAncestor = 0\nAncestor = 1\n"

# Two paths 0 -> 1 -> 3 and 0 -> 2 -> 3: step applies per term, so the
# contracted sum counts both.
DIAMOND = """
Parent[0,1] = 1
Parent[0,2] = 1
Parent[1,3] = 1
Parent[2,3] = 1
Parent[9,9] = 0
Ancestor[x,y] = step(Parent[x,y])
Ancestor[x,z] max= step(Parent[x,y] Ancestor[y,z])
Ancestor[0,3]?
Ancestor[0,1]?
"""
DIAMOND_OUT = "Ancestor = 2\nAncestor = 1\n"

# The relation is declared `sparse` before its facts: the recursion reads the
# global, which stays zero.
SPARSE_DECL = """
domain n: 6
sparse Link[n, n]
Link[0,1] = 1
Link[1,2] = 1
Link[2,3] = 1
Reach[x,y] = step(Link[x,y])
Reach[x,z] max= step(Link[x,y] Reach[y,z])
Reach[0,3]?
Reach[0,1]?
"""
SPARSE_DECL_OUT = "Reach = 0\nReach = 0\n"

# Accumulation operators, two contracted indices and a comparison.
ACCUM = """
domain i: 3
domain j: 3
domain k: 3
A[0] = 2
A[1] = -1
A[2] = 0.5
S[i] = A[i]
S[i] += 10
S[i] max= 3
M[i] = A[i]
M[i] min= 0
P[i] = A[i]
P[i] *= 4
T[i] = A[j] A[k]
G[i] = A[i] > 0
S[0]?
S[1]?
M[0]?
M[1]?
P[0]?
T[0]?
G[1]?
"""
ACCUM_OUT = "S = 12\nS = 9\nM = 0\nM = -1\nP = 8\nT = 2.25\nG = -1\n"

# A cycle 0 <-> 1 and the path 1 -> 2 -> 3.  Asking (1, 3) first computes
# (0, 3) while (1, 3) is still in progress with memo 0, so (0, 3) is memoised
# as 0 and the later query returns it; asked the other way round both are 1.
CYCLE = """
domain x: 4
domain y: 4
domain z: 4
E[0,1] = 1
E[1,0] = 1
E[1,2] = 1
E[2,3] = 1
E[3,3] = 0
R[x,y] = step(E[x,y])
R[x,z] max= step(E[x,y] R[y,z])
"""
CYCLE_LATE = CYCLE + "R[1,3]?\nR[0,3]?\n"
CYCLE_LATE_OUT = "R = 1\nR = 0\n"
CYCLE_EARLY = CYCLE + "R[0,3]?\nR[1,3]?\n"
CYCLE_EARLY_OUT = "R = 1\nR = 1\n"

KNOWN = [
    ("chain", CHAIN, CHAIN_OUT),
    ("cycle_late", CYCLE_LATE, CYCLE_LATE_OUT),
    ("cycle_early", CYCLE_EARLY, CYCLE_EARLY_OUT),
    ("diamond", DIAMOND, DIAMOND_OUT),
    ("sparse_decl", SPARSE_DECL, SPARSE_DECL_OUT),
    ("accum", ACCUM, ACCUM_OUT),
]

# Forward and backward queries interleave in statement order.
MIXED = """
domain x: 4
domain y: 4
domain z: 4
E[0,1] = 1
E[1,2] = 1
E[3,3] = 0
R[x,y] = step(E[x,y])
R[x,z] max= step(R[x,y] E[y,z])
R?
R[0,2]?
E?
R[2,0]?
"""

# Out-of-range constant: the memo offset falls outside the table (undefined
# in the reference); this implementation returns 0.0 without evaluating.
OUT_OF_RANGE = CHAIN.replace("Ancestor[1,3]?", "Ancestor[20,3]?\nAncestor[1,3]?")

NO_EQUATION = """
domain i: 3
A[0] = 1
Q[2]?
"""


def graph_program(n, edges, queries, form="right"):
    """A reachability program over `n` nodes with edge facts and constant queries."""
    lines = [f"domain x: {n}", f"domain y: {n}", f"domain z: {n}"]
    lines += [f"E[{a},{b}] = 1" for a, b in edges]
    lines.append(f"E[{n - 1},{n - 1}] = 0")
    lines.append("R[x,y] = step(E[x,y])")
    if form == "right":
        lines.append("R[x,z] max= step(E[x,y] R[y,z])")
    else:
        lines.append("R[x,z] max= step(R[x,y] E[y,z])")
    lines += [f"R[{a},{b}]?" for a, b in queries]
    return "\n".join(lines) + "\n"


def random_graph(n, m, n_queries, seed, cyclic):
    import numpy as np
    rng = np.random.default_rng(seed)
    edges = set()
    while len(edges) < m:
        a, b = (int(v) for v in rng.integers(0, n, 2))
        if a == b:
            continue
        if not cyclic and a > b:
            a, b = b, a
        edges.add((a, b))
    queries = [tuple(int(v) for v in rng.integers(0, n, 2)) for _ in range(n_queries)]
    return sorted(edges), queries


def float_program(n, seed):
    """Real-valued equations over loaded inputs: nonlinearities per term."""
    import numpy as np
    rng = np.random.default_rng(seed)
    W = rng.standard_normal((n, n)) * 0.5
    X = rng.standard_normal(n)
    src = (f"domain i: {n}\ndomain j: {n}\n"
           "W[i,j] = 0\nload W \"W.bin\"\nX[i] = 0\nload X \"X.bin\"\n"
           "Y[i] = sigmoid(W[i,j] X[j])\n"
           "Y[i] += tanh(X[i]) * 0.5\n"
           "Z[i] = Y[j] W[j,i] - exp(X[i]) / 4\n"
           "Z[i] max= relu(X[i])\n"
           "Y[0]?\nY[3]?\nZ[1]?\nZ[2]?\n")
    return src, {"W": W, "X": X}
