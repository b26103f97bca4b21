"""Each kernel family against the f64 oracle on seeded inputs, incl. tails and odd shapes."""
import numpy as np
import pytest

from tensor_logic_lang_b200 import inputs as gen
from tensor_logic_lang_b200 import lang

from gpu_helpers import TOL_FP32, TOL_TF32, assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx(gpu_ctx_factory):
    c = gpu_ctx_factory()
    yield c
    c.close()


def both(ctx, oracle_lib, src, data=None, sparse=None):
    p = lang.Program(src, inputs=data, sparse_inputs=sparse)
    ctx.run(p)
    return oracle_lib.OracleRun(p)


def decl(**dom):
    return "".join(f"domain {k}: {v}\n" for k, v in dom.items())


def inputs_src(names):
    return "".join(f"{n}[{','.join(ix)}] = 0\nload {n} \"{n}.bin\"\n" for n, ix in names)


# ----------------------------------------------------------------------------- GEMM
GEMM_CASES = [
    # (M, N, K, A index order, B index order, LHS order, extra)
    (300, 200, 100, "mk", "kn", "mn", ""),          # SIMT, tails
    (1024, 512, 784, "mk", "kn", "mn", ""),         # tcgen05: A K-major, B MN-major
    (1024, 512, 784, "mk", "nk", "mn", ""),         # tcgen05: both K-major
    (784, 1024, 512, "km", "kn", "mn", ""),         # tcgen05: both MN-major (dW-style)
    (512, 1024, 256, "km", "nk", "nm", ""),         # transposed output
    (1000, 600, 300, "mk", "kn", "mn", ""),         # tails in M, N, K
    (1024, 768, 200, "mk", "kn", "mn", "relu"),     # per-term relu: sign split
    (512, 512, 128, "mk", "kn", "mn", "scale"),     # literal scale
    (512, 512, 130, "mk", "kn", "mn", "accum"),     # += into existing values, K not /4
    (2048, 64, 2048, "mk", "kn", "mn", ""),         # N = 64 tile, long K
    (1024, 10, 4096, "mk", "kn", "mn", ""),         # skinny N, A k-contiguous, split K
    (4096, 10, 1024, "km", "kn", "mn", ""),         # skinny N, A row-contiguous (weight gradient)
    (1000, 13, 777, "mk", "nk", "mn", "accum"),     # skinny N, unaligned rows, strided B, +=
    (512, 16, 300, "km", "nk", "nm", "scale"),      # skinny N, transposed output, scale
    (1024, 4096, 10, "mk", "nk", "mn", ""),         # thin K (input gradient of a 10-wide layer)
    (1000, 1000, 7, "mk", "kn", "mn", "accum"),     # thin K, tails, +=
]


@pytest.mark.parametrize("case", GEMM_CASES, ids=[f"{c[0]}x{c[1]}x{c[2]}-{c[3]}{c[4]}{c[5]}-{c[6]}" for c in GEMM_CASES])
def test_gemm(ctx, oracle_lib, case):
    M, N, K, ao, bo, lo, extra = case
    size = dict(m=M, n=N, k=K)
    A = gen.normal(1, "A", tuple(size[c] for c in ao))
    B = gen.normal(1, "B", tuple(size[c] for c in bo))
    a = f"A[{ao[0]},{ao[1]}]"
    b = f"B[{bo[0]},{bo[1]}]"
    rhs = f"{a} {b}"
    if extra == "relu":
        rhs = f"relu({a} {b})"
    if extra == "scale":
        rhs = f"{a} {b} / 8.0"
    src = decl(m=M, n=N, k=K) + inputs_src([("A", ao), ("B", bo)])
    if extra == "accum":
        C0 = gen.normal(2, "C0", (M, N))
        src += inputs_src([("C", "mn")]) + f"C[m,n] += {rhs}\n"
        data = dict(A=A, B=B, C=C0)
        out = "C"
    else:
        src += f"C[{lo[0]},{lo[1]}] = {rhs}\n"
        data = dict(A=A, B=B)
        out = "C"
    p = lang.Program(src, inputs=data)
    ctx.run(p)
    got = ctx.tensor(out)
    # reference values from the oracle's reference-order f64 loop
    Am = A if ao == "mk" else A.T
    Bm = B if bo == "kn" else B.T
    want = oracle_lib.gemm(Am, Bm, C_init=data.get("C"), relu_per_term=(extra == "relu"),
                           scale=0.125 if extra == "scale" else 1.0)
    if lo == "nm":
        want = want.T
    tol = TOL_TF32 if M * N * K >= (1 << 25) else TOL_FP32
    assert_close(got, want, tol, "C")


MN_CASES = [c for c in GEMM_CASES if "km" in (c[3],) or c[4] == "kn"]


@pytest.mark.parametrize("case", MN_CASES, ids=[f"{c[0]}x{c[1]}x{c[2]}-{c[3]}{c[4]}{c[5]}-{c[6]}" for c in MN_CASES])
def test_gemm_mn_major_descriptors(ctx, oracle_lib, case, monkeypatch):
    """The same GEMMs with MN-major operands read by the tensor cores directly
    (128-byte swizzle with 32-byte atoms) instead of through a transposing copy."""
    monkeypatch.setenv("TL_GEMM_MN", "1")
    test_gemm(ctx, oracle_lib, case)


STORE_CASES = [c for c in GEMM_CASES if c[0] * c[1] * c[2] >= (1 << 25) and c[1] >= 64]


@pytest.mark.parametrize("case", STORE_CASES, ids=[f"{c[0]}x{c[1]}x{c[2]}-{c[3]}{c[4]}{c[5]}-{c[6]}" for c in STORE_CASES])
def test_gemm_plain_store_epilogue(ctx, oracle_lib, case, monkeypatch):
    """The tensor-core GEMMs with the epilogue's per-thread stores instead of
    TMA stores (the path for unaligned or strided outputs)."""
    monkeypatch.setenv("TL_GEMM_NO_TMA_STORE", "1")
    test_gemm(ctx, oracle_lib, case)


# ----------------------------------------------------------------------------- row-wise
# (6, 2052) .. (3, 8192): rows held in a block's registers; (2, 8196): the
# multi-pass block path
ROW_CASES = [(3, 10), (2048, 2048), (64, 1000), (5, 5000), (1024, 10), (7, 129), (6, 2052), (9, 4096),
             (3, 8192), (2, 8196)]


@pytest.mark.parametrize("rows,cols", ROW_CASES)
@pytest.mark.parametrize("op", ["softmax", "lnorm"])
def test_rowwise(ctx, oracle_lib, rows, cols, op):
    X = gen.normal(3, "X", (rows, cols), 2.0)
    src = decl(r=rows, c=cols) + inputs_src([("X", "rc")]) + f"Y[r,c.] = {op}(X[r,c])\nYt[r.,c] = {op}(X[r,c])\n"
    ref = both(ctx, oracle_lib, src, dict(X=X))
    assert_close(ctx.tensor("Y"), ref.tensor("Y"), TOL_FP32 * 10, "Y")
    assert_close(ctx.tensor("Yt"), ref.tensor("Yt"), TOL_FP32 * 10, "Yt")


# ----------------------------------------------------------------------------- generic
GENERIC = [
    ("S[i] = A[i,j] B[j]", "sum"),
    ("S[i] += exp(A[i,j] B[j])", "exp per term"),
    ("S[i] max= A[i,j] B[j]", "max"),
    ("S[i] min= A[i,j] - B[j]", "min"),
    ("S[i] *= sigmoid(A[i,j])", "mul"),
    ("S[i] = tanh(A[i,j] B[j]) + abs(B[j])", "tanh+abs"),
    ("S[i] = step(A[i,j]) B[j]", "step factor"),
    ("S[i] = sqrt(abs(A[i,j])) * cos(B[j]) - sin(A[i,j])", "mixed"),
    ("S[i] = A[i,3] + A[i+1,0] - A[i-1,2]", "const and offset"),
    ("S[i] = A[i,j] > B[j]", "comparison"),
    ("S[i] = log(abs(A[i,j]) + 1.0) ^ 2", "log pow"),
    ("S[i] = -A[i,j]", "negate"),
]


@pytest.mark.parametrize("eq,what", GENERIC, ids=[g[1] for g in GENERIC])
def test_generic_einsum(ctx, oracle_lib, eq, what):
    A = gen.normal(4, "A", (37, 23))
    B = gen.normal(4, "B", (23,))
    src = decl(i=37, j=23) + inputs_src([("A", "ij"), ("B", "j")]) + "S[i] = 0\n" + eq + "\n"
    ref = both(ctx, oracle_lib, src, dict(A=A, B=B))
    assert_close(ctx.tensor("S"), ref.tensor("S"), TOL_FP32, what)


def test_avg_pool_and_scalar_assign(ctx, oracle_lib):
    X = gen.normal(5, "X", (32, 6))
    src = decl(i=32, j=6) + inputs_src([("X", "ij")]) + \
        "P[i/4, j] avg= X[i,j]\nX[3,2] = 7.5\nQ[i,j] = X[i,j] * 2.0\nT = X[i,j]\n"
    ref = both(ctx, oracle_lib, src, dict(X=X))
    for n in ("P", "Q", "T"):
        assert_close(ctx.tensor(n), ref.tensor(n), TOL_FP32, n)


# ----------------------------------------------------------------------------- fixpoint
@pytest.mark.parametrize("n,deg,seed", [(100, 3, 1), (1000, 4, 2), (4096, 4, 3), (2000, 1, 4)])
def test_closure_bits(ctx, oracle_lib, n, deg, seed):
    rows, cols = gen.random_dag(n, deg, seed)
    src = decl(x=n, y=n, z=n) + "sparse Edge[x, y]\nReach[x,y] = step(Edge[x,y])\n" \
                                "Reach[x,z] max= step(Reach[x,y] Edge[y,z])\n"
    p = lang.Program(src, sparse_inputs={"Edge": (rows, cols, None)})
    ctx.run(p)
    got = ctx.bits("Reach")
    colptr, rowidx = gen.csr_from_coo(n, cols, rows)
    W = (n + 31) // 32
    R = np.zeros((n, W), dtype=np.uint32)
    np.bitwise_or.at(R, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
    sweeps = oracle_lib.closure_right(n, colptr, rowidx, R)
    np.testing.assert_array_equal(got, R)
    assert ctx.sweeps == sweeps == 2


def test_closure_with_cycles(ctx, oracle_lib):
    n = 300
    rng = np.random.default_rng(9)
    pairs = np.unique(rng.integers(0, n, size=(900, 2)), axis=0)
    pairs = pairs[pairs[:, 0] != pairs[:, 1]]
    rows, cols = pairs[:, 0], pairs[:, 1]
    src = decl(x=n, y=n, z=n) + "sparse Edge[x, y]\nReach[x,y] = step(Edge[x,y])\n" \
                                "Reach[x,z] max= step(Reach[x,y] Edge[y,z])\n"
    ref = both(ctx, oracle_lib, src, sparse={"Edge": (rows, cols, None)})
    np.testing.assert_array_equal(ctx.tensor("Reach"), ref.tensor("Reach"))


def _closure_case(ctx, oracle_lib, n, rows, cols):
    src = decl(x=n, y=n, z=n) + "sparse Edge[x, y]\nReach[x,y] = step(Edge[x,y])\n" \
                                "Reach[x,z] max= step(Reach[x,y] Edge[y,z])\n"
    ctx.run(lang.Program(src, sparse_inputs={"Edge": (rows, cols, None)}))
    got = ctx.bits("Reach")
    colptr, rowidx = gen.csr_from_coo(n, cols, rows)
    R = np.zeros((n, (n + 31) // 32), dtype=np.uint32)
    np.bitwise_or.at(R, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
    sweeps = oracle_lib.closure_right(n, colptr, rowidx, R)
    np.testing.assert_array_equal(got, R)
    return sweeps


def test_closure_high_degree_nodes(ctx, oracle_lib):
    # nodes with more successors than the successor table holds inline
    n, rng = 3000, np.random.default_rng(21)
    pairs = set()
    for u in range(n - 1):
        d = 40 if u % 50 == 0 else int(rng.integers(0, 6))
        for v in rng.integers(u + 1, n, size=d):
            pairs.add((u, int(v)))
    pr = np.array(sorted(pairs), dtype=np.int64)
    sweeps = _closure_case(ctx, oracle_lib, n, pr[:, 0], pr[:, 1])
    assert ctx.sweeps == sweeps == 2


@pytest.mark.parametrize("mode", ["default", "teams"])
def test_closure_large_frontier(ctx, oracle_lib, monkeypatch, mode):
    # rows whose first frontier and later frontiers outgrow the queue (spill
    # set); "teams" hands rows past the lone-warp budget to whole blocks
    if mode == "teams":
        monkeypatch.setenv("TL_CLOSURE_TEAMS", "1")
    n, rng = 4096, np.random.default_rng(22)
    pairs = set()
    for u in range(8):
        for v in rng.choice(np.arange(u + 1, n), 2500, replace=False):
            pairs.add((u, int(v)))
    r2, c2 = gen.random_dag(n, 6, 23)
    pairs.update(zip(r2.tolist(), c2.tolist()))
    pr = np.array(sorted(pairs), dtype=np.int64)
    sweeps = _closure_case(ctx, oracle_lib, n, pr[:, 0], pr[:, 1])
    assert ctx.sweeps == sweeps == 2


@pytest.mark.parametrize("n", [33, 1000, 2017])
def test_closure_odd_widths_and_cycles(ctx, oracle_lib, n):
    # row widths that are not a multiple of 128 bits, with back edges
    rng = np.random.default_rng(n)
    pairs = np.unique(rng.integers(0, n, size=(3 * n, 2)), axis=0)
    pairs = pairs[pairs[:, 0] != pairs[:, 1]]
    _closure_case(ctx, oracle_lib, n, pairs[:, 0], pairs[:, 1])


def test_closure_explicit_zero_edges(ctx, oracle_lib):
    # stored 0.0 entries are not edges of step(Edge): the closure must not follow them
    n = 200
    rows, cols = gen.random_dag(n, 3, 31)
    vals = np.ones(len(rows))
    vals[::3] = 0.0
    src = decl(x=n, y=n, z=n) + "sparse Edge[x, y]\nReach[x,y] = step(Edge[x,y])\n" \
                                "Reach[x,z] max= step(Reach[x,y] Edge[y,z])\n"
    ref = both(ctx, oracle_lib, src, sparse={"Edge": (rows, cols, vals)})
    np.testing.assert_array_equal(ctx.tensor("Reach"), ref.tensor("Reach"))


@pytest.mark.parametrize("long_row", [False, True])
def test_sparse_upload_device_build(ctx, oracle_lib, long_row):
    # unsorted COO entries with repeated (row, column) pairs, the last value
    # counting; zero and negative values; long_row puts more than 32 entries in
    # one row, which sends the upload to the host build
    n, m = 600, 5000
    rng = np.random.default_rng(41)
    rows = rng.integers(0, n, m)
    cols = rng.integers(0, n, m)
    if long_row:
        rows[:200] = 7
    rows = np.concatenate([rows, rows[:300]])
    cols = np.concatenate([cols, cols[:300]])
    vals = rng.normal(size=len(rows))
    vals[::17] = 0.0
    src = decl(i=n, j=n) + "sparse A[i, j]\nB[i,j] = A[i,j]\n"
    ref = both(ctx, oracle_lib, src, sparse={"A": (rows, cols, vals)})
    D = np.zeros((n, n))
    for r, c, v in zip(rows, cols, vals):
        D[r, c] = v   # in input order: the last entry of a pair stays
    np.testing.assert_array_equal(ctx.tensor("B"), D.astype(np.float32).astype(np.float64))
    np.testing.assert_allclose(ref.tensor("B"), D, rtol=1e-7, atol=0)


def test_closure_one_launch_matches_per_sweep(ctx, oracle_lib, monkeypatch):
    # the one-launch fixpoint and the per-sweep launches give the same bits and sweeps
    n = 2048
    rows, cols = gen.random_dag(n, 5, 24)
    src = decl(x=n, y=n, z=n) + "sparse Edge[x, y]\nReach[x,y] = step(Edge[x,y])\n" \
                                "Reach[x,z] max= step(Reach[x,y] Edge[y,z])\n"
    p = lang.Program(src, sparse_inputs={"Edge": (rows, cols, None)})
    ctx.run(p)
    one, s1 = ctx.bits("Reach"), ctx.sweeps
    monkeypatch.setenv("TL_CLOSURE_PER_SWEEP", "1")
    ctx.run(p)
    np.testing.assert_array_equal(ctx.bits("Reach"), one)
    assert ctx.sweeps == s1 == 2


def test_generic_recursive_dense(ctx, oracle_lib):
    # a dense relation takes the generic recursive kernel: same fixpoint
    n = 40
    E = np.zeros((n, n))
    rng = np.random.default_rng(5)
    for u in range(n):
        for v in rng.choice(n, 2, replace=False):
            if u < v:
                E[u, v] = 1.0
    src = decl(x=n, y=n, z=n) + inputs_src([("E", "xy")]) + \
        "R[x,y] = step(E[x,y])\nR[x,z] max= step(R[x,y] E[y,z])\n"
    ref = both(ctx, oracle_lib, src, dict(E=E))
    np.testing.assert_array_equal(ctx.tensor("R"), ref.tensor("R"))


# ----------------------------------------------------------------------------- attention block
ATTN_CASES = [
    # (queries, keys, d, scores expression, note).  The scores keep the 1/sqrt(d)
    # scale: unscaled N(0, 1) inputs give scores of deviation 8, where the TF32
    # rounding of Q and K alone moves the softmax past the 1e-3 tolerance (in
    # the tiled pipeline and one equation at a time alike)
    (256, 384, 64, "Q[q,d] K[k,d] / 8.0", "the tiled pipeline"),
    (128, 128, 64, "Q[q,d] K[k,d] * 0.125", "one tile, a multiplied scale"),
    (384, 256, 64, "K[k,d] Q[q,d] / 8.0", "operands swapped"),
    (200, 256, 64, "Q[q,d] K[k,d] / 8.0", "queries not a multiple of 128: one by one"),
    (256, 256, 32, "Q[q,d] K[k,d] / 8.0", "d = 32: one by one"),
]


@pytest.mark.parametrize("nq,nk,d,expr,note", ATTN_CASES)
def test_attention_block(ctx, oracle_lib, nq, nk, d, expr, note):
    Q = gen.normal(11, "Q", (nq, d))
    K = gen.normal(12, "K", (nk, d))
    V = gen.normal(13, "V", (nk, d))
    src = decl(q=nq, k=nk, d=d) + inputs_src([("Q", "qd"), ("K", "kd"), ("V", "kd")]) + \
        f"S[q,k] = {expr}\nA[q,k.] = softmax(S[q,k])\nO[q,d] = A[q,k] V[k,d]\n"
    ref = both(ctx, oracle_lib, src, dict(Q=Q, K=K, V=V))
    for n in ("S", "A", "O"):
        assert_close(ctx.tensor(n), ref.tensor(n), TOL_TF32, f"{n} ({note})")


def test_attention_block_matches_one_by_one(ctx, monkeypatch):
    # the tiled pipeline and the three equations run one by one agree; a
    # second run of the same program (outputs no longer fresh) too
    nq, nk, d = 256, 512, 64
    data = dict(Q=gen.normal(21, "Q", (nq, d)), K=gen.normal(22, "K", (nk, d)), V=gen.normal(23, "V", (nk, d)))
    src = decl(q=nq, k=nk, d=d) + inputs_src([("Q", "qd"), ("K", "kd"), ("V", "kd")]) + \
        "Scores[q,k] = Q[q,d] K[k,d] / 8.0\nAttn[q,k.] = softmax(Scores[q,k])\nOut[q,d] = Attn[q,k] V[k,d]\n"
    p = lang.Program(src, inputs=data)
    ctx.run(p)
    fused = {n: ctx.tensor(n) for n in ("Scores", "Attn", "Out")}
    ctx.run(p)
    for n in fused:
        np.testing.assert_allclose(ctx.tensor(n), fused[n], rtol=0, atol=0)
    monkeypatch.setenv("TL_NO_FUSED_ATTENTION", "1")
    ctx.run(p)
    for n in fused:
        assert_close(fused[n], ctx.tensor(n), TOL_TF32, n)


def test_attention_block_accumulating_scores(ctx, oracle_lib):
    # S defined earlier in the run: `=` with a contraction adds into it, so
    # the block runs one equation at a time
    nq, nk, d = 128, 128, 64
    data = dict(Q=gen.normal(31, "Q", (nq, d)), K=gen.normal(32, "K", (nk, d)), V=gen.normal(33, "V", (nk, d)))
    src = decl(q=nq, k=nk, d=d) + inputs_src([("Q", "qd"), ("K", "kd"), ("V", "kd")]) + \
        "S[q,k] = 0.5\nS[q,k] = Q[q,d] K[k,d] / 8.0\nA[q,k.] = softmax(S[q,k])\nO[q,d] = A[q,k] V[k,d]\n"
    ref = both(ctx, oracle_lib, src, data)
    for n in ("S", "A", "O"):
        assert_close(ctx.tensor(n), ref.tensor(n), TOL_TF32, n)


@pytest.mark.parametrize("i", [256, 250], ids=["pairs", "k_not_mult_4"])
def test_fp32_class_gemm_hi_lo_pairs(ctx, oracle_lib, monkeypatch, i):
    # Z1's sign feeds relu's gradient, so Z1 runs as 3xTF32: hi*hi + hi*lo +
    # lo*hi.  With K a multiple of 4 a stage holds the hi and lo tiles of A and
    # B and takes the three products (TL_GEMM_NO_PAIRS=1: three concatenated
    # segments instead); both against the oracle and against each other
    from tensor_logic_lang_b200 import configs
    p, _, _, _ = configs.program(configs.mlp_train, b=256, i=i, h=1024, o=10)
    ctx.run(p)
    got = {n: ctx.tensor(n) for n in ("Z1", "dL_dW1", "dL_dW2")}
    ref = oracle_lib.OracleRun(p)
    for n in ("Z1", "dL_dW1", "dL_dW2"):
        assert_close(got[n], ref.tensor(n), TOL_TF32, n)
    monkeypatch.setenv("TL_GEMM_NO_PAIRS", "1")
    ctx.run(p)
    # both 3xTF32: fp32-class agreement on Z1
    assert_close(got["Z1"], ctx.tensor("Z1"), 1e-5, "Z1 (concatenated segments)")


HEAD_CASES = [(32, 784, 256, 10, "relu(X[b,i] W1[i,h])"), (64, 20, 100, 32, "relu(X[b,i] W1[i,h] / 4)"),
              (1, 300, 33, 1, "X[b,i] W1[i,h]"), (17, 1024, 600, 7, "relu(X[b,i] W1[i,h])")]


@pytest.mark.parametrize("b,i,h,o,first", HEAD_CASES, ids=[f"b{c[0]}-i{c[1]}-h{c[2]}-o{c[3]}" for c in HEAD_CASES])
def test_small_batch_head(ctx, oracle_lib, monkeypatch, b, i, h, o, first):
    # H = [relu per term](X W1), Z = H W2, Y = softmax(Z) at batch <= 64 runs
    # as two launches (k_head_h, k_head_zy); all three tensors against the
    # oracle, and against the statement-by-statement kernels
    src = (f"domain b: {b}\ndomain i: {i}\ndomain h: {h}\ndomain o: {o}\n"
           "X[b,i] = 0\nload X \"x.bin\"\nW1[i,h] = 0\nload W1 \"w1.bin\"\nW2[h,o] = 0\nload W2 \"w2.bin\"\n"
           f"H[b,h] = {first}\nZ[b,o] = H[b,h] W2[h,o]\nY[b,o.] = softmax(Z[b,o])\n")
    rng = np.random.default_rng(b * 7 + i)
    data = {"X": rng.uniform(-1, 1, (b, i)), "W1": rng.normal(0, np.sqrt(2 / i), (i, h)),
            "W2": rng.normal(0, np.sqrt(2 / h), (h, o))}
    p = lang.Program(src, inputs=data)
    ctx.profile(True)
    ctx.profile_reset()
    ctx.run(p)
    ctx.sync()
    assert ctx.profile_read().get("head_hidden", {}).get("launches", 0) == 1
    ctx.profile(False)
    fused = {n: ctx.tensor(n) for n in ("H", "Z", "Y")}
    ref = oracle_lib.OracleRun(p)
    for n in ("H", "Z", "Y"):
        assert_close(fused[n], ref.tensor(n), TOL_FP32, n)
    monkeypatch.setenv("TL_NO_FUSED_HEAD", "1")
    ctx.run(p)
    for n in ("H", "Z", "Y"):
        assert_close(fused[n], ctx.tensor(n), TOL_FP32, n + " (one statement at a time)")


@pytest.mark.parametrize("signs", ["x_nonneg", "w_nonneg", "mixed"])
def test_relu_per_term_with_a_nonnegative_operand(ctx, oracle_lib, signs):
    # relu(x w) per term needs both sign halves of x and w (K doubled) unless
    # one operand has no negative value: then x relu(w) or relu(x) w, one K
    # segment.  H0 >= 0 (uploaded), W1 >= 0, or neither; H1 >= 0 always (a
    # non-negative Adj times a sum of relus), so layer 2 takes the one-segment
    # form in every case.  Both layers against the oracle.
    from tensor_logic_lang_b200 import configs
    from tensor_logic_lang_b200 import inputs as gen
    from tensor_logic_lang_b200.lang import Program
    n, f = 8192, 128
    src, d, sp, _ = configs.gnn(n=n, f=f)
    d = dict(d)
    if signs == "x_nonneg":
        d["H0"] = np.abs(d["H0"])
    elif signs == "w_nonneg":
        d["W1"] = np.abs(d["W1"])
    ctx.run(Program(src, inputs=d, sparse_inputs=sp))
    rows, cols, _ = sp["Adj"]
    rowptr, colidx = gen.csr_from_coo(n, rows, cols)
    h1 = oracle_lib.gnn_layer(rowptr, colidx, d["H0"], d["W1"])
    h2 = oracle_lib.gnn_layer(rowptr, colidx, h1, d["W2"])
    assert_close(ctx.tensor_f32("H1"), h1, TOL_TF32, "H1")
    assert_close(ctx.tensor_f32("H2"), h2, TOL_TF32, "H2")


@pytest.mark.parametrize("n,f", [(16384, 256), (16384, 128), (700, 64)])
def test_spmm_tma_gathers_match_register_gathers(ctx, oracle_lib, monkeypatch, n, f):
    # the message-passing SpMM gathers rows of P by tile::gather4 copies for
    # f = 128 / 256 (TL_SPMM_REGS=1 forces the register-gather kernel).  Both
    # sum each element's terms in nonzero order, so with the same P they give
    # identical results; P's GEMM has one CTA per output tile at n = 16384
    # (no split K, whose atomic adds would reorder sums), so both runs see
    # the same P.  Both match the oracle.
    from tensor_logic_lang_b200 import configs
    from tensor_logic_lang_b200 import inputs as gen
    p, d, sp, _ = configs.program(configs.gnn, n=n, f=f)
    monkeypatch.setenv("TL_SPMM_REGS", "1")
    ctx.run(p)
    regs = (ctx.tensor_f32("H1"), ctx.tensor_f32("H2"))
    monkeypatch.delenv("TL_SPMM_REGS")
    ctx.run(p)
    tma = (ctx.tensor_f32("H1"), ctx.tensor_f32("H2"))
    if n >= 16384:
        np.testing.assert_array_equal(tma[0], regs[0])
        np.testing.assert_array_equal(tma[1], regs[1])
    rows, cols, _ = sp["Adj"]
    rowptr, colidx = gen.csr_from_coo(n, rows, cols)
    h1 = oracle_lib.gnn_layer(rowptr, colidx, d["H0"], d["W1"])
    h2 = oracle_lib.gnn_layer(rowptr, colidx, h1, d["W2"])
    for got in (regs, tma):
        assert_close(got[0], h1, TOL_TF32, "H1")
        assert_close(got[1], h2, TOL_TF32, "H2")
