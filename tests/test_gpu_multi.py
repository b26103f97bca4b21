"""Row-sharded closure and message passing on 2+ GPUs (one process per GPU,
changed word per sweep through peer memory or an NCCL all-reduce, NCCL
all-gather of the per-node transform per layer), reassembled and checked
against the f64 oracle; and the bounded waits of the sharded fixpoint when a
rank skips a run.  Skipped when the box has fewer than two GPUs."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tensor_logic_lang_b200 import abi, configs, shard
from tensor_logic_lang_b200 import inputs as gen

from gpu_helpers import TOL_TF32, assert_close

pytestmark = pytest.mark.gpu


def _world():
    return min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0


def _closure_src(n):
    return (f"domain x: {n}\ndomain y: {n}\ndomain z: {n}\nsparse Edge[x, y]\n"
            "Reach[x,y] = step(Edge[x,y])\nReach[x,z] max= step(Reach[x,y] Edge[y,z])\n")


def _graph(n, kind):
    if kind == "dag":
        _, _, sp, _ = configs.closure(n=n)
        rows, cols, _ = sp["Edge"]
        return rows, cols
    # a DAG plus back edges: cycles, rows that reach themselves
    rows, cols = gen.random_dag(n, 3, 41)
    rng = np.random.default_rng(42)
    b = rng.integers(0, n, size=(n // 50, 2))
    b = b[b[:, 0] > b[:, 1]]
    return np.concatenate([rows, b[:, 0]]), np.concatenate([cols, b[:, 1]])


def _closure_worker(rank, world, nid, n, kind, mode, q):
    os.environ["TL_CLOSURE_SHARDED"] = mode
    from tensor_logic_lang_b200 import lang
    from tensor_logic_lang_b200.runtime import Context
    ctx = Context(device=rank, rank=rank, world_size=world, nccl_id=nid, comm_timeout_ms=60000)
    try:
        # "cols": this rank keeps its slice of the columns of every row
        ctx.set_sharding("Reach", abi.SHARD_COLS if mode == "cols" else abi.SHARD_ROWS)
        rows, cols = _graph(n, kind)
        p = lang.Program(_closure_src(n), sparse_inputs={"Edge": (rows, cols, None)})
        out = []
        for _ in range(2):          # a second run: the next epoch of closed words
            ctx.run(p)
            if mode == "cols":
                out.append((ctx.bits("Reach", words=n // 32 // world), ctx.sweeps))
            else:
                out.append((ctx.bits("Reach", rows=shard.local_count(n, rank, world)), ctx.sweeps))
        q.put((rank, "closure", out))
    finally:
        ctx.close()


def _gnn_worker(rank, world, nid, n, f, mode, q):
    if mode == "nccl":
        os.environ["TL_GNN_NCCL"] = "1"
    if mode == "pushed":
        os.environ["TL_GNN_FAN"] = "push"
    from tensor_logic_lang_b200.runtime import Context
    ctx = Context(device=rank, rank=rank, world_size=world, nccl_id=nid, comm_timeout_ms=60000)
    try:
        for name in ("Adj", "H0", "H1", "H2"):
            ctx.set_sharding(name, abi.SHARD_ROWS)
        p, _, _, _ = configs.program(configs.gnn, n=n, f=f)
        ctx.run(p)
        ctx.run(p)          # a second run: the next pair of gathered buffers and tile counts
        rows = shard.local_count(n, rank, world)
        q.put((rank, "gnn", ctx.tensor("H1", rows=rows), ctx.tensor("H2", rows=rows)))
    finally:
        ctx.close()


def _run(target, world, *args):
    from tensor_logic_lang_b200.runtime import unique_id
    nid = unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, nid) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return sorted(out, key=lambda t: t[0])


CLOSURE_CASES = [(8192, "dag", "replicate"), (5000, "cyclic", "replicate"), (8192, "dag", "peer"),
                 (5000, "cyclic", "peer"), (5000, "cyclic", "local"), (4099, "dag", "bfs"),
                 (8192, "dag", "cols"), (5120, "cyclic", "cols")]


@pytest.mark.skipif(_world() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("n,kind,mode", CLOSURE_CASES, ids=[f"{c[1]}{c[0]}-{c[2]}" for c in CLOSURE_CASES])
def test_sharded_closure(oracle_lib, n, kind, mode):
    # every lazy-sweep mode of a row-sharded relation, and the column split,
    # against the oracle, bit for bit, on a DAG (2 sweeps) and on a graph
    # with cycles
    world = _world()
    out = _run(_closure_worker, world, n, kind, mode)
    rows, cols = _graph(n, kind)
    colptr, rowidx = gen.csr_from_coo(n, cols, rows)
    R = np.zeros((n, (n + 31) // 32), dtype=np.uint32)
    np.bitwise_or.at(R, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
    sweeps = oracle_lib.closure_right(n, colptr, rowidx, R)
    for run in range(2):
        if mode == "cols":
            got = np.concatenate([o[2][run][0] for o in out], axis=1)
        else:
            got = shard.assemble([o[2][run][0] for o in out], n)
        np.testing.assert_array_equal(got, R)
        got_sweeps = {o[2][run][1] for o in out}
        assert len(got_sweeps) == 1
        if kind == "dag":
            assert got_sweeps == {sweeps} == {2}
        else:
            # every row closes in its first sweep: the count can be lower than
            # the reference's in-place order needs, never higher
            assert 2 <= got_sweeps.pop() <= sweeps


GNN_CASES = [(4096, 128, "epilogue"), (16384, 256, "epilogue"), (4096, 128, "pushed"), (4096, 128, "nccl"),
             (3001, 64, "epilogue")]


@pytest.mark.skipif(_world() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("n,f,mode", GNN_CASES, ids=[f"n{c[0]}-f{c[1]}-{c[2]}" for c in GNN_CASES])
def test_sharded_gnn(oracle_lib, n, f, mode):
    # epilogue: each rank's GEMM epilogue stores its block of P into every
    # rank's gathered copy over NVLink and counts its tiles there; pushed: a
    # kernel after the GEMM does those stores; nccl: the all-gather
    # runs as an NCCL collective (n = 3001, f = 64 has shares too small for
    # the tensor-core GEMM, so it takes the NCCL path in every mode)
    world = _world()
    out = _run(_gnn_worker, world, n, f, mode)
    h1 = shard.assemble([o[2] for o in out], n)
    h2 = shard.assemble([o[3] for o in out], n)
    _, d, sp, _ = configs.gnn(n=n, f=f)
    rows, cols, _ = sp["Adj"]
    rowptr, colidx = gen.csr_from_coo(n, rows, cols)
    r1 = oracle_lib.gnn_layer(rowptr, colidx, d["H0"], d["W1"])
    r2 = oracle_lib.gnn_layer(rowptr, colidx, r1, d["W2"])
    assert_close(h1, r1, TOL_TF32, "H1")
    assert_close(h2, r2, TOL_TF32, "H2")


def _skip_worker(rank, world, nid, mode, q, done):
    # a rank that skips the second fixpoint: it stays alive, with none of its
    # kernels or collectives in flight, until rank 0 has seen its wait run out
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    # peer: the scheme whose changed words cross GPUs inside the launch (the
    # default replicated scheme needs no exchange, so nothing would wait)
    os.environ["TL_CLOSURE_SHARDED"] = "peer"
    if mode == "nccl":
        os.environ["TL_NO_PEER_FLAGS"] = "1"
    from tensor_logic_lang_b200 import abi as A
    from tensor_logic_lang_b200.runtime import Context
    ctx = Context(device=rank, rank=rank, world_size=world, nccl_id=nid, comm_timeout_ms=1000)
    try:
        ctx.set_sharding("Reach", A.SHARD_ROWS)
        p, _, _, _ = configs.program(configs.closure, n=4096)
        ctx.run(p)
        ctx.sync()
        first = ctx.sweeps
        status = A.TL_OK
        if rank == 0:
            try:
                ctx.run(p)
                ctx.sync()
            except A.TLError as e:
                status = e.status
            done.set()
        else:
            done.wait(120)
        q.put((rank, first, status))
    finally:
        ctx.close()


@pytest.mark.skipif(_world() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["peer", "nccl"])
def test_skipped_rank_ends_the_wait_with_comm_error(mode):
    # peer: the one-launch fixpoint's wait for the other rank's changed word
    # (ld.acquire.sys on its own slot array) gives up after comm_timeout_ms of
    # %globaltimer, every block returns, and tl_sync reports TL_ERR_COMM.
    # nccl: the per-sweep all-reduce's host wait gives up after
    # comm_timeout_ms, aborts the communicator and returns TL_ERR_COMM.
    from tensor_logic_lang_b200.runtime import unique_id
    nid = unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    procs = [ctx.Process(target=_skip_worker, args=(r, 2, nid, mode, q, done)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=300) for _ in range(2)])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert out[0][1] == out[1][1] == 2                  # the first run converged on both ranks
    assert out[0][2] == abi.TL_ERR_COMM and out[1][2] == abi.TL_OK


def _grow_worker(rank, world, nid, sizes, q):
    # the peer-row buffer is sized for the first relation, then grown (every
    # rank unmaps its peers' buffers, a barrier, then a new mapping)
    os.environ["TL_CLOSURE_SHARDED"] = "peer"
    from tensor_logic_lang_b200 import lang
    from tensor_logic_lang_b200.runtime import Context
    ctx = Context(device=rank, rank=rank, world_size=world, nccl_id=nid, comm_timeout_ms=60000)
    try:
        ctx.set_sharding("Reach", abi.SHARD_ROWS)
        out = []
        for n in sizes:
            rows, cols = _graph(n, "dag")
            ctx.run(lang.Program(_closure_src(n), sparse_inputs={"Edge": (rows, cols, None)}))
            out.append((ctx.bits("Reach", rows=shard.local_count(n, rank, world)), ctx.sweeps))
        q.put((rank, "grow", out))
    finally:
        ctx.close()


@pytest.mark.skipif(_world() < 2, reason="needs two GPUs")
def test_sharded_closure_peer_buffer_grows(oracle_lib):
    world, sizes = _world(), (2048, 8192)
    out = _run(_grow_worker, world, sizes)
    for k, n in enumerate(sizes):
        rows, cols = _graph(n, "dag")
        colptr, rowidx = gen.csr_from_coo(n, cols, rows)
        R = np.zeros((n, (n + 31) // 32), dtype=np.uint32)
        np.bitwise_or.at(R, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
        sweeps = oracle_lib.closure_right(n, colptr, rowidx, R)
        np.testing.assert_array_equal(shard.assemble([o[2][k][0] for o in out], n), R)
        assert all(o[2][k][1] == sweeps for o in out)
