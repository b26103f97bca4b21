"""The N > 1 path on CPU: two gloo ranks shard the closure rows cyclically,
sweep their rows with the f64 oracle and all-reduce the changed flag; the
assembled relation and the sweep count equal the single-process fixpoint."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from tensor_logic_lang_b200 import inputs as gen
from tensor_logic_lang_b200 import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _bits(n, rows, cols):
    W = (n + 31) // 32
    R = np.zeros((n, W), dtype=np.uint32)
    np.bitwise_or.at(R, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
    return R


def _worker(rank, world, port, n, rows, cols, q):
    import torch
    import torch.distributed as td
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    td.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import oracle
    colptr, rowidx = gen.csr_from_coo(n, cols, rows)
    full = _bits(n, rows, cols)
    mine = np.ascontiguousarray(full[shard.global_rows(n, rank, world)])

    def sweep_local():
        before = mine.copy()
        # one sweep of this rank's rows (rows are independent in the right form)
        for i, x in enumerate(shard.global_rows(n, rank, world)):
            row = mine[i:i + 1]
            oracle.closure_right(n, colptr, rowidx, row, 0, 1, max_sweeps=1)
        return int(not np.array_equal(before, mine))

    def allreduce_max(x):
        t = torch.tensor([x], dtype=torch.int32)
        td.all_reduce(t, op=td.ReduceOp.MAX)
        return int(t.item())

    sweeps = shard.sharded_fixpoint(sweep_local, allreduce_max)
    gathered = [None] * world
    td.all_gather_object(gathered, mine)
    if rank == 0:
        q.put((sweeps, shard.assemble(gathered, n)))
    td.destroy_process_group()


@pytest.mark.parametrize("n,world", [(300, 2)])
def test_sharded_closure_matches_single(oracle_lib, n, world):
    rows, cols = gen.random_dag(n, 3, 21)
    # add back edges so some rows need more than one sweep
    extra = np.array([[200, 10], [150, 3], [290, 120]])
    rows = np.concatenate([rows, extra[:, 0]])
    cols = np.concatenate([cols, extra[:, 1]])
    colptr, rowidx = gen.csr_from_coo(n, cols, rows)
    ref = _bits(n, rows, cols)
    ref_sweeps = oracle_lib.closure_right(n, colptr, rowidx, ref)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, rows, cols, q)) for r in range(world)]
    for p in procs:
        p.start()
    sweeps, got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    np.testing.assert_array_equal(got, ref)
    assert sweeps == ref_sweeps


def test_partition_helpers():
    n, world = 10, 3
    counts = [shard.local_count(n, r, world) for r in range(world)]
    assert counts == [4, 3, 3] and sum(counts) == n
    blocks = [np.arange(n)[shard.global_rows(n, r, world)] for r in range(world)]
    np.testing.assert_array_equal(shard.assemble(blocks, n), np.arange(n))
    per = (n + world - 1) // world
    layout = np.full(world * per, -1)
    for r in range(world):
        layout[r * per: r * per + counts[r]] = shard.global_rows(n, r, world)
    for u in range(n):
        assert layout[shard.gathered_row(u, world, per)] == u


def _parity_worker(rank, world, port, n, rows, cols, swap, col_split, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import bench
    from oracle import oracle
    bench.N_CLOSURE = n
    dist = bench.Dist(world, rank, rank)
    colptr, rowidx = gen.csr_from_coo(n, cols, rows)
    full = _bits(n, rows, cols)
    sweeps = oracle.closure_right(n, colptr, rowidx, full)
    if col_split:
        # this rank's slice of the columns of every row
        w = n // 32 // world
        mine = np.ascontiguousarray(full[:, rank * w:(rank + 1) * w])
    else:
        mine = np.ascontiguousarray(full[shard.global_rows(n, rank, world)])
    if swap and rank == 1:
        mine[[3, 4]] = mine[[4, 3]]          # two rows in the wrong places, same pair count
    res = bench.closure_parity(dist, mine, sweeps, rows, cols, col_split)
    if rank == 0:
        q.put(res)
    dist.close()


@pytest.mark.parametrize("swap", [False, True], ids=["exact", "rows_swapped"])
@pytest.mark.parametrize("col_split", [False, True], ids=["rows", "columns"])
def test_bench_closure_parity_over_gloo(oracle_lib, swap, col_split):
    # bench.py's N > 1 parity leg: per-row digests (of a row, or of a row's
    # column slice) gathered from every rank and compared with the oracle's;
    # a swap of two rows on one rank keeps the pair count but must read as a
    # mismatch
    n, world = 256, 2
    rows, cols = gen.random_dag(n, 3, 22)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_parity_worker, args=(r, world, port, n, rows, cols, swap, col_split, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res["rows_checked"] == n
    if swap:
        assert res["closure"] == "MISMATCH" and res["rows_differing"] == 2
    else:
        assert res["closure"] == "bit-exact" and res["sweeps"] == [res["oracle_sweeps"]] * world
