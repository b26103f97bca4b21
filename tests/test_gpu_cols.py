"""Column-sharded closure on one GPU: each slice r of W (TL_SHARD_COLS_OF=r/W)
is closed by the one-launch fixpoint alone, with no exchange, and must equal
columns [r c / W, (r + 1) c / W) of the f64 oracle's closure, bit for bit; the
sweep count is the same on every slice (it comes from the graph, not from the
slice).  The reference fixpoint (fixpoint.zig:46-98) has no distribution:
the whole relation is the parity target."""
import os

import numpy as np
import pytest
import torch

from tensor_logic_lang_b200 import abi, configs
from tensor_logic_lang_b200 import inputs as gen

pytestmark = pytest.mark.gpu


def _closure_src(n):
    return (f"domain x: {n}\ndomain y: {n}\ndomain z: {n}\nsparse Edge[x, y]\n"
            "Reach[x,y] = step(Edge[x,y])\nReach[x,z] max= step(Reach[x,y] Edge[y,z])\n")


def _graph(n, kind):
    if kind == "dag":
        _, _, sp, _ = configs.closure(n=n)
        rows, cols, _ = sp["Edge"]
        return rows, cols
    if kind == "transitive":
        # a graph that is its own closure: every i -> j with i < j inside
        # blocks of 8 nodes (the first sweep changes nothing)
        i, j = np.meshgrid(np.arange(8), np.arange(8), indexing="ij")
        keep = i < j
        base = np.arange(0, n, 8)[:, None]
        return (base + i[keep][None, :]).ravel(), (base + j[keep][None, :]).ravel()
    rows, cols = gen.random_dag(n, 3, 41)
    rng = np.random.default_rng(42)
    b = rng.integers(0, n, size=(n // 50, 2))
    b = b[b[:, 0] > b[:, 1]]
    return np.concatenate([rows, b[:, 0]]), np.concatenate([cols, b[:, 1]])


def _oracle(oracle_lib, n, rows, cols):
    colptr, rowidx = gen.csr_from_coo(n, cols, rows)
    R = np.zeros((n, n // 32), dtype=np.uint32)
    np.bitwise_or.at(R, (rows, cols >> 5), (np.uint32(1) << (cols & 31).astype(np.uint32)))
    sweeps = oracle_lib.closure_right(n, colptr, rowidx, R)
    return R, sweeps


CASES = [(8192, "dag", 4), (5120, "cyclic", 2), (5120, "cyclic", 5), (4096, "transitive", 2), (32768, "dag", 8),
         (24576, "dag", 2)]


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("n,kind,world", CASES, ids=[f"{c[1]}{c[0]}-of{c[2]}" for c in CASES])
def test_column_slices(oracle_lib, monkeypatch, n, kind, world):
    from tensor_logic_lang_b200 import lang
    from tensor_logic_lang_b200.runtime import Context
    rows, cols = _graph(n, kind)
    R, osw = _oracle(oracle_lib, n, rows, cols)
    w = n // 32 // world
    p = lang.Program(_closure_src(n), sparse_inputs={"Edge": (rows, cols, None)})
    sweeps = set()
    with Context(device=0) as ctx:
        for r in range(world):
            monkeypatch.setenv("TL_SHARD_COLS_OF", f"{r}/{world}")
            ctx.set_sharding("Reach", abi.SHARD_COLS)
            for _ in range(2):      # a second run: the next epoch of closed words
                ctx.run(p)
                got = ctx.bits("Reach", words=w)
                np.testing.assert_array_equal(got, R[:, r * w:(r + 1) * w])
                sweeps.add(ctx.sweeps)
    assert len(sweeps) == 1
    sw = sweeps.pop()
    if kind == "dag":
        assert sw == osw == 2
    elif kind == "transitive":
        assert sw == osw == 1
    else:
        assert 2 <= sw <= osw


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_column_slices_need_whole_blocks(monkeypatch):
    # 1000 columns do not split into 2 slices of whole 128-column blocks: the
    # run fails with TL_ERR_UNSUPPORTED before anything launches
    from tensor_logic_lang_b200 import lang
    from tensor_logic_lang_b200.abi import TLError
    from tensor_logic_lang_b200.runtime import Context
    n = 1000
    rows, cols = gen.random_dag(n, 3, 7)
    p = lang.Program(_closure_src(n), sparse_inputs={"Edge": (rows, cols, None)})
    with Context(device=0) as ctx:
        monkeypatch.setenv("TL_SHARD_COLS_OF", "1/2")
        ctx.set_sharding("Reach", abi.SHARD_COLS)
        with pytest.raises(TLError) as e:
            ctx.run(p)
        assert e.value.status == abi.TL_ERR_UNSUPPORTED
