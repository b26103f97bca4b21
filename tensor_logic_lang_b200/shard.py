"""Row sharding of the closure relation and GNN features across ranks.

Rank r of `world` holds rows r, r + world, r + 2*world, ... (cyclic).  On a
DAG with edges u < v the reach sets shrink with the row index, so contiguous
blocks would leave rank 0 with most of the work; dealing rows cyclically
balances it.  The runtime (csrc/) applies the same mapping; these helpers
give the host the same view (sizes, global row ids, reassembly).
"""
import numpy as np


def local_count(n, rank, world):
    """Rows of an n-row tensor held by `rank`."""
    return 0 if n <= rank else (n - rank + world - 1) // world


def global_rows(n, rank, world):
    return np.arange(rank, n, world, dtype=np.int64)


def assemble(blocks, n):
    """Interleave per-rank local row blocks (rank order) into the full n-row array."""
    world = len(blocks)
    shape = (n,) + tuple(blocks[0].shape[1:])
    out = np.empty(shape, dtype=blocks[0].dtype)
    for r, b in enumerate(blocks):
        out[r::world] = b
    return out


def gathered_row(u, world, per_rank):
    """Row of global node u in an all-gathered [world][per_rank] block layout."""
    return (u % world) * per_rank + u // world


def sharded_fixpoint(sweep_local, allreduce_max, max_sweeps=1000):
    """The convergence protocol of a row-sharded fixpoint.

    sweep_local() runs one sweep over this rank's rows and returns 1 if any of
    them changed; allreduce_max(x) returns the maximum of x over all ranks.
    Every rank runs the same number of sweeps and stops together, exactly
    when no row anywhere changed (fixpoint.zig:46-98 with a global flag).
    """
    sweeps = 0
    changed = 1
    while sweeps < max_sweeps and changed:
        changed = allreduce_max(sweep_local())
        sweeps += 1
    return sweeps
