"""Seeded synthetic inputs for the benchmark configurations.

Dense values come from a counter-based generator: SplitMix64 of
(seed, stream, flat index), so any consumer regenerates identical values
without shared state.  Every value is rounded to fp32 and kept as f64, so the
f64 oracle and the fp32 device path see the same operands.  Graphs use
numpy's PCG64 seeded per configuration.
"""
import numpy as np

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def _splitmix(x):
    with np.errstate(over="ignore"):
        z = x + _GOLD
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def _stream_key(seed, stream):
    h = np.uint64(seed & 0xFFFFFFFFFFFFFFFF)
    for ch in stream.encode():
        h = _splitmix(h ^ np.uint64(ch))
    return h


def _bits(seed, stream, n, salt=0):
    key = _stream_key(seed, stream)
    idx = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _splitmix(idx * np.uint64(2) + np.uint64(salt) + key * np.uint64(0x100000001B3))


def uniform(seed, stream, shape):
    n = int(np.prod(shape))
    u = (_bits(seed, stream, n) >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
    return u.astype(np.float32).astype(np.float64).reshape(shape)


def normal(seed, stream, shape, std=1.0):
    n = int(np.prod(shape))
    u1 = ((_bits(seed, stream, n, 0) >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / (1 << 53))
    u2 = ((_bits(seed, stream, n, 1) >> np.uint64(11)).astype(np.float64)) * (1.0 / (1 << 53))
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (z * std).astype(np.float32).astype(np.float64).reshape(shape)


def labels_onehot(seed, stream, rows, classes):
    lab = (_bits(seed, stream, rows) % np.uint64(classes)).astype(np.int64)
    t = np.zeros((rows, classes))
    t[np.arange(rows), lab] = 1.0
    return t


def er_graph(n, mean_degree, seed):
    """Directed Erdos-Renyi: each ordered pair (v, u) independently with p = d/n."""
    rng = np.random.default_rng(seed)
    p = mean_degree / n
    counts = rng.binomial(n, p, size=n)
    rows = np.repeat(np.arange(n, dtype=np.int64), counts)
    cols = np.empty(rows.shape[0], dtype=np.int64)
    off = 0
    for v in range(n):
        k = counts[v]
        if k:
            cols[off:off + k] = np.sort(rng.choice(n, size=k, replace=False))
        off += k
    return rows, cols


def random_dag(n, mean_out_degree, seed):
    """Exactly d*n distinct edges u -> v with u < v, uniform over pairs."""
    rng = np.random.default_rng(seed)
    m = int(mean_out_degree * n)
    if m > n * (n - 1) // 2:
        raise ValueError("too many edges for a DAG of this size")
    out = np.empty((0, 2), dtype=np.int64)
    while out.shape[0] < m:
        k = int((m - out.shape[0]) * 1.1) + 16
        a = rng.integers(0, n, size=k)
        b = rng.integers(0, n, size=k)
        keep = a != b
        u = np.minimum(a, b)[keep]
        v = np.maximum(a, b)[keep]
        cand = np.concatenate([out, np.stack([u, v], axis=1)])
        _, first = np.unique(cand[:, 0] * n + cand[:, 1], return_index=True)
        out = cand[np.sort(first)]
    out = out[:m]
    return out[:, 0].copy(), out[:, 1].copy()


def csr_from_coo(n_rows, rows, cols):
    order = np.lexsort((cols, rows))
    r, c = rows[order], cols[order]
    rowptr = np.zeros(n_rows + 1, dtype=np.int64)
    np.add.at(rowptr, r + 1, 1)
    return np.cumsum(rowptr), c.astype(np.int32)
