"""Shared helpers of the GPU parity tests (comparison metrics, runners)."""
import numpy as np

from tensor_logic_lang_b200 import lang

# Float tolerance of the fp32 / TF32 device path against the f64 oracle.
TOL_TF32 = 1e-3
TOL_FP32 = 1e-5


def normwise(got, want):
    """max|g - r| / max|r| (0 when both are all zero)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    scale = np.max(np.abs(want)) if want.size else 0.0
    err = np.max(np.abs(got - want)) if want.size else 0.0
    return 0.0 if scale == 0 and err == 0 else err / (scale if scale > 0 else 1.0)


def assert_close(got, want, tol, what=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    assert np.all(np.isfinite(got)), what
    e = normwise(got, want)
    assert e <= tol, f"{what}: norm-wise rel err {e:.3e} > {tol}"
    return e


def run_gpu(ctx, src, inputs=None, sparse=None):
    p = lang.Program(src, inputs=inputs, sparse_inputs=sparse)
    ctx.run(p)
    return p
