"""Generate the committed golden fixtures ``tests/golden/glm_golden.npz``.

Run once, where a checkout of the reference is available, giving its root
as the argument (or in GPU_ALGOS_REFERENCE)::

    python tests/golden/make_golden.py <path-to-gpu_algos-checkout>

Source of truth.  The reference's CPU product goes through Eigen, which is
absent from this image, so its C++ host path cannot be run here.  The
reference's Python test-suite ships NumPy reference functions for the same
operations (``python/py-gpu-algos/tests/utils.py:255-309``:
``get_numpy_reference_glm_predict`` and ``get_numpy_reference_glm_gradient``);
this script imports those functions from the reference checkout and records
their outputs.  Conventions, read from the two sources:

* index order: the NumPy functions index ``X[f, task, obs]``, ``Y[t, task, obs]``,
  ``M[f, t, task]`` -- the same logical indices as the C++ ``Tensor3D.at(col,
  row, sheet)``; the fixtures store arrays in the C++ memory order, i.e. the
  NumPy arrays transposed ``(2, 1, 0)``;
* sign and scale: the NumPy gradient is ``X (Y - Yhat)^T`` while the C++ host
  path computes ``2 (Yhat - Y) X`` (``glm_gradient_naive.cuh:454``), so
  ``grad_cpp = -2 * grad_numpy``.  Integer arrays are multiplied modulo 2^bits,
  exactly as the C++ integer product wraps.

Input generation follows the reference tests: ``default_rng(42).normal(1, 1)``
for floats and ``integers(-100, 100)`` for integers
(``python/py-gpu-algos/tests/conftest.py:200-217``), the shape list of
``test_glm_ops.py:232-237`` and the single-dimension cases of
``test_glm_ops.py:504-549``.  Two further cases are recorded: the
single-task, single-target shape of the reference's CPU-checkable driver
(nobs 8192, nfeatures 32, float32, X ~ U(-1, 1), y = X b_true + N(0, 0.01^2),
current b ~ N(0, 1)), and the driver's "increasing" initialisation
(``benchmark_tensor3d_3in_1out.cuh:180-184``) for int32/int64 whose exact
answer is computed with Python integers.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "glm_golden.npz")


def _load_reference_utils(ref_root: str):
    path = os.path.join(ref_root, "python", "py-gpu-algos", "tests", "utils.py")
    spec = importlib.util.spec_from_file_location("ref_py_gpu_algos_test_utils", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _to_cpp(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(np.transpose(a, (2, 1, 0)))


def _exact_increasing(dtype, nf, nt, ntasks, nobs):
    """Driver 'increasing' init: A[i] = i, B[i] = i, C[i] = i in memory order."""
    bits = np.dtype(dtype).itemsize * 8
    mod = 1 << bits
    X = [i % mod for i in range(nf * ntasks * nobs)]
    M = [i % mod for i in range(nf * nt * ntasks)]
    Y = [i % mod for i in range(nt * ntasks * nobs)]
    grad = []
    yhat = []
    for task in range(ntasks):
        for t in range(nt):
            for f in range(nf):
                s = 0
                for obs in range(nobs):
                    xrow = (obs * ntasks + task) * nf
                    dot = sum(M[(task * nt + t) * nf + k] * X[xrow + k] for k in range(nf))
                    e = dot - Y[(obs * ntasks + task) * nt + t]
                    s += e * X[xrow + f]
                grad.append((2 * s) % mod)
    for obs in range(nobs):
        for task in range(ntasks):
            for t in range(nt):
                xrow = (obs * ntasks + task) * nf
                yhat.append(sum(M[(task * nt + t) * nf + k] * X[xrow + k] for k in range(nf)) % mod)

    unsigned = {8: np.uint8, 16: np.uint16, 32: np.uint32, 64: np.uint64}[bits]

    def wrap(vals):
        return np.array([v % mod for v in vals], dtype=unsigned).view(dtype)

    return (
        wrap(X).reshape(nobs, ntasks, nf),
        wrap(M).reshape(ntasks, nt, nf),
        wrap(Y).reshape(nobs, ntasks, nt),
        wrap(yhat).reshape(nobs, ntasks, nt),
        wrap(grad).reshape(ntasks, nt, nf),
    )


def main(ref_root: str) -> None:
    ref = _load_reference_utils(ref_root)
    cases = {}

    def add(name, X, M, Y):
        # X, M, Y in the NumPy reference's index order
        yhat = ref.get_numpy_reference_glm_predict(X, M)
        g_np = ref.get_numpy_reference_glm_gradient(X, Y, M)
        if np.issubdtype(X.dtype, np.integer):
            with np.errstate(over="ignore"):
                g_cpp = (g_np * X.dtype.type(-2)).astype(X.dtype)
        else:
            g_cpp = (-2 * g_np).astype(X.dtype)
        cases[f"{name}/X"] = _to_cpp(X)
        cases[f"{name}/M"] = _to_cpp(M)
        cases[f"{name}/Y"] = _to_cpp(Y)
        cases[f"{name}/yhat"] = _to_cpp(yhat)
        cases[f"{name}/grad"] = _to_cpp(g_cpp)

    dtypes = [np.float32, np.float64, np.int32, np.int64]
    shapes = [(10, 3, 4, 100), (5, 3, 2, 50), (20, 8, 4, 100), (10, 1, 5, 200), (15, 5, 1, 100),
              (1, 2, 3, 100), (5, 2, 1, 100), (5, 2, 3, 1), (33, 2, 3, 257)]
    for dt in dtypes:
        for (nf, nt, ntasks, nobs) in shapes:
            g = np.random.default_rng(42)
            if np.issubdtype(dt, np.floating):
                X = g.normal(1, 1, (nf, ntasks, nobs)).astype(dt)
                Y = g.normal(1, 1, (nt, ntasks, nobs)).astype(dt)
                M = g.normal(1, 1, (nf, nt, ntasks)).astype(dt)
            else:
                X = g.integers(-100, 100, (nf, ntasks, nobs)).astype(dt)
                Y = g.integers(-100, 100, (nt, ntasks, nobs)).astype(dt)
                M = g.integers(-100, 100, (nf, nt, ntasks)).astype(dt)
            add(f"ref_{np.dtype(dt).name}_{nf}x{nt}x{ntasks}x{nobs}", X, M, Y)

    # the reference driver's CPU-checkable single-task shape
    g = np.random.default_rng(20250101)
    nf, nobs = 32, 8192
    Xc = g.uniform(-1.0, 1.0, (nobs, 1, nf)).astype(np.float32)
    b_true = g.normal(0.0, 1.0, (1, 1, nf)).astype(np.float32)
    y = (Xc[:, 0, :].astype(np.float64) @ b_true[0, 0, :].astype(np.float64)
         + g.normal(0.0, 0.01, nobs)).astype(np.float32).reshape(nobs, 1, 1)
    b = g.normal(0.0, 1.0, (1, 1, nf)).astype(np.float32)
    add("driver_f32_32x1x1x8192", np.transpose(Xc, (2, 1, 0)), np.transpose(b, (2, 1, 0)),
        np.transpose(y, (2, 1, 0)))

    # exact integer known answers for the driver's "increasing" init
    for dt in (np.int32, np.int64):
        X, M, Y, yhat, grad = _exact_increasing(dt, 3, 2, 2, 5)
        name = f"increasing_{np.dtype(dt).name}_3x2x2x5"
        cases[f"{name}/X"], cases[f"{name}/M"], cases[f"{name}/Y"] = X, M, Y
        cases[f"{name}/yhat"], cases[f"{name}/grad"] = yhat, grad
        # cross-check the NumPy reference on the same exact case
        add(f"{name}_numpy", np.transpose(X, (2, 1, 0)), np.transpose(M, (2, 1, 0)),
            np.transpose(Y, (2, 1, 0)))
        assert np.array_equal(cases[f"{name}_numpy/grad"], grad)
        assert np.array_equal(cases[f"{name}_numpy/yhat"], yhat)

    np.savez_compressed(OUT, **cases)
    total = sum(v.nbytes for v in cases.values())
    print(f"wrote {OUT}: {len(cases) // 5} cases, {total / 1e6:.2f} MB raw")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GPU_ALGOS_REFERENCE")
    if not root:
        sys.exit("usage: make_golden.py <path-to-gpu_algos-checkout>  (or set GPU_ALGOS_REFERENCE)")
    main(root)
