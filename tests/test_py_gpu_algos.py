"""The NumPy mirror of the reference Python package's GLM functions
(gpu_algos_b200/py_gpu_algos.py).

CPU: the reference's validation rules and messages
(python/py-gpu-algos/py_gpu_algos/glm_ops.py:61-104) and a loud failure
without a device.  GPU: the golden fixtures -- outputs of the reference's own
NumPy functions (python/py-gpu-algos/tests/utils.py:255-309), stored in the
C++ memory order -- fed in the documented index order (X[f, task, obs],
Y[t, task, obs], M[f, t, task], also as non-contiguous views), with the C++
sign and scale; integers bit-exact, floats within 1e-4 (float32) / 1e-11
(float64) of the oracle.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from gpu_algos_b200 import py_gpu_algos as P  # noqa: E402


def _doc(a):
    """C++ memory order (obs, task, col) -> the documented index order (col, task, obs)."""
    return np.transpose(a, (2, 1, 0))


def test_names_match_the_reference_package():
    for base in ("glm_predict_naive", "glm_gradient_naive", "glm_gradient_xyyhat"):
        for sfx in ("", "_float32", "_float64", "_int32", "_int64"):
            assert callable(getattr(P, base + sfx))


def test_validation_messages():
    X = np.zeros((4, 2, 10), np.float32)
    M = np.zeros((4, 3, 2), np.float32)
    Y = np.zeros((3, 2, 10), np.float32)
    with pytest.raises(ValueError, match="3-dimensional"):
        P.glm_predict_naive(X[0], M)
    with pytest.raises(ValueError, match="same dtype"):
        P.glm_predict_naive(X, M.astype(np.float64))
    with pytest.raises(ValueError, match="Unsupported dtype"):
        P.glm_gradient_naive(X.astype(np.float16), Y.astype(np.float16), M.astype(np.float16))
    with pytest.raises(ValueError, match="Feature dimensions must match"):
        P.glm_predict_naive(X, np.zeros((5, 3, 2), np.float32))
    with pytest.raises(ValueError, match="compatible task/obs"):
        P.glm_gradient_xyyhat(X, np.zeros((3, 2, 11), np.float32), M)
    with pytest.raises(ValueError, match="Tensor dimensions must be compatible"):
        P.glm_gradient_naive(X, np.zeros((2, 2, 10), np.float32), M)
    with pytest.raises(ValueError, match="expected float64"):
        P.glm_gradient_naive_float64(X, Y, M)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the failure without a device")
def test_no_device_fails_loudly():
    X = np.zeros((4, 2, 10), np.float32)
    M = np.zeros((4, 3, 2), np.float32)
    with pytest.raises(RuntimeError, match="no CUDA device"):
        P.glm_predict_naive(X, M)


@pytest.mark.gpu
def test_golden_cases_in_the_documented_layout(golden, oracle):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    checked = 0
    for name, c in golden.items():
        X, M, Y = c["X"], c["M"], c["Y"]
        if X.dtype not in (np.float32, np.float64, np.int32, np.int64):
            continue
        Xd, Md, Yd = _doc(X), _doc(M), _doc(Y)  # non-contiguous views, read by their indices
        g = _doc(P.glm_gradient_naive(Xd, Yd, Md))
        yh = _doc(P.glm_predict_naive(Xd, Md))
        gx = _doc(P.glm_gradient_xyyhat(Xd, Yd, Md, 2.0 if np.issubdtype(X.dtype, np.integer) else 0.3, 0.25))
        if np.issubdtype(X.dtype, np.integer):
            assert np.array_equal(g, c["grad"]), name
            assert np.array_equal(yh, c["yhat"]), name
            assert np.array_equal(gx, oracle.gradient(X, M, Y, 2.0, 0.25, True)), name
        else:
            tol = 1e-4 if X.dtype == np.float32 else 1e-11
            og = oracle.gradient(X, M, Y, with_reg=False)
            floor = 1e-3 * np.abs(og.astype(np.float64)).max()
            rel = np.max(np.abs(g.astype(np.float64) - og) / np.maximum(np.abs(og), floor))
            assert rel <= tol, (name, rel)
            ogx = oracle.gradient(X, M, Y, 0.3, 0.25, True)
            relx = np.max(np.abs(gx.astype(np.float64) - ogx) / np.maximum(np.abs(ogx), floor))
            assert relx <= tol, (name, relx)
            scale = np.einsum("otf,tkf->otk", np.abs(X.astype(np.float64)), np.abs(M.astype(np.float64)))
            assert np.all(np.abs(yh.astype(np.float64) - c["yhat"]) <= tol * (np.abs(c["yhat"]) + scale)), name
        checked += 1
    assert checked >= 10
