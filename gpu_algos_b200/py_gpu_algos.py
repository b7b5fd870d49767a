"""NumPy GLM functions with the reference Python package's names and shapes.

The reference ships pybind11 bindings (``python/py-gpu-algos``) whose GLM
functions are ``glm_predict_naive(X, M)``, ``glm_gradient_naive(X, Y, M)`` and
``glm_gradient_xyyhat(X, Y, M)`` plus typed variants ``*_float32``,
``*_float64``, ``*_int32``, ``*_int64``
(``python/py-gpu-algos/py_gpu_algos/glm_ops.py:114-330``), documented with
arrays indexed ``X[feature, task, obs]``, ``Y[target, task, obs]`` and
``M[feature, target, task]``.  Those bindings do not compute what they
document:

* ``glm_ops.cu:271-280,404-413`` pass ``(X, Y, M)`` to
  ``run_device_kernel(X, M, Y, ...)``: Y and M trade places;
* they copy the C-ordered NumPy buffers (observations fastest) to a device
  layout whose fastest index is the feature
  (``include/common/types/tensor3d.hpp:107-112``);
* ``glm_gradient_xyyhat`` in ``glm_ops.py`` calls the binding without the
  ``lambda`` and ``alpha`` it requires.

This module keeps the names, argument order, shapes, validation and error
messages, and computes what the documentation says, through the library's
C ABI (``include/glm_b200.h``): arrays are read by their documented indices
(any strides), laid out as the library expects, computed on the current CUDA
device and returned in the documented shapes:

* ``glm_predict_naive(X, M) -> Yhat[target, task, obs]``;
* ``glm_gradient_naive(X, Y, M) -> grad[feature, target, task]``
  ``= 2 sum_obs (Yhat - Y) X`` -- the C++ kernel classes' convention
  (``glm_gradient_naive.cuh:454``);
* ``glm_gradient_xyyhat(X, Y, M, lam=0, alpha=0)``: the same plus the
  elastic-net term ``lam*(alpha*sign(M) + 2*(1-alpha)*M)``
  (``glm_gradient_xyyhat.cuh:839-851``).

There is no host fallback: without the built library or a CUDA device the
calls raise.
"""
from __future__ import annotations

import numpy as np
import torch

from . import capi, glm

_GLM_TYPES = {
    np.dtype(np.float32): "float32",
    np.dtype(np.float64): "float64",
    np.dtype(np.int32): "int32",
    np.dtype(np.int64): "int64",
}


def _validate_predict(X: np.ndarray, M: np.ndarray, name: str) -> None:
    if X.ndim != 3 or M.ndim != 3:
        raise ValueError(f"{name}: Input arrays must be 3-dimensional")
    if X.dtype != M.dtype:
        raise ValueError(f"{name}: Input arrays must have the same dtype")
    if X.dtype not in _GLM_TYPES:
        raise ValueError(f"{name}: Unsupported dtype {X.dtype}. GLM operations support: float32, float64, int32, int64")
    nf_x, ntasks_x, _ = X.shape
    nf_m, _, ntasks_m = M.shape
    if nf_x != nf_m:
        raise ValueError(f"{name}: Feature dimensions must match: X({nf_x}) vs M({nf_m})")
    if ntasks_x != ntasks_m:
        raise ValueError(f"{name}: Task dimensions must match: X({ntasks_x}) vs M({ntasks_m})")


def _validate_gradient(X: np.ndarray, Y: np.ndarray, M: np.ndarray, name: str) -> None:
    if X.ndim != 3 or Y.ndim != 3 or M.ndim != 3:
        raise ValueError(f"{name}: Input arrays must be 3-dimensional")
    if X.dtype != Y.dtype or X.dtype != M.dtype:
        raise ValueError(f"{name}: All input arrays must have the same dtype")
    if X.dtype not in _GLM_TYPES:
        raise ValueError(f"{name}: Unsupported dtype {X.dtype}. GLM operations support: float32, float64, int32, int64")
    nf_x, ntasks_x, nobs_x = X.shape
    nt_y, ntasks_y, nobs_y = Y.shape
    nf_m, nt_m, ntasks_m = M.shape
    if ntasks_x != ntasks_y or nobs_x != nobs_y:
        raise ValueError(f"{name}: X and Y must have compatible task/obs dimensions: "
                         f"X({ntasks_x}, {nobs_x}) vs Y({ntasks_y}, {nobs_y})")
    if nf_x != nf_m or nt_y != nt_m or ntasks_x != ntasks_m:
        raise ValueError(f"{name}: Tensor dimensions must be compatible: "
                         f"X({nf_x}, {ntasks_x}), Y({nt_y}, {ntasks_y}), M({nf_m}, {nt_m}, {ntasks_m})")


def _to_device(a: np.ndarray) -> torch.Tensor:
    """a[i, j, k] (documented index order) -> the library's layout, C order (k, j, i)."""
    host = np.ascontiguousarray(np.transpose(a, (2, 1, 0)))
    return torch.from_numpy(host).to(device=torch.device("cuda", torch.cuda.current_device()))


def _to_host(t: torch.Tensor) -> np.ndarray:
    return np.ascontiguousarray(np.transpose(t.cpu().numpy(), (2, 1, 0)))


def _require_cuda(name: str) -> None:
    if not torch.cuda.is_available():
        raise RuntimeError(f"{name}: no CUDA device (this library has no host fallback)")


def glm_predict_naive(X: np.ndarray, M: np.ndarray) -> np.ndarray:
    """Yhat[t, task, obs] = sum_f M[f, t, task] X[f, task, obs]; X (nf, ntasks, nobs), M (nf, nt, ntasks)."""
    _validate_predict(X, M, "glm_predict_naive")
    _require_cuda("glm_predict_naive")
    Yhat = glm.predict(_to_device(X), _to_device(M))
    torch.cuda.current_stream().synchronize()
    return _to_host(Yhat)


def _gradient(X, Y, M, lam, alpha, regularize, name):
    _validate_gradient(X, Y, M, name)
    _require_cuda(name)
    grad = glm.gradient(_to_device(X), _to_device(M), _to_device(Y), float(lam), float(alpha), regularize)
    torch.cuda.current_stream().synchronize()
    return _to_host(grad)


def glm_gradient_naive(X: np.ndarray, Y: np.ndarray, M: np.ndarray) -> np.ndarray:
    """grad[f, t, task] = 2 sum_obs (Yhat - Y)[t, task, obs] X[f, task, obs] (no regularisation)."""
    return _gradient(X, Y, M, 0.0, 0.0, False, "glm_gradient_naive")


def glm_gradient_xyyhat(X: np.ndarray, Y: np.ndarray, M: np.ndarray, lam: float = 0.0,
                        alpha: float = 0.0) -> np.ndarray:
    """glm_gradient_naive's value plus lam*(alpha*sign(M) + 2*(1-alpha)*M)."""
    return _gradient(X, Y, M, lam, alpha, True, "glm_gradient_xyyhat")


def _typed(fn, dtype, name):
    def typed(*args, **kwargs):
        for a in args[:3]:
            if isinstance(a, np.ndarray) and a.dtype != np.dtype(dtype):
                raise ValueError(f"{name}: expected {np.dtype(dtype).name} arrays, got {a.dtype}")
        return fn(*args, **kwargs)

    typed.__name__ = name
    typed.__doc__ = f"{fn.__name__} for {np.dtype(dtype).name} arrays."
    return typed


for _dt in (np.float32, np.float64, np.int32, np.int64):
    _sfx = np.dtype(_dt).name
    for _fn in (glm_predict_naive, glm_gradient_naive, glm_gradient_xyyhat):
        _name = f"{_fn.__name__}_{_sfx}"
        globals()[_name] = _typed(_fn, _dt, _name)

__all__ = [f"{f}{s}" for f in ("glm_predict_naive", "glm_gradient_naive", "glm_gradient_xyyhat")
           for s in ("", "_float32", "_float64", "_int32", "_int64")]

# the library must be present: importing this module without it fails loudly
capi.lib()
