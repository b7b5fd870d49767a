"""NumPy-facing wrapper of the C oracle (``libglm_oracle.so``).

TEST INFRASTRUCTURE ONLY: the checker used by ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``.  The
product never imports this module.

Arrays use the reference's memory layout (``include/common/types/tensor3d.hpp:107-112``),
expressed here as C-ordered NumPy arrays indexed ``[sheet, row, col]``:

* ``X``     shape ``(nobs, ntasks, nfeatures)``
* ``Y``     shape ``(nobs, ntasks, ntargets)``   (``Yhat`` alike)
* ``M``     shape ``(ntasks, ntargets, nfeatures)``   (``grad`` alike)

NumPy has no bfloat16 type: bfloat16 arrays travel as ``np.uint16`` bit
patterns, and ``predict`` / ``gradient`` / ``loss`` take ``bf16=True`` to read
them so (``bf16_bits`` and ``bf16_to_f32`` convert).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libglm_oracle.so")

SUFFIX = {
    np.dtype(np.float32): "f32",
    np.dtype(np.float64): "f64",
    np.dtype(np.float16): "f16",
    np.dtype(np.int8): "i8",
    np.dtype(np.int16): "i16",
    np.dtype(np.int32): "i32",
    np.dtype(np.int64): "i64",
    np.dtype(np.uint8): "u8",
    np.dtype(np.uint16): "u16",
    np.dtype(np.uint32): "u32",
    np.dtype(np.uint64): "u64",
}

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_D = ctypes.c_double
_INT = ctypes.c_int


def _declare(L: ctypes.CDLL) -> None:
    for sfx in list(SUFFIX.values()) + ["bf16"]:
        getattr(L, f"oracle_glm_predict_{sfx}").argtypes = [_P, _P, _P, _I64, _I64, _I64, _I64]
        getattr(L, f"oracle_glm_gradient_{sfx}").argtypes = [
            _P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _INT]
        getattr(L, f"oracle_glm_loss_{sfx}").argtypes = [
            _P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D]
    L.oracle_glm_gradient_f32_acc64.argtypes = [
        _P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _INT]
    for sfx in ("f32", "f64"):
        getattr(L, f"oracle_prox_step_{sfx}").argtypes = [_P, _P, _I64, _D, _D]
        getattr(L, f"oracle_power_norm_{sfx}").argtypes = [_P, _P, _I64, _I64, _I64, _INT, _P]
        getattr(L, f"oracle_fit_{sfx}").argtypes = [
            _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _P, _INT, _INT, _P]
    L.oracle_power_start.argtypes = [_P, _I64, ctypes.c_uint64]
    L.oracle_set_threads.argtypes = [_INT]
    L.oracle_get_threads.restype = _INT


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def _sfx(dtype, bf16: bool = False) -> str:
    if bf16:
        assert np.dtype(dtype) == np.uint16, "bfloat16 arrays are uint16 bit patterns"
        return "bf16"
    return SUFFIX[np.dtype(dtype)]


def bf16_bits(a) -> np.ndarray:
    """float32 values -> bfloat16 bit patterns (round to nearest even; NaN stays NaN)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_to_f32(b) -> np.ndarray:
    """bfloat16 bit patterns -> float32 (exact)."""
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def get_threads() -> int:
    return int(lib().oracle_get_threads())


def _dims(X, M):
    nobs, ntasks, nf = X.shape
    ntasks2, nt, nf2 = M.shape
    assert ntasks == ntasks2 and nf == nf2, (X.shape, M.shape)
    return nf, nt, ntasks, nobs


def predict(X: np.ndarray, M: np.ndarray, bf16: bool = False) -> np.ndarray:
    """Yhat[obs, task, t] = sum_f M[task, t, f] * X[obs, task, f]."""
    X = np.ascontiguousarray(X)
    M = np.ascontiguousarray(M, dtype=X.dtype)
    nf, nt, ntasks, nobs = _dims(X, M)
    Yhat = np.zeros((nobs, ntasks, nt), dtype=X.dtype)
    getattr(lib(), f"oracle_glm_predict_{_sfx(X.dtype, bf16)}")(
        _ptr(X), _ptr(M), _ptr(Yhat), nf, nt, ntasks, nobs)
    return Yhat


def gradient(X, M, Y, lam: float = 0.0, alpha: float = 0.0, with_reg: bool = True,
             bf16: bool = False) -> np.ndarray:
    """grad = 2*sum_obs (Yhat - Y) X  [+ lam*(alpha*sign(M) + 2(1-alpha) M)].

    ``Y=None`` stands for an all-zero Y.
    """
    X = np.ascontiguousarray(X)
    M = np.ascontiguousarray(M, dtype=X.dtype)
    nf, nt, ntasks, nobs = _dims(X, M)
    if Y is not None:
        Y = np.ascontiguousarray(Y, dtype=X.dtype)
        assert Y.shape == (nobs, ntasks, nt), Y.shape
    grad = np.zeros((ntasks, nt, nf), dtype=X.dtype)
    getattr(lib(), f"oracle_glm_gradient_{_sfx(X.dtype, bf16)}")(
        _ptr(X), _ptr(M), _ptr(Y), _ptr(grad), nf, nt, ntasks, nobs,
        float(lam), float(alpha), int(bool(with_reg)))
    return grad


def gradient_acc64(X, M, Y, lam: float = 0.0, alpha: float = 0.0, with_reg: bool = True) -> np.ndarray:
    """Same as :func:`gradient` for float32 inputs, carried in double."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    M = np.ascontiguousarray(M, dtype=np.float32)
    nf, nt, ntasks, nobs = _dims(X, M)
    if Y is not None:
        Y = np.ascontiguousarray(Y, dtype=np.float32)
    grad = np.zeros((ntasks, nt, nf), dtype=np.float64)
    lib().oracle_glm_gradient_f32_acc64(
        _ptr(X), _ptr(M), _ptr(Y), _ptr(grad), nf, nt, ntasks, nobs,
        float(lam), float(alpha), int(bool(with_reg)))
    return grad


def loss(M, Y, Yhat, lam: float = 0.0, alpha: float = 0.0, bf16: bool = False) -> np.ndarray:
    M = np.ascontiguousarray(M)
    Y = np.ascontiguousarray(Y, dtype=M.dtype)
    Yhat = np.ascontiguousarray(Yhat, dtype=M.dtype)
    ntasks, nt, nf = M.shape
    nobs = Y.shape[0]
    out = np.zeros((1,), dtype=M.dtype)
    getattr(lib(), f"oracle_glm_loss_{_sfx(M.dtype, bf16)}")(
        _ptr(M), _ptr(Y), _ptr(Yhat), _ptr(out), nf, nt, ntasks, nobs, float(lam), float(alpha))
    return out


def prox_step(beta, grad_smooth, inv_L: float, l1: float) -> np.ndarray:
    beta = np.array(beta, copy=True, order="C")
    g = np.ascontiguousarray(grad_smooth, dtype=beta.dtype)
    getattr(lib(), f"oracle_prox_step_{_sfx(beta.dtype)}")(
        _ptr(beta), _ptr(g), beta.size, float(inv_L), float(l1))
    return beta


def power_start(n: int, seed: int) -> np.ndarray:
    v0 = np.zeros((n,), dtype=np.float64)
    lib().oracle_power_start(_ptr(v0), int(n), ctypes.c_uint64(int(seed) & (2**64 - 1)))
    return v0


def power_norm(X, v0, n_power: int) -> np.ndarray:
    X = np.ascontiguousarray(X)
    nobs, ntasks, nf = X.shape
    v0 = np.ascontiguousarray(v0, dtype=X.dtype).reshape(ntasks, nf)
    out = np.zeros((ntasks,), dtype=np.float64)
    getattr(lib(), f"oracle_power_norm_{_sfx(X.dtype)}")(
        _ptr(X), _ptr(v0), nf, ntasks, nobs, int(n_power), _ptr(out))
    return out


def fit(X, Y, lambda1: float, lambda2: float, v0, n_power: int, n_iter: int):
    """ISTA elastic-net fit; returns (beta, lipschitz per task)."""
    X = np.ascontiguousarray(X)
    Y = np.ascontiguousarray(Y, dtype=X.dtype)
    nobs, ntasks, nf = X.shape
    nt = Y.shape[2]
    v0 = np.ascontiguousarray(v0, dtype=X.dtype).reshape(ntasks, nf)
    beta = np.zeros((ntasks, nt, nf), dtype=X.dtype)
    lip = np.zeros((ntasks,), dtype=np.float64)
    getattr(lib(), f"oracle_fit_{_sfx(X.dtype)}")(
        _ptr(X), _ptr(Y), _ptr(beta), nf, nt, ntasks, nobs, float(lambda1), float(lambda2),
        _ptr(v0), int(n_power), int(n_iter), _ptr(lip))
    return beta, lip
