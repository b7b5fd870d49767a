"""Torch-facing wrappers of the GLM C ABI.

Tensors follow the reference's Tensor3D memory layout
(``include/common/types/tensor3d.hpp:107-112``), written as C-contiguous
torch shapes ``[sheet, row, col]``:

* ``X``           ``(nobs, ntasks, nfeatures)``
* ``Y``, ``Yhat``  ``(nobs, ntasks, ntargets)``
* ``M``, ``grad``  ``(ntasks, ntargets, nfeatures)``

Every call launches asynchronously on ``stream`` (default: torch's current
stream) and goes to ``libglm_b200.so``; there is no host or torch fallback.
"""
from __future__ import annotations

import torch

from . import capi

SUFFIX = {
    torch.float16: "f16",
    torch.bfloat16: "bf16",
    torch.float32: "f32",
    torch.float64: "f64",
    torch.int8: "i8",
    torch.int16: "i16",
    torch.int32: "i32",
    torch.int64: "i64",
    torch.uint8: "u8",
    torch.uint16: "u16",
    torch.uint32: "u32",
    torch.uint64: "u64",
}


def _stream(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, name: str, shape, dtype) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    if t.dtype != dtype:
        raise ValueError(f"{name} has dtype {t.dtype}, expected {dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _dims(X: torch.Tensor, M: torch.Tensor):
    nobs, ntasks, nf = X.shape
    ntasks2, nt, nf2 = M.shape
    if ntasks2 != ntasks or nf2 != nf:
        raise ValueError(f"X {tuple(X.shape)} and M {tuple(M.shape)} disagree")
    return nf, nt, ntasks, nobs


def predict(X, M, out=None, stream=None):
    """Yhat[obs, task, t] = sum_f M[task, t, f] X[obs, task, f]."""
    sfx = SUFFIX[X.dtype]
    nf, nt, ntasks, nobs = _dims(X, M)
    _need(X, "X", (nobs, ntasks, nf), X.dtype)
    _need(M, "M", (ntasks, nt, nf), X.dtype)
    if out is None:
        out = torch.empty((nobs, ntasks, nt), dtype=X.dtype, device=X.device)
    _need(out, "out", (nobs, ntasks, nt), X.dtype)
    capi.call(f"glmb_predict_{sfx}", _ptr(X), _ptr(M), _ptr(out), nf, nt, ntasks, nobs, _stream(stream))
    return out


def workspace_bytes(dtype, nf: int, nt: int, ntasks: int, nobs: int) -> int:
    return int(getattr(capi.lib(), f"glmb_gradient_workspace_size_{SUFFIX[dtype]}")(nf, nt, ntasks, nobs))


def gradient(X, M, Y, lam: float = 0.0, alpha: float = 0.0, regularize: bool = True,
             yhat_out=None, out=None, workspace=None, stream=None, logistic: bool = False):
    """Fused prediction + gradient (+ elastic-net term when ``regularize``).

    ``Y=None`` means an all-zero Y.  ``yhat_out`` (optional) receives the
    predictions.  ``workspace`` is an optional CUDA uint8 tensor of at least
    :func:`workspace_bytes` bytes.  ``logistic``: logistic link (mu =
    sigmoid(X M), gradient sum (mu - Y) X of the log-likelihood; predictions mu).
    """
    sfx = SUFFIX[X.dtype]
    nf, nt, ntasks, nobs = _dims(X, M)
    _need(X, "X", (nobs, ntasks, nf), X.dtype)
    _need(M, "M", (ntasks, nt, nf), X.dtype)
    flags = capi.GRAD_REGULARIZE if regularize else 0
    if logistic:
        flags |= capi.GRAD_LOGISTIC
    if Y is None:
        flags |= capi.GRAD_Y_ZERO
    else:
        _need(Y, "Y", (nobs, ntasks, nt), X.dtype)
    if yhat_out is not None:
        _need(yhat_out, "yhat_out", (nobs, ntasks, nt), X.dtype)
        flags |= capi.GRAD_WRITE_YHAT
    if out is None:
        out = torch.empty((ntasks, nt, nf), dtype=X.dtype, device=X.device)
    _need(out, "out", (ntasks, nt, nf), X.dtype)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    capi.call(f"glmb_gradient_{sfx}", _ptr(X), _ptr(M), _ptr(Y), _ptr(out), _ptr(yhat_out),
              nf, nt, ntasks, nobs, float(lam), float(alpha), flags, ws_ptr, ws_bytes, _stream(stream))
    return out


def loss(M, Y, Yhat, lam: float = 0.0, alpha: float = 0.0, out=None, workspace=None, stream=None):
    """sum (Yhat - Y)^2 + lam * (alpha * sum|M| + (1 - alpha) * sum M^2), as a
    one-element tensor of M's dtype (``Y=None``: zeros)."""
    sfx = SUFFIX[M.dtype]
    ntasks, nt, nf = M.shape
    nobs = Yhat.shape[0]
    _need(Yhat, "Yhat", (nobs, ntasks, nt), M.dtype)
    if Y is not None:
        _need(Y, "Y", (nobs, ntasks, nt), M.dtype)
    if out is None:
        out = torch.empty((1,), dtype=M.dtype, device=M.device)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    capi.call(f"glmb_loss_{sfx}", _ptr(M), _ptr(Y), _ptr(Yhat), _ptr(out), nf, nt, ntasks, nobs,
              float(lam), float(alpha), ws_ptr, ws_bytes, _stream(stream))
    return out


def gradient_loss(X, M, Y, lam: float = 0.0, alpha: float = 0.0, regularize: bool = True,
                  yhat_out=None, out=None, loss_out=None, workspace=None, stream=None):
    """Gradient (as :func:`gradient`) and loss (as :func:`loss`, always with
    the elastic-net term) from one call; returns (grad, loss, yhat).  On the
    rows path the squared residuals are summed in the gradient's own pass."""
    sfx = SUFFIX[X.dtype]
    nf, nt, ntasks, nobs = _dims(X, M)
    _need(X, "X", (nobs, ntasks, nf), X.dtype)
    _need(M, "M", (ntasks, nt, nf), X.dtype)
    flags = capi.GRAD_REGULARIZE if regularize else 0
    if Y is None:
        flags |= capi.GRAD_Y_ZERO
    else:
        _need(Y, "Y", (nobs, ntasks, nt), X.dtype)
    if yhat_out is None:
        yhat_out = torch.empty((nobs, ntasks, nt), dtype=X.dtype, device=X.device)
    _need(yhat_out, "yhat_out", (nobs, ntasks, nt), X.dtype)
    if out is None:
        out = torch.empty((ntasks, nt, nf), dtype=X.dtype, device=X.device)
    if loss_out is None:
        loss_out = torch.empty((1,), dtype=X.dtype, device=X.device)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    capi.call(f"glmb_gradient_loss_{sfx}", _ptr(X), _ptr(M), _ptr(Y), _ptr(out), _ptr(yhat_out), _ptr(loss_out),
              nf, nt, ntasks, nobs, float(lam), float(alpha), flags, ws_ptr, ws_bytes, _stream(stream))
    return out, loss_out, yhat_out


def gradient_partial(X, M, Y, out=None, yhat_out=None, workspace=None, stream=None):
    """sum_obs (Yhat - Y) X as float64 (no factor 2, no elastic-net term)."""
    sfx = SUFFIX[X.dtype]
    nf, nt, ntasks, nobs = _dims(X, M)
    flags = 0
    if Y is None:
        flags |= capi.GRAD_Y_ZERO
    else:
        _need(Y, "Y", (nobs, ntasks, nt), X.dtype)
    if yhat_out is not None:
        flags |= capi.GRAD_WRITE_YHAT
    if out is None:
        out = torch.empty((ntasks, nt, nf), dtype=torch.float64, device=X.device)
    _need(out, "out", (ntasks, nt, nf), torch.float64)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    capi.call(f"glmb_gradient_partial_{sfx}", _ptr(X), _ptr(M), _ptr(Y), _ptr(out), _ptr(yhat_out),
              nf, nt, ntasks, nobs, flags, ws_ptr, ws_bytes, _stream(stream))
    return out


def gradient_finalize(partial, M, lam: float = 0.0, alpha: float = 0.0, regularize: bool = True,
                      out=None, stream=None):
    """grad = 2*partial + lam*(alpha*sign(M) + 2*(1-alpha)*M)."""
    sfx = SUFFIX[M.dtype]
    ntasks, nt, nf = M.shape
    _need(partial, "partial", (ntasks, nt, nf), torch.float64)
    if out is None:
        out = torch.empty_like(M)
    capi.call(f"glmb_gradient_finalize_{sfx}", _ptr(partial), _ptr(M), _ptr(out), nf, nt, ntasks,
              float(lam), float(alpha), capi.GRAD_REGULARIZE if regularize else 0, _stream(stream))
    return out


def prox_step(beta, grad_smooth, inv_L: float, l1: float, stream=None):
    sfx = SUFFIX[beta.dtype]
    capi.call(f"glmb_prox_step_{sfx}", _ptr(beta), _ptr(grad_smooth), beta.numel(), float(inv_L),
              float(l1), _stream(stream))
    return beta


def prox_update(partial, beta, lipschitz, lambda1: float, lambda2: float, stream=None):
    sfx = SUFFIX[beta.dtype]
    ntasks, nt, nf = beta.shape
    capi.call(f"glmb_prox_update_{sfx}", _ptr(partial), _ptr(beta), _ptr(lipschitz), nf, nt, ntasks,
              float(lambda1), float(lambda2), _stream(stream))
    return beta


def power_init(v, seed: int, stream=None):
    """v: (ntasks, 1, nfeatures) start vector of the power iteration."""
    sfx = SUFFIX[v.dtype]
    ntasks, _, nf = v.shape
    capi.call(f"glmb_power_init_{sfx}", _ptr(v), nf, ntasks, int(seed) & (2**64 - 1), _stream(stream))
    return v


def power_step(partial, v, norm, lipschitz, lambda2: float, stream=None):
    sfx = SUFFIX[v.dtype]
    ntasks, _, nf = v.shape
    capi.call(f"glmb_power_step_{sfx}", _ptr(partial), _ptr(v), _ptr(norm), _ptr(lipschitz), nf,
              ntasks, float(lambda2), _stream(stream))
    return v


def fit_elastic_net(X, Y, lambda1: float, lambda2: float, n_power: int = 20, n_iter: int = 200,
                    seed: int = 42, beta=None, lipschitz=None, workspace=None, stream=None):
    """Single-GPU ISTA fit; returns (beta, lipschitz per task)."""
    sfx = SUFFIX[X.dtype]
    nobs, ntasks, nf = X.shape
    nt = Y.shape[2]
    if beta is None:
        beta = torch.empty((ntasks, nt, nf), dtype=X.dtype, device=X.device)
    if lipschitz is None:
        lipschitz = torch.empty((ntasks,), dtype=torch.float64, device=X.device)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    capi.call(f"glmb_fit_elastic_net_{sfx}", _ptr(X), _ptr(Y), _ptr(beta), _ptr(lipschitz), nf, nt,
              ntasks, nobs, float(lambda1), float(lambda2), int(n_power), int(n_iter),
              int(seed) & (2**64 - 1), ws_ptr, ws_bytes, _stream(stream))
    return beta, lipschitz
