"""Helpers for the GPU tests: move NumPy arrays through raw device buffers
and call the C ABI (``include/glm_b200.h``) by name."""
from __future__ import annotations

import numpy as np
import torch

from gpu_algos_b200 import capi

SFX = {
    np.dtype(np.float16): "f16",
    np.dtype(np.float32): "f32",
    np.dtype(np.float64): "f64",
    np.dtype(np.int8): "i8",
    np.dtype(np.int16): "i16",
    np.dtype(np.int32): "i32",
    np.dtype(np.int64): "i64",
    np.dtype(np.uint8): "u8",
    np.dtype(np.uint16): "u16",
    np.dtype(np.uint32): "u32",
    np.dtype(np.uint64): "u64",
}

CANARY = 8  # guard elements after every device output


class Dev:
    """A device byte buffer holding a NumPy array, with a guard band."""

    def __init__(self, arr: np.ndarray | None = None, shape=None, dtype=None, fill: int = 0xA5):
        if arr is not None:
            arr = np.ascontiguousarray(arr)
            shape, dtype = arr.shape, arr.dtype
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        total = self.nbytes + CANARY * self.dtype.itemsize
        self.buf = torch.full((max(total, 16),), fill, dtype=torch.uint8, device="cuda")
        if arr is not None and self.nbytes:
            self.buf[: self.nbytes].copy_(torch.from_numpy(arr.reshape(-1).view(np.uint8)))

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    def numpy(self) -> np.ndarray:
        host = self.buf[: self.nbytes].cpu().numpy()
        return host.view(self.dtype).reshape(self.shape).copy()

    def canary_intact(self, fill: int = 0xA5) -> bool:
        tail = self.buf[self.nbytes:].cpu().numpy()
        return bool(np.all(tail == fill))


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def predict(X, M, sfx=None):
    """``sfx`` names the C-ABI type when the dtype does not (``"bf16"`` for
    bfloat16 bit patterns held as uint16)."""
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    dX, dM = Dev(X), Dev(M)
    out = Dev(shape=(nobs, ntasks, nt), dtype=X.dtype)
    capi.call(f"glmb_predict_{sfx or SFX[X.dtype]}", dX.ptr, dM.ptr, out.ptr, nf, nt, ntasks, nobs, stream())
    torch.cuda.synchronize()
    assert out.canary_intact()
    return out.numpy()


def gradient(X, M, Y, lam=0.0, alpha=0.0, reg=True, want_yhat=False, workspace=None, sfx=None, flags=0):
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    dX, dM = Dev(X), Dev(M)
    dY = Dev(Y) if Y is not None else None
    g = Dev(shape=(ntasks, nt, nf), dtype=X.dtype)
    yh = Dev(shape=(nobs, ntasks, nt), dtype=X.dtype) if want_yhat else None
    flags |= (capi.GRAD_REGULARIZE if reg else 0) | (capi.GRAD_WRITE_YHAT if want_yhat else 0)
    if Y is None:
        flags |= capi.GRAD_Y_ZERO
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel())
    capi.call(f"glmb_gradient_{sfx or SFX[X.dtype]}", dX.ptr, dM.ptr, dY.ptr if dY else None, g.ptr,
              yh.ptr if yh else None, nf, nt, ntasks, nobs, float(lam), float(alpha), flags,
              ws_ptr, ws_bytes, stream())
    torch.cuda.synchronize()
    assert g.canary_intact()
    if yh is not None:
        assert yh.canary_intact()
        return g.numpy(), yh.numpy()
    return g.numpy()


def rel_err(actual, expected, floor=0.0):
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    den = np.maximum(np.abs(e), floor)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(den > 0, np.abs(a - e) / den, np.abs(a - e))
    return float(np.max(r)) if r.size else 0.0
