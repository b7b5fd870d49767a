"""glmb_gradient_noalloc_f32: the gradient entry point that allocates no
device memory, for callers that may not allocate (a host that owns every
device buffer and passes only inputs and outputs, a fixed memory budget, a
path that must not wait on the allocator).

It is checked through the C ABI against glmb_gradient_f32 -- the entry point
that takes scratch from the caller or from cudaMallocAsync -- on two calls in
a row with different shapes, so the second call runs over the first call's
leftovers in the shared scratch array.  Tolerance: the float32 bar of the
parity tests, max relative error <= 1e-4 (on all-positive data, where no
gradient element is near zero).  This file is collected last on purpose.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_algos_b200 import capi  # noqa: E402
from tests import gpu_util as G  # noqa: E402

RTOL = 1e-4


def _positive(nobs, ntasks, nf, nt, seed):
    rng = np.random.default_rng(seed)
    X = rng.uniform(0, 1, (nobs, ntasks, nf)).astype(np.float32)
    M = rng.uniform(0, 1, (ntasks, nt, nf)).astype(np.float32)
    Y = rng.uniform(0, 1, (nobs, ntasks, nt)).astype(np.float32)
    return X, M, Y


def _both(X, M, Y, lam, alpha, flags):
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    dX, dM, dY = G.Dev(X), G.Dev(M), G.Dev(Y)
    out = {}
    for name in ("glmb_gradient_f32", "glmb_gradient_noalloc_f32"):
        g = G.Dev(shape=(ntasks, nt, nf), dtype=np.float32)
        yh = G.Dev(shape=(nobs, ntasks, nt), dtype=np.float32)
        args = [dX.ptr, dM.ptr, dY.ptr, g.ptr, yh.ptr, nf, nt, ntasks, nobs, lam, alpha, flags]
        if name == "glmb_gradient_f32":
            args += [None, 0]
        capi.call(name, *args, G.stream())
        torch.cuda.synchronize()
        assert g.canary_intact() and yh.canary_intact()
        out[name] = (g.numpy(), yh.numpy())
    return out["glmb_gradient_f32"], out["glmb_gradient_noalloc_f32"]


def test_noalloc_matches_allocating_entry_point_twice():
    # call 1: the benchmark's single-task shape, smaller nobs
    X, M, Y = _positive(300_000, 1, 128, 1, seed=1)
    (g_ref, _), (g_na, _) = _both(X, M, Y, 0.01, 0.0, capi.GRAD_REGULARIZE)
    assert G.rel_err(g_na, g_ref) <= RTOL
    # call 2: another shape (3 tasks, 2 targets, 64 features) with predictions
    X, M, Y = _positive(50_001, 3, 64, 2, seed=2)
    flags = capi.GRAD_REGULARIZE | capi.GRAD_WRITE_YHAT
    (g_ref, y_ref), (g_na, y_na) = _both(X, M, Y, 0.2, 0.5, flags)
    assert G.rel_err(g_na, g_ref) <= RTOL
    assert G.rel_err(y_na, y_ref) <= RTOL


def test_noalloc_rejects_sizes_beyond_its_scratch():
    buf = torch.zeros(64, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    L = capi.lib()
    # 1024 tasks x 1 target x 1024 features = 1,048,576 partial sums > 524,288
    st = L.glmb_gradient_noalloc_f32(p, p, p, p, None, 1024, 1, 1024, 16, 0.0, 0.0, 0, G.stream())
    assert st == capi.GLMB_ERR_TOO_LARGE
