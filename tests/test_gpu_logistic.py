"""Logistic link (GLMB_GRAD_LOGISTIC): mu = sigmoid(X M), gradient
sum_obs (mu - Y) X [+ lambda (alpha sign M + 2 (1 - alpha) M)] -- the
gradient of the logistic negative log-likelihood -- against a float64
NumPy evaluation, on the fused rows kernel (half/float/double) and on the
generic path."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_algos_b200 import capi  # noqa: E402
from tests import gpu_util as G  # noqa: E402


def _problem(dt, nobs, ntasks, nf, nt, seed):
    rng = np.random.default_rng(seed)
    X = (rng.normal(size=(nobs, ntasks, nf)) / np.sqrt(nf)).astype(dt)
    beta = rng.normal(size=(ntasks, nt, nf))
    eta = np.einsum("otf,tkf->otk", X.astype(np.float64), beta)
    Y = (rng.uniform(size=eta.shape) < 1 / (1 + np.exp(-eta))).astype(dt)  # Bernoulli labels
    M = (rng.normal(size=(ntasks, nt, nf)) * 0.5).astype(dt)
    return X, M, Y


def _reference(X, M, Y, lam, alpha, reg):
    x, m, y = X.astype(np.float64), M.astype(np.float64), Y.astype(np.float64)
    mu = 1 / (1 + np.exp(-np.einsum("otf,tkf->otk", x, m)))
    g = np.einsum("otk,otf->tkf", mu - y, x)
    if reg:
        g = g + lam * (alpha * np.sign(m) + 2 * (1 - alpha) * m)
    return g, mu


def _logistic_gradient(X, M, Y, lam, alpha, reg, want_yhat):
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    dX, dM = G.Dev(X), G.Dev(M)
    dY = G.Dev(Y) if Y is not None else None
    g = G.Dev(shape=(ntasks, nt, nf), dtype=X.dtype)
    yh = G.Dev(shape=(nobs, ntasks, nt), dtype=X.dtype) if want_yhat else None
    flags = capi.GRAD_LOGISTIC | (capi.GRAD_REGULARIZE if reg else 0) | (capi.GRAD_WRITE_YHAT if want_yhat else 0)
    if Y is None:
        flags |= capi.GRAD_Y_ZERO
    capi.call(f"glmb_gradient_{G.SFX[X.dtype]}", dX.ptr, dM.ptr, dY.ptr if dY else None, g.ptr,
              yh.ptr if yh else None, nf, nt, ntasks, nobs, float(lam), float(alpha), flags, None, 0, G.stream())
    torch.cuda.synchronize()
    path = capi.last_path()
    assert g.canary_intact()
    return g.numpy(), (yh.numpy() if yh else None), path


CASES = [
    (np.float32, (50000, 1, 128, 1), "rows"),
    (np.float32, (3000, 3, 64, 4), "rows"),
    (np.float32, (2000, 2, 64, 16), "generic"),   # many targets: dense is identity-link only
    (np.float64, (20000, 2, 96, 2), "rows"),
    (np.float64, (1500, 2, 64, 16), "generic"),   # tiles is identity-link only
    (np.float16, (20000, 1, 128, 1), "rows"),
    (np.float16, (700, 2, 40, 3), "rows"),
]


@pytest.mark.parametrize("dt,shape,path", CASES, ids=[f"{np.dtype(d).name}-{s}" for d, s, _ in CASES])
def test_logistic_gradient(dt, shape, path):
    nobs, ntasks, nf, nt = shape
    X, M, Y = _problem(dt, nobs, ntasks, nf, nt, seed=nobs + nt)
    g, mu, got_path = _logistic_gradient(X, M, Y, 0.3, 0.4, True, True)
    assert got_path == path
    ref, ref_mu = _reference(X, M, Y, 0.3, 0.4, True)
    tol = {np.float16: 2.0 ** -7, np.float32: 1e-4, np.float64: 1e-11}[dt]
    floor = 1e-3 * np.abs(ref).max()
    assert G.rel_err(g, ref, floor=floor) <= tol
    assert G.rel_err(mu, ref_mu) <= tol * (4 if dt == np.float16 else 1)
    # without Y (labels all 0) and without the elastic-net term
    g0, _, _ = _logistic_gradient(X, M, None, 0.0, 0.0, False, False)
    ref0, _ = _reference(X, M, np.zeros_like(Y), 0.0, 0.0, False)
    assert G.rel_err(g0, ref0, floor=1e-3 * np.abs(ref0).max()) <= tol


def test_logistic_rejections():
    X, M, Y = _problem(np.float32, 100, 1, 8, 1, seed=1)
    Xi, Mi, Yi = (a.astype(np.int32) for a in (X, M, Y))
    dX, dM, dY = G.Dev(Xi), G.Dev(Mi), G.Dev(Yi)
    g = G.Dev(shape=(1, 1, 8), dtype=np.int32)
    st = capi.lib().glmb_gradient_i32(dX.ptr, dM.ptr, dY.ptr, g.ptr, None, 8, 1, 1, 100, 0.0, 0.0,
                                      capi.GRAD_LOGISTIC, None, 0, G.stream())
    assert st == capi.GLMB_ERR_INVALID_VALUE
    dX, dM, dY = G.Dev(X), G.Dev(M), G.Dev(Y)
    g, yh, loss = G.Dev(shape=(1, 1, 8), dtype=np.float32), G.Dev(shape=(100, 1, 1), dtype=np.float32), \
        G.Dev(shape=(1,), dtype=np.float32)
    st = capi.lib().glmb_gradient_loss_f32(dX.ptr, dM.ptr, dY.ptr, g.ptr, yh.ptr, loss.ptr, 8, 1, 1, 100, 0.0, 0.0,
                                           capi.GRAD_LOGISTIC, None, 0, G.stream())
    assert st == capi.GLMB_ERR_UNSUPPORTED
