"""Parity of the loss kernels (``glmb_loss_<type>``, ``glmb_gradient_loss_<f32|f64>``)
with the oracle's restatement of the reference's loss
(include/cuda/kernels/glm/glm_loss_myyhat.cuh:365-401), through the C ABI.

Integer types are bit-exact (arithmetic modulo 2^bits); float32 within
1e-4 and float64 within 1e-11 of the oracle, and both close to the exact
(float64 / long) sum; half within its own rounding.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_algos_b200 import capi  # noqa: E402
from tests import gpu_util as G  # noqa: E402

TYPES = [np.float16, np.float32, np.float64, np.int8, np.int16, np.int32, np.int64,
         np.uint8, np.uint16, np.uint32, np.uint64]


def _arrays(dt, nobs, ntasks, nf, nt, seed):
    rng = np.random.default_rng(seed)
    if np.issubdtype(dt, np.integer):
        info = np.iinfo(dt)
        lo, hi = (0, 60) if info.min == 0 else (-60, 60)
        mk = lambda s: rng.integers(lo, hi, s).astype(dt)  # noqa: E731
    else:
        mk = lambda s: rng.uniform(-1, 1, s).astype(dt)  # noqa: E731
    return mk((ntasks, nt, nf)), mk((nobs, ntasks, nt)), mk((nobs, ntasks, nt))


def _gpu_loss(M, Y, Yhat, lam, alpha, workspace=None):
    dt = M.dtype
    ntasks, nt, nf = M.shape
    nobs = Yhat.shape[0]
    dM, dYh = G.Dev(M), G.Dev(Yhat)
    dY = G.Dev(Y) if Y is not None else None
    out = G.Dev(shape=(1,), dtype=dt)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel())
    capi.call(f"glmb_loss_{G.SFX[dt]}", dM.ptr, dY.ptr if dY else None, dYh.ptr, out.ptr, nf, nt, ntasks,
              nobs, float(lam), float(alpha), ws_ptr, ws_bytes, G.stream())
    torch.cuda.synchronize()
    assert out.canary_intact()
    return out.numpy()[0]


def _exact_float_loss(M, Y, Yhat, lam, alpha):
    e = Yhat.astype(np.float64) - Y.astype(np.float64)
    m = M.astype(np.float64)
    lam_t, alp_t = float(M.dtype.type(lam)), float(M.dtype.type(alpha))
    return float(np.sum(e * e) + lam_t * (alp_t * np.abs(m).sum() + (1 - alp_t) * (m * m).sum()))


@pytest.mark.parametrize("dt", TYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("shape", [(1, 1, 1, 1), (1000, 3, 7, 5), (4097, 2, 33, 9), (70000, 1, 16, 3)])
@pytest.mark.parametrize("lam_alpha", [(0.0, 0.0), (0.7, 0.3), (2.0, 0.0), (3.0, 1.0)])
def test_loss_matches_oracle(dt, shape, lam_alpha, oracle):
    nobs, ntasks, nf, nt = shape
    lam, alpha = lam_alpha
    M, Y, Yhat = _arrays(np.dtype(dt), nobs, ntasks, nf, nt, seed=nobs + nt)
    if dt == np.float16 and _exact_float_loss(M, Y, Yhat, lam, alpha) > 6e4:
        pytest.skip("the loss of this shape overflows half")
    got = _gpu_loss(M, Y, Yhat, lam, alpha)
    ref = oracle.loss(M, Y, Yhat, lam, alpha)[0]
    if np.issubdtype(dt, np.integer):
        assert got == ref, (got, ref)
    else:
        exact = _exact_float_loss(M, Y, Yhat, lam, alpha)
        tol = {np.float16: 2e-3, np.float32: 1e-4, np.float64: 1e-11}[dt]
        assert abs(float(got) - float(ref)) <= tol * abs(float(ref)) + 1e-30
        # the device sums in double: as close to the exact sum as the output type allows
        tight = {np.float16: 1e-3, np.float32: 1e-6, np.float64: 1e-13}[dt]
        assert abs(float(got) - exact) <= tight * abs(exact) + 1e-30


@pytest.mark.parametrize("dt", [np.float32, np.float64, np.int32, np.uint8])
def test_loss_edge_cases(dt, oracle):
    dt = np.dtype(dt)
    # no observations: the model term alone; Y absent: zeros
    M, Y, Yhat = _arrays(dt, 0, 2, 5, 3, seed=3)
    got = _gpu_loss(M, Y, Yhat, 2.0, 0.5)
    ref = oracle.loss(M, Y, Yhat, 2.0, 0.5)[0]
    assert got == ref if dt.kind in "iu" else abs(float(got) - float(ref)) <= 1e-5 * abs(float(ref))
    M, Y, Yhat = _arrays(dt, 300, 2, 5, 3, seed=4)
    got = _gpu_loss(M, None, Yhat, 0.0, 0.0)
    ref = oracle.loss(M, np.zeros_like(Yhat), Yhat, 0.0, 0.0)[0]
    assert got == ref if dt.kind in "iu" else abs(float(got) - float(ref)) <= 1e-5 * abs(float(ref))
    # a caller workspace of the gradient's size is enough
    ntasks, nt, nf = M.shape
    ws_bytes = getattr(capi.lib(), f"glmb_gradient_workspace_size_{G.SFX[dt]}")(nf, nt, ntasks, 300)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    assert _gpu_loss(M, Y, Yhat, 0.7, 0.2, workspace=ws) == _gpu_loss(M, Y, Yhat, 0.7, 0.2)


def test_loss_is_deterministic():
    M, Y, Yhat = _arrays(np.dtype(np.float32), 200000, 1, 8, 8, seed=9)
    a = _gpu_loss(M, Y, Yhat, 0.1, 0.5)
    b = _gpu_loss(M, Y, Yhat, 0.1, 0.5)
    assert a.tobytes() == b.tobytes()


def _gradient_loss(X, M, Y, lam, alpha, reg=True, workspace=None):
    dt = X.dtype
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    dX, dM = G.Dev(X), G.Dev(M)
    dY = G.Dev(Y) if Y is not None else None
    g = G.Dev(shape=(ntasks, nt, nf), dtype=dt)
    yh = G.Dev(shape=(nobs, ntasks, nt), dtype=dt)
    loss = G.Dev(shape=(1,), dtype=dt)
    flags = (capi.GRAD_REGULARIZE if reg else 0) | (capi.GRAD_Y_ZERO if Y is None else 0)
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel())
    capi.call(f"glmb_gradient_loss_{G.SFX[dt]}", dX.ptr, dM.ptr, dY.ptr if dY else None, g.ptr, yh.ptr,
              loss.ptr, nf, nt, ntasks, nobs, float(lam), float(alpha), flags, ws_ptr, ws_bytes, G.stream())
    torch.cuda.synchronize()
    path = capi.last_path()
    assert g.canary_intact() and yh.canary_intact() and loss.canary_intact()
    return g.numpy(), loss.numpy()[0], yh.numpy(), path


# On the rows path the kernel sums the squared residuals itself (each r formed
# in the input precision, squared and summed in double): the same value as
# glmb_loss on the written Yhat up to the rounding of r and the order of the
# sum.  The other paths run glmb_loss's own kernels on that Yhat: identical.
FUSED_TOL = {np.float32: 1e-6, np.float64: 1e-13}


@pytest.mark.parametrize("dt,shape,path", [
    (np.float32, (5000, 2, 64, 3), "rows"),      # 16-lane row segments
    (np.float32, (5000, 2, 8, 3), "rows"),       # 2-lane row segments
    (np.float32, (5000, 2, 128, 3), "rows"),     # one row per warp
    (np.float32, (70001, 1, 128, 1), "rows"),    # one row per warp, 8-row batches, ragged end
    (np.float32, (3001, 3, 33, 2), "rows"),      # unaligned rows: scalar loads
    (np.float64, (5000, 2, 64, 3), "rows"),
    (np.float64, (9999, 1, 20, 7), "rows"),
    (np.float32, (3000, 2, 128, 40), "dense"),
    (np.float64, (3000, 3, 64, 16), "tiles"),
    (np.float32, (2000, 2, 30, 12), "generic"),
])
def test_gradient_loss_on_every_path(dt, shape, path, oracle):
    nobs, ntasks, nf, nt = shape
    rng = np.random.default_rng(nobs + nf)
    X = rng.uniform(-1, 1, (nobs, ntasks, nf)).astype(dt)
    M = rng.normal(size=(ntasks, nt, nf)).astype(dt)
    Y = rng.normal(size=(nobs, ntasks, nt)).astype(dt)
    g, loss, yh, got_path = _gradient_loss(X, M, Y, 0.3, 0.4)
    assert got_path == path
    # the gradient is exactly the plain call's; on the rows path so is the
    # prediction (the same kernel's dot products)
    assert np.array_equal(g, G.gradient(X, M, Y, 0.3, 0.4, reg=True))
    if path == "rows":
        assert np.array_equal(yh, G.predict(X, M))
    two_pass = _gpu_loss(M, Y, yh, 0.3, 0.4)
    if path == "rows":
        assert abs(float(loss) - float(two_pass)) <= FUSED_TOL[dt] * abs(float(two_pass))
    else:
        assert two_pass.tobytes() == np.asarray(loss).tobytes()
    # and the loss agrees with the oracle's on the oracle's own prediction
    ref = oracle.loss(M, Y, oracle.predict(X, M), 0.3, 0.4)[0]
    tol = 1e-4 if dt == np.float32 else 1e-11
    assert abs(float(loss) - float(ref)) <= tol * abs(float(ref))


@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_gradient_loss_fused_edge_cases(dt, oracle):
    dt = np.dtype(dt)
    rng = np.random.default_rng(21)
    nobs, ntasks, nf, nt = 4099, 2, 32, 2
    X = rng.uniform(-1, 1, (nobs, ntasks, nf)).astype(dt)
    M = rng.normal(size=(ntasks, nt, nf)).astype(dt)
    Y = rng.normal(size=(nobs, ntasks, nt)).astype(dt)
    tol = 1e-4 if dt == np.float32 else 1e-11
    # Y absent (zeros); the gradient unregularised while the loss keeps its elastic-net term
    g, loss, _, path = _gradient_loss(X, M, None, 0.5, 0.25, reg=False)
    assert path == "rows"
    assert np.array_equal(g, G.gradient(X, M, None, 0.0, 0.0, reg=False))
    ref = oracle.loss(M, np.zeros((nobs, ntasks, nt), dt), oracle.predict(X, M), 0.5, 0.25)[0]
    assert abs(float(loss) - float(ref)) <= tol * abs(float(ref))
    # no observations: the model term alone, the gradient the elastic-net term alone
    g0, loss0, _, path = _gradient_loss(X[:0], M, Y[:0], 0.5, 0.25)
    ref0 = oracle.loss(M, Y[:0], Y[:0], 0.5, 0.25)[0]
    assert abs(float(loss0) - float(ref0)) <= tol * abs(float(ref0))
    assert np.array_equal(g0, G.gradient(X[:0], M, Y[:0], 0.5, 0.25, reg=True))
    # a caller workspace of the gradient's queried size holds the loss partials too; deterministic
    ws_bytes = getattr(capi.lib(), f"glmb_gradient_workspace_size_{G.SFX[dt]}")(nf, nt, ntasks, nobs)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    before = capi.launch_count()
    a = _gradient_loss(X, M, Y, 0.3, 0.4, workspace=ws)
    b = _gradient_loss(X, M, Y, 0.3, 0.4)
    assert a[3] == "rows"
    assert a[1].tobytes() == b[1].tobytes() and np.array_equal(a[0], b[0])
    # fused: rows kernel, finalize, loss scalar -- three launches per call
    assert capi.launch_count() - before == 6
