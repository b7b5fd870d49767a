"""Parity of the sm_100a GLM kernels with the oracle, through the C ABI.

Bars: max relative error <= 1e-4 for float32 and
<= 1e-11 for float64 against the oracle on the same inputs; integer types
bit-exact; half within the reference driver's own tolerance
2^-(11 - tol_bits) with tol_bits = 4.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_algos_b200 import capi  # noqa: E402
from tests import gpu_util as G  # noqa: E402

RTOL = {np.dtype(np.float32): 1e-4, np.dtype(np.float64): 1e-11, np.dtype(np.float16): 2.0 ** -7}


def _inputs(dt, nobs, ntasks, nf, nt, seed=0, positive=True):
    rng = np.random.default_rng(seed)
    if np.issubdtype(dt, np.integer):
        info = np.iinfo(dt)
        lo, hi = (0, 100) if info.min == 0 else (-100, 100)
        mk = lambda s: rng.integers(lo, hi, s).astype(dt)  # noqa: E731
    elif positive:
        mk = lambda s: rng.uniform(0, 1, s).astype(dt)  # noqa: E731
    else:
        mk = lambda s: rng.uniform(-1, 1, s).astype(dt)  # noqa: E731
    return mk((nobs, ntasks, nf)), mk((ntasks, nt, nf)), mk((nobs, ntasks, nt))


def _check_float(actual, expected, dt, scale=None, what=""):
    rtol = RTOL[np.dtype(dt)]
    a = actual.astype(np.float64)
    e = expected.astype(np.float64)
    if scale is None:
        r = G.rel_err(a, e)
        assert r <= rtol, f"{what}: max rel err {r:.3e} > {rtol:.1e}"
    else:
        err = np.abs(a - e)
        assert np.all(err <= rtol * (np.abs(e) + scale)), f"{what}: {np.max(err / (np.abs(e) + scale)):.3e}"


def test_golden_cases_through_cabi(golden, oracle):
    for name, c in golden.items():
        X, M, Y = c["X"], c["M"], c["Y"]
        g, yh = G.gradient(X, M, Y, reg=False, want_yhat=True)
        p = G.predict(X, M)
        if np.issubdtype(X.dtype, np.integer):
            assert np.array_equal(g, c["grad"]), name
            assert np.array_equal(p, c["yhat"]), name
            assert np.array_equal(yh, c["yhat"]), name
        else:
            Xd, Md = X.astype(np.float64), M.astype(np.float64)
            pscale = np.einsum("otf,tkf->otk", np.abs(Xd), np.abs(Md))
            _check_float(p, c["yhat"], X.dtype, pscale, name + " predict")
            _check_float(yh, c["yhat"], X.dtype, pscale, name + " yhat")
            og = oracle.gradient(X, M, Y, with_reg=False)
            _check_float(g, og, X.dtype, what=name + " grad vs oracle")
            _check_float(g, c["grad"], X.dtype, what=name + " grad vs golden")


@pytest.mark.parametrize("dt", [np.float32, np.float64])
@pytest.mark.parametrize("nf", [1, 3, 4, 8, 20, 24, 32, 33, 48, 60, 64, 100, 128, 255, 256, 512, 1000, 1025])
@pytest.mark.parametrize("nt", [1, 2, 3, 8, 9])
def test_shapes_float(dt, nf, nt, oracle):
    for (nobs, ntasks) in ((1, 1), (33, 3), (1025, 1), (4097, 2)):
        X, M, Y = _inputs(dt, nobs, ntasks, nf, nt, seed=nf * 31 + nt)
        g, yh = G.gradient(X, M, Y, lam=0.3, alpha=0.4, reg=True, want_yhat=True)
        path = capi.last_path()
        _check_float(g, oracle.gradient(X, M, Y, 0.3, 0.4, True), dt, what=f"grad {nobs},{ntasks},{nf},{nt} [{path}]")
        _check_float(yh, oracle.predict(X, M), dt, what=f"yhat {nobs},{ntasks},{nf},{nt}")
        _check_float(G.predict(X, M), oracle.predict(X, M), dt, what=f"predict {nobs},{ntasks},{nf},{nt}")


def test_rows_path_is_used_for_hot_shapes():
    X, M, Y = _inputs(np.float32, 4096, 1, 128, 1)
    G.gradient(X, M, Y)
    assert capi.last_path() == "rows"
    X, M, Y = _inputs(np.float64, 4096, 3, 256, 1)
    G.gradient(X, M, Y)
    assert capi.last_path() == "rows"
    X, M, Y = _inputs(np.float32, 512, 2, 64, 16)
    G.gradient(X, M, Y)
    assert capi.last_path() == "dense"
    X, M, Y = _inputs(np.float32, 512, 2, 30, 16)  # features not a multiple of 4
    G.gradient(X, M, Y)
    assert capi.last_path() == "generic"


@pytest.mark.parametrize("dt", [np.float16, np.int8, np.int16, np.int32, np.int64,
                                np.uint8, np.uint16, np.uint32, np.uint64])
@pytest.mark.parametrize("shape", [(1, 1, 1, 1), (8, 2, 8, 3), (33, 3, 33, 2), (1025, 1, 24, 1)])
def test_other_types(dt, shape, oracle):
    nobs, ntasks, nf, nt = shape
    X, M, Y = _inputs(dt, nobs, ntasks, nf, nt, seed=nobs + nf)
    if dt == np.float16:
        # keep sums representable in binary16
        X = (X.astype(np.float32) / 8).astype(dt)
        Y = (Y.astype(np.float32) / 8).astype(dt)
    lam, alpha = (2.9, 0.5) if np.issubdtype(dt, np.integer) else (0.25, 0.5)
    g, yh = G.gradient(X, M, Y, lam, alpha, reg=True, want_yhat=True)
    og = oracle.gradient(X, M, Y, lam, alpha, True)
    oy = oracle.predict(X, M)
    if np.issubdtype(dt, np.integer):
        assert np.array_equal(g, og)
        assert np.array_equal(yh, oy)
        assert np.array_equal(G.predict(X, M), oy)
    else:
        _check_float(g, og, dt, scale=np.abs(og.astype(np.float64)).max() * 1e-2, what="half grad")
        _check_float(yh, oy, dt, what="half yhat")


def test_driver_shape_config1(golden, oracle):
    c = golden["driver_f32_32x1x1x8192"]
    X, M, Y = c["X"], c["M"], c["Y"]
    g = G.gradient(X, M, Y, lam=0.1, alpha=0.0, reg=True)
    og = oracle.gradient(X, M, Y, 0.1, 0.0, True)
    assert G.rel_err(g, og) <= 1e-4
    g0 = G.gradient(X, M, Y, reg=False)
    assert G.rel_err(g0, c["grad"]) <= 1e-4


def test_large_nobs_against_double_oracle(oracle):
    rng = np.random.default_rng(1)
    nobs, nf = 1 << 20, 128
    X = rng.uniform(-1, 1, (nobs, 1, nf)).astype(np.float32)
    b = rng.normal(size=(1, 1, nf)).astype(np.float32)
    Y = (X[:, 0, :].astype(np.float64) @ b[0, 0].astype(np.float64) + rng.normal(0, 0.1, nobs))
    Y = Y.astype(np.float32).reshape(nobs, 1, 1)
    g = G.gradient(X, b, Y, lam=0.01, alpha=0.0, reg=True)
    ref = oracle.gradient_acc64(X, b, Y, 0.01, 0.0, True)
    # elementwise, with the conditioning of each sum as the floor
    resid = np.abs(X[:, 0, :].astype(np.float64) @ b[0, 0].astype(np.float64) - Y[:, 0, 0])
    scale = 2 * (resid @ np.abs(X[:, 0, :].astype(np.float64)))
    err = np.abs(g.astype(np.float64) - ref)[0, 0]
    assert np.all(err <= 1e-4 * np.abs(ref[0, 0]) + 1e-6 * scale)
    assert np.linalg.norm(g - ref) / np.linalg.norm(ref) < 1e-5


def test_partial_finalize_matches_single_call():
    X, M, Y = _inputs(np.float32, 3000, 2, 128, 2, positive=False)
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    dX, dM, dY = G.Dev(X), G.Dev(M), G.Dev(Y)
    part = G.Dev(shape=(ntasks, nt, nf), dtype=np.float64)
    capi.call("glmb_gradient_partial_f32", dX.ptr, dM.ptr, dY.ptr, part.ptr, None, nf, nt, ntasks, nobs,
              0, None, 0, G.stream())
    g = G.Dev(shape=(ntasks, nt, nf), dtype=np.float32)
    capi.call("glmb_gradient_finalize_f32", part.ptr, dM.ptr, g.ptr, nf, nt, ntasks, 0.2, 0.3,
              capi.GRAD_REGULARIZE, G.stream())
    torch.cuda.synchronize()
    single = G.gradient(X, M, Y, 0.2, 0.3, reg=True)
    assert np.array_equal(g.numpy(), single)


def test_obs_shards_sum_to_full_gradient(oracle):
    X, M, Y = _inputs(np.float64, 5000, 1, 64, 1, positive=False)
    nf, nt, ntasks = 64, 1, 1
    total = np.zeros((ntasks, nt, nf))
    for lo, hi in ((0, 1234), (1234, 3000), (3000, 5000)):
        dX, dM, dY = G.Dev(X[lo:hi]), G.Dev(M), G.Dev(Y[lo:hi])
        part = G.Dev(shape=(ntasks, nt, nf), dtype=np.float64)
        capi.call("glmb_gradient_partial_f64", dX.ptr, dM.ptr, dY.ptr, part.ptr, None, nf, nt, ntasks,
                  hi - lo, 0, None, 0, G.stream())
        torch.cuda.synchronize()
        total += part.numpy()
    dP, dM = G.Dev(total), G.Dev(M)
    g = G.Dev(shape=(ntasks, nt, nf), dtype=np.float64)
    capi.call("glmb_gradient_finalize_f64", dP.ptr, dM.ptr, g.ptr, nf, nt, ntasks, 0.5, 0.5,
              capi.GRAD_REGULARIZE, G.stream())
    torch.cuda.synchronize()
    og = oracle.gradient(X, M, Y, 0.5, 0.5, True)
    assert G.rel_err(g.numpy(), og, floor=1e-6 * np.abs(og).max()) <= 1e-11


def test_y_zero_flag_and_explicit_workspace(oracle):
    X, M, _ = _inputs(np.float32, 2049, 2, 96, 3)
    g = G.gradient(X, M, None, reg=False)
    assert G.rel_err(g, oracle.gradient(X, M, None, with_reg=False)) <= 1e-4
    nbytes = capi.lib().glmb_gradient_workspace_size_f32(96, 3, 2, 2049)
    assert nbytes > 0
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    Xp, Mp, Yp = _inputs(np.float32, 2049, 2, 96, 3, seed=4)
    a = G.gradient(Xp, Mp, Yp, 0.1, 0.2, workspace=ws)
    b = G.gradient(Xp, Mp, Yp, 0.1, 0.2)
    assert np.array_equal(a, b)


def test_deterministic():
    X, M, Y = _inputs(np.float32, 100000, 1, 128, 1, positive=False)
    a = G.gradient(X, M, Y, 0.01, 0.0)
    b = G.gradient(X, M, Y, 0.01, 0.0)
    assert np.array_equal(a, b)


def test_invalid_arguments_return_status():
    L = capi.lib()
    s = G.stream()
    assert L.glmb_gradient_f32(None, None, None, None, None, -1, 1, 1, 1, 0.0, 0.0, 0, None, 0, s) == capi.GLMB_ERR_INVALID_VALUE
    assert L.glmb_gradient_f32(None, None, None, None, None, 4, 1, 1, 8, 0.0, 0.0, 0, None, 0, s) == capi.GLMB_ERR_INVALID_VALUE
    assert L.glmb_gradient_f32(None, None, None, None, None, 4, 1, 1, 8, 0.0, 0.0, 0x80, None, 0, s) == capi.GLMB_ERR_INVALID_VALUE
    assert L.glmb_predict_f64(None, None, None, 4, 1, 1, 8, s) == capi.GLMB_ERR_INVALID_VALUE
    X, M, Y = _inputs(np.float32, 4096, 1, 128, 1)
    dX, dM, dY = G.Dev(X), G.Dev(M), G.Dev(Y)
    g = G.Dev(shape=(1, 1, 128), dtype=np.float32)
    tiny = torch.empty(8, dtype=torch.uint8, device="cuda")
    st = L.glmb_gradient_f32(dX.ptr, dM.ptr, dY.ptr, g.ptr, None, 128, 1, 1, 4096, 0.0, 0.0, 0,
                             tiny.data_ptr(), 8, s)
    assert st == capi.GLMB_ERR_WORKSPACE
    # empty problems are valid no-ops; nobs == 0 gives the regularisation term alone
    assert L.glmb_gradient_f32(None, None, None, None, None, 4, 0, 1, 8, 0.0, 0.0, 0, None, 0, s) == 0
    g2 = G.gradient(np.zeros((0, 1, 4), np.float32), np.ones((1, 1, 4), np.float32),
                    np.zeros((0, 1, 1), np.float32), lam=0.5, alpha=0.0)
    assert np.allclose(g2, 1.0)


@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_fit_matches_oracle(dt, oracle):
    rng = np.random.default_rng(5)
    nobs, nf = 8192, 48
    X = rng.normal(size=(nobs, 1, nf)).astype(dt)
    bt = np.where(rng.uniform(size=nf) < 0.2, rng.normal(size=nf), 0.0)
    Y = (X[:, 0, :].astype(np.float64) @ bt + rng.normal(0, 0.1, nobs)).astype(dt).reshape(nobs, 1, 1)
    l1, l2, seed = 50.0, 10.0, 77
    v0 = oracle.power_start(nf, seed)
    ob, olip = oracle.fit(X, Y, l1, l2, v0, n_power=20, n_iter=100)
    from gpu_algos_b200 import glm
    tX, tY = torch.from_numpy(X).cuda(), torch.from_numpy(Y).cuda()
    beta, lip = glm.fit_elastic_net(tX, tY, l1, l2, n_power=20, n_iter=100, seed=seed)
    torch.cuda.synchronize()
    tol = 1e-4 if dt == np.float32 else 1e-10
    assert abs(lip.item() - olip[0]) <= tol * olip[0]
    b = beta.cpu().numpy()
    assert np.max(np.abs(b - ob)) <= tol * np.max(np.abs(ob))
    assert np.array_equal(b == 0, ob == 0) or dt == np.float32


def test_tiles_path_multitask_f64(oracle):
    # the multi-task float64 shape (64 tasks x 256 features x 16 targets), fewer observations
    rng = np.random.default_rng(33)
    nobs, ntasks, nf, nt = 1500, 64, 256, 16
    X = rng.normal(size=(nobs, ntasks, nf))
    bt = rng.normal(size=(ntasks, nt, nf))
    Y = np.einsum("otf,tkf->otk", X, bt) + 0.05 * rng.normal(size=(nobs, ntasks, nt))
    M = rng.normal(size=(ntasks, nt, nf))
    g, yh = G.gradient(X, M, Y, lam=0.1, alpha=0.0, reg=True, want_yhat=True)
    assert capi.last_path() == "tiles"
    og = oracle.gradient(X, M, Y, 0.1, 0.0, True)
    # mixed-sign data: elements far below the gradient's scale are compared
    # relative to 1e-3 of its largest element (cancellation floor)
    assert G.rel_err(g, og, floor=1e-3 * np.abs(og).max()) <= 1e-11
    pscale = np.einsum("otf,tkf->otk", np.abs(X), np.abs(M))
    assert np.all(np.abs(yh - oracle.predict(X, M)) <= 1e-12 * pscale)
    # ragged tiles and a target count below 8
    for (nobs, ntasks, nf, nt) in ((33, 3, 10, 9), (100, 2, 256, 12), (70, 5, 64, 16), (45, 1, 2, 16)):
        X = rng.uniform(0, 1, (nobs, ntasks, nf))
        M = rng.uniform(0, 1, (ntasks, nt, nf))
        Y = rng.uniform(0, 1, (nobs, ntasks, nt))
        g = G.gradient(X, M, Y, 0.2, 0.5, reg=True)
        assert capi.last_path() == "tiles"
        assert G.rel_err(g, oracle.gradient(X, M, Y, 0.2, 0.5, True)) <= 1e-11
        g0 = G.gradient(X, M, None, reg=False)
        assert G.rel_err(g0, oracle.gradient(X, M, None, with_reg=False)) <= 1e-11


@pytest.mark.parametrize("shape", [(1, 1, 32, 9), (129, 1, 64, 16), (1000, 3, 96, 40), (4097, 1, 256, 256),
                                   (700, 2, 4096, 12), (3000, 1, 128, 300), (257, 5, 36, 129), (500, 1, 64, 700)])
def test_dense_path_float32(shape, oracle):
    """tcgen05 3xTF32 path (many targets): gradient, predictions, partials."""
    nobs, ntasks, nf, nt = shape
    X, M, Y = _inputs(np.float32, nobs, ntasks, nf, nt, seed=nobs * 7 + nt)
    g, yh = G.gradient(X, M, Y, 0.2, 0.3, reg=True, want_yhat=True)
    assert capi.last_path() == "dense"
    ref = oracle.gradient_acc64(X, M, Y, 0.2, 0.3, True)
    assert G.rel_err(g, ref) <= 1e-4
    assert G.rel_err(g, oracle.gradient(X, M, Y, 0.2, 0.3, True)) <= 1e-4
    assert G.rel_err(yh, oracle.predict(X.astype(np.float64), M.astype(np.float64))) <= 1e-4
    assert G.rel_err(G.gradient(X, M, None, reg=False), oracle.gradient_acc64(X, M, None, with_reg=False)) <= 1e-4


def _dense_problem(nobs, nf, nt, at_solution, seed=44):
    """Config-4-like data: X ~ U(-1,1)/sqrt(nf), Y = X beta + N(0, 0.01^2);
    the gradient is taken at beta itself (residuals are the noise: a small
    difference of large terms) or at an independent N(0,1) draw."""
    rng = np.random.default_rng(seed)
    X = (rng.uniform(-1, 1, (nobs, 1, nf)) / np.sqrt(nf)).astype(np.float32)
    bt = rng.normal(size=(1, nt, nf))
    Y = (np.einsum("otf,tkf->otk", X.astype(np.float64), bt) + 0.01 * rng.normal(size=(nobs, 1, nt))).astype(np.float32)
    M = (bt if at_solution else rng.normal(size=(1, nt, nf))).astype(np.float32)
    return X, M, Y


def test_dense_path_mixed_sign_with_cancellation_floor(oracle):
    X, M, Y = _dense_problem(20000, 512, 64, at_solution=False)
    g = G.gradient(X, M, Y, 0.001, 0.0, reg=True)
    assert capi.last_path() == "dense"
    ref = oracle.gradient_acc64(X, M, Y, 0.001, 0.0, True)
    assert G.rel_err(g, ref, floor=1e-3 * np.abs(ref).max()) <= 1e-4
    assert np.linalg.norm(g - ref) / np.linalg.norm(ref) <= 2e-6


def test_dense_path_at_the_solution(oracle):
    """Residuals of order 0.01 against predictions of order 0.6: the tensor
    core's round-toward-zero accumulation is bounded by the per-block drains;
    the result stays within 1e-4 of the exact gradient in norm (the fp32
    host algorithm: about 1e-5)."""
    X, M, Y = _dense_problem(20000, 512, 64, at_solution=True)
    g = G.gradient(X, M, Y, 0.001, 0.0, reg=True)
    assert capi.last_path() == "dense"
    ref = oracle.gradient_acc64(X, M, Y, 0.001, 0.0, True)
    assert np.linalg.norm(g - ref) / np.linalg.norm(ref) <= 1e-4
    assert np.abs(g - ref).max() <= 2e-4 * np.abs(ref).max()


@pytest.mark.parametrize("shape", [(100000, 1, 128, 1), (20000, 2, 64, 4), (5001, 3, 1024, 1), (777, 2, 40, 3)])
def test_half_rows_path(shape, oracle):
    """float16 inputs on the fused rows kernel (8 values per 16-byte load,
    float arithmetic): within the driver's half tolerance of the oracle."""
    nobs, ntasks, nf, nt = shape
    rng = np.random.default_rng(nobs + nf)
    X = (rng.uniform(-1, 1, (nobs, ntasks, nf)) / 4).astype(np.float16)
    M = rng.normal(size=(ntasks, nt, nf)).astype(np.float16)
    Y = (np.einsum("otf,tkf->otk", X.astype(np.float64), M.astype(np.float64))
         + 0.05 * rng.normal(size=(nobs, ntasks, nt))).astype(np.float16)
    g, yh = G.gradient(X, M, Y, 0.1, 0.5, reg=True, want_yhat=True)
    assert capi.last_path() == "rows"
    og = oracle.gradient(X, M, Y, 0.1, 0.5, True)
    exact = (2 * np.einsum("otk,otf->tkf", np.einsum("otf,tkf->otk", X.astype(np.float64), M.astype(np.float64))
                           - Y.astype(np.float64), X.astype(np.float64))
             + 0.1 * (0.5 * np.sign(M.astype(np.float64)) + 2 * 0.5 * M.astype(np.float64)))
    scale = np.abs(exact).max()
    # float arithmetic (residuals ~0.05 out of predictions ~5 lose a few bits
    # to cancellation), one rounding to half at the end: within 2^-8, tighter
    # than the driver's half tolerance 2^-7
    assert np.all(np.abs(g.astype(np.float64) - exact) <= 2.0 ** -8 * (np.abs(exact) + 1e-2 * scale))
    _check_float(g, og, np.float16, scale=scale * 1e-2, what="half grad vs oracle")
    oy = oracle.predict(X, M)  # mixed signs: predictions near zero are judged on the data's scale
    _check_float(yh, oy, np.float16, scale=np.abs(oy.astype(np.float64)).max() * 1e-2, what="half yhat")
