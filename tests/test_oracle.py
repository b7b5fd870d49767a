"""CPU tests that pin the oracle before it is trusted as the checker.

The oracle restates the reference's host path (see ``oracle/glm_oracle.h``).
It is pinned here against

* the reference's own NumPy reference functions, through the committed
  fixtures of ``tests/golden/make_golden.py`` (float: tolerance below;
  integer: bit-exact),
* exact integer known answers of the driver's "increasing" initialisation,
* hand-computed cases for the elastic-net term, the sign rule and the loss,
* closed forms for the proximal-gradient fit (soft threshold, ridge solution,
  largest eigenvalue).
"""
import numpy as np
import pytest

RTOL = {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}


def _cond_close(actual, expected, scale, rtol):
    """|actual - expected| <= rtol * (|expected| + scale) elementwise.

    ``scale`` is the sum of absolute values of the terms that produced each
    element (the conditioning of a dot product): a near-zero dot product of
    large terms legitimately carries an absolute rounding error of order
    eps * scale.
    """
    err = np.abs(actual.astype(np.float64) - expected.astype(np.float64))
    bound = rtol * (np.abs(expected.astype(np.float64)) + scale)
    assert np.all(err <= bound), float(np.max(err / np.maximum(bound, 1e-300)))


def test_golden_predict_and_gradient(oracle, golden):
    assert len(golden) >= 40
    for name, c in golden.items():
        X, M, Y = c["X"], c["M"], c["Y"]
        yhat = oracle.predict(X, M)
        grad = oracle.gradient(X, M, Y, with_reg=False)
        if np.issubdtype(X.dtype, np.integer):
            assert np.array_equal(yhat, c["yhat"]), name
            assert np.array_equal(grad, c["grad"]), name
        else:
            rtol = RTOL[X.dtype]
            Xd, Md = X.astype(np.float64), M.astype(np.float64)
            pred_scale = np.einsum("otf,tkf->otk", np.abs(Xd), np.abs(Md))
            _cond_close(yhat, c["yhat"], pred_scale, rtol)
            resid = np.einsum("otf,tkf->otk", Xd, Md) - Y.astype(np.float64)
            grad_scale = 2 * np.einsum("otk,otf->tkf", np.abs(resid), np.abs(Xd))
            _cond_close(grad, c["grad"], grad_scale, rtol)
            # on these well-conditioned cases the plain relative error is small too
            rel = np.abs(grad - c["grad"]) / np.abs(c["grad"])
            assert rel.max() < 10 * rtol, (name, rel.max())


def test_golden_covers_edge_shapes(golden):
    shapes = {tuple(c["X"].shape) for c in golden.values()}
    # single observation, single feature, single task, ragged (33 features, 257 obs)
    assert (1, 3, 5) in shapes and (100, 3, 1) in shapes and (100, 1, 5) in shapes
    assert (257, 3, 33) in shapes and (8192, 1, 32) in shapes


def test_increasing_init_exact(oracle, golden):
    for dt in ("int32", "int64"):
        c = golden[f"increasing_{dt}_3x2x2x5"]
        assert np.array_equal(oracle.predict(c["X"], c["M"]), c["yhat"])
        assert np.array_equal(oracle.gradient(c["X"], c["M"], c["Y"], with_reg=False), c["grad"])


def test_integer_wraparound_matches_modular_arithmetic(oracle):
    rng = np.random.default_rng(7)
    for dt in (np.int8, np.uint8, np.int16, np.uint16, np.uint32, np.int32, np.int64, np.uint64):
        info = np.iinfo(dt)
        nobs, ntasks, nf, nt = 9, 2, 5, 3
        X = rng.integers(info.min, info.max, (nobs, ntasks, nf), dtype=dt, endpoint=True)
        M = rng.integers(info.min, info.max, (ntasks, nt, nf), dtype=dt, endpoint=True)
        Y = rng.integers(info.min, info.max, (nobs, ntasks, nt), dtype=dt, endpoint=True)
        bits = np.dtype(dt).itemsize * 8
        mod = 1 << bits
        Xi, Mi, Yi = (a.astype(object) for a in (X, M, Y))
        yhat = np.einsum("otf,tkf->otk", Xi, Mi)
        grad = 2 * np.einsum("otk,otf->tkf", yhat - Yi, Xi)
        to = np.vectorize(lambda v: v % mod, otypes=[object])
        exp_g = np.array(to(grad).astype(np.uint64) if bits == 64 else to(grad).astype(np.int64))
        exp_y = np.array(to(yhat).astype(np.uint64) if bits == 64 else to(yhat).astype(np.int64))
        unsigned = {8: np.uint8, 16: np.uint16, 32: np.uint32, 64: np.uint64}[bits]
        exp_g = exp_g.astype(unsigned).view(dt)
        exp_y = exp_y.astype(unsigned).view(dt)
        assert np.array_equal(oracle.predict(X, M), exp_y), dt
        assert np.array_equal(oracle.gradient(X, M, Y, with_reg=False), exp_g), dt


def test_hand_computed_2x2_with_elastic_net(oracle):
    # nobs=2, ntasks=1, nf=2, nt=1
    X = np.array([[[1.0, 2.0]], [[3.0, -1.0]]])
    M = np.array([[[0.5, 0.0]]])
    Y = np.array([[[1.0]], [[0.0]]])
    # yhat = [0.5, 1.5]; e = [-0.5, 1.5]
    # sum e*x = [-0.5*1 + 1.5*3, -0.5*2 + 1.5*(-1)] = [4.0, -2.5]; grad = 2*that = [8, -5]
    assert np.allclose(oracle.predict(X, M)[:, 0, 0], [0.5, 1.5])
    g0 = oracle.gradient(X, M, Y, with_reg=False)
    assert np.array_equal(g0[0, 0], [8.0, -5.0])
    # lambda=0.5, alpha=0.25: + 0.5*(0.25*sign(M) + 2*0.75*M); sign(0)=0
    g = oracle.gradient(X, M, Y, lam=0.5, alpha=0.25)
    assert np.allclose(g[0, 0], [8.0 + 0.5 * (0.25 * 1 + 1.5 * 0.5), -5.0 + 0.0])
    # alpha = 1: pure L1, no L2 term; alpha = 0: pure L2
    assert np.allclose(oracle.gradient(X, M, Y, lam=0.5, alpha=1.0)[0, 0], [8.5, -5.0])
    assert np.allclose(oracle.gradient(X, M, Y, lam=0.5, alpha=0.0)[0, 0], [8.5, -5.0])
    # the naive class never adds the term
    assert np.array_equal(oracle.gradient(X, M, Y, lam=0.5, alpha=0.25, with_reg=False), g0)
    for dt in (np.float32,):
        g32 = oracle.gradient(X.astype(dt), M.astype(dt), Y.astype(dt), lam=0.5, alpha=0.25)
        assert np.allclose(g32, g)


def test_integer_reg_truncates_lambda(oracle):
    # Number(lambda) for an integer Number truncates: lambda=2.9 -> 2, alpha=0.5 -> 0
    X = np.array([[[1, 2]], [[3, -1]]], dtype=np.int32)
    M = np.array([[[-3, 0]]], dtype=np.int32)
    Y = np.array([[[1]], [[0]]], dtype=np.int32)
    base = oracle.gradient(X, M, Y, with_reg=False)
    g = oracle.gradient(X, M, Y, lam=2.9, alpha=0.5)
    # alpha truncates to 0 -> pure L2 with 2*lambda*(1-alpha) = 4
    assert np.array_equal(g, base + 4 * M)
    # unsigned: sign is never negative
    Xu, Mu, Yu = X.astype(np.uint32), np.array([[[3, 0]]], dtype=np.uint32), Y.astype(np.uint32)
    gu = oracle.gradient(Xu, Mu, Yu, lam=2.0, alpha=1.0)
    bu = oracle.gradient(Xu, Mu, Yu, with_reg=False)
    assert np.array_equal(gu, bu + np.array([[[2, 0]]], dtype=np.uint32))


def test_f32_acc64_twin_matches_float64_math(oracle):
    rng = np.random.default_rng(3)
    X = rng.uniform(-1, 1, (3000, 2, 17)).astype(np.float32)
    M = rng.normal(size=(2, 3, 17)).astype(np.float32)
    Y = rng.normal(size=(3000, 2, 3)).astype(np.float32)
    g64 = oracle.gradient_acc64(X, M, Y, lam=0.1, alpha=0.3)
    ref = oracle.gradient(X.astype(np.float64), M.astype(np.float64), Y.astype(np.float64),
                          lam=0.1, alpha=0.3)
    assert np.allclose(g64, ref, rtol=1e-12, atol=1e-9)
    g32 = oracle.gradient(X, M, Y, lam=0.1, alpha=0.3)
    assert np.allclose(g32, g64, rtol=1e-4)


def test_gradient_zero_at_exact_fit_and_linearity(oracle):
    rng = np.random.default_rng(11)
    X = rng.normal(size=(500, 3, 8))
    M = rng.normal(size=(3, 2, 8))
    Y = oracle.predict(X, M)
    assert np.max(np.abs(oracle.gradient(X, M, Y, with_reg=False))) < 1e-10
    # predict is linear in M
    M2 = rng.normal(size=M.shape)
    assert np.allclose(oracle.predict(X, 2 * M + M2), 2 * oracle.predict(X, M) + oracle.predict(X, M2))
    assert np.array_equal(oracle.predict(np.zeros_like(X), M), np.zeros((500, 3, 2)))


def test_loss_hand_computed(oracle):
    M = np.array([[[1.0, -2.0]]])
    Y = np.array([[[1.0]], [[0.0]]])
    Yhat = np.array([[[0.5]], [[1.5]]])
    # sq error = 0.25 + 2.25 = 2.5; |M|_1 = 3; |M|^2 = 5; lambda=0.1, alpha=0.4 -> 0.1*(1.2+3.0)
    assert np.isclose(oracle.loss(M, Y, Yhat, lam=0.1, alpha=0.4)[0], 2.5 + 0.42)


def test_soft_threshold_and_prox_step(oracle):
    beta = np.array([1.0, -1.0, 0.2, -0.2, 0.0])
    g = np.array([0.0, 0.0, 0.0, 0.0, 1.0])
    out = oracle.prox_step(beta, g, inv_L=0.5, l1=1.0)  # threshold 0.5
    assert np.allclose(out, [0.5, -0.5, 0.0, 0.0, 0.0])
    out = oracle.prox_step(beta, g, inv_L=1.0, l1=0.0)
    assert np.allclose(out, [1.0, -1.0, 0.2, -0.2, -1.0])


def test_power_iteration_matches_eigenvalue(oracle):
    rng = np.random.default_rng(5)
    X = rng.normal(size=(400, 2, 6))
    v0 = oracle.power_start(2 * 6, seed=1234)
    nrm = oracle.power_norm(X, v0, n_power=200)
    for task in range(2):
        lmax = np.linalg.eigvalsh(X[:, task, :].T @ X[:, task, :])[-1]
        assert np.isclose(nrm[task], 2 * lmax, rtol=1e-6)


def test_power_start_is_deterministic_uniform(oracle):
    a = oracle.power_start(1000, 42)
    b = oracle.power_start(1000, 42)
    assert np.array_equal(a, b)
    assert a.min() >= -1 and a.max() < 1 and abs(a.mean()) < 0.1
    assert not np.array_equal(a, oracle.power_start(1000, 43))


def test_fit_converges_to_ridge_closed_form(oracle):
    rng = np.random.default_rng(9)
    nobs, nf = 300, 5
    X = rng.normal(size=(nobs, 1, nf))
    bt = rng.normal(size=nf)
    Y = (X[:, 0, :] @ bt + 0.1 * rng.normal(size=nobs)).reshape(nobs, 1, 1)
    lam2 = 3.0
    v0 = oracle.power_start(nf, 7)
    beta, lip = oracle.fit(X, Y, 0.0, lam2, v0, n_power=50, n_iter=3000)
    A = X[:, 0, :]
    closed = np.linalg.solve(A.T @ A + lam2 * np.eye(nf), A.T @ Y[:, 0, 0])
    assert np.allclose(beta[0, 0], closed, rtol=1e-6, atol=1e-8)
    assert lip[0] > 2 * np.linalg.eigvalsh(A.T @ A)[-1]


def test_fit_lasso_kkt_conditions(oracle):
    rng = np.random.default_rng(13)
    nobs, nf = 400, 8
    X = rng.normal(size=(nobs, 1, nf))
    bt = np.zeros(nf)
    bt[:3] = [2.0, -1.5, 1.0]
    Y = (X[:, 0, :] @ bt + 0.1 * rng.normal(size=nobs)).reshape(nobs, 1, 1)
    l1, l2 = 40.0, 1.0
    beta, _ = oracle.fit(X, Y, l1, l2, oracle.power_start(nf, 3), n_power=50, n_iter=4000)
    b = beta[0, 0]
    A = X[:, 0, :]
    g = 2 * A.T @ (A @ b - Y[:, 0, 0]) + 2 * l2 * b
    nz = b != 0
    # stationarity: g + l1*sign(b) = 0 on the support, |g| <= l1 off it
    assert np.allclose(g[nz] + l1 * np.sign(b[nz]), 0, atol=1e-6)
    assert np.all(np.abs(g[~nz]) <= l1 + 1e-6)
    assert nz.sum() >= 3 and not nz.all()


def test_bf16_conversions_and_hand_computed_case(oracle):
    """bfloat16 (an input type beyond the reference's set, treated like half):
    the NumPy conversions round to nearest even like torch's, and the oracle's
    bfloat16 gradient of the hand-computed 2x2 case is exact (every value and
    intermediate is representable)."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    a = np.concatenate([rng.normal(size=20000).astype(np.float32) * 1e3,
                        np.array([0.0, -0.0, np.inf, -np.inf, 3.0e38, 1e-40, 1.00390625, 1.01171875], np.float32)])
    ref = torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle.bf16_bits(a), ref)
    assert np.array_equal(oracle.bf16_to_f32(ref), torch.from_numpy(ref.view(np.int16)).view(torch.bfloat16).float().numpy())
    assert np.isnan(oracle.bf16_to_f32(oracle.bf16_bits(np.array([np.nan], np.float32))))[0]
    X = oracle.bf16_bits(np.array([[[1.0, 2.0]], [[3.0, -1.0]]], np.float32))
    M = oracle.bf16_bits(np.array([[[0.5, 0.0]]], np.float32))
    Y = oracle.bf16_bits(np.array([[[1.0]], [[0.0]]], np.float32))
    assert np.array_equal(oracle.bf16_to_f32(oracle.predict(X, M, bf16=True))[:, 0, 0], [0.5, 1.5])
    assert np.array_equal(oracle.bf16_to_f32(oracle.gradient(X, M, Y, with_reg=False, bf16=True))[0, 0], [8.0, -5.0])
    # lambda 0.5, alpha 0.25 (both exact in bfloat16): 8 + 0.5*(0.25 + 1.5*0.5) = 8.5
    g = oracle.bf16_to_f32(oracle.gradient(X, M, Y, lam=0.5, alpha=0.25, bf16=True))
    assert np.array_equal(g[0, 0], [8.5, -5.0])
    # loss: e = [-0.5, 1.5] -> 2.5, + 0.5*(0.25*0.5 + 0.75*0.25) = 2.65625 -> bfloat16 2.65625
    yh = oracle.predict(X, M, bf16=True)
    assert oracle.bf16_to_f32(oracle.loss(M, Y, yh, 0.5, 0.25, bf16=True))[0] == 2.65625


def test_bf16_gradient_within_its_rounding(oracle):
    """float arithmetic and one rounding to bfloat16: within 2^-8 of the exact
    gradient of the same rounded inputs, on the data's scale."""
    rng = np.random.default_rng(6)
    X = oracle.bf16_bits(rng.uniform(-1, 1, (3000, 2, 24)).astype(np.float32))
    M = oracle.bf16_bits(rng.normal(size=(2, 3, 24)).astype(np.float32))
    Y = oracle.bf16_bits(rng.normal(size=(3000, 2, 3)).astype(np.float32))
    Xf, Mf, Yf = (oracle.bf16_to_f32(v).astype(np.float64) for v in (X, M, Y))
    exact = 2 * np.einsum("otk,otf->tkf", np.einsum("otf,tkf->otk", Xf, Mf) - Yf, Xf)
    g = oracle.bf16_to_f32(oracle.gradient(X, M, Y, with_reg=False, bf16=True)).astype(np.float64)
    assert np.all(np.abs(g - exact) <= 2.0 ** -8 * (np.abs(exact) + 1e-3 * np.abs(exact).max()))
