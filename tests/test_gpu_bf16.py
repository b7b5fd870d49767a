"""bfloat16 inputs (glmb_*_bf16): the reduced-precision input type beside
float16, with float arithmetic and one rounding to bfloat16 on store.

bfloat16 is not in the reference's type set (include/cuda/type_traits.cuh:44-46
lists the eleven types of its mains), so the bar is the oracle's bfloat16
restatement -- the half algorithm with bfloat16 rounding -- and the exact
(float64) gradient of the same rounded inputs, with lambda and alpha taken in
bfloat16 as the kernels take them (the reference's Number(double)).
bfloat16 carries 8 significant bits: unit roundoff 2^-8, one unit in the
last place at most 2^-7 of the value.  Tolerances, stated per check: against
the exact gradient 2^-7 relative on the data's scale (one rounding plus float
arithmetic); against the oracle 2^-6 (both round once at the end, from float
sums in different orders, so they may land one unit in the last place
apart).

bfloat16 arrays travel as uint16 bit patterns (NumPy has no bfloat16).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_algos_b200 import capi, glm  # noqa: E402
from oracle import pyoracle as O  # noqa: E402
from tests import gpu_util as G  # noqa: E402

TOL_EXACT = 2.0 ** -7
TOL_ORACLE = 2.0 ** -6


def _b(v):
    """A double as the kernels take it: rounded to bfloat16."""
    return float(O.bf16_to_f32(O.bf16_bits(np.array([v], np.float32)))[0])


def _problem(nobs, ntasks, nf, nt, seed):
    rng = np.random.default_rng(seed)
    X = O.bf16_bits(rng.uniform(-1, 1, (nobs, ntasks, nf)) / 4)
    M = O.bf16_bits(rng.normal(size=(ntasks, nt, nf)))
    Xf, Mf = O.bf16_to_f32(X).astype(np.float64), O.bf16_to_f32(M).astype(np.float64)
    Y = O.bf16_bits(np.einsum("otf,tkf->otk", Xf, Mf) + 0.05 * rng.normal(size=(nobs, ntasks, nt)))
    return X, M, Y


def _exact(X, M, Y, lam, alpha, reg):
    Xf, Mf, Yf = (O.bf16_to_f32(a).astype(np.float64) for a in (X, M, Y))
    g = 2 * np.einsum("otk,otf->tkf", np.einsum("otf,tkf->otk", Xf, Mf) - Yf, Xf)
    if reg:
        lam, alpha = _b(lam), _b(alpha)
        g = g + lam * (alpha * np.sign(Mf) + 2 * (1 - alpha) * Mf)
    return g, np.einsum("otf,tkf->otk", Xf, Mf)


def _within(actual_bits, expected, tol, scale, what):
    a = O.bf16_to_f32(actual_bits).astype(np.float64)
    e = np.asarray(expected, dtype=np.float64)
    err = np.abs(a - e)
    bound = tol * (np.abs(e) + scale)
    assert np.all(err <= bound), f"{what}: {np.max(err / (np.abs(e) + scale)):.3e} > {tol:.1e}"


@pytest.mark.parametrize("shape", [(100000, 1, 128, 1), (20000, 2, 64, 4), (5001, 3, 1024, 1), (777, 2, 40, 3),
                                   (3000, 1, 32, 4), (1000, 2, 96, 2), (64, 1, 7, 2)])
def test_bf16_rows_path(shape, oracle):
    """Packed pairs in 4-, 8- and 16-byte loads over full warps and over
    shorter segments, and (7 features) one element per lane."""
    nobs, ntasks, nf, nt = shape
    X, M, Y = _problem(nobs, ntasks, nf, nt, seed=nobs + nf)
    g, yh = G.gradient(X, M, Y, 0.1, 0.5, reg=True, want_yhat=True, sfx="bf16")
    assert capi.last_path() == "rows"
    exact, yexact = _exact(X, M, Y, 0.1, 0.5, True)
    scale = np.abs(exact).max()
    _within(g, exact, TOL_EXACT, 1e-2 * scale, "bf16 grad vs exact")
    og = O.bf16_to_f32(O.gradient(X, M, Y, 0.1, 0.5, True, bf16=True))
    _within(g, og, TOL_ORACLE, 1e-2 * scale, "bf16 grad vs oracle")
    oy = O.bf16_to_f32(O.predict(X, M, bf16=True))
    yscale = 1e-2 * np.abs(yexact).max()
    _within(yh, yexact, TOL_EXACT, yscale, "bf16 yhat vs exact")
    _within(yh, oy, TOL_ORACLE, yscale, "bf16 yhat vs oracle")
    p = G.predict(X, M, sfx="bf16")
    _within(p, oy, TOL_ORACLE, yscale, "bf16 predict vs oracle")


@pytest.mark.parametrize("shape", [(500, 2, 40, 9), (300, 3, 2000, 1)])
def test_bf16_generic_path(shape, oracle):
    """Shapes the rows kernel does not serve (more than 8 targets; 2000
    features, beyond its register budget): the generic pair of kernels."""
    nobs, ntasks, nf, nt = shape
    X, M, Y = _problem(nobs, ntasks, nf, nt, seed=nobs * 7 + nf)
    g = G.gradient(X, M, Y, 0.2, 0.25, reg=True, sfx="bf16")
    assert capi.last_path() != "rows"
    exact, _ = _exact(X, M, Y, 0.2, 0.25, True)
    scale = np.abs(exact).max()
    _within(g, exact, TOL_EXACT, 1e-2 * scale, f"bf16 grad vs exact ({capi.last_path()})")
    og = O.bf16_to_f32(O.gradient(X, M, Y, 0.2, 0.25, True, bf16=True))
    _within(g, og, TOL_ORACLE, 1e-2 * scale, f"bf16 grad vs oracle ({capi.last_path()})")


def test_bf16_through_the_torch_api_and_loss(oracle):
    """glm.gradient / glm.loss on torch.bfloat16 tensors: the same bits as the
    C-ABI call on the same bytes; the loss within 2^-6 of the oracle's."""
    X, M, Y = _problem(20000, 1, 128, 1, seed=3)
    to_t = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()  # noqa: E731
    Xt, Mt, Yt = to_t(X), to_t(M), to_t(Y)
    yh = torch.empty((20000, 1, 1), dtype=torch.bfloat16, device="cuda")
    g = glm.gradient(Xt, Mt, Yt, 0.1, 0.5, yhat_out=yh)
    L = glm.loss(Mt, Yt, yh, 0.1, 0.5)
    torch.cuda.synchronize()
    bits = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    g_abi, yh_abi = G.gradient(X, M, Y, 0.1, 0.5, reg=True, want_yhat=True, sfx="bf16")
    assert np.array_equal(bits(g), g_abi)
    assert np.array_equal(bits(yh), yh_abi)
    ol = O.bf16_to_f32(O.loss(M, Y, bits(yh), 0.1, 0.5, bf16=True))[0]
    assert abs(float(O.bf16_to_f32(bits(L))[0]) - ol) <= TOL_ORACLE * abs(ol)


def test_bf16_specials_propagate(oracle):
    """Inf and NaN inputs reach the outputs as they do in the oracle: the
    rows kernel widens bfloat16 by a shift, which keeps them."""
    X, M, Y = _problem(2000, 2, 64, 1, seed=11)
    X = X.copy()
    X[5, 0, 3] = 0x7F80  # +inf in task 0: its gradient is +-inf
    X[9, 1, 10] = 0x7FC0  # NaN in task 1: its gradient is NaN
    g = G.gradient(X, M, Y, 0.0, 0.0, reg=False, sfx="bf16")
    og = O.gradient(X, M, Y, with_reg=False, bf16=True)
    gf, of = O.bf16_to_f32(g), O.bf16_to_f32(og)
    assert np.isinf(gf[0]).sum() > 32 and np.isnan(gf[1]).all()
    assert np.array_equal(np.isnan(gf), np.isnan(of))
    assert np.array_equal(np.isinf(gf), np.isinf(of))
    assert np.array_equal(np.signbit(gf[np.isinf(gf)]), np.signbit(of[np.isinf(of)]))


@pytest.mark.parametrize("shape,path", [((20000, 1, 128, 1), "rows"), ((700, 2, 40, 3), "rows"),
                                        ((900, 2, 48, 12), "generic")])
def test_bf16_logistic(shape, path):
    """GLMB_GRAD_LOGISTIC on bfloat16: mu = sigmoid(X M) and sum (mu - Y) X
    (+ elastic net) against float64 NumPy on the same rounded inputs, within
    2^-6 (floor 1e-3 of the largest element); mu within 2^-7 absolute."""
    nobs, ntasks, nf, nt = shape
    rng = np.random.default_rng(nobs + nt)
    X = O.bf16_bits(rng.normal(size=(nobs, ntasks, nf)) / np.sqrt(nf))
    Xf = O.bf16_to_f32(X).astype(np.float64)
    eta = np.einsum("otf,tkf->otk", Xf, rng.normal(size=(ntasks, nt, nf)))
    Y = O.bf16_bits((rng.uniform(size=eta.shape) < 1 / (1 + np.exp(-eta))).astype(np.float32))
    M = O.bf16_bits(rng.normal(size=(ntasks, nt, nf)) * 0.5)
    Mf, Yf = O.bf16_to_f32(M).astype(np.float64), O.bf16_to_f32(Y).astype(np.float64)
    g, mu = G.gradient(X, M, Y, 0.3, 0.4, reg=True, want_yhat=True, sfx="bf16", flags=capi.GRAD_LOGISTIC)
    assert capi.last_path() == path
    ref_mu = 1 / (1 + np.exp(-np.einsum("otf,tkf->otk", Xf, Mf)))
    lam, alpha = _b(0.3), _b(0.4)
    ref = np.einsum("otk,otf->tkf", ref_mu - Yf, Xf) + lam * (alpha * np.sign(Mf) + 2 * (1 - alpha) * Mf)
    assert G.rel_err(O.bf16_to_f32(g), ref, floor=1e-3 * np.abs(ref).max()) <= TOL_ORACLE
    assert np.abs(O.bf16_to_f32(mu) - ref_mu).max() <= TOL_EXACT
