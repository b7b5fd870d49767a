"""Parity at the benchmark configurations' full sizes, through properties that
do not depend on size (the oracle cannot run there in seconds):

* checksum identity: for any vector v, v . grad[task, t, :] = 2 sum_obs
  r[obs, task, t] (X[obs, task, :] . v) with r = Yhat - Y -- the right side
  from the library's predict kernel (a different code path) and float64
  reductions in torch, the left side from the gradient;
* shard additivity: the partial sums of disjoint observation blocks add up to
  the partial sum of the whole.

Inputs are seeded and generated on the device with the configurations'
distributions (the reference names no dataset).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_algos_b200 import capi, glm  # noqa: E402


def _problem(nobs, ntasks, nf, nt, dtype, x_dist, x_scale, noise, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    X = torch.empty((nobs, ntasks, nf), dtype=dtype, device="cuda")
    if x_dist == "uniform":
        X.uniform_(-1.0, 1.0, generator=g)
    else:
        X.normal_(generator=g)
    if x_scale != 1.0:
        X.mul_(x_scale)
    beta = torch.randn((ntasks, nt, nf), generator=g, dtype=dtype, device="cuda")
    Y = torch.empty((nobs, ntasks, nt), dtype=dtype, device="cuda")
    for task in range(ntasks):
        Y[:, task, :] = X[:, task, :] @ beta[task].T
    Y.add_(torch.randn(Y.shape, generator=g, dtype=dtype, device="cuda") * noise)
    M = torch.randn((ntasks, nt, nf), generator=g, dtype=dtype, device="cuda")  # away from the solution
    return X, M, Y


def _checksum(X, M, Y, grad, nvec=3, seed=7):
    """max over tasks/targets/vectors of |v.g - 2 r.(Xv)| / (|v| |2 r| |Xv|-scale)."""
    ntasks, nt, nf = M.shape
    r = (glm.predict(X, M).double() - Y.double())  # (nobs, ntasks, nt)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    worst = 0.0
    for _ in range(nvec):
        v = torch.randn((ntasks, 1, nf), generator=g, dtype=X.dtype, device="cuda")
        xv = glm.predict(X, v).double()  # (nobs, ntasks, 1)
        rhs = 2.0 * (r * xv).sum(dim=0)  # (ntasks, nt)
        lhs = (grad.double() * v.double()).sum(dim=2)  # (ntasks, nt)
        scale = 2.0 * (r.abs() * xv.abs()).sum(dim=0)  # the sum's own conditioning
        worst = max(worst, float(((lhs - rhs).abs() / scale).max()))
        del xv
    return worst


@pytest.mark.parametrize("cfg", ["gradient_f32_2^24x128", "multitask_f64_64x2^18x256x16", "dense_f32_2^20x4096x256"])
def test_full_size_checksum_identity(cfg):
    if cfg.startswith("gradient"):
        X, M, Y = _problem(1 << 24, 1, 128, 1, torch.float32, "uniform", 1.0, 0.1, 11)
        tol, path = 1e-5, "rows"
    elif cfg.startswith("multitask"):
        X, M, Y = _problem(1 << 18, 64, 256, 16, torch.float64, "normal", 1.0, 0.05, 12)
        tol, path = 1e-12, "tiles"
    else:
        X, M, Y = _problem(1 << 20, 1, 4096, 256, torch.float32, "uniform", 4096 ** -0.5, 0.01, 13)
        tol, path = 1e-5, "dense"
    grad = glm.gradient(X, M, Y, 0.0, 0.0, regularize=False)
    assert capi.last_path() == path
    assert bool(torch.isfinite(grad).all())
    assert _checksum(X, M, Y, grad) <= tol
    # regularised: the elastic-net term is added elementwise on top
    reg = glm.gradient(X, M, Y, 0.01, 0.0, regularize=True)
    expect = grad.double() + 2 * 0.01 * M.double()
    rel = float(((reg.double() - expect).abs() / (expect.abs() + grad.double().abs().max() * 1e-6)).max())
    assert rel <= (1e-5 if X.dtype == torch.float32 else 1e-12)


def test_full_size_shard_additivity():
    X, M, Y = _problem(1 << 24, 1, 128, 1, torch.float32, "uniform", 1.0, 0.1, 14)
    whole = glm.gradient_partial(X, M, Y)
    cuts = [0, 5_000_000, 11_111_111, 1 << 24]
    parts = sum(glm.gradient_partial(X[a:b], M, Y[a:b]) for a, b in zip(cuts[:-1], cuts[1:]))
    # the blocks' float runs are grouped differently: agreement to float accumulation accuracy
    scale = float(whole.abs().max())
    assert float((parts - whole).abs().max()) <= 1e-6 * scale
