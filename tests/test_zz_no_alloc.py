"""glmb_gradient_noalloc_f32: the gradient entry point that allocates no
device memory, for callers that may not allocate (a host that owns every
device buffer and passes only inputs and outputs, a fixed memory budget, a
path that must not wait on the allocator).

It is checked through the C ABI against glmb_gradient_f32 -- the entry point
that takes scratch from the caller or from cudaMallocAsync -- and against the
oracle, on calls in a row with different shapes, so each call runs over the
previous call's leftovers in the shared scratch array.  Tolerance: the
float32 bar of the parity tests, max relative error <= 1e-4 (on all-positive
data, where no gradient element is near zero).  Also covered: the branch
that trades CTAs for longer row ranges when a shape's CTA partials would not
fit the 4 MiB array, the early-return paths (no features, no observations,
Y all zero), the rejected options, and that a call leaves the device's
memory use unchanged.  This file is collected last on purpose.
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
SCRATCH_DOUBLES = 1 << 19  # the array's stated size: 4 MiB of doubles


def _positive(nobs, ntasks, nf, nt, seed):
    rng = np.random.default_rng(seed)
    X = rng.uniform(0, 1, (nobs, ntasks, nf)).astype(np.float32)
    M = rng.uniform(0, 1, (ntasks, nt, nf)).astype(np.float32)
    Y = rng.uniform(0, 1, (nobs, ntasks, nt)).astype(np.float32)
    return X, M, Y


def _both(X, M, Y, lam, alpha, flags):
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    dX, dM = G.Dev(X), G.Dev(M)
    dY = G.Dev(Y) if Y is not None else None
    out = {}
    for name in ("glmb_gradient_f32", "glmb_gradient_noalloc_f32"):
        g = G.Dev(shape=(ntasks, nt, nf), dtype=np.float32)
        yh = G.Dev(shape=(nobs, ntasks, nt), dtype=np.float32)
        args = [dX.ptr, dM.ptr, dY.ptr if dY else None, g.ptr, yh.ptr, nf, nt, ntasks, nobs, lam, alpha, flags]
        if name == "glmb_gradient_f32":
            args += [None, 0]
        capi.call(name, *args, G.stream())
        torch.cuda.synchronize()
        assert g.canary_intact() and yh.canary_intact()
        out[name] = (g.numpy(), yh.numpy())
    return out["glmb_gradient_f32"], out["glmb_gradient_noalloc_f32"]


def _check(X, M, Y, lam, alpha, flags, oracle):
    (g_ref, y_ref), (g_na, y_na) = _both(X, M, Y, lam, alpha, flags)
    assert G.rel_err(g_na, g_ref) <= RTOL
    og = oracle.gradient(X, M, Y, lam, alpha, bool(flags & capi.GRAD_REGULARIZE))
    assert G.rel_err(g_na, og) <= RTOL
    if flags & capi.GRAD_WRITE_YHAT:
        assert G.rel_err(y_na, y_ref) <= RTOL
        assert G.rel_err(y_na, oracle.predict(X, M)) <= RTOL
    return g_na


def test_noalloc_matches_allocating_entry_point_twice(oracle):
    # call 1: the benchmark's single-task shape, smaller nobs
    X, M, Y = _positive(300_000, 1, 128, 1, seed=1)
    _check(X, M, Y, 0.01, 0.0, capi.GRAD_REGULARIZE, oracle)
    # call 2: another shape (3 tasks, 2 targets, 64 features) with predictions
    X, M, Y = _positive(50_001, 3, 64, 2, seed=2)
    _check(X, M, Y, 0.2, 0.5, capi.GRAD_REGULARIZE | capi.GRAD_WRITE_YHAT, oracle)


@pytest.mark.parametrize("big", [(64, 257, 512, 2), (64, 257, 256, 4), (64, 257, 128, 8), (100, 512, 1024, 1)])
def test_noalloc_fewer_longer_ctas_then_smaller_call(big, oracle):
    """Shapes at the array's limit.  257 tasks x 1024 partials per task: two
    CTAs per task would need 526,336 doubles, more than the 524,288 the array
    holds, so wherever the planner gives each task two or more CTAs (kernels
    that fit two or more CTAs per SM on 148 SMs) the call cuts the plan to
    one longer CTA per task.  512 tasks x 1024 features fill the array
    exactly.  A smaller call follows, over the cut plan's leftovers."""
    nobs, ntasks, nf, nt = big
    assert nf * nt * ntasks <= SCRATCH_DOUBLES
    X, M, Y = _positive(nobs, ntasks, nf, nt, seed=nobs + ntasks + nf)
    _check(X, M, Y, 0.1, 0.3, capi.GRAD_REGULARIZE | capi.GRAD_WRITE_YHAT, oracle)
    X, M, Y = _positive(40_000, 2, 96, 3, seed=5)
    _check(X, M, Y, 0.0, 0.0, 0, oracle)


def test_noalloc_early_return_paths(oracle):
    L = capi.lib()
    s = G.stream()
    # no features: Yhat is all zeros and nothing else is touched
    M0 = G.Dev(shape=(1, 2, 0), dtype=np.float32)
    yh = G.Dev(np.full((7, 1, 2), 3.0, np.float32))
    g0 = G.Dev(shape=(1, 2, 0), dtype=np.float32)
    assert L.glmb_gradient_noalloc_f32(None, M0.ptr, None, g0.ptr, yh.ptr, 0, 2, 1, 7, 0.0, 0.0,
                                       capi.GRAD_WRITE_YHAT, s) == 0
    torch.cuda.synchronize()
    assert np.all(yh.numpy() == 0) and yh.canary_intact() and g0.canary_intact()
    # no observations: the elastic-net term alone
    M = np.array([[[0.5, -1.0, 0.0, 2.0]]], np.float32)
    dM, g = G.Dev(M), G.Dev(shape=(1, 1, 4), dtype=np.float32)
    assert L.glmb_gradient_noalloc_f32(None, dM.ptr, None, g.ptr, None, 4, 1, 1, 0, 0.5, 0.25,
                                       capi.GRAD_REGULARIZE, s) == 0
    torch.cuda.synchronize()
    expect = 0.5 * (0.25 * np.sign(M) + 2 * 0.75 * M)
    assert np.allclose(g.numpy(), expect, rtol=1e-6, atol=0) and g.canary_intact()
    # Y all zero (Y may be NULL)
    X, M, _ = _positive(5000, 2, 64, 3, seed=9)
    (g_ref, _), (g_na, _) = _both(X, M, None, 0.0, 0.0, capi.GRAD_Y_ZERO)
    assert G.rel_err(g_na, g_ref) <= RTOL
    assert G.rel_err(g_na, oracle.gradient(X, M, None, with_reg=False)) <= RTOL


def test_noalloc_rejects_what_it_does_not_offer():
    L = capi.lib()
    s = G.stream()
    X, M, Y = _positive(64, 1, 16, 9, seed=3)
    dX, dM, dY = G.Dev(X), G.Dev(M), G.Dev(Y)
    g = G.Dev(shape=(1, 9, 16), dtype=np.float32)
    # the logistic link is not offered here
    st = L.glmb_gradient_noalloc_f32(dX.ptr, dM.ptr, dY.ptr, g.ptr, None, 16, 9, 1, 64, 0.0, 0.0,
                                     capi.GRAD_LOGISTIC, s)
    assert st == capi.GLMB_ERR_INVALID_VALUE
    # more than 8 targets: not a shape of the single-pass kernel
    st = L.glmb_gradient_noalloc_f32(dX.ptr, dM.ptr, dY.ptr, g.ptr, None, 16, 9, 1, 64, 0.0, 0.0, 0, s)
    assert st == capi.GLMB_ERR_UNSUPPORTED
    torch.cuda.synchronize()
    assert g.canary_intact()
    assert np.all(g.numpy().view(np.uint8) == 0xA5)  # untouched


def test_noalloc_rejects_sizes_beyond_its_scratch():
    buf = torch.zeros(64, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    L = capi.lib()
    # 1024 tasks x 1 target x 1024 features = 1,048,576 partial sums > 524,288
    st = L.glmb_gradient_noalloc_f32(p, p, p, p, None, 1024, 1, 1024, 16, 0.0, 0.0, 0, G.stream())
    assert st == capi.GLMB_ERR_TOO_LARGE


def test_noalloc_call_leaves_device_memory_unchanged():
    """No cudaMalloc / cudaMallocAsync behind the call: the device's free
    memory, torch's allocations and the default stream-ordered pool's use
    (its high-water mark, reset just before) are the same after two calls."""
    rt = pytest.importorskip("cuda.bindings.runtime")
    drv = pytest.importorskip("cuda.bindings.driver")
    X, M, Y = _positive(200_000, 2, 128, 2, seed=11)
    dX, dM, dY = G.Dev(X), G.Dev(M), G.Dev(Y)
    g = G.Dev(shape=(2, 2, 128), dtype=np.float32)
    yh = G.Dev(shape=(200_000, 2, 2), dtype=np.float32)
    L = capi.lib()
    s = G.stream()
    flags = capi.GRAD_REGULARIZE | capi.GRAD_WRITE_YHAT
    # first call on this device done earlier in the file or here: the array's address is set up
    assert L.glmb_gradient_noalloc_f32(dX.ptr, dM.ptr, dY.ptr, g.ptr, yh.ptr, 128, 2, 2, 200_000, 0.1, 0.5,
                                       flags, s) == 0
    torch.cuda.synchronize()
    err, dev = rt.cudaGetDevice()
    assert err == rt.cudaError_t.cudaSuccess
    err, pool = rt.cudaDeviceGetDefaultMemPool(dev)
    assert err == rt.cudaError_t.cudaSuccess
    high = rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh
    cur = rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent
    err, used0 = rt.cudaMemPoolGetAttribute(pool, cur)
    assert err == rt.cudaError_t.cudaSuccess
    (err,) = rt.cudaMemPoolSetAttribute(pool, high, drv.cuuint64_t(0))
    assert err == rt.cudaError_t.cudaSuccess
    free0, _ = torch.cuda.mem_get_info()
    torch0 = torch.cuda.memory_allocated()
    for _ in range(2):
        assert L.glmb_gradient_noalloc_f32(dX.ptr, dM.ptr, dY.ptr, g.ptr, yh.ptr, 128, 2, 2, 200_000, 0.1, 0.5,
                                           flags, s) == 0
    torch.cuda.synchronize()
    err, peak = rt.cudaMemPoolGetAttribute(pool, high)
    assert err == rt.cudaError_t.cudaSuccess
    assert int(peak) <= int(used0)  # nothing taken from the stream-ordered pool
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == torch0
    assert g.canary_intact() and yh.canary_intact()
