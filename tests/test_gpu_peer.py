"""The peer-memory exchange on one GPU: a one-rank group reproduces the
plain gradient bit for bit, and a wait for a peer that never arrives ends
after the group's timeout with the status set and NaN outputs (the GPU and
the context stay usable).  Multi-rank exchanges are covered by
tests/test_gpu_sharded.py on two GPUs."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_algos_b200 import capi  # noqa: E402
from tests import gpu_util as G  # noqa: E402


def _group(rank, world, max_elems, timeout_ms):
    ptr = ctypes.c_void_p()
    capi.call("glmb_peer_group_create", rank, world, max_elems, timeout_ms, ctypes.byref(ptr), None)
    return ptr


def _status(g):
    st = ctypes.c_int(-1)
    capi.call("glmb_peer_group_status", g, ctypes.byref(st), 1)
    return st.value


def _sharded(g, X, M, Y, lam, alpha, partial=False, sfx=None):
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    sfx = sfx or G.SFX[X.dtype]
    dX, dM, dY = G.Dev(X), G.Dev(M), G.Dev(Y)
    out = G.Dev(shape=(ntasks, nt, nf), dtype=np.float64 if partial else X.dtype)
    capi.call(f"glmb_gradient_sharded_{sfx}", dX.ptr, dM.ptr, dY.ptr, None if partial else out.ptr,
              out.ptr if partial else None, None, nf, nt, ntasks, nobs, lam, alpha,
              0 if partial else capi.GRAD_REGULARIZE, g, None, 0, G.stream())
    torch.cuda.synchronize()
    assert out.canary_intact()
    return out.numpy()


def test_single_rank_group_equals_plain_gradient():
    g = _group(0, 1, 1 << 15, 1000.0)
    try:
        capi.call("glmb_peer_group_connect_local", g, (ctypes.c_void_p * 1)(capi.lib().glmb_peer_group_buffer(g)))
        rng = np.random.default_rng(2)
        for dt, shape in ((np.float32, (20000, 1, 128, 1)), (np.float64, (3000, 4, 256, 16)),
                          (np.float32, (777, 3, 50, 12))):
            nobs, ntasks, nf, nt = shape
            X = rng.uniform(-1, 1, (nobs, ntasks, nf)).astype(dt)
            M = rng.normal(size=(ntasks, nt, nf)).astype(dt)
            Y = rng.normal(size=(nobs, ntasks, nt)).astype(dt)
            for _ in range(3):  # successive calls alternate slot parities
                got = _sharded(g, X, M, Y, 0.3, 0.2)
                assert np.array_equal(got, G.gradient(X, M, Y, 0.3, 0.2))
            P = _sharded(g, X, M, Y, 0.0, 0.0, partial=True)
            g0 = G.gradient(X, M, Y, reg=False)
            assert np.allclose(2 * P, g0, rtol=1e-5 if dt == np.float32 else 1e-12, atol=1e-3)
        # the 16-bit types (bfloat16 as uint16 bit patterns)
        for dt, sfx in ((np.float16, None), (np.uint16, "bf16")):
            Xf = rng.uniform(-1, 1, (5000, 2, 64)) / 4
            Mf, Yf = rng.normal(size=(2, 3, 64)), rng.normal(size=(5000, 2, 3))
            if sfx == "bf16":
                from oracle import pyoracle as O

                X, M, Y = O.bf16_bits(Xf), O.bf16_bits(Mf), O.bf16_bits(Yf)
            else:
                X, M, Y = Xf.astype(dt), Mf.astype(dt), Yf.astype(dt)
            for _ in range(2):
                got = _sharded(g, X, M, Y, 0.3, 0.2, sfx=sfx)
                assert np.array_equal(got, G.gradient(X, M, Y, 0.3, 0.2, sfx=sfx))
        assert _status(g) == 0
    finally:
        capi.call("glmb_peer_group_destroy", g)


def test_wait_for_absent_peer_times_out_with_status():
    # rank 0 of a two-rank group whose rank 1 never runs: its flag never arrives
    a = _group(0, 2, 1024, 200.0)
    b = _group(1, 2, 1024, 200.0)
    try:
        L = capi.lib()
        bufs = (ctypes.c_void_p * 2)(L.glmb_peer_group_buffer(a), L.glmb_peer_group_buffer(b))
        capi.call("glmb_peer_group_connect_local", a, bufs)
        capi.call("glmb_peer_group_connect_local", b, bufs)
        rng = np.random.default_rng(3)
        X = rng.uniform(-1, 1, (4096, 1, 64)).astype(np.float32)
        M = rng.normal(size=(1, 1, 64)).astype(np.float32)
        Y = rng.normal(size=(4096, 1, 1)).astype(np.float32)
        got = _sharded(a, X, M, Y, 0.1, 0.0)
        assert np.all(np.isnan(got))
        assert _status(a) == 1
        assert _status(a) == 0  # reset by the previous read
        # the context is still usable
        assert np.isfinite(G.gradient(X, M, Y, 0.1, 0.0)).all()
    finally:
        capi.call("glmb_peer_group_destroy", a)
        capi.call("glmb_peer_group_destroy", b)


def test_group_argument_checks():
    ptr = ctypes.c_void_p()
    L = capi.lib()
    assert L.glmb_peer_group_create(2, 2, 16, 100.0, ctypes.byref(ptr), None) == capi.GLMB_ERR_INVALID_VALUE
    assert L.glmb_peer_group_create(0, 0, 16, 100.0, ctypes.byref(ptr), None) == capi.GLMB_ERR_INVALID_VALUE
    assert L.glmb_peer_group_create(0, 1, 0, 100.0, ctypes.byref(ptr), None) == capi.GLMB_ERR_INVALID_VALUE
    g = _group(0, 1, 8, 100.0)
    try:
        capi.call("glmb_peer_group_connect_local", g, (ctypes.c_void_p * 1)(L.glmb_peer_group_buffer(g)))
        X = np.ones((10, 1, 16), np.float32)
        M = np.ones((1, 1, 16), np.float32)
        Y = np.ones((10, 1, 1), np.float32)
        dX, dM, dY = G.Dev(X), G.Dev(M), G.Dev(Y)
        out = G.Dev(shape=(1, 1, 16), dtype=np.float32)
        # 16 gradient elements exceed the group's capacity of 8
        st = L.glmb_gradient_sharded_f32(dX.ptr, dM.ptr, dY.ptr, out.ptr, None, None, 16, 1, 1, 10, 0.0, 0.0, 0,
                                         g, None, 0, G.stream())
        assert st == capi.GLMB_ERR_TOO_LARGE
    finally:
        capi.call("glmb_peer_group_destroy", g)
