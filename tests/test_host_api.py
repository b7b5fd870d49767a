"""CPU tests of the C++ host mirror of the reference's kernel-class API:
the option parser, Tensor3D's seeded initialisation, the kernel classes'
host computations (run_host_kernel) against the oracle, and the
executables' command-line behaviour.  No GPU is used."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "gpu_algos_b200")
BIN = os.path.join(PKG, "bin")


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    out = tmp_path_factory.mktemp("probe") / "libhost_api_probe.so"
    cuda_inc = "/usr/local/cuda/include"
    subprocess.run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-fopenmp",
                    f"-I{PKG}/include", f"-I{REPO}/include", f"-I{cuda_inc}",
                    os.path.join(REPO, "tests", "cpp", "host_api_probe.cpp"), "-o", str(out),
                    f"-L{PKG}/lib", "-lglm_b200", f"-Wl,-rpath,{PKG}/lib"], check=True)
    L = ctypes.CDLL(str(out))
    P, L64, D, I = ctypes.c_void_p, ctypes.c_long, ctypes.c_double, ctypes.c_int
    for s in ("f32", "f64", "i32", "u8", "i64"):
        getattr(L, f"probe_gradient_{s}").argtypes = [P, P, P, P, L64, L64, L64, L64, D, D, I, I]
        getattr(L, f"probe_predict_{s}").argtypes = [P, P, P, L64, L64, L64, L64]
        getattr(L, f"probe_randomize_{s}").argtypes = [P, L64, L64]
        getattr(L, f"probe_loss_{s}").argtypes = [P, P, P, P, L64, L64, L64, L64, D, D]
    L.probe_parse.argtypes = [I, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p)]
    L.probe_parse.restype = I
    return L


SFX = {np.dtype(np.float32): "f32", np.dtype(np.float64): "f64", np.dtype(np.int32): "i32",
       np.dtype(np.uint8): "u8", np.dtype(np.int64): "i64"}


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _host_gradient(L, X, M, Y, lam, alpha, reg, matrix=True):
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    g = np.zeros((ntasks, nt, nf), dtype=X.dtype)
    getattr(L, f"probe_gradient_{SFX[X.dtype]}")(_p(X), _p(M), _p(Y), _p(g), nf, nt, ntasks, nobs, lam, alpha,
                                                int(reg), int(matrix))
    return g


def _host_predict(L, X, M):
    nobs, ntasks, nf = X.shape
    nt = M.shape[1]
    y = np.zeros((nobs, ntasks, nt), dtype=X.dtype)
    getattr(L, f"probe_predict_{SFX[X.dtype]}")(_p(X), _p(M), _p(y), nf, nt, ntasks, nobs)
    return y


def _parse(L, *args):
    argv = (ctypes.c_char_p * (len(args) + 1))(b"probe", *[a.encode() for a in args])
    out = ctypes.c_char_p()
    rc = L.probe_parse(len(args) + 1, argv, ctypes.byref(out))
    return rc, out.value.decode()


def test_host_kernels_match_oracle(probe, oracle, golden):
    for name, c in golden.items():
        X, M, Y = c["X"], c["M"], c["Y"]
        if X.dtype not in SFX:
            continue
        g = _host_gradient(probe, X, M, Y, 0.0, 0.0, reg=False)
        yh = _host_predict(probe, X, M)
        if np.issubdtype(X.dtype, np.integer):
            assert np.array_equal(g, c["grad"]), name
            assert np.array_equal(yh, c["yhat"]), name
        else:
            tol = 1e-5 if X.dtype == np.float32 else 1e-12
            og = oracle.gradient(X, M, Y, with_reg=False)
            assert np.max(np.abs(g - og) / np.abs(og)) < tol, name
            if X.dtype == np.float32:  # host sums are carried in double
                o64 = oracle.gradient_acc64(X, M, Y, with_reg=False)
                assert np.max(np.abs(g - o64) / np.abs(o64)) < 2e-7, name
    rng = np.random.default_rng(0)
    X = rng.uniform(0, 1, (700, 3, 20))
    M = rng.uniform(-1, 1, (3, 4, 20))
    Y = rng.uniform(0, 1, (700, 3, 4))
    for matrix in (True, False):
        g = _host_gradient(probe, X, M, Y, 0.3, 0.25, reg=True, matrix=matrix)
        assert np.allclose(g, oracle.gradient(X, M, Y, 0.3, 0.25, True), rtol=1e-12, atol=1e-9)
    for dt in (np.uint8, np.int64):
        Xi = rng.integers(0, 100, (50, 2, 7)).astype(dt)
        Mi = rng.integers(0, 100, (2, 3, 7)).astype(dt)
        Yi = rng.integers(0, 100, (50, 2, 3)).astype(dt)
        assert np.array_equal(_host_gradient(probe, Xi, Mi, Yi, 2.9, 0.5, True),
                              oracle.gradient(Xi, Mi, Yi, 2.9, 0.5, True))


def test_host_loss_matches_oracle(probe, oracle):
    rng = np.random.default_rng(5)
    for dt in (np.float32, np.float64, np.int32, np.uint8, np.int64):
        dt = np.dtype(dt)
        for (nobs, ntasks, nf, nt) in [(1, 1, 1, 1), (300, 3, 7, 5), (0, 2, 4, 3)]:
            if dt.kind in "iu":
                lo = 0 if dt.kind == "u" else -50
                mk = lambda s: rng.integers(lo, 50, s).astype(dt)  # noqa: E731
            else:
                mk = lambda s: rng.uniform(-1, 1, s).astype(dt)  # noqa: E731
            M, Y, Yh = mk((ntasks, nt, nf)), mk((nobs, ntasks, nt)), mk((nobs, ntasks, nt))
            for lam, alpha in [(0.0, 0.0), (2.0, 0.5), (3.0, 1.0)]:
                got = np.zeros((1,), dtype=dt)
                getattr(probe, f"probe_loss_{SFX[dt]}")(_p(M), _p(Y), _p(Yh), _p(got), nf, nt, ntasks, nobs,
                                                      lam, alpha)
                ref = oracle.loss(M, Y, Yh, lam, alpha)
                if dt.kind in "iu":
                    assert got[0] == ref[0], (dt, lam, alpha)
                else:
                    assert abs(float(got[0]) - float(ref[0])) <= 1e-5 * abs(float(ref[0])) + 1e-30


def test_seeded_initialisation_is_mt19937_64_uniform(probe):
    a = np.zeros(1000, np.float32)
    probe.probe_randomize_f32(_p(a), 1000, 42)
    b = np.zeros(1000, np.float32)
    probe.probe_randomize_f32(_p(b), 1000, 42)
    assert np.array_equal(a, b) and a.min() >= 0 and a.max() < 1
    d = np.zeros(1000, np.float64)
    probe.probe_randomize_f64(_p(d), 1000, 43)
    assert d.min() >= 0 and d.max() < 1 and not np.allclose(d[:10], a[:10])
    u = np.zeros(1000, np.uint8)
    probe.probe_randomize_u8(_p(u), 1000, 42)
    assert u.min() >= 0 and u.max() <= 100 and len(set(u.tolist())) > 50


def test_option_parser(probe):
    rc, out = _parse(probe, "-X", "32", "--ntargets=1", "-T1", "--nobs", "8192", "--lambda", "0.1",
                     "--type", "double", "--verbose", "-f", "--seed", "7", "--block-dim-x=4")
    assert rc == 0, out
    kv = dict(p.split("=") for p in out.split(";"))
    assert kv["nfeatures"] == "32" and kv["ntargets"] == "1" and kv["ntasks"] == "1" and kv["nobs"] == "8192"
    assert kv["lambda"] == "0.1" and kv["type"] == "double" and kv["verbose"] == "1" and kv["force"] == "1"
    assert kv["seed"] == "7" and kv["bx"] == "4" and kv["gpu_algo"] == "fused" and kv["cpu_algo"] == "matrix"
    rc, out = _parse(probe)
    kv = dict(p.split("=") for p in out.split(";"))
    assert rc == 0 and kv["nfeatures"] == "25" and kv["nobs"] == "1000" and kv["seed"] == "42"
    assert kv["init"] == "random" and kv["help"] == "0"
    assert _parse(probe, "--gpu-algo", "warp")[0] == 0
    for bad in (["--gpu-algo", "nope"], ["--type", "quad"], ["--cpu-algo", "x"], ["--nobs"], ["--nobs", "abc"],
                ["--unknown"], ["--alpha", "2"], ["--block-dim-x", "-3"]):
        rc, out = _parse(probe, *bad)
        assert rc == 1, (bad, out)


@pytest.mark.parametrize("exe", ["glm_predict_naive", "glm_gradient_naive", "glm_gradient_xyyhat", "glm_loss_myyhat"])
def test_executables_help_and_bad_options(exe):
    path = os.path.join(BIN, exe)
    assert os.path.exists(path), "build with make -C gpu_algos_b200"
    r = subprocess.run([path, "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0
    # the sweep harness finds the size flags with the regex -[A-Z][ ,] in --help
    import re
    assert set(re.findall(r"-([A-Z])[ ,]", r.stdout)) >= {"X", "Y", "T", "N"}
    r = subprocess.run([path, "--no-such-option"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
