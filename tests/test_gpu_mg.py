"""The single-process multi-GPU context (glmb_mg_*) driven from C++.

tests/cpp/mg_probe.cpp is a plain C++ host (one thread, no torch) that
splits observations over the GPUs, runs the sharded gradient and the
sharded elastic-net fit through the context with the library's peer
exchange and with NCCL, and compares them with the one-GPU entry points on
the whole data: max relative error <= 1e-4 (float32) / 1e-11 (float64) for
the gradient, cancellation floor 1e-3 of the largest element; every device
must hold bit-identical results.  Needs two GPUs (skipped otherwise); the
probe is compiled here against include/glm_b200.h and libglm_b200.so.
"""
import os
import subprocess

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "gpu_algos_b200", "lib")


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    out = tmp_path_factory.mktemp("mg") / "mg_probe"
    subprocess.run(["g++", "-std=c++20", "-O2", f"-I{REPO}/include", "-I/usr/local/cuda/include",
                    os.path.join(REPO, "tests", "cpp", "mg_probe.cpp"), "-o", str(out),
                    f"-L{LIB}", "-lglm_b200", "-L/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{LIB}"],
                   check=True)
    return str(out)


@pytest.mark.parametrize("mode", ["peer", "nccl"])
def test_mg_context_matches_one_gpu(probe, mode):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([probe, "2", mode], capture_output=True, text=True, timeout=600, env=env)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL PASS" in r.stdout
    assert r.stdout.count("PASS") >= 8
