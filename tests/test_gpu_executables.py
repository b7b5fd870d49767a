"""The C++ GLM executables (the reference's drivers rebuilt on the C ABI)
run on the GPU and pass their own CPU check, the way the reference's sweep
harness (test/gpu_algo_test/gpu_algo_test.py) exercises them: it parses
"Max error rel", "Compute kernel: <ms> ms" and the [SUCCESS] / [FAILURE]
verdict from stdout."""
import os
import re
import subprocess

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

BIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "gpu_algos_b200", "bin")


def _run(exe, *args):
    r = subprocess.run([os.path.join(BIN, exe), *args], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    out = r.stdout
    m = re.search(r"Max error rel\s*:\s*([\d.e+-]+|nan|inf)", out)
    k = re.search(r"Compute kernel:\s*([\d.]+)\s*ms", out)
    assert m and k, out[-2000:]
    return out, float(m.group(1))


CASES = [
    ("glm_gradient_xyyhat", []),  # reference defaults: 25 x 25 x 10 x 1000, float
    ("glm_gradient_xyyhat", ["-X", "32", "-Y", "1", "-T", "1", "-N", "8192", "--lambda", "0.1"]),
    ("glm_gradient_xyyhat", ["-X", "128", "-Y", "1", "-T", "1", "-N", "65536", "--lambda", "0.01"]),
    ("glm_gradient_xyyhat", ["-X", "1025", "-Y", "3", "-T", "2", "-N", "24", "--lambda", "0.5", "--alpha", "0.5"]),
    ("glm_gradient_xyyhat", ["--type", "double", "-X", "256", "-Y", "16", "-T", "4", "-N", "1500", "--lambda", "0.1"]),
    ("glm_gradient_xyyhat", ["--type", "half", "-X", "16", "-Y", "2", "-T", "2", "-N", "64"]),
    ("glm_gradient_xyyhat", ["--type", "int32", "-X", "24", "-Y", "8", "-T", "3", "-N", "2500", "--lambda", "3", "--alpha", "1"]),
    ("glm_gradient_xyyhat", ["--type", "uint8", "--init-method", "increasing", "-X", "8", "-Y", "16", "-T", "24", "-N", "8"]),
    ("glm_gradient_xyyhat", ["--type", "int64", "--init-method", "decreasing", "-X", "33", "-Y", "2", "-T", "1", "-N", "1025"]),
    ("glm_gradient_xyyhat", ["--cpu-algo", "nested-loop", "-X", "8", "-Y", "2", "-T", "2", "-N", "100", "--lambda", "0.2", "--alpha", "0.3"]),
    ("glm_gradient_naive", []),
    ("glm_gradient_naive", ["--type", "double", "-X", "100", "-Y", "1", "-T", "3", "-N", "5000"]),
    ("glm_gradient_naive", ["--type", "int16", "-X", "16", "-Y", "1", "-T", "1", "-N", "1500"]),
    ("glm_predict_naive", []),
    ("glm_predict_naive", ["-X", "128", "-Y", "1", "-T", "1", "-N", "100000"]),
    ("glm_predict_naive", ["--type", "uint64", "-X", "24", "-Y", "8", "-T", "16", "-N", "1025"]),
    ("glm_predict_naive", ["--type", "half", "-X", "8", "-Y", "1", "-T", "1", "-N", "2500"]),
    ("glm_loss_myyhat", []),
    ("glm_loss_myyhat", ["--lambda", "0.5", "--alpha", "0.3"]),
    ("glm_loss_myyhat", ["--type", "double", "-X", "64", "-Y", "16", "-T", "4", "-N", "100000", "--lambda", "0.1"]),
    ("glm_loss_myyhat", ["--type", "int32", "-X", "24", "-Y", "8", "-T", "3", "-N", "2500", "--lambda", "3", "--alpha", "1"]),
    ("glm_loss_myyhat", ["--type", "uint8", "--init-method", "increasing", "-X", "8", "-Y", "16", "-T", "24", "-N", "8"]),
    ("glm_loss_myyhat", ["--type", "half", "-X", "8", "-Y", "2", "-T", "2", "-N", "100"]),
]


@pytest.mark.parametrize("exe,args", CASES, ids=[f"{e}:{' '.join(a) or 'defaults'}" for e, a in CASES])
def test_executable_passes_its_cpu_check(exe, args):
    out, rel = _run(exe, *args)
    assert "[SUCCESS]" in out, out[-1500:]
    if any(t in args for t in ("int16", "int32", "int64", "uint8", "uint64")):
        assert rel == 0.0
    if "--type" not in args or "float" in args:
        assert rel <= 1e-4
    if exe != "glm_loss_myyhat":
        assert "path=" in out
