"""Sweep of the GLM executables the way the reference's regression harness
(test/gpu_algo_test/gpu_algo_test.py in gpu_algos) drives executables: the
size flags are discovered from --help (options matching -[A-Z][ ,]), sizes
straddling warp and block boundaries are cycled through them with the
product of all dimensions capped, every element type is passed with --type
(and --tol-bits for floating types), and a run passes when it exits 0 and
prints [SUCCESS]."""
import os
import re
import subprocess

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

BIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "gpu_algos_b200", "bin")
EXES = ["glm_predict_naive", "glm_gradient_naive", "glm_gradient_xyyhat", "glm_loss_myyhat"]
TYPES = ["half", "float", "double", "int8", "int16", "int32", "int64", "uint8", "uint16", "uint32", "uint64"]
# below, at and across warp (32) and block (1024) boundaries
SIZES = [8, 24, 32, 33, 100, 128, 1024, 1025, 2500]
MAX_PRODUCT = 1 << 21
TOL_BITS = 6


def _size_flags(exe):
    out = subprocess.run([os.path.join(BIN, exe), "--help"], capture_output=True, text=True, timeout=60).stdout
    flags = []
    for m in re.findall(r"-([A-Z])[ ,]", out):
        if f"-{m}" not in flags:
            flags.append(f"-{m}")
    return flags


def _command(exe, dtype, size_i):
    cmd = [os.path.join(BIN, exe)]
    product = 1
    for k, flag in enumerate(_size_flags(exe)):
        size = min(SIZES[(size_i + k) % len(SIZES)], MAX_PRODUCT // product)
        product *= max(size, 1)
        cmd += [flag, str(size)]
    cmd += ["--type", dtype]
    if dtype in ("half", "float", "double"):
        cmd += ["--tol-bits", str(TOL_BITS)]
    return cmd


@pytest.mark.parametrize("exe", EXES)
@pytest.mark.parametrize("dtype", TYPES)
def test_sweep(exe, dtype):
    assert set(_size_flags(exe)) >= {"-X", "-Y", "-T", "-N"}
    for size_i in (0, 3, 6):
        cmd = _command(exe, dtype, size_i)
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0 and "[SUCCESS]" in r.stdout, " ".join(cmd) + "\n" + r.stdout[-1500:] + r.stderr[-800:]
