"""The f64 tensor-core MMA shapes that the tiled float64 gradient relies on.

tests/cpp/f64_mma_probe.cu multiplies known 16 x 16 / 16 x 8 (and smaller)
double matrices with one mma.sync of each f64 shape, loading and storing the
fragments by the lane layout that gpu_algos_b200/csrc/glm_tiles.cu uses, and
compares every element with the host product (relative 1e-9: the products
are exact, only the summation order differs).  It also prints each shape's
throughput with operands in registers -- the FP64 tensor pipe's peak, the
bound of the tiled kernel.  Compiled here with nvcc for sm_100a.
"""
import os
import re
import shutil
import subprocess

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    out = tmp_path_factory.mktemp("mma") / "f64_mma_probe"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-o", str(out),
                    os.path.join(REPO, "tests", "cpp", "f64_mma_probe.cu")], check=True)
    return str(out)


def test_f64_mma_layouts_and_throughput(probe):
    r = subprocess.run([probe], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    layouts = re.findall(r"^layout (\S+)\s*: (\S+)", r.stdout, re.M)
    assert [s for s, _ in layouts] == ["m8n8k4", "m16n8k4", "m16n8k8", "m16n8k16"]
    assert all(v == "ok" for _, v in layouts), r.stdout
    tputs = [float(x) for x in re.findall(r"([0-9.]+) TFLOP/s", r.stdout)]
    assert len(tputs) == 9 and all(t > 0 for t in tputs)
