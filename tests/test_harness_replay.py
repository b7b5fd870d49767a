"""The reference's sweep harness over this package's GLM executables.

``tests/golden/harness_commands.json`` holds the 704 command lines that the
reference's harness (``test/gpu_algo_test/gpu_algo_test.py``) builds for
``gpu_algos_b200/bin`` -- its size classes (``:89-97``) cycled through the
executables' ``-X -Y -T -N`` options under a product cap of 2^20, every
``--type`` of the eleven, ``--tol-bits 4`` for floating types -- and
``tests/golden/harness_outputs.json.gz`` what they printed on a B200
(``tests/golden/harness_run.py``).

* Everywhere: every recorded run exited 0 and printed the stdout contract the
  harness parses (``Max error``, ``Max error rel``, ``Compute kernel:``,
  ``[SUCCESS]``; ``gpu_algo_test.py:569-600``).
* Where a checkout of the reference is named by ``GPU_ALGOS_REFERENCE``: the
  harness's own loop (``test_all_sizes_and_types``), parser
  (``_extract_performance_metrics``) and verdict (``_check_correctness``) run
  unmodified over the recorded outputs, and every run must come out
  ``run_success`` and ``correct``.
* On a GPU (``-m gpu``): every 11th recorded command line is run again
  against the current build and must still print ``[SUCCESS]``.
"""
import gzip
import json
import os
import re
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
BIN = os.path.join(REPO, "gpu_algos_b200", "bin")
GOLD = os.path.join(HERE, "golden")


def _commands():
    with open(os.path.join(GOLD, "harness_commands.json")) as f:
        return json.load(f)["commands"]


def _outputs():
    with gzip.open(os.path.join(GOLD, "harness_outputs.json.gz"), "rt") as f:
        return {" ".join(r["cmd"]): r for r in json.load(f)["outputs"]}


def test_every_recorded_run_meets_the_stdout_contract():
    cmds, outs = _commands(), _outputs()
    assert len(cmds) == 704
    for cmd in cmds:
        r = outs[" ".join(cmd)]
        assert r["return_code"] == 0, cmd
        s = r["stdout"]
        assert "[SUCCESS]" in s and "[FAILURE]" not in s, cmd
        assert re.search(r"Max error\s*:\s*([\d.e+-]+)", s), cmd
        assert re.search(r"Max error rel\s*:\s*([\d.e+-]+|nan|inf)", s), cmd
        assert re.search(r"Compute kernel:\s*([\d.]+)\s*ms", s), cmd


def test_reference_harness_over_recorded_outputs():
    root = os.environ.get("GPU_ALGOS_REFERENCE")
    if not root or not os.path.exists(os.path.join(root, "test", "gpu_algo_test", "gpu_algo_test.py")):
        pytest.skip("GPU_ALGOS_REFERENCE does not name a checkout of the reference")
    import sys

    sys.path.insert(0, GOLD)
    try:
        import harness_record
    finally:
        sys.path.remove(GOLD)
    mod = harness_record.load_harness(root)
    outs = _outputs()
    real_run = subprocess.run
    served = []

    class Done:
        def __init__(self, rec):
            self.returncode, self.stdout, self.stderr = rec["return_code"], rec["stdout"], rec["stderr"]

    def run(cmd, *args, **kwargs):
        if len(cmd) == 2 and cmd[1] == "--help":
            return real_run(cmd, *args, **kwargs)
        key = " ".join([os.path.basename(cmd[0])] + list(cmd[1:]))
        served.append(key)
        return Done(outs[key])

    mod.subprocess.run = run
    try:
        tester = mod.GPUAlgoTest(bin_dir=BIN, max_problem_size=harness_record.MAX_PROBLEM_SIZE)
        results = []
        for exe in tester.executables:
            results += tester.test_all_sizes_and_types(exe)
    finally:
        mod.subprocess.run = real_run
    assert len(results) == len(served) == 704
    bad = [r["cmdline"] for r in results if not (r["run_success"] and r.get("correct"))]
    assert not bad, bad[:5]


@pytest.mark.gpu
def test_recorded_commands_still_succeed_on_the_gpu():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    for cmd in _commands()[::11]:
        r = subprocess.run([os.path.join(BIN, cmd[0])] + cmd[1:], capture_output=True, text=True, timeout=300,
                           cwd=BIN)
        assert r.returncode == 0 and "[SUCCESS]" in r.stdout, (cmd, r.stdout[-500:], r.stderr[-500:])
