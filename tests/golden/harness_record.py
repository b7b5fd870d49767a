"""Record the command lines the reference's sweep harness issues for this
package's GLM executables (``gpu_algos_b200/bin``).

The reference tests its executables with ``test/gpu_algo_test/gpu_algo_test.py``:
it reads each executable's ``--help`` for its size options (``-X``, ``-Y``,
``-T``, ``-N`` here), cycles the warp- and block-boundary size classes
(``gpu_algo_test.py:89-97``) through them under a cap on the product,
adds ``--type`` and ``--tol-bits`` and parses the stdout lines ``Max error``,
``Max error rel``, ``Compute kernel:`` and ``[SUCCESS]`` (``:569-600``).
The harness is a Python script of the reference checkout and does not
travel to a GPU host, so its use is split in three steps:

1. this script, where the reference checkout is available, runs the
   harness's own executable discovery and command construction against
   ``gpu_algos_b200/bin`` (the ``--help`` calls really run; the test runs are
   only recorded) and writes ``tests/golden/harness_commands.json``;
2. ``tests/golden/harness_run.py`` runs those command lines on a GPU host
   and writes their outputs to ``tests/golden/harness_outputs.json.gz``;
3. ``tests/test_harness_replay.py`` feeds the recorded outputs back through
   the harness's own loop, parser and verdict (where the checkout is
   available), and checks them with the same stdout contract otherwise.

Usage::

    python tests/golden/harness_record.py <path-to-gpu_algos-checkout>   (or GPU_ALGOS_REFERENCE)
"""
from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
BIN = os.path.join(REPO, "gpu_algos_b200", "bin")
OUT = os.path.join(HERE, "harness_commands.json")
MAX_PROBLEM_SIZE = 1 << 20  # product of the four GLM dimensions (the harness's --max-problem-size)


def load_harness(ref_root: str):
    path = os.path.join(ref_root, "test", "gpu_algo_test", "gpu_algo_test.py")
    spec = importlib.util.spec_from_file_location("reference_gpu_algo_test", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _Done:
    def __init__(self, cmd, stdout=""):
        self.args, self.returncode, self.stdout, self.stderr = cmd, 0, stdout, ""


def main(ref_root: str) -> None:
    mod = load_harness(ref_root)
    real_run = subprocess.run
    recorded = []

    def run(cmd, *args, **kwargs):
        if len(cmd) == 2 and cmd[1] == "--help":
            return real_run(cmd, *args, **kwargs)
        recorded.append([os.path.basename(cmd[0])] + list(cmd[1:]))
        return _Done(cmd)

    mod.subprocess.run = run
    try:
        tester = mod.GPUAlgoTest(bin_dir=BIN, max_problem_size=MAX_PROBLEM_SIZE)
        for exe in tester.executables:
            tester.test_all_sizes_and_types(exe)
    finally:
        mod.subprocess.run = real_run
    with open(OUT, "w") as f:
        json.dump({"max_problem_size": MAX_PROBLEM_SIZE, "commands": recorded}, f, indent=0)
    print(f"{len(recorded)} command lines -> {OUT}")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GPU_ALGOS_REFERENCE")
    if not root:
        sys.exit("usage: harness_record.py <path-to-gpu_algos-checkout>  (or set GPU_ALGOS_REFERENCE)")
    main(root)
