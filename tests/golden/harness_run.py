"""Run the command lines recorded by ``harness_record.py`` against
``gpu_algos_b200/bin`` on a GPU host and store their outputs in
``tests/golden/harness_outputs.json.gz`` (return code, stdout, stderr per
command line), the input of ``tests/test_harness_replay.py``.

Usage (on a host with a B200 and the built executables)::

    python tests/golden/harness_run.py [--jobs 8] [--out PATH]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import gzip
import json
import os
import subprocess
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
BIN = os.path.join(REPO, "gpu_algos_b200", "bin")
COMMANDS = os.path.join(HERE, "harness_commands.json")
OUT = os.path.join(HERE, "harness_outputs.json.gz")


def run_one(cmd, timeout=300):
    argv = [os.path.join(BIN, cmd[0])] + cmd[1:]
    t0 = time.time()
    try:
        r = subprocess.run(argv, capture_output=True, text=True, timeout=timeout, cwd=BIN)
        rc, out, err = r.returncode, r.stdout, r.stderr
    except subprocess.TimeoutExpired:
        rc, out, err = -1, "", f"timeout after {timeout} s"
    return {"cmd": cmd, "return_code": rc, "stdout": out, "stderr": err, "seconds": round(time.time() - t0, 3)}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--jobs", type=int, default=8)
    p.add_argument("--out", default=OUT)
    a = p.parse_args()
    with open(COMMANDS) as f:
        commands = json.load(f)["commands"]
    with cf.ThreadPoolExecutor(max_workers=a.jobs) as ex:
        results = list(ex.map(run_one, commands))
    results.sort(key=lambda r: " ".join(r["cmd"]))
    with gzip.open(a.out, "wt") as f:
        json.dump({"outputs": results}, f)
    bad = [r for r in results if r["return_code"] != 0 or "[SUCCESS]" not in r["stdout"]]
    print(f"{len(results)} runs, {len(bad)} without [SUCCESS] -> {a.out}")
    for r in bad[:10]:
        print(" ".join(r["cmd"]), r["return_code"], r["stdout"][-300:], r["stderr"][-300:])
    return 1 if bad else 0


if __name__ == "__main__":
    raise SystemExit(main())
