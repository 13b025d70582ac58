"""Build ``libckv.so`` in-tree for sm_100a (``python -m submission_folder_b200.build``)."""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")


def build(verbose: bool = False) -> str:
    """Run the csrc Makefile (nvcc -gencode arch=compute_100a,code=sm_100a); returns the .so path."""
    jobs = str(max(1, min(8, os.cpu_count() or 1)))
    cmd = ["make", "-C", CSRC, "-j", jobs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stdout.write(res.stdout)
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError("building libckv.so failed")
    return os.path.join(HERE, "libckv.so")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
