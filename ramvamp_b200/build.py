"""Build the in-tree CUDA library (sm_100a) with its Makefile."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")


def build(force: bool = False) -> str:
    """Compile ramvamp_b200/libramvamp_b200.so (nvcc, -gencode sm_100a).

    The Makefile also generates the SiLU exception table from the host libm.
    """
    if force:
        subprocess.run(["make", "-C", CSRC, "clean"], check=True)
    subprocess.run(["make", "-C", CSRC, "-s"], check=True)
    return os.path.join(HERE, "libramvamp_b200.so")


if __name__ == "__main__":
    print(build())
