"""Build recipe for the CPU oracle (test infrastructure only).

Compiles ``oracle/csrc/oracle.c`` into ``oracle/liboracle.so`` with
``-ffp-contract=off`` so that every floating-point operation rounds exactly
once in program order.  The product library never links this file.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCE = os.path.join(HERE, "csrc", "oracle.c")
LIBRARY = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    """Compile the oracle shared library if it is missing or stale."""
    if (not force and os.path.exists(LIBRARY)
            and os.path.getmtime(LIBRARY) >= os.path.getmtime(SOURCE)):
        return LIBRARY
    command = [
        "gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off",
        "-fno-fast-math", "-Wall", "-Wextra", "-o", LIBRARY, SOURCE, "-lm",
    ]
    subprocess.run(command, check=True)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
