"""Build the oracle's C helpers (oracle/_build/libcsynth.so) with gcc.

TEST INFRASTRUCTURE ONLY.  `python -m oracle.build`; called by __graft_entry__.build().
"""

import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_build")
LIB = os.path.join(OUT, "libcsynth.so")
SRC = os.path.join(HERE, "csynth.c")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(OUT, exist_ok=True)
    cc = shutil.which("gcc") or "cc"
    cmd = [cc, "-O3", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", SRC, "-o", LIB + ".tmp"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
