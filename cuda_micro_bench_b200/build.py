"""Builds the native parts in-tree with make: the sm_100a library and CLI
(``lib/libcmb_b200.so``, ``bin/cmb_b200``)."""

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 8, verbose: bool = False) -> None:
    cmd = ["make", "-C", HERE, f"-j{jobs}"]
    out = None if verbose else subprocess.PIPE
    proc = subprocess.run(cmd, stdout=out, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"native build failed ({' '.join(cmd)}):\n{proc.stdout}")


if __name__ == "__main__":
    build(verbose=True)
