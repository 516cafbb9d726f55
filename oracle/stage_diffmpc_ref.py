"""TEST AND BASELINE INFRASTRUCTURE ONLY -- stages the reference DiffMPC
solver's pure-Python sources into oracle/_ref/diffmpc/, so that the CPU
baseline can time the reference itself on the GPU machine, where the
reference tree is absent:

    python oracle/stage_diffmpc_ref.py <reference root>

Copies, unchanged:
  DifferentialMPC/*.py                              -> _ref/diffmpc/DifferentialMPC/
  acmpc_public-master/diff_mpc_drones/drone.py      -> _ref/diffmpc/drone.py
  acmpc_public-master/mpc.pytorch/mpc/*.py          -> _ref/diffmpc/mpc/   (drone.py imports mpc.util)

oracle/_ref/ is git-ignored: the copies are never part of the repository's
history; they travel to the GPU machine with the working tree, as the built
reference FastMPC kernels beside them do. Returns the staged directory, or
None (with a message) when the reference tree is absent.
"""

from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "diffmpc")
SOURCES = (
    ("DifferentialMPC", "DifferentialMPC"),
    (os.path.join("acmpc_public-master", "mpc.pytorch", "mpc"), "mpc"),
)
DRONE = os.path.join("acmpc_public-master", "diff_mpc_drones", "drone.py")


def stage(reference_root: str) -> str | None:
    if not all(os.path.isdir(os.path.join(reference_root, src)) for src, _ in SOURCES) or \
            not os.path.isfile(os.path.join(reference_root, DRONE)):
        print(f"reference DiffMPC sources not found under {reference_root}; oracle/_ref/diffmpc not staged")
        return None
    for src, dst in SOURCES:
        d = os.path.join(OUT, dst)
        os.makedirs(d, exist_ok=True)
        for f in sorted(glob.glob(os.path.join(reference_root, src, "*.py"))):
            shutil.copy2(f, os.path.join(d, os.path.basename(f)))
    shutil.copy2(os.path.join(reference_root, DRONE), os.path.join(OUT, "drone.py"))
    return OUT


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python oracle/stage_diffmpc_ref.py <reference root>")
    print(stage(sys.argv[1]))
