"""Install the unmodified reference package into baseline/_ref (git-ignored;
it travels to the GPU box with the working tree).  Used by bench.py to time
the reference's own CPU path (pytm, src/pytm/base.py) on the box's host cores.

    python oracle/install_reference.py [--ref PATH]

First tries the offline pip install
    pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
        --target baseline/_ref <copy of the reference>
The reference declares `hatchling` as its build backend (pyproject.toml
[build-system]); when that backend is not installed the wheel cannot be built,
and the script then lays out in baseline/_ref exactly the packages the wheel
would hold ([tool.hatch.build.targets.wheel] packages = src/ytm, src/cutm,
src/pytm, src/tm_utils), unmodified.  Nothing of the reference is committed.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
TARGET = os.path.join(ROOT, "baseline", "_ref")
PACKAGES = ("ytm", "cutm", "pytm", "tm_utils")


def main() -> int:
    from ref_build import DEFAULT_REF
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=DEFAULT_REF)
    a = ap.parse_args()
    if not os.path.isdir(os.path.join(a.ref, "src", "pytm")):
        print(f"no reference checkout at {a.ref}", file=sys.stderr)
        return 1
    os.makedirs(TARGET, exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:  # the build may write into the source tree
        src = os.path.join(tmp, "ref")
        shutil.copytree(a.ref, src, ignore=shutil.ignore_patterns(".git", ".pixi"))
        r = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                            "--no-deps", "--find-links", "/opt/wheelhouse", "--target", TARGET, src],
                           capture_output=True, text=True)
        if r.returncode == 0:
            print("pip install: ok")
            return 0
        why = (r.stderr.strip().splitlines() or ["?"])[-1]
        print(f"pip install failed ({why}); laying out the wheel's packages instead")
        for p in PACKAGES:
            d = os.path.join(src, "src", p)
            if os.path.isdir(d):
                shutil.copytree(d, os.path.join(TARGET, p), dirs_exist_ok=True,
                                ignore=shutil.ignore_patterns("__pycache__"))
    with open(os.path.join(TARGET, "INSTALL_NOTE.txt"), "w") as f:
        f.write("packages of the reference's wheel, unmodified (pip could not build it: no hatchling backend)\n")
    print("installed:", sorted(os.listdir(TARGET)))
    return 0


if __name__ == "__main__":
    sys.path.insert(0, HERE)
    raise SystemExit(main())
